// Device-side building blocks shared by the slab kernels.
//
// Slab wire formats (reference docs/format.md:15-30, src/c_api.cpp:18-28 and
// 44-65):
//   serial  "bf16-huffman-tile16":  u64 count | u64 bit_count | u8 len[256] |
//            u8 sm[count] | exponent bits, MSB first, ceil(bit_count/8) bytes
//   parallel "bf16-huffman-parallel32": "XKSP2\0\0\0" | u64 rows | u64 cols |
//            u64 chunks | u64 seg_len[chunks] | chunks serial segments, segment
//            i covering tiled elements [n*i/chunks, n*(i+1)/chunks)
// Elements are in 16x16 tile order (src/layout.cpp:32-50).  A BF16 word is
// (sm & 0x80) << 8 | exponent << 7 | (sm & 0x7f) (src/codec.cpp:70).
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

#include "xksv_types.h"

namespace xksv {

// --------------------------------------------------------------- loads ----
__device__ __forceinline__ uint32_t bswap32(uint32_t x) { return __byte_perm(x, 0, 0x0123); }

__device__ __forceinline__ uint4 ldg16(const void* p) {
  return __ldg(reinterpret_cast<const uint4*>(p));
}

// Little-endian u64 from any byte address (header fields only).
__device__ __forceinline__ uint64_t ld_le64(const uint8_t* p) {
  uint64_t v = 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) v |= uint64_t(__ldg(p + i)) << (8 * i);
  return v;
}

// Eight bytes starting at an arbitrary address, assembled little-endian from
// two aligned 8-byte loads.  `lo_ok`/`hi_ok` gate loads that would fall
// outside the owning buffer (the gated word reads as zero).
__device__ __forceinline__ uint64_t ld8_any(const uint8_t* p, const uint8_t* end) {
  uintptr_t a = reinterpret_cast<uintptr_t>(p);
  const uint64_t* w = reinterpret_cast<const uint64_t*>(a & ~uintptr_t(7));
  int sh = int(a & 7) * 8;
  uint64_t lo = __ldg(w);
  if (sh == 0) return lo;
  uint64_t hi = (reinterpret_cast<const uint8_t*>(w + 1) < end) ? __ldg(w + 1) : 0ull;
  return (lo >> sh) | (hi << (64 - sh));
}

// ------------------------------------------------------- bit reader -------
// MSB-first bit stream in global memory, read through aligned 16-byte chunks
// with one chunk always in flight ahead of the one being consumed.  Fetches
// are unconditional (the address is clamped to the stream's last chunk), so a
// fetch never stalls on a select of its own result; bits past the stream end
// are whatever the last chunk holds, which only a corrupt stream can reach and
// which the caller's final bit count rejects.  `buf` holds the next bits
// left-aligned, `nb` how many are valid.
struct BitReader {
  const uint4* next;   // next aligned chunk to fetch
  const uint4* last;   // last chunk holding stream bytes
  uint4 nxt;           // fetched, not yet consumed
  uint4 cur;           // current chunk, big-endian words, consumed from .x
  int cw;              // words left in cur
  uint32_t taken;      // words moved into buf so far
  uint32_t skip0;      // bits of the first words that precede the stream start
  uint64_t buf;
  int nb;

  __device__ __forceinline__ uint4 fetch() {
    const uint4* q = next <= last ? next : last;
    ++next;
    return ldg16(q);
  }
  __device__ __forceinline__ void load_chunk() {
    const uint4 c = nxt;
    nxt = fetch();
    cur = make_uint4(bswap32(c.x), bswap32(c.y), bswap32(c.z), bswap32(c.w));
    cw = 4;
  }
  // Takes the next word; `cur` always holds at least one word afterwards.
  __device__ __forceinline__ uint32_t take_word() {
    const uint32_t w = cur.x;
    cur.x = cur.y;
    cur.y = cur.z;
    cur.z = cur.w;
    --cw;
    ++taken;
    if (cw == 0) load_chunk();
    return w;
  }
  __device__ __forceinline__ void init(const uint8_t* base, uint64_t nbytes) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(base);
    const uint4* first = reinterpret_cast<const uint4*>(a & ~uintptr_t(15));
    next = first;
    last = reinterpret_cast<const uint4*>((a + (nbytes ? nbytes - 1 : 0)) & ~uintptr_t(15));
    const int skipb = int(a & 15) * 8;
    taken = 0;
    skip0 = uint32_t(skipb);
    nxt = fetch();
    load_chunk();
    for (int i = 0; i < (skipb >> 5); ++i) take_word();
    buf = uint64_t(take_word()) << 32;
    buf |= take_word();
    const int sb = skipb & 31;
    buf <<= sb;
    nb = 64 - sb;
  }
  // Ensures nb > 32 (a branch: use where lanes rarely get here together).
  __device__ __forceinline__ void refill() {
    if (nb <= 32) {
      buf |= uint64_t(take_word()) << (32 - nb);
      nb += 32;
    }
  }
  // Same effect without a data-dependent branch around the word move; the
  // chunk load below it is the only per-lane branch, one in four refills.
  __device__ __forceinline__ void refill_uniform() {
    const bool need = nb <= 32;
    const uint32_t w = cur.x;
    const uint64_t add = uint64_t(w) << (need ? 32 - nb : 0);
    buf |= need ? add : 0ull;
    nb += need ? 32 : 0;
    cur.x = need ? cur.y : cur.x;
    cur.y = need ? cur.z : cur.y;
    cur.z = need ? cur.w : cur.z;
    cw -= need ? 1 : 0;
    taken += need ? 1u : 0u;
    if (cw == 0) load_chunk();
  }
  __device__ __forceinline__ uint32_t peek32() const { return uint32_t(buf >> 32); }
  __device__ __forceinline__ void skip(int n) {
    buf <<= n;
    nb -= n;
  }
  // Bits consumed from the stream start.
  __device__ __forceinline__ uint64_t consumed() const {
    return uint64_t(taken) * 32 - uint64_t(nb) - skip0;
  }
};

// Sequential 8-byte groups of a byte stream starting at any address, fetched
// two aligned words ahead of use; fetch addresses are clamped to `lastw` (the
// aligned word holding the stream's final byte).
struct ByteReader8 {
  const uint64_t* next;
  const uint64_t* lastw;
  uint64_t w0, w1, w2;
  int sh;
  __device__ __forceinline__ uint64_t fetch() {
    const uint64_t* q = next <= lastw ? next : lastw;
    ++next;
    return __ldg(q);
  }
  __device__ __forceinline__ void init(const uint8_t* p, const uint8_t* end) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(p);
    next = reinterpret_cast<const uint64_t*>(a & ~uintptr_t(7));
    lastw = reinterpret_cast<const uint64_t*>((reinterpret_cast<uintptr_t>(end) - 1) & ~uintptr_t(7));
    sh = int(a & 7) * 8;
    w0 = fetch();
    w1 = fetch();
    w2 = fetch();
  }
  // The next 8 bytes, little-endian.
  __device__ __forceinline__ uint64_t take() {
    const uint64_t v = sh ? (w0 >> sh) | (w1 << (64 - sh)) : w0;
    w0 = w1;
    w1 = w2;
    w2 = fetch();
    return v;
  }
};

// Sequential 16-byte groups of a byte stream starting at any address.  Raw
// aligned chunks sit in a 3-deep register ring (two loads in flight); the
// funnel that realigns them runs only when a group is consumed, so no load is
// waited on early.  Fetch addresses are clamped to the chunk holding the
// stream's final byte.
struct ByteReader16 {
  const uint4* next;
  const uint4* lastc;
  uint4 r0, r1, r2;
  int q, bs;  // word and bit offset of the stream start inside a chunk
  __device__ __forceinline__ uint4 fetch() {
    const uint4* p = next <= lastc ? next : lastc;
    ++next;
    return ldg16(p);
  }
  __device__ __forceinline__ void init(const uint8_t* p, const uint8_t* end) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(p);
    next = reinterpret_cast<const uint4*>(a & ~uintptr_t(15));
    lastc = reinterpret_cast<const uint4*>((reinterpret_cast<uintptr_t>(end) - 1) & ~uintptr_t(15));
    q = int((a >> 2) & 3);
    bs = int(a & 3) * 8;
    r0 = fetch();
    r1 = fetch();
    r2 = fetch();
  }
  // The next 16 bytes, little-endian words.
  __device__ __forceinline__ uint4 take() {
    uint32_t w0 = r0.x, w1 = r0.y, w2 = r0.z, w3 = r0.w, w4 = r1.x, w5 = r1.y, w6 = r1.z, w7 = r1.w;
    if (q & 2) {
      w0 = w2; w1 = w3; w2 = w4; w3 = w5; w4 = w6; w5 = w7;
    }
    if (q & 1) {
      w0 = w1; w1 = w2; w2 = w3; w3 = w4; w4 = w5;
    }
    const uint4 v = make_uint4(__funnelshift_r(w0, w1, bs), __funnelshift_r(w1, w2, bs),
                               __funnelshift_r(w2, w3, bs), __funnelshift_r(w3, w4, bs));
    r0 = r1;
    r1 = r2;
    r2 = fetch();
    return v;
  }
};

// MSB-first bit stream held in shared memory as big-endian 32-bit words,
// read through a 64-bit register window (one shared load per refill).
struct SmemBitReader {
  const uint32_t* win;
  uint32_t wi;  // next word to append
  uint64_t buf;
  int nb;
  __device__ __forceinline__ void init(const uint32_t* w, uint32_t pos) {
    win = w;
    wi = pos >> 5;
    const int sb = int(pos & 31);
    buf = ((uint64_t(win[wi]) << 32) | win[wi + 1]) << sb;
    nb = 64 - sb;
    wi += 2;
  }
  __device__ __forceinline__ void refill_uniform() {
    const bool need = nb <= 32;
    const uint32_t w = win[wi];
    buf |= need ? uint64_t(w) << (need ? 32 - nb : 0) : 0ull;
    nb += need ? 32 : 0;
    wi += need ? 1u : 0u;
  }
  __device__ __forceinline__ uint32_t peek32() const { return uint32_t(buf >> 32); }
  __device__ __forceinline__ void skip(int n) {
    buf <<= n;
    nb -= n;
  }
};

// ------------------------------------------------------------ cp.async -----
// 16-byte global -> shared copies that bypass registers (and L1: .cg), with
// per-thread commit groups.
__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gmem_src) {
  const uint32_t d = static_cast<uint32_t>(__cvta_generic_to_shared(smem_dst));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(d), "l"(gmem_src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;\n" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_1() { asm volatile("cp.async.wait_group 1;\n" ::: "memory"); }

// 96-bit MSB-first bit window w0:w1:w2 (nb valid bits) over a stream held in
// shared memory as big-endian words; wi is the next word to append, so the
// window head sits at bit 32*wi - nb.  One refill() keeps nb >= 65 when nb was
// >= 33, enough for several table-sized codes without further checks.
struct SmemWin96 {
  const uint32_t* win;
  uint32_t wi, w0, w1, w2;
  int nb;
  __device__ __forceinline__ void init(const uint32_t* w, uint32_t pos) {
    win = w;
    const uint32_t k = pos >> 5, sb = pos & 31;
    const uint32_t a = win[k], b = win[k + 1], c = win[k + 2];
    w0 = __funnelshift_l(b, a, sb);
    w1 = __funnelshift_l(c, b, sb);
    w2 = __funnelshift_l(0u, c, sb);
    nb = 96 - int(sb);
    wi = k + 3;
  }
  // Appends the next word when nb <= 64, without a branch (the word past the
  // window is always readable: callers keep padding words after their data).
  __device__ __forceinline__ void refill() {
    const bool need = nb <= 64;
    const uint32_t word = win[wi];  // unconditional load (in bounds), then a select
    const uint32_t t = need ? word : 0u;
    const bool low = nb < 32;
    // t lands at bit nb: its head ORs into w0 (nb < 32) or w1, its tail into
    // the next word; clamped funnel shifts keep every nb well defined
    const uint32_t k = uint32_t(low ? nb : nb - 32);
    const uint32_t head = __funnelshift_rc(t, 0u, k), tail = __funnelshift_rc(0u, t, k);
    w0 |= low ? head : 0u;
    w1 |= low ? tail : head;
    w2 |= low ? 0u : tail;
    nb += need ? 32 : 0;
    wi += need ? 1u : 0u;
  }
  // nb >= 65 afterwards from any nb >= 1.
  __device__ __forceinline__ void refill2() {
    refill();
    if (nb < 65) refill();
  }
  // nb >= NEED (<= 64) afterwards from any nb >= 1; the second word is
  // rarely needed, so the branch is almost always uniform.
  template <int NEED>
  __device__ __forceinline__ void refill_to() {
    refill();
    if (nb < NEED) refill();
  }
  __device__ __forceinline__ void skip(uint32_t n) {  // uses the low 5 bits of n
    w0 = __funnelshift_l(w1, w0, n);
    w1 = __funnelshift_l(w2, w1, n);
    w2 = __funnelshift_l(0u, w2, n);
    nb -= int(n & 31u);
  }
  // Shift only; the caller subtracts the consumed bits from nb later.
  __device__ __forceinline__ void shift(uint32_t n) {
    w0 = __funnelshift_l(w1, w0, n);
    w1 = __funnelshift_l(w2, w1, n);
    w2 = __funnelshift_l(0u, w2, n);
  }
  __device__ __forceinline__ uint32_t pos() const { return 32 * wi - uint32_t(nb); }
};

// The 16 bytes at byte offset off (0..15) of the 32 bytes lo:hi.
__device__ __forceinline__ uint4 realign16(const uint4& lo, const uint4& hi, int off) {
  if (off == 0) return lo;
  uint32_t w0 = lo.x, w1 = lo.y, w2 = lo.z, w3 = lo.w, w4 = hi.x, w5 = hi.y, w6 = hi.z, w7 = hi.w;
  if (off & 8) {
    w0 = w2; w1 = w3; w2 = w4; w3 = w5; w4 = w6; w5 = w7;
  }
  if (off & 4) {
    w0 = w1; w1 = w2; w2 = w3; w3 = w4; w4 = w5;
  }
  const int bs = (off & 3) * 8;
  return make_uint4(__funnelshift_r(w0, w1, bs), __funnelshift_r(w1, w2, bs),
                    __funnelshift_r(w2, w3, bs), __funnelshift_r(w3, w4, bs));
}

// 16 bytes from any address (two aligned loads and a byte funnel).
__device__ __forceinline__ uint4 ld16_any(const uint8_t* p) {
  const uintptr_t a = reinterpret_cast<uintptr_t>(p);
  const uint4* q = reinterpret_cast<const uint4*>(a & ~uintptr_t(15));
  const int off = int(a & 15);
  const uint4 lo = ldg16(q);
  if (off == 0) return lo;
  const uint4 hi = ldg16(q + 1);
  uint32_t w0 = lo.x, w1 = lo.y, w2 = lo.z, w3 = lo.w, w4 = hi.x, w5 = hi.y, w6 = hi.z, w7 = hi.w;
  if (off & 8) {
    w0 = w2; w1 = w3; w2 = w4; w3 = w5; w4 = w6; w5 = w7;
  }
  if (off & 4) {
    w0 = w1; w1 = w2; w2 = w3; w3 = w4; w4 = w5;
  }
  const int bs = (off & 3) * 8;
  return make_uint4(__funnelshift_r(w0, w1, bs), __funnelshift_r(w1, w2, bs),
                    __funnelshift_r(w2, w3, bs), __funnelshift_r(w3, w4, bs));
}

// One 32-byte store (a whole L2 sector) from eight words; dst must be 32-byte
// aligned.  sm_100 has 256-bit global stores: a lane's tile row then reaches
// L2 as one full-sector write instead of two half-sector writes.
__device__ __forceinline__ void st_global_32B(void* dst, const uint4& a, const uint4& b) {
  asm volatile("st.global.v8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"l"(dst), "r"(a.x), "r"(a.y),
               "r"(a.z), "r"(a.w), "r"(b.x), "r"(b.y), "r"(b.z), "r"(b.w)
               : "memory");
}

// ---------------------------------------------------- BF16 assembly -------
// Two BF16 words from two exponent bytes (e0 in bits 0-7, e1 in bits 8-15)
// and two sign/mantissa bytes (same places), packed low word first.
__device__ __forceinline__ uint32_t merge2(uint32_t e01, uint32_t s01) {
  uint32_t e = __byte_perm(e01, 0, 0x4140);  // [e0, 0, e1, 0]
  uint32_t s = __byte_perm(s01, 0, 0x1100);  // [s0, s0, s1, s1]
  return (e << 7) | (s & 0x807F807Fu);
}

// One BF16 word from a table entry holding exponent << 7 in bits 7-14.
__device__ __forceinline__ uint32_t merge1(uint32_t entry, uint32_t sm) {
  return (entry & 0x7F80u) | ((sm * 0x101u) & 0x807Fu);
}

// ---------------------------------------------------- tile geometry -------
// Row-major element index of tiled (packed) element p of a rows x cols slab
// (src/layout.cpp:32-50 visit order: 16-row blocks, 16-column tiles inside,
// rows inside a tile; edge tiles narrower/shorter).
__device__ __forceinline__ uint64_t untile_index(uint64_t p, uint64_t rows, uint64_t cols) {
  uint64_t blk = p / (16 * cols);
  uint64_t q = p - blk * 16 * cols;
  uint64_t nr = rows - blk * 16;
  nr = nr < 16 ? nr : 16;
  uint64_t t = q / (16 * nr);
  uint64_t w = cols - t * 16;
  w = w < 16 ? w : 16;
  uint64_t local = q - t * 16 * nr;
  uint64_t i = local / w, j = local - i * w;
  return (blk * 16 + i) * cols + t * 16 + j;
}

// -------------------------------------------------- generic decoder -------
// Bit-serial canonical decoding valid for every code length the format
// allows (1..255).  cnt[l] = number of codes of length l, sorted[] = symbols
// ordered by (length, symbol) (the canonical order of src/codec.cpp:11-29).
// Walking one bit at a time, d is the position of the current prefix among
// the prefixes not yet assigned at this length; d < cnt[l] is a hit.
// Returns the symbol and sets *len, or returns -1 for a prefix that no code
// can complete.
template <class BitFn>
__device__ __forceinline__ int generic_decode(BitFn bit_at, const uint16_t* cnt,
                                              const uint8_t* sorted, int maxlen, int* len) {
  uint32_t d = 0, idx = 0;
  for (int l = 1; l <= maxlen; ++l) {
    d = (d << 1) | bit_at(l - 1);
    uint32_t c = cnt[l];
    if (d < c) {
      *len = l;
      return sorted[idx + d];
    }
    d -= c;
    idx += c;
    if (d >= 256) return -1;  // more open prefixes than symbols remain
  }
  return -1;
}

}  // namespace xksv
