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
// MSB-first bit stream read through aligned 16-byte chunks.  `buf` holds the
// next bits left-aligned; `nb` is how many are valid (>= 32 after refill()).
// Reads past `end` (the stream's last byte + 1) return zero bits, so a
// corrupt stream can be decoded to its (wrong) end without leaving the buffer.
struct BitReader {
  const uint4* next;   // next aligned chunk to load
  const uint4* last;   // last chunk holding stream bytes
  uint4 cur;           // current chunk (byte-swapped to big-endian words)
  int cw;              // words of `cur` not yet moved into buf
  uint64_t buf;
  int nb;

  __device__ __forceinline__ void load_chunk() {
    uint4 c = make_uint4(0, 0, 0, 0);
    if (next <= last) c = ldg16(next);
    ++next;
    cur = make_uint4(bswap32(c.x), bswap32(c.y), bswap32(c.z), bswap32(c.w));
    cw = 4;
  }
  __device__ __forceinline__ uint32_t take_word() {
    if (cw == 0) load_chunk();
    uint32_t w = cur.x;
    cur.x = cur.y;
    cur.y = cur.z;
    cur.z = cur.w;
    --cw;
    return w;
  }
  // Positions the reader at bit `bit` of the stream starting at `base`.
  __device__ __forceinline__ void init(const uint8_t* base, uint64_t nbytes, uint64_t bit) {
    uintptr_t a = reinterpret_cast<uintptr_t>(base);
    const uint8_t* first = reinterpret_cast<const uint8_t*>(a & ~uintptr_t(15));
    uint64_t skip = uint64_t(a & 15) * 8 + bit;  // bits from `first`
    next = reinterpret_cast<const uint4*>(first) + (skip >> 7);
    last = reinterpret_cast<const uint4*>((a + (nbytes ? nbytes - 1 : 0)) & ~uintptr_t(15));
    if (nbytes == 0) last = reinterpret_cast<const uint4*>(first) - 1;
    load_chunk();
    int sw = int((skip >> 5) & 3);
    for (int i = 0; i < sw; ++i) take_word();
    buf = uint64_t(take_word()) << 32;
    buf |= take_word();
    int sb = int(skip & 31);
    buf <<= sb;
    nb = 64 - sb;
    refill();
  }
  __device__ __forceinline__ void refill() {
    if (nb <= 32) {
      uint64_t w = take_word();
      buf |= w << (32 - nb);
      nb += 32;
    }
  }
  __device__ __forceinline__ uint32_t peek32() const { return uint32_t(buf >> 32); }
  __device__ __forceinline__ void skip(int n) {
    buf <<= n;
    nb -= n;
  }
};

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
