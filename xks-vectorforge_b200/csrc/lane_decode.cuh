// Lane-private canonical-Huffman decoding: one lane decodes one independent
// bit stream with its own codebook, all lanes of a warp at a common cadence.
// Used by the parallel-codec kernels (a lane per substream of a slab) and the
// fused tensor-core GEMM (a lane per serial-codec slab, from the tile index).
//
// Per lane, in shared memory and lane-minor ([entry][lane], so lane l only
// touches bank l/2 of a 16-bit table and bank l of a 32-bit one):
//   * canonical tables built from the codebook's 256 code lengths (the
//     canonical assignment of src/codec.cpp:11-29): a 2^PK-entry first level
//     for codes of length <= PK, a second level for lengths PK+1..PK+K2 under
//     the first NE escape prefixes, and a compact (length, symbol) list for
//     lengths up to PK+PNL (at most PLONG symbols);
//   * a 16-word ring of the stream's bits as big-endian words, fed by aligned
//     32-byte global loads held one chunk ahead in registers;
//   * a 4-slot ring of 16-byte cp.async copies of the sign/mantissa bytes.
// Codes are decoded four at a time from one 32-bit snapshot of the ring: four
// table lookups, each followed by a one-instruction shift; one check per block
// (total length <= 32 and a non-zero last entry) proves every code of the
// block, otherwise the block is redone code by code.
#pragma once
#include <cstdint>

#include "xksv_device.cuh"

namespace xksv {
namespace ldec {

template <int PK_, int K2_, int NE_, int PNL_, int PLONG_>
struct Cfg {
  static constexpr int PK = PK_;        // first-level table bits
  static constexpr int K2 = K2_;        // second level covers lengths PK+1 .. PK+K2
  static constexpr int NE = NE_;        // escape prefixes with a second-level table
  static constexpr int PNL = PNL_;      // long lengths held per lane: PK+1 .. PK+PNL
  static constexpr int PLONG = PLONG_;  // long symbols held per lane
  static constexpr int NROW2 = (NE << K2) + 1;  // second-level rows (the last is all zero)
  static_assert(PK == 6, "packed short-length counters cover lengths 1-4 and 5-6");
  static_assert(PK + PNL <= 32, "a code fits one 32-bit snapshot");
  static_assert(PLONG <= 255, "u8 long-symbol cursors");
};

template <class C>
struct Tables {
  uint16_t lut[1 << C::PK][32];  // exponent << 7 | length; 0 = no code of length <= PK
  uint16_t lut2[C::NROW2][32];   // second level: (PK+K2)-bit prefix - (L << K2); last row 0
  uint8_t cnt[C::PNL][32];       // number of codes of length PK+1+j (<= PLONG)
  uint8_t lsym[C::PLONG][32];    // long-code symbols, canonical (length, symbol) order
};

constexpr int BR = 16;            // bit-ring words per lane (power of two)
constexpr uint32_t kRingLow = 8;  // unread ring words kept at each 16-code group
constexpr int SMR = 4;            // 16-byte sign/mantissa slots per lane
static_assert(kRingLow + 8 <= BR, "a staged chunk fits whenever maintain() adds one");
using Ring = uint32_t (*)[32];    // [BR][32]
using SmRing = uint4 (*)[32];     // [SMR][32]

struct Code {
  uint32_t F;   // first code of length PK+1
  uint32_t L2;  // first escape prefix << K2 (second-level index origin)
  int maxlen;
};

// Where a lane's 256 code lengths come from, as 16-byte chunks (little-endian
// words): take() returns the next chunk in order; keep(k, v) is told the k-th
// non-zero chunk and kept(k, c16) must return it again (chunk c16) for the
// fill pass.
//
// From global memory: streamed through ByteReader16; the first three
// non-zero chunks are saved in 12 rows of the lane's column of `save` and
// later ones re-read.
struct GlobalLens {
  ByteReader16 rd;
  const uint8_t* lens;
  uint32_t (*save)[32];
  int lane;
  static constexpr bool kZeroLut2 = false;  // the caller zeroes lut2 before the build
  __device__ __forceinline__ GlobalLens(const uint8_t* l, uint32_t (*s)[32], int ln) : lens(l), save(s), lane(ln) {
    rd.init(l, l + 256);
  }
  __device__ __forceinline__ uint4 take() { return rd.take(); }
  __device__ __forceinline__ void keep(uint32_t k, const uint4& v) {
    if (k < 3) {
      const int r = 4 * int(k);
      save[r][lane] = v.x;
      save[r + 1][lane] = v.y;
      save[r + 2][lane] = v.z;
      save[r + 3][lane] = v.w;
    }
  }
  __device__ __forceinline__ uint4 kept(uint32_t k, int c16) const {
    if (k < 3) {
      const int r = 4 * int(k);
      return make_uint4(save[r][lane], save[r + 1][lane], save[r + 2][lane], save[r + 3][lane]);
    }
    return ld16_any(lens + 16 * c16);
  }
};

// From shared memory: the 17 aligned 16-byte chunks that cover the lengths,
// chunk c of this lane at chunk(c): areas of `per_area` chunks x 32 lanes,
// `stride` bytes apart, realigned by the lengths' offset in their first chunk.
struct SmemLens {
  static constexpr bool kZeroLut2 = false;  // the caller zeroes lut2 before the build
  const uint8_t* base;  // this lane's chunk 0
  uint32_t stride, per_area;
  int q, bs;            // word / bit offset of the first length in chunk 0
  int next;
  __device__ __forceinline__ SmemLens(const uint8_t* b, uint32_t s, uint32_t pa, uintptr_t lens_addr)
      : base(b), stride(s), per_area(pa), q(int((lens_addr >> 2) & 3)), bs(int(lens_addr & 3) * 8), next(0) {}
  __device__ __forceinline__ uint4 chunk(int c) const {
    const uint32_t a = uint32_t(c) / per_area, r = uint32_t(c) - a * per_area;
    return *reinterpret_cast<const uint4*>(base + a * stride + r * 512);
  }
  __device__ __forceinline__ uint4 at(int c) const {
    const uint4 r0 = chunk(c), r1 = chunk(c + 1);
    uint32_t w0 = r0.x, w1 = r0.y, w2 = r0.z, w3 = r0.w, w4 = r1.x, w5 = r1.y, w6 = r1.z, w7 = r1.w;
    if (q & 2) {
      w0 = w2; w1 = w3; w2 = w4; w3 = w5; w4 = w6; w5 = w7;
    }
    if (q & 1) {
      w0 = w1; w1 = w2; w2 = w3; w3 = w4; w4 = w5;
    }
    return make_uint4(__funnelshift_r(w0, w1, bs), __funnelshift_r(w1, w2, bs), __funnelshift_r(w2, w3, bs),
                      __funnelshift_r(w3, w4, bs));
  }
  __device__ __forceinline__ uint4 take() { return at(next++); }
  __device__ __forceinline__ void keep(uint32_t, const uint4&) {}
  __device__ __forceinline__ uint4 kept(uint32_t, int c16) const { return at(c16); }
};

// Staged in the lane's own table memory, idle until the fill pass: chunks
// 0-7 in the first-level table, 8-15 in the second-level table, 16 in the
// long-symbol list (each as [chunk][lane] 16-byte cells; stage_lengths()
// issues the copies).  The first three non-zero chunks are saved in 12 rows of
// `save` during the count pass, later ones re-read from global memory, since
// the fill pass overwrites the staging; the build zeroes this lane's column of
// the second-level table after the count pass.
template <class C>
struct TabLens {
  static constexpr bool kZeroLut2 = true;
  const uint4* lo;  // chunks 0-7: lo[32 * c]
  const uint4* mid; // chunks 8-15
  const uint4* hi;  // chunk 16
  const uint8_t* lens;
  uint32_t (*save)[32];
  int lane, q, bs, next;
  __device__ __forceinline__ TabLens(Tables<C>& T, const uint8_t* l, uint32_t (*s)[32], int ln)
      : lo(reinterpret_cast<const uint4*>(&T.lut[0][0]) + ln),
        mid(reinterpret_cast<const uint4*>(&T.lut2[0][0]) + ln),
        hi(reinterpret_cast<const uint4*>(&T.lsym[0][0]) + ln),
        lens(l), save(s), lane(ln),
        q(int((reinterpret_cast<uintptr_t>(l) >> 2) & 3)), bs(int(reinterpret_cast<uintptr_t>(l) & 3) * 8), next(0) {}
  __device__ __forceinline__ uint4 chunk(int c) const { return c < 8 ? lo[32 * c] : c < 16 ? mid[32 * (c - 8)] : *hi; }
  __device__ __forceinline__ uint4 take() {
    const uint4 r0 = chunk(next), r1 = chunk(next + 1);
    ++next;
    uint32_t w0 = r0.x, w1 = r0.y, w2 = r0.z, w3 = r0.w, w4 = r1.x, w5 = r1.y, w6 = r1.z, w7 = r1.w;
    if (q & 2) {
      w0 = w2; w1 = w3; w2 = w4; w3 = w5; w4 = w6; w5 = w7;
    }
    if (q & 1) {
      w0 = w1; w1 = w2; w2 = w3; w3 = w4; w4 = w5;
    }
    return make_uint4(__funnelshift_r(w0, w1, bs), __funnelshift_r(w1, w2, bs), __funnelshift_r(w2, w3, bs),
                      __funnelshift_r(w3, w4, bs));
  }
  __device__ __forceinline__ void keep(uint32_t k, const uint4& v) {
    if (k < 3) {
      const int r = 4 * int(k);
      save[r][lane] = v.x;
      save[r + 1][lane] = v.y;
      save[r + 2][lane] = v.z;
      save[r + 3][lane] = v.w;
    }
  }
  __device__ __forceinline__ uint4 kept(uint32_t k, int c16) const {
    if (k < 3) {
      const int r = 4 * int(k);
      return make_uint4(save[r][lane], save[r + 1][lane], save[r + 2][lane], save[r + 3][lane]);
    }
    return ld16_any(lens + 16 * c16);
  }
};

// Issues the cp.async copies TabLens reads: the aligned 16-byte chunks that
// hold the 256 code lengths at `lens` (the 17th only when the lengths are not
// 16-byte aligned, so every chunk read holds a length byte).
template <class C>
__device__ __forceinline__ void stage_lengths(Tables<C>& T, const uint8_t* lens, int lane) {
  static_assert(sizeof(T.lut) >= 8 * 512 && sizeof(T.lut2) >= 8 * 512 && sizeof(T.lsym) >= 512,
                "the tables hold the 17 staged chunks");
  static_assert(offsetof(Tables<C>, lut2) % 16 == 0 && offsetof(Tables<C>, lsym) % 16 == 0, "16-byte cells");
  const uintptr_t a = reinterpret_cast<uintptr_t>(lens);
  const uint8_t* c0 = reinterpret_cast<const uint8_t*>(a & ~uintptr_t(15));
  uint4* lo = reinterpret_cast<uint4*>(&T.lut[0][0]) + lane;
  uint4* mid = reinterpret_cast<uint4*>(&T.lut2[0][0]) + lane;
#pragma unroll
  for (int c = 0; c < 8; ++c) cp_async16(lo + 32 * c, c0 + 16 * c);
#pragma unroll
  for (int c = 0; c < 8; ++c) cp_async16(mid + 32 * c, c0 + 128 + 16 * c);
  if (a & 15) cp_async16(reinterpret_cast<uint4*>(&T.lsym[0][0]) + lane, c0 + 256);
}

// Builds lane `lane`'s tables from its 256 code lengths (read through `rd`).
// Returns 0 when built, 1 when the codebook does not fit them (a length
// above PK+PNL or more than PLONG long codes), -1 when the lengths are
// oversubscribed (the canonical assignment fails exactly then).  Only the
// non-zero length bytes are visited (a codebook uses a few dozen symbols at
// most).  Short-length counters and fill cursors are 8-bit fields of two
// registers (lengths 1-4 | 5-6); a field that wraps (256 codes of one
// length) shows as a count mismatch.  lut2 starts all zero: zeroed by the
// caller before the build, or here after the count pass (R::kZeroLut2).
template <class C, class R>
__device__ int build_tables(R& rd, Tables<C>& T, uint8_t (*lpos)[32], int lane, uint32_t& F, int& maxlen,
                            uint32_t& Lout) {
  constexpr int PK = C::PK, K2 = C::K2, NE = C::NE, PNL = C::PNL, PLONG = C::PLONG;
  uint32_t c14 = 0, c56 = 0, nshort = 0, nlong = 0;
  bool generic = false;
  uint32_t mx = 0;
#pragma unroll
  for (int j = 0; j < PNL; ++j) T.cnt[j][lane] = 0;
  uint32_t nz = 0;      // chunks holding a non-zero length
  uint32_t nkept = 0;   // non-zero chunks seen
  for (int c16 = 0; c16 < 16; ++c16) {
    const uint4 v = rd.take();
    if ((v.x | v.y | v.z | v.w) == 0) continue;
    nz |= 1u << c16;
    rd.keep(nkept++, v);
    const uint32_t wv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      uint32_t w = wv[q];
      while (w) {
        const uint32_t sh = uint32_t(__ffs(w) - 1) & ~7u;
        const uint32_t l = (w >> sh) & 255u;
        w &= ~(255u << sh);
        mx = max(mx, l);
        if (l <= PK) {
          ++nshort;
          if (l <= 4)
            c14 += 1u << (8 * (l - 1));
          else
            c56 += 1u << (8 * (l - 5));
        } else if (l <= PK + PNL) {
          // a u8 counter: more than PLONG long codes send the lane to the
          // caller's fallback, before any count is used
          T.cnt[l - PK - 1][lane] += 1;
          ++nlong;
        } else {
          generic = true;
        }
      }
    }
  }
  maxlen = int(mx);
  if (generic || nlong > PLONG) return 1;
  // first-level start row per short length (8-bit fields); Kraft check
  uint32_t s14 = 0, s56 = 0, L = 0, tot = 0;
#pragma unroll
  for (int l = 1; l <= PK; ++l) {
    const uint32_t c = (l <= 4 ? c14 >> (8 * (l - 1)) : c56 >> (8 * (l - 5))) & 255u;
    if (l <= 4)
      s14 |= (L & 255u) << (8 * (l - 1));
    else
      s56 |= (L & 255u) << (8 * (l - 5));
    L += c << (PK - l);
    tot += c;
  }
  if (tot != nshort || L > (1u << PK)) return -1;
  uint64_t used = L;
  uint32_t pos = 0;
  for (int l = PK + 1; l <= maxlen; ++l) {
    const uint32_t c = T.cnt[l - PK - 1][lane];
    used = (used << 1) + c;
    lpos[l - PK - 1][lane] = uint8_t(pos);
    pos += c;
  }
  if (maxlen > PK && used > (1ull << maxlen)) return -1;
  F = L << 1;
  if (R::kZeroLut2) {  // the second level held staged lengths until now
    for (int r = 0; r < C::NROW2; ++r) T.lut2[r][lane] = 0;
  }
  // fill pass over the non-zero chunks again
  uint32_t k = 0;
  while (nz) {
    const int c16 = __ffs(nz) - 1;
    nz &= nz - 1;
    const uint4 v = rd.kept(k, c16);
    ++k;
    const uint32_t wv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      uint32_t w = wv[q];
      while (w) {
        const uint32_t sh = uint32_t(__ffs(w) - 1) & ~7u;
        const uint32_t l = (w >> sh) & 255u;
        w &= ~(255u << sh);
        const uint32_t sym = uint32_t(c16 * 16 + q * 4) + (sh >> 3);
        if (l <= PK) {
          const bool lo = l <= 4;
          const uint32_t fs = 8 * (lo ? l - 1 : l - 5);
          const uint32_t run = 1u << (PK - l);
          const uint32_t st = ((lo ? s14 : s56) >> fs) & 255u;
          s14 += lo ? run << fs : 0u;
          s56 += lo ? 0u : run << fs;
          const uint16_t e = uint16_t((sym << 7) | l);
          for (uint32_t r = 0; r < run; ++r) T.lut[st + r][lane] = e;
        } else {
          const int j = int(l) - PK - 1;
          T.lsym[lpos[j][lane]][lane] = uint8_t(sym);
          lpos[j][lane] += 1;
        }
      }
    }
  }
  // rows past the short codes: prefixes of long codes or unused code space
  for (uint32_t z = L; z < (1u << PK); ++z) T.lut[z][lane] = 0;
  // second level (zeroed before the fill): codes of length
  // PK+1..PK+K2 whose (PK+K2)-bit prefixes fall in the first NE escape prefixes
  uint32_t cf = F, idx = 0;
  const uint32_t base = L << K2;
  for (int l = PK + 1; l <= maxlen && l <= PK + K2; ++l) {
    const uint32_t c = T.cnt[l - PK - 1][lane];
    for (uint32_t q = 0; q < c; ++q) {
      const uint32_t code = cf + q;
      const uint32_t run = 1u << (PK + K2 - l);
      const uint32_t st = (code << (PK + K2 - l)) - base;
      if (st + run <= uint32_t(NE << K2)) {
        const uint16_t e = uint16_t((uint32_t(T.lsym[idx + q][lane]) << 7) | uint32_t(l));
        for (uint32_t r = 0; r < run; ++r) T.lut2[st + r][lane] = e;
      }
    }
    idx += c;
    cf = (cf + c) << 1;
  }
  Lout = L;
  return 0;
}

// Entry for a code longer than PK bits at the top of w: exponent << 7 |
// length, or 0.
template <class C>
__device__ __noinline__ uint32_t long_entry(uint32_t w, const Tables<C>& T, int lane, uint32_t F, int maxlen) {
  uint32_t cf = F, idx = 0;
  for (int l = C::PK + 1; l <= maxlen; ++l) {
    const uint32_t v = w >> (32 - l);
    const uint32_t c = T.cnt[l - C::PK - 1][lane];
    if (v - cf < c) return (uint32_t(T.lsym[idx + v - cf][lane]) << 7) | uint32_t(l);
    idx += c;
    cf = (cf + c) << 1;
  }
  return 0;
}

// 32 bytes at a 32-byte aligned address (one sm_100 256-bit load).
struct Chunk32 {
  uint4 a, b;
};
__device__ __forceinline__ Chunk32 ldg32(const void* p) {
  Chunk32 c;
  asm volatile("ld.global.nc.v8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=r"(c.a.x), "=r"(c.a.y), "=r"(c.a.z), "=r"(c.a.w), "=r"(c.b.x), "=r"(c.b.y), "=r"(c.b.z),
                 "=r"(c.b.w)
               : "l"(p));
  return c;
}

// A lane's exponent bit stream.  Word w (counted from the 32-byte aligned
// chunk holding the stream's first byte) sits big-endian in ring[w % BR]; fw
// words have entered the ring and the next aligned chunk (`stage`) is already
// loaded into registers.  `pos` counts bits from that aligned start, so the
// stream's own bits begin at pos0 = 8 * (start & 31) + the first bit's offset
// in its byte.  Chunk loads are clamped to the last chunk holding stream
// bytes: only a corrupt stream reads past its end, and the final bit count
// rejects it.
struct Stream {
  const Chunk32* src;   // next chunk to load
  const Chunk32* last;  // last chunk holding stream bytes
  Chunk32 c0;           // first chunk (loaded before the table build)
  Chunk32 stage;        // next chunk, loaded, not yet in the ring
  uint32_t fw, pos, pos0;

  __device__ __forceinline__ Chunk32 fetch() {
    const Chunk32* q = src <= last ? src : last;
    ++src;
    return ldg32(q);
  }
  // Issues the first loads of the nbytes-byte stream at base (its first bit
  // is bit `bit0` < 8 of the first byte, MSB first); the ring is written by
  // init_ring() once the memory it may share is free.
  __device__ __forceinline__ void start(const uint8_t* base, uint64_t nbytes, uint32_t bit0 = 0) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(base);
    src = reinterpret_cast<const Chunk32*>(a & ~uintptr_t(31));
    last = reinterpret_cast<const Chunk32*>((a + (nbytes ? nbytes - 1 : 0)) & ~uintptr_t(31));
    pos0 = pos = uint32_t(a & 31) * 8 + bit0;
    c0 = fetch();
    stage = fetch();
  }
  // fw is always a multiple of 8 (chunks of 8 words from word 0), so a chunk
  // fills ring rows (fw % BR) .. +7 from one base address.
  __device__ __forceinline__ void put(Ring ring, int lane, const Chunk32& c) {
    static_assert(BR == 16, "a chunk fills one half of the ring");
    uint32_t* r = &ring[fw & 8][lane];
    r[0 * 32] = bswap32(c.a.x);
    r[1 * 32] = bswap32(c.a.y);
    r[2 * 32] = bswap32(c.a.z);
    r[3 * 32] = bswap32(c.a.w);
    r[4 * 32] = bswap32(c.b.x);
    r[5 * 32] = bswap32(c.b.y);
    r[6 * 32] = bswap32(c.b.z);
    r[7 * 32] = bswap32(c.b.w);
    fw += 8;
  }
  __device__ __forceinline__ void init_ring(Ring ring, int lane) {
    fw = 0;
    put(ring, lane, c0);
  }
  // Moves the staged chunk into the ring and loads the next one.
  __device__ __forceinline__ void advance(Ring ring, int lane) {
    put(ring, lane, stage);
    stage = fetch();
  }
  // Keeps at least kRingLow unread words in the ring: four checked blocks
  // (<= 32 bits each) and the last snapshot's second word need five; a chunk
  // enters only when it fits (fw - word <= BR - 8), so the chunk staged here
  // was loaded several groups earlier.
  __device__ __forceinline__ void maintain(Ring ring, int lane) {
    while (fw - (pos >> 5) < kRingLow) advance(ring, lane);
  }
  // The 32 bits at pos.
  __device__ __forceinline__ uint32_t snap(const uint32_t (*ring)[32], int lane) const {
    const uint32_t j = pos >> 5;
    const uint32_t a = ring[j & (BR - 1)][lane], b = ring[(j + 1) & (BR - 1)][lane];
    return __funnelshift_l(b, a, pos);
  }
};

// A lane's sign/mantissa bytes for 16-code groups: aligned 16-byte chunks
// staged by cp.async three groups ahead, realigned when a group is consumed.
struct SmStream {
  const uint4* src;
  const uint4* last;
  uint32_t g;   // chunk index of the next group's first byte
  int q, bs;    // word / bit offset of the stream start inside a chunk
  __device__ __forceinline__ void fetch(SmRing sr, int lane, uint32_t k) {
    const uint4* p = src + k <= last ? src + k : last;
    cp_async16(&sr[k & (SMR - 1)][lane], p);
  }
  __device__ __forceinline__ void init(SmRing sr, int lane, const uint8_t* p, const uint8_t* end) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(p);
    src = reinterpret_cast<const uint4*>(a & ~uintptr_t(15));
    last = reinterpret_cast<const uint4*>((reinterpret_cast<uintptr_t>(end) - 1) & ~uintptr_t(15));
    q = int((a >> 2) & 3);
    bs = int(a & 3) * 8;
    g = 0;
    fetch(sr, lane, 0);
    fetch(sr, lane, 1);
    fetch(sr, lane, 2);
  }
  // Stages the chunk three ahead of the group about to be consumed (its slot
  // held the chunk the previous group read first).
  __device__ __forceinline__ void stage(SmRing sr, int lane) { fetch(sr, lane, g + 3); }
  __device__ __forceinline__ uint4 take(const uint4 (*sr)[32], int lane) {
    const uint4 r0 = sr[g & (SMR - 1)][lane];
    const uint4 r1 = sr[(g + 1) & (SMR - 1)][lane];
    ++g;
    uint32_t w0 = r0.x, w1 = r0.y, w2 = r0.z, w3 = r0.w, w4 = r1.x, w5 = r1.y, w6 = r1.z, w7 = r1.w;
    if (q & 2) {
      w0 = w2; w1 = w3; w2 = w4; w3 = w5; w4 = w6; w5 = w7;
    }
    if (q & 1) {
      w0 = w1; w1 = w2; w2 = w3; w3 = w4; w4 = w5;
    }
    return make_uint4(__funnelshift_r(w0, w1, bs), __funnelshift_r(w1, w2, bs),
                      __funnelshift_r(w2, w3, bs), __funnelshift_r(w3, w4, bs));
  }
};

__device__ __forceinline__ void cp_async_wait_2() { asm volatile("cp.async.wait_group 2;\n" ::: "memory"); }

// Table lookup of the code at the top of w: exponent << 7 | length, or 0
// when neither level holds it.  No branch: a prefix outside the second level
// reads its all-zero last row, and a short code (first level) always has a
// prefix below the escape rows, so at most one level is non-zero.
template <class C>
__device__ __forceinline__ uint32_t lookup(uint32_t w, const Tables<C>& T, int lane, uint32_t L2) {
  const uint32_t e1 = T.lut[w >> (32 - C::PK)][lane];
  // min(prefix - L2, NE << K2) in one add-min (DPX) instruction
  const uint32_t i2 = __viaddmin_u32(w >> (32 - C::PK - C::K2), 0u - L2, uint32_t(C::NE << C::K2));
  return e1 | uint32_t(T.lut2[i2][lane]);
}

// One code at pos, with the compact long-code list behind the tables and a
// ring top-up first (any code the lane can hold has <= PK+PNL <= 32 bits).
template <class C>
__device__ __forceinline__ uint32_t dec_one(Stream& b, Ring ring, const Tables<C>& T, int lane, const Code& lc,
                                            bool& bad) {
  if (b.fw - (b.pos >> 5) < 2u) b.advance(ring, lane);  // the ring keeps >= 2 unread words
  const uint32_t w = b.snap(ring, lane);
  uint32_t e = lookup<C>(w, T, lane, lc.L2);
  if (e == 0) {
    e = long_entry<C>(w, T, lane, lc.F, lc.maxlen);
    if ((e & 31u) == 0) bad = true;
  }
  b.pos += e & 31u;
  return e;
}

// Four codes from one 32-bit snapshot.  A code k read from bits past the
// snapshot (its start s_k plus its length above 32) makes the block's total
// exceed 32; a code it decodes with s_k + length <= 32 used only real bits and
// is the true code (prefix property).  So total <= 32 and a non-zero last
// entry prove the whole block; anything else is redone code by code.
template <class C>
__device__ __forceinline__ void dec4(Stream& b, Ring ring, const Tables<C>& T, int lane, const Code& lc, bool& bad,
                                     uint32_t& e0, uint32_t& e1, uint32_t& e2, uint32_t& e3) {
  uint32_t w = b.snap(ring, lane);
  e0 = lookup<C>(w, T, lane, lc.L2);
  w = __funnelshift_l(0u, w, e0);  // w << (length & 31)
  e1 = lookup<C>(w, T, lane, lc.L2);
  w = __funnelshift_l(0u, w, e1);
  e2 = lookup<C>(w, T, lane, lc.L2);
  w = __funnelshift_l(0u, w, e2);
  e3 = lookup<C>(w, T, lane, lc.L2);
  // lengths sit in bits 0-4 above zero bits 5-6, so one sum carries all four
  const uint32_t s = (e0 + e1 + e2 + e3) & 127u;
  if (s > 32u || e3 == 0) {
    e0 = dec_one<C>(b, ring, T, lane, lc, bad);
    e1 = dec_one<C>(b, ring, T, lane, lc, bad);
    e2 = dec_one<C>(b, ring, T, lane, lc, bad);
    e3 = dec_one<C>(b, ring, T, lane, lc, bad);
    b.maintain(ring, lane);
  } else {
    b.pos += s;
  }
}

// Two BF16 words (e_lo, e_hi table entries; sign/mantissa bytes at byte
// positions `sel` of sw, 0x1100 for bytes 0-1 or 0x3322 for bytes 2-3).
__device__ __forceinline__ uint32_t merge2(uint32_t e_lo, uint32_t e_hi, uint32_t sw, uint32_t sel) {
  return (__byte_perm(e_lo, e_hi, 0x5410) & 0x7F807F80u) | (__byte_perm(sw, 0, sel) & 0x807F807Fu);
}

// One tile row of 16 BF16 words from 16 entries and 16 sign/mantissa bytes.
__device__ __forceinline__ void merge16(const uint32_t* e, const uint4& s16, uint4& v0, uint4& v1) {
  v0.x = merge2(e[0], e[1], s16.x, 0x1100);
  v0.y = merge2(e[2], e[3], s16.x, 0x3322);
  v0.z = merge2(e[4], e[5], s16.y, 0x1100);
  v0.w = merge2(e[6], e[7], s16.y, 0x3322);
  v1.x = merge2(e[8], e[9], s16.z, 0x1100);
  v1.y = merge2(e[10], e[11], s16.z, 0x3322);
  v1.z = merge2(e[12], e[13], s16.w, 0x1100);
  v1.w = merge2(e[14], e[15], s16.w, 0x3322);
}

}  // namespace ldec
}  // namespace xksv
