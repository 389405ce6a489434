// "bf16-huffman-parallel32" (XKSP2) slabs: decode and fused GEMV/GEMM.
//
// Reference behaviour: cuda/parallel.cu:13-31 (one thread per substream,
// per-substream tree walk, packed->(row, col) mapping :23-24), header checks
// cuda/parallel.cu:33-53, CPU semantics src/c_api.cpp:66-85.
//
// B200 design: one warp per slab, one lane per substream (the format's up to
// 32 independently coded substreams are a warp's worth of independent work);
// many slabs in flight per SM.  Every per-lane event in the inner loop runs at
// a cadence shared by all lanes, so the warp never serialises on one lane:
//   * each lane builds its own canonical tables: a 2^PK-entry first level for
//     codes of length <= PK, a second level for lengths PK+1..PK+K2 under the
//     first NE escape prefixes, and a compact list for lengths up to PK+PNL.
//     Tables are lane-minor ([entry][lane]) so lookups never share a bank
//     beyond lane pairs;
//   * a lane's exponent bits are staged in a 4-slot shared ring by 16-byte
//     cp.async copies issued once per 16 codes, and read through a 64-bit
//     register window refilled from the ring once per 4 codes without a
//     data-dependent branch;
//   * sign/mantissa bytes arrive 16 at a time through a 3-deep register ring;
//   * 16 decoded BF16 words (one tile row) leave as one 32-byte store (two
//     16-byte stores when the output is only 16-byte aligned), un-tiled on the
//     fly, for 16-row slabs with cols % 16 == 0; other shapes use an
//     element-wise store path.
// A substream whose codebook the compact tables cannot hold (a length above
// PK+PNL or more than PLONG long codes, e.g. near-uniform exponents) is decoded
// afterwards by lane 0 with the bit-serial canonical decoder.
#include "kernels.h"
#include "xksv_device.cuh"

namespace xksv {
namespace {

constexpr int PK = 7;      // first-level table bits
constexpr int K2 = 5;      // second level covers lengths PK+1 .. PK+K2
constexpr int NE = 2;      // escape prefixes with a second-level table
constexpr int PNL = 16;    // long lengths held per lane: PK+1 .. PK+PNL
constexpr int PLONG = 32;  // long symbols held per lane
constexpr int RING = 4;    // 16-byte bit-stream slots per lane
constexpr int SMR = 4;     // 16-byte sign/mantissa slots per lane
constexpr int PWARPS = 2;  // slabs (warps) per CTA: small CTAs free their tables sooner
constexpr int PMAXB = 8;   // GEMM columns per pass

// One warp's tables, lane-minor so that lane l always touches bank l/2.
struct WarpTabs {
  uint16_t lut[1 << PK][32];      // exponent << 7 | length; 0 = no code of length <= PK
  uint16_t lut2[(NE << K2) + 1][32];  // second level: 12-bit prefix - (L << K2); last row 0
  uint16_t cnt[PNL][32];          // number of codes of length PK+1+j
  uint8_t lsym[PLONG][32];        // long-code symbols, canonical (length, symbol) order
  union {
    uint8_t lpos[PNL][32];        // fill cursor per long length (table build only)
    uint4 ring[RING][32];         // staged exponent-bit chunks (little-endian bytes)
  };
  uint4 smring[SMR][32];          // staged sign/mantissa chunks
};
// decode: the warps' tables; GEMM adds [16][PMAXB] row accumulators per warp
constexpr size_t kSmemTabs = PWARPS * sizeof(WarpTabs);
constexpr size_t kSmemBytes[2] = {kSmemTabs, kSmemTabs + PWARPS * 16 * PMAXB * sizeof(float)};

// Bit-serial tables for a substream the compact tables cannot hold; they
// overlay the warp's first-level tables once the fast lanes are done.
struct GenericTab {
  uint16_t cnt[256];
  uint16_t off[257];
  uint8_t sorted[256];
};
static_assert(sizeof(GenericTab) <= sizeof(WarpTabs::lut), "generic table fits");

struct Seg {
  const uint8_t* lens;
  const uint8_t* sm;
  const uint8_t* bits;
  uint32_t count;
  uint32_t start;  // packed index of the substream's first element
  uint64_t nbits;
  uint64_t ebytes;
};

__device__ __forceinline__ uint32_t byte_of(const uint4& v, int b) {
  const uint32_t w = b < 4 ? v.x : b < 8 ? v.y : b < 12 ? v.z : v.w;
  return (w >> (8 * (b & 3))) & 255u;
}

// Builds the lane's tables.  Returns 0 when built, 1 when the codebook needs
// the generic decoder, -1 when the lengths are oversubscribed (the canonical
// assignment of src/codec.cpp:11-29 fails exactly then).
__device__ int build_lane_tables(const uint8_t* lens, WarpTabs& W, int lane, uint32_t& F,
                                 int& maxlen, uint32_t& Lout) {
  uint64_t c_lo = 0, c_hi = 0;  // 16-bit counters: lengths 1-4 | 5-PK
  uint32_t nlong = 0;
  bool generic = false;
  maxlen = 0;
#pragma unroll
  for (int j = 0; j < PNL; ++j) W.cnt[j][lane] = 0;
  uint32_t nz = 0;  // chunks holding a non-zero length
  for (int g = 0; g < 16; g += 4) {
    uint4 vv[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) vv[k] = ld16_any(lens + 16 * (g + k));
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const uint4 v = vv[k];
      if ((v.x | v.y | v.z | v.w) == 0) continue;
      nz |= 1u << (g + k);
#pragma unroll
      for (int b = 0; b < 16; ++b) {
        const uint32_t l = byte_of(v, b);
        if (!l) continue;
        maxlen = max(maxlen, int(l));
        if (l <= 4)
          c_lo += 1ull << (16 * (l - 1));
        else if (l <= PK)
          c_hi += 1ull << (16 * (l - 5));
        else if (l <= PK + PNL) {
          W.cnt[l - PK - 1][lane] += 1;
          ++nlong;
        } else
          generic = true;
      }
    }
  }
  if (generic || nlong > PLONG) return 1;
  // first-level start row per short length; Kraft check
  uint64_t s_lo = 0, s_hi = 0;
  uint32_t L = 0;
#pragma unroll
  for (int l = 1; l <= PK; ++l) {
    const uint32_t c = l <= 4 ? uint32_t(c_lo >> (16 * (l - 1))) & 0xFFFFu
                              : uint32_t(c_hi >> (16 * (l - 5))) & 0xFFFFu;
    if (l <= 4)
      s_lo |= uint64_t(L) << (16 * (l - 1));
    else
      s_hi |= uint64_t(L) << (16 * (l - 5));
    L += c << (PK - l);
  }
  if (L > (1u << PK)) return -1;
  uint64_t used = L;
  uint32_t pos = 0;
  for (int l = PK + 1; l <= maxlen; ++l) {
    const uint32_t c = W.cnt[l - PK - 1][lane];
    used = (used << 1) + c;
    W.lpos[l - PK - 1][lane] = uint8_t(pos);
    pos += c;
  }
  if (maxlen > PK && used > (1ull << maxlen)) return -1;
  F = L << 1;
  // fill, re-reading only the non-zero chunks
  while (nz) {
    const int c16 = __ffs(nz) - 1;
    nz &= nz - 1;
    const uint4 v = ld16_any(lens + 16 * c16);
#pragma unroll
    for (int b = 0; b < 16; ++b) {
      const uint32_t l = byte_of(v, b);
      if (!l) continue;
      const uint32_t s = uint32_t(c16 * 16 + b);
      if (l <= PK) {
        uint32_t st;
        if (l <= 4) {
          st = uint32_t(s_lo >> (16 * (l - 1))) & 0xFFFFu;
          s_lo += uint64_t(1u << (PK - l)) << (16 * (l - 1));
        } else {
          st = uint32_t(s_hi >> (16 * (l - 5))) & 0xFFFFu;
          s_hi += uint64_t(1u << (PK - l)) << (16 * (l - 5));
        }
        const uint16_t e = uint16_t((s << 7) | l);
        const uint32_t run = 1u << (PK - l);
        for (uint32_t k = 0; k < run; ++k) W.lut[st + k][lane] = e;
      } else {
        const int j = int(l) - PK - 1;
        W.lsym[W.lpos[j][lane]][lane] = uint8_t(s);
        W.lpos[j][lane] += 1;
      }
    }
  }
  // rows past the short codes: prefixes of long codes or unused code space
  for (uint32_t z = L; z < (1u << PK); ++z) W.lut[z][lane] = 0;
  // second level: codes of length PK+1..PK+K2 whose (PK+K2)-bit prefixes fall
  // in the first NE escape prefixes
  for (int z = 0; z <= (NE << K2); ++z) W.lut2[z][lane] = 0;
  if (NE == 0) {
    Lout = L;
    return 0;
  }
  uint32_t cf = F, idx = 0;
  const uint32_t base = L << K2;
  for (int l = PK + 1; l <= maxlen && l <= PK + K2; ++l) {
    const uint32_t c = W.cnt[l - PK - 1][lane];
    for (uint32_t k = 0; k < c; ++k) {
      const uint32_t code = cf + k;
      const uint32_t run = 1u << (PK + K2 - l);
      const uint32_t st = (code << (PK + K2 - l)) - base;
      if (st + run <= uint32_t(NE << K2)) {
        const uint16_t e = uint16_t((uint32_t(W.lsym[idx + k][lane]) << 7) | uint32_t(l));
        for (uint32_t q = 0; q < run; ++q) W.lut2[st + q][lane] = e;
      }
    }
    idx += c;
    cf = (cf + c) << 1;
  }
  Lout = L;
  return 0;
}

// Entry for a code longer than PK bits: exponent << 7 | length, or 0.
__device__ __noinline__ uint32_t long_entry(uint32_t w, const WarpTabs& W, int lane, uint32_t F,
                                            int maxlen) {
  uint32_t cf = F, idx = 0;
  for (int l = PK + 1; l <= maxlen; ++l) {
    const uint32_t v = w >> (32 - l);
    const uint32_t c = W.cnt[l - PK - 1][lane];
    if (v - cf < c) return (uint32_t(W.lsym[idx + v - cf][lane]) << 7) | uint32_t(l);
    idx += c;
    cf = (cf + c) << 1;
  }
  return 0;
}

// A lane's exponent bits: 16-byte chunks staged by cp.async into the lane's
// RING slots (fw = words fetched, rw = words consumed), read through a 96-bit
// window w0:w1:w2 holding nb valid bits (MSB first).  One refill per four
// codes keeps nb >= 65, so four codes of up to PK+K2 bits need no check.
struct LaneBits {
  const uint4* src;   // next chunk to fetch
  const uint4* last;  // last chunk holding stream bytes (fetches are clamped to it)
  uint32_t fw, rw, rw0, skipb;
  uint32_t w0, w1, w2;
  int nb;

  __device__ __forceinline__ void fetch(WarpTabs& W, int lane) {
    const uint4* q = src <= last ? src : last;
    cp_async16(&W.ring[(fw >> 2) & (RING - 1)][lane], q);
    ++src;
    fw += 4;
  }
  __device__ __forceinline__ uint32_t word(const WarpTabs& W, int lane, uint32_t k) const {
    return bswap32(reinterpret_cast<const uint32_t*>(&W.ring[(k >> 2) & (RING - 1)][lane])[k & 3]);
  }
  __device__ __forceinline__ void init(WarpTabs& W, int lane, const uint8_t* base, uint64_t nbytes) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(base);
    src = reinterpret_cast<const uint4*>(a & ~uintptr_t(15));
    last = reinterpret_cast<const uint4*>((a + (nbytes ? nbytes - 1 : 0)) & ~uintptr_t(15));
    fw = 0;
    for (int k = 0; k < RING; ++k) fetch(W, lane);
    cp_async_commit();
    cp_async_wait_all();
    rw0 = rw = uint32_t(a & 15) >> 2;
    skipb = uint32_t(a & 3) * 8;
    w0 = word(W, lane, rw);
    w1 = word(W, lane, rw + 1);
    w2 = word(W, lane, rw + 2);
    rw += 3;
    w0 = __funnelshift_l(w1, w0, skipb);
    w1 = __funnelshift_l(w2, w1, skipb);
    w2 = __funnelshift_l(0u, w2, skipb);
    nb = 96 - int(skipb);
  }
  // Once per 16 codes (every lane at the same point): keep >= 8 unread words
  // staged, and make sure every staged word this stretch may read has landed.
  __device__ __forceinline__ void maintain(WarpTabs& W, int lane) {
    int nf = 0;
    while (fw - rw <= uint32_t(4 * RING - 4)) {
      fetch(W, lane);
      ++nf;
    }
    cp_async_commit();
    if (nf <= 1 && fw - rw >= uint32_t(4 * RING - 4))
      cp_async_wait_1();
    else
      cp_async_wait_all();
  }
  // Inserts the next word at bit nb when nb <= 64, without a data-dependent
  // branch (needs nb >= 1).
  __device__ __forceinline__ void refill(const WarpTabs& W, int lane) {
    const bool need = nb <= 64;
    const uint32_t wd = word(W, lane, rw);  // unconditional load of a ring slot, then a select
    const uint32_t t = need ? wd : 0u;
    const bool low = nb < 32;  // lands in w0:w1, else in w1:w2
    const uint32_t k = uint32_t(low ? nb : nb - 32);
    const uint32_t head = __funnelshift_rc(t, 0u, k), tail = __funnelshift_rc(0u, t, k);
    w0 |= low ? head : 0u;
    w1 |= low ? tail : head;
    w2 |= low ? 0u : tail;
    nb += need ? 32 : 0;
    rw += need ? 1u : 0u;
  }
  __device__ __forceinline__ void skip(uint32_t n) {  // n: low 5 bits used
    w0 = __funnelshift_l(w1, w0, n);
    w1 = __funnelshift_l(w2, w1, n);
    w2 = __funnelshift_l(0u, w2, n);
    nb -= int(n & 31u);
  }
  __device__ __forceinline__ void shift(uint32_t n) {  // skip without updating nb
    w0 = __funnelshift_l(w1, w0, n);
    w1 = __funnelshift_l(w2, w1, n);
    w2 = __funnelshift_l(0u, w2, n);
  }
  __device__ __forceinline__ uint64_t consumed() const {
    return uint64_t(rw - rw0) * 32 - uint64_t(nb) - skipb;
  }
};

// A lane's sign/mantissa bytes for 16-code groups: aligned 16-byte chunks
// staged by cp.async two groups ahead, realigned when a group is consumed.
struct LaneSm {
  const uint4* src;
  const uint4* last;
  uint32_t g;   // chunk index of the next group's first byte
  int q, bs;    // word / bit offset of the stream start inside a chunk
  __device__ __forceinline__ void fetch(WarpTabs& W, int lane, uint32_t k) {
    const uint4* p = src + k <= last ? src + k : last;
    cp_async16(&W.smring[k & (SMR - 1)][lane], p);
  }
  __device__ __forceinline__ void init(WarpTabs& W, int lane, const uint8_t* p, const uint8_t* end) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(p);
    src = reinterpret_cast<const uint4*>(a & ~uintptr_t(15));
    last = reinterpret_cast<const uint4*>((reinterpret_cast<uintptr_t>(end) - 1) & ~uintptr_t(15));
    q = int((a >> 2) & 3);
    bs = int(a & 3) * 8;
    g = 0;
    fetch(W, lane, 0);
    fetch(W, lane, 1);
    fetch(W, lane, 2);
  }
  // Called in step with LaneBits::maintain (same commit group): stages the
  // chunk three ahead of the group about to be consumed.
  __device__ __forceinline__ void stage(WarpTabs& W, int lane) { fetch(W, lane, g + 3); }
  __device__ __forceinline__ uint4 take(const WarpTabs& W, int lane) {
    const uint4 r0 = W.smring[g & (SMR - 1)][lane];
    const uint4 r1 = W.smring[(g + 1) & (SMR - 1)][lane];
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

struct LaneCode {
  uint32_t F;  // first code of length PK+1
  uint32_t L;  // first escape prefix (PK-bit units)
  int maxlen;
};

// Codes the two table levels do not hold (longer than PK+K2 bits, or beyond
// the covered escape prefixes): the compact list, then a top-up of the window
// and the ring so the rest of the group still has its bits.
__device__ __forceinline__ void top_up(LaneBits& b, WarpTabs& W, int lane) {
  if (b.nb < 65) {
    if (b.rw + 1 >= b.fw) {
      b.fetch(W, lane);
      cp_async_commit();
    }
    if (b.rw + 4 >= b.fw) cp_async_wait_all();
    b.refill(W, lane);
  }
}

__device__ __forceinline__ uint32_t rare_entry(LaneBits& b, WarpTabs& W, int lane,
                                            const LaneCode& lc, bool& bad) {
  top_up(b, W, lane);  // >= 33 bits: a whole long code (<= PK+PNL bits) is in w0
  uint32_t e = long_entry(b.w0, W, lane, lc.F, lc.maxlen);
  if ((e & 31u) == 0) bad = true;
  b.skip(e);
  top_up(b, W, lane);
  return e;
}

// Table lookup of the code at the window head: exponent << 7 | length, or 0
// when neither level holds it.  No branch: a prefix outside the second level
// reads its all-zero last row, and a short code (first level) always has a
// prefix below the escape rows, so at most one level is non-zero.
__device__ __forceinline__ uint32_t lookup(const LaneBits& b, const WarpTabs& W, int lane,
                                          uint32_t L5) {
  const uint32_t h = b.w0;
  const uint32_t e1 = W.lut[h >> (32 - PK)][lane];
  const uint32_t i2 = min((h >> (32 - PK - K2)) - L5, uint32_t(NE << K2));
  return e1 | uint32_t(W.lut2[i2][lane]);
}

// One code with the rare path.
__device__ __forceinline__ uint32_t dec(LaneBits& b, WarpTabs& W, int lane, const LaneCode& lc,
                                       bool& bad) {
  const uint32_t e = lookup(b, W, lane, lc.L << K2);
  if (e == 0) return rare_entry(b, W, lane, lc, bad);
  b.skip(e);
  return e;
}

// Four codes from a window holding >= 4*(PK+K2) bits, without a branch in the
// common case.  A code neither level holds has entry 0, which skips no bits,
// so the rest of the block looks up the same code and is 0 too: e3 == 0 tells
// that the window stopped at such a code, and the block finishes code by code
// from there.
__device__ __forceinline__ void dec4(LaneBits& b, WarpTabs& W, int lane, const LaneCode& lc,
                                     bool& bad, uint32_t& e0, uint32_t& e1, uint32_t& e2,
                                     uint32_t& e3) {
  const uint32_t L5 = lc.L << K2;
  e0 = lookup(b, W, lane, L5);
  b.shift(e0);
  e1 = lookup(b, W, lane, L5);
  b.shift(e1);
  e2 = lookup(b, W, lane, L5);
  b.shift(e2);
  e3 = lookup(b, W, lane, L5);
  b.shift(e3);
  // lengths sit in bits 0-4 above zero bits 5-6, so one sum carries all four
  b.nb -= int((e0 + e1 + e2 + e3) & 127u);
  if (e3 == 0) {
    if (e0 == 0) e0 = dec(b, W, lane, lc, bad);
    if (e1 == 0) e1 = dec(b, W, lane, lc, bad);
    if (e2 == 0) e2 = dec(b, W, lane, lc, bad);
    e3 = dec(b, W, lane, lc, bad);
  }
}

struct Out {
  uint16_t* out;   // decode: slab output
  const float* x;  // GEMM: X at this slab's column 0 (row stride ld)
  float* ysm;      // GEMM: [16][PMAXB] warp accumulators
  uint32_t rows, cols, ld, nb;
  bool xvec;       // GEMM: nb == 1, ld == 1, 16-byte aligned x
  bool out32;      // decode: 32-byte aligned output (one 256-bit store per tile row)
};

template <int MODE>
__device__ __forceinline__ void emit_one(const Out& o, uint32_t p, uint32_t word) {
  const uint64_t idx = untile_index(p, o.rows, o.cols);
  if (MODE == 0) {
    o.out[idx] = uint16_t(word);
  } else {
    const uint32_t r = uint32_t(idx / o.cols), c = uint32_t(idx - uint64_t(r) * o.cols);
    const float w = __uint_as_float(word << 16);
    for (uint32_t b = 0; b < o.nb; ++b)
      atomicAdd(&o.ysm[r * PMAXB + b], w * __ldg(&o.x[uint64_t(c) * o.ld + b]));
  }
}

// Decodes one substream.  `nice`: 16-row slab, cols % 16 == 0 and (decode)
// 16-byte aligned output; whole tile rows then leave as two 16-byte stores.
template <int MODE>
__device__ void decode_segment(const Seg& s, WarpTabs& W, int lane, const LaneCode& lc,
                               bool nice, const Out& o, bool& bad) {
  const bool rows16 = nice && (s.start & 15) == 0;
  LaneSm smr;
  if (rows16) smr.init(W, lane, s.sm, s.sm + s.count);
  LaneBits b;
  b.init(W, lane, s.bits, s.ebytes);  // its commit/wait also covers the first sm chunks
  uint32_t i = 0, p = s.start;
  while (i < s.count) {
    if (rows16) smr.stage(W, lane);
    b.maintain(W, lane);
    const uint32_t n = min(16u, s.count - i);
    if (rows16 && n == 16) {
      const uint4 s16 = smr.take(W, lane);
      uint32_t e[16];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        b.refill(W, lane);
        if (b.nb < 4 * (PK + K2)) b.refill(W, lane);  // rare: four codes of <= PK+K2 bits
        dec4(b, W, lane, lc, bad, e[4 * k], e[4 * k + 1], e[4 * k + 2], e[4 * k + 3]);
      }
      const uint32_t r = (p >> 4) & 15, c = (p >> 8) * 16;
      if (MODE == 0) {
        uint4 v0, v1;
        v0.x = (__byte_perm(e[0], e[1], 0x5410) & 0x7F807F80u) | (__byte_perm(s16.x, 0, 0x1100) & 0x807F807Fu);
        v0.y = (__byte_perm(e[2], e[3], 0x5410) & 0x7F807F80u) | (__byte_perm(s16.x, 0, 0x3322) & 0x807F807Fu);
        v0.z = (__byte_perm(e[4], e[5], 0x5410) & 0x7F807F80u) | (__byte_perm(s16.y, 0, 0x1100) & 0x807F807Fu);
        v0.w = (__byte_perm(e[6], e[7], 0x5410) & 0x7F807F80u) | (__byte_perm(s16.y, 0, 0x3322) & 0x807F807Fu);
        v1.x = (__byte_perm(e[8], e[9], 0x5410) & 0x7F807F80u) | (__byte_perm(s16.z, 0, 0x1100) & 0x807F807Fu);
        v1.y = (__byte_perm(e[10], e[11], 0x5410) & 0x7F807F80u) | (__byte_perm(s16.z, 0, 0x3322) & 0x807F807Fu);
        v1.z = (__byte_perm(e[12], e[13], 0x5410) & 0x7F807F80u) | (__byte_perm(s16.w, 0, 0x1100) & 0x807F807Fu);
        v1.w = (__byte_perm(e[14], e[15], 0x5410) & 0x7F807F80u) | (__byte_perm(s16.w, 0, 0x3322) & 0x807F807Fu);
        uint4* dst = reinterpret_cast<uint4*>(o.out + size_t(r) * o.cols + c);
        if (o.out32) {
          st_global_32B(dst, v0, v1);
        } else {
          dst[0] = v0;
          dst[1] = v1;
        }
      } else {
        float wf[16];
        const uint32_t sw[4] = {s16.x, s16.y, s16.z, s16.w};
#pragma unroll
        for (int k = 0; k < 16; ++k)
          wf[k] = __uint_as_float(merge1(e[k], (sw[k >> 2] >> (8 * (k & 3))) & 255u) << 16);
        if (o.xvec) {
          const float4* xv = reinterpret_cast<const float4*>(o.x + c);
          float acc = 0.f;
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const float4 xq = __ldg(xv + q);
            acc = fmaf(wf[4 * q], xq.x, acc);
            acc = fmaf(wf[4 * q + 1], xq.y, acc);
            acc = fmaf(wf[4 * q + 2], xq.z, acc);
            acc = fmaf(wf[4 * q + 3], xq.w, acc);
          }
          atomicAdd(&o.ysm[r * PMAXB], acc);
        } else {
          for (uint32_t bb = 0; bb < o.nb; ++bb) {
            float acc = 0.f;
#pragma unroll
            for (int k = 0; k < 16; ++k) acc = fmaf(wf[k], __ldg(&o.x[uint64_t(c + k) * o.ld + bb]), acc);
            atomicAdd(&o.ysm[r * PMAXB + bb], acc);
          }
        }
      }
    } else {
      for (uint32_t k = 0; k < n; ++k) {
        b.refill(W, lane);
        if (b.nb < 65) b.refill(W, lane);
        const uint32_t e = dec(b, W, lane, lc, bad);
        emit_one<MODE>(o, p + k, merge1(e, __ldg(s.sm + i + k)));
      }
    }
    i += n;
    p += n;
  }
  cp_async_wait_all();
  if (b.consumed() != s.nbits) bad = true;
}

// Lane 0 decodes a substream whose codebook needs the generic decoder.
template <int MODE>
__device__ bool decode_segment_generic(const Seg& s, GenericTab& G, const Out& o) {
  for (int l = 0; l < 256; ++l) G.cnt[l] = 0;
  int maxlen = 0;
  for (int sym = 0; sym < 256; ++sym) {
    const int l = __ldg(s.lens + sym);
    if (l) {
      G.cnt[l] += 1;
      maxlen = max(maxlen, l);
    }
  }
  int64_t avail = 1;  // Kraft check: open prefixes per level, clamped past 256
  for (int l = 1; l <= maxlen; ++l) {
    avail = 2 * avail - G.cnt[l];
    if (avail < 0) return false;
    if (avail > 4096) avail = 4096;
  }
  G.off[0] = 0;
  for (int l = 1; l <= 256; ++l) G.off[l] = uint16_t(G.off[l - 1] + G.cnt[l - 1]);
  for (int sym = 0; sym < 256; ++sym) {
    const int l = __ldg(s.lens + sym);
    if (l) G.sorted[G.off[l]++] = uint8_t(sym);
  }
  uint64_t pos = 0;
  for (uint32_t i = 0; i < s.count; ++i) {
    int len = 0;
    auto bit_at = [&](int k) -> uint32_t {
      const uint64_t q = pos + uint64_t(k);
      return q < s.nbits ? (__ldg(s.bits + (q >> 3)) >> (7 - (q & 7))) & 1u : 0u;
    };
    const int sym = generic_decode(bit_at, G.cnt, G.sorted, maxlen, &len);
    if (sym < 0) return false;
    pos += uint64_t(len);
    if (pos > s.nbits) return false;
    emit_one<MODE>(o, s.start + i, merge1(uint32_t(sym) << 7, __ldg(s.sm + i)));
  }
  return pos == s.nbits;
}

__device__ __forceinline__ uint64_t warp_incl_scan(uint64_t v, int lane) {
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    const uint64_t t = __shfl_up_sync(0xffffffffu, v, d);
    if (lane >= d) v += t;
  }
  return v;
}

template <int MODE>
__global__ void __launch_bounds__(PWARPS * 32)
    parallel_slab_kernel(const Slab* __restrict__ slabs, uint32_t nslabs,
                         const uint8_t* __restrict__ payload, uint8_t* __restrict__ out,
                         const float* __restrict__ x, float* __restrict__ y, uint32_t ld,
                         uint32_t nb, int* __restrict__ status) {
  extern __shared__ __align__(16) uint8_t smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  WarpTabs& W = reinterpret_cast<WarpTabs*>(smem)[warp];
  float* ysm = MODE == 1 ? reinterpret_cast<float*>(smem + kSmemTabs) + warp * 16 * PMAXB : nullptr;

  for (uint32_t si = blockIdx.x * PWARPS + warp; si < nslabs; si += gridDim.x * PWARPS) {
    const Slab sd = slabs[si];
    const uint8_t* p = payload + sd.src;
    const uint64_t n = sd.size;
    // ---- container header (cuda/parallel.cu:34-36) ----
    bool ok = n >= 32;
    uint64_t rows = 0, cols = 0, chunks = 0;
    if (ok) {
      ok = ld_le64(p) == 0x0000003250534B58ull;  // "XKSP2\0\0\0"
      rows = ld_le64(p + 8);
      cols = ld_le64(p + 16);
      chunks = ld_le64(p + 24);
      ok = ok && rows && rows <= 16 && cols && chunks && chunks <= 32 &&
           cols <= ~0ull / rows && chunks <= rows * cols && rows * cols <= n &&
           rows * cols <= ~0ull / 32 && n >= 32 + 8 * chunks && rows == sd.rows &&
           cols == sd.cols;
    }
    if (!ok) {
      if (lane == 0) atomicOr(status, kStatusHeader);
      continue;
    }
    if (rows * cols >= (1ull << 31)) {  // this implementation indexes elements in 32 bits
      if (lane == 0) atomicOr(status, kStatusInternal);
      continue;
    }
    // ---- substream table (cuda/parallel.cu:39-51) ----
    const uint32_t total = uint32_t(rows * cols);
    const bool active = uint64_t(lane) < chunks;
    const uint64_t len = active ? ld_le64(p + 32 + 8 * lane) : 0;
    bool lok = !active || (len >= kHdr && len <= n);
    const uint64_t incl = warp_incl_scan(lok ? len : 0, lane);
    const uint64_t base = 32 + 8 * chunks + incl - len;
    Seg s{};
    if (active && lok) {
      lok = base + len <= n;
      if (lok) {
        const uint8_t* q = p + base;
        const uint64_t count = ld_le64(q);
        s.nbits = ld_le64(q + 8);
        s.start = uint32_t(uint64_t(total) * uint64_t(lane) / chunks);
        const uint64_t expect = uint64_t(total) * uint64_t(lane + 1) / chunks - s.start;
        s.ebytes = s.nbits / 8 + (s.nbits % 8 != 0);
        lok = count == expect && count <= len - kHdr && s.ebytes == len - kHdr - count;
        s.count = uint32_t(count);
        s.lens = q + 16;
        s.sm = q + kHdr;
        s.bits = q + kHdr + count;
      }
    }
    const uint64_t end_all = __shfl_sync(0xffffffffu, base + len, int(chunks - 1));
    if (!(__all_sync(0xffffffffu, lok) && end_all == n)) {
      if (lane == 0) atomicOr(status, kStatusHeader);
      continue;
    }
    // ---- per-lane tables ----
    LaneCode lc{0, 0, 0};
    const int tb = active ? build_lane_tables(s.lens, W, lane, lc.F, lc.maxlen, lc.L) : 0;
    if (__any_sync(0xffffffffu, tb < 0)) {
      if (lane == 0) atomicOr(status, kStatusCodebook);
      continue;
    }
    __syncwarp();  // every lane's build is done before the bit ring (over lpos) fills
    Out o;
    o.out = reinterpret_cast<uint16_t*>(out + sd.dst);
    o.x = MODE == 1 ? x + sd.xoff * ld : nullptr;
    o.ysm = ysm;
    o.rows = uint32_t(rows);
    o.cols = uint32_t(cols);
    o.ld = ld;
    o.nb = nb;
    o.xvec = nb == 1 && ld == 1 && (reinterpret_cast<uintptr_t>(o.x) & 15) == 0;
    o.out32 = (reinterpret_cast<uintptr_t>(o.out) & 31) == 0;
    if (MODE == 1) {
      for (int k = lane; k < 16 * PMAXB; k += 32) ysm[k] = 0.f;
      __syncwarp();
    }
    const bool nice = rows == 16 && (cols & 15) == 0 &&
                      (MODE == 1 || (reinterpret_cast<uintptr_t>(o.out) & 15) == 0);
    bool bad = false;
    if (active && tb == 0) decode_segment<MODE>(s, W, lane, lc, nice, o, bad);
    // ---- substreams that need the generic decoder ----
    uint32_t gmask = __ballot_sync(0xffffffffu, active && tb == 1);
    __syncwarp();
    while (gmask) {
      const int g = __ffs(gmask) - 1;
      gmask &= gmask - 1;
      Seg sg;
      sg.lens = reinterpret_cast<const uint8_t*>(__shfl_sync(0xffffffffu, reinterpret_cast<uintptr_t>(s.lens), g));
      sg.sm = reinterpret_cast<const uint8_t*>(__shfl_sync(0xffffffffu, reinterpret_cast<uintptr_t>(s.sm), g));
      sg.bits = reinterpret_cast<const uint8_t*>(__shfl_sync(0xffffffffu, reinterpret_cast<uintptr_t>(s.bits), g));
      sg.count = __shfl_sync(0xffffffffu, s.count, g);
      sg.start = __shfl_sync(0xffffffffu, s.start, g);
      sg.nbits = __shfl_sync(0xffffffffu, s.nbits, g);
      sg.ebytes = __shfl_sync(0xffffffffu, s.ebytes, g);
      if (lane == 0 && !decode_segment_generic<MODE>(sg, *reinterpret_cast<GenericTab*>(&W.lut[0][0]), o))
        bad = true;
      __syncwarp();
    }
    if (__any_sync(0xffffffffu, bad)) {
      if (lane == 0) atomicOr(status, kStatusStream);
      continue;
    }
    if (MODE == 1) {
      __syncwarp();
      for (uint32_t k = lane; k < uint32_t(rows) * nb; k += 32) {
        const uint32_t r = k / nb, b = k - r * nb;
        y[(sd.dst + r) * ld + b] = ysm[r * PMAXB + b];
      }
      __syncwarp();
    }
  }
}

void set_attr_once() {
  static int done_mask = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 31 && ((done_mask >> dev) & 1)) return;
  cudaFuncSetAttribute(parallel_slab_kernel<0>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kSmemBytes[0]));
  cudaFuncSetAttribute(parallel_slab_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kSmemBytes[1]));
  if (dev < 31) done_mask |= 1 << dev;
}

}  // namespace

size_t parallel_smem_bytes() { return kSmemBytes[0]; }

cudaError_t launch_parallel_decode(const Slab* slabs, uint32_t n, const uint8_t* payload,
                                   uint8_t* out, int* status, int grid, cudaStream_t st) {
  if (!n) return cudaSuccess;
  set_attr_once();
  const int need = int((n + PWARPS - 1) / PWARPS);
  parallel_slab_kernel<0><<<grid < need ? grid : need, PWARPS * 32, kSmemBytes[0], st>>>(
      slabs, n, payload, out, nullptr, nullptr, 1, 1, status);
  return cudaGetLastError();
}

cudaError_t launch_parallel_gemm(const Slab* slabs, uint32_t n, const uint8_t* payload,
                                 const float* x, float* y, uint32_t ld, uint32_t b0, uint32_t nb,
                                 int* status, int grid, cudaStream_t st) {
  if (!n) return cudaSuccess;
  set_attr_once();
  const int need = int((n + PWARPS - 1) / PWARPS);
  parallel_slab_kernel<1><<<grid < need ? grid : need, PWARPS * 32, kSmemBytes[1], st>>>(
      slabs, n, payload, nullptr, x + b0, y + b0, ld, nb, status);
  return cudaGetLastError();
}

}  // namespace xksv
