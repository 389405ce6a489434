// "bf16-huffman-parallel32" (XKSP2) slabs: decode and fused GEMV/GEMM.
//
// Reference behaviour: cuda/parallel.cu:13-31 (one thread per substream,
// per-substream tree walk, packed->(row, col) mapping :23-24), header checks
// cuda/parallel.cu:33-53, CPU semantics src/c_api.cpp:66-85.
//
// B200 design: one warp per slab, one lane per substream (the format's up to
// 32 independently coded substreams are a warp's worth of independent work);
// many slabs in flight per SM.  Every per-lane step of the inner loop runs at
// a cadence shared by all lanes, so the warp never serialises on one lane:
//   * each lane builds its own canonical tables: a 2^PK-entry first level for
//     codes of length <= PK, a second level for lengths PK+1..PK+K2 under the
//     first NE escape prefixes (12-bit codes: the long tails of large slabs
//     and heavy-tailed weights stay on the fast path), and a compact list for
//     lengths up to PK+PNL.  Tables are lane-minor ([entry][lane]);
//   * a lane's exponent bits live in a 16-word ring in shared memory laid out
//     [word][lane], so every lane reads only its own bank.  Words arrive as
//     aligned 32-byte global loads (sm_100 256-bit loads: a warp-wide load of
//     32 separate streams costs one L1 wavefront per lane, so wider loads move
//     more bytes per wavefront) held ahead in registers and are byte-swapped
//     once when they enter the ring;
//   * codes are decoded four at a time from one 32-bit snapshot of the ring
//     at the lane's bit position (two shared loads and a funnel shift): four
//     table lookups each followed by a one-instruction shift.  One check per
//     block -- total length <= 32 and a non-zero last entry -- proves that
//     every code of the block was read from real bits and found in the
//     tables (an entry of 0 consumes no bits, so an unresolved code zeroes
//     the block's last entry); otherwise the block is redone code by code;
//   * sign/mantissa bytes arrive 16 at a time through a shared cp.async ring
//     (asynchronous copies: nothing waits on a register load);
//   * 16 decoded BF16 words (one tile row) leave as one 32-byte store (two
//     16-byte stores when the output is only 16-byte aligned), un-tiled on the
//     fly, for 16-row slabs with cols % 16 == 0; other shapes use an
//     element-wise store path.
// A substream whose codebook the compact tables cannot hold (a length above
// PK+PNL or more than PLONG long codes, e.g. near-uniform exponents) is decoded
// afterwards by lane 0 with the bit-serial canonical decoder.
// A slab's setup is a chain of dependent loads (container header, substream
// table, substream headers, length tables); while one slab's tables are built
// the warp already reads its next slab's substream table and prefetches that
// slab's substream headers and length tables into L2.
#include <atomic>

#include "kernels.h"
#include "xksv_device.cuh"

namespace xksv {
namespace {

constexpr int PK = 6;       // first-level table bits
constexpr int K2 = 5;       // second level covers lengths PK+1 .. PK+K2
constexpr int NE = 2;       // escape prefixes with a second-level table
constexpr int NROW2 = (NE << K2) + 1;  // second-level rows (the last is all zero)
constexpr int PNL = 16;     // long lengths held per lane: PK+1 .. PK+PNL
constexpr int PLONG = 16;   // long symbols held per lane
constexpr int BR = 16;      // bit-ring words per lane (power of two)
constexpr uint32_t kRingLow = 8;  // unread ring words kept at each 16-code group
constexpr int kSaveChunk = 4;     // first ring row holding length chunks saved by the table build
constexpr int SMR = 4;      // 16-byte sign/mantissa slots per lane
constexpr int PWARPS = 2;   // slabs (warps) per CTA: small CTAs free their tables sooner
constexpr int PMAXB = 8;    // GEMM columns per pass

// One warp's tables, lane-minor so that lane l always touches bank l/2
// (16-bit tables) or bank l (the bit ring).
struct WarpTabs {
  uint16_t lut[1 << PK][32];     // exponent << 7 | length; 0 = no code of length <= PK
  uint16_t lut2[NROW2][32];      // second level: (PK+K2)-bit prefix - (L << K2); last row 0
  uint8_t cnt[PNL][32];          // number of codes of length PK+1+j (<= PLONG)
  uint8_t lsym[PLONG][32];       // long-code symbols, canonical (length, symbol) order
  union {
    uint8_t lpos[PNL][32];       // fill cursor per long length (table build only)
    uint32_t ring[BR][32];       // exponent bits, big-endian words, word w at [w % BR]
  };
  uint4 smring[SMR][32];         // staged sign/mantissa chunks
};
static_assert(sizeof(WarpTabs) % 16 == 0, "warp tables keep 16-byte alignment");
static_assert(kRingLow + 8 <= BR, "a staged chunk fits whenever maintain() adds one");
static_assert(kSaveChunk * 128 >= PNL * 32, "saved length chunks do not overlap lpos");
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

// Builds the lane's tables.  Returns 0 when built, 1 when the codebook needs
// the generic decoder, -1 when the lengths are oversubscribed (the canonical
// assignment of src/codec.cpp:11-29 fails exactly then).  The 256 length
// bytes arrive through 17 aligned 16-byte loads issued together (one memory
// round trip instead of a short stream of dependent ones) and only their
// non-zero bytes are visited (a slab's exponents use a dozen or so symbols); the first three
// non-zero chunks are kept in the lane's column of the bit ring (rows
// kSaveChunk.., clear of lpos) for the fill pass.  Short-length counters and
// fill cursors are 8-bit fields of two registers (lengths 1-4 | 5-PK); a field
// that wraps (256 codes of one length) shows as a count mismatch.
__device__ int build_lane_tables(const uint8_t* lens, WarpTabs& W, int lane, uint32_t& F,
                                 int& maxlen, uint32_t& Lout) {
  static_assert(PK == 6, "packed counters cover lengths 1-4 and 5-6");
  uint32_t c14 = 0, c56 = 0, nshort = 0, nlong = 0;
  bool generic = false;
  uint32_t mx = 0;
#pragma unroll
  for (int j = 0; j < PNL; ++j) W.cnt[j][lane] = 0;
  uint32_t nz = 0;      // chunks holding a non-zero length
  uint32_t nsaved = 0;  // non-zero chunks kept in the ring rows
  ByteReader16 rd;
  rd.init(lens, lens + 256);
  for (int c16 = 0; c16 < 16; ++c16) {
    const uint4 v = rd.take();
    if ((v.x | v.y | v.z | v.w) == 0) continue;
    nz |= 1u << c16;
    if (nsaved < 3) {
      const int r = kSaveChunk + 4 * int(nsaved);
      W.ring[r][lane] = v.x;
      W.ring[r + 1][lane] = v.y;
      W.ring[r + 2][lane] = v.z;
      W.ring[r + 3][lane] = v.w;
      ++nsaved;
    }
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
          // generic decoder, before any count is used
          W.cnt[l - PK - 1][lane] += 1;
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
    const uint32_t c = W.cnt[l - PK - 1][lane];
    used = (used << 1) + c;
    W.lpos[l - PK - 1][lane] = uint8_t(pos);
    pos += c;
  }
  if (maxlen > PK && used > (1ull << maxlen)) return -1;
  F = L << 1;
  // fill from the saved chunks (re-reading any beyond the first three)
  uint32_t k = 0;
  while (nz) {
    const int c16 = __ffs(nz) - 1;
    nz &= nz - 1;
    uint4 v;
    if (k < 3) {
      const int r = kSaveChunk + 4 * int(k);
      v = make_uint4(W.ring[r][lane], W.ring[r + 1][lane], W.ring[r + 2][lane], W.ring[r + 3][lane]);
    } else {
      v = ld16_any(lens + 16 * c16);
    }
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
          for (uint32_t r = 0; r < run; ++r) W.lut[st + r][lane] = e;
        } else {
          const int j = int(l) - PK - 1;
          W.lsym[W.lpos[j][lane]][lane] = uint8_t(sym);
          W.lpos[j][lane] += 1;
        }
      }
    }
  }
  // rows past the short codes: prefixes of long codes or unused code space
  for (uint32_t z = L; z < (1u << PK); ++z) W.lut[z][lane] = 0;
  // second level (zeroed by the whole warp before the build): codes of length
  // PK+1..PK+K2 whose (PK+K2)-bit prefixes fall in the first NE escape prefixes
  uint32_t cf = F, idx = 0;
  const uint32_t base = L << K2;
  for (int l = PK + 1; l <= maxlen && l <= PK + K2; ++l) {
    const uint32_t c = W.cnt[l - PK - 1][lane];
    for (uint32_t q = 0; q < c; ++q) {
      const uint32_t code = cf + q;
      const uint32_t run = 1u << (PK + K2 - l);
      const uint32_t st = (code << (PK + K2 - l)) - base;
      if (st + run <= uint32_t(NE << K2)) {
        const uint16_t e = uint16_t((uint32_t(W.lsym[idx + q][lane]) << 7) | uint32_t(l));
        for (uint32_t r = 0; r < run; ++r) W.lut2[st + r][lane] = e;
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
// stream's own bits begin at pos0 = 8 * (start & 31).  Chunk loads are clamped
// to the last chunk holding stream bytes: only a corrupt stream reads past its
// end, and the final bit count rejects it.
struct LaneStream {
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
  // Issues the first loads; the ring is written by init_ring() once the
  // table build no longer needs the memory it shares.
  __device__ __forceinline__ void start(const uint8_t* base, uint64_t nbytes) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(base);
    src = reinterpret_cast<const Chunk32*>(a & ~uintptr_t(31));
    last = reinterpret_cast<const Chunk32*>((a + (nbytes ? nbytes - 1 : 0)) & ~uintptr_t(31));
    pos0 = pos = uint32_t(a & 31) * 8;
    c0 = fetch();
    stage = fetch();
  }
  // fw is always a multiple of 8 (chunks of 8 words from word 0), so a chunk
  // fills ring rows (fw % BR) .. +7 from one base address.
  __device__ __forceinline__ void put(WarpTabs& W, int lane, const Chunk32& c) {
    static_assert(BR == 16, "a chunk fills one half of the ring");
    uint32_t* r = &W.ring[fw & 8][lane];
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
  __device__ __forceinline__ void init_ring(WarpTabs& W, int lane) {
    fw = 0;
    put(W, lane, c0);
  }
  // Moves the staged chunk into the ring and loads the next one.
  __device__ __forceinline__ void advance(WarpTabs& W, int lane) {
    put(W, lane, stage);
    stage = fetch();
  }
  // Keeps at least kRingLow unread words in the ring: four checked blocks
  // (<= 32 bits each) and the last snapshot's second word need five; a chunk
  // enters only when it fits (fw - word <= BR - 8), so the chunk staged here
  // was loaded several groups earlier.
  __device__ __forceinline__ void maintain(WarpTabs& W, int lane) {
    while (fw - (pos >> 5) < kRingLow) advance(W, lane);
  }
  // The 32 bits at pos.
  __device__ __forceinline__ uint32_t snap(const WarpTabs& W, int lane) const {
    const uint32_t j = pos >> 5;
    const uint32_t a = W.ring[j & (BR - 1)][lane], b = W.ring[(j + 1) & (BR - 1)][lane];
    return __funnelshift_l(b, a, pos);
  }
};

// A lane's sign/mantissa bytes for 16-code groups: aligned 16-byte chunks
// staged by cp.async three groups ahead, realigned when a group is consumed.
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
  // Stages the chunk three ahead of the group about to be consumed (its slot
  // held the chunk the previous group read first).
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

__device__ __forceinline__ void cp_async_wait_2() { asm volatile("cp.async.wait_group 2;\n" ::: "memory"); }

struct LaneCode {
  uint32_t F;   // first code of length PK+1
  uint32_t L2;  // first escape prefix << K2 (second-level index origin)
  int maxlen;
};

// Table lookup of the code at the top of w: exponent << 7 | length, or 0
// when neither level holds it.  No branch: a prefix outside the second level
// reads its all-zero last row, and a short code (first level) always has a
// prefix below the escape rows, so at most one level is non-zero.
__device__ __forceinline__ uint32_t lookup(uint32_t w, const WarpTabs& W, int lane, uint32_t L2) {
  const uint32_t e1 = W.lut[w >> (32 - PK)][lane];
  // min(prefix - L2, NE << K2) in one add-min (DPX) instruction
  const uint32_t i2 = __viaddmin_u32(w >> (32 - PK - K2), 0u - L2, uint32_t(NE << K2));
  return e1 | uint32_t(W.lut2[i2][lane]);
}

// One code at pos, with the compact long-code list behind the tables and a
// ring top-up first (any code the lane can hold has <= PK+PNL <= 32 bits).
__device__ __forceinline__ uint32_t dec_one(LaneStream& b, WarpTabs& W, int lane, const LaneCode& lc,
                                            bool& bad) {
  if (b.fw - (b.pos >> 5) < 2u) b.advance(W, lane);  // the ring keeps >= 2 unread words
  const uint32_t w = b.snap(W, lane);
  uint32_t e = lookup(w, W, lane, lc.L2);
  if (e == 0) {
    e = long_entry(w, W, lane, lc.F, lc.maxlen);
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
__device__ __forceinline__ void dec4(LaneStream& b, WarpTabs& W, int lane, const LaneCode& lc, bool& bad,
                                     uint32_t& e0, uint32_t& e1, uint32_t& e2, uint32_t& e3) {
  uint32_t w = b.snap(W, lane);
  e0 = lookup(w, W, lane, lc.L2);
  w = __funnelshift_l(0u, w, e0);  // w << (length & 31)
  e1 = lookup(w, W, lane, lc.L2);
  w = __funnelshift_l(0u, w, e1);
  e2 = lookup(w, W, lane, lc.L2);
  w = __funnelshift_l(0u, w, e2);
  e3 = lookup(w, W, lane, lc.L2);
  // lengths sit in bits 0-4 above zero bits 5-6, so one sum carries all four
  const uint32_t s = (e0 + e1 + e2 + e3) & 127u;
  if (s > 32u || e3 == 0) {
    e0 = dec_one(b, W, lane, lc, bad);
    e1 = dec_one(b, W, lane, lc, bad);
    e2 = dec_one(b, W, lane, lc, bad);
    e3 = dec_one(b, W, lane, lc, bad);
    b.maintain(W, lane);
  } else {
    b.pos += s;
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

// Decodes one substream.  `rows16`: 16-row slab, cols % 16 == 0, the
// substream starts on a tile row and (decode) the output is 16-byte aligned;
// whole tile rows then leave as 32-byte stores.  The caller has started `b`
// and `smr` (sign/mantissa bytes, 16 per group) and put the first words into
// the ring.
template <int MODE>
__device__ void decode_segment(const Seg& s, WarpTabs& W, int lane, const LaneCode& lc, bool rows16,
                               LaneStream& b, LaneSm& smr, const Out& o, bool& bad) {
  uint32_t i = 0;
  if (rows16) {
    const uint32_t ng = s.count >> 4;
    uint32_t p = s.start;
    for (uint32_t g = 0; g < ng; ++g, p += 16) {
      smr.stage(W, lane);
      cp_async_commit();
      b.maintain(W, lane);
      cp_async_wait_2();  // this group's two chunks were committed two groups ago
      const uint4 s16 = smr.take(W, lane);
      uint32_t e[16];
#pragma unroll
      for (int k = 0; k < 4; ++k) dec4(b, W, lane, lc, bad, e[4 * k], e[4 * k + 1], e[4 * k + 2], e[4 * k + 3]);
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
          for (int qq = 0; qq < 4; ++qq) {
            const float4 xq = __ldg(xv + qq);
            acc = fmaf(wf[4 * qq], xq.x, acc);
            acc = fmaf(wf[4 * qq + 1], xq.y, acc);
            acc = fmaf(wf[4 * qq + 2], xq.z, acc);
            acc = fmaf(wf[4 * qq + 3], xq.w, acc);
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
    }
    i = ng << 4;
  }
  for (; i < s.count; ++i) {
    const uint32_t e = dec_one(b, W, lane, lc, bad);
    emit_one<MODE>(o, s.start + i, merge1(e, __ldg(s.sm + i)));
  }
  cp_async_wait_all();
  if (uint64_t(b.pos - b.pos0) != s.nbits) bad = true;
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

__device__ __forceinline__ void prefetch_l2(const void* p) {
  asm volatile("prefetch.global.L2 [%0];" ::"l"(p));
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
__global__ void __launch_bounds__(PWARPS * 32, MODE == 0 ? 8 : 1)
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
    // ---- the warp's next slab: its header lines go to L2 now and its
    // substream table is read here, so that once this slab's tables are built
    // the next slab's substream headers and length tables can be prefetched
    // too; its setup then finds every dependent load in L2 ----
    const uint32_t sn = si + gridDim.x * PWARPS;
    const uint8_t* np = nullptr;
    uint64_t nsize = 0, nlen = 0, ntotal = 0;
    if (sn < nslabs) {
      const Slab nd = slabs[sn];
      np = payload + nd.src;
      nsize = nd.size;
      ntotal = nd.rows * nd.cols;
      if (uint64_t(lane) * 128 < (nsize < 288 ? nsize : 288)) prefetch_l2(np + 128 * lane);
      if (40 + 8 * uint64_t(lane) <= nsize) nlen = ld8_any(np + 32 + 8 * lane, np + nsize);
    }
    // ---- container header (cuda/parallel.cu:34-36) ----
    bool ok = n >= 32;
    uint64_t rows = 0, cols = 0, chunks = 0;
    if (ok) {
      // header fields through aligned 8-byte loads (the slab may sit at any
      // byte offset; n >= 32 keeps every read inside the slab's words)
      const uint8_t* pe = p + n;
      ok = ld8_any(p, pe) == 0x0000003250534B58ull;  // "XKSP2\0\0\0"
      rows = ld8_any(p + 8, pe);
      cols = ld8_any(p + 16, pe);
      chunks = ld8_any(p + 24, pe);
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
    const uint64_t len = active ? ld8_any(p + 32 + 8 * lane, p + n) : 0;
    bool lok = !active || (len >= kHdr && len <= n);
    const uint64_t incl = warp_incl_scan(lok ? len : 0, lane);
    const uint64_t base = 32 + 8 * chunks + incl - len;
    Seg s{};
    if (active && lok) {
      lok = base + len <= n;
      if (lok) {
        const uint8_t* q = p + base;
        const uint64_t count = ld8_any(q, p + n);
        s.nbits = ld8_any(q + 8, p + n);
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
    // bit positions are 32-bit (the slab format bounds them far lower: a
    // substream's bits fit in its slab, and compiled slabs are <= 1 MiB)
    if (__any_sync(0xffffffffu, s.nbits >= (1ull << 32) - 256)) {
      if (lane == 0) atomicOr(status, kStatusInternal);
      continue;
    }
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
    const bool nice = rows == 16 && (cols & 15) == 0 &&
                      (MODE == 1 || (reinterpret_cast<uintptr_t>(o.out) & 15) == 0);
    const bool rows16 = nice && (s.start & 15) == 0;
    // ---- first bit and sign/mantissa loads, overlapping the table build ----
    LaneStream b;
    LaneSm smr;
    if (active) {
      b.start(s.bits, s.ebytes);
      if (rows16) smr.init(W, lane, s.sm, s.sm + s.count);
    }
    cp_async_commit();
    // ---- per-lane tables ----
    // the second-level table starts all zero: 16-byte stores by the warp
    {
      static_assert(sizeof(WarpTabs::lut2) % 16 == 0 && offsetof(WarpTabs, lut2) % 16 == 0, "lut2 as uint4");
      uint4* z = reinterpret_cast<uint4*>(&W.lut2[0][0]);
      for (uint32_t k = lane; k < sizeof(WarpTabs::lut2) / 16; k += 32) z[k] = make_uint4(0, 0, 0, 0);
      __syncwarp();
    }
    LaneCode lc{0, 0, 0};
    uint32_t L = 0;
    const int tb = active ? build_lane_tables(s.lens, W, lane, lc.F, lc.maxlen, L) : 0;
    lc.L2 = L << K2;
    __syncwarp();
    if (np) {  // next slab's substream headers and length tables to L2
      const uint64_t nch = ntotal < 32 ? ntotal : 32;
      const bool na = uint64_t(lane) < nch;
      const uint64_t nl = na ? nlen : 0;
      const uint64_t off = 32 + 8 * nch + warp_incl_scan(nl, lane) - nl;
      if (na && nl >= kHdr && off <= nsize && kHdr <= nsize - off) {
        prefetch_l2(np + off);
        prefetch_l2(np + off + 128);
        prefetch_l2(np + off + kHdr - 1);
      }
    }
    if (__any_sync(0xffffffffu, tb < 0)) {
      cp_async_wait_all();
      __syncwarp();
      if (lane == 0) atomicOr(status, kStatusCodebook);
      continue;
    }
    __syncwarp();  // every lane's build is done before the bit ring (over lpos) fills
    if (MODE == 1) {
      for (int k = lane; k < 16 * PMAXB; k += 32) ysm[k] = 0.f;
      __syncwarp();
    }
    bool bad = false;
    if (active && tb == 0) {
      b.init_ring(W, lane);
      cp_async_wait_all();
      decode_segment<MODE>(s, W, lane, lc, rows16, b, smr, o, bad);
    }
    cp_async_wait_all();
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
        const uint32_t r = k / nb, bb = k - r * nb;
        y[(sd.dst + r) * ld + bb] = ysm[r * PMAXB + bb];
      }
      __syncwarp();
    }
  }
}

// Dynamic shared memory opt-in, once per device (concurrent first calls both
// set the same value, which is harmless).
void set_attr_once() {
  static std::atomic<uint64_t> done{0};
  int dev = 0;
  cudaGetDevice(&dev);
  const uint64_t bit = dev < 64 ? (1ull << dev) : 0ull;
  if (bit && (done.load(std::memory_order_acquire) & bit)) return;
  cudaFuncSetAttribute(parallel_slab_kernel<0>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kSmemBytes[0]));
  cudaFuncSetAttribute(parallel_slab_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kSmemBytes[1]));
  if (bit) done.fetch_or(bit, std::memory_order_release);
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
