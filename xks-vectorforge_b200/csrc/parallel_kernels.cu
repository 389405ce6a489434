// "bf16-huffman-parallel32" (XKSP2) slabs: decode and fused GEMV/GEMM.
//
// Reference behaviour: cuda/parallel.cu:13-31 (one thread per substream,
// per-substream tree walk, packed->(row, col) mapping :23-24), header checks
// cuda/parallel.cu:33-53, CPU semantics src/c_api.cpp:66-85.
//
// B200 design: one warp per slab, one lane per substream (the format's up to
// 32 independently coded substreams are a warp's worth of independent work);
// many slabs in flight per SM.  Each lane
//   * builds its own canonical decode table: a 2^PK-entry first-level table
//     for codes of length <= PK and a compact table for lengths PK+1..PK+PNL
//     (at most PLONG symbols).  Tables are stored transposed ([entry][lane])
//     so a warp's 32 lookups never conflict on shared-memory banks;
//   * streams its exponent bits through a 64-bit register window fed by
//     16-byte loads issued one chunk ahead, refilled once per 4 codes without
//     a data-dependent branch (codes of length <= PK need <= 28 bits);
//   * streams its sign/mantissa bytes through 8-byte loads two words ahead;
//   * writes 8 BF16 words (half a tile row) per 16-byte store, un-tiled on the
//     fly, for 16-row slabs with cols % 16 == 0 and 16-byte aligned output;
//     other shapes use an element-wise store path.
// A substream whose codebook does not fit the compact table (a length above
// PK+PNL or more than PLONG long codes, e.g. near-uniform exponents) is decoded
// afterwards by lane 0 with the bit-serial canonical decoder.
#include "kernels.h"
#include "xksv_device.cuh"

namespace xksv {
namespace {

constexpr int PK = 7;      // first-level table bits
constexpr int PNL = 16;    // long lengths held per lane: PK+1 .. PK+PNL
constexpr int PLONG = 32;  // long symbols held per lane
constexpr int PWARPS = 4;  // slabs (warps) per CTA
constexpr int PMAXB = 8;   // GEMM columns per pass

// One warp's tables, lane-minor so that lane l always touches bank l/2.
struct WarpTabs {
  uint16_t lut[1 << PK][32];  // exponent << 7 | length; 0 = no code of length <= PK
  uint16_t cnt[PNL][32];      // number of codes of length PK+1+j
  uint8_t lpos[PNL][32];      // fill cursor per long length (build only)
  uint8_t lsym[PLONG][32];    // long-code symbols, canonical (length, symbol) order
  float y[16 * PMAXB];        // GEMM accumulators for the slab's rows
};
constexpr size_t kSmemBytes = PWARPS * sizeof(WarpTabs);

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

// Builds the lane's tables.  Returns 0 when built, 1 when the codebook needs
// the generic decoder, -1 when the lengths are oversubscribed (the canonical
// assignment of src/codec.cpp:11-29 fails exactly then).
__device__ int build_lane_tables(const uint8_t* lens, WarpTabs& W, int lane, uint32_t& F,
                                 int& maxlen) {
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

// Next entry (exponent << 7 | length) of the lane's stream.  Needs >= PK valid
// bits in the window; a long code refills around itself.
__device__ __forceinline__ uint32_t dec(BitReader& br, const WarpTabs& W, int lane, uint32_t F,
                                       int maxlen, bool& bad) {
  uint32_t e = W.lut[br.peek32() >> (32 - PK)][lane];
  if ((e & 31u) == 0) {
    br.refill();
    e = long_entry(br.peek32(), W, lane, F, maxlen);
    bad |= (e & 31u) == 0;
    br.skip(int(e & 31u));
    br.refill();
  } else {
    br.skip(int(e & 31u));
  }
  return e;
}

struct Out {
  uint16_t* out;   // decode: slab output
  const float* x;  // GEMM: X at this slab's column 0 (row stride ld)
  float* ysm;      // GEMM: [16][PMAXB] warp accumulators
  uint32_t rows, cols, ld, nb;
  bool xvec;       // GEMM: nb == 1, ld == 1, 16-byte aligned x
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
// 16-byte aligned output.
template <int MODE>
__device__ void decode_segment(const Seg& s, const WarpTabs& W, int lane, uint32_t F, int maxlen,
                               bool nice, const Out& o, bool& bad) {
  BitReader br;
  br.init(s.bits, s.ebytes);
  uint32_t i = 0, p = s.start;
  if (nice) {
    for (; i < s.count && (p & 7); ++i, ++p) {
      br.refill();
      const uint32_t e = dec(br, W, lane, F, maxlen, bad);
      emit_one<MODE>(o, p, merge1(e, __ldg(s.sm + i)));
    }
    ByteReader16 smr;
    smr.init(s.sm + i, s.sm + s.count);
    uint4 s16 = make_uint4(0, 0, 0, 0);
    const uint32_t i0 = i;
    for (; i + 8 <= s.count; i += 8, p += 8) {
      const bool second = ((i - i0) & 8) != 0;
      if (!second) s16 = smr.take();
      const uint64_t s8 = second ? (uint64_t(s16.w) << 32 | s16.z) : (uint64_t(s16.y) << 32 | s16.x);
      uint32_t e[8];
      br.refill_uniform();
#pragma unroll
      for (int k = 0; k < 4; ++k) e[k] = dec(br, W, lane, F, maxlen, bad);
      br.refill_uniform();
#pragma unroll
      for (int k = 4; k < 8; ++k) e[k] = dec(br, W, lane, F, maxlen, bad);
      const uint32_t slo = uint32_t(s8), shi = uint32_t(s8 >> 32);
      const uint32_t r = (p >> 4) & 15, c = (p >> 8) * 16 + (p & 15);
      if (MODE == 0) {
        uint4 v;
        v.x = (__byte_perm(e[0], e[1], 0x5410) & 0x7F807F80u) | (__byte_perm(slo, 0, 0x1100) & 0x807F807Fu);
        v.y = (__byte_perm(e[2], e[3], 0x5410) & 0x7F807F80u) | (__byte_perm(slo, 0, 0x3322) & 0x807F807Fu);
        v.z = (__byte_perm(e[4], e[5], 0x5410) & 0x7F807F80u) | (__byte_perm(shi, 0, 0x1100) & 0x807F807Fu);
        v.w = (__byte_perm(e[6], e[7], 0x5410) & 0x7F807F80u) | (__byte_perm(shi, 0, 0x3322) & 0x807F807Fu);
        *reinterpret_cast<uint4*>(o.out + size_t(r) * o.cols + c) = v;
      } else {
        float wf[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const uint32_t sb = (k < 4 ? slo : shi) >> (8 * (k & 3));
          wf[k] = __uint_as_float(merge1(e[k], sb & 255u) << 16);
        }
        if (o.xvec) {
          const float4* xv = reinterpret_cast<const float4*>(o.x + c);
          const float4 x0 = __ldg(xv), x1 = __ldg(xv + 1);
          float acc = wf[0] * x0.x;
          acc = fmaf(wf[1], x0.y, acc);
          acc = fmaf(wf[2], x0.z, acc);
          acc = fmaf(wf[3], x0.w, acc);
          acc = fmaf(wf[4], x1.x, acc);
          acc = fmaf(wf[5], x1.y, acc);
          acc = fmaf(wf[6], x1.z, acc);
          acc = fmaf(wf[7], x1.w, acc);
          atomicAdd(&o.ysm[r * PMAXB], acc);
        } else {
          for (uint32_t b = 0; b < o.nb; ++b) {
            float acc = 0.f;
#pragma unroll
            for (int k = 0; k < 8; ++k) acc = fmaf(wf[k], __ldg(&o.x[uint64_t(c + k) * o.ld + b]), acc);
            atomicAdd(&o.ysm[r * PMAXB + b], acc);
          }
        }
      }
    }
  }
  for (; i < s.count; ++i, ++p) {
    br.refill();
    const uint32_t e = dec(br, W, lane, F, maxlen, bad);
    emit_one<MODE>(o, p, merge1(e, __ldg(s.sm + i)));
  }
  if (br.consumed() != s.nbits) bad = true;
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
    uint32_t F = 0;
    int maxlen = 0;
    const int tb = active ? build_lane_tables(s.lens, W, lane, F, maxlen) : 0;
    if (__any_sync(0xffffffffu, tb < 0)) {
      if (lane == 0) atomicOr(status, kStatusCodebook);
      continue;
    }
    Out o;
    o.out = reinterpret_cast<uint16_t*>(out + sd.dst);
    o.x = MODE == 1 ? x + sd.xoff * ld : nullptr;
    o.ysm = W.y;
    o.rows = uint32_t(rows);
    o.cols = uint32_t(cols);
    o.ld = ld;
    o.nb = nb;
    o.xvec = nb == 1 && ld == 1 && (reinterpret_cast<uintptr_t>(o.x) & 15) == 0;
    if (MODE == 1) {
      for (int k = lane; k < 16 * PMAXB; k += 32) W.y[k] = 0.f;
      __syncwarp();
    }
    const bool nice = rows == 16 && (cols & 15) == 0 &&
                      (MODE == 1 || (reinterpret_cast<uintptr_t>(o.out) & 15) == 0);
    bool bad = false;
    if (active && tb == 0) decode_segment<MODE>(s, W, lane, F, maxlen, nice, o, bad);
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
        y[(sd.dst + r) * ld + b] = W.y[r * PMAXB + b];
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
  cudaFuncSetAttribute(parallel_slab_kernel<0>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kSmemBytes));
  cudaFuncSetAttribute(parallel_slab_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kSmemBytes));
  if (dev < 31) done_mask |= 1 << dev;
}

}  // namespace

size_t parallel_smem_bytes() { return kSmemBytes; }

cudaError_t launch_parallel_decode(const Slab* slabs, uint32_t n, const uint8_t* payload,
                                   uint8_t* out, int* status, int grid, cudaStream_t st) {
  if (!n) return cudaSuccess;
  set_attr_once();
  const int need = int((n + PWARPS - 1) / PWARPS);
  parallel_slab_kernel<0><<<grid < need ? grid : need, PWARPS * 32, kSmemBytes, st>>>(
      slabs, n, payload, out, nullptr, nullptr, 1, 1, status);
  return cudaGetLastError();
}

cudaError_t launch_parallel_gemm(const Slab* slabs, uint32_t n, const uint8_t* payload,
                                 const float* x, float* y, uint32_t ld, uint32_t b0, uint32_t nb,
                                 int* status, int grid, cudaStream_t st) {
  if (!n) return cudaSuccess;
  set_attr_once();
  const int need = int((n + PWARPS - 1) / PWARPS);
  parallel_slab_kernel<1><<<grid < need ? grid : need, PWARPS * 32, kSmemBytes, st>>>(
      slabs, n, payload, nullptr, x + b0, y + b0, ld, nb, status);
  return cudaGetLastError();
}

}  // namespace xksv
