// "bf16-huffman-parallel32" (XKSP2) slabs: decode and fused GEMV/GEMM.
//
// Reference behaviour: cuda/parallel.cu:13-31 (one thread per substream,
// per-substream tree walk, packed->(row, col) mapping :23-24), header checks
// cuda/parallel.cu:33-53, CPU semantics src/c_api.cpp:66-85.
//
// B200 design: one warp per slab and one lane per substream (the format's
// up-to-32 independently coded substreams are exactly a warp's worth of
// independent work), many slabs in flight per SM.  Each lane
//   * builds its own canonical decode table in shared memory: a 2^PK-entry
//     first-level table for codes of length <= PK plus a compact table for
//     longer codes (lengths PK+1..PK+PNL, at most PLONG symbols);
//   * streams its exponent bits through 16-byte loads into a 64-bit window,
//     its sign/mantissa bytes through aligned 8-byte loads;
//   * writes 8 decoded BF16 words (one 16-byte store, half a tile row) at a
//     time, un-tiled on the fly, for the common slab shape (16 rows, cols a
//     multiple of 16, 16-byte aligned output).  Other shapes take an
//     element-wise store path.
// A substream whose codebook does not fit the compact table (lengths > PK+PNL
// or more than PLONG long codes, e.g. near-uniform exponents) is decoded
// afterwards by lane 0 with a bit-serial canonical decoder.
#include "kernels.h"
#include "xksv_device.cuh"

namespace xksv {
namespace {

constexpr int PK = 7;      // first-level table bits
constexpr int PNL = 16;    // long lengths held per lane: PK+1 .. PK+PNL
constexpr int PLONG = 32;  // long symbols held per lane
constexpr int PWARPS = 4;  // slabs (warps) per CTA
constexpr int PMAXB = 8;   // GEMM columns per pass

struct __align__(16) LaneTab {
  uint16_t lut[1 << PK];  // exponent << 7 | length; 0 = no code of length <= PK
  uint16_t cnt[PNL];      // number of codes of length PK+1+j
  uint8_t lpos[PNL];      // fill cursor per long length (build time only)
  uint8_t lsym[PLONG];    // long-code symbols in canonical (length, symbol) order
};
static_assert(sizeof(LaneTab) % 16 == 0, "LaneTab alignment");

struct WarpShared {
  float y[16 * PMAXB];  // GEMM accumulators for the slab's rows
};

constexpr size_t kWarpTabBytes = sizeof(LaneTab) * 32;
constexpr size_t kSmemBytes = PWARPS * (kWarpTabBytes + sizeof(WarpShared));

// Generic (bit-serial) tables overlay a warp's 32 LaneTabs once the fast lanes
// are done.
struct GenericTab {
  uint16_t cnt[256];
  uint16_t off[257];
  uint8_t sorted[256];
};
static_assert(sizeof(GenericTab) <= kWarpTabBytes, "generic table fits");

struct Seg {
  const uint8_t* lens;
  const uint8_t* sm;
  const uint8_t* bits;
  uint64_t count;
  uint64_t nbits;
  uint64_t ebytes;
  uint64_t start;  // packed index of the substream's first element
};

__device__ __forceinline__ uint32_t byte_of(const uint4& v, int b) {
  uint32_t w = b < 4 ? v.x : b < 8 ? v.y : b < 12 ? v.z : v.w;
  return (w >> (8 * (b & 3))) & 255u;
}

// 16 bytes from any address, as little-endian words (two aligned loads and a
// byte funnel).
__device__ __forceinline__ uint4 ld16_any(const uint8_t* p) {
  uintptr_t a = reinterpret_cast<uintptr_t>(p);
  const uint4* q = reinterpret_cast<const uint4*>(a & ~uintptr_t(15));
  int off = int(a & 15);
  uint4 lo = ldg16(q);
  if (off == 0) return lo;
  uint4 hi = ldg16(q + 1);
  uint32_t w0 = lo.x, w1 = lo.y, w2 = lo.z, w3 = lo.w, w4 = hi.x, w5 = hi.y, w6 = hi.z, w7 = hi.w;
  if (off & 8) {
    w0 = w2; w1 = w3; w2 = w4; w3 = w5; w4 = w6; w5 = w7;
  }
  if (off & 4) {
    w0 = w1; w1 = w2; w2 = w3; w3 = w4; w4 = w5;
  }
  int bs = (off & 3) * 8;
  return make_uint4(__funnelshift_r(w0, w1, bs), __funnelshift_r(w1, w2, bs),
                    __funnelshift_r(w2, w3, bs), __funnelshift_r(w3, w4, bs));
}

// Builds the lane's fast tables.  Returns 0 when built, 1 when the codebook
// needs the generic decoder, -1 when the lengths are oversubscribed.
__device__ int build_lane_tables(const uint8_t* lens, LaneTab& T, uint32_t& F, int& maxlen) {
  uint64_t c_lo = 0, c_hi = 0;  // 16-bit counters: lengths 1-4 | 5-8
  uint32_t nlong = 0;
  bool generic = false;
  maxlen = 0;
  reinterpret_cast<uint4*>(T.cnt)[0] = make_uint4(0, 0, 0, 0);
  reinterpret_cast<uint4*>(T.cnt)[1] = make_uint4(0, 0, 0, 0);
  for (int c16 = 0; c16 < 16; ++c16) {
    uint4 v = ld16_any(lens + 16 * c16);
    if ((v.x | v.y | v.z | v.w) == 0) continue;
#pragma unroll
    for (int b = 0; b < 16; ++b) {
      uint32_t l = byte_of(v, b);
      if (!l) continue;
      maxlen = max(maxlen, int(l));
      if (l <= 4)
        c_lo += 1ull << (16 * (l - 1));
      else if (l <= PK)
        c_hi += 1ull << (16 * (l - 5));
      else if (l <= PK + PNL) {
        T.cnt[l - PK - 1] += 1;
        ++nlong;
      } else
        generic = true;
    }
  }
  if (generic || nlong > PLONG) return 1;
  // first-level start index per short length; Kraft check
  uint64_t s_lo = 0, s_hi = 0;
  uint32_t L = 0;
#pragma unroll
  for (int l = 1; l <= PK; ++l) {
    uint32_t c = l <= 4 ? uint32_t(c_lo >> (16 * (l - 1))) & 0xFFFFu
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
    uint32_t c = T.cnt[l - PK - 1];
    used = (used << 1) + c;
    T.lpos[l - PK - 1] = uint8_t(pos);
    pos += c;
  }
  if (maxlen > PK && used > (1ull << maxlen)) return -1;
  F = L << 1;
  // fill
  for (int c16 = 0; c16 < 16; ++c16) {
    uint4 v = ld16_any(lens + 16 * c16);
    if ((v.x | v.y | v.z | v.w) == 0) continue;
#pragma unroll
    for (int b = 0; b < 16; ++b) {
      uint32_t l = byte_of(v, b);
      if (!l) continue;
      uint32_t s = uint32_t(c16 * 16 + b);
      if (l <= PK) {
        uint32_t st;
        if (l <= 4) {
          st = uint32_t(s_lo >> (16 * (l - 1))) & 0xFFFFu;
          s_lo += uint64_t(1u << (PK - l)) << (16 * (l - 1));
        } else {
          st = uint32_t(s_hi >> (16 * (l - 5))) & 0xFFFFu;
          s_hi += uint64_t(1u << (PK - l)) << (16 * (l - 5));
        }
        uint32_t e = (s << 7) | l, run = 1u << (PK - l);
        uint32_t e2 = e | (e << 16);
        if (run == 1)
          T.lut[st] = uint16_t(e);
        else if (run == 2)
          *reinterpret_cast<uint32_t*>(&T.lut[st]) = e2;
        else if (run == 4)
          *reinterpret_cast<uint2*>(&T.lut[st]) = make_uint2(e2, e2);
        else
          for (uint32_t k = 0; k < run; k += 8)
            *reinterpret_cast<uint4*>(&T.lut[st + k]) = make_uint4(e2, e2, e2, e2);
      } else {
        T.lsym[T.lpos[l - PK - 1]++] = uint8_t(s);
      }
    }
  }
  // entries past the short codes: prefixes of long codes or unused space
  uint32_t z = L;
  for (; z < (1u << PK) && (z & 7); ++z) T.lut[z] = 0;
  for (; z < (1u << PK); z += 8) *reinterpret_cast<uint4*>(&T.lut[z]) = make_uint4(0, 0, 0, 0);
  return 0;
}

// Next table entry (exponent << 7 | length) of the lane's stream.
__device__ __forceinline__ uint32_t next_entry(BitReader& br, const LaneTab& T, uint32_t F,
                                               int maxlen, uint64_t& used, bool& bad) {
  uint32_t w = br.peek32();
  uint32_t e = T.lut[w >> (32 - PK)];
  uint32_t len = e & 31u;
  if (len == 0) {
    uint32_t cf = F, idx = 0;
    for (int l = PK + 1; l <= maxlen; ++l) {
      uint32_t v = w >> (32 - l);
      uint32_t c = T.cnt[l - PK - 1];
      if (v - cf < c) {
        e = (uint32_t(T.lsym[idx + v - cf]) << 7) | uint32_t(l);
        break;
      }
      idx += c;
      cf = (cf + c) << 1;
    }
    len = e & 31u;
    if (len == 0) bad = true;
  }
  br.skip(int(len));
  br.refill();
  used += len;
  return e;
}

// Output of one decoded element (packed index p).
struct DecodeOut {
  uint16_t* out;  // slab output (row-major)
  uint64_t rows, cols;
  __device__ __forceinline__ void one(uint64_t p, uint32_t word) const {
    out[untile_index(p, rows, cols)] = uint16_t(word);
  }
};

struct GemmOut {
  const float* x;  // X at this slab's column 0, row stride ld
  float* ysm;      // [16][PMAXB] warp accumulators
  uint64_t rows, cols;
  uint32_t ld, nb;
  __device__ __forceinline__ void one(uint64_t p, uint32_t word) const {
    uint64_t o = untile_index(p, rows, cols);
    uint64_t r = o / cols, c = o - r * cols;
    float w = __uint_as_float(word << 16);
    for (uint32_t b = 0; b < nb; ++b) atomicAdd(&ysm[r * PMAXB + b], w * __ldg(&x[c * ld + b]));
  }
};

// Decodes one substream with the lane tables; `nice` = 16-row slab, cols %
// 16 == 0, 16-byte aligned output (decode) / contiguous 16-byte aligned x
// with nb == 1 (GEMV).
template <int MODE>
__device__ void decode_segment(const Seg& s, const LaneTab& T, uint32_t F, int maxlen, bool nice,
                               const DecodeOut& dout, const GemmOut& gout, bool& bad) {
  BitReader br;
  br.init(s.bits, s.ebytes, 0);
  uint64_t used = 0, i = 0, p = s.start;
  if (nice) {
    for (; i < s.count && (p & 7); ++i, ++p) {
      uint32_t e = next_entry(br, T, F, maxlen, used, bad);
      uint32_t w = merge1(e, __ldg(s.sm + i));
      if (MODE == 0) dout.one(p, w); else gout.one(p, w);
    }
    const uintptr_t a = reinterpret_cast<uintptr_t>(s.sm + i);
    const uint64_t* sw = reinterpret_cast<const uint64_t*>(a & ~uintptr_t(7));
    const int sh = int(a & 7) * 8;
    uint64_t s_lo = (i + 8 <= s.count) ? __ldg(sw) : 0ull;
    for (; i + 8 <= s.count && !bad; i += 8, p += 8) {
      uint64_t s_hi = sh ? __ldg(sw + 1) : 0ull;
      uint64_t s8 = sh ? (s_lo >> sh) | (s_hi << (64 - sh)) : s_lo;
      ++sw;
      s_lo = sh ? s_hi : ((i + 16 <= s.count) ? __ldg(sw) : 0ull);
      uint32_t e[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) e[k] = next_entry(br, T, F, maxlen, used, bad);
      const uint32_t slo = uint32_t(s8), shi = uint32_t(s8 >> 32);
      uint64_t t = p >> 8, r = (p >> 4) & 15, c = t * 16 + (p & 15);
      if (MODE == 0) {
        uint4 o;
        o.x = (__byte_perm(e[0], e[1], 0x5410) & 0x7F807F80u) | (__byte_perm(slo, 0, 0x1100) & 0x807F807Fu);
        o.y = (__byte_perm(e[2], e[3], 0x5410) & 0x7F807F80u) | (__byte_perm(slo, 0, 0x3322) & 0x807F807Fu);
        o.z = (__byte_perm(e[4], e[5], 0x5410) & 0x7F807F80u) | (__byte_perm(shi, 0, 0x1100) & 0x807F807Fu);
        o.w = (__byte_perm(e[6], e[7], 0x5410) & 0x7F807F80u) | (__byte_perm(shi, 0, 0x3322) & 0x807F807Fu);
        *reinterpret_cast<uint4*>(dout.out + r * dout.cols + c) = o;
      } else {
        const float4* xv = reinterpret_cast<const float4*>(gout.x + c);
        float4 x0 = __ldg(xv), x1 = __ldg(xv + 1);
        float xs[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
        float acc = 0.f;
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          uint32_t sb = (k < 4 ? slo : shi) >> (8 * (k & 3));
          uint32_t w = merge1(e[k], sb & 255u);
          acc = fmaf(__uint_as_float(w << 16), xs[k], acc);
        }
        atomicAdd(&gout.ysm[r * PMAXB], acc);
      }
    }
  }
  for (; i < s.count && !bad; ++i, ++p) {
    uint32_t e = next_entry(br, T, F, maxlen, used, bad);
    uint32_t w = merge1(e, __ldg(s.sm + i));
    if (MODE == 0) dout.one(p, w); else gout.one(p, w);
  }
  if (used != s.nbits) bad = true;
}

// Lane 0 decodes a substream whose codebook needs the generic decoder.
template <int MODE>
__device__ bool decode_segment_generic(const Seg& s, GenericTab& G, const DecodeOut& dout,
                                       const GemmOut& gout) {
  for (int l = 0; l < 256; ++l) G.cnt[l] = 0;
  int maxlen = 0;
  for (int sym = 0; sym < 256; ++sym) {
    int l = __ldg(s.lens + sym);
    if (l) {
      G.cnt[l] += 1;
      maxlen = max(maxlen, l);
    }
  }
  // Kraft check: open prefixes per level, clamped once they exceed 256
  int64_t avail = 1;
  for (int l = 1; l <= maxlen; ++l) {
    avail = 2 * avail - G.cnt[l];
    if (avail < 0) return false;
    if (avail > 4096) avail = 4096;
  }
  G.off[0] = 0;
  for (int l = 1; l <= 256; ++l) G.off[l] = uint16_t(G.off[l - 1] + G.cnt[l - 1]);
  for (int sym = 0; sym < 256; ++sym) {
    int l = __ldg(s.lens + sym);
    if (l) G.sorted[G.off[l]++] = uint8_t(sym);
  }
  uint64_t pos = 0;
  const uint8_t* bits = s.bits;
  const uint64_t nbits = s.nbits;
  for (uint64_t i = 0; i < s.count; ++i) {
    int len = 0;
    auto bit_at = [&](int k) -> uint32_t {
      uint64_t q = pos + uint64_t(k);
      return q < nbits ? (__ldg(bits + (q >> 3)) >> (7 - (q & 7))) & 1u : 0u;
    };
    int sym = generic_decode(bit_at, G.cnt, G.sorted, maxlen, &len);
    if (sym < 0) return false;
    pos += uint64_t(len);
    if (pos > nbits) return false;
    uint32_t w = merge1(uint32_t(sym) << 7, __ldg(s.sm + i));
    if (MODE == 0) dout.one(s.start + i, w); else gout.one(s.start + i, w);
  }
  return pos == nbits;
}

__device__ __forceinline__ uint64_t warp_incl_scan(uint64_t v, int lane) {
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    uint64_t t = __shfl_up_sync(0xffffffffu, v, d);
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
  LaneTab* tabs = reinterpret_cast<LaneTab*>(smem + warp * kWarpTabBytes);
  WarpShared* ws = reinterpret_cast<WarpShared*>(smem + PWARPS * kWarpTabBytes) + warp;

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
    // ---- substream table (cuda/parallel.cu:39-51) ----
    const uint64_t total = rows * cols;
    const bool active = uint64_t(lane) < chunks;
    uint64_t len = active ? ld_le64(p + 32 + 8 * lane) : 0;
    bool lok = !active || (len >= kHdr && len <= n);
    uint64_t incl = warp_incl_scan(lok ? len : 0, lane);
    uint64_t base = 32 + 8 * chunks + incl - len;
    Seg s{};
    if (active && lok) {
      lok = base + len <= n;
      if (lok) {
        const uint8_t* q = p + base;
        s.count = ld_le64(q);
        s.nbits = ld_le64(q + 8);
        s.start = total * uint64_t(lane) / chunks;
        uint64_t expect = total * uint64_t(lane + 1) / chunks - s.start;
        s.ebytes = s.nbits / 8 + (s.nbits % 8 != 0);
        lok = s.count == expect && s.count <= len - kHdr && s.ebytes == len - kHdr - s.count;
        s.lens = q + 16;
        s.sm = q + kHdr;
        s.bits = q + kHdr + s.count;
      }
    }
    uint64_t end_all = __shfl_sync(0xffffffffu, base + len, int(chunks - 1));
    bool all_ok = __all_sync(0xffffffffu, lok) && end_all == n;
    if (!all_ok) {
      if (lane == 0) atomicOr(status, kStatusHeader);
      continue;
    }
    // ---- per-lane tables ----
    LaneTab& T = tabs[lane];
    uint32_t F = 0;
    int maxlen = 0;
    int tb = active ? build_lane_tables(s.lens, T, F, maxlen) : 0;
    if (__any_sync(0xffffffffu, tb < 0)) {
      if (lane == 0) atomicOr(status, kStatusCodebook);
      continue;
    }
    uint16_t* o16 = reinterpret_cast<uint16_t*>(out + sd.dst);
    DecodeOut dout{o16, rows, cols};
    GemmOut gout{x + sd.xoff * ld, ws->y, rows, cols, ld, nb};
    if (MODE == 1) {
      for (int k = lane; k < 16 * PMAXB; k += 32) ws->y[k] = 0.f;
      __syncwarp();
    }
    bool nice;
    if (MODE == 0)
      nice = rows == 16 && (cols & 15) == 0 && ((reinterpret_cast<uintptr_t>(o16)) & 15) == 0;
    else
      nice = rows == 16 && (cols & 15) == 0 && nb == 1 && ld == 1 &&
             ((reinterpret_cast<uintptr_t>(gout.x)) & 15) == 0;
    bool bad = false;
    if (active && tb == 0) decode_segment<MODE>(s, T, F, maxlen, nice, dout, gout, bad);
    // ---- substreams that need the generic decoder ----
    uint32_t gmask = __ballot_sync(0xffffffffu, active && tb == 1);
    __syncwarp();
    while (gmask) {
      int g = __ffs(gmask) - 1;
      gmask &= gmask - 1;
      Seg sg;
      sg.lens = reinterpret_cast<const uint8_t*>(__shfl_sync(0xffffffffu, reinterpret_cast<uintptr_t>(s.lens), g));
      sg.sm = reinterpret_cast<const uint8_t*>(__shfl_sync(0xffffffffu, reinterpret_cast<uintptr_t>(s.sm), g));
      sg.bits = reinterpret_cast<const uint8_t*>(__shfl_sync(0xffffffffu, reinterpret_cast<uintptr_t>(s.bits), g));
      sg.count = __shfl_sync(0xffffffffu, s.count, g);
      sg.nbits = __shfl_sync(0xffffffffu, s.nbits, g);
      sg.ebytes = __shfl_sync(0xffffffffu, s.ebytes, g);
      sg.start = __shfl_sync(0xffffffffu, s.start, g);
      if (lane == 0) {
        bool gok = decode_segment_generic<MODE>(sg, *reinterpret_cast<GenericTab*>(tabs), dout, gout);
        if (!gok) bad = true;
      }
      __syncwarp();
    }
    if (__any_sync(0xffffffffu, bad)) {
      if (lane == 0) atomicOr(status, kStatusStream);
      continue;
    }
    if (MODE == 1) {
      __syncwarp();
      for (uint32_t k = lane; k < rows * nb; k += 32) {
        uint32_t r = k / nb, b = k - r * nb;
        y[(sd.dst + r) * ld + b] = ws->y[r * PMAXB + b];
      }
      __syncwarp();
    }
  }
}

}  // namespace

size_t parallel_smem_bytes() { return kSmemBytes; }

cudaError_t launch_parallel_decode(const Slab* slabs, uint32_t n, const uint8_t* payload,
                                   uint8_t* out, int* status, int grid, cudaStream_t st) {
  if (!n) return cudaSuccess;
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(parallel_slab_kernel<0>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kSmemBytes));
    cudaFuncSetAttribute(parallel_slab_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kSmemBytes));
    attr = true;
  }
  int need = int((n + PWARPS - 1) / PWARPS);
  parallel_slab_kernel<0><<<grid < need ? grid : need, PWARPS * 32, kSmemBytes, st>>>(
      slabs, n, payload, out, nullptr, nullptr, 1, 1, status);
  return cudaGetLastError();
}

cudaError_t launch_parallel_gemm(const Slab* slabs, uint32_t n, const uint8_t* payload,
                                 const float* x, float* y, uint32_t ld, uint32_t b0, uint32_t nb,
                                 int* status, int grid, cudaStream_t st) {
  if (!n) return cudaSuccess;
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(parallel_slab_kernel<0>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kSmemBytes));
    cudaFuncSetAttribute(parallel_slab_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kSmemBytes));
    attr = true;
  }
  int need = int((n + PWARPS - 1) / PWARPS);
  parallel_slab_kernel<1><<<grid < need ? grid : need, PWARPS * 32, kSmemBytes, st>>>(
      slabs, n, payload, nullptr, x + b0, y + b0, ld, nb, status);
  return cudaGetLastError();
}

}  // namespace xksv
