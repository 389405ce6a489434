// Fused decode -> tcgen05 GEMM: Y[rows, batch] = W X for indexed 16-row
// serial-codec slabs, with no decoded weight ever leaving the SM.
//
// Reference behaviour: xksv_cuda_gemm (cuda/decode.cu:28-45, 94-98) decodes
// and multiplies in one pass, one thread per slab row block.  Here the decode
// runs on the CUDA cores and the multiply on the 5th-generation tensor cores
// of the same SM:
//   * a CTA owns a group of up to 32 slabs that read the same X columns and a
//     run of their half tiles (8 rows x 16 columns); lane j of every producer
//     warp decodes slab j with the lane-private canonical tables of
//     lane_decode.cuh, built once per group when the tile index is built and
//     copied into the CTA's shared memory (one set, shared by its warps); a
//     warp's bit stream starts at the tile index's offset of its first half
//     tile and runs contiguously through the following ones;
//   * every producer warp takes its own contiguous share of the CTA's half
//     tiles and decodes tile rows in lock step over its lanes: after row s of
//     a tile, lane j holds the 16 BF16 weights of row 16 j' + s (j' = its
//     slab) for the tile's 16 columns and stores them as row 32 (s % 4) + j of
//     a 128 x 16 stage in the UMMA canonical K-major layout, so four tile rows
//     of 32 slabs fill one stage: the A operand of one M = 128, K = 16 MMA;
//   * stage q (rows 4q .. 4q+3 of every slab) of every tile accumulates into
//     TMEM accumulator D_q (four of them, 128 lanes x npad FP32 columns);
//     B is the tile's 16 rows of X^T (BF16), staged per warp by cp.async;
//   * one thread issues each warp's stages in that warp's order, serving the
//     warps as their stages become ready, and commits each stage back to its
//     producer through an mbarrier (one stage slot per warp: the MMA finishes
//     while the producer decodes its next row);
//   * the epilogue reads D_q with tcgen05.ld (warp r of the first four holds
//     TMEM lanes 32 r .., i.e. row 4q + r of every slab) and adds into Y
//     (several CTAs share a group's rows when its tiles are split).
// Shared memory holds the tables once and, per producer warp, one stage, two
// B slices and the lane rings; no decoded tile is buffered whole, so 19
// producer warps fit one SM beside the stages.  Every wait is bounded: on a
// timeout the CTA sets an error bit, lets its issued MMAs drain, frees its
// TMEM and returns.
#include <cuda_bf16.h>

#include <algorithm>
#include <atomic>

#include "kernels.h"
#include "lane_decode.cuh"
#include "tcgen05.cuh"
#include "xksv_device.cuh"

namespace xksv {
namespace {

// A serial slab's codebook covers up to 16 x 28672 weights: lengths to 32
// bits and up to 32 long codes (measured: <= 20 bits, <= 19 codes above 6
// bits on the BASELINE distributions).
using FCfg = ldec::Cfg<6, 5, 2, 26, 32>;
using ldec::BR;
using ldec::SMR;
constexpr int FR = 1;                           // stage slots per producer warp
constexpr int FMAXP = 19;                       // producer warps at most (20 warps: 5 per SM sub-partition keep 96 registers)
constexpr int FTHREADS = (FMAXP + 1) * 32;      // + the MMA warp
constexpr uint32_t kStageBytes = 128 * 16 * 2;  // 128 rows x K 16, BF16
constexpr size_t kSmemLimit = 232448;           // dynamic shared memory per CTA (227 KB)
constexpr uint32_t kIdleLimit = 1u << 21;       // MMA-thread polls without progress: about a second

// A group's lane tables (lane j: slab j), built once per plan when the tile
// index is built (fused_tables_kernel) and copied into each CTA's shared
// memory at its start.
struct FusedTabs {
  ldec::Tables<FCfg> T;
  uint32_t F[32], L2[32];
  int maxlen[32];
};
static_assert(sizeof(FusedTabs) % 16 == 0, "copied as 16-byte chunks");

struct FusedShared {
  FusedTabs tabs;
  uint32_t hb[FMAXP + 1];  // producer warp w decodes half tiles [hb[w], hb[w + 1]) of the segment
  uint32_t mc[FMAXP];      // MMA thread: stages of warp w consumed in earlier segments
  uint32_t mi[FMAXP];      // MMA thread: stages of warp w issued in this segment
  uint64_t full[FMAXP][FR], empty[FMAXP][FR], done;
  uint32_t tmem_base;
  uint32_t qmask;  // accumulators D_q written by some MMA (a one-half-tile task writes two)
  int abort_flag;
};
constexpr size_t kHdrBytes = (sizeof(FusedShared) + 127) & ~size_t(127);

__host__ __device__ constexpr size_t warp_bytes(uint32_t npad) {
  return FR * kStageBytes + 2 * size_t(npad) * 32 + BR * 32 * 4 + SMR * 32 * 16;
}

// Polls an mbarrier phase; gives up after kSpin polls or when another thread
// of the CTA has aborted.
__device__ __forceinline__ bool mbar_wait_or_abort(uint32_t bar, uint32_t parity, const volatile int* abort_flag) {
  for (uint32_t i = 0; i < kSpin; ++i) {
    uint32_t done;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
        " selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(done)
        : "r"(bar), "r"(parity)
        : "memory");
    if (done) return true;
    if ((i & 255) == 255 && *abort_flag) return false;
    if (i > 64) __nanosleep(64);
  }
  return false;
}

// Non-blocking probe of an mbarrier phase.
__device__ __forceinline__ bool mbar_test(uint32_t bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(done)
      : "r"(bar), "r"(parity)
      : "memory");
  return done != 0;
}

__device__ __forceinline__ void fence_proxy_async() {
  asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
}

// Canonical K-major offset of (row r, 8-element K half h) in a stage or B
// slice: 8-row core matrices of 16-byte rows, K halves 128 bytes apart (LBO),
// 8-row groups 256 bytes apart (SBO).
__device__ __forceinline__ uint32_t kmajor_off(uint32_t r, uint32_t h) {
  return (r >> 3) * 256 + h * 128 + (r & 7) * 16;
}

__global__ void __launch_bounds__(FTHREADS, 1) fused_gemm_kernel(FusedArgs a, uint32_t nprod) {
  extern __shared__ __align__(128) uint8_t smem[];
  FusedShared& S = *reinterpret_cast<FusedShared*>(smem);
  const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t P = nprod, npad = a.npad;
  const uint32_t tmem_cols = 4 * npad <= 32 ? 32 : 4 * npad <= 64 ? 64 : 4 * npad <= 128 ? 128 : 4 * npad <= 256 ? 256 : 512;
  uint8_t* wr = smem + kHdrBytes + size_t(warp) * warp_bytes(npad);  // this producer warp's region
  uint8_t* stage = wr;                                               // [FR][kStageBytes]
  uint8_t* bring = wr + FR * kStageBytes;                            // [2][npad * 32]
  ldec::Ring ring = reinterpret_cast<ldec::Ring>(bring + 2 * npad * 32);
  ldec::SmRing smring = reinterpret_cast<ldec::SmRing>(bring + 2 * npad * 32 + BR * 32 * 4);
  const bool prod = warp < P;

  if (warp == P) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(smem_addr(&S.tmem_base)),
                 "r"(tmem_cols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::: "memory");
  }
  if (threadIdx.x == 0) {
    for (uint32_t w = 0; w < P; ++w) {
      for (int r = 0; r < FR; ++r) {
        mbar_init(smem_addr(&S.full[w][r]), 32);
        mbar_init(smem_addr(&S.empty[w][r]), 1);
      }
      S.mc[w] = 0;
    }
    mbar_init(smem_addr(&S.done), 1);
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    S.abort_flag = 0;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = S.tmem_base;
  uint32_t gm = 0;    // producer: stages this warp has written (all segments)
  uint32_t nseg = 0;  // segments finished (the phase of `done`)

  for (uint32_t sg = a.seg0[blockIdx.x]; sg < a.seg0[blockIdx.x + 1]; ++sg, ++nseg) {
    const FusedTask task = a.tasks[sg];
    const FusedGroup grp = a.groups[task.group];
    const uint32_t span = task.h1 - task.h0;
    if (threadIdx.x == 0) {
      S.qmask = 0;
      for (uint32_t w = 0; w <= P; ++w) S.hb[w] = task.h0 + uint32_t(uint64_t(span) * w / P);
    }
    // ---- producers: this warp's run of half tiles [ha, hb) (half h = rows
    // 8 (h % 2) .. +7 of tile h / 2) and its first loads ----
    const bool active = prod && lane < grp.nslabs;
    uint32_t ha = 0, hb = 0, b0 = 0, b1 = 0;
    ldec::Stream b;
    ldec::SmStream smr;
    if (prod) {
      ha = task.h0 + uint32_t(uint64_t(span) * warp / P);
      hb = task.h0 + uint32_t(uint64_t(span) * (warp + 1) / P);
    }
    auto load_b = [&](uint32_t k, uint32_t slot) {  // X^T rows 0..npad-1, columns of tile k
      const __nv_bfloat16* xt = static_cast<const __nv_bfloat16*>(a.xt) + grp.xoff + 16 * uint64_t(k);
      for (uint32_t i = lane; i < 2 * npad; i += 32) {
        const uint32_t n = i >> 1, h = i & 1;
        cp_async16(bring + slot * npad * 32 + kmajor_off(n, h), xt + uint64_t(n) * a.xt_ld + 8 * h);
      }
    };
    if (active && ha < hb) {
      const uint32_t si = a.members[grp.m0 + lane];
      const Slab sd = a.slabs[si];
      const uint8_t* sm = a.payload + sd.src + kHdr;
      const uint8_t* bits = sm + sd.rows * sd.cols;
      const uint32_t* ti = a.tidx + a.tbase[si];
      const uint32_t* tm = a.tmid + a.tbase[si];
      b0 = (ha & 1) ? tm[ha >> 1] : ti[ha >> 1];
      b1 = (hb & 1) ? tm[hb >> 1] : ti[hb >> 1];
      if (b1 < b0) b1 = b0;  // an index that does not describe this payload: the bit count check rejects it
      b.start(bits + (b0 >> 3), uint64_t((b1 + 7) >> 3) - (b0 >> 3), b0 & 7);
      // a half tile's 128 sign/mantissa bytes follow the previous half's
      smr.init(smring, lane, sm + 128 * uint64_t(ha), sm + 128 * uint64_t(hb));
    }
    // the group's lane tables, built when the index was: one round trip
    {
      const uint4* src = static_cast<const uint4*>(a.tabs) + size_t(task.group) * (sizeof(FusedTabs) / 16);
      uint4* dst = reinterpret_cast<uint4*>(&S.tabs);
      for (uint32_t i = threadIdx.x; i < sizeof(FusedTabs) / 16; i += blockDim.x) cp_async16(dst + i, src + i);
    }
    cp_async_commit();
    cp_async_wait_all();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const bool go = S.abort_flag == 0;
    // X^T and the zeroed Y come from the preceding prep kernel, launched as
    // this grid's programmatic prerequisite: everything above overlapped it
    asm volatile("griddepcontrol.wait;\n" ::: "memory");

    if (prod && go && ha < hb) {
      // ---- decode tile rows into the stage ring ----
      const ldec::Code lc{S.tabs.F[lane], S.tabs.L2[lane], S.tabs.maxlen[lane]};
      if (active) b.init_ring(ring, int(lane));
      load_b(ha >> 1, 0);  // later tiles' slices are loaded eight rows ahead
      bool bad = false, ok = true;
      const uint32_t t0 = ha >> 1, tlast = (hb - 1) >> 1;  // the warp's first and last tile
      for (uint32_t h = ha; h < hb && ok; ++h) {
        const uint32_t k = h >> 1, tl = k - t0;
        for (uint32_t s = 8 * (h & 1); s < 8 * (h & 1) + 8; ++s) {
          uint4 v0 = make_uint4(0, 0, 0, 0), v1 = v0;
          if (active) smr.stage(smring, int(lane));
          cp_async_commit();
          if (active) b.maintain(ring, int(lane));
          ldec::cp_async_wait_2();
          if (active) {
            const uint4 s16 = smr.take(smring, int(lane));
            uint32_t e[16];
#pragma unroll
            for (int q = 0; q < 4; ++q)
              ldec::dec4<FCfg>(b, ring, S.tabs.T, int(lane), lc, bad, e[4 * q], e[4 * q + 1], e[4 * q + 2], e[4 * q + 3]);
            ldec::merge16(e, s16, v0, v1);
          }
          const uint32_t slot = gm % FR;
          if ((s & 3) == 0) {
            // the slot's previous stage (gm - FR) has been multiplied
            if (gm >= FR && !mbar_wait_or_abort(smem_addr(&S.empty[warp][slot]), ((gm / FR) - 1) & 1, &S.abort_flag)) {
              ok = false;
              break;
            }
            // at row 8 that also retired every MMA of the previous tile (or
            // this is the warp's first stage of the segment): the other B
            // slot is free
            if (s == 8 && k + 1 <= tlast) load_b(k + 1, (tl + 1) & 1);
          }
          uint8_t* row = stage + slot * kStageBytes;
          const uint32_t r = 32 * (s & 3) + lane;
          *reinterpret_cast<uint4*>(row + kmajor_off(r, 0)) = v0;
          *reinterpret_cast<uint4*>(row + kmajor_off(r, 1)) = v1;
          if ((s & 3) == 3) {
            // this lane's stage rows and its share of the tile's B slice (its
            // cp.async group completed at least five rows ago) reach the
            // tensor cores
            fence_proxy_async();
            mbar_arrive(smem_addr(&S.full[warp][slot]));
            ++gm;
          }
        }
      }
      cp_async_wait_all();
      if (!ok) {
        if (lane == 0) atomicOr(a.status, kStatusInternal);
        S.abort_flag = 1;
      }
      if (active && ok && (bad || b.pos - b.pos0 != b1 - b0)) atomicOr(a.status, kStatusStream);
    } else if (warp == P && lane == 0 && go) {
      // ---- MMA issue: every warp's stages in its own order, the warps
      // served as their stages become ready.  Stage m of warp w is half tile
      // h = hb[w] + m / 2, rows 4 (m % 2) .. of it, i.e. tile rows 4 q ..
      // 4 q + 3 with q = 2 (h % 2) + m % 2 ----
      const uint32_t idesc = umma_idesc_bf16(128, npad);
      uint32_t left = 0;
      for (uint32_t w = 0; w < P; ++w) {
        S.mi[w] = 0;
        left += 2 * (S.hb[w + 1] - S.hb[w]);
      }
      uint32_t init = 0;  // D_q written once already
      bool ok = true;
      uint32_t idle = 0;
      while (left && ok) {
        bool issued = false;
        for (uint32_t w = 0; w < P; ++w) {
          const uint32_t m = S.mi[w];
          if (m >= 2 * (S.hb[w + 1] - S.hb[w])) continue;
          const uint32_t mg = S.mc[w] + m;  // the warp's stage count over all segments
          const uint32_t slot = mg % FR;
          if (!mbar_test(smem_addr(&S.full[w][slot]), (mg / FR) & 1)) continue;
          tc_fence_after();
          const uint32_t h = S.hb[w] + (m >> 1);
          const uint32_t q = 2 * (h & 1) + (m & 1), tl = (h >> 1) - (S.hb[w] >> 1);
          const uint8_t* wr_w = smem + kHdrBytes + size_t(w) * warp_bytes(npad);
          const uint64_t ad = umma_desc(smem_addr(wr_w + slot * kStageBytes), 128, 256);
          const uint64_t bd = umma_desc(smem_addr(wr_w + FR * kStageBytes + (tl & 1) * npad * 32), 128, 256);
          umma_bf16(tmem + q * npad, ad, bd, idesc, (init >> q) & 1);
          init |= 1u << q;
          umma_commit(smem_addr(&S.empty[w][slot]));
          S.mi[w] = m + 1;
          --left;
          issued = true;
        }
        if (issued) {
          idle = 0;
        } else if (++idle > kIdleLimit || S.abort_flag) {
          ok = false;
        } else if (idle > 32) {
          __nanosleep(64);
        }
      }
      for (uint32_t w = 0; w < P; ++w) S.mc[w] += 2 * (S.hb[w + 1] - S.hb[w]);
      if (!ok) {
        atomicOr(a.status, kStatusInternal);
        S.abort_flag = 1;
      }
      S.qmask = init;
      // every MMA issued above is complete once `done` flips (bounded wait)
      umma_commit(smem_addr(&S.done));
      if (!mbar_wait(smem_addr(&S.done), nseg & 1)) {
        atomicOr(a.status, kStatusInternal);
        S.abort_flag = 1;
      }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    // ---- epilogue: warp r < 4 holds TMEM lanes 32 r .. 32 r + 31 ----
    if (warp < 4 && S.abort_flag == 0) {
      const bool mine = lane < grp.nslabs;
      const uint64_t row0 = mine ? a.slabs[a.members[grp.m0 + lane]].dst : 0;
      for (uint32_t q = 0; q < 4; ++q) {
        if (!((S.qmask >> q) & 1)) continue;  // no MMA wrote D_q: nothing to add
        for (uint32_t n0 = 0; n0 < npad; n0 += 16) {
          float v[16];
          tmem_ld16(tmem + ((warp * 32) << 16) + q * npad + n0, v);
          if (mine) {
            float* yr = a.y + (row0 + 4 * q + warp) * uint64_t(a.ld);
#pragma unroll
            for (int i = 0; i < 16; ++i)
              if (n0 + uint32_t(i) < a.nb) atomicAdd(yr + n0 + i, v[i]);
          }
        }
      }
    }
    // the accumulators, stage areas and tables are free for the next segment
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (S.abort_flag) break;
  }
  if (warp == P) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tmem), "r"(tmem_cols) : "memory");
  }
}

// X^T in BF16 (xt[n][c] = bf16(x[c * ld + n]), zero for nb <= n < npad) and
// Y[rows of every group, 0..nb) = 0, in one launch that first lets the fused
// kernel launch behind it (programmatic dependent launch): the fused CTAs
// start their stream loads and table builds while this runs.
__global__ void fused_prep_kernel(const float* __restrict__ x, uint32_t ld, uint32_t nb, uint64_t cols,
                                  uint32_t npad, __nv_bfloat16* __restrict__ xt, uint64_t xt_ld,
                                  const TcGroup* __restrict__ groups, uint32_t ngroups, float* __restrict__ y) {
  asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");
  const uint64_t stride = uint64_t(gridDim.x) * blockDim.x;
  const uint64_t total = cols * npad;
  for (uint64_t i = blockIdx.x * uint64_t(blockDim.x) + threadIdx.x; i < total; i += stride) {
    const uint64_t n = i / cols, c = i - n * cols;
    xt[n * xt_ld + c] = __float2bfloat16_rn(n < nb ? x[c * ld + n] : 0.f);
  }
  for (uint32_t gi = blockIdx.x; gi < ngroups; gi += gridDim.x) {
    const TcGroup g = groups[gi];
    for (uint32_t i = threadIdx.x; i < g.rows * nb; i += blockDim.x) {
      const uint32_t m = i / nb, n = i - m * nb;
      y[(g.y_row0 + m) * uint64_t(ld) + n] = 0.f;
    }
  }
}

// One warp per group: lane j builds slab j's tables (the codes of its 256
// lengths, read from the payload) and the warp writes the group's FusedTabs.
// A lane whose codebook does not fit or is oversubscribed sets the status.
__global__ void __launch_bounds__(32) fused_tables_kernel(const FusedGroup* __restrict__ groups,
                                                          const uint32_t* __restrict__ members,
                                                          const Slab* __restrict__ slabs,
                                                          const uint8_t* __restrict__ payload, FusedTabs* tabs,
                                                          int* status) {
  __shared__ __align__(16) FusedTabs t;
  __shared__ uint8_t lpos[FCfg::PNL][32];
  __shared__ uint32_t save[12][32];
  const int lane = threadIdx.x;
  const FusedGroup g = groups[blockIdx.x];
  uint4* z = reinterpret_cast<uint4*>(&t.T.lut2[0][0]);
  for (uint32_t k = lane; k < sizeof(t.T.lut2) / 16; k += 32) z[k] = make_uint4(0, 0, 0, 0);
  __syncwarp();
  uint32_t F = 0, L = 0;
  int mx = 0, tb = 0;
  if (uint32_t(lane) < g.nslabs) {
    ldec::GlobalLens lens(payload + slabs[members[g.m0 + lane]].src + 16, save, lane);
    tb = ldec::build_tables<FCfg>(lens, t.T, lpos, lane, F, mx, L);
  }
  t.F[lane] = F;
  t.L2[lane] = L << FCfg::K2;
  t.maxlen[lane] = mx;
  if (tb != 0) atomicOr(status, tb < 0 ? kStatusCodebook : kStatusInternal);
  __syncwarp();
  const uint4* src = reinterpret_cast<const uint4*>(&t);
  uint4* dst = reinterpret_cast<uint4*>(tabs + blockIdx.x);
  for (uint32_t i = lane; i < sizeof(FusedTabs) / 16; i += 32) dst[i] = src[i];
}

// ok[i] = 1 when slab i's codebook fits the fused decoder's lane tables
// (lengths <= PK + PNL, at most PLONG codes longer than PK).
__global__ void fused_check_kernel(const Slab* __restrict__ slabs, uint32_t n, const uint8_t* __restrict__ payload,
                                   uint8_t* __restrict__ ok) {
  for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    const uint8_t* lens = payload + slabs[i].src + 16;
    uint32_t nlong = 0, mx = 0;
    for (int s = 0; s < 256; ++s) {
      const uint32_t l = __ldg(lens + s);
      mx = max(mx, l);
      nlong += l > uint32_t(FCfg::PK);
    }
    ok[i] = mx <= uint32_t(FCfg::PK + FCfg::PNL) && nlong <= uint32_t(FCfg::PLONG);
  }
}

}  // namespace

uint32_t fused_producers(uint32_t npad, size_t* smem_bytes) {
  if (npad < 16 || npad > 128 || npad % 16) return 0;
  const size_t per = warp_bytes(npad);
  const uint32_t p = uint32_t(std::min<size_t>(FMAXP, (kSmemLimit - kHdrBytes) / per));
  if (p < 4) return 0;  // the epilogue needs warps 0-3
  if (smem_bytes) *smem_bytes = kHdrBytes + p * per;
  return p;
}

size_t fused_tables_bytes() { return sizeof(FusedTabs); }

cudaError_t launch_fused_tables(const FusedGroup* groups, uint32_t ngroups, const uint32_t* members,
                                const Slab* slabs, const uint8_t* payload, void* tabs, int* status,
                                cudaStream_t st) {
  if (!ngroups) return cudaSuccess;
  fused_tables_kernel<<<ngroups, 32, 0, st>>>(groups, members, slabs, payload, static_cast<FusedTabs*>(tabs), status);
  return cudaGetLastError();
}

cudaError_t launch_fused_check(const Slab* slabs, uint32_t n, const uint8_t* payload, uint8_t* ok,
                               cudaStream_t st) {
  if (!n) return cudaSuccess;
  fused_check_kernel<<<(n + 127) / 128, 128, 0, st>>>(slabs, n, payload, ok);
  return cudaGetLastError();
}

cudaError_t launch_fused_gemm(const FusedArgs& args, uint32_t nctas, const float* x, uint64_t x_cols,
                              const TcGroup* groups, uint32_t ngroups, cudaStream_t st) {
  if (!nctas) return cudaSuccess;
  size_t smem = 0;
  const uint32_t p = fused_producers(args.npad, &smem);
  if (!p) return cudaErrorInvalidValue;
  // dynamic shared memory opt-in, once per device (concurrent first calls set the same value)
  static std::atomic<uint64_t> done{0};
  int dev = 0;
  cudaGetDevice(&dev);
  const uint64_t bit = dev < 64 ? (1ull << dev) : 0ull;
  if (!bit || !(done.load(std::memory_order_acquire) & bit)) {
    const cudaError_t e =
        cudaFuncSetAttribute(fused_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kSmemLimit));
    if (e != cudaSuccess) return e;
    if (bit) done.fetch_or(bit, std::memory_order_release);
  }
  const uint64_t work = std::max<uint64_t>(x_cols * args.npad, uint64_t(ngroups) * 256);
  const int pb = int(std::min<uint64_t>((work + 255) / 256, 1024));
  fused_prep_kernel<<<pb, 256, 0, st>>>(x, args.ld, args.nb, x_cols, args.npad,
                                        static_cast<__nv_bfloat16*>(const_cast<void*>(args.xt)), args.xt_ld, groups,
                                        ngroups, args.y);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(nctas);
  cfg.blockDim = dim3((p + 1) * 32);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, fused_gemm_kernel, args, p);
}

}  // namespace xksv
