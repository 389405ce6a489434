// Tensor-core (tcgen05 / TMEM) GEMM stage of the batch >= 16 fused GEMM.
//
// Y[rows, batch] = W X for a plan's slabs runs as decode -> tensor-core GEMM:
// the plan's decoders (running at full occupancy) write each row group of up
// to 128 weight rows as BF16 into a plan-owned scratch buffer, sized so that
// a linear stays resident in the 126 MB L2, and this kernel multiplies it by X
// on the 5th-generation tensor cores.  (Feeding tcgen05 straight from the
// decoder would need every in-flight decoded tile resident in shared memory,
// ~128 KB per CTA for 256 tiles, leaving one CTA per SM: the decoders are
// latency-bound and need ~32 warps per SM, so the L2 hand-off is faster.)
//
// Per CTA: one 128-row group x one K split.  A (W rows, K-major) and B (X^T,
// K-major) stream through a two-stage shared-memory ring by cp.async in the
// UMMA canonical no-swizzle layout (8-row x 16-byte core matrices); one
// thread issues tcgen05.mma kind::f16 (BF16 x BF16 -> FP32) into a TMEM
// accumulator of 128 lanes x N columns and commits each stage to an
// mbarrier; the epilogue reads TMEM with tcgen05.ld and adds into Y.  Every
// wait is bounded: on a timeout the CTA sets an error bit, drains its copies
// and MMAs (bounded), frees its TMEM and returns.
#include <cuda_bf16.h>

#include <algorithm>

#include "kernels.h"
#include "tcgen05.cuh"

namespace xksv {
namespace {

constexpr int TC_THREADS = 128;
constexpr int TC_KC = 64;              // K per stage (4 MMAs of K = 16)
constexpr int TC_M = 128;              // rows per MMA tile (TMEM lanes)

// Byte offset of (row m, 16-byte K chunk c of a 64-wide stage) in a stage
// buffer holding `rows` rows: K step j = c / 2 occupies rows * 32 bytes; in
// it, 8-row groups are 256 bytes apart (SBO) and the two 8-element halves of
// the K step 128 bytes apart (LBO).
__device__ __forceinline__ uint32_t stage_off(uint32_t m, uint32_t c, uint32_t rows) {
  return (c >> 1) * rows * 32 + (m >> 3) * 256 + (c & 1) * 128 + (m & 7) * 16;
}

__global__ void __launch_bounds__(TC_THREADS) tc_gemm_kernel(TcGemmArgs a) {
  extern __shared__ __align__(1024) uint8_t smem[];
  __shared__ __align__(8) uint64_t bars[2];
  __shared__ uint32_t tmem_base;
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  const TcGroup g = a.groups[blockIdx.x / a.ksplit];
  const uint32_t split = blockIdx.x % a.ksplit;
  const uint32_t npad = a.npad;
  const uint32_t a_bytes = TC_M * TC_KC * 2, b_bytes = npad * TC_KC * 2;
  uint8_t* sA[2] = {smem, smem + a_bytes + b_bytes};
  uint8_t* sB[2] = {smem + a_bytes, smem + 2 * a_bytes + b_bytes};
  // K range of this split, in whole 64-wide chunks
  const uint32_t nchunk_all = (g.cols + TC_KC - 1) / TC_KC;
  const uint32_t per = (nchunk_all + a.ksplit - 1) / a.ksplit;
  const uint32_t c0 = split * per, c1 = min(nchunk_all, c0 + per);
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(
                     smem_addr(&tmem_base)),
                 "r"(a.tmem_cols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::: "memory");
  }
  if (t == 0) {
    mbar_init(smem_addr(&bars[0]), 1);
    mbar_init(smem_addr(&bars[1]), 1);
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_d = tmem_base;
  const uint32_t idesc = umma_idesc_bf16(TC_M, npad);
  const __nv_bfloat16* W = reinterpret_cast<const __nv_bfloat16*>(a.scratch + g.a_off);
  const __nv_bfloat16* XT = static_cast<const __nv_bfloat16*>(a.xt) + g.xoff;
  auto load_stage = [&](uint32_t c, int s) {
    const uint32_t k0 = c * TC_KC;
    const uint32_t dA = smem_addr(sA[s]), dB = smem_addr(sB[s]);
    for (uint32_t i = t; i < TC_M * 8; i += TC_THREADS) {  // A: 128 rows x 8 chunks of 16 B
      const uint32_t m = i >> 3, cc = i & 7, k = k0 + cc * 8;
      const bool ok = m < g.rows && k < g.cols;
      cp_async16_zfill(dA + stage_off(m, cc, TC_M), ok ? W + uint64_t(m) * g.cols + k : W, ok ? 16u : 0u);
    }
    for (uint32_t i = t; i < npad * 8; i += TC_THREADS) {  // B: npad rows of X^T
      const uint32_t n = i >> 3, cc = i & 7, k = k0 + cc * 8;
      const bool ok = k < g.cols;
      cp_async16_zfill(dB + stage_off(n, cc, npad), ok ? XT + uint64_t(n) * a.xt_ld + k : XT, ok ? 16u : 0u);
    }
    asm volatile("cp.async.commit_group;\n" ::: "memory");
  };
  bool ok = true;
  int last_commit = -1;  // thread 0: index (chunk - c0) of its last commit
  if (c0 < c1) load_stage(c0, 0);
  for (uint32_t c = c0; c < c1 && ok; ++c) {
    const int s = int((c - c0) & 1);
    if (c + 1 < c1) {
      const int s1 = s ^ 1;
      if (c + 1 - c0 >= 2) {  // the MMAs that read stage s1 (chunk c - 1) are done
        const uint32_t k = (c - 1 - c0) >> 1;
        if (!mbar_wait(smem_addr(&bars[s1]), k & 1)) ok = false;
      }
      if (__syncthreads_and(ok)) load_stage(c + 1, s1);
      else ok = false;
      asm volatile("cp.async.wait_group 1;\n" ::: "memory");
    } else {
      asm volatile("cp.async.wait_group 0;\n" ::: "memory");
    }
    // this thread's copies are visible to the tensor cores' async proxy
    asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
    ok = __syncthreads_and(ok);
    if (!ok) break;
    if (t == 0) {
      tc_fence_after();
      const uint32_t dA = smem_addr(sA[s]), dB = smem_addr(sB[s]);
#pragma unroll
      for (uint32_t j = 0; j < TC_KC / 16; ++j) {
        const uint64_t ad = umma_desc(dA + j * TC_M * 32, 128, 256);
        const uint64_t bd = umma_desc(dB + j * npad * 32, 128, 256);
        umma_bf16(tmem_d, ad, bd, idesc, (c > c0 || j > 0) ? 1u : 0u);
      }
      umma_commit(smem_addr(&bars[s]));
      last_commit = int(c - c0);
    }
  }
  // all MMAs done (they complete in order: wait for the last commit)
  if (ok && c1 > c0) {
    const uint32_t last = c1 - 1 - c0;
    ok = mbar_wait(smem_addr(&bars[last & 1]), (last >> 1) & 1);
  }
  ok = __syncthreads_and(ok);
  tc_fence_after();
  if (ok && c1 > c0) {
    // epilogue: warp w holds rows 32w..32w+31 (TMEM lanes), one row per lane
    const uint32_t m = uint32_t(warp) * 32 + uint32_t(lane);
    for (uint32_t n0 = 0; n0 < npad; n0 += 16) {
      float v[16];
      tmem_ld16(tmem_d + ((uint32_t(warp) * 32) << 16) + n0, v);
      if (m < g.rows) {
        float* yr = a.y + (g.y_row0 + m) * uint64_t(a.ld);
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const uint32_t n = n0 + uint32_t(i);
          if (n < a.nb) {
            if (a.ksplit > 1)
              atomicAdd(yr + n, v[i]);
            else
              yr[n] = v[i];
          }
        }
      }
    }
  } else if (!ok) {
    if (t == 0) {
      atomicOr(a.status, kStatusInternal);
    }
    asm volatile("cp.async.wait_group 0;\n" ::: "memory");
    // let committed MMAs drain before the accumulator is freed (bounded)
    if (t == 0 && last_commit >= 0)
      mbar_wait(smem_addr(&bars[last_commit & 1]), (uint32_t(last_commit) >> 1) & 1);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tmem_d), "r"(a.tmem_cols)
                 : "memory");
  }
}

// X^T in BF16: xt[n][c] = bf16(x[c * ld + n]) for n < nb, 0 for nb <= n < npad.
__global__ void xt_convert_kernel(const float* __restrict__ x, uint32_t ld, uint32_t nb, uint64_t cols,
                                  uint32_t npad, __nv_bfloat16* __restrict__ xt, uint64_t xt_ld) {
  const uint64_t total = cols * npad;
  for (uint64_t i = blockIdx.x * uint64_t(blockDim.x) + threadIdx.x; i < total;
       i += uint64_t(gridDim.x) * blockDim.x) {
    const uint64_t n = i / cols, c = i - n * cols;
    xt[n * xt_ld + c] = __float2bfloat16_rn(n < nb ? x[c * ld + n] : 0.f);
  }
}

// Zeroes Y[y_row0 + m, 0..nb) of every group (split-K accumulates into Y).
__global__ void zero_rows_kernel(const TcGroup* __restrict__ groups, uint32_t ngroups, float* __restrict__ y,
                                 uint32_t ld, uint32_t nb) {
  for (uint32_t gi = blockIdx.x; gi < ngroups; gi += gridDim.x) {
    const TcGroup g = groups[gi];
    for (uint32_t i = threadIdx.x; i < g.rows * nb; i += blockDim.x) {
      const uint32_t m = i / nb, n = i - m * nb;
      y[(g.y_row0 + m) * uint64_t(ld) + n] = 0.f;
    }
  }
}

}  // namespace

size_t tc_gemm_smem_bytes(uint32_t npad) { return 2 * (size_t(TC_M) * TC_KC * 2 + size_t(npad) * TC_KC * 2); }

cudaError_t launch_tc_gemm(const TcGemmArgs& args, uint32_t ngroups, const float* x, uint64_t x_cols,
                           cudaStream_t st) {
  if (!ngroups) return cudaSuccess;
  if (args.npad < 16 || args.npad > 256 || args.npad % 16) return cudaErrorInvalidValue;
  // shared memory sized so that the CTAs resident on one SM never ask for
  // more than its 512 TMEM columns (an allocation would otherwise stall)
  const size_t per_sm = 233472, fit = 512 / args.tmem_cols;
  const size_t smem = std::max(tc_gemm_smem_bytes(args.npad), per_sm / (fit + 1) + 1024);
  cudaError_t e = cudaFuncSetAttribute(tc_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
  if (e != cudaSuccess) return e;
  e = launch_xt_convert(x, args.ld, args.nb, x_cols, args.npad, const_cast<void*>(args.xt), args.xt_ld, st);
  if (e == cudaSuccess && args.ksplit > 1) e = launch_zero_rows(args.groups, ngroups, args.y, args.ld, args.nb, st);
  if (e != cudaSuccess) return e;
  tc_gemm_kernel<<<ngroups * args.ksplit, TC_THREADS, smem, st>>>(args);
  return cudaGetLastError();
}

cudaError_t launch_xt_convert(const float* x, uint32_t ld, uint32_t nb, uint64_t cols, uint32_t npad, void* xt,
                              uint64_t xt_ld, cudaStream_t st) {
  const uint64_t total = cols * npad;
  if (!total) return cudaSuccess;
  const int cb = int(std::min<uint64_t>((total + 255) / 256, 4096));
  xt_convert_kernel<<<cb, 256, 0, st>>>(x, ld, nb, cols, npad, static_cast<__nv_bfloat16*>(xt), xt_ld);
  return cudaGetLastError();
}

cudaError_t launch_zero_rows(const TcGroup* groups, uint32_t ngroups, float* y, uint32_t ld, uint32_t nb,
                             cudaStream_t st) {
  if (!ngroups) return cudaSuccess;
  zero_rows_kernel<<<std::min<uint32_t>(ngroups, 1024), 256, 0, st>>>(groups, ngroups, y, ld, nb);
  return cudaGetLastError();
}

}  // namespace xksv
