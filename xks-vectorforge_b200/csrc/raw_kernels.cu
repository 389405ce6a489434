// Raw blocks: archive blocks stored as the source bytes (src/compile.cpp:268-
// 275 keeps the original bytes whenever encoding does not shrink a slab).
// Decode copies them (any byte alignment on either side); GEMV/GEMM reads them
// as BF16 row-major [rows, cols] (python/runtime.py:280-282 does this with a
// torch matmul).
#include "kernels.h"
#include "xksv_device.cuh"

namespace xksv {
namespace {

constexpr int RT = 256;

__global__ void __launch_bounds__(RT) raw_copy_kernel(const Slab* __restrict__ slabs, uint32_t n,
                                                      const uint8_t* __restrict__ payload,
                                                      uint8_t* __restrict__ out) {
  for (uint32_t si = blockIdx.x; si < n; si += gridDim.x) {
    const Slab sd = slabs[si];
    const uint8_t* src = payload + sd.src;
    uint8_t* dst = out + sd.dst;
    const uint64_t size = sd.size;
    // head: bytes until dst is 16-byte aligned
    uint64_t head = (16 - (reinterpret_cast<uintptr_t>(dst) & 15)) & 15;
    if (head > size) head = size;
    if (threadIdx.x < head) dst[threadIdx.x] = __ldg(src + threadIdx.x);
    const uint64_t body = (size - head) / 16;
    const uint8_t* s = src + head;
    uint4* d = reinterpret_cast<uint4*>(dst + head);
    const uint8_t* send = src + size;
    if ((reinterpret_cast<uintptr_t>(s) & 15) == 0) {
      const uint4* s4 = reinterpret_cast<const uint4*>(s);
      for (uint64_t k = threadIdx.x; k < body; k += RT) d[k] = ldg16(s4 + k);
    } else {
      // misaligned source: aligned 8-byte loads and funnel shifts
      for (uint64_t k = threadIdx.x; k < body; k += RT) {
        uint64_t lo = ld8_any(s + 16 * k, send), hi = ld8_any(s + 16 * k + 8, send);
        d[k] = make_uint4(uint32_t(lo), uint32_t(lo >> 32), uint32_t(hi), uint32_t(hi >> 32));
      }
    }
    const uint64_t tail0 = head + body * 16;
    for (uint64_t k = tail0 + threadIdx.x; k < size; k += RT) dst[k] = __ldg(src + k);
  }
}

// One warp per output row of one raw BF16 slab.
__global__ void __launch_bounds__(RT) raw_gemm_kernel(const Slab* __restrict__ slabs, uint32_t n,
                                                      const uint8_t* __restrict__ payload,
                                                      const float* __restrict__ x,
                                                      float* __restrict__ y, uint32_t ld,
                                                      uint32_t nb) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (uint32_t si = blockIdx.x; si < n; si += gridDim.x) {
    const Slab sd = slabs[si];
    const uint8_t* src = payload + sd.src;
    for (uint64_t r = warp; r < sd.rows; r += RT / 32) {
      float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
      for (uint64_t c = lane; c < sd.cols; c += 32) {
        const uint8_t* e = src + 2 * (r * sd.cols + c);
        uint32_t word = uint32_t(__ldg(e)) | (uint32_t(__ldg(e + 1)) << 8);
        float w = __uint_as_float(word << 16);
        const float* xr = x + (sd.xoff + c) * ld;
#pragma unroll
        for (int b = 0; b < 8; ++b)
          if (uint32_t(b) < nb) acc[b] = fmaf(w, __ldg(xr + b), acc[b]);
      }
#pragma unroll
      for (int b = 0; b < 8; ++b) {
        float v = acc[b];
        for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if (lane == 0 && uint32_t(b) < nb) y[(sd.dst + r) * ld + b] = v;
      }
    }
  }
}

}  // namespace

cudaError_t launch_raw_decode(const Slab* slabs, uint32_t n, const uint8_t* payload, uint8_t* out,
                              int grid, cudaStream_t st) {
  if (!n) return cudaSuccess;
  raw_copy_kernel<<<grid < int(n) ? grid : int(n), RT, 0, st>>>(slabs, n, payload, out);
  return cudaGetLastError();
}

cudaError_t launch_raw_gemm(const Slab* slabs, uint32_t n, const uint8_t* payload, const float* x,
                            float* y, uint32_t ld, uint32_t b0, uint32_t nb, int grid,
                            cudaStream_t st) {
  if (!n) return cudaSuccess;
  raw_gemm_kernel<<<grid < int(n) ? grid : int(n), RT, 0, st>>>(slabs, n, payload, x + b0, y + b0,
                                                                ld, nb);
  return cudaGetLastError();
}

}  // namespace xksv
