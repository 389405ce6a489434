// Launchers for the slab kernels (host side, one per codec and mode).
#pragma once
#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

#include "xksv_types.h"

namespace xksv {

size_t parallel_smem_bytes();
size_t serial_smem_bytes();

// Decode slabs[0..n) from payload into out (+ slab.dst bytes each).
cudaError_t launch_parallel_decode(const Slab* slabs, uint32_t n, const uint8_t* payload,
                                   uint8_t* out, int* status, int grid, cudaStream_t st);
cudaError_t launch_serial_decode(const Slab* slabs, uint32_t n, const uint8_t* payload,
                                 uint8_t* out, int* status, int grid, cudaStream_t st);
cudaError_t launch_raw_decode(const Slab* slabs, uint32_t n, const uint8_t* payload, uint8_t* out,
                              int grid, cudaStream_t st);

// Y[dst + r, b0 + b] = sum_c W[r, c] X[xoff + c, b0 + b] for b < nb (nb <= 8),
// X and Y row-major with leading dimension ld.
cudaError_t launch_parallel_gemm(const Slab* slabs, uint32_t n, const uint8_t* payload,
                                 const float* x, float* y, uint32_t ld, uint32_t b0, uint32_t nb,
                                 int* status, int grid, cudaStream_t st);
cudaError_t launch_serial_gemm(const Slab* slabs, uint32_t n, const uint8_t* payload,
                               const float* x, float* y, uint32_t ld, uint32_t b0, uint32_t nb,
                               int* status, int grid, cudaStream_t st);
cudaError_t launch_raw_gemm(const Slab* slabs, uint32_t n, const uint8_t* payload, const float* x,
                            float* y, uint32_t ld, uint32_t b0, uint32_t nb, int grid,
                            cudaStream_t st);

}  // namespace xksv
