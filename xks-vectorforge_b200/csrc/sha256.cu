// SHA-256 (FIPS 180-4) of decoded output ranges on the GPU: the integrity
// check of the .xksv index, whose blocks and tensors carry the SHA-256 of
// their decoded BF16 bytes (reference src/compile.cpp:255 hashes each block's
// raw bytes, :483 the tensor's; src/verify.cpp:262-273 recomputes both after
// decoding).  Hashing on the device avoids copying the decoded weights back
// to the host to verify them.
//
// A message is hashed sequentially (each 64-byte chunk depends on the
// previous state), so the parallelism is one thread per range: a checkpoint's
// slabs are thousands of independent ranges.  Message words are read as
// aligned 32-bit loads, realigned with a funnel shift when the range starts
// off a 4-byte boundary, and byte-swapped to the standard's big-endian order;
// the padding (0x80, zeros, 64-bit bit length) is generated on the fly.
#include <cstdint>

#include "kernels.h"

namespace xksv {
namespace {

// FIPS 180-4 section 4.2.2: first 32 bits of the fractional parts of the cube
// roots of the first 64 primes.
__constant__ uint32_t kSha[64] = {
    0x428a2f98u, 0x71374491u, 0xb5c0fbcfu, 0xe9b5dba5u, 0x3956c25bu, 0x59f111f1u, 0x923f82a4u,
    0xab1c5ed5u, 0xd807aa98u, 0x12835b01u, 0x243185beu, 0x550c7dc3u, 0x72be5d74u, 0x80deb1feu,
    0x9bdc06a7u, 0xc19bf174u, 0xe49b69c1u, 0xefbe4786u, 0x0fc19dc6u, 0x240ca1ccu, 0x2de92c6fu,
    0x4a7484aau, 0x5cb0a9dcu, 0x76f988dau, 0x983e5152u, 0xa831c66du, 0xb00327c8u, 0xbf597fc7u,
    0xc6e00bf3u, 0xd5a79147u, 0x06ca6351u, 0x14292967u, 0x27b70a85u, 0x2e1b2138u, 0x4d2c6dfcu,
    0x53380d13u, 0x650a7354u, 0x766a0abbu, 0x81c2c92eu, 0x92722c85u, 0xa2bfe8a1u, 0xa81a664bu,
    0xc24b8b70u, 0xc76c51a3u, 0xd192e819u, 0xd6990624u, 0xf40e3585u, 0x106aa070u, 0x19a4c116u,
    0x1e376c08u, 0x2748774cu, 0x34b0bcb5u, 0x391c0cb3u, 0x4ed8aa4au, 0x5b9cca4fu, 0x682e6ff3u,
    0x748f82eeu, 0x78a5636fu, 0x84c87814u, 0x8cc70208u, 0x90befffau, 0xa4506cebu, 0xbef9a3f7u,
    0xc67178f2u};

__device__ __forceinline__ uint32_t rotr(uint32_t x, int n) { return __funnelshift_r(x, x, n); }

// Big-endian message word i of the padded message of length len at base.
struct MsgReader {
  const uint32_t* w;  // aligned words covering the range
  uint32_t sh;        // byte misalignment * 8
  uint64_t len, nwords_full;
  __device__ __forceinline__ uint32_t word(uint64_t i, uint64_t total_words) const {
    if (i < nwords_full) {  // four message bytes
      const uint32_t lo = __ldg(w + i);
      const uint32_t v = sh ? __funnelshift_r(lo, __ldg(w + i + 1), sh) : lo;
      return __byte_perm(v, 0, 0x0123);
    }
    if (i >= total_words - 2)  // bit length, big-endian 64-bit
      return i == total_words - 2 ? uint32_t((len * 8) >> 32) : uint32_t(len * 8);
    // the word holding the message tail and/or the 0x80 marker
    uint32_t v = 0;
    for (int k = 0; k < 4; ++k) {
      const uint64_t b = i * 4 + uint64_t(k);
      uint32_t byte = 0;
      if (b < len) {
        const uint64_t q = b + (sh >> 3);  // byte index from the aligned base
        byte = (__ldg(w + (q >> 2)) >> (8 * (q & 3))) & 0xFFu;
      } else if (b == len) {
        byte = 0x80u;
      }
      v = (v << 8) | byte;
    }
    return v;
  }
};

__device__ void sha256_range(const uint8_t* p, uint64_t len, uint32_t* out) {
  uint32_t h[8] = {0x6a09e667u, 0xbb67ae85u, 0x3c6ef372u, 0xa54ff53au,
                   0x510e527fu, 0x9b05688cu, 0x1f83d9abu, 0x5be0cd19u};
  const uintptr_t a = reinterpret_cast<uintptr_t>(p);
  MsgReader m;
  m.w = reinterpret_cast<const uint32_t*>(a & ~uintptr_t(3));
  m.sh = uint32_t(a & 3) * 8;
  m.len = len;
  m.nwords_full = len / 4;
  const uint64_t nchunks = (len + 8) / 64 + 1;
  const uint64_t total_words = nchunks * 16;
  for (uint64_t c = 0; c < nchunks; ++c) {
    uint32_t W[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) W[j] = m.word(c * 16 + uint64_t(j), total_words);
    uint32_t A = h[0], B = h[1], C = h[2], D = h[3], E = h[4], F = h[5], G = h[6], H = h[7];
#pragma unroll
    for (int t = 0; t < 64; ++t) {
      uint32_t wt;
      if (t < 16) {
        wt = W[t];
      } else {
        const uint32_t w15 = W[(t - 15) & 15], w2 = W[(t - 2) & 15];
        const uint32_t s0 = rotr(w15, 7) ^ rotr(w15, 18) ^ (w15 >> 3);
        const uint32_t s1 = rotr(w2, 17) ^ rotr(w2, 19) ^ (w2 >> 10);
        wt = W[t & 15] + s0 + W[(t - 7) & 15] + s1;
        W[t & 15] = wt;
      }
      const uint32_t S1 = rotr(E, 6) ^ rotr(E, 11) ^ rotr(E, 25);
      const uint32_t ch = (E & F) ^ (~E & G);
      const uint32_t t1 = H + S1 + ch + kSha[t] + wt;
      const uint32_t S0 = rotr(A, 2) ^ rotr(A, 13) ^ rotr(A, 22);
      const uint32_t maj = (A & B) ^ (A & C) ^ (B & C);
      const uint32_t t2 = S0 + maj;
      H = G;
      G = F;
      F = E;
      E = D + t1;
      D = C;
      C = B;
      B = A;
      A = t1 + t2;
    }
    h[0] += A;
    h[1] += B;
    h[2] += C;
    h[3] += D;
    h[4] += E;
    h[5] += F;
    h[6] += G;
    h[7] += H;
  }
#pragma unroll
  for (int k = 0; k < 8; ++k) out[k] = h[k];
}

__global__ void sha256_kernel(const uint64_t* __restrict__ ranges, uint32_t n, const uint8_t* __restrict__ base,
                              uint8_t* __restrict__ digests) {
  for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    uint32_t h[8];
    sha256_range(base + ranges[2 * i], ranges[2 * i + 1], h);
    uint8_t* d = digests + 32 * uint64_t(i);
#pragma unroll
    for (int k = 0; k < 8; ++k) {  // digest bytes big-endian
      d[4 * k] = uint8_t(h[k] >> 24);
      d[4 * k + 1] = uint8_t(h[k] >> 16);
      d[4 * k + 2] = uint8_t(h[k] >> 8);
      d[4 * k + 3] = uint8_t(h[k]);
    }
  }
}

}  // namespace

cudaError_t launch_sha256(const uint64_t* d_ranges, uint32_t n, const uint8_t* d_base, uint8_t* d_digests,
                          cudaStream_t st) {
  if (!n) return cudaSuccess;
  const uint32_t threads = 64;
  const uint32_t blocks = (n + threads - 1) / threads;
  sha256_kernel<<<blocks, threads, 0, st>>>(d_ranges, n, d_base, d_digests);
  return cudaGetLastError();
}

}  // namespace xksv
