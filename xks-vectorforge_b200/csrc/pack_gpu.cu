// Archive-side encoder on the GPU: the slabs of xksv_host_pack_tensor, byte
// for byte, built from a row-major BF16 tensor already in device memory (the
// compile step of src/compile.cpp:247-285, 449-479 with the block encoders of
// src/c_api.cpp:18-28, 44-65 and src/codec.cpp:32-58).
//
// Coding blocks are the serial codec's slabs, or the <= 32 substreams of each
// parallel-codec slab (tiled ranges [n*i/c, n*(i+1)/c)).  Steps:
//   1. histogram of the exponent bytes per block (one CTA per block);
//   2. Huffman code lengths with the reference's tie order -- leaves sorted by
//      (frequency, symbol) with a bitonic sort in shared memory, then the
//      two-queue merge (leaves and internal nodes, the smaller (frequency,
//      node index) first) by one thread -- and canonical codes;
//   3. sizes and raw-fallback decisions on the host (the encoding is kept only
//      when smaller than the raw bytes), payload offsets;
//   4. headers, sign/mantissa bytes in tile order, container headers, raw copies;
//   5. the exponent bit stream: each thread packs a contiguous run of codes at
//      the bit offset a block scan gives it, OR-ing whole big-endian 32-bit
//      words, so words shared with a neighbour's run merge without a race.
#include <algorithm>
#include <cstring>
#include <vector>

#include "kernels.h"
#include "xksv_cuda.h"
#include "xksv_device.cuh"

namespace xksv {
namespace {

struct PackBlock {
  uint64_t data_off;  // first element of the slab in the tensor (row-major)
  uint32_t rows, cols;  // the slab
  uint32_t start, count;  // tiled range of the block inside the slab
  uint64_t out_off;   // byte offset of the block's serial header in the payload; ~0 = raw slab
};

__device__ __forceinline__ uint32_t word_at(const uint16_t* d, const PackBlock& b, uint32_t p) {
  const uint64_t idx = untile_index(p, b.rows, b.cols);
  return d[b.data_off + idx];
}

__global__ void pack_hist_kernel(const PackBlock* __restrict__ blocks, const uint16_t* __restrict__ d,
                                 uint32_t* __restrict__ freq) {
  __shared__ uint32_t h[256];
  const PackBlock b = blocks[blockIdx.x];
  h[threadIdx.x] = 0;
  __syncthreads();
  for (uint32_t i = threadIdx.x; i < b.count; i += blockDim.x)
    atomicAdd(&h[(word_at(d, b, b.start + i) >> 7) & 255u], 1u);
  __syncthreads();
  freq[blockIdx.x * 256ull + threadIdx.x] = h[threadIdx.x];
}

// Code lengths (<= 32) and canonical codes per block; bits[b] = total code
// bits, or ~0 when a length exceeds 32 (beyond this encoder's word packing;
// not reachable for <= 1 MiB slabs).
__global__ void pack_codes_kernel(const uint32_t* __restrict__ freq, uint8_t* __restrict__ lens_out,
                                  uint32_t* __restrict__ codes_out, uint64_t* __restrict__ bits_out) {
  __shared__ uint64_t key[256];  // (frequency << 8 | symbol), zero-frequency last
  __shared__ uint64_t nf[512];   // node frequencies
  __shared__ int16_t par[512];   // node parents
  __shared__ int16_t lsym[256];  // leaf node -> symbol
  __shared__ uint8_t lens[256];
  __shared__ int nleaf_s;
  const int t = threadIdx.x;
  const uint32_t f = freq[blockIdx.x * 256ull + t];
  key[t] = f ? (uint64_t(f) << 8) | uint64_t(t) : ~0ull;
  lens[t] = 0;
  __syncthreads();
  // bitonic sort of 256 keys, ascending
  for (int k = 2; k <= 256; k <<= 1) {
    for (int j = k >> 1; j > 0; j >>= 1) {
      const int q = t ^ j;
      if (q > t) {
        const uint64_t a = key[t], c = key[q];
        const bool up = (t & k) == 0;
        if ((a > c) == up) {
          key[t] = c;
          key[q] = a;
        }
      }
      __syncthreads();
    }
  }
  if (t == 0) {
    // leaves are nodes 0..n-1 in symbol order; sorted queue `key` holds them
    // in (frequency, symbol) = (frequency, node index) order
    int n = 0;
    for (int s = 0; s < 256; ++s)
      if (freq[blockIdx.x * 256ull + s]) {
        nf[n] = freq[blockIdx.x * 256ull + s];
        lsym[n] = int16_t(s);
        ++n;
      }
    nleaf_s = n;
    // node index of the sorted leaf at position i: the rank of its symbol
    // among present symbols (leaf indices follow symbol order)
    int li = 0, ii = n, m = n;
    auto leaf_node = [&](int i) -> int {
      const int sym = int(key[i] & 255u);
      int r = 0;
      while (lsym[r] != sym) ++r;
      return r;
    };
    int cur_leaf = n > 0 ? leaf_node(0) : 0;
    auto pick = [&]() -> int {
      const bool lok = li < n, iok = ii < m;
      if (lok && (!iok || nf[cur_leaf] < nf[ii] || (nf[cur_leaf] == nf[ii] && cur_leaf < ii))) {
        const int r = cur_leaf;
        ++li;
        if (li < n) cur_leaf = leaf_node(li);
        return r;
      }
      return ii++;
    };
    while ((n - li) + (m - ii) > 1) {
      const int a = pick(), c = pick();
      nf[m] = nf[a] + nf[c];
      par[a] = int16_t(m);
      par[c] = int16_t(m);
      ++m;
    }
    // depths: the root is the last node; parents come after children
    bool ok = true;
    if (n == 1) {
      lens[lsym[0]] = 1;
    } else if (n > 1) {
      int dep[512];
      dep[m - 1] = 0;
      for (int i = m - 2; i >= 0; --i) dep[i] = dep[par[i]] + 1;
      for (int i = 0; i < n; ++i) {
        if (dep[i] > 32) ok = false;
        lens[lsym[i]] = uint8_t(dep[i] > 255 ? 255 : dep[i]);
      }
    }
    if (!ok) nleaf_s = -1;
  }
  __syncthreads();
  lens_out[blockIdx.x * 256ull + t] = lens[t];
  if (t == 0) {
    uint64_t bits = 0;
    if (nleaf_s < 0) {
      bits = ~0ull;
    } else {
      // canonical codes: by (length, symbol), each the previous plus one, left-aligned
      uint32_t code = 0;
      int prev = 0;
      bool first = true;
      for (int l = 1; l <= 32; ++l)
        for (int s = 0; s < 256; ++s)
          if (lens[s] == l) {
            if (!first) code = (code + 1) << (l - prev);
            first = false;
            prev = l;
            codes_out[blockIdx.x * 256ull + s] = code;
            bits += uint64_t(freq[blockIdx.x * 256ull + s]) * uint64_t(l);
          }
    }
    bits_out[blockIdx.x] = bits;
  }
}

__device__ __forceinline__ void put64d(uint8_t* p, uint64_t v) {
  for (int i = 0; i < 8; ++i) p[i] = uint8_t(v >> (8 * i));
}

// Serial headers and sign/mantissa bytes of every coded block.
__global__ void pack_body_kernel(const PackBlock* __restrict__ blocks, const uint16_t* __restrict__ d,
                                 const uint8_t* __restrict__ lens, const uint64_t* __restrict__ bits,
                                 uint8_t* __restrict__ out) {
  const PackBlock b = blocks[blockIdx.x];
  if (b.out_off == ~0ull) return;  // the slab is stored raw
  uint8_t* o = out + b.out_off;
  if (threadIdx.x == 0) {
    put64d(o, b.count);
    put64d(o + 8, bits[blockIdx.x]);
  }
  for (uint32_t s = threadIdx.x; s < 256; s += blockDim.x) o[16 + s] = lens[blockIdx.x * 256ull + s];
  uint8_t* sm = o + 272;
  for (uint32_t i = threadIdx.x; i < b.count; i += blockDim.x) {
    const uint32_t w = word_at(d, b, b.start + i);
    sm[i] = uint8_t(((w >> 8) & 0x80u) | (w & 0x7Fu));
  }
}

// The exponent bit stream of every coded block.
__global__ void pack_bits_kernel(const PackBlock* __restrict__ blocks, const uint16_t* __restrict__ d,
                                 const uint8_t* __restrict__ lens_all, const uint32_t* __restrict__ codes_all,
                                 uint8_t* __restrict__ out) {
  __shared__ uint8_t lens[256];
  __shared__ uint32_t codes[256];
  __shared__ uint64_t wsum[32];
  const PackBlock b = blocks[blockIdx.x];
  if (b.out_off == ~0ull) return;  // the slab is stored raw
  const int t = threadIdx.x, nt = blockDim.x;
  for (int s = t; s < 256; s += nt) {
    lens[s] = lens_all[blockIdx.x * 256ull + s];
    codes[s] = codes_all[blockIdx.x * 256ull + s];
  }
  __syncthreads();
  // thread t codes elements [i0, i1) of the block
  const uint32_t per = (b.count + nt - 1) / nt;
  const uint32_t i0 = min(b.count, uint32_t(t) * per), i1 = min(b.count, i0 + per);
  uint64_t mine = 0;
  for (uint32_t i = i0; i < i1; ++i) mine += lens[(word_at(d, b, b.start + i) >> 7) & 255u];
  // exclusive scan of the runs' bit counts
  uint64_t v = mine;
  const int lane = t & 31, warp = t >> 5;
  for (int k = 1; k < 32; k <<= 1) {
    const uint64_t u = __shfl_up_sync(0xffffffffu, v, k);
    if (lane >= k) v += u;
  }
  if (lane == 31) wsum[warp] = v;
  __syncthreads();
  uint64_t pre = 0;
  for (int w = 0; w < warp; ++w) pre += wsum[w];
  uint64_t G = pre + v - mine;  // bit offset of this run in the stream
  // stream words: big-endian 32-bit values from the aligned address below the stream start
  uint8_t* e = out + b.out_off + 272 + b.count;
  const uintptr_t ea = reinterpret_cast<uintptr_t>(e);
  uint32_t* words = reinterpret_cast<uint32_t*>(ea & ~uintptr_t(3));
  G += uint64_t(ea & 3) * 8;
  uint64_t stage = 0;  // bits of words sw, sw + 1 (bit 63 = word sw's first bit)
  uint64_t sw = G >> 5;
  auto flush = [&](uint64_t widx, uint32_t val) {
    if (val) atomicOr(words + widx, __byte_perm(val, 0, 0x0123));
  };
  for (uint32_t i = i0; i < i1; ++i) {
    const uint32_t s = (word_at(d, b, b.start + i) >> 7) & 255u;
    const uint32_t l = lens[s];
    const uint64_t w = G >> 5;
    if (w != sw) {
      flush(sw, uint32_t(stage >> 32));
      if (w == sw + 1) {
        stage <<= 32;
      } else {
        flush(sw + 1, uint32_t(stage));
        stage = 0;
      }
      sw = w;
    }
    stage |= uint64_t(codes[s]) << (64 - (G & 31) - l);
    G += l;
  }
  flush(sw, uint32_t(stage >> 32));
  flush(sw + 1, uint32_t(stage));
}

// Parallel-codec container headers and raw-fallback slabs.
struct PackSlab {
  uint64_t data_off, out_off, raw_bytes;
  uint32_t rows, cols, kind, chunks;  // kind: 0 raw, 1 serial, 2 parallel
  uint32_t first_block;
};

__global__ void pack_slab_kernel(const PackSlab* __restrict__ slabs, const PackBlock* __restrict__ blocks,
                                 const uint64_t* __restrict__ block_bytes, const uint8_t* __restrict__ dbytes,
                                 uint8_t* __restrict__ out) {
  const PackSlab s = slabs[blockIdx.x];
  uint8_t* o = out + s.out_off;
  if (s.kind == 0) {
    for (uint64_t i = threadIdx.x; i < s.raw_bytes; i += blockDim.x) o[i] = dbytes[s.data_off * 2 + i];
  } else if (s.kind == 2 && threadIdx.x == 0) {
    const char magic[8] = {'X', 'K', 'S', 'P', '2', 0, 0, 0};
    for (int i = 0; i < 8; ++i) o[i] = uint8_t(magic[i]);
    put64d(o + 8, s.rows);
    put64d(o + 16, s.cols);
    put64d(o + 24, s.chunks);
    for (uint32_t i = 0; i < s.chunks; ++i) put64d(o + 32 + 8 * i, block_bytes[s.first_block + i]);
  }
}

}  // namespace
}  // namespace xksv

extern "C" {

int xksv_cuda_pack_tensor(const void* d_data, size_t rows, size_t cols, int codec, uint64_t dst_base,
                          void** d_payload, size_t* payload_size, xksv_slab** table, size_t* nslabs,
                          void* stream) {
  using namespace xksv;
  if (!d_data || !d_payload || !payload_size || !table || !nslabs) return 1;
  if (codec != XKSV_CODEC_TILE16 && codec != XKSV_CODEC_PARALLEL32) return 1;
  if (!rows || !cols || (reinterpret_cast<uintptr_t>(d_data) & 1)) return 1;
  constexpr uint64_t chunk = 1 << 20;  // slab geometry of src/compile.cpp:449-457, 471-479
  if (cols > chunk / 2 || rows > (1ull << 40) / cols) return 1;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const uint64_t rows_per = std::min<uint64_t>(16, chunk / (cols * 2));
  const size_t ns = (rows + rows_per - 1) / rows_per;
  std::vector<PackBlock> blocks;
  std::vector<PackSlab> slabs(ns);
  for (size_t i = 0; i < ns; ++i) {
    const uint64_t r0 = i * rows_per, nr = std::min<uint64_t>(rows_per, rows - r0);
    const uint64_t n = nr * cols;
    PackSlab& s = slabs[i];
    s.data_off = r0 * cols;
    s.rows = uint32_t(nr);
    s.cols = uint32_t(cols);
    s.raw_bytes = n * 2;
    s.first_block = uint32_t(blocks.size());
    s.kind = uint32_t(codec);
    s.chunks = codec == XKSV_CODEC_PARALLEL32 ? uint32_t(std::min<uint64_t>(32, n)) : 1;
    for (uint32_t k = 0; k < s.chunks; ++k) {
      const uint64_t a = codec == XKSV_CODEC_PARALLEL32 ? n * k / s.chunks : 0;
      const uint64_t z = codec == XKSV_CODEC_PARALLEL32 ? n * (k + 1) / s.chunks : n;
      blocks.push_back(PackBlock{s.data_off, s.rows, s.cols, uint32_t(a), uint32_t(z - a), 0});
    }
  }
  const size_t nb = blocks.size();
  PackBlock* d_blocks = nullptr;
  uint32_t *d_freq = nullptr, *d_codes = nullptr;
  uint8_t* d_lens = nullptr;
  uint64_t *d_bits = nullptr, *d_bbytes = nullptr;
  PackSlab* d_slabs = nullptr;
  uint8_t* d_out = nullptr;
  auto cleanup = [&] {
    cudaFree(d_blocks);
    cudaFree(d_freq);
    cudaFree(d_codes);
    cudaFree(d_lens);
    cudaFree(d_bits);
    cudaFree(d_bbytes);
    cudaFree(d_slabs);
  };
  const uint16_t* d = static_cast<const uint16_t*>(d_data);
  bool ok = cudaMalloc(&d_blocks, nb * sizeof(PackBlock)) == cudaSuccess &&
            cudaMalloc(&d_freq, nb * 256 * 4) == cudaSuccess && cudaMalloc(&d_codes, nb * 256 * 4) == cudaSuccess &&
            cudaMalloc(&d_lens, nb * 256) == cudaSuccess && cudaMalloc(&d_bits, nb * 8) == cudaSuccess &&
            cudaMalloc(&d_bbytes, nb * 8) == cudaSuccess &&
            cudaMemsetAsync(d_codes, 0, nb * 256 * 4, st) == cudaSuccess &&
            cudaMemcpyAsync(d_blocks, blocks.data(), nb * sizeof(PackBlock), cudaMemcpyHostToDevice, st) ==
                cudaSuccess;
  if (ok) {
    pack_hist_kernel<<<unsigned(nb), 256, 0, st>>>(d_blocks, d, d_freq);
    pack_codes_kernel<<<unsigned(nb), 256, 0, st>>>(d_freq, d_lens, d_codes, d_bits);
    ok = cudaGetLastError() == cudaSuccess;
  }
  std::vector<uint64_t> bits(nb);
  ok = ok && cudaMemcpyAsync(bits.data(), d_bits, nb * 8, cudaMemcpyDeviceToHost, st) == cudaSuccess &&
       cudaStreamSynchronize(st) == cudaSuccess;
  if (!ok) {
    cleanup();
    return 1;
  }
  // sizes, raw fallback (src/compile.cpp:268-275), offsets
  std::vector<uint64_t> bbytes(nb);
  uint64_t total = 0;
  std::vector<uint64_t> sizes(ns);
  for (size_t i = 0; i < ns; ++i) {
    PackSlab& s = slabs[i];
    uint64_t size = s.kind == XKSV_CODEC_PARALLEL32 ? 32 + 8 * uint64_t(s.chunks) : 0;
    for (uint32_t k = 0; k < s.chunks; ++k) {
      const size_t b = s.first_block + k;
      if (bits[b] == ~0ull) {  // code longer than 32 bits: not produced by this encoder
        cleanup();
        return 1;
      }
      bbytes[b] = 272 + blocks[b].count + bits[b] / 8 + (bits[b] % 8 != 0);
      size += bbytes[b];
    }
    if (size >= s.raw_bytes) {
      s.kind = XKSV_CODEC_RAW;
      size = s.raw_bytes;
    }
    s.out_off = total;
    uint64_t pos = s.kind == XKSV_CODEC_PARALLEL32 ? total + 32 + 8 * uint64_t(s.chunks) : total;
    for (uint32_t k = 0; k < s.chunks; ++k) {
      blocks[s.first_block + k].out_off = pos;
      pos += bbytes[s.first_block + k];
    }
    sizes[i] = size;
    total += size;
  }
  for (size_t i = 0; i < ns; ++i)  // blocks of raw slabs are not written
    if (slabs[i].kind == XKSV_CODEC_RAW)
      for (uint32_t k = 0; k < slabs[i].chunks; ++k) blocks[slabs[i].first_block + k].out_off = ~0ull;
  ok = cudaMalloc(&d_out, total + 16) == cudaSuccess && cudaMemsetAsync(d_out, 0, total + 16, st) == cudaSuccess &&
       cudaMalloc(&d_slabs, ns * sizeof(PackSlab)) == cudaSuccess &&
       cudaMemcpyAsync(d_slabs, slabs.data(), ns * sizeof(PackSlab), cudaMemcpyHostToDevice, st) == cudaSuccess &&
       cudaMemcpyAsync(d_bbytes, bbytes.data(), nb * 8, cudaMemcpyHostToDevice, st) == cudaSuccess &&
       cudaMemcpyAsync(d_blocks, blocks.data(), nb * sizeof(PackBlock), cudaMemcpyHostToDevice, st) == cudaSuccess;
  if (ok) {
    pack_body_kernel<<<unsigned(nb), 256, 0, st>>>(d_blocks, d, d_lens, d_bits, d_out);
    pack_slab_kernel<<<unsigned(ns), 256, 0, st>>>(d_slabs, d_blocks, d_bbytes,
                                                    static_cast<const uint8_t*>(d_data), d_out);
    // after the bodies: the stream words may share bytes with the sign/mantissa section
    pack_bits_kernel<<<unsigned(nb), 256, 0, st>>>(d_blocks, d, d_lens, d_codes, d_out);
    ok = cudaGetLastError() == cudaSuccess;
  }
  ok = ok && cudaStreamSynchronize(st) == cudaSuccess;
  cleanup();
  auto* tab = ok ? static_cast<xksv_slab*>(std::malloc(sizeof(xksv_slab) * (ns ? ns : 1))) : nullptr;
  if (!tab) {
    cudaFree(d_out);
    return 1;
  }
  for (size_t i = 0; i < ns; ++i) {
    tab[i].src_offset = slabs[i].out_off;
    tab[i].src_size = sizes[i];
    tab[i].rows = slabs[i].rows;
    tab[i].cols = slabs[i].cols;
    tab[i].dst_offset = dst_base + slabs[i].data_off * 2;
    tab[i].x_offset = 0;
    tab[i].codec = slabs[i].kind;
    tab[i].flags = 0;
  }
  *d_payload = d_out;
  *payload_size = total;
  *table = tab;
  *nslabs = ns;
  return 0;
}

void xksv_cuda_free(void* d) {
  if (d) cudaFree(d);
}

}  // extern "C"
