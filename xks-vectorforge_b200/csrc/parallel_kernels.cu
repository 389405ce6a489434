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
// A slab's setup takes two memory round trips: the container header together
// with each lane's substream-table entry, then each lane's substream header
// together with its 256 code lengths (cp.async copies into the lane's own
// table memory, idle until the tables are filled) and its first sign/mantissa
// chunks.  A warp that goes on to another slab (grids smaller than the slab
// count) prefetches that slab's headers and length tables into L2 meanwhile.
#include <atomic>

#include "kernels.h"
#include "lane_decode.cuh"
#include "xksv_device.cuh"

namespace xksv {
namespace {

using PCfg = ldec::Cfg<6, 5, 2, 16, 16>;  // first level 6 bits, second 7-11 bits, 16 long codes to 22 bits
using ldec::BR;
using ldec::SMR;
constexpr int kSaveChunk = 4;  // first ring row holding length chunks saved by the table build
constexpr int PWARPS = 2;      // slabs (warps) per CTA: small CTAs free their tables sooner
constexpr int PMAXB = 8;       // GEMM columns per pass

// One warp's tables and rings, lane-minor so that lane l always touches bank
// l/2 (16-bit tables) or bank l (the bit ring).
struct WarpTabs {
  ldec::Tables<PCfg> t;
  union {
    uint8_t lpos[PCfg::PNL][32];  // fill cursor per long length (table build only)
    uint32_t ring[BR][32];        // exponent bits, big-endian words, word w at [w % BR]
  };
  uint4 smring[SMR][32];          // staged sign/mantissa chunks
};
static_assert(sizeof(WarpTabs) % 16 == 0, "warp tables keep 16-byte alignment");
static_assert(kSaveChunk * 128 >= PCfg::PNL * 32, "saved length chunks do not overlap lpos");
static_assert(kSaveChunk + 12 <= BR, "three saved chunks fit the ring");
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
static_assert(sizeof(GenericTab) <= sizeof(ldec::Tables<PCfg>::lut), "generic table fits");

struct Seg {
  const uint8_t* lens;
  const uint8_t* sm;
  const uint8_t* bits;
  uint32_t count;
  uint32_t start;  // packed index of the substream's first element
  uint64_t nbits;
  uint64_t ebytes;
};

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
__device__ void decode_segment(const Seg& s, WarpTabs& W, int lane, const ldec::Code& lc, bool rows16,
                               ldec::Stream& b, ldec::SmStream& smr, const Out& o, bool& bad) {
  uint32_t i = 0;
  if (rows16) {
    const uint32_t ng = s.count >> 4;
    uint32_t p = s.start;
    for (uint32_t g = 0; g < ng; ++g, p += 16) {
      smr.stage(W.smring, lane);
      cp_async_commit();
      b.maintain(W.ring, lane);
      ldec::cp_async_wait_2();  // this group's two chunks were committed two groups ago
      const uint4 s16 = smr.take(W.smring, lane);
      uint32_t e[16];
#pragma unroll
      for (int k = 0; k < 4; ++k)
        ldec::dec4<PCfg>(b, W.ring, W.t, lane, lc, bad, e[4 * k], e[4 * k + 1], e[4 * k + 2], e[4 * k + 3]);
      const uint32_t r = (p >> 4) & 15, c = (p >> 8) * 16;
      if (MODE == 0) {
        uint4 v0, v1;
        ldec::merge16(e, s16, v0, v1);
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
    const uint32_t e = ldec::dec_one<PCfg>(b, W.ring, W.t, lane, lc, bad);
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
    // ---- container header (cuda/parallel.cu:34-36) and, in the same round
    // trip, this lane's substream-table entry (read when it lies inside the
    // slab; the header checks below decide whether it is one) ----
    bool ok = n >= 32;
    uint64_t rows = 0, cols = 0, chunks = 0, entry = 0;
    if (ok) {
      // header fields through aligned 8-byte loads (the slab may sit at any
      // byte offset; n >= 32 keeps every read inside the slab's words)
      const uint8_t* pe = p + n;
      const uint64_t magic = ld8_any(p, pe);
      rows = ld8_any(p + 8, pe);
      cols = ld8_any(p + 16, pe);
      chunks = ld8_any(p + 24, pe);
      if (40 + 8 * uint64_t(lane) <= n) entry = ld8_any(p + 32 + 8 * lane, pe);
      ok = magic == 0x0000003250534B58ull &&  // "XKSP2\0\0\0"
           rows && rows <= 16 && cols && chunks && chunks <= 32 &&
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
    const uint64_t len = active ? entry : 0;  // n >= 32 + 8 * chunks: every active entry was read
    bool lok = !active || (len >= kHdr && len <= n);
    const uint64_t incl = warp_incl_scan(lok ? len : 0, lane);
    const uint64_t base = 32 + 8 * chunks + incl - len;
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
    Seg s{};
    s.start = uint32_t(uint64_t(total) * uint64_t(lane) / chunks);
    const uint64_t expect = uint64_t(total) * uint64_t(lane + 1) / chunks - s.start;
    const bool rows16 = nice && (s.start & 15) == 0;
    ldec::Stream b;
    ldec::SmStream smr;
    if (active && lok) {
      lok = base + len <= n;
      if (lok) {
        const uint8_t* q = p + base;
        // one round trip for the substream's header, its code lengths (into
        // the warp's table memory, idle until the fill pass) and its first
        // sign/mantissa chunks (the substream holds `expect` of them when
        // the slab is well formed; the copies stay inside the slab anyway)
        ldec::stage_lengths<PCfg>(W.t, q + 16, lane);
        if (rows16) {
          const uint8_t* sm = q + kHdr;
          const uint8_t* sme = sm + expect <= p + n ? sm + expect : p + n;
          smr.init(W.smring, lane, sm, sme > sm ? sme : sm + 1);
        }
        const uint64_t count = ld8_any(q, p + n);
        s.nbits = ld8_any(q + 8, p + n);
        s.ebytes = s.nbits / 8 + (s.nbits % 8 != 0);
        lok = count == expect && count <= len - kHdr && s.ebytes == len - kHdr - count;
        s.count = uint32_t(count);
        s.lens = q + 16;
        s.sm = q + kHdr;
        s.bits = q + kHdr + count;
      }
    }
    cp_async_commit();
    const uint64_t end_all = __shfl_sync(0xffffffffu, base + len, int(chunks - 1));
    if (!(__all_sync(0xffffffffu, lok) && end_all == n)) {
      cp_async_wait_all();
      __syncwarp();
      if (lane == 0) atomicOr(status, kStatusHeader);
      continue;
    }
    // bit positions are 32-bit (the slab format bounds them far lower: a
    // substream's bits fit in its slab, and compiled slabs are <= 1 MiB)
    if (__any_sync(0xffffffffu, s.nbits >= (1ull << 32) - 256)) {
      cp_async_wait_all();
      __syncwarp();
      if (lane == 0) atomicOr(status, kStatusInternal);
      continue;
    }
    // ---- first bit loads, overlapping the table build ----
    if (active) b.start(s.bits, s.ebytes);
    // ---- per-lane tables, from the staged lengths ----
    cp_async_wait_all();
    ldec::Code lc{0, 0, 0};
    uint32_t L = 0;
    int tb = 0;
    if (active) {
      ldec::TabLens<PCfg> lens(W.t, s.lens, &W.ring[kSaveChunk], lane);
      tb = ldec::build_tables<PCfg>(lens, W.t, W.lpos, lane, lc.F, lc.maxlen, L);
    }
    lc.L2 = L << PCfg::K2;
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
      b.init_ring(W.ring, lane);
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
      if (lane == 0 && !decode_segment_generic<MODE>(sg, *reinterpret_cast<GenericTab*>(&W.t.lut[0][0]), o))
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
