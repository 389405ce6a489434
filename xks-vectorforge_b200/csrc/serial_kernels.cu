// "bf16-huffman-tile16" (serial codec) slabs: decode and fused GEMV/GEMM.
//
// Reference behaviour: cuda/decode.cu:12-45 (one thread walks the whole slab
// bit stream; errors at :20, :22, :26), host checks cuda/decode.cu:47-66, CPU
// semantics src/codec.cpp:59-74 and src/c_api.cpp:29-40.
//
// B200 design: a slab has ONE Huffman bit stream and no substream offsets, so
// one CTA decodes it cooperatively by self-synchronising speculative decoding
// (after Weissenberger & Schmidt, "Massively Parallel Huffman Decoding on
// GPUs", ICPP 2018).  The stream is processed in rounds of ST*S bits held in
// shared memory:
//   1. every thread decodes its own S-bit range from the range's first bit
//      (thread 0 from the exact round start), marking each code start in a
//      bitmap and counting codes;
//   2. thread t re-decodes from the true end of thread t-1's last code until it
//      lands on a position it marked itself: from there its first pass was on
//      the true code sequence, so its count is corrected by the marks it
//      skipped (a popcount); repeated until no end position changes (each
//      repetition makes at least one more thread exact, so the loop is
//      bounded; Huffman codes resynchronise within a few codes in practice);
//   3. a block scan of the corrected counts gives each thread's output index,
//      and the threads decode their exact ranges again into a shared staging
//      buffer of exponent bytes;
//   4. the staged exponents are merged with the sign/mantissa bytes and
//      written un-tiled with 16-byte stores (or fed to the GEMV/GEMM).
// Decode tables: a 2^SK-entry table for codes of length <= SK, canonical
// limits for lengths up to 32, and a bit-serial decoder beyond that (the
// format allows lengths up to 255).
#include "kernels.h"
#include "xksv_device.cuh"

namespace xksv {
namespace {

constexpr int SK = 11;         // first-level table bits
constexpr int ST = 256;        // threads per CTA
constexpr int SCAP = 16384;    // staged symbols per round (=> S = 64 * min length)
constexpr int SMAXS = 256;     // max bits per thread per round
constexpr int PADW = 12;       // window words past the round end (255-bit code + read-ahead)
constexpr int WINW = ST * SMAXS / 32 + PADW;
constexpr int SMAXB = 8;       // GEMM columns per pass
constexpr uint32_t kDead = 0xFFFFFFFFu;

struct SerialShared {
  uint16_t lut[1 << SK];
  uint64_t lim[33];      // left-aligned limit of codes with length <= l (l <= 32)
  uint64_t firstc[33];   // canonical first code of length l (l <= 32)
  alignas(16) uint16_t cnt[256];  // codes per length
  uint16_t offs[257];    // index in sorted[] of the first code of length l
  uint8_t sorted[256];   // symbols in canonical (length, symbol) order
  uint32_t win[WINW];    // the round's bits, big-endian words
  uint32_t marks[ST * SMAXS / 32];
  uint32_t endpos[ST];   // relative end of each thread's last code (or kDead)
  uint32_t warpsum[ST / 32];
  float y[16 * SMAXB];
  int maxlen, minlen, flag;
  uint32_t total;
  alignas(16) uint8_t stage[SCAP + 16];
  uint8_t hist[ST / 32][256];  // rank scratch at table build
};

__device__ __forceinline__ uint32_t win32(const SerialShared& S, uint32_t pos) {
  uint32_t i = pos >> 5;
  return __funnelshift_l(S.win[i + 1], S.win[i], pos & 31);
}

// Codes longer than SK bits.  Returns (symbol << 7 | 0) with *len set, or -1.
__device__ int slow_decode(const SerialShared& S, uint32_t w, uint32_t pos, int* len) {
  int top = S.maxlen < 32 ? S.maxlen : 32;
  for (int l = SK + 1; l <= top; ++l) {
    if (uint64_t(w) < S.lim[l]) {
      uint64_t v = uint64_t(w) >> (32 - l);
      *len = l;
      return S.sorted[S.offs[l] + uint32_t(v - S.firstc[l])];
    }
  }
  if (S.maxlen <= 32) return -1;
  auto bit_at = [&](int k) -> uint32_t {
    uint32_t q = pos + uint32_t(k);
    return (S.win[q >> 5] >> (31 - (q & 31))) & 1u;
  };
  return generic_decode(bit_at, S.cnt, S.sorted, S.maxlen, len);
}

// Decodes the code at relative bit `pos`; returns symbol and length, or -1.
__device__ __forceinline__ int decode_at(const SerialShared& S, uint32_t pos, int* len) {
  uint32_t w = win32(S, pos);
  uint32_t e = S.lut[w >> (32 - SK)];
  if (e & 31u) {
    *len = int(e & 31u);
    return int(e >> 7);
  }
  return slow_decode(S, w, pos, len);
}

__device__ __forceinline__ bool marked(const SerialShared& S, uint32_t pos) {
  return (S.marks[pos >> 5] >> (pos & 31)) & 1u;
}

// Marks in [from, to) (both inside one thread's range).
__device__ __forceinline__ uint32_t count_marks(const SerialShared& S, uint32_t from, uint32_t to) {
  uint32_t n = 0;
  uint32_t w0 = from >> 5, w1 = to >> 5;
  for (uint32_t w = w0; w <= w1 && w < ST * SMAXS / 32; ++w) {
    uint32_t m = S.marks[w];
    if (w == w0) m &= ~0u << (from & 31);
    if (w == w1) m &= (to & 31) ? (~0u >> (32 - (to & 31))) : 0u;
    n += __popc(m);
  }
  return n;
}

// Builds canonical tables for the slab's code lengths.  Returns false for an
// oversubscribed codebook.
__device__ bool build_tables(SerialShared& S, const uint8_t* lens) {
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  S.cnt[t] = 0;
  if (t == 0) {
    S.maxlen = 0;
    S.minlen = 256;
  }
  uint8_t* hist = &S.hist[0][0];
  for (int k = t; k < (ST / 32) * 256; k += ST) hist[k] = 0;
  __syncthreads();
  const int l = __ldg(lens + t);
  // per-length counts (16-bit fields) via 32-bit atomics on the containing word
  if (l) {
    uint32_t* w = reinterpret_cast<uint32_t*>(&S.cnt[l & ~1]);
    atomicAdd(w, (l & 1) ? 0x10000u : 1u);
    atomicMax(&S.maxlen, l);
    atomicMin(&S.minlen, l);
  }
  // rank of symbol t among earlier symbols with the same length
  const uint32_t same = __match_any_sync(0xffffffffu, l);
  const uint32_t rank_w = __popc(same & ((1u << lane) - 1));
  if (l && rank_w == 0) S.hist[warp][l] = uint8_t(__popc(same));
  __syncthreads();
  // offs[] = exclusive scan of cnt[] (one length per thread)
  const uint32_t c = S.cnt[t];
  uint32_t v = c;
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    uint32_t u = __shfl_up_sync(0xffffffffu, v, d);
    if (lane >= d) v += u;
  }
  if (lane == 31) S.warpsum[warp] = v;
  __syncthreads();
  uint32_t pre = 0;
  for (int w = 0; w < warp; ++w) pre += S.warpsum[w];
  S.offs[t] = uint16_t(pre + v - c);
  if (t == ST - 1) S.offs[256] = uint16_t(pre + v);
  if (t == 0) {
    int64_t avail = 1;
    bool ok = true;
    for (int k = 1; k <= S.maxlen; ++k) {
      avail = 2 * avail - S.cnt[k];
      if (avail < 0) ok = false;
      if (avail > 4096) avail = 4096;
    }
    uint64_t code = 0;
    for (int k = 1; k <= 32; ++k) {
      uint64_t ck = S.cnt[k];
      S.firstc[k] = code;
      S.lim[k] = (code + ck) << (32 - k);
      code = (code + ck) << 1;
    }
    S.lim[0] = 0;
    S.firstc[0] = 0;
    S.flag = ok ? 0 : 1;
  }
  __syncthreads();
  if (S.flag) return false;
  if (l) {
    uint32_t r = rank_w;
    for (int w = 0; w < warp; ++w) r += S.hist[w][l];
    S.sorted[S.offs[l] + r] = uint8_t(t);
  }
  __syncthreads();
  // first-level table: thread t fills entries [PER*t, PER*t + PER)
  constexpr int PER = (1 << SK) / ST;
  int len = S.minlen;
  for (int k = 0; k < PER; ++k) {
    uint32_t e = uint32_t(t * PER + k);
    uint64_t W = uint64_t(e) << (32 - SK);
    while (len <= SK && W >= S.lim[len]) ++len;
    uint16_t val = 0;
    if (len <= SK) {
      uint32_t code = e >> (SK - len);
      val = uint16_t((uint32_t(S.sorted[S.offs[len] + code - uint32_t(S.firstc[len])]) << 7) |
                     uint32_t(len));
    }
    S.lut[e] = val;
  }
  __syncthreads();
  return true;
}

struct SerialArgs {
  const uint8_t* payload;
  uint8_t* out;
  const float* x;
  float* y;
  uint32_t ld, nb;
  int* status;
};

template <int MODE>
__global__ void __launch_bounds__(ST) serial_slab_kernel(const Slab* __restrict__ slabs,
                                                         uint32_t nslabs, SerialArgs a) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  SerialShared& S = *reinterpret_cast<SerialShared*>(smem_raw);
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;

  for (uint32_t si = blockIdx.x; si < nslabs; si += gridDim.x) {
    const Slab sd = slabs[si];
    const uint8_t* p = a.payload + sd.src;
    const uint64_t size = sd.size, rows = sd.rows, cols = sd.cols;
    // ---- header (cuda/decode.cu:49-51) ----
    bool ok = size >= kHdr && rows && cols && cols <= ~0ull / rows;
    uint64_t count = 0, nbits = 0;
    if (ok) {
      count = ld_le64(p);
      nbits = ld_le64(p + 8);
      ok = count == rows * cols && count <= size - kHdr &&
           nbits / 8 + (nbits % 8 != 0) == size - kHdr - count && count < (1ull << 40);
    }
    if (!ok) {
      if (t == 0) atomicOr(a.status, kStatusHeader);
      continue;
    }
    if (!build_tables(S, p + 16)) {
      if (t == 0) atomicOr(a.status, kStatusCodebook);
      __syncthreads();
      continue;
    }
    const uint8_t* sm = p + kHdr;
    const uint8_t* bits = p + kHdr + count;
    const uint8_t* end = p + size;
    uint16_t* o16 = reinterpret_cast<uint16_t*>(a.out + sd.dst);
    const float* xs = MODE == 1 ? a.x + sd.xoff * a.ld : nullptr;
    bool nice;
    if (MODE == 0)
      nice = rows == 16 && (cols & 15) == 0 && (reinterpret_cast<uintptr_t>(o16) & 15) == 0;
    else
      nice = rows == 16 && (cols & 15) == 0;
    if (MODE == 1) {
      for (int k = t; k < 16 * SMAXB; k += ST) S.y[k] = 0.f;
      if (!nice)
        for (uint64_t k = t; k < rows * a.nb; k += ST) {
          uint64_t r = k / a.nb, b = k - r * a.nb;
          a.y[(sd.dst + r) * a.ld + b] = 0.f;
        }
      __syncthreads();
    }
    // bits per thread per round: at most SCAP codes start in a round
    const uint32_t S_bits = uint32_t(min(SMAXS, 32 * max(1, (SCAP / ST) * S.minlen / 32)));
    const uint32_t round_bits = ST * S_bits;
    uint64_t R0 = 0, p0 = 0, base = 0;
    int err = 0;
    while (R0 < nbits) {
      // ---- 1. window ----
      const uint32_t nw = round_bits / 32 + PADW;
      for (uint32_t j = t; j < nw; j += ST) {
        const uint8_t* q = bits + (R0 >> 3) + 4 * uint64_t(j);
        uint32_t v = 0;
        if (q < end) {
          uintptr_t qa = reinterpret_cast<uintptr_t>(q);
          const uint32_t* qw = reinterpret_cast<const uint32_t*>(qa & ~uintptr_t(3));
          int sh = int(qa & 3) * 8;
          uint32_t lo = __ldg(qw);
          uint32_t hi = (sh && reinterpret_cast<const uint8_t*>(qw + 1) < end) ? __ldg(qw + 1) : 0u;
          v = bswap32(sh ? __funnelshift_r(lo, hi, sh) : lo);
        }
        S.win[j] = v;
      }
      const uint32_t lim_rel = uint32_t(nbits - R0 < round_bits ? nbits - R0 : round_bits);
      const uint32_t my_lo = uint32_t(t) * S_bits;
      const uint32_t my_hi = min(my_lo + S_bits, lim_rel);
      for (uint32_t w = my_lo / 32; w < (my_lo + S_bits) / 32; ++w) S.marks[w] = 0;
      __syncthreads();
      // ---- 2. speculative pass ----
      const uint32_t p0rel = uint32_t(p0 - R0);
      uint32_t st0 = t == 0 ? p0rel : my_lo;
      uint32_t e1 = st0, n1 = 0;
      bool d1 = false;
      {
        uint32_t pos = st0, mw = pos >> 5, m = 0;
        while (pos < my_hi) {
          int len;
          int sym = decode_at(S, pos, &len);
          if (sym < 0) {
            d1 = true;
            break;
          }
          if ((pos >> 5) != mw) {
            S.marks[mw] = m;
            mw = pos >> 5;
            m = 0;
          }
          m |= 1u << (pos & 31);
          ++n1;
          pos += uint32_t(len);
        }
        if (pos > st0 || d1) S.marks[mw] |= m;
        e1 = pos;
      }
      __syncthreads();
      // ---- 3. resynchronisation ----
      uint32_t myE = d1 ? kDead : e1, myN = n1, last_start = st0;
      bool myD = d1;
      S.endpos[t] = myE;
      for (int iter = 0; iter <= ST; ++iter) {
        __syncthreads();
        uint32_t A = t == 0 ? p0rel : S.endpos[t - 1];
        bool redo = t > 0 && A != last_start;
        __syncthreads();
        if (redo) {
          last_start = A;
          if (A == kDead) {
            myD = true;
            myE = kDead;
            myN = 0;
          } else if (A >= my_hi) {
            myD = false;
            myE = A;
            myN = 0;
          } else if (A < my_lo) {
            myD = true;
            myE = kDead;
            myN = 0;
          } else {
            uint32_t pos = A, k = 0;
            bool synced = false, dead = false;
            while (pos < my_hi) {
              if (marked(S, pos)) {
                synced = true;
                break;
              }
              int len;
              if (decode_at(S, pos, &len) < 0) {
                dead = true;
                break;
              }
              pos += uint32_t(len);
              ++k;
            }
            if (synced) {
              myN = k + n1 - count_marks(S, my_lo, pos);
              myE = d1 ? kDead : e1;
              myD = d1;
            } else {
              myN = k;
              myE = dead ? kDead : pos;
              myD = dead;
            }
          }
          S.endpos[t] = myE;
        }
        if (!__syncthreads_or(redo)) break;
      }
      // ---- 4. scan ----
      uint32_t v = myN;
#pragma unroll
      for (int d = 1; d < 32; d <<= 1) {
        uint32_t u = __shfl_up_sync(0xffffffffu, v, d);
        if (lane >= d) v += u;
      }
      if (lane == 31) S.warpsum[warp] = v;
      const int any_dead = __syncthreads_or(myD);
      uint32_t wpre = 0, tot = 0;
      for (int w = 0; w < ST / 32; ++w) {
        uint32_t ws = S.warpsum[w];
        if (w < warp) wpre += ws;
        tot += ws;
      }
      const uint32_t my_off = wpre + v - myN;
      const uint32_t last_end = S.endpos[ST - 1];
      if (any_dead || base + tot > count) {
        err = kStatusStream;
        break;
      }
      // ---- 5. exact decode into the staging buffer ----
      const uint32_t a0 = uint32_t(base & 7);
      {
        uint32_t pos = t == 0 ? p0rel : S.endpos[t - 1];
        uint8_t* dst = S.stage + a0 + my_off;
        for (uint32_t k = 0; k < myN; ++k) {
          int len;
          int sym = decode_at(S, pos, &len);
          dst[k] = uint8_t(sym);
          pos += uint32_t(len);
        }
      }
      __syncthreads();
      // ---- 6. write out ----
      const uint64_t g0 = base & ~7ull;
      const uint64_t fin = base + tot;
      const uint32_t ngroups = uint32_t((fin - g0 + 7) >> 3);
      for (uint32_t g = t; g < ngroups; g += ST) {
        const uint64_t q = g0 + 8ull * g;
        const bool full = q >= base && q + 8 <= fin;
        if (nice && full) {
          uint64_t e8 = *reinterpret_cast<const uint64_t*>(S.stage + (q - g0));
          uint64_t s8 = ld8_any(sm + q, end);
          const uint32_t elo = uint32_t(e8), ehi = uint32_t(e8 >> 32);
          const uint32_t slo = uint32_t(s8), shi = uint32_t(s8 >> 32);
          const uint64_t tt = q >> 8, r = (q >> 4) & 15, c = tt * 16 + (q & 15);
          uint4 o;
          o.x = (__byte_perm(elo, 0, 0x4140) << 7) | (__byte_perm(slo, 0, 0x1100) & 0x807F807Fu);
          o.y = (__byte_perm(elo, 0, 0x4342) << 7) | (__byte_perm(slo, 0, 0x3322) & 0x807F807Fu);
          o.z = (__byte_perm(ehi, 0, 0x4140) << 7) | (__byte_perm(shi, 0, 0x1100) & 0x807F807Fu);
          o.w = (__byte_perm(ehi, 0, 0x4342) << 7) | (__byte_perm(shi, 0, 0x3322) & 0x807F807Fu);
          if (MODE == 0) {
            *reinterpret_cast<uint4*>(o16 + r * cols + c) = o;
          } else {
            uint32_t wv[4] = {o.x, o.y, o.z, o.w};
            for (uint32_t b = 0; b < a.nb; ++b) {
              float acc = 0.f;
#pragma unroll
              for (int k = 0; k < 8; ++k) {
                uint32_t word = (wv[k >> 1] >> (16 * (k & 1))) & 0xFFFFu;
                acc = fmaf(__uint_as_float(word << 16), __ldg(&xs[(c + k) * a.ld + b]), acc);
              }
              atomicAdd(&S.y[r * SMAXB + b], acc);
            }
          }
        } else {
          const uint64_t lo = q > base ? q : base, hi = q + 8 < fin ? q + 8 : fin;
          for (uint64_t e = lo; e < hi; ++e) {
            uint32_t word = merge1(uint32_t(S.stage[e - g0]) << 7, __ldg(sm + e));
            uint64_t o = untile_index(e, rows, cols);
            if (MODE == 0) {
              o16[o] = uint16_t(word);
            } else {
              uint64_t r = o / cols, c = o - r * cols;
              float wf = __uint_as_float(word << 16);
              for (uint32_t b = 0; b < a.nb; ++b) {
                float pv = wf * __ldg(&xs[c * a.ld + b]);
                if (nice)
                  atomicAdd(&S.y[r * SMAXB + b], pv);
                else
                  atomicAdd(&a.y[(sd.dst + r) * a.ld + b], pv);
              }
            }
          }
        }
      }
      base += tot;
      p0 = R0 + last_end;
      R0 += round_bits;
      __syncthreads();
    }
    if (!err && (base != count || p0 != nbits)) err = kStatusStream;
    if (err) {
      if (t == 0) atomicOr(a.status, err);
    } else if (MODE == 1 && nice) {
      for (uint32_t k = t; k < 16 * a.nb; k += ST) {
        uint32_t r = k / a.nb, b = k - r * a.nb;
        a.y[(sd.dst + r) * a.ld + b] = S.y[r * SMAXB + b];
      }
    }
    __syncthreads();
  }
}

}  // namespace

size_t serial_smem_bytes() { return sizeof(SerialShared); }

static void serial_set_attr() {
  static int done_mask = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 31 && (done_mask >> dev) & 1) return;
  cudaFuncSetAttribute(serial_slab_kernel<0>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(sizeof(SerialShared)));
  cudaFuncSetAttribute(serial_slab_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(sizeof(SerialShared)));
  if (dev < 31) done_mask |= 1 << dev;
}

cudaError_t launch_serial_decode(const Slab* slabs, uint32_t n, const uint8_t* payload,
                                 uint8_t* out, int* status, int grid, cudaStream_t st) {
  if (!n) return cudaSuccess;
  serial_set_attr();
  SerialArgs a{payload, out, nullptr, nullptr, 1, 1, status};
  int g = grid < int(n) ? grid : int(n);
  serial_slab_kernel<0><<<g, ST, sizeof(SerialShared), st>>>(slabs, n, a);
  return cudaGetLastError();
}

cudaError_t launch_serial_gemm(const Slab* slabs, uint32_t n, const uint8_t* payload,
                               const float* x, float* y, uint32_t ld, uint32_t b0, uint32_t nb,
                               int* status, int grid, cudaStream_t st) {
  if (!n) return cudaSuccess;
  serial_set_attr();
  SerialArgs a{payload, nullptr, x + b0, y + b0, ld, nb, status};
  int g = grid < int(n) ? grid : int(n);
  serial_slab_kernel<1><<<g, ST, sizeof(SerialShared), st>>>(slabs, n, a);
  return cudaGetLastError();
}

}  // namespace xksv
