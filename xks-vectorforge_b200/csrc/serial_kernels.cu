// "bf16-huffman-tile16" (serial codec) slabs: decode and fused GEMV/GEMM.
//
// Reference behaviour: cuda/decode.cu:12-45 (one thread walks the whole slab
// bit stream; errors at :20, :22, :26), host checks cuda/decode.cu:47-66, CPU
// semantics src/codec.cpp:59-74 and src/c_api.cpp:29-40.
//
// B200 design: a slab has ONE Huffman bit stream and no substream offsets, so
// one CTA decodes it cooperatively by self-synchronising speculative decoding
// (after Weissenberger & Schmidt, "Massively Parallel Huffman Decoding on
// GPUs", ICPP 2018).  The stream is cut into rounds of ST*S bits (S chosen per
// slab so rounds are balanced), each held in shared memory:
//   1. count pass: every thread walks its own S-bit range from the range's
//      first bit (thread 0 from the exact round start) with a count table that
//      consumes every whole code inside the next CK bits at once, and records
//      where its first REC lookups start and how many codes preceded each;
//   2. thread t re-decodes code by code from the true end of thread t-1's walk
//      until it lands on one of its recorded lookup starts: from there its walk
//      followed the true code sequence, so its count only loses the codes
//      before that point.  Repeated until no end position changes: each
//      repetition makes at least one more thread exact (bounded by ST); in
//      practice codes resynchronise within a few codes and one suffices;
//   3. a block scan of the counts gives every thread its output index; each
//      thread decodes its exact range code by code (four codes per branch-free
//      block), merges exponents with the sign/mantissa bytes and writes 8 BF16
//      words (half a tile row) per 16-byte store, un-tiled on the fly (or feeds
//      the GEMV/GEMM).
// Bits reach the threads through a 96-bit register window over the round's
// shared copy, refilled once per four codes.  Tables: 2^SK-entry single-code
// table, 2^CK-entry count table, canonical limits up to 32 bits and a
// bit-serial decoder beyond (the format allows lengths up to 255).
#include <atomic>

#include "kernels.h"
#include "tcgen05.cuh"
#include "xksv_device.cuh"

namespace xksv {
namespace {

constexpr int SK = 11;         // single-code table bits
constexpr int CK = 10;         // count table bits
constexpr int ST = 256;        // threads per CTA
constexpr int SMAXS = 1024;    // max bits per thread per round
constexpr int PADW = 16;       // window words past the round end (255-bit code + window)
constexpr int WINW = ST * SMAXS / 32 + PADW;
constexpr int REC = 16;        // lookup starts recorded per thread in the count pass
constexpr int SMAXB = 8;       // GEMM columns per pass
constexpr uint32_t kDead = 0xFFFFFFFFu;

struct SerialShared {
  uint16_t lut[1 << SK];  // exponent << 7 | length for codes <= SK bits; 0 = none
  uint8_t clut[1 << CK];  // n << 4 | total length of the n whole codes in CK bits; 0 = none
  uint64_t lim[33];       // left-aligned limit of codes with length <= l (l <= 32)
  uint64_t firstc[33];    // canonical first code of length l (l <= 32)
  alignas(16) uint16_t cnt[256];  // codes per length
  uint16_t offs[257];     // index in sorted[] of the first code of length l
  uint8_t sorted[256];    // symbols in canonical (length, symbol) order
  alignas(16) uint32_t win[WINW + 16];  // the round's bits, big-endian words (+ room for the raw copy's offset)
  union {
    struct {
      uint16_t pos[REC][ST];  // lookup start, relative to the thread's range start
      uint16_t cnt[REC][ST];  // codes counted before that lookup
    } rec;
    uint8_t hist[8][256];  // rank scratch while building tables
  };
  uint32_t endpos[ST];  // relative end of each thread's walk (or kDead)
  uint32_t warpsum[ST / 32];
  float y[16 * SMAXB];
  int maxlen, minlen, flag;
};

template <class SH>
__device__ __forceinline__ uint32_t win32(const SH& S, uint32_t pos) {
  const uint32_t i = pos >> 5;
  return __funnelshift_l(S.win[i + 1], S.win[i], pos & 31);
}

// Codes longer than SK bits at relative bit `pos`.  Returns the symbol with
// *len set, or -1.
template <class SH>
__device__ __noinline__ int slow_decode(const SH& S, uint32_t pos, int* len) {
  const uint32_t w = win32(S, pos);
  const int top = S.maxlen < 32 ? S.maxlen : 32;
  for (int l = SK + 1; l <= top; ++l) {
    if (uint64_t(w) < S.lim[l]) {
      const uint64_t v = uint64_t(w) >> (32 - l);
      *len = l;
      return S.sorted[S.offs[l] + uint32_t(v - S.firstc[l])];
    }
  }
  if (S.maxlen <= 32) return -1;
  auto bit_at = [&](int k) -> uint32_t {
    const uint32_t q = pos + uint32_t(k);
    return (S.win[q >> 5] >> (31 - (q & 31))) & 1u;
  };
  return generic_decode(bit_at, S.cnt, S.sorted, S.maxlen, len);
}

// One code at the window head (>= SK valid bits).  Table entries hold the
// exponent at bit XS and the code length in bits 0-4; the result holds the
// exponent at bit XS.  A code longer than SK bits re-positions the window
// after it.
template <int XS, class SH>
__device__ __forceinline__ uint32_t code1(const SH& S, SmemWin96& r, bool& dead) {
  const uint32_t e = S.lut[r.w0 >> (32 - SK)];
  if (e) {
    r.skip(e);
    return e;
  }
  const uint32_t pos = r.pos();
  int l = 1;
  int sym = slow_decode(S, pos, &l);
  if (sym < 0) {
    dead = true;
    sym = 0;
    l = 1;
  }
  r.init(S.win, pos + uint32_t(l));
  return uint32_t(sym) << XS;
}

// Four codes from a window holding >= 4*SK bits, without a branch in the
// common case.  A code the table does not hold has entry 0, which skips no
// bits, so every later lookup of the block sees the same code and is 0 too:
// the window stops at the first such code, and e3 == 0 tells that one did.
// Those codes are then decoded one by one from where the window stopped.
template <int XS, class SH>
__device__ __forceinline__ void code4(const SH& S, SmemWin96& r, bool& dead, uint32_t& e0,
                                      uint32_t& e1, uint32_t& e2, uint32_t& e3) {
  e0 = S.lut[r.w0 >> (32 - SK)];
  r.shift(e0);
  e1 = S.lut[r.w0 >> (32 - SK)];
  r.shift(e1);
  e2 = S.lut[r.w0 >> (32 - SK)];
  r.shift(e2);
  e3 = S.lut[r.w0 >> (32 - SK)];
  r.shift(e3);
  // lengths sit in bits 0-4 above zero bits, so one sum carries all four
  r.nb -= int((e0 + e1 + e2 + e3) & 127u);
  if (e3 == 0) {
    if (e0 == 0) {
      e0 = code1<XS>(S, r, dead);
      r.refill();
    }
    if (e1 == 0) {
      e1 = code1<XS>(S, r, dead);
      r.refill();
    }
    if (e2 == 0) {
      e2 = code1<XS>(S, r, dead);
      r.refill();
    }
    e3 = code1<XS>(S, r, dead);
  }
}

// Builds canonical tables for the slab's code lengths with NT threads (128 or
// 256).  Returns false for an oversubscribed codebook.
template <int XS, bool COUNT_TABLE, int NT = ST, class SH>
__device__ bool build_tables(SH& S, const uint8_t* lens) {
  constexpr int NW = NT / 32, R = 256 / NT, E = 256 / NT;
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
#pragma unroll
  for (int j = 0; j < E; ++j) S.cnt[t * E + j] = 0;
  if (t == 0) {
    S.maxlen = 0;
    S.minlen = 256;
  }
  uint8_t* hist = &S.hist[0][0];
  for (int k = t; k < 8 * 256; k += NT) hist[k] = 0;
  __syncthreads();
  // symbol chunk c = j * NW + warp holds symbols 32c .. 32c + 31
  int l[R];
  uint32_t rank_w[R];
#pragma unroll
  for (int j = 0; j < R; ++j) {
    const int c = j * NW + warp;
    l[j] = __ldg(lens + 32 * c + lane);
    // per-length counts (16-bit fields) via 32-bit atomics on the containing word
    if (l[j]) {
      uint32_t* w = reinterpret_cast<uint32_t*>(&S.cnt[l[j] & ~1]);
      atomicAdd(w, (l[j] & 1) ? 0x10000u : 1u);
      atomicMax(&S.maxlen, l[j]);
      atomicMin(&S.minlen, l[j]);
    }
    // rank of the symbol among earlier symbols of its chunk with the same length
    const uint32_t same = __match_any_sync(0xffffffffu, l[j]);
    rank_w[j] = __popc(same & ((1u << lane) - 1));
    if (l[j] && rank_w[j] == 0) S.hist[c][l[j]] = uint8_t(__popc(same));
  }
  __syncthreads();
  // offs[] = exclusive scan of cnt[] (E consecutive lengths per thread)
  uint32_t cl[E], tsum = 0;
#pragma unroll
  for (int j = 0; j < E; ++j) {
    cl[j] = S.cnt[t * E + j];
    tsum += cl[j];
  }
  uint32_t v = tsum;
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    const uint32_t u = __shfl_up_sync(0xffffffffu, v, d);
    if (lane >= d) v += u;
  }
  if (lane == 31) S.warpsum[warp] = v;
  __syncthreads();
  uint32_t pre = 0;
  for (int w = 0; w < warp; ++w) pre += S.warpsum[w];
  uint32_t run = pre + v - tsum;
#pragma unroll
  for (int j = 0; j < E; ++j) {
    S.offs[t * E + j] = uint16_t(run);
    run += cl[j];
  }
  if (t == NT - 1) S.offs[256] = uint16_t(run);
  if (t == 0) {
    int64_t avail = 1;  // Kraft check: open prefixes per level, clamped past 256
    bool ok = true;
    for (int k = 1; k <= S.maxlen; ++k) {
      avail = 2 * avail - S.cnt[k];
      if (avail < 0) ok = false;
      if (avail > 4096) avail = 4096;
    }
    uint64_t code = 0;
    for (int k = 1; k <= 32; ++k) {
      const uint64_t ck = S.cnt[k];
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
#pragma unroll
  for (int j = 0; j < R; ++j) {
    const int c = j * NW + warp;
    if (l[j]) {
      uint32_t r = rank_w[j];
      for (int w = 0; w < c; ++w) r += S.hist[w][l[j]];
      S.sorted[S.offs[l[j]] + r] = uint8_t(32 * c + lane);
    }
  }
  __syncthreads();
  // single-code table: thread t fills entries [PER*t, PER*t + PER)
  constexpr int PER = (1 << SK) / NT;
  int len = S.minlen;
  for (int k = 0; k < PER; ++k) {
    const uint32_t e = uint32_t(t * PER + k);
    const uint64_t W = uint64_t(e) << (32 - SK);
    while (len <= SK && W >= S.lim[len]) ++len;
    uint32_t val = 0;
    if (len <= SK) {
      const uint32_t code = e >> (SK - len);
      val = (uint32_t(S.sorted[S.offs[len] + code - uint32_t(S.firstc[len])]) << XS) | uint32_t(len);
    }
    S.lut[e] = decltype(+S.lut[0])(val);
  }
  __syncthreads();
  if constexpr (COUNT_TABLE) {
  // count table: the whole codes inside each CK-bit window
  constexpr int CPER = (1 << CK) / NT;
  for (int k = 0; k < CPER; ++k) {
    const uint32_t v0 = uint32_t(t * CPER + k);
    uint32_t used = 0, n = 0;
    for (;;) {
      const uint32_t idx = ((v0 << used) & ((1u << CK) - 1)) << (SK - CK);
      const uint32_t ln = S.lut[idx] & 31u;
      if (ln == 0 || ln > uint32_t(CK) - used) break;
      used += ln;
      ++n;
    }
    S.clut[v0] = uint8_t(n ? (n << 4) | used : 0);
  }
    __syncthreads();
  }
  return true;
}

struct SerialArgs {
  const uint8_t* payload;
  uint8_t* out;
  const float* x;
  float* y;
  uint32_t ld, nb;
  int* status;
  uint32_t* tidx;         // MODE 2: tile index (bit offset of each 16x16 tile's first code)
  const uint64_t* tbase;  // MODE 2: first index entry of each slab
  uint32_t* tmid;         // MODE 2: bit offset of each tile's row 8 (same entry positions)
  GemvTabs* gtabs;        // MODE 2: each slab's tables for the tile GEMV kernel
};

struct SOut {
  uint16_t* out;
  const float* x;
  float* ysm;
  float* yg;
  uint64_t rows, cols;
  uint32_t ld, nb;
  bool nice, xvec;
  bool out32;  // decode: 32-byte aligned slab output (one 256-bit store per tile row)
};

template <int MODE>
__device__ __forceinline__ void semit_one(const SOut& o, uint32_t p, uint32_t word) {
  const uint64_t idx = untile_index(p, o.rows, o.cols);
  if (MODE == 0) {
    o.out[idx] = uint16_t(word);
  } else {
    const uint64_t r = idx / o.cols, c = idx - r * o.cols;
    const float wf = __uint_as_float(word << 16);
    for (uint32_t b = 0; b < o.nb; ++b) {
      const float pv = wf * __ldg(&o.x[c * o.ld + b]);
      if (o.nice)
        atomicAdd(&o.ysm[r * SMAXB + b], pv);
      else
        atomicAdd(&o.yg[r * o.ld + b], pv);
    }
  }
}

template <int MODE>
__global__ void __launch_bounds__(ST, 3) serial_slab_kernel(const Slab* __restrict__ slabs,
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
           nbits / 8 + (nbits % 8 != 0) == size - kHdr - count;
    }
    if (!ok) {
      if (t == 0) atomicOr(a.status, kStatusHeader);
      continue;
    }
    if (count >= (1ull << 31) || nbits >= (1ull << 32)) {  // 32-bit element / bit indexing
      if (t == 0) atomicOr(a.status, kStatusInternal);
      continue;
    }
    // warm L2 with the whole slab (at most 1 MiB, 32 lines per thread) while
    // its tables are built: each round's bit staging and the exact pass's
    // sign/mantissa loads then hit L2 instead of waiting on DRAM
    for (uint64_t off = uint64_t(t) * 128; off < size; off += uint64_t(ST) * 128)
      asm volatile("prefetch.global.L2 [%0];" ::"l"(p + off));
    if (!build_tables<7, true>(S, p + 16)) {
      if (t == 0) atomicOr(a.status, kStatusCodebook);
      __syncthreads();
      continue;
    }
    if (MODE == 2) {  // the tile GEMV kernel's copy of the tables (the same layout)
      GemvTabs& g = a.gtabs[si];
      for (int k = t; k < (1 << SK); k += ST) g.lut[k] = S.lut[k];
      for (int k = t; k < 33; k += ST) {
        g.lim[k] = S.lim[k];
        g.firstc[k] = S.firstc[k];
      }
      for (int k = t; k < 256; k += ST) {
        g.cnt[k] = S.cnt[k];
        g.sorted[k] = S.sorted[k];
      }
      for (int k = t; k < 257; k += ST) g.offs[k] = S.offs[k];
      if (t == 0) {
        g.maxlen = S.maxlen;
        g.minlen = S.minlen;
      }
    }
    const uint8_t* sm = p + kHdr;
    const uint8_t* bits = p + kHdr + count;
    const uint8_t* end = p + size;
    SOut o;
    o.out = reinterpret_cast<uint16_t*>(a.out + sd.dst);
    o.x = MODE == 1 ? a.x + sd.xoff * a.ld : nullptr;
    o.ysm = S.y;
    o.yg = MODE == 1 ? a.y + sd.dst * a.ld : nullptr;
    o.rows = rows;
    o.cols = cols;
    o.ld = a.ld;
    o.nb = a.nb;
    o.nice = rows == 16 && (cols & 15) == 0 &&
             (MODE == 1 || (reinterpret_cast<uintptr_t>(o.out) & 15) == 0);
    o.xvec = MODE == 1 && a.nb == 1 && a.ld == 1 && (reinterpret_cast<uintptr_t>(o.x) & 15) == 0;
    o.out32 = MODE == 0 && (reinterpret_cast<uintptr_t>(o.out) & 31) == 0;
    if (MODE == 1) {
      for (int k = t; k < 16 * SMAXB; k += ST) S.y[k] = 0.f;
      if (!o.nice)
        for (uint64_t k = t; k < rows * a.nb; k += ST) {
          const uint64_t r = k / a.nb, b = k - r * a.nb;
          o.yg[r * a.ld + b] = 0.f;
        }
      __syncthreads();
    }
    // balanced rounds of ST * S bits, S a multiple of 32 in [64, SMAXS]
    const uint32_t nb32 = uint32_t(nbits);
    const uint32_t nrounds = uint32_t((uint64_t(nb32) + ST * SMAXS - 1) / (ST * SMAXS));
    const uint32_t per_round = nrounds ? uint32_t((uint64_t(nb32) + nrounds - 1) / nrounds) : 0;
    const uint32_t S_bits = max(64u, ((per_round + ST - 1) / ST + 31) & ~31u);
    const uint32_t round_bits = ST * S_bits;
    uint32_t R0 = 0, p0 = 0, base = 0;
    int err = 0;
    const uint32_t cnt32 = uint32_t(count);
    while (R0 < nb32) {
      // ---- 1. the round's bits into shared memory (zero past the slab) ----
      // The 16-byte aligned chunks that hold them arrive by cp.async four
      // words into the window (one memory round trip), then passes of 1024
      // words realign them to the round's first byte and byte-swap them into
      // big-endian words: each pass reads 4+ words ahead of what it writes,
      // and writes after a barrier, so the window is rewritten in place.
      const uint32_t nw = round_bits / 32 + PADW;
      {
        const uintptr_t qa = reinterpret_cast<uintptr_t>(bits + (R0 >> 3));
        const uint8_t* qc = reinterpret_cast<const uint8_t*>(qa & ~uintptr_t(15));
        const uint32_t sb = uint32_t(qa & 15);  // bytes of the first chunk before the round
        const uint32_t nc = (4 * nw + sb + 4 + 15) / 16;
        for (uint32_t c = t; c < nc; c += ST) {
          const uint8_t* src = qc + 16 * c;
          const uint32_t valid = src >= end ? 0u : end - src >= 16 ? 16u : uint32_t(end - src);
          cp_async16_zfill(smem_addr(&S.win[4 + 4 * c]), valid ? src : qc, valid);
        }
        cp_async_commit();
        cp_async_wait_all();
        __syncthreads();
        const uint32_t wq = 4 + (sb >> 2), sh = (sb & 3) * 8;
        for (uint32_t j0 = 0; j0 < nw; j0 += 4 * ST) {
          uint32_t v[4];
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const uint32_t j = j0 + uint32_t(t) + uint32_t(k) * ST;
            if (j < nw) {
              const uint32_t lo = S.win[wq + j], hi = S.win[wq + j + 1];
              v[k] = bswap32(sh ? __funnelshift_r(lo, hi, sh) : lo);
            }
          }
          __syncthreads();
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const uint32_t j = j0 + uint32_t(t) + uint32_t(k) * ST;
            if (j < nw) S.win[j] = v[k];
          }
        }
      }
      const uint32_t lim_rel = min(nb32 - R0, round_bits);
      const uint32_t my_lo = uint32_t(t) * S_bits;
      const uint32_t my_hi = min(my_lo + S_bits, lim_rel);
      const uint32_t p0rel = p0 - R0;
      __syncthreads();
      // ---- 2. count pass ----
      const uint32_t st0 = t == 0 ? p0rel : my_lo;
      uint32_t e1 = st0, n1 = 0, nrec = 0;
      bool d1 = false;
      if (st0 < my_hi) {
        SmemWin96 r;
        r.init(S.win, st0);
        uint32_t pos = st0;
        bool go = true;
        while (go) {
          r.refill_to<4 * SK>();  // four lookups of <= SK bits
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            if (go) {
              if (nrec < REC) {
                S.rec.pos[nrec][t] = uint16_t(pos - my_lo);
                S.rec.cnt[nrec][t] = uint16_t(n1);
                ++nrec;
              }
              // near the stream end whole-window lookups could count padding
              const uint32_t c = pos + CK <= lim_rel ? uint32_t(S.clut[r.w0 >> (32 - CK)]) : 0u;
              if (c) {
                n1 += c >> 4;
                pos += c & 15u;
                r.skip(c & 15u);
              } else {
                code1<7>(S, r, d1);
                ++n1;
                pos = r.pos();
              }
              go = !d1 && pos < my_hi;
            }
          }
        }
        e1 = pos;
      }
      // ---- 3. resynchronisation ----
      uint32_t myE = d1 ? kDead : e1, myN = n1, last_start = st0;
      bool myD = d1;
      S.endpos[t] = myE;
      for (int iter = 0; iter <= ST; ++iter) {
        __syncthreads();
        const uint32_t A = t == 0 ? p0rel : S.endpos[t - 1];
        const bool redo = t > 0 && A != last_start;
        __syncthreads();
        if (redo) {
          last_start = A;
          if (A != kDead && A >= my_hi) {
            myD = false;  // no code of the true sequence starts in this range
            myE = A;
            myN = 0;
          } else if (A == kDead || A < my_lo) {
            myD = true;   // predecessor hit an invalid code
            myE = kDead;
            myN = 0;
          } else {
            SmemWin96 r;
            r.init(S.win, A);
            uint32_t pos = A, k = 0, j = 0;
            const uint32_t m = nrec;
            bool synced = false, dead = false;
            while (pos < my_hi) {
              const uint32_t rel = pos - my_lo;
              while (j < m && S.rec.pos[j][t] < rel) ++j;
              if (j < m && S.rec.pos[j][t] == rel) {
                synced = true;
                break;
              }
              r.refill();
              code1<7>(S, r, dead);
              if (dead) break;
              pos = r.pos();
              ++k;
            }
            if (synced) {
              myN = k + n1 - S.rec.cnt[j][t];
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
        const uint32_t u = __shfl_up_sync(0xffffffffu, v, d);
        if (lane >= d) v += u;
      }
      if (lane == 31) S.warpsum[warp] = v;
      const int any_dead = __syncthreads_or(myD);
      uint32_t wpre = 0, tot = 0;
      for (int w = 0; w < ST / 32; ++w) {
        const uint32_t ws = S.warpsum[w];
        if (w < warp) wpre += ws;
        tot += ws;
      }
      const uint32_t my_off = wpre + v - myN;
      const uint32_t last_end = S.endpos[ST - 1];
      if (any_dead || uint64_t(base) + tot > count) {
        err = kStatusStream;
        break;
      }
      // ---- 5. exact decode straight to the output ----
      if (MODE == 2 && myN) {
        // tile index: the stream offset of every 256th code (a 16x16 tile
        // start) and of every tile's 129th code (its row 8)
        SmemWin96 r;
        r.init(S.win, t == 0 ? p0rel : S.endpos[t - 1]);
        bool dead = false;
        uint32_t* ti = a.tidx + a.tbase[si];
        uint32_t* tm = a.tmid + a.tbase[si];
        const uint32_t gend = base + my_off + myN;
        for (uint32_t g = base + my_off; g < gend; ++g) {
          if ((g & 127u) == 0) ((g & 128u) ? tm : ti)[g >> 8] = R0 + r.pos();
          r.refill();
          code1<7>(S, r, dead);
        }
      } else if (myN) {
        SmemWin96 r;
        r.init(S.win, t == 0 ? p0rel : S.endpos[t - 1]);
        bool dead = false;
        uint32_t g = base + my_off;
        const uint32_t gend = g + myN;
        if (MODE == 0 && o.nice) {
          // whole tile rows: 16 codes -> one 32-byte store (two 16-byte
          // stores when the output is only 16-byte aligned)
          for (; g < gend && (g & 15); ++g) {
            r.refill();
            const uint32_t e = code1<7>(S, r, dead);
            semit_one<MODE>(o, g, merge1(e, __ldg(sm + g)));
          }
          if (g + 16 <= gend) {
            ByteReader8 smr;
            smr.init(sm + g, sm + cnt32);
            for (; g + 16 <= gend; g += 16) {
              uint4 wv[2];
#pragma unroll
              for (int hh = 0; hh < 2; ++hh) {
                const uint64_t s8 = smr.take();
                uint32_t e[8];
                r.refill_to<4 * SK>();
                code4<7>(S, r, dead, e[0], e[1], e[2], e[3]);
                r.refill_to<4 * SK>();
                code4<7>(S, r, dead, e[4], e[5], e[6], e[7]);
                const uint32_t slo = uint32_t(s8), shi = uint32_t(s8 >> 32);
                wv[hh].x = (__byte_perm(e[0], e[1], 0x5410) & 0x7F807F80u) | (__byte_perm(slo, 0, 0x1100) & 0x807F807Fu);
                wv[hh].y = (__byte_perm(e[2], e[3], 0x5410) & 0x7F807F80u) | (__byte_perm(slo, 0, 0x3322) & 0x807F807Fu);
                wv[hh].z = (__byte_perm(e[4], e[5], 0x5410) & 0x7F807F80u) | (__byte_perm(shi, 0, 0x1100) & 0x807F807Fu);
                wv[hh].w = (__byte_perm(e[6], e[7], 0x5410) & 0x7F807F80u) | (__byte_perm(shi, 0, 0x3322) & 0x807F807Fu);
              }
              uint16_t* dst = o.out + size_t((g >> 4) & 15) * cols + (g >> 8) * 16;
              if (o.out32) {
                st_global_32B(dst, wv[0], wv[1]);
              } else {
                reinterpret_cast<uint4*>(dst)[0] = wv[0];
                reinterpret_cast<uint4*>(dst)[1] = wv[1];
              }
            }
          }
        } else if (o.nice) {
          for (; g < gend && (g & 7); ++g) {
            r.refill();
            const uint32_t e = code1<7>(S, r, dead);
            semit_one<MODE>(o, g, merge1(e, __ldg(sm + g)));
          }
          if (g + 8 <= gend) {
            ByteReader8 smr;
            smr.init(sm + g, sm + cnt32);
            for (; g + 8 <= gend; g += 8) {
              const uint64_t s8 = smr.take();
              uint32_t e[8];
              r.refill_to<4 * SK>();
              code4<7>(S, r, dead, e[0], e[1], e[2], e[3]);
              r.refill_to<4 * SK>();
              code4<7>(S, r, dead, e[4], e[5], e[6], e[7]);
              const uint32_t slo = uint32_t(s8), shi = uint32_t(s8 >> 32);
              const uint32_t rr = (g >> 4) & 15, c = (g >> 8) * 16 + (g & 15);
              if (MODE == 0) {
                uint4 w;
                w.x = (__byte_perm(e[0], e[1], 0x5410) & 0x7F807F80u) | (__byte_perm(slo, 0, 0x1100) & 0x807F807Fu);
                w.y = (__byte_perm(e[2], e[3], 0x5410) & 0x7F807F80u) | (__byte_perm(slo, 0, 0x3322) & 0x807F807Fu);
                w.z = (__byte_perm(e[4], e[5], 0x5410) & 0x7F807F80u) | (__byte_perm(shi, 0, 0x1100) & 0x807F807Fu);
                w.w = (__byte_perm(e[6], e[7], 0x5410) & 0x7F807F80u) | (__byte_perm(shi, 0, 0x3322) & 0x807F807Fu);
                *reinterpret_cast<uint4*>(o.out + size_t(rr) * cols + c) = w;
              } else {
                float wf[8];
#pragma unroll
                for (int q = 0; q < 8; ++q) {
                  const uint32_t sb = (q < 4 ? slo : shi) >> (8 * (q & 3));
                  wf[q] = __uint_as_float(merge1(e[q], sb & 255u) << 16);
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
                  atomicAdd(&S.y[rr * SMAXB], acc);
                } else {
                  for (uint32_t b = 0; b < o.nb; ++b) {
                    float acc = 0.f;
#pragma unroll
                    for (int q = 0; q < 8; ++q)
                      acc = fmaf(wf[q], __ldg(&o.x[uint64_t(c + q) * o.ld + b]), acc);
                    atomicAdd(&S.y[rr * SMAXB + b], acc);
                  }
                }
              }
            }
          }
        }
        for (; g < gend; ++g) {
          r.refill();
          const uint32_t e = code1<7>(S, r, dead);
          semit_one<MODE>(o, g, merge1(e, __ldg(sm + g)));
        }
      }
      base += tot;
      p0 = R0 + last_end;
      R0 += round_bits;
      __syncthreads();
    }
    if (!err && (base != cnt32 || p0 != nb32)) err = kStatusStream;
    if (err) {
      if (t == 0) atomicOr(a.status, err);
    } else if (MODE == 2) {
      if (t == 0) a.tidx[a.tbase[si] + (cnt32 >> 8)] = nb32;  // end sentinel
    } else if (MODE == 1 && o.nice) {
      for (uint32_t k = t; k < 16 * a.nb; k += ST) {
        const uint32_t r = k / a.nb, b = k - r * a.nb;
        a.y[(sd.dst + r) * a.ld + b] = S.y[r * SMAXB + b];
      }
    }
    __syncthreads();
  }
}

// ------------------------------------------------ indexed tile GEMV ------
// With a tile index (the bit offsets of every 16x16 tile's first code and of
// its row 8, and each slab's decode tables, built once per plan by
// serial_slab_kernel<2>), every tile of a 16-row slab can be decoded on its
// own: one thread per tile (or two, rows 0-7 and 8-15), no speculative pass.
// A CTA takes up to GT consecutive tiles of one slab, copies the slab's
// tables and stages the tiles' bits in shared memory (in several rounds when
// they do not fit), and each thread walks its rows: 16 codes a row, 16 FP32
// weights assembled from the table entry (exponent at bit 23) and the
// sign/mantissa bytes, 16 FMAs with x held in registers, then a warp sum per
// row.  Slabs split over several CTAs combine their row sums in a fixed order
// in the last CTA to finish (deterministic, and Y is overwritten as
// cuda/decode.cu:31 requires).
constexpr int GT = 256;                  // tiles per GEMV item (CTA)
constexpr int GPAD = 160;                // zero words past a round: one row of 16 maximal codes + window
constexpr int GWINW = 6144 + GPAD;       // staged bit words per round
constexpr uint32_t GCAP = uint32_t(GWINW - GPAD - 9) * 32;  // bits per round (+ up to 4 words of alignment)
constexpr int GNB = 4;                   // batch columns per pass
// Threads per tile (SPLIT): one, or, for launches at batch <= 1 whose items
// fill under one wave of 256-thread CTAs, two -- rows 0-7 from the tile's
// first code and rows 8-15 from its row-8 offset (both in the index) -- so
// that such a launch has twice the threads (a 4096 x 4096 weight is 65536
// tiles, under half of the 148 x 1024 threads the GPU holds).  Measured on
// 16 x 4096 slabs at batch 1: 256 slabs 31.2 us split against 50.0; 1024
// slabs (1.7 waves) 102.5 against 97.7, hence one thread per tile there.
constexpr int GTMAX = 2 * GT;            // threads per CTA at most

// The tables (16-bit single-code entries: fewer bank conflicts) lead, in the
// layout the index pass writes them to global memory.
static_assert((1 << SK) == sizeof(GemvTabs::lut) / 2, "the exported table has SK bits");
struct GemvShared : GemvTabs {
  alignas(16) uint32_t win[GWINW];
  float red[16][GTMAX / 32][GNB];
  int flag;
};

// FP32 weight from a table entry (exponent at bit 7, length in bits 0-4) and
// the sign/mantissa byte K of sw: byte -> bits 16-23 and 24-31, then one
// bit-select keeps sign (31) and mantissa (16-22) from it, exponent from e << 16.
template <int K>
__device__ __forceinline__ float wfloat(uint32_t e, uint32_t sw) {
  constexpr uint32_t sel = 0x0044u | (uint32_t(K) << 8) | (uint32_t(K) << 12);
  const uint32_t s = __byte_perm(sw, 0u, sel);
  return __uint_as_float((s & 0x807FFFFFu) | ((e << 16) & 0x7F800000u));
}

// Y[row, b] = v: the local output, or (fused tensor parallel) this rank's
// block of its own gathered buffer.
__device__ __forceinline__ void store_y(const GemvArgs& a, uint64_t row, uint32_t b, float v) {
  float* y = a.npeers ? a.peer_y[a.rank] + a.peer_row0 * a.ld : a.y;
  y[row * a.ld + b] = v;
}

// acc[b] += w(e_k, byte k of sw) * x[4q + k][b] for the block's four codes;
// xr4 holds the block's x values, column-major in k then b (NB per column).
template <int NB>
__device__ __forceinline__ void fma4(float* acc, uint32_t e0, uint32_t e1, uint32_t e2, uint32_t e3,
                                     uint32_t sw, const float* xr4) {
  const float w0 = wfloat<0>(e0, sw), w1 = wfloat<1>(e1, sw);
  const float w2 = wfloat<2>(e2, sw), w3 = wfloat<3>(e3, sw);
#pragma unroll
  for (int b = 0; b < NB; ++b) {
    acc[b] = fmaf(w0, xr4[b], acc[b]);
    acc[b] = fmaf(w1, xr4[NB + b], acc[b]);
    acc[b] = fmaf(w2, xr4[2 * NB + b], acc[b]);
    acc[b] = fmaf(w3, xr4[3 * NB + b], acc[b]);
  }
}

// NB == 0: decode mode (BF16 tile rows to a.out + slab dst); NB >= 1: GEMV/GEMM.
template <int NB, int SPLIT>
__global__ void __launch_bounds__(GT * SPLIT, SPLIT == 2 || NB > 1 ? 2 : 4) serial_tile_gemv_kernel(GemvArgs a) {
  static_assert(SPLIT == 1 || (SPLIT == 2 && NB <= 1), "two threads per tile at batch <= 1");
  constexpr int NT = GT * SPLIT;   // threads
  constexpr int RPT = 16 / SPLIT;  // tile rows per thread
  extern __shared__ __align__(16) uint8_t smem_raw[];
  GemvShared& S = *reinterpret_cast<GemvShared*>(smem_raw);
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const int tl = t % GT;    // this thread's tile of the item
  const int part = t / GT;  // and its rows: part * RPT .. + RPT - 1
  // the stream's next kernel may start launching once every CTA of this one
  // has started (it waits for this grid before touching what it shares)
  asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");
  for (uint32_t ii = blockIdx.x; ii < a.nitems; ii += gridDim.x) {
    const GemvItem it = a.items[ii];
    const Slab sd = a.slabs[it.slab];
    const uint8_t* p = a.payload + sd.src;
    const uint32_t count = uint32_t(sd.rows * sd.cols);
    const uint32_t nbits = uint32_t(ld_le64(p + 8));
    // warm L2 with the item's sign/mantissa tiles and bit range (the tile
    // index bounds it; clamped to the slab) while its tables arrive, in
    // launches of under one wave (two threads per tile): measured on the
    // Llama-3-8B forward of linears +3 % tokens/s from those launches, while a
    // full 1024-slab launch loses ~3 % to the extra L2 requests.
    if (SPLIT == 2) {
      const uint8_t* smp = p + kHdr + uint64_t(it.tile0) * 256;
      const uint64_t smn = uint64_t(it.ntiles) * 256;
      for (uint64_t off = uint64_t(t) * 128; off < smn; off += uint64_t(NT) * 128)
        asm volatile("prefetch.global.L2 [%0];" ::"l"(smp + off));
      const uint32_t* tix = a.tidx + a.tbase[it.slab];
      const uint64_t nbb = sd.size - kHdr - count;
      const uint64_t pb0 = tix[it.tile0] >> 3, pb1 = min(uint64_t(tix[it.tile0 + it.ntiles] + 7) >> 3, nbb);
      const uint8_t* bp = p + kHdr + count;
      for (uint64_t off = pb0 + uint64_t(t) * 128; off < pb1; off += uint64_t(NT) * 128)
        asm volatile("prefetch.global.L2 [%0];" ::"l"(bp + off));
    }
    const uint32_t* ti = a.tidx + a.tbase[it.slab];
    const uint8_t* sm = p + kHdr;
    const uint8_t* bits = sm + count;
    const uint8_t* end = p + sd.size;
    const bool mine = uint32_t(tl) < it.ntiles;
    const uint32_t tile = it.tile0 + uint32_t(mine ? tl : 0);
    const uint32_t b0 = ti[tile], b1 = ti[tile + 1];
    // where this thread's rows start: the tile's first code, or its row 8
    const uint32_t bs = part ? a.tmid[a.tbase[it.slab] + tile] : b0;
    // A round: the tiles [ta, tb) whose bits fit the window, staged as the
    // 16-byte aligned chunks that hold them by cp.async (bytes past the slab
    // read as zero); the first round's copies overlap the table build.
    struct Round {
      uint32_t tb, base_bit, slack;
      bool ok;
    };
    auto issue_round = [&](uint32_t ta) {
      Round rd;
      rd.base_bit = ti[it.tile0 + ta] & ~31u;
      const bool fits = mine && part == 0 && uint32_t(tl) >= ta && b1 - rd.base_bit <= GCAP;
      rd.tb = ta + uint32_t(__syncthreads_count(fits));
      const uint32_t end_bit = ti[it.tile0 + rd.tb];
      // an index that does not describe this payload fails here (uniformly)
      rd.ok = !(rd.tb == ta || end_bit < rd.base_bit || end_bit - rd.base_bit > GCAP);
      const uintptr_t qa = reinterpret_cast<uintptr_t>(bits + (rd.base_bit >> 3));
      const uint8_t* qc = reinterpret_cast<const uint8_t*>(qa & ~uintptr_t(15));
      rd.slack = uint32_t(qa & 15) * 8;  // staged bits before the round's first bit
      const uint32_t nc = rd.ok ? ((end_bit - rd.base_bit + rd.slack + 31) / 32 + GPAD + 3) / 4 : 0u;
      for (uint32_t c = t; c < nc; c += NT) {
        const uint8_t* src = qc + 16 * c;
        const uint32_t valid = src >= end ? 0u : end - src >= 16 ? 16u : uint32_t(end - src);
        cp_async16_zfill(smem_addr(&S.win[4 * c]), valid ? src : qc, valid);
      }
      cp_async_commit();
      return rd;
    };
    // every staged word byte-swapped in place into the window's big-endian words
    auto finish_round = [&](const Round& rd) {
      const uint32_t end_bit = ti[it.tile0 + rd.tb];
      const uint32_t nc = ((end_bit - rd.base_bit + rd.slack + 31) / 32 + GPAD + 3) / 4;
      cp_async_wait_all();
      __syncthreads();
      for (uint32_t j = t; j < 4 * nc; j += NT) S.win[j] = bswap32(S.win[j]);
      __syncthreads();
    };
    Round rd = issue_round(0);
    {
      // the slab's tables from the index pass, landing with the round's bits
      // (the previous item's last barrier has retired every read of them)
      const uint4* src = reinterpret_cast<const uint4*>(a.gtabs + it.slab);
      uint4* dst = reinterpret_cast<uint4*>(static_cast<GemvTabs*>(&S));
      for (int k = t; k < int(sizeof(GemvTabs) / 16); k += NT) cp_async16(dst + k, src + k);
      cp_async_commit();
    }
    if (NB > 0)
      for (int k = t; k < 16 * (GTMAX / 32) * GNB; k += NT) (&S.red[0][0][0])[k] = 0.f;
    // Launched behind the stream's previous kernel (programmatic dependent
    // launch), everything above read only the payload, the index and the
    // plan; x, Y, the partials and the output are touched after that kernel
    // has completed and its writes are visible.
    asm volatile("griddepcontrol.wait;\n" ::: "memory");
    // x for this tile's 16 columns
    const float* xs = a.x + (sd.xoff + uint64_t(tile) * 16) * a.ld;
    // x[c][b] for the tile's 16 columns and the pass's nb <= NB batch columns
    // (zero beyond nb), in registers for the whole tile
    float xr[NB > 0 ? 16 * NB : 1];
    if (NB == 0) {
      // decode mode: no x
    } else if (NB == 1 && a.ld == 1 && (reinterpret_cast<uintptr_t>(xs) & 15) == 0) {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float4 v = __ldg(reinterpret_cast<const float4*>(xs) + q);
        xr[4 * q] = v.x;
        xr[4 * q + 1] = v.y;
        xr[4 * q + 2] = v.z;
        xr[4 * q + 3] = v.w;
      }
    } else {
#pragma unroll
      for (int c = 0; c < 16; ++c)
#pragma unroll
        for (int b = 0; b < NB; ++b)
          xr[c * NB + b] = uint32_t(b) < a.nb ? __ldg(xs + uint64_t(c) * a.ld + b) : 0.f;
    }
    // the tile's 256 sign/mantissa bytes, one 16-byte row per step from
    // aligned 16-byte loads (the misalignment is the same for the whole slab;
    // the chunk past the tile is the slab's next bytes, so loads stay inside)
    const uintptr_t sma = reinterpret_cast<uintptr_t>(sm + uint64_t(tile) * 256);
    const int soff = int(sma & 15);
    const uint4* sq = reinterpret_cast<const uint4*>(sma & ~uintptr_t(15));
    const bool ostore16 = NB == 0 && ((reinterpret_cast<uintptr_t>(a.out + sd.dst) | (sd.cols * 2)) & 15) == 0;
    const bool ostore32 = NB == 0 && ((reinterpret_cast<uintptr_t>(a.out + sd.dst) | (sd.cols * 2)) & 31) == 0;
    uint32_t ta = 0;
    while (ta < it.ntiles) {  // rounds (one, unless the tiles' bits exceed GCAP)
      if (ta) rd = issue_round(ta);
      if (!rd.ok) {
        if (t == 0) atomicOr(a.status, kStatusInternal);
        cp_async_wait_all();
        break;
      }
      finish_round(rd);
      const uint32_t tb = rd.tb, base_bit = rd.base_bit, slack = rd.slack;
      bool act = mine && uint32_t(tl) >= ta && uint32_t(tl) < tb && b0 >= base_bit && b1 >= b0 && bs >= b0 &&
                 bs <= b1;
      SmemWin96 r;
      r.init(S.win, act ? bs - base_bit + slack : 0u);
      bool dead = false;
      // sign/mantissa rows loaded one row ahead of use
      const int row0 = part * RPT;
      uint4 nlo = ldg16(sq + row0), nhi = soff ? ldg16(sq + row0 + 1) : make_uint4(0, 0, 0, 0);
      for (int row = row0; row < row0 + RPT; ++row) {
        const uint4 lo = nlo, hi = nhi;
        const int nr = row < 15 ? row + 1 : 15;
        nlo = ldg16(sq + nr);
        if (soff) nhi = ldg16(sq + nr + 1);
        float acc[NB > 0 ? NB : 1];
#pragma unroll
        for (int b = 0; b < NB; ++b) acc[b] = 0.f;
        // a row starts inside the staged bits: its 16 codes stay inside GPAD
        if (act && r.pos() > b1 - base_bit + slack) {
          atomicOr(a.status, kStatusStream);
          act = false;
        }
        if (act && NB == 0) {
          // decode: tile row `row` = 16 BF16 words, two 16-byte halves
          const uint4 s16 = realign16(lo, hi, soff);
          const uint32_t sw[4] = {s16.x, s16.y, s16.z, s16.w};
          uint8_t* orow = a.out + sd.dst + (uint64_t(row) * sd.cols + uint64_t(tile) * 16) * 2;
          uint4 wrow[2];
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {
            uint32_t e[8];
            r.refill_to<4 * SK>();
            code4<7>(S, r, dead, e[0], e[1], e[2], e[3]);
            r.refill_to<4 * SK>();
            code4<7>(S, r, dead, e[4], e[5], e[6], e[7]);
            const uint32_t slo = sw[2 * hh], shi = sw[2 * hh + 1];
            uint4 w;
            w.x = (__byte_perm(e[0], e[1], 0x5410) & 0x7F807F80u) | (__byte_perm(slo, 0, 0x1100) & 0x807F807Fu);
            w.y = (__byte_perm(e[2], e[3], 0x5410) & 0x7F807F80u) | (__byte_perm(slo, 0, 0x3322) & 0x807F807Fu);
            w.z = (__byte_perm(e[4], e[5], 0x5410) & 0x7F807F80u) | (__byte_perm(shi, 0, 0x1100) & 0x807F807Fu);
            w.w = (__byte_perm(e[6], e[7], 0x5410) & 0x7F807F80u) | (__byte_perm(shi, 0, 0x3322) & 0x807F807Fu);
            wrow[hh] = w;
          }
          if (ostore32) {
            st_global_32B(orow, wrow[0], wrow[1]);
          } else if (ostore16) {
            reinterpret_cast<uint4*>(orow)[0] = wrow[0];
            reinterpret_cast<uint4*>(orow)[1] = wrow[1];
          } else {  // 2-byte aligned output
            uint16_t* o2 = reinterpret_cast<uint16_t*>(orow);
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
              const uint4 w = wrow[hh];
              o2[8 * hh + 0] = uint16_t(w.x); o2[8 * hh + 1] = uint16_t(w.x >> 16);
              o2[8 * hh + 2] = uint16_t(w.y); o2[8 * hh + 3] = uint16_t(w.y >> 16);
              o2[8 * hh + 4] = uint16_t(w.z); o2[8 * hh + 5] = uint16_t(w.z >> 16);
              o2[8 * hh + 6] = uint16_t(w.w); o2[8 * hh + 7] = uint16_t(w.w >> 16);
            }
          }
        } else if (act) {
          const uint4 s16 = realign16(lo, hi, soff);
          const uint32_t sw[4] = {s16.x, s16.y, s16.z, s16.w};
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            uint32_t e0, e1, e2, e3;
            r.refill_to<4 * SK>();
            code4<7>(S, r, dead, e0, e1, e2, e3);
            fma4<NB>(acc, e0, e1, e2, e3, sw[q], xr + 4 * q * NB);
          }
        }
#pragma unroll
        for (int b = 0; b < NB; ++b) {
          float v = acc[b];
#pragma unroll
          for (int d = 16; d >= 1; d >>= 1) v += __shfl_xor_sync(0xffffffffu, v, d);
          if (lane == 0) S.red[row][warp][b] += v;
        }
      }
      __syncthreads();
      ta = tb;
    }
    (void)nbits;
    if (NB == 0) {
      __syncthreads();
      continue;
    }
    // combine: row r, column b
    const bool comb = uint32_t(t) < 16u * a.nb;
    const uint32_t rr = uint32_t(t) / a.nb, bb = uint32_t(t) - rr * a.nb;
    float v = 0.f;
    if (comb)
      for (int w = 0; w < NT / 32; ++w) v += S.red[rr][w][bb];
    if (it.nitems == 1) {
      if (comb) store_y(a, sd.dst + rr, bb, v);
    } else {
      if (comb) a.partials[uint64_t(ii) * 16 * GNB + rr * GNB + bb] = v;
      __threadfence();
      __syncthreads();
      if (t == 0) S.flag = atomicAdd(&a.counters[it.slab], 1u) == it.nitems - 1;
      __syncthreads();
      if (S.flag) {
        __threadfence();
        if (comb) {
          float sum = 0.f;
          for (uint32_t j = 0; j < it.nitems; ++j)
            sum += __ldcg(&a.partials[uint64_t(it.first + j) * 16 * GNB + rr * GNB + bb]);
          store_y(a, sd.dst + rr, bb, sum);
        }
        if (t == 0) a.counters[it.slab] = 0;
      }
    }
    __syncthreads();
  }
  if (NB > 0 && a.npeers) {
    // fused all-gather: the last CTA to finish copies this rank's block of Y
    // into every other rank's gathered buffer (peer stores over NVLink), makes
    // them visible system-wide, and publishes the new epoch to every rank
    __threadfence();
    __syncthreads();
    if (t == 0) S.flag = atomicAdd(a.done, 1u) == gridDim.x - 1;
    __syncthreads();
    if (S.flag) {
      __threadfence();
      const uint64_t n = a.peer_rows * a.ld, off = a.peer_row0 * a.ld;
      const float* src = a.peer_y[a.rank] + off;
      for (uint64_t i = t; i < n; i += NT) {
        const float v = __ldcg(src + i);
        for (uint32_t g = 0; g < a.npeers; ++g)
          if (g != a.rank) a.peer_y[g][off + i] = v;
      }
      __threadfence_system();
      __syncthreads();
      if (t == 0) {
        *a.done = 0;
        const uint32_t e = *reinterpret_cast<volatile uint32_t*>(a.epoch) + 1;
        *reinterpret_cast<volatile uint32_t*>(a.epoch) = e;
        __threadfence_system();
        for (uint32_t g = 0; g < a.npeers; ++g)
          *reinterpret_cast<volatile uint32_t*>(a.peer_flags[g] + a.rank) = e;
      }
    }
  }
}

// One thread per rank polls that rank's flag until it reaches this rank's
// epoch (every rank makes the same sequence of fused calls); the wait is
// bounded (about a second), after which the status word gets an error bit.
__global__ void tp_wait_kernel(const uint32_t* flags, uint32_t world, const uint32_t* epoch, int* status) {
  const uint32_t g = threadIdx.x;
  if (g < world) {
    const uint32_t target = *reinterpret_cast<const volatile uint32_t*>(epoch);
    const volatile uint32_t* f = flags + g;
    uint32_t i = 0;
    while (int32_t(*f - target) < 0) {
      if (++i > (1u << 23)) {
        atomicOr(status, kStatusInternal);
        break;
      }
      __nanosleep(128);
    }
  }
  __threadfence_system();
}

// Dynamic shared memory opt-in, once per device (concurrent first calls both
// set the same values, which is harmless).
void serial_set_attr() {
  static std::atomic<uint64_t> done{0};
  int dev = 0;
  cudaGetDevice(&dev);
  const uint64_t bit = dev < 64 ? (1ull << dev) : 0ull;
  if (bit && (done.load(std::memory_order_acquire) & bit)) return;
  cudaFuncSetAttribute(serial_slab_kernel<0>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(sizeof(SerialShared)));
  cudaFuncSetAttribute(serial_slab_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(sizeof(SerialShared)));
  cudaFuncSetAttribute(serial_slab_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(sizeof(SerialShared)));
  cudaFuncSetAttribute(serial_tile_gemv_kernel<0, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(sizeof(GemvShared)));
  cudaFuncSetAttribute(serial_tile_gemv_kernel<0, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(sizeof(GemvShared)));
  cudaFuncSetAttribute(serial_tile_gemv_kernel<1, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(sizeof(GemvShared)));
  cudaFuncSetAttribute(serial_tile_gemv_kernel<1, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(sizeof(GemvShared)));
  cudaFuncSetAttribute(serial_tile_gemv_kernel<2, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(sizeof(GemvShared)));
  cudaFuncSetAttribute(serial_tile_gemv_kernel<4, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(sizeof(GemvShared)));
  if (bit) done.fetch_or(bit, std::memory_order_release);
}

}  // namespace

size_t serial_smem_bytes() { return sizeof(SerialShared); }

cudaError_t launch_serial_decode(const Slab* slabs, uint32_t n, const uint8_t* payload,
                                 uint8_t* out, int* status, int grid, cudaStream_t st) {
  if (!n) return cudaSuccess;
  serial_set_attr();
  SerialArgs a{payload, out, nullptr, nullptr, 1, 1, status, nullptr, nullptr};
  const int g = grid < int(n) ? grid : int(n);
  serial_slab_kernel<0><<<g, ST, sizeof(SerialShared), st>>>(slabs, n, a);
  return cudaGetLastError();
}

cudaError_t launch_serial_gemm(const Slab* slabs, uint32_t n, const uint8_t* payload,
                               const float* x, float* y, uint32_t ld, uint32_t b0, uint32_t nb,
                               int* status, int grid, cudaStream_t st) {
  if (!n) return cudaSuccess;
  serial_set_attr();
  SerialArgs a{payload, nullptr, x + b0, y + b0, ld, nb, status, nullptr, nullptr};
  const int g = grid < int(n) ? grid : int(n);
  serial_slab_kernel<1><<<g, ST, sizeof(SerialShared), st>>>(slabs, n, a);
  return cudaGetLastError();
}

cudaError_t launch_serial_index(const Slab* slabs, uint32_t n, const uint8_t* payload,
                                uint32_t* tidx, uint32_t* tmid, const uint64_t* tbase, GemvTabs* gtabs,
                                int* status, cudaStream_t st) {
  if (!n) return cudaSuccess;
  serial_set_attr();
  SerialArgs a{payload, nullptr, nullptr, nullptr, 1, 1, status, tidx, tbase, tmid, gtabs};
  serial_slab_kernel<2><<<n, ST, sizeof(SerialShared), st>>>(slabs, n, a);
  return cudaGetLastError();
}

// The indexed kernel is launched with programmatic stream serialisation: its
// CTAs may start (table build, bit staging) while the stream's previous
// kernel finishes, and wait for it before touching shared data.
template <int NB, int SPLIT>
cudaError_t launch_tile_kernel(const GemvArgs& args, cudaStream_t st) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(args.nitems);
  cfg.blockDim = dim3(GT * SPLIT);
  cfg.dynamicSmemBytes = sizeof(GemvShared);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, serial_tile_gemv_kernel<NB, SPLIT>, args);
}

// Two threads per tile when the items fill under one wave of 256-thread CTAs
// (4 per SM).
bool tile_split(uint32_t nitems) {
  static std::atomic<int> sms{0};
  int n = sms.load(std::memory_order_relaxed);
  if (!n) {
    int dev = 0;
    cudaGetDevice(&dev);
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    sms.store(n, std::memory_order_relaxed);
  }
  return nitems <= uint32_t(4 * n);
}

cudaError_t launch_serial_tile_gemm(const GemvArgs& args, cudaStream_t st) {
  if (!args.nitems) return cudaSuccess;
  if (args.nb < 1 || args.nb > uint32_t(GNB)) return cudaErrorInvalidValue;
  if (!args.gtabs || !args.tmid) return cudaErrorInvalidValue;  // the index pass's tables and row-8 offsets
  serial_set_attr();
  if (args.nb == 1)
    return tile_split(args.nitems) ? launch_tile_kernel<1, 2>(args, st) : launch_tile_kernel<1, 1>(args, st);
  if (args.nb == 2) return launch_tile_kernel<2, 1>(args, st);
  return launch_tile_kernel<4, 1>(args, st);
}

cudaError_t launch_serial_tile_decode(const GemvArgs& args, cudaStream_t st) {
  if (!args.nitems) return cudaSuccess;
  if (!args.gtabs || !args.tmid) return cudaErrorInvalidValue;
  serial_set_attr();
  return tile_split(args.nitems) ? launch_tile_kernel<0, 2>(args, st) : launch_tile_kernel<0, 1>(args, st);
}

cudaError_t launch_tp_wait(const uint32_t* flags, uint32_t world, const uint32_t* epoch, int* status,
                           cudaStream_t st) {
  tp_wait_kernel<<<1, 32 * ((world + 31) / 32), 0, st>>>(flags, world, epoch, status);
  return cudaGetLastError();
}

}  // namespace xksv
