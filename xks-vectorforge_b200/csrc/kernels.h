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
struct GemvTabs;

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

// Tile index of 16-row serial-codec slabs: tidx[tbase[i] + k] = bit offset of
// tile k's first code in slab i's stream, tidx[tbase[i] + tiles] = bit count;
// tmid[tbase[i] + k] = bit offset of tile k's row 8 (its 129th code).
cudaError_t launch_serial_index(const Slab* slabs, uint32_t n, const uint8_t* payload,
                                uint32_t* tidx, uint32_t* tmid, const uint64_t* tbase, GemvTabs* gtabs,
                                int* status, cudaStream_t st);

// A 16-row serial-codec slab's decode tables as the tile GEMV kernel holds
// them in shared memory: the 2^11-entry single-code table (exponent << 7 |
// length; 0 = longer code) and the canonical data of longer codes (limits,
// first codes, counts, offsets, symbols in (length, symbol) order).  Written
// once per slab by the tile-index pass (xksv_plan_index) and copied in by each
// GEMV item instead of being rebuilt from the code lengths.
struct alignas(16) GemvTabs {
  uint16_t lut[1 << 11];
  uint64_t lim[33];
  uint64_t firstc[33];
  alignas(16) uint16_t cnt[256];
  uint16_t offs[257];
  uint8_t sorted[256];
  int maxlen, minlen;
};
static_assert(sizeof(GemvTabs) == 5920, "per-slab table bytes, as documented and counted by bench.py");

struct GemvArgs {
  const GemvItem* items;
  uint32_t nitems;
  const Slab* slabs;       // slabs the items refer to
  const uint64_t* tbase;   // per slab: first tile-index entry
  const uint32_t* tidx;    // tile index
  const uint8_t* payload;
  const float* x;          // X at batch column b0 (row stride ld)
  float* y;                // Y at batch column b0 (row stride ld)
  uint32_t ld, nb;         // nb <= 4 columns this pass
  float* partials;         // [item][16][4] row sums of slabs split over several items
  uint32_t* counters;      // per slab, zero between launches
  int* status;
  uint8_t* out;            // indexed decode: output base (slab dst = byte offset)
  const GemvTabs* gtabs;   // per slab: its tables (from the index pass)
  const uint32_t* tmid;    // bit offset of each tile's row 8 (tile-index positions)
  // fused tensor-parallel all-gather (npeers > 0): output rows go to this
  // rank's block (rows peer_row0 ..) of its own gathered buffer; the grid's
  // last CTA copies the block into every other rank's buffer over NVLink and
  // raises this rank's flag on every rank
  float* const* peer_y;    // [npeers] gathered buffers (this call's half)
  uint32_t* const* peer_flags;  // [npeers] flag arrays, indexed by source rank
  uint32_t npeers, rank;
  uint64_t peer_row0, peer_rows;  // this rank's block of the gathered Y
  uint32_t* done;          // grid completion counter (zero between launches)
  uint32_t* epoch;         // this rank's completed fused calls
};
// Indexed fused GEMV/GEMM (nb <= 4) over 16-row serial-codec slabs.
cudaError_t launch_serial_tile_gemm(const GemvArgs& args, cudaStream_t st);
// Fused TP: waits (bounded) until every rank's flag reaches this rank's epoch.
cudaError_t launch_tp_wait(const uint32_t* flags, uint32_t world, const uint32_t* epoch, int* status,
                           cudaStream_t st);
// Indexed decode of the same slabs to BF16 at args.out + slab dst (x, y,
// partials and counters unused).
cudaError_t launch_serial_tile_decode(const GemvArgs& args, cudaStream_t st);

// Tensor-core GEMM over decoded row groups (batch >= 16 path).
struct TcGroup {
  uint64_t a_off;   // byte offset of the group's BF16 rows [rows, cols] in the scratch
  uint64_t y_row0;  // first output row
  uint64_t xoff;    // first column of X (element offset into X^T rows)
  uint32_t rows, cols;
};
struct TcGemmArgs {
  const TcGroup* groups;
  const uint8_t* scratch;
  const void* xt;        // BF16 X^T [npad][xt_ld]
  uint64_t xt_ld;
  float* y;              // Y at batch column b0 (row stride ld)
  uint32_t ld, nb, npad, ksplit, tmem_cols;
  int* status;
};
size_t tc_gemm_smem_bytes(uint32_t npad);
// Converts X (FP32, [x_cols, ld] at column b0) to X^T BF16, zeroes Y rows when
// K is split, then runs the tensor-core GEMM: ngroups * ksplit CTAs.
cudaError_t launch_tc_gemm(const TcGemmArgs& args, uint32_t ngroups, const float* x, uint64_t x_cols,
                           cudaStream_t st);

// X (FP32, [cols, ld] from column 0 of the pass) to X^T BF16 [npad][xt_ld],
// zero for batch columns nb <= n < npad; and Y[rows of every group, 0..nb) = 0.
cudaError_t launch_xt_convert(const float* x, uint32_t ld, uint32_t nb, uint64_t cols, uint32_t npad, void* xt,
                              uint64_t xt_ld, cudaStream_t st);
cudaError_t launch_zero_rows(const TcGroup* groups, uint32_t ngroups, float* y, uint32_t ld, uint32_t nb,
                             cudaStream_t st);

// Fused decode -> tensor-core GEMM of indexed 16-row serial-codec slabs.  A
// group is up to 32 slabs reading the same X columns; a CTA runs one or more
// segments, each a range of one group's half tiles (8 rows x 16 columns).
struct FusedGroup {
  uint32_t m0;       // first member in the members array (slab indices)
  uint32_t nslabs;   // <= 32
  uint32_t tiles;    // cols / 16
  uint32_t pad;
  uint64_t xoff;     // X^T column of the group's column 0
};
struct FusedTask {  // one segment of a CTA's work
  uint32_t group, h0, h1, pad;  // half tiles [h0, h1) of the group (half h: rows 8 (h % 2).. of tile h / 2)
};
struct FusedArgs {
  const uint32_t* seg0;  // CTA c runs segments tasks[seg0[c] .. seg0[c + 1])
  const FusedTask* tasks;
  const FusedGroup* groups;
  const uint32_t* members;
  const Slab* slabs;
  const uint64_t* tbase;
  const uint32_t* tidx;
  const uint32_t* tmid;  // row-8 offsets of the tiles
  const void* tabs;      // per group: its lane tables (launch_fused_tables)
  const uint8_t* payload;
  const void* xt;        // BF16 X^T [npad][xt_ld]
  uint64_t xt_ld;
  float* y;              // Y at batch column b0 (row stride ld), rows zeroed
  uint32_t ld, nb, npad;
  int* status;
};
// Producer warps and dynamic shared memory for a batch pass of npad columns
// (16 <= npad <= 128, a multiple of 16); 0 producers when it does not fit.
uint32_t fused_producers(uint32_t npad, size_t* smem_bytes);
// Bytes of one group's lane tables, and their build (one warp per group, at
// index time; a codebook that does not fit sets the status word).
size_t fused_tables_bytes();
cudaError_t launch_fused_tables(const FusedGroup* groups, uint32_t ngroups, const uint32_t* members,
                                const Slab* slabs, const uint8_t* payload, void* tabs, int* status,
                                cudaStream_t st);
// The codebook of every slab fits the fused decoder's lane tables: ok[i] = 1.
cudaError_t launch_fused_check(const Slab* slabs, uint32_t n, const uint8_t* payload, uint8_t* ok,
                               cudaStream_t st);
// X (FP32 [x_cols, ld] at the pass's first column) to args.xt, zeroed Y rows
// of `groups`, then `nctas` fused CTAs (args.seg0 has nctas + 1 entries),
// launched to overlap the prep kernel: two launches.
cudaError_t launch_fused_gemm(const FusedArgs& args, uint32_t nctas, const float* x, uint64_t x_cols,
                              const TcGroup* groups, uint32_t ngroups, cudaStream_t st);

// SHA-256 (FIPS 180-4) of n ranges {offset, length} (device array of 2n u64)
// of d_base; 32-byte big-endian digests to d_digests.
cudaError_t launch_sha256(const uint64_t* d_ranges, uint32_t n, const uint8_t* d_base, uint8_t* d_digests,
                          cudaStream_t st);

}  // namespace xksv
