/*
 * xksv_cuda.h -- C ABI of the B200 slab decoder (libxksv_cuda.so).
 *
 * Part 1 keeps the reference's GPU entry points: same names, signatures,
 * argument meaning and return codes, so ctypes callers of the reference
 * library (python/runtime.py:40-44, 251-255; python/tune.py:16-19) load this
 * library unchanged through XKSV_CUDA_LIBRARY.  `input` is a HOST pointer to
 * one encoded slab; `output`, `x` are DEVICE pointers on the current device.
 * Each call is synchronous and returns 0 on success, 1 on any failure
 * (null pointer, bad header or size, invalid codebook or bit stream, CUDA
 * error).  Outputs are written only through device kernels of this library.
 *
 * Part 2 adds a device-resident batched interface (no counterpart in the
 * reference): a plan describes many slabs of one payload buffer already in
 * device memory; decode / GEMV / GEMM are enqueued on a caller stream
 * without host synchronisation, and errors are collected in a device status
 * word read back by xksv_plan_status().
 */
#ifndef XKSV_CUDA_H
#define XKSV_CUDA_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---------------- Part 1: reference-compatible entry points ------------- */

/* Serial-codec ("bf16-huffman-tile16") slab -> BF16 row-major [rows, cols]
 * at output.  Replaces reference cuda/decode.cu:85-87 (validation :47-66). */
int xksv_cuda_decode(const void* input, size_t size, size_t rows, size_t cols, void* output);

/* Serial-codec slab fused with y = W x: x is FP32 [cols], output FP32 [rows]
 * (overwritten).  Replaces reference cuda/decode.cu:89-92. */
int xksv_cuda_gemv(const void* input, size_t size, size_t rows, size_t cols, const float* x,
                   float* output);

/* Serial-codec slab fused with Y = W X: x is FP32 row-major [cols, batch],
 * output FP32 row-major [rows, batch] (overwritten).  Replaces reference
 * cuda/decode.cu:94-98. */
int xksv_cuda_gemm(const void* input, size_t size, size_t rows, size_t cols, size_t batch,
                   const float* x, float* output);

/* Parallel-codec ("bf16-huffman-parallel32", XKSP2) slab -> BF16 row-major
 * [rows, cols] (dimensions read from the slab header).  Replaces reference
 * cuda/parallel.cu:68-70 (validation :33-53). */
int xksv_cuda_decode_parallel(const void* input, size_t n, void* output);

/* Parallel-codec slab fused with y = W x, x FP32 [cols], output FP32 [rows]
 * (overwritten).  Replaces reference cuda/parallel.cu:71-74. */
int xksv_cuda_gemv_parallel(const void* input, size_t n, const float* x, float* output);

/* ---------------- Part 2: batched, device-resident interface ------------ */

enum {
  XKSV_CODEC_RAW = 0,        /* block stores the source bytes unchanged */
  XKSV_CODEC_TILE16 = 1,     /* "bf16-huffman-tile16" (serial codec) */
  XKSV_CODEC_PARALLEL32 = 2  /* "bf16-huffman-parallel32" (XKSP2) */
};

/* One archive block, as listed in the archive index (src/compile.cpp:459-470):
 * where its bytes sit in the payload buffer, its slab shape, and where its
 * result goes.  For decode, dst_offset is a byte offset into the output.
 * For GEMV/GEMM, dst_offset is the first output row and x_offset the element
 * offset of this slab's column 0 inside x (so one plan can serve several
 * weight matrices).  Raw blocks used by GEMV/GEMM must give rows and cols
 * (BF16 row-major data); raw blocks used by decode only need src_size. */
typedef struct xksv_slab {
  uint64_t src_offset;
  uint64_t src_size;
  uint64_t rows;
  uint64_t cols;
  uint64_t dst_offset;
  uint64_t x_offset;
  uint32_t codec;
  uint32_t flags; /* must be 0 */
} xksv_slab;

typedef struct xksv_plan xksv_plan;

/* Validates the host table, copies it to the current device and groups it by
 * codec.  Returns 0 and a plan, or 1.  The plan records the extents its
 * table needs: payload bytes (largest src_offset + src_size), decoded bytes
 * (largest dst_offset + rows * cols * 2, or + src_size for raw blocks), X rows
 * (largest x_offset + cols) and Y rows (largest dst_offset + rows).  Every call
 * below is given the size of each device buffer it reads or writes and
 * returns 1 without launching anything when a slab lies outside one: a bad
 * table entry never reaches a kernel as an out-of-bounds access. */
int xksv_plan_create(const xksv_slab* slabs, size_t n, xksv_plan** plan);
void xksv_plan_destroy(xksv_plan* plan);

/* Enqueues decode of every slab of the plan from d_payload (device,
 * payload_size bytes) into d_out (device, out_size bytes) on `stream` (a
 * cudaStream_t; NULL = legacy default stream).  Returns 1 for launch errors
 * and, without launching, when a slab lies outside either buffer or when
 * d_out or a coded slab's dst_offset is odd (BF16 words need 2-byte
 * alignment); stream errors are found by xksv_plan_status(). */
int xksv_plan_decode(const xksv_plan* plan, const void* d_payload, size_t payload_size, void* d_out,
                     size_t out_size, void* stream);

/* The same decode from a HOST payload (pinned memory for overlap): the first
 * payload_size bytes at h_payload are copied into d_payload (device, at least
 * as large) in 8 pieces on a plan-owned stream while the slabs of each piece
 * that has landed are decoded on `stream`, so the copy and the decode
 * overlap.  The copies wait for work already enqueued on `stream`.  Needs
 * each codec's slabs in increasing payload order (an archive's block order;
 * otherwise, and for a plan indexed on d_payload, it copies once and then
 * decodes).  Returns 1 as xksv_plan_decode does (a slab past payload_size or
 * past out_size included).  No reference counterpart (the reference stages
 * one slab per blocking call, cuda/decode.cu:47-83). */
int xksv_plan_decode_host(const xksv_plan* plan, const void* h_payload, size_t payload_size,
                          void* d_payload, void* d_out, size_t out_size, void* stream);

/* Enqueues Y[dst_offset + r, b] = sum_c W[r, c] * X[x_offset + c, b] for every
 * slab, X FP32 row-major [x_rows, batch] and Y FP32 row-major [y_rows, batch]
 * (rows of Y not covered by a slab are left untouched).  Returns 1 without
 * launching when a slab lies outside the payload, X or Y. */
int xksv_plan_gemm(const xksv_plan* plan, const void* d_payload, size_t payload_size, const float* d_x,
                   size_t x_rows, float* d_y, size_t y_rows, size_t batch, void* stream);

/* The tensor-core path (batch >= 4) decodes the plan's weights into a BF16
 * scratch before its GEMM; by default each plan allocates its own on first
 * use and keeps it, i.e. a decoded copy of its weights.  Plans whose calls
 * are serialised on one stream can share one caller-owned scratch instead:
 * xksv_plan_scratch_bytes gives the bytes a plan needs (0 when it has no
 * tensor-core path) and xksv_plan_set_scratch lends it a device buffer of at
 * least that size, 256-byte aligned (the plan's own scratch, if any, is
 * freed; NULL returns to an own scratch).  Returns 1 for a buffer too small
 * or misaligned.  The caller keeps the buffer alive while the plan uses it. */
size_t xksv_plan_scratch_bytes(const xksv_plan* plan);
int xksv_plan_set_scratch(xksv_plan* plan, void* d_scratch, size_t bytes);

/* Tensor-core routing of xksv_plan_gemm for 4 <= batch <= 128 on a plan
 * indexed for the payload (xksv_plan_index) whose slabs are all 16-row
 * serial-codec slabs: XKSV_GEMM_FUSED decodes each tile row straight into
 * the shared-memory operand stages of the tensor-core MMAs (one kernel, no
 * decoded weight written to memory); XKSV_GEMM_SCRATCH decodes into the BF16
 * scratch and runs the tensor-core GEMM on it (also the route for larger
 * batches and other plans); XKSV_GEMM_AUTO (the default) picks the fused
 * kernel wherever it applies.  Returns 1 for an unknown route. */
enum { XKSV_GEMM_AUTO = 0, XKSV_GEMM_SCRATCH = 1, XKSV_GEMM_FUSED = 2 };
int xksv_plan_set_gemm_route(xksv_plan* plan, int route);
/* 1 when the fused route applies to this plan and payload (after
 * xksv_plan_index), else 0. */
int xksv_plan_fused_ready(const xksv_plan* plan, const void* d_payload);

/* Synchronises `stream`, returns 0 when no slab reported an error since the
 * last call (then clears the word), else 1. */
int xksv_plan_status(const xksv_plan* plan, void* stream);

/* Number of kernel launches the last xksv_plan_decode / xksv_plan_gemm call
 * enqueued (for accounting in benchmarks). */
int xksv_plan_launches(const xksv_plan* plan);

/* Builds the plan's tile index for resident weights: one decode pass over
 * the plan's 16-row serial-codec slabs with cols % 16 == 0 records the bit
 * offsets at which every 16x16 tile's codes and its row 8 start (8 bytes per
 * tile) and each slab's decode tables (5920 bytes per slab), all kept on the
 * device with the plan.  Afterwards xksv_plan_gemm and xksv_plan_decode with
 * the same d_payload pointer decode those slabs tile-parallel (one or two
 * threads per tile) instead of re-synchronising each slab's single bit
 * stream on every call.
 * The index describes the payload's contents at this call: rebuild it if they
 * change.  No reference counterpart (the reference decodes every slab from
 * its first bit, cuda/decode.cu:12-45); it is an acceleration structure on
 * the side, the slab format is unchanged.  Synchronises `stream`; 0 on
 * success, 1 on a bad slab or CUDA error (no index is kept then).  Calls on
 * one plan must not overlap. */
int xksv_plan_index(xksv_plan* plan, const void* d_payload, size_t payload_size, void* stream);


/* ---------------- Part 3: archive-side encoder (host CPU) --------------- */
/* The compile step that produces slabs for the decoder; byte-identical to the
 * reference's xksv_pack (codec XKSV_CODEC_TILE16, src/c_api.cpp:18-28) and
 * xksv_pack_parallel (XKSV_CODEC_PARALLEL32, src/c_api.cpp:44-65): same
 * argument checks, 0 on success and 1 on failure (the reference returns -1),
 * output malloc'd and released with xksv_host_free. */
int xksv_host_pack(const void* data, size_t n, size_t rows, size_t cols, int codec, void** out,
                   size_t* out_size);
void xksv_host_free(void* p);

/* Splits a row-major BF16 [rows, cols] tensor into the compiler's slabs
 * (whole rows, at most 16 rows and 1 MiB each: src/compile.cpp:449-479),
 * encodes them on `threads` host threads (0 = all cores), keeps an encoding
 * only when smaller than the raw bytes (src/compile.cpp:268-275), and returns
 * the concatenated payload plus one xksv_slab per slab (dst_offset =
 * dst_base + the slab's byte offset in the tensor).  Both outputs are
 * malloc'd; release them with xksv_host_free. */
int xksv_host_pack_tensor(const void* data, size_t nbytes, size_t rows, size_t cols, int codec,
                          int threads, uint64_t dst_base, void** payload, size_t* payload_size,
                          xksv_slab** table, size_t* nslabs);

/* GPU encoder: the slabs of xksv_host_pack_tensor, byte-identical, built on
 * the current device from a row-major BF16 [rows, cols] tensor in device
 * memory (histograms, Huffman lengths with the reference's tie order,
 * canonical codes and bit packing in kernels; src/compile.cpp:247-285,
 * 449-479, src/c_api.cpp:18-28, 44-65, src/codec.cpp:32-58).  *d_payload is
 * device memory allocated by the library (release with xksv_cuda_free), the
 * slab table host memory as for xksv_host_pack_tensor.  Synchronises
 * `stream`; 0 on success, 1 on bad arguments, a CUDA error, or a code longer
 * than 32 bits (not produced for the compiler's <= 1 MiB slabs). */
int xksv_cuda_pack_tensor(const void* d_data, size_t rows, size_t cols, int codec, uint64_t dst_base,
                          void** d_payload, size_t* payload_size, xksv_slab** table, size_t* nslabs,
                          void* stream);
void xksv_cuda_free(void* d_ptr);

/* ---------------- Part 4: decode without device allocation -------------- */
/* No counterpart in the reference.  For callers that cannot let a library
 * allocate device memory -- a server that has reserved the whole GPU for its
 * own allocator, or code that cannot afford cudaMalloc's implicit
 * device-wide synchronisation.  Decodes the n slabs of `slabs` (host array,
 * same fields as for xksv_plan_create) from d_payload into d_out (both device
 * buffers owned by the caller) on `stream`, then waits for the stream and
 * returns 0 on success, 1 on a bad table entry (a slab outside the
 * payload_size bytes at d_payload or the out_size bytes at d_out included,
 * found before any launch), a launch error or a slab that fails to decode,
 * and 2 when n exceeds XKSV_NOALLOC_MAX_SLABS.
 * Besides the caller's buffers it uses only a fixed scratch array compiled
 * into the library (the slab table and a status word, about 192 KiB on every
 * GPU that loads the library, kept until the process exits).  The first call
 * on a device looks that array up (cudaGetSymbolAddress) and keeps its
 * address: make it before any stream capture, and make no call on a device
 * after a cudaDeviceReset of it (the address is stale then).  All calls
 * share the array: calls that overlap on the GPU race, so issue them one at
 * a time. */
#define XKSV_NOALLOC_MAX_SLABS 4096
int xksv_cuda_decode_noalloc(const xksv_slab* slabs, size_t n, const void* d_payload, size_t payload_size,
                             void* d_out, size_t out_size, void* stream);

/* Fused variant: no separate collective.  The indexed GEMV kernel writes its
 * output rows into this rank's block of its own gathered buffer; the grid's
 * last CTA copies the block into every other rank's buffer (CUDA IPC peer
 * mappings, stores over NVLink), fences once and raises this rank's flag on
 * every rank; a one-warp kernel on each rank then waits (bounded, about a
 * second; an error bit in the plan's status word after that) until all
 * ranks' flags reach this call.  Plain peer stores only, no multicast.  The
 * gathered buffers alternate between two halves on successive calls, so a
 * result stays valid until the call after next on any rank. */
#define XKSV_TP_IPC_BYTES 64
typedef struct xksv_tp_fused xksv_tp_fused;

/* Allocates this rank's gathered buffers (2 x nranks * max_rows_shard *
 * max_batch floats, max_batch <= 4) and flags on the current device and
 * returns its IPC handle (XKSV_TP_IPC_BYTES) for the other ranks.  0 or 1. */
int xksv_tp_fused_create(int nranks, int rank, size_t max_rows_shard, size_t max_batch, xksv_tp_fused** ctx,
                         void* ipc_handle);
/* Opens the peers' buffers: handles = every rank's handle, in rank order. */
int xksv_tp_fused_open(xksv_tp_fused* ctx, const void* handles);
/* Enqueues the fused GEMV/GEMM (batch <= max_batch) of this rank's plan,
 * which must hold only 16-row serial-codec slabs with a tile index for
 * d_payload (xksv_plan_index) and write no row at or past rows_shard.  X is
 * FP32 [x_rows, batch].  The gathered Y [nranks * rows_shard, batch] (rank
 * order) is copied to d_y_full when it is not NULL, and its address in the
 * context's buffers is stored to *d_gathered when that is not NULL.
 * Collective: every rank makes the same calls in the same order.  1 for bad
 * arguments (a slab outside the payload, X or the rank's rows included) or
 * launch errors. */
int xksv_tp_fused_gemm(xksv_tp_fused* ctx, const xksv_plan* plan, const void* d_payload, size_t payload_size,
                       const float* d_x, size_t x_rows, size_t rows_shard, size_t batch, float* d_y_full,
                       float** d_gathered, void* stream);
void xksv_tp_fused_destroy(xksv_tp_fused* ctx);

/* ---------------- Part 6: SHA-256 of decoded bytes on the GPU ----------- */
/* The archive index stores the SHA-256 of every block's and tensor's decoded
 * BF16 bytes (reference src/compile.cpp:255, 483; checked after decoding in
 * src/verify.cpp:262-273 on the CPU).  These compute FIPS 180-4 SHA-256 on
 * the device, so decoded weights are verified without copying them back.
 * No reference counterpart.  Enqueued on `stream`; 0 on success, 1 on bad
 * arguments or a CUDA error. */

/* n ranges of device memory at d_base: ranges[2i] = byte offset,
 * ranges[2i + 1] = length (a HOST array); 32-byte digests to d_digests
 * (device, n * 32 bytes). */
int xksv_cuda_sha256(const uint64_t* ranges, size_t n, const void* d_base, void* d_digests, void* stream);

/* Digest i (slab order of xksv_plan_create) = SHA-256 of slab i's decoded
 * bytes in d_out (out_size bytes): [dst_offset, dst_offset + rows * cols * 2),
 * or src_size bytes for a raw slab. */
int xksv_plan_sha256(const xksv_plan* plan, const void* d_out, size_t out_size, void* d_digests, void* stream);

/* ---------------- Part 5: tensor-parallel fused GEMV / GEMM ------------- */
/* One process per GPU; each rank's plan holds the slabs of its own rows
 * [g*R/G, (g+1)*R/G) of W with dst_offset rebased to the shard's first row.
 * No reference counterpart (the reference has no multi-GPU path); the NCCL
 * library is opened at run time (libnccl.so.2, reusing an already loaded
 * copy), so these return 1 when it is absent. */
#define XKSV_TP_ID_BYTES 128

/* A fresh NCCL unique id (XKSV_TP_ID_BYTES bytes) for xksv_tp_comm_create:
 * made by one rank and sent to the others by the caller. 0 or 1. */
int xksv_tp_unique_id(void* id);

/* Collective over nranks processes: creates this rank's communicator on the
 * current CUDA device.  0 or 1. */
int xksv_tp_comm_create(const void* id, int nranks, int rank, void** comm);
void xksv_tp_comm_destroy(void* comm);

/* Enqueues on `stream`: d_y_shard[rows_shard, batch] = W_shard X (the fused
 * plan GEMM, X FP32 [x_rows, batch]), then one all-gather of every rank's
 * shard into d_y_full[nranks * rows_shard, batch] (rank order = row order;
 * all ranks pass the same rows_shard).  Returns 1 for launch errors and,
 * without launching, for a slab outside the payload, X or the shard's rows;
 * slab errors are read with xksv_plan_status. */
int xksv_tp_gemm(const xksv_plan* plan, const void* d_payload, size_t payload_size, const float* d_x,
                 size_t x_rows, float* d_y_shard, size_t rows_shard, float* d_y_full, size_t batch, void* comm,
                 void* stream);

#ifdef __cplusplus
}
#endif
#endif /* XKSV_CUDA_H */
