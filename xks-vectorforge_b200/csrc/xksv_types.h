// Plan entry as stored on the device, and kernel status bits.
#pragma once
#include <cstdint>

namespace xksv {

// Serial block header: u64 count, u64 bit_count, u8 lengths[256].
constexpr uint32_t kHdr = 272;

// One block of a plan (device copy).  Mirrors the public xksv_slab, with the
// codec implied by which per-codec list the entry sits in.
struct Slab {
  uint64_t src;   // byte offset of the block in the payload
  uint64_t size;  // block bytes
  uint64_t rows;  // slab rows
  uint64_t cols;  // slab cols
  uint64_t dst;   // decode: byte offset in the output; GEMV/GEMM: first row of Y
  uint64_t xoff;  // GEMV/GEMM: element offset of column 0 in X
};

// Indexed GEMV work item: tiles [tile0, tile0 + ntiles) of slab `slab`
// (16-row slab, tile k = columns 16k..16k+15); the slab's items are
// first .. first + nitems - 1.
struct GemvItem {
  uint32_t slab, tile0, ntiles, first, nitems, pad0, pad1, pad2;
};

// Status bits OR-ed into the plan's device status word.
enum StatusBit : int {
  kStatusHeader = 1,    // malformed header / sizes / shape disagreement
  kStatusCodebook = 2,  // oversubscribed code lengths
  kStatusStream = 4,    // bad code, truncated stream, leftover bits, count mismatch
  kStatusInternal = 8,  // a limit of this implementation was exceeded
};

}  // namespace xksv
