// xksv_cuda_decode_noalloc: batched decode that allocates no device memory.
//
// Some callers cannot let a library call cudaMalloc: serving stacks that
// reserve all of a GPU's memory up front for their own allocator (a library
// cudaMalloc then fails or fragments their pool), and code that must not hit
// cudaMalloc's implicit device-wide synchronisation in the middle of a
// latency-critical stream of work.  This entry point serves them: the caller
// passes device buffers for the payload and the output, and the only device
// memory the call uses besides those is a fixed, file-scope scratch array
// (the slab table and the status word), created when the library is loaded
// on a device and kept until the process exits.
//
// The first call on each device looks up that array's device address with
// cudaGetSymbolAddress (with the device current) and caches it for the life
// of the process; make that first call before any stream capture.  A
// cudaDeviceReset unloads the library's device code with the array, so the
// cached address is stale afterwards: a process that resets a device must
// not call this entry point on it again.  Every call shares the one array
// and overwrites it, so calls that overlap on the GPU (different streams, or
// other host threads) race on it: issue them one after another.
#include <mutex>

#include "kernels.h"
#include "xksv_cuda.h"

namespace xksv {
namespace {

constexpr size_t kNoallocStatusBytes = 256;  // status word, padded to the array's alignment
constexpr size_t kNoallocBytes = kNoallocStatusBytes + size_t(XKSV_NOALLOC_MAX_SLABS) * sizeof(Slab);

// Device scratch: [status int | pad to 256 B | Slab table (serial, parallel, raw)].
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoallocBytes];

constexpr int kMaxDev = 64;
std::mutex g_noalloc_mu;
unsigned char* g_noalloc_dev[kMaxDev] = {};  // device address of the array, per device
Slab g_noalloc_host[XKSV_NOALLOC_MAX_SLABS];  // host-side grouping buffer (guarded by the mutex)
int g_noalloc_status_host = 0;

}  // namespace
}  // namespace xksv

extern "C" int xksv_cuda_decode_noalloc(const xksv_slab* slabs, size_t n, const void* d_payload,
                                        size_t payload_size, void* d_out, size_t out_size, void* stream) {
  using namespace xksv;
  constexpr uint64_t kMax = ~uint64_t(0);
  if (n > size_t(XKSV_NOALLOC_MAX_SLABS)) return 2;  // beyond the scratch array
  if ((n && !slabs) || !d_payload || !d_out || (reinterpret_cast<uintptr_t>(d_out) & 1)) return 1;
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDev) return 1;
  if (!g_noalloc_dev[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || !p) return 1;
    g_noalloc_dev[dev] = static_cast<unsigned char*>(p);
  }
  unsigned char* base = g_noalloc_dev[dev];
  int* d_status = reinterpret_cast<int*>(base);
  Slab* d_tab = reinterpret_cast<Slab*>(base + kNoallocStatusBytes);
  // group by codec into the host buffer: serial | parallel | raw
  uint32_t counts[3] = {0, 0, 0};
  for (size_t i = 0; i < n; ++i) {
    const xksv_slab& s = slabs[i];
    if (s.flags || s.codec > XKSV_CODEC_PARALLEL32) return 1;
    if (s.codec != XKSV_CODEC_RAW && (s.dst_offset & 1)) return 1;  // BF16 stores need even offsets
    if (s.codec == XKSV_CODEC_TILE16 && (!s.rows || !s.cols || s.src_size < kHdr)) return 1;
    if (s.codec == XKSV_CODEC_PARALLEL32 && (!s.rows || s.rows > 16 || !s.cols || s.src_size < 32))
      return 1;
    // every slab inside the caller's buffers, checked before any launch
    if (s.src_offset > kMax - s.src_size || s.src_offset + s.src_size > payload_size) return 1;
    if (s.codec != XKSV_CODEC_RAW && s.cols > kMax / 2 / s.rows) return 1;
    const uint64_t dec = s.codec == XKSV_CODEC_RAW ? s.src_size : s.rows * s.cols * 2;
    if (s.dst_offset > kMax - dec || s.dst_offset + dec > out_size) return 1;
    ++counts[s.codec == XKSV_CODEC_TILE16 ? 0 : s.codec == XKSV_CODEC_PARALLEL32 ? 1 : 2];
  }
  uint32_t pos[3] = {0, counts[0], counts[0] + counts[1]};
  for (size_t i = 0; i < n; ++i) {
    const xksv_slab& s = slabs[i];
    const int k = s.codec == XKSV_CODEC_TILE16 ? 0 : s.codec == XKSV_CODEC_PARALLEL32 ? 1 : 2;
    g_noalloc_host[pos[k]++] = Slab{s.src_offset, s.src_size, s.rows, s.cols, s.dst_offset, s.x_offset};
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (n && cudaMemcpyAsync(d_tab, g_noalloc_host, n * sizeof(Slab), cudaMemcpyHostToDevice, st) != cudaSuccess)
    return 1;
  if (cudaMemsetAsync(d_status, 0, sizeof(int), st) != cudaSuccess) return 1;
  const uint8_t* pay = static_cast<const uint8_t*>(d_payload);
  uint8_t* out = static_cast<uint8_t*>(d_out);
  const int grid = 1 << 30;
  cudaError_t e = launch_serial_decode(d_tab, counts[0], pay, out, d_status, grid, st);
  if (e == cudaSuccess) e = launch_parallel_decode(d_tab + counts[0], counts[1], pay, out, d_status, grid, st);
  if (e == cudaSuccess) e = launch_raw_decode(d_tab + counts[0] + counts[1], counts[2], pay, out, grid, st);
  if (e != cudaSuccess) return 1;
  if (cudaMemcpyAsync(&g_noalloc_status_host, d_status, sizeof(int), cudaMemcpyDeviceToHost, st) != cudaSuccess)
    return 1;
  if (cudaStreamSynchronize(st) != cudaSuccess) return 1;
  return g_noalloc_status_host == 0 ? 0 : 1;
}
