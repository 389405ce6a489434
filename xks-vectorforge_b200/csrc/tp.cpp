// Tensor-parallel fused GEMV/GEMM: every rank (one process per GPU) holds the
// slabs of its own rows of W, computes its row shard of Y with the plan API,
// and one NCCL all-gather over NVLink assembles the full Y on every rank
// (row-major [rows, batch] shards concatenate in rank order).  K is not
// split, so no reduction is needed.
//
// NCCL is opened at run time (dlopen of libnccl.so.2, reusing a copy the
// process already loaded, e.g. PyTorch's), so the library has no link-time
// NCCL dependency and the rest of it works without NCCL installed.
#include <dlfcn.h>
#include <nccl.h>

#include <cstring>
#include <mutex>

#include "xksv_cuda.h"

namespace {

struct NcclApi {
  ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
  ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
  ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t,
                             cudaStream_t) = nullptr;
  bool ok = false;
};

const NcclApi& nccl() {
  static NcclApi api;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!h) return;
    api.get_unique_id = reinterpret_cast<decltype(api.get_unique_id)>(dlsym(h, "ncclGetUniqueId"));
    api.comm_init_rank = reinterpret_cast<decltype(api.comm_init_rank)>(dlsym(h, "ncclCommInitRank"));
    api.comm_destroy = reinterpret_cast<decltype(api.comm_destroy)>(dlsym(h, "ncclCommDestroy"));
    api.all_gather = reinterpret_cast<decltype(api.all_gather)>(dlsym(h, "ncclAllGather"));
    api.ok = api.get_unique_id && api.comm_init_rank && api.comm_destroy && api.all_gather;
  });
  return api;
}

static_assert(sizeof(ncclUniqueId) == XKSV_TP_ID_BYTES, "NCCL unique id size");

}  // namespace

extern "C" {

int xksv_tp_unique_id(void* id) {
  const NcclApi& n = nccl();
  if (!id || !n.ok) return 1;
  ncclUniqueId u;
  if (n.get_unique_id(&u) != ncclSuccess) return 1;
  std::memcpy(id, &u, sizeof(u));
  return 0;
}

int xksv_tp_comm_create(const void* id, int nranks, int rank, void** comm) {
  const NcclApi& n = nccl();
  if (!id || !comm || nranks < 1 || rank < 0 || rank >= nranks || !n.ok) return 1;
  *comm = nullptr;
  ncclUniqueId u;
  std::memcpy(&u, id, sizeof(u));
  ncclComm_t c = nullptr;
  if (n.comm_init_rank(&c, nranks, u, rank) != ncclSuccess) return 1;
  *comm = c;
  return 0;
}

void xksv_tp_comm_destroy(void* comm) {
  const NcclApi& n = nccl();
  if (comm && n.ok) n.comm_destroy(static_cast<ncclComm_t>(comm));
}

int xksv_tp_gemm(const xksv_plan* plan, const void* d_payload, size_t payload_size, const float* d_x,
                 size_t x_rows, float* d_y_shard, size_t rows_shard, float* d_y_full, size_t batch, void* comm,
                 void* stream) {
  const NcclApi& n = nccl();
  if (!plan || !d_y_shard || !d_y_full || !comm || !batch || !n.ok) return 1;
  // the shard's rows bound the plan's output rows (checked by the GEMM)
  if (xksv_plan_gemm(plan, d_payload, payload_size, d_x, x_rows, d_y_shard, rows_shard, batch, stream)) return 1;
  return n.all_gather(d_y_shard, d_y_full, rows_shard * batch, ncclFloat32,
                      static_cast<ncclComm_t>(comm), static_cast<cudaStream_t>(stream)) == ncclSuccess
             ? 0
             : 1;
}

}  // extern "C"
