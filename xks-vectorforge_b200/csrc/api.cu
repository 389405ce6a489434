// C ABI of libxksv_cuda.so (declared in include/xksv_cuda.h).
//
// The five reference entry points keep the reference's validation order and
// 0/1 return contract (cuda/decode.cu:47-98, cuda/parallel.cu:33-74).  Unlike
// the reference they do not cudaMalloc/cudaFree per call: each device keeps a
// growable staging buffer, a one-entry slab table and a status word, guarded
// by a mutex (calls stay synchronous on the legacy default stream, like the
// reference).  The batched plan interface enqueues work on a caller stream.
#include <algorithm>
#include <cstring>
#include <limits>
#include <map>
#include <mutex>
#include <queue>
#include <vector>

#include "xksv_cuda.h"
#include "kernels.h"

namespace xksv {
namespace {

constexpr size_t kMaxDevices = 64;
constexpr uint64_t kMax = std::numeric_limits<uint64_t>::max();

uint64_t get64(const uint8_t* p) {
  uint64_t v = 0;
  for (int i = 0; i < 8; ++i) v |= uint64_t(p[i]) << (8 * i);
  return v;
}

// Canonical assignment succeeds iff the Kraft sum of the lengths is <= 1
// (src/codec.cpp:11-29 / cuda/decode.cu:52-66 fail exactly on carry-out).
bool lengths_ok(const uint8_t* lens) {
  uint32_t cnt[256] = {0};
  int maxlen = 0;
  for (int s = 0; s < 256; ++s)
    if (lens[s]) {
      ++cnt[lens[s]];
      maxlen = std::max(maxlen, int(lens[s]));
    }
  int64_t avail = 1;
  for (int l = 1; l <= maxlen; ++l) {
    avail = 2 * avail - cnt[l];
    if (avail < 0) return false;
    avail = std::min<int64_t>(avail, 4096);
  }
  return true;
}

// cuda/decode.cu:49-66 for a host slab.
bool serial_header_ok(const uint8_t* p, size_t size, size_t rows, size_t cols, size_t batch) {
  if (!p || size < kHdr || !rows || !cols || !batch || cols > kMax / rows || batch > kMax / rows ||
      batch > kMax / cols)
    return false;
  uint64_t n = get64(p), nbits = get64(p + 8);
  if (n != uint64_t(rows) * cols || n > size - kHdr || nbits / 8 + (nbits % 8 != 0) != size - kHdr - n)
    return false;
  return lengths_ok(p + 16);
}

// cuda/parallel.cu:34-53 for a host slab; returns rows/cols.
bool parallel_header_ok(const uint8_t* p, size_t n, uint64_t* rows_out, uint64_t* cols_out) {
  if (!p || n < 32 || std::memcmp(p, "XKSP2\0\0\0", 8)) return false;
  uint64_t rows = get64(p + 8), cols = get64(p + 16), count = get64(p + 24);
  if (!rows || rows > 16 || !cols || !count || count > 32 || cols > kMax / rows ||
      count > rows * cols || rows * cols > n || rows * cols > kMax / 32 || n < 32 + 8 * count)
    return false;
  size_t pos = 32 + 8 * count;
  for (uint64_t k = 0; k < count; ++k) {
    uint64_t len = get64(p + 32 + 8 * k);
    if (len < kHdr || len > n - pos) return false;
    uint64_t elements = get64(p + pos), bits = get64(p + pos + 8);
    uint64_t start = rows * cols * k / count;
    if (elements != rows * cols * (k + 1) / count - start || elements > len - kHdr ||
        bits / 8 + (bits % 8 != 0) != len - kHdr - elements)
      return false;
    if (!lengths_ok(p + pos + 16)) return false;
    pos += len;
  }
  if (pos != n) return false;
  *rows_out = rows;
  *cols_out = cols;
  return true;
}

struct DevCtx {
  std::mutex mu;
  bool init = false;
  uint8_t* stage = nullptr;
  size_t cap = 0;
  Slab* d_slab = nullptr;
  int* d_status = nullptr;
  int* h_status = nullptr;  // pinned
  int sms = 148;
};
DevCtx g_ctx[kMaxDevices];

DevCtx* ctx_current() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || size_t(dev) >= kMaxDevices) return nullptr;
  DevCtx& c = g_ctx[dev];
  if (!c.init) {
    if (cudaMalloc(&c.d_slab, sizeof(Slab)) != cudaSuccess) return nullptr;
    if (cudaMalloc(&c.d_status, sizeof(int)) != cudaSuccess) return nullptr;
    if (cudaMallocHost(&c.h_status, sizeof(int)) != cudaSuccess) return nullptr;
    cudaDeviceGetAttribute(&c.sms, cudaDevAttrMultiProcessorCount, dev);
    c.init = true;
  }
  return &c;
}

bool is_device_ptr(const void* p) {
  cudaPointerAttributes a;
  if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  return a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged;
}

enum class Kind { Serial, Parallel };

// Stages one slab, launches the kernel on the legacy default stream, and
// returns the reference's 0/1 result.
int run_single(Kind kind, const void* input, size_t size, uint64_t rows, uint64_t cols,
               void* output, const float* x, size_t batch, bool gemm) {
  DevCtx* c = ctx_current();
  if (!c) return 1;
  std::lock_guard<std::mutex> lock(c->mu);
  cudaStream_t st = 0;
  const uint8_t* payload;
  if (is_device_ptr(input)) {
    payload = static_cast<const uint8_t*>(input);
  } else {
    if (size > c->cap) {
      if (c->stage) cudaFree(c->stage);
      size_t cap = std::max<size_t>(size + 64, c->cap * 2);
      if (cudaMalloc(&c->stage, cap) != cudaSuccess) {
        c->stage = nullptr;
        c->cap = 0;
        return 1;
      }
      c->cap = cap;
    }
    if (cudaMemcpyAsync(c->stage, input, size, cudaMemcpyHostToDevice, st) != cudaSuccess) return 1;
    payload = c->stage;
  }
  Slab s{0, size, rows, cols, 0, 0};
  if (cudaMemcpyAsync(c->d_slab, &s, sizeof(Slab), cudaMemcpyHostToDevice, st) != cudaSuccess) return 1;
  if (cudaMemsetAsync(c->d_status, 0, sizeof(int), st) != cudaSuccess) return 1;
  cudaError_t e = cudaSuccess;
  if (!gemm) {
    e = kind == Kind::Serial
            ? launch_serial_decode(c->d_slab, 1, payload, static_cast<uint8_t*>(output), c->d_status, 1, st)
            : launch_parallel_decode(c->d_slab, 1, payload, static_cast<uint8_t*>(output), c->d_status, 1, st);
  } else {
    float* y = static_cast<float*>(output);
    for (size_t b0 = 0; b0 < batch && e == cudaSuccess; b0 += 8) {
      uint32_t nb = uint32_t(std::min<size_t>(8, batch - b0));
      e = kind == Kind::Serial
              ? launch_serial_gemm(c->d_slab, 1, payload, x, y, uint32_t(batch), uint32_t(b0), nb, c->d_status, 1, st)
              : launch_parallel_gemm(c->d_slab, 1, payload, x, y, uint32_t(batch), uint32_t(b0), nb, c->d_status, 1, st);
    }
  }
  if (e != cudaSuccess) return 1;
  if (cudaMemcpyAsync(c->h_status, c->d_status, sizeof(int), cudaMemcpyDeviceToHost, st) != cudaSuccess) return 1;
  if (cudaStreamSynchronize(st) != cudaSuccess) return 1;
  return *c->h_status == 0 ? 0 : 1;
}

}  // namespace
}  // namespace xksv

struct xksv_plan {
  int device = 0;
  xksv::Slab* d_slabs = nullptr;  // [serial | parallel | raw]
  uint32_t n_ser = 0, n_par = 0, n_raw = 0;
  bool raw_gemm_ok = true;
  bool odd_dst = false;  // a coded slab with an odd byte offset: decode refused
  // buffer extents the slab table needs, checked against the sizes every call
  // is given before anything is launched: payload bytes (max src end),
  // decoded bytes (max dst end, decode and SHA-256), X rows (max x_offset +
  // cols) and Y rows (max dst_offset + rows) of GEMV/GEMM
  uint64_t need_payload = 0, need_out = 0, need_x_rows = 0, need_y_rows = 0;
  int* d_status = nullptr;
  int* h_status = nullptr;
  int grid_ser = 148, grid_par = 148, grid_raw = 148;
  int launches = 0;
  // tile index (xksv_plan_index): the first n_ser_idx serial slabs are
  // 16-row slabs with cols % 16 == 0
  uint32_t n_ser_idx = 0;
  std::vector<xksv::Slab> h_slabs;  // host copy of d_slabs
  const void* indexed_payload = nullptr;
  uint32_t* d_tidx = nullptr;
  uint32_t* d_tmid = nullptr;  // row-8 offsets of the tiles (fused GEMM work split)
  xksv::GemvTabs* d_gtabs = nullptr;  // per indexed slab: the tile GEMV kernel's tables
  uint64_t* d_tbase = nullptr;
  xksv::GemvItem* d_items = nullptr;
  uint32_t n_items = 0;
  float* d_partials = nullptr;
  uint32_t* d_counters = nullptr;
  // tensor-core GEMM path (batch >= 16): the plan's slabs decoded into BF16
  // row groups of <= 128 rows in a scratch buffer, then tcgen05 GEMM
  bool tc_ok = false;
  uint32_t ngroups = 0, tc_ksplit = 1;
  xksv::TcGroup* d_groups = nullptr;
  xksv::Slab* d_tc_slabs = nullptr;  // d_slabs with dst = scratch byte offsets
  uint64_t scratch_bytes = 0, x_cols = 0, x_base = 0;  // X rows [x_base, x_base + x_cols)
  uint8_t* d_scratch = nullptr;
  bool scratch_owned = true;  // false: lent by the caller (xksv_plan_set_scratch)
  void* d_xt = nullptr;  // BF16 X^T [256][x_cols] of X rows from x_base
  // fused decode -> tensor-core GEMM (xksv_plan_index of an all-serial,
  // all-indexable plan whose codebooks fit the fused decoder)
  bool fused_ok = false;
  int gemm_route = 0;  // XKSV_GEMM_*
  uint32_t n_fctas = 0;
  uint32_t* d_fseg0 = nullptr;  // CTA c's segments: d_ftasks[d_fseg0[c] .. d_fseg0[c + 1])
  xksv::FusedTask* d_ftasks = nullptr;
  xksv::FusedGroup* d_fgroups = nullptr;
  uint32_t* d_fmembers = nullptr;
  void* d_ftabs = nullptr;  // per group: its lane tables, built with the index
  uint64_t* d_hash_ranges = nullptr;  // per slab in creation order: {dst, decoded bytes}
  // xksv_plan_decode_host: copy stream and per-chunk events (created on first use)
  cudaStream_t copy_st = nullptr;
  cudaEvent_t chunk_ev[9] = {};
};

namespace {
void free_index(xksv_plan* p) {
  if (p->d_tidx) cudaFree(p->d_tidx);
  if (p->d_tmid) cudaFree(p->d_tmid);
  if (p->d_gtabs) cudaFree(p->d_gtabs);
  if (p->d_tbase) cudaFree(p->d_tbase);
  if (p->d_items) cudaFree(p->d_items);
  if (p->d_partials) cudaFree(p->d_partials);
  if (p->d_counters) cudaFree(p->d_counters);
  if (p->d_fseg0) cudaFree(p->d_fseg0);
  if (p->d_ftasks) cudaFree(p->d_ftasks);
  if (p->d_fgroups) cudaFree(p->d_fgroups);
  if (p->d_fmembers) cudaFree(p->d_fmembers);
  if (p->d_ftabs) cudaFree(p->d_ftabs);
  p->d_ftabs = nullptr;
  p->d_fseg0 = nullptr;
  p->d_ftasks = nullptr;
  p->d_fgroups = nullptr;
  p->d_fmembers = nullptr;
  p->n_fctas = 0;
  p->fused_ok = false;
  p->d_tidx = nullptr;
  p->d_tmid = nullptr;
  p->d_gtabs = nullptr;
  p->d_tbase = nullptr;
  p->d_items = nullptr;
  p->d_partials = nullptr;
  p->d_counters = nullptr;
  p->n_items = 0;
  p->indexed_payload = nullptr;
}

bool tile_indexable(const xksv::Slab& s) {
  return s.rows == 16 && s.cols % 16 == 0 && s.cols < (1ull << 27);
}

// Row groups for the tensor-core GEMM: slabs sharing X columns (x_offset,
// cols) whose output rows are contiguous, up to 128 rows per group; fills
// the scratch slab table (same order as `all`).  The X columns the plan reads
// are [x_base, x_base + x_cols); groups hold offsets relative to x_base.
// False when a slab is not 16-byte aligned for cp.async (cols or x_offset not
// a multiple of 8).
bool build_tc_groups(const std::vector<xksv::Slab>& all, std::vector<xksv::TcGroup>& groups,
                     std::vector<xksv::Slab>& tc_slabs, uint64_t& scratch, uint64_t& x_cols,
                     uint64_t& x_base) {
  using xksv::Slab;
  const size_t n = all.size();
  if (!n) return false;
  for (const Slab& s : all)
    if (s.cols % 8 || s.xoff % 8 || !s.rows || s.rows > 128 || s.cols >= (1u << 31)) return false;
  std::vector<size_t> idx(n);
  for (size_t i = 0; i < n; ++i) idx[i] = i;
  std::sort(idx.begin(), idx.end(), [&](size_t a, size_t b) {
    const Slab &x = all[a], &y = all[b];
    if (x.xoff != y.xoff) return x.xoff < y.xoff;
    if (x.cols != y.cols) return x.cols < y.cols;
    return x.dst < y.dst;
  });
  tc_slabs = all;
  scratch = 0;
  x_base = ~uint64_t(0);
  for (const Slab& s : all) x_base = std::min(x_base, s.xoff);
  x_cols = 0;
  xksv::TcGroup cur{};
  bool open = false;
  for (size_t k = 0; k < n; ++k) {
    const Slab& s = all[idx[k]];
    x_cols = std::max<uint64_t>(x_cols, s.xoff + s.cols - x_base);
    const bool extend = open && s.xoff - x_base == cur.xoff && s.cols == cur.cols &&
                        s.dst == cur.y_row0 + cur.rows && cur.rows + s.rows <= 128;
    if (!extend) {
      if (open) groups.push_back(cur);
      cur = xksv::TcGroup{scratch, s.dst, s.xoff - x_base, 0, uint32_t(s.cols)};
      open = true;
    }
    tc_slabs[idx[k]].dst = cur.a_off + uint64_t(cur.rows) * s.cols * 2;
    cur.rows += uint32_t(s.rows);
    scratch += s.rows * s.cols * 2;
  }
  groups.push_back(cur);
  return true;
}
// Fused-GEMM groups and CTA work: slabs reading the same X columns
// (x_offset, cols) in groups of up to 32 (one slab per lane).  The work unit
// is a half tile of a group (8 rows x 16 columns of all its slabs; the same
// instruction count whatever the group's slab count, since a warp issues for
// all its lanes).  A CTA's producer warps share each of its segments (one
// group's run of half tiles), so a CTA's time follows the sum over its
// segments of the largest warp share plus a start-up per segment (stream
// starts, length staging, table build: measured about half a unit).  Two
// schedules are built and the one whose slowest CTA is cheaper is kept:
//   * by group: every group gets one CTA, then the group whose CTAs carry
//     the most half tiles gets another, until there are `sms` CTAs;
//   * equal shares: the groups' units in order cut into `sms` equal ranges,
//     a range that crosses a group boundary becoming several segments.
// seg0[c] .. seg0[c + 1] are CTA c's segments.  X columns are relative to
// x_base.
void build_fused(const std::vector<xksv::Slab>& all, uint64_t x_base, int sms, uint32_t warps,
                 std::vector<xksv::FusedGroup>& groups, std::vector<uint32_t>& members,
                 std::vector<xksv::FusedTask>& segs, std::vector<uint32_t>& seg0) {
  std::map<std::pair<uint64_t, uint64_t>, std::vector<uint32_t>> by_x;
  std::vector<std::pair<uint64_t, uint64_t>> order;
  for (uint32_t i = 0; i < all.size(); ++i) {
    const auto key = std::make_pair(all[i].xoff, all[i].cols);
    auto it = by_x.find(key);
    if (it == by_x.end()) {
      order.push_back(key);
      it = by_x.emplace(key, std::vector<uint32_t>()).first;
    }
    it->second.push_back(i);
  }
  for (const auto& key : order) {
    const std::vector<uint32_t>& v = by_x[key];
    for (size_t k = 0; k < v.size(); k += 32) {
      xksv::FusedGroup g{};
      g.m0 = uint32_t(members.size());
      g.nslabs = uint32_t(std::min<size_t>(32, v.size() - k));
      g.tiles = uint32_t(key.second / 16);
      g.xoff = key.first - x_base;
      members.insert(members.end(), v.begin() + k, v.begin() + k + g.nslabs);
      groups.push_back(g);
    }
  }
  const size_t ng = groups.size();
  auto units = [&](size_t g) { return 2 * uint64_t(groups[g].tiles); };
  using Sched = std::pair<std::vector<xksv::FusedTask>, std::vector<uint32_t>>;
  // cost of a schedule in units: the slowest CTA's segments, each its
  // largest warp share + a start-up of half a unit
  auto cost = [&](const Sched& sc) {
    double worst = 0;
    for (size_t c = 0; c + 1 < sc.second.size(); ++c) {
      double t = 0;
      for (uint32_t i = sc.second[c]; i < sc.second[c + 1]; ++i)
        t += double((sc.first[i].h1 - sc.first[i].h0 + warps - 1) / warps) + 0.5;
      worst = std::max(worst, t);
    }
    return worst;
  };
  Sched by_group, shares;
  {
    std::vector<uint32_t> parts(ng, 1);
    auto load = [&](size_t g) { return (units(g) + parts[g] - 1) / parts[g]; };
    std::priority_queue<std::pair<uint64_t, size_t>> q;  // (half tiles per CTA, group)
    for (size_t g = 0; g < ng; ++g) q.emplace(load(g), g);
    size_t total = ng;
    while (total < size_t(sms) && !q.empty()) {
      const size_t g = q.top().second;
      q.pop();
      if (parts[g] >= units(g)) continue;  // one half tile per CTA already
      ++parts[g];
      ++total;
      q.emplace(load(g), g);
    }
    for (size_t g = 0; g < ng; ++g)
      for (uint32_t j = 0; j < parts[g]; ++j) {
        const uint64_t u = units(g);
        by_group.second.push_back(uint32_t(by_group.first.size()));
        by_group.first.push_back(xksv::FusedTask{uint32_t(g), uint32_t(u * j / parts[g]), uint32_t(u * (j + 1) / parts[g]), 0});
      }
    by_group.second.push_back(uint32_t(by_group.first.size()));
  }
  {
    std::vector<uint64_t> unit0(ng);
    uint64_t all_units = 0;
    for (size_t g = 0; g < ng; ++g) {
      unit0[g] = all_units;
      all_units += units(g);
    }
    const uint64_t nctas = std::min<uint64_t>(uint64_t(std::max(sms, 1)), all_units);
    size_t g = 0;
    for (uint64_t c = 0; c < nctas; ++c) {
      shares.second.push_back(uint32_t(shares.first.size()));
      const uint64_t u0 = all_units * c / nctas, u1 = all_units * (c + 1) / nctas;
      while (g < ng && unit0[g] + units(g) <= u0) ++g;
      for (size_t h = g; h < ng && unit0[h] < u1; ++h) {
        const uint64_t a = std::max(u0, unit0[h]), b = std::min(u1, unit0[h] + units(h));
        if (a < b) shares.first.push_back(xksv::FusedTask{uint32_t(h), uint32_t(a - unit0[h]), uint32_t(b - unit0[h]), 0});
      }
    }
    shares.second.push_back(uint32_t(shares.first.size()));
  }
  const Sched& best = cost(shares) < cost(by_group) ? shares : by_group;
  segs = best.first;
  seg0 = best.second;
}
}  // namespace

using namespace xksv;

extern "C" {

// Pointers the kernels store BF16 (2-byte) or FP32 (4-byte) words through.
static bool misaligned(const void* ptr, uintptr_t align) {
  return (reinterpret_cast<uintptr_t>(ptr) & (align - 1)) != 0;
}

int xksv_cuda_decode(const void* input, size_t size, size_t rows, size_t cols, void* output) {
  const uint8_t* p = static_cast<const uint8_t*>(input);
  if (!p || !output || misaligned(output, 2)) return 1;
  if (!is_device_ptr(input) && !serial_header_ok(p, size, rows, cols, 1)) return 1;
  if (is_device_ptr(input) && (size < kHdr || !rows || !cols || cols > kMax / rows)) return 1;
  return run_single(Kind::Serial, input, size, rows, cols, output, nullptr, 1, false);
}

int xksv_cuda_gemv(const void* input, size_t size, size_t rows, size_t cols, const float* x,
                   float* output) {
  return xksv_cuda_gemm(input, size, rows, cols, 1, x, output);
}

int xksv_cuda_gemm(const void* input, size_t size, size_t rows, size_t cols, size_t batch,
                   const float* x, float* output) {
  const uint8_t* p = static_cast<const uint8_t*>(input);
  if (!x || !p || !output || misaligned(x, 4) || misaligned(output, 4)) return 1;
  if (batch > std::numeric_limits<uint32_t>::max()) return 1;
  if (!is_device_ptr(input) && !serial_header_ok(p, size, rows, cols, batch)) return 1;
  if (is_device_ptr(input) && (size < kHdr || !rows || !cols || !batch || cols > kMax / rows)) return 1;
  return run_single(Kind::Serial, input, size, rows, cols, output, x, batch, true);
}

int xksv_cuda_decode_parallel(const void* input, size_t n, void* output) {
  const uint8_t* p = static_cast<const uint8_t*>(input);
  if (!p || !output || misaligned(output, 2)) return 1;
  uint64_t rows = 0, cols = 0;
  if (is_device_ptr(input)) {
    uint8_t h[32];
    if (n < 32 || cudaMemcpy(h, input, 32, cudaMemcpyDeviceToHost) != cudaSuccess) return 1;
    rows = get64(h + 8);
    cols = get64(h + 16);
  } else if (!parallel_header_ok(p, n, &rows, &cols)) {
    return 1;
  }
  return run_single(Kind::Parallel, input, n, rows, cols, output, nullptr, 1, false);
}

int xksv_cuda_gemv_parallel(const void* input, size_t n, const float* x, float* output) {
  const uint8_t* p = static_cast<const uint8_t*>(input);
  if (!x || !p || !output || misaligned(x, 4) || misaligned(output, 4)) return 1;
  uint64_t rows = 0, cols = 0;
  if (is_device_ptr(input)) {
    uint8_t h[32];
    if (n < 32 || cudaMemcpy(h, input, 32, cudaMemcpyDeviceToHost) != cudaSuccess) return 1;
    rows = get64(h + 8);
    cols = get64(h + 16);
  } else if (!parallel_header_ok(p, n, &rows, &cols)) {
    return 1;
  }
  return run_single(Kind::Parallel, input, n, rows, cols, output, x, 1, true);
}

int xksv_plan_create(const xksv_slab* slabs, size_t n, xksv_plan** out) {
  if (!out || (!slabs && n) || n > std::numeric_limits<uint32_t>::max()) return 1;
  *out = nullptr;
  std::vector<Slab> ser, par, raw;
  bool raw_gemm_ok = true, odd_dst = false;
  uint64_t need_payload = 0, need_out = 0, need_x = 0, need_y = 0;
  for (size_t i = 0; i < n; ++i) {
    const xksv_slab& s = slabs[i];
    if (s.flags || s.src_offset > kMax - s.src_size) return 1;
    need_payload = std::max(need_payload, s.src_offset + s.src_size);
    // the bytes a decode of this slab writes at dst_offset, and the X / Y
    // rows a GEMV/GEMM reads and writes (raw decode-only slabs: src_size
    // bytes, no rows); an extent that does not fit in 64 bits is refused
    const bool shaped = s.rows && s.cols && s.cols <= kMax / 2 / s.rows;
    if ((s.rows || s.cols) && !shaped) return 1;
    const uint64_t dec = s.codec == XKSV_CODEC_RAW ? s.src_size : s.rows * s.cols * 2;
    if (s.dst_offset > kMax - dec) return 1;
    need_out = std::max(need_out, s.dst_offset + dec);
    if (shaped) {
      if (s.x_offset > kMax - s.cols || s.dst_offset > kMax - s.rows) return 1;
      need_x = std::max(need_x, s.x_offset + s.cols);
      need_y = std::max(need_y, s.dst_offset + s.rows);
    }
    // decode writes BF16 words: an odd byte offset would be a misaligned store
    if (s.codec != XKSV_CODEC_RAW && (s.dst_offset & 1)) odd_dst = true;
    Slab d{s.src_offset, s.src_size, s.rows, s.cols, s.dst_offset, s.x_offset};
    switch (s.codec) {
      case XKSV_CODEC_TILE16:
        if (!s.rows || !s.cols || s.cols > kMax / s.rows || s.src_size < kHdr) return 1;
        ser.push_back(d);
        break;
      case XKSV_CODEC_PARALLEL32:
        if (!s.rows || s.rows > 16 || !s.cols || s.src_size < 32) return 1;
        par.push_back(d);
        break;
      case XKSV_CODEC_RAW:
        if (!s.rows || !s.cols || s.cols > kMax / s.rows || s.rows * s.cols * 2 != s.src_size)
          raw_gemm_ok = false;
        raw.push_back(d);
        break;
      default:
        return 1;
    }
  }
  // indexable serial slabs first (the order of slabs within a codec is free:
  // every slab carries its own output offset)
  std::stable_partition(ser.begin(), ser.end(), tile_indexable);
  auto* p = new xksv_plan();
  cudaGetDevice(&p->device);
  p->n_ser_idx = uint32_t(std::count_if(ser.begin(), ser.end(), tile_indexable));
  int sms = 148;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, p->device);
  // one CTA per slab (per PWARPS slabs for the parallel codec): the block
  // scheduler balances slabs of different cost
  p->grid_ser = 1 << 30;
  p->grid_par = 1 << 30;
  p->grid_raw = 1 << 30;
  p->n_ser = uint32_t(ser.size());
  p->n_par = uint32_t(par.size());
  p->n_raw = uint32_t(raw.size());
  p->raw_gemm_ok = raw_gemm_ok;
  p->odd_dst = odd_dst;
  p->need_payload = need_payload;
  p->need_out = need_out;
  p->need_x_rows = need_x;
  p->need_y_rows = need_y;
  std::vector<Slab> all;
  all.reserve(n);
  all.insert(all.end(), ser.begin(), ser.end());
  all.insert(all.end(), par.begin(), par.end());
  all.insert(all.end(), raw.begin(), raw.end());
  bool ok = cudaMalloc(&p->d_status, sizeof(int)) == cudaSuccess &&
            cudaMallocHost(&p->h_status, sizeof(int)) == cudaSuccess &&
            cudaMemset(p->d_status, 0, sizeof(int)) == cudaSuccess;
  if (ok && n) {
    ok = cudaMalloc(&p->d_slabs, n * sizeof(Slab)) == cudaSuccess &&
         cudaMemcpy(p->d_slabs, all.data(), n * sizeof(Slab), cudaMemcpyHostToDevice) == cudaSuccess;
  }
  // decoded byte ranges in the caller's slab order (xksv_plan_sha256)
  if (ok && n) {
    std::vector<uint64_t> hr(2 * n);
    for (size_t i = 0; i < n; ++i) {
      hr[2 * i] = slabs[i].dst_offset;
      hr[2 * i + 1] = slabs[i].codec == XKSV_CODEC_RAW ? slabs[i].src_size : slabs[i].rows * slabs[i].cols * 2;
    }
    ok = cudaMalloc(&p->d_hash_ranges, hr.size() * sizeof(uint64_t)) == cudaSuccess &&
         cudaMemcpy(p->d_hash_ranges, hr.data(), hr.size() * sizeof(uint64_t), cudaMemcpyHostToDevice) ==
             cudaSuccess;
  }
  // tensor-core GEMM groups (raw slabs must hold exactly rows * cols BF16)
  {
    std::vector<TcGroup> groups;
    std::vector<Slab> tc_slabs;
    if (ok && raw_gemm_ok && build_tc_groups(all, groups, tc_slabs, p->scratch_bytes, p->x_cols, p->x_base)) {
      p->ngroups = uint32_t(groups.size());
      uint32_t minch = ~0u;
      for (const TcGroup& g : groups) minch = std::min<uint32_t>(minch, (g.cols + 63) / 64);
      const uint32_t want = (2 * uint32_t(sms) + p->ngroups - 1) / p->ngroups;
      p->tc_ksplit = std::max<uint32_t>(1, std::min<uint32_t>(want, minch));
      p->tc_ok = cudaMalloc(&p->d_groups, groups.size() * sizeof(TcGroup)) == cudaSuccess &&
                 cudaMalloc(&p->d_tc_slabs, n * sizeof(Slab)) == cudaSuccess &&
                 cudaMemcpy(p->d_groups, groups.data(), groups.size() * sizeof(TcGroup),
                            cudaMemcpyHostToDevice) == cudaSuccess &&
                 cudaMemcpy(p->d_tc_slabs, tc_slabs.data(), n * sizeof(Slab), cudaMemcpyHostToDevice) ==
                     cudaSuccess;
    }
  }
  // the copies above ran on the legacy default stream, which callers' non-blocking
  // streams do not wait for: finish them before the plan is used anywhere
  ok = ok && cudaStreamSynchronize(nullptr) == cudaSuccess;
  p->h_slabs = std::move(all);
  if (!ok) {
    xksv_plan_destroy(p);
    return 1;
  }
  *out = p;
  return 0;
}

void xksv_plan_destroy(xksv_plan* p) {
  if (!p) return;
  free_index(p);
  if (p->d_groups) cudaFree(p->d_groups);
  if (p->d_tc_slabs) cudaFree(p->d_tc_slabs);
  if (p->d_scratch && p->scratch_owned) cudaFree(p->d_scratch);
  if (p->d_xt) cudaFree(p->d_xt);
  if (p->d_hash_ranges) cudaFree(p->d_hash_ranges);
  if (p->d_slabs) cudaFree(p->d_slabs);
  if (p->d_status) cudaFree(p->d_status);
  if (p->h_status) cudaFreeHost(p->h_status);
  for (cudaEvent_t ev : p->chunk_ev)
    if (ev) cudaEventDestroy(ev);
  if (p->copy_st) cudaStreamDestroy(p->copy_st);
  delete p;
}

namespace {
// Indexed decode of the plan's 16-row serial slabs (slabs[0, n_ser_idx)) to
// out + slab dst; the caller decodes the remaining serial slabs.
cudaError_t tile_decode(xksv_plan* p, const xksv::Slab* slabs, const uint8_t* pay, uint8_t* out,
                        cudaStream_t st) {
  xksv::GemvArgs g{};
  g.items = p->d_items;
  g.nitems = p->n_items;
  g.slabs = slabs;
  g.tbase = p->d_tbase;
  g.tidx = p->d_tidx;
  g.gtabs = p->d_gtabs;
  g.tmid = p->d_tmid;
  g.payload = pay;
  g.status = p->d_status;
  g.out = out;
  g.nb = 1;
  return xksv::launch_serial_tile_decode(g, st);
}
}  // namespace

int xksv_plan_decode(const xksv_plan* pc, const void* d_payload, size_t payload_size, void* d_out,
                     size_t out_size, void* stream) {
  auto* p = const_cast<xksv_plan*>(pc);
  if (!p || !d_payload || !d_out || p->odd_dst || misaligned(d_out, 2)) return 1;
  if (p->need_payload > payload_size || p->need_out > out_size) return 1;  // a slab outside a buffer
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const uint8_t* pay = static_cast<const uint8_t*>(d_payload);
  uint8_t* out = static_cast<uint8_t*>(d_out);
  p->launches = 0;
  cudaError_t e = cudaSuccess;
  // with a tile index of this payload, the 16-row serial slabs decode one
  // thread per tile; the other serial slabs resynchronise their streams
  const bool indexed = p->d_tidx && d_payload == p->indexed_payload && p->n_items;
  const uint32_t ser0 = indexed ? p->n_ser_idx : 0;
  if (indexed) {
    e = tile_decode(p, p->d_slabs, pay, out, st);
    ++p->launches;
  }
  if (e == cudaSuccess && p->n_ser > ser0) {
    e = launch_serial_decode(p->d_slabs + ser0, p->n_ser - ser0, pay, out, p->d_status, p->grid_ser, st);
    ++p->launches;
  }
  if (e == cudaSuccess && p->n_par) {
    e = launch_parallel_decode(p->d_slabs + p->n_ser, p->n_par, pay, out, p->d_status, p->grid_par, st);
    ++p->launches;
  }
  if (e == cudaSuccess && p->n_raw) {
    e = launch_raw_decode(p->d_slabs + p->n_ser + p->n_par, p->n_raw, pay, out, p->grid_raw, st);
    ++p->launches;
  }
  return e == cudaSuccess ? 0 : 1;
}


// Host payload -> device -> decode, with the copy and the decode overlapped:
// the payload crosses PCIe in kHostChunks pieces on the plan's copy stream,
// and the slabs that end inside each piece are decoded on the caller's
// stream as soon as it has landed (event wait), so only the last piece's
// decode is exposed.  Needs each codec group's slabs in increasing payload
// order (an archive's block order); otherwise one copy, then the decode.
namespace {
constexpr int kHostChunks = 8;
static_assert(sizeof(xksv_plan::chunk_ev) / sizeof(cudaEvent_t) == kHostChunks + 1, "one event per chunk + 1");
uint64_t chunk_end(uint64_t end, int c) {  // end * (c + 1) / kHostChunks without overflow
  const uint64_t q = end / kHostChunks, r = end % kHostChunks;
  return q * uint64_t(c + 1) + r * uint64_t(c + 1) / kHostChunks;
}
}  // namespace

int xksv_plan_decode_host(const xksv_plan* pc, const void* h_payload, size_t payload_size, void* d_payload,
                          void* d_out, size_t out_size, void* stream) {
  auto* p = const_cast<xksv_plan*>(pc);
  if (!p || !h_payload || !d_payload || !d_out || p->odd_dst || misaligned(d_out, 2)) return 1;
  if (p->need_payload > payload_size || p->need_out > out_size) return 1;  // a slab outside a buffer
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const auto& hs = p->h_slabs;
  uint64_t end = 0;
  for (const Slab& s : hs) end = std::max(end, s.src + s.size);
  if (end > payload_size) return 1;  // a slab outside the host payload
  // groups: tile-indexable serial slabs, the other serial slabs (plan
  // creation keeps each part in table order), parallel, raw
  constexpr int NG = 4;
  const uint32_t lo[NG] = {0, p->n_ser_idx, p->n_ser, p->n_ser + p->n_par};
  const uint32_t hi[NG] = {p->n_ser_idx, p->n_ser, p->n_ser + p->n_par, p->n_ser + p->n_par + p->n_raw};
  const bool indexed = p->d_tidx && d_payload == p->indexed_payload && p->n_items;
  bool ordered = !indexed && end > 0;
  for (int g = 0; g < NG && ordered; ++g)
    for (uint32_t i = lo[g] + 1; i < hi[g] && ordered; ++i)
      ordered = hs[i].src + hs[i].size >= hs[i - 1].src + hs[i - 1].size;
  if (!ordered) {
    if (end && cudaMemcpyAsync(d_payload, h_payload, end, cudaMemcpyHostToDevice, st) != cudaSuccess) return 1;
    return xksv_plan_decode(p, d_payload, payload_size, d_out, out_size, stream);
  }
  if (!p->copy_st && cudaStreamCreateWithFlags(&p->copy_st, cudaStreamNonBlocking) != cudaSuccess) return 1;
  for (cudaEvent_t& ev : p->chunk_ev)
    if (!ev && cudaEventCreateWithFlags(&ev, cudaEventDisableTiming) != cudaSuccess) return 1;
  const uint8_t* h = static_cast<const uint8_t*>(h_payload);
  uint8_t* pay = static_cast<uint8_t*>(d_payload);
  uint8_t* out = static_cast<uint8_t*>(d_out);
  // the copies must not overwrite bytes that earlier work on `st` still reads
  cudaError_t e = cudaEventRecord(p->chunk_ev[kHostChunks], st);
  if (e == cudaSuccess) e = cudaStreamWaitEvent(p->copy_st, p->chunk_ev[kHostChunks], 0);
  uint64_t a = 0;
  for (int c = 0; c < kHostChunks && e == cudaSuccess; ++c) {
    const uint64_t b = chunk_end(end, c);
    if (b > a) e = cudaMemcpyAsync(pay + a, h + a, b - a, cudaMemcpyHostToDevice, p->copy_st);
    if (e == cudaSuccess) e = cudaEventRecord(p->chunk_ev[c], p->copy_st);
    a = b;
  }
  p->launches = 0;
  uint32_t done[NG] = {lo[0], lo[1], lo[2], lo[3]};
  for (int c = 0; c < kHostChunks && e == cudaSuccess; ++c) {
    const uint64_t b = chunk_end(end, c);
    uint32_t upto[NG];
    bool any = false;
    for (int g = 0; g < NG; ++g) {
      upto[g] = done[g];
      while (upto[g] < hi[g] && hs[upto[g]].src + hs[upto[g]].size <= b) ++upto[g];
      any = any || upto[g] > done[g];
    }
    if (!any) continue;
    e = cudaStreamWaitEvent(st, p->chunk_ev[c], 0);
    for (int g = 0; g < 2 && e == cudaSuccess; ++g)
      if (upto[g] > done[g]) {
        e = launch_serial_decode(p->d_slabs + done[g], upto[g] - done[g], pay, out, p->d_status, p->grid_ser, st);
        ++p->launches;
      }
    if (e == cudaSuccess && upto[2] > done[2]) {
      e = launch_parallel_decode(p->d_slabs + done[2], upto[2] - done[2], pay, out, p->d_status, p->grid_par, st);
      ++p->launches;
    }
    if (e == cudaSuccess && upto[3] > done[3]) {
      e = launch_raw_decode(p->d_slabs + done[3], upto[3] - done[3], pay, out, p->grid_raw, st);
      ++p->launches;
    }
    for (int g = 0; g < NG; ++g) done[g] = upto[g];
  }
  return e == cudaSuccess ? 0 : 1;
}

int xksv_plan_gemm(const xksv_plan* pc, const void* d_payload, size_t payload_size, const float* d_x,
                   size_t x_rows, float* d_y, size_t y_rows, size_t batch, void* stream) {
  auto* p = const_cast<xksv_plan*>(pc);
  if (!p || !d_payload || !d_x || !d_y || !batch || batch > std::numeric_limits<uint32_t>::max() ||
      misaligned(d_x, 4) || misaligned(d_y, 4))
    return 1;
  if (p->need_payload > payload_size || p->need_x_rows > x_rows || p->need_y_rows > y_rows) return 1;
  if (p->n_raw && !p->raw_gemm_ok) return 1;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const uint8_t* pay = static_cast<const uint8_t*>(d_payload);
  p->launches = 0;
  cudaError_t e = cudaSuccess;
  const uint32_t ld = uint32_t(batch);
  // routing (measured on B200 with the tile index): up to batch 3 the
  // CUDA-core kernels with FP32 X (1024 slabs of 16x4096: 116 us at batch 1,
  // 182 / 190 us at 2 / 3); from batch 4, decode + tensor-core GEMM with X
  // rounded to BF16 (200 us for any batch <= 256, against 230 us for batch 4
  // on the CUDA cores; the 70B linears: 164 ms against 226 ms at batch 4)
  const bool indexed = p->d_tidx && d_payload == p->indexed_payload;
  const bool fused = p->fused_ok && indexed && batch >= 4 && batch <= 128 && p->gemm_route != XKSV_GEMM_SCRATCH;
  if (fused) {
    // one kernel decodes every tile row into tensor-core operand stages,
    // after a prep kernel (X^T in BF16, zeroed Y rows) that it overlaps
    if (!p->d_xt && cudaMalloc(&p->d_xt, 256 * p->x_cols * 2) != cudaSuccess) return 1;
    FusedArgs f{};
    f.seg0 = p->d_fseg0;
    f.tasks = p->d_ftasks;
    f.groups = p->d_fgroups;
    f.members = p->d_fmembers;
    f.slabs = p->d_slabs;
    f.tbase = p->d_tbase;
    f.tidx = p->d_tidx;
    f.tmid = p->d_tmid;
    f.tabs = p->d_ftabs;
    f.payload = pay;
    f.xt = p->d_xt;
    f.xt_ld = p->x_cols;
    f.y = d_y;
    f.ld = ld;
    f.nb = uint32_t(batch);
    f.npad = (f.nb + 15) / 16 * 16;
    f.status = p->d_status;
    e = launch_fused_gemm(f, p->n_fctas, d_x + p->x_base * ld, p->x_cols, p->d_groups, p->ngroups, st);
    p->launches = 2;
    return e == cudaSuccess ? 0 : 1;
  }
  if (p->tc_ok && batch >= 4) {
    // decode every slab into its BF16 row group, then the tensor-core GEMM,
    // up to 256 batch columns per pass over the same decoded scratch
    if (!p->d_scratch && cudaMalloc(&p->d_scratch, std::max<uint64_t>(16, p->scratch_bytes)) != cudaSuccess)
      return 1;
    if (!p->d_xt && cudaMalloc(&p->d_xt, 256 * p->x_cols * 2) != cudaSuccess) return 1;
    const uint32_t tser0 = indexed && p->n_items ? p->n_ser_idx : 0;
    if (tser0) {
      e = tile_decode(p, p->d_tc_slabs, pay, p->d_scratch, st);
      ++p->launches;
    }
    if (e == cudaSuccess && p->n_ser > tser0) {
      e = launch_serial_decode(p->d_tc_slabs + tser0, p->n_ser - tser0, pay, p->d_scratch, p->d_status,
                               p->grid_ser, st);
      ++p->launches;
    }
    if (e == cudaSuccess && p->n_par) {
      e = launch_parallel_decode(p->d_tc_slabs + p->n_ser, p->n_par, pay, p->d_scratch, p->d_status,
                                 p->grid_par, st);
      ++p->launches;
    }
    if (e == cudaSuccess && p->n_raw) {
      e = launch_raw_decode(p->d_tc_slabs + p->n_ser + p->n_par, p->n_raw, pay, p->d_scratch,
                            p->grid_raw, st);
      ++p->launches;
    }
    for (size_t b0 = 0; b0 < batch && e == cudaSuccess; b0 += 256) {
      TcGemmArgs g{};
      g.groups = p->d_groups;
      g.scratch = p->d_scratch;
      g.xt = p->d_xt;
      g.xt_ld = p->x_cols;
      g.y = d_y + b0;
      g.ld = ld;
      g.nb = uint32_t(std::min<size_t>(256, batch - b0));
      g.npad = (g.nb + 15) / 16 * 16;
      g.ksplit = p->tc_ksplit;
      g.tmem_cols = 32;
      while (g.tmem_cols < g.npad) g.tmem_cols *= 2;
      g.status = p->d_status;
      e = launch_tc_gemm(g, p->ngroups, d_x + p->x_base * ld + b0, p->x_cols, st);
      p->launches += g.ksplit > 1 ? 3 : 2;
    }
    return e == cudaSuccess ? 0 : 1;
  }
  // indexed serial slabs: tile-parallel kernel, 4 batch columns per pass
  const uint32_t ser0 = indexed ? p->n_ser_idx : 0;
  if (indexed && p->n_items) {
    for (size_t b0 = 0; b0 < batch && e == cudaSuccess; b0 += 4) {
      GemvArgs g{};
      g.items = p->d_items;
      g.nitems = p->n_items;
      g.slabs = p->d_slabs;
      g.tbase = p->d_tbase;
      g.tidx = p->d_tidx;
      g.gtabs = p->d_gtabs;
      g.tmid = p->d_tmid;
      g.payload = pay;
      g.x = d_x + b0;
      g.y = d_y + b0;
      g.ld = ld;
      g.nb = uint32_t(std::min<size_t>(4, batch - b0));
      g.partials = p->d_partials;
      g.counters = p->d_counters;
      g.status = p->d_status;
      e = launch_serial_tile_gemm(g, st);
      ++p->launches;
    }
  }
  for (size_t b0 = 0; b0 < batch && e == cudaSuccess; b0 += 8) {
    const uint32_t nb = uint32_t(std::min<size_t>(8, batch - b0));
    if (p->n_ser > ser0) {
      e = launch_serial_gemm(p->d_slabs + ser0, p->n_ser - ser0, pay, d_x, d_y, ld, uint32_t(b0), nb,
                             p->d_status, p->grid_ser, st);
      ++p->launches;
    }
    if (e == cudaSuccess && p->n_par) {
      e = launch_parallel_gemm(p->d_slabs + p->n_ser, p->n_par, pay, d_x, d_y, ld, uint32_t(b0), nb,
                               p->d_status, p->grid_par, st);
      ++p->launches;
    }
    if (e == cudaSuccess && p->n_raw) {
      e = launch_raw_gemm(p->d_slabs + p->n_ser + p->n_par, p->n_raw, pay, d_x, d_y, ld, uint32_t(b0),
                          nb, p->grid_raw, st);
      ++p->launches;
    }
  }
  return e == cudaSuccess ? 0 : 1;
}

int xksv_plan_set_gemm_route(xksv_plan* p, int route) {
  if (!p || route < XKSV_GEMM_AUTO || route > XKSV_GEMM_FUSED) return 1;
  p->gemm_route = route;
  return 0;
}

int xksv_plan_fused_ready(const xksv_plan* p, const void* d_payload) {
  return p && p->fused_ok && p->d_tidx && d_payload == p->indexed_payload ? 1 : 0;
}

size_t xksv_plan_scratch_bytes(const xksv_plan* p) {
  return p && p->tc_ok ? size_t(std::max<uint64_t>(16, p->scratch_bytes)) : 0;
}

int xksv_plan_set_scratch(xksv_plan* p, void* d_scratch, size_t bytes) {
  if (!p) return 1;
  if (!p->tc_ok) return 0;  // no tensor-core path: nothing uses a scratch
  if (d_scratch && (bytes < xksv_plan_scratch_bytes(p) || misaligned(d_scratch, 256))) return 1;
  if (p->d_scratch && p->scratch_owned) cudaFree(p->d_scratch);
  p->d_scratch = static_cast<uint8_t*>(d_scratch);  // null: allocate an own one on next use
  p->scratch_owned = d_scratch == nullptr;
  return 0;
}

int xksv_plan_status(const xksv_plan* pc, void* stream) {
  auto* p = const_cast<xksv_plan*>(pc);
  if (!p) return 1;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (cudaMemcpyAsync(p->h_status, p->d_status, sizeof(int), cudaMemcpyDeviceToHost, st) != cudaSuccess)
    return 1;
  if (cudaStreamSynchronize(st) != cudaSuccess) return 1;
  int v = *p->h_status;
  if (cudaMemsetAsync(p->d_status, 0, sizeof(int), st) != cudaSuccess) return 1;
  if (cudaStreamSynchronize(st) != cudaSuccess) return 1;
  return v == 0 ? 0 : 1;
}

int xksv_plan_launches(const xksv_plan* p) { return p ? p->launches : 0; }

int xksv_cuda_sha256(const uint64_t* ranges, size_t n, const void* d_base, void* d_digests, void* stream) {
  if (!n) return 0;
  if (!ranges || !d_base || !d_digests || n > std::numeric_limits<uint32_t>::max()) return 1;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  void* d_r = nullptr;  // stream-ordered: no device-wide synchronisation
  if (cudaMallocAsync(&d_r, 2 * n * sizeof(uint64_t), st) != cudaSuccess) return 1;
  cudaError_t e = cudaMemcpyAsync(d_r, ranges, 2 * n * sizeof(uint64_t), cudaMemcpyHostToDevice, st);
  if (e == cudaSuccess)
    e = launch_sha256(static_cast<const uint64_t*>(d_r), uint32_t(n), static_cast<const uint8_t*>(d_base),
                      static_cast<uint8_t*>(d_digests), st);
  const cudaError_t f = cudaFreeAsync(d_r, st);
  // the host ranges must outlive the copy
  const cudaError_t g = cudaStreamSynchronize(st);
  return e == cudaSuccess && f == cudaSuccess && g == cudaSuccess ? 0 : 1;
}

int xksv_plan_sha256(const xksv_plan* p, const void* d_out, size_t out_size, void* d_digests, void* stream) {
  if (!p || !d_out || !d_digests || p->need_out > out_size) return 1;
  const uint32_t n = p->n_ser + p->n_par + p->n_raw;
  return launch_sha256(p->d_hash_ranges, n, static_cast<const uint8_t*>(d_out), static_cast<uint8_t*>(d_digests),
                       static_cast<cudaStream_t>(stream)) == cudaSuccess
             ? 0
             : 1;
}

// After a successful index: the fused decode -> tensor-core GEMM applies
// when every slab of the plan is on the tile path, the plan has a
// tensor-core path and every codebook fits the fused decoder's tables; each
// group's lane tables are built here, once.  Any failure here only leaves
// the fused route off.
static void setup_fused(xksv_plan* p, const uint8_t* d_payload, cudaStream_t st) {
  const uint32_t n = p->n_ser + p->n_par + p->n_raw;
  if (!p->tc_ok || !n || p->n_ser_idx != n) return;
  uint8_t* d_ok = nullptr;
  std::vector<uint8_t> ok(n, 0);
  bool good = cudaMalloc(&d_ok, n) == cudaSuccess && launch_fused_check(p->d_slabs, n, d_payload, d_ok, st) == cudaSuccess &&
              cudaMemcpyAsync(ok.data(), d_ok, n, cudaMemcpyDeviceToHost, st) == cudaSuccess &&
              cudaStreamSynchronize(st) == cudaSuccess;
  if (d_ok) cudaFree(d_ok);
  for (uint32_t i = 0; i < n && good; ++i) good = ok[i] == 1;
  if (!good) return;
  int sms = 148;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, p->device);
  std::vector<FusedGroup> groups;
  std::vector<uint32_t> members, seg0;
  std::vector<FusedTask> tasks;
  build_fused(p->h_slabs, p->x_base, sms, fused_producers(16, nullptr), groups, members, tasks, seg0);
  good = !tasks.empty() && seg0.size() >= 2 &&
         cudaMalloc(&p->d_fseg0, seg0.size() * sizeof(uint32_t)) == cudaSuccess &&
         cudaMemcpyAsync(p->d_fseg0, seg0.data(), seg0.size() * sizeof(uint32_t), cudaMemcpyHostToDevice, st) ==
             cudaSuccess &&
         cudaMalloc(&p->d_ftasks, tasks.size() * sizeof(FusedTask)) == cudaSuccess &&
         cudaMalloc(&p->d_fgroups, groups.size() * sizeof(FusedGroup)) == cudaSuccess &&
         cudaMalloc(&p->d_fmembers, members.size() * sizeof(uint32_t)) == cudaSuccess &&
         cudaMemcpyAsync(p->d_ftasks, tasks.data(), tasks.size() * sizeof(FusedTask), cudaMemcpyHostToDevice, st) ==
             cudaSuccess &&
         cudaMemcpyAsync(p->d_fgroups, groups.data(), groups.size() * sizeof(FusedGroup), cudaMemcpyHostToDevice,
                         st) == cudaSuccess &&
         cudaMemcpyAsync(p->d_fmembers, members.data(), members.size() * sizeof(uint32_t), cudaMemcpyHostToDevice,
                         st) == cudaSuccess &&
         cudaMalloc(&p->d_ftabs, groups.size() * fused_tables_bytes()) == cudaSuccess &&
         cudaMemsetAsync(p->d_status, 0, sizeof(int), st) == cudaSuccess &&
         launch_fused_tables(p->d_fgroups, uint32_t(groups.size()), p->d_fmembers, p->d_slabs, d_payload, p->d_ftabs,
                             p->d_status, st) == cudaSuccess &&
         cudaMemcpyAsync(p->h_status, p->d_status, sizeof(int), cudaMemcpyDeviceToHost, st) == cudaSuccess &&
         cudaStreamSynchronize(st) == cudaSuccess && *p->h_status == 0;
  cudaMemsetAsync(p->d_status, 0, sizeof(int), st);
  cudaStreamSynchronize(st);
  if (!good) {
    if (p->d_fseg0) cudaFree(p->d_fseg0);
    p->d_fseg0 = nullptr;
    if (p->d_ftasks) cudaFree(p->d_ftasks);
    if (p->d_fgroups) cudaFree(p->d_fgroups);
    if (p->d_fmembers) cudaFree(p->d_fmembers);
    if (p->d_ftabs) cudaFree(p->d_ftabs);
    p->d_ftabs = nullptr;
    p->d_ftasks = nullptr;
    p->d_fgroups = nullptr;
    p->d_fmembers = nullptr;
    return;
  }
  p->n_fctas = uint32_t(seg0.size() - 1);
  p->fused_ok = true;
}

int xksv_plan_index(xksv_plan* p, const void* d_payload, size_t payload_size, void* stream) {
  if (!p || !d_payload || p->need_payload > payload_size) return 1;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (cudaStreamSynchronize(st) != cudaSuccess) return 1;
  free_index(p);
  const uint32_t n = p->n_ser_idx;
  if (!n) {
    p->indexed_payload = d_payload;
    return 0;
  }
  const std::vector<Slab>& sl = p->h_slabs;
  // index layout: per slab (tiles + 1) entries; items: <= 256 tiles each,
  // tiles spread evenly over the slab's items
  std::vector<uint64_t> tbase(n);
  std::vector<GemvItem> items;
  uint64_t total = 0;
  for (uint32_t i = 0; i < n; ++i) {
    const uint32_t tiles = uint32_t(sl[i].cols / 16);
    tbase[i] = total;
    total += uint64_t(tiles) + 1;  // every tile's first code + end
    const uint32_t ni = (tiles + 255) / 256;  // one 256-thread CTA per item
    const uint32_t per = (tiles + ni - 1) / ni;
    const uint32_t first = uint32_t(items.size());
    for (uint32_t k = 0; k < ni; ++k) {
      const uint32_t t0 = k * per;
      items.push_back(GemvItem{i, t0, std::min(per, tiles - t0), first, ni, 0, 0, 0});
    }
  }
  if (total > std::numeric_limits<uint32_t>::max() || items.size() > (1u << 31)) return 1;
  // every copy and fill on the caller's stream, ahead of the index kernel
  // (a non-blocking stream does not wait for the legacy default stream)
  bool ok = cudaMalloc(&p->d_tidx, total * sizeof(uint32_t)) == cudaSuccess &&
            cudaMalloc(&p->d_tmid, total * sizeof(uint32_t)) == cudaSuccess &&
            cudaMalloc(&p->d_tbase, n * sizeof(uint64_t)) == cudaSuccess &&
            cudaMalloc(&p->d_gtabs, n * sizeof(GemvTabs)) == cudaSuccess &&
            cudaMalloc(&p->d_items, items.size() * sizeof(GemvItem)) == cudaSuccess &&
            cudaMalloc(&p->d_partials, items.size() * 16 * 4 * sizeof(float)) == cudaSuccess &&
            cudaMalloc(&p->d_counters, n * sizeof(uint32_t)) == cudaSuccess &&
            cudaMemcpyAsync(p->d_tbase, tbase.data(), n * sizeof(uint64_t), cudaMemcpyHostToDevice, st) == cudaSuccess &&
            cudaMemcpyAsync(p->d_items, items.data(), items.size() * sizeof(GemvItem), cudaMemcpyHostToDevice, st) == cudaSuccess &&
            cudaMemsetAsync(p->d_counters, 0, n * sizeof(uint32_t), st) == cudaSuccess &&
            cudaMemsetAsync(p->d_tidx, 0, total * sizeof(uint32_t), st) == cudaSuccess &&
            cudaMemsetAsync(p->d_tmid, 0, total * sizeof(uint32_t), st) == cudaSuccess &&
            cudaMemsetAsync(p->d_status, 0, sizeof(int), st) == cudaSuccess;
  if (ok)
    ok = launch_serial_index(p->d_slabs, n, static_cast<const uint8_t*>(d_payload), p->d_tidx, p->d_tmid,
                             p->d_tbase, p->d_gtabs, p->d_status, st) == cudaSuccess;
  if (ok)
    ok = cudaMemcpyAsync(p->h_status, p->d_status, sizeof(int), cudaMemcpyDeviceToHost, st) == cudaSuccess &&
         cudaStreamSynchronize(st) == cudaSuccess;
  const bool bad = !ok || *p->h_status != 0;
  cudaMemsetAsync(p->d_status, 0, sizeof(int), st);
  cudaStreamSynchronize(st);
  if (bad) {
    free_index(p);
    return 1;
  }
  p->n_items = uint32_t(items.size());
  p->indexed_payload = d_payload;
  setup_fused(p, static_cast<const uint8_t*>(d_payload), st);
  return 0;
}

// ------------------------------------------------ fused tensor parallel ---
}  // extern "C"

struct xksv_tp_fused {
  int device = 0, world = 1, rank = 0;
  size_t max_rows = 0, max_batch = 0;
  uint8_t* base = nullptr;  // [2 gathered buffers][flags per rank][epoch][done]
  size_t buf_bytes = 0, flags_off = 0, epoch_off = 0, done_off = 0;
  std::vector<void*> opened;  // peers' mappings (nullptr for this rank)
  float** d_peer_y[2] = {nullptr, nullptr};
  uint32_t** d_peer_flags = nullptr;
  uint64_t calls = 0;
};

extern "C" {

int xksv_tp_fused_create(int world, int rank, size_t max_rows_shard, size_t max_batch, xksv_tp_fused** out,
                         void* ipc_handle) {
  if (!out || !ipc_handle || world < 1 || rank < 0 || rank >= world || !max_rows_shard || !max_batch ||
      max_batch > 4)
    return 1;
  *out = nullptr;
  auto* c = new xksv_tp_fused();
  cudaGetDevice(&c->device);
  c->world = world;
  c->rank = rank;
  c->max_rows = max_rows_shard;
  c->max_batch = max_batch;
  auto up = [](size_t v) { return (v + 255) & ~size_t(255); };
  c->buf_bytes = up(size_t(world) * max_rows_shard * max_batch * sizeof(float));
  c->flags_off = 2 * c->buf_bytes;
  c->epoch_off = c->flags_off + up(size_t(world) * sizeof(uint32_t));
  c->done_off = c->epoch_off + 256;
  const size_t total = c->done_off + 256;
  cudaIpcMemHandle_t h;
  const bool ok = cudaMalloc(&c->base, total) == cudaSuccess && cudaMemset(c->base, 0, total) == cudaSuccess &&
                  cudaIpcGetMemHandle(&h, c->base) == cudaSuccess && cudaDeviceSynchronize() == cudaSuccess;
  if (!ok) {
    xksv_tp_fused_destroy(c);
    return 1;
  }
  std::memcpy(ipc_handle, &h, sizeof(h));
  *out = c;
  return 0;
}

int xksv_tp_fused_open(xksv_tp_fused* c, const void* handles) {
  if (!c || !handles) return 1;
  c->opened.assign(c->world, nullptr);
  std::vector<float*> y0(c->world), y1(c->world);
  std::vector<uint32_t*> fl(c->world);
  for (int g = 0; g < c->world; ++g) {
    uint8_t* b = c->base;
    if (g != c->rank) {
      cudaIpcMemHandle_t h;
      std::memcpy(&h, static_cast<const uint8_t*>(handles) + g * sizeof(h), sizeof(h));
      void* p = nullptr;
      if (cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) return 1;
      c->opened[g] = p;
      b = static_cast<uint8_t*>(p);
    }
    y0[g] = reinterpret_cast<float*>(b);
    y1[g] = reinterpret_cast<float*>(b + c->buf_bytes);
    fl[g] = reinterpret_cast<uint32_t*>(b + c->flags_off);
  }
  const size_t pb = c->world * sizeof(void*);
  const bool ok = cudaMalloc(&c->d_peer_y[0], pb) == cudaSuccess && cudaMalloc(&c->d_peer_y[1], pb) == cudaSuccess &&
                  cudaMalloc(&c->d_peer_flags, pb) == cudaSuccess &&
                  cudaMemcpy(c->d_peer_y[0], y0.data(), pb, cudaMemcpyHostToDevice) == cudaSuccess &&
                  cudaMemcpy(c->d_peer_y[1], y1.data(), pb, cudaMemcpyHostToDevice) == cudaSuccess &&
                  cudaMemcpy(c->d_peer_flags, fl.data(), pb, cudaMemcpyHostToDevice) == cudaSuccess &&
                  cudaStreamSynchronize(nullptr) == cudaSuccess;
  return ok ? 0 : 1;
}

int xksv_tp_fused_gemm(xksv_tp_fused* c, const xksv_plan* pc, const void* d_payload, size_t payload_size,
                       const float* d_x, size_t x_rows, size_t rows_shard, size_t batch, float* d_y_full,
                       float** d_gathered, void* stream) {
  auto* p = const_cast<xksv_plan*>(pc);
  if (!c || !p || !d_payload || !d_x || !c->d_peer_flags || !batch || batch > c->max_batch ||
      rows_shard > c->max_rows || misaligned(d_x, 4) || misaligned(d_y_full, 4))
    return 1;
  // the epilogue stores row r of this rank's block at rank * rows_shard + r of
  // every gathered buffer: a plan row past rows_shard would land in the next
  // rank's block or past the buffer, onto the flags
  if (p->need_y_rows > rows_shard || p->need_payload > payload_size || p->need_x_rows > x_rows) return 1;
  // every slab must be on the indexed tile path for this payload
  const uint32_t n = p->n_ser + p->n_par + p->n_raw;
  if (!p->d_tidx || d_payload != p->indexed_payload || p->n_ser_idx != n || !p->n_items) return 1;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int parity = int(c->calls & 1);
  GemvArgs g{};
  g.items = p->d_items;
  g.nitems = p->n_items;
  g.slabs = p->d_slabs;
  g.tbase = p->d_tbase;
  g.tidx = p->d_tidx;
  g.gtabs = p->d_gtabs;
  g.tmid = p->d_tmid;
  g.payload = static_cast<const uint8_t*>(d_payload);
  g.x = d_x;
  g.ld = uint32_t(batch);
  g.nb = uint32_t(batch);
  g.partials = p->d_partials;
  g.counters = p->d_counters;
  g.status = p->d_status;
  g.peer_y = c->d_peer_y[parity];
  g.peer_flags = c->d_peer_flags;
  g.npeers = uint32_t(c->world);
  g.rank = uint32_t(c->rank);
  g.peer_row0 = uint64_t(c->rank) * rows_shard;
  g.peer_rows = rows_shard;
  g.done = reinterpret_cast<uint32_t*>(c->base + c->done_off);
  g.epoch = reinterpret_cast<uint32_t*>(c->base + c->epoch_off);
  cudaError_t e = launch_serial_tile_gemm(g, st);
  if (e == cudaSuccess)
    e = launch_tp_wait(reinterpret_cast<const uint32_t*>(c->base + c->flags_off), uint32_t(c->world), g.epoch,
                       p->d_status, st);
  p->launches = 2;
  float* gathered = reinterpret_cast<float*>(c->base + parity * c->buf_bytes);
  if (e == cudaSuccess && d_y_full)
    e = cudaMemcpyAsync(d_y_full, gathered, size_t(c->world) * rows_shard * batch * sizeof(float),
                        cudaMemcpyDeviceToDevice, st);
  if (e != cudaSuccess) return 1;
  if (d_gathered) *d_gathered = gathered;
  ++c->calls;
  return 0;
}

void xksv_tp_fused_destroy(xksv_tp_fused* c) {
  if (!c) return;
  for (void* q : c->opened)
    if (q) cudaIpcCloseMemHandle(q);
  if (c->d_peer_y[0]) cudaFree(c->d_peer_y[0]);
  if (c->d_peer_y[1]) cudaFree(c->d_peer_y[1]);
  if (c->d_peer_flags) cudaFree(c->d_peer_flags);
  if (c->base) cudaFree(c->base);
  delete c;
}

}  // extern "C"
