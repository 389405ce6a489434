// Archive-side encoder (host CPU): builds the slab payload that the decode
// kernels consume.  This is the compile step of the format, not a decode path
// -- the reference runs it on the CPU too (src/compile.cpp:247-285 calling
// src/c_api.cpp:18-28 and 44-65).  Outputs are byte-identical to the
// reference's xksv_pack / xksv_pack_parallel (checked by tests/test_pack.py
// against the reference's golden vectors).
//
// Algorithm restated from the reference (src/codec.cpp:32-58): exponent byte
// (w >> 7) & 255 is Huffman coded with leaves in symbol order and the two
// smallest (frequency, node index) pairs merged first; a leaf's code length is
// max(depth, 1); codes are canonical (sorted by (length, symbol), each the
// previous plus one, left-aligned); sign+mantissa go to one raw byte.
#include <algorithm>
#include <atomic>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <limits>
#include <thread>
#include <vector>

#include "xksv_cuda.h"

namespace {

constexpr uint64_t kHdr = 272;

void put64(uint8_t* p, uint64_t v) {
  for (int i = 0; i < 8; ++i) p[i] = uint8_t(v >> (8 * i));
}

// Row-major -> 16x16 tile order (src/layout.cpp:32-50).
void tile16(const uint16_t* in, uint16_t* out, size_t rows, size_t cols) {
  size_t k = 0;
  for (size_t r = 0; r < rows; r += 16) {
    const size_t nr = std::min<size_t>(16, rows - r);
    for (size_t c = 0; c < cols; c += 16) {
      const size_t nc = std::min<size_t>(16, cols - c);
      for (size_t i = 0; i < nr; ++i) {
        std::memcpy(out + k, in + (r + i) * cols + c, nc * 2);
        k += nc;
      }
    }
  }
}

// Huffman code lengths for a frequency table, with the reference's tie
// order.  Returns false when a depth exceeds 255.
bool code_lengths(const uint64_t* freq, uint8_t* lens) {
  std::memset(lens, 0, 256);
  // The priority queue pops the smallest (freq, node); leaves get indices in
  // symbol order and internal nodes are appended, so two sorted queues (leaves
  // by (freq, index), internal nodes in creation order -- their frequencies
  // never decrease) reproduce the pop order exactly.
  struct Node {
    uint64_t f;
    int left, right, sym;
  };
  Node nodes[512];
  int nleaf = 0;
  int order[256];
  for (int s = 0; s < 256; ++s)
    if (freq[s]) {
      nodes[nleaf] = {freq[s], -1, -1, s};
      order[nleaf] = nleaf;
      ++nleaf;
    }
  if (nleaf == 0) return true;
  std::sort(order, order + nleaf, [&](int a, int b) {
    return nodes[a].f < nodes[b].f || (nodes[a].f == nodes[b].f && a < b);
  });
  int li = 0, ii = nleaf, n = nleaf;  // leaf cursor, internal cursor, next node
  auto pick = [&]() -> int {
    const bool leaf_ok = li < nleaf;
    const bool int_ok = ii < n;
    if (leaf_ok && (!int_ok || nodes[order[li]].f < nodes[ii].f ||
                    (nodes[order[li]].f == nodes[ii].f && order[li] < ii)))
      return order[li++];
    return ii++;
  };
  while ((nleaf - li) + (n - ii) > 1) {
    const int a = pick(), b = pick();
    nodes[n] = {nodes[a].f + nodes[b].f, a, b, -1};
    ++n;
  }
  // depths from the root (last node)
  int depth[512];
  depth[n - 1] = 0;
  for (int i = n - 1; i >= nleaf; --i) {
    depth[nodes[i].left] = depth[i] + 1;
    depth[nodes[i].right] = depth[i] + 1;
  }
  for (int i = 0; i < nleaf; ++i) {
    if (depth[i] > 255) return false;
    lens[nodes[i].sym] = uint8_t(std::max(depth[i], 1));
  }
  return true;
}

// Canonical codes (MSB-first values) for lengths <= 64; false if a length
// exceeds 64 (not reachable for slabs below ~10^13 elements).
bool canonical_codes(const uint8_t* lens, uint64_t* code) {
  int order[256], n = 0;
  for (int s = 0; s < 256; ++s)
    if (lens[s]) order[n++] = s;
  std::sort(order, order + n, [&](int a, int b) {
    return lens[a] < lens[b] || (lens[a] == lens[b] && a < b);
  });
  uint64_t c = 0;
  int prev = 0;
  for (int k = 0; k < n; ++k) {
    const int l = lens[order[k]];
    if (l > 64) return false;
    if (k) c = (c + 1) << (l - prev);
    code[order[k]] = c;
    prev = l;
  }
  return true;
}

// One serial block for already-tiled words into `out` (resized).
bool encode_block(const uint16_t* w, uint64_t count, std::vector<uint8_t>& out) {
  uint64_t freq[256] = {0};
  for (uint64_t i = 0; i < count; ++i) ++freq[(w[i] >> 7) & 255];
  uint8_t lens[256];
  if (!code_lengths(freq, lens)) return false;
  uint64_t code[256] = {0};
  if (!canonical_codes(lens, code)) return false;
  uint64_t bits = 0;
  for (int s = 0; s < 256; ++s) bits += freq[s] * lens[s];
  const uint64_t ebytes = bits / 8 + (bits % 8 != 0);
  out.assign(kHdr + count + ebytes, 0);
  put64(out.data(), count);
  put64(out.data() + 8, bits);
  std::memcpy(out.data() + 16, lens, 256);
  uint8_t* sm = out.data() + kHdr;
  uint8_t* e = sm + count;
  uint64_t acc = 0;  // pending bits, right-aligned
  int nacc = 0;
  size_t o = 0;
  for (uint64_t i = 0; i < count; ++i) {
    const uint16_t x = w[i];
    sm[i] = uint8_t(((x >> 8) & 0x80) | (x & 0x7F));
    const int s = (x >> 7) & 255;
    const int l = lens[s];
    const uint64_t c = code[s];
    if (l <= 32) {
      acc = (acc << l) | c;
      nacc += l;
    } else {  // very long code: emit in two parts
      acc = (acc << (l - 32)) | (c >> 32);
      nacc += l - 32;
      while (nacc >= 8) {
        nacc -= 8;
        e[o++] = uint8_t(acc >> nacc);
      }
      acc = (acc << 32) | (c & 0xFFFFFFFFu);
      nacc += 32;
    }
    while (nacc >= 8) {
      nacc -= 8;
      e[o++] = uint8_t(acc >> nacc);
    }
  }
  if (nacc) e[o++] = uint8_t(acc << (8 - nacc));
  return true;
}

bool pack_serial(const uint16_t* rowmajor, size_t rows, size_t cols, std::vector<uint8_t>& out) {
  std::vector<uint16_t> t(rows * cols);
  tile16(rowmajor, t.data(), rows, cols);
  return encode_block(t.data(), t.size(), out);
}

bool pack_parallel(const uint16_t* rowmajor, size_t rows, size_t cols, std::vector<uint8_t>& out) {
  const uint64_t total = uint64_t(rows) * cols;
  std::vector<uint16_t> t(total);
  tile16(rowmajor, t.data(), rows, cols);
  const uint64_t chunks = std::min<uint64_t>(32, total);
  std::vector<std::vector<uint8_t>> seg(chunks);
  size_t size = 32 + 8 * chunks;
  for (uint64_t i = 0; i < chunks; ++i) {
    const uint64_t s = total * i / chunks, e = total * (i + 1) / chunks;
    if (!encode_block(t.data() + s, e - s, seg[i])) return false;
    size += seg[i].size();
  }
  out.resize(size);
  std::memcpy(out.data(), "XKSP2\0\0\0", 8);
  put64(out.data() + 8, rows);
  put64(out.data() + 16, cols);
  put64(out.data() + 24, chunks);
  size_t pos = 32 + 8 * chunks;
  for (uint64_t i = 0; i < chunks; ++i) {
    put64(out.data() + 32 + 8 * i, seg[i].size());
    std::memcpy(out.data() + pos, seg[i].data(), seg[i].size());
    pos += seg[i].size();
  }
  return true;
}

void* copy_out(const std::vector<uint8_t>& v, size_t* size) {
  void* p = std::malloc(v.empty() ? 1 : v.size());
  if (p && !v.empty()) std::memcpy(p, v.data(), v.size());
  *size = v.size();
  return p;
}

std::vector<uint16_t> load_words(const void* data, size_t n) {
  std::vector<uint16_t> w(n / 2);
  const uint8_t* p = static_cast<const uint8_t*>(data);
  for (size_t i = 0; i < w.size(); ++i) w[i] = uint16_t(p[2 * i] | (p[2 * i + 1] << 8));
  return w;
}

}  // namespace

extern "C" {

int xksv_host_pack(const void* data, size_t n, size_t rows, size_t cols, int codec, void** out,
                   size_t* out_size) {
  if (!out || !out_size || (n && !data)) return 1;
  if (codec == XKSV_CODEC_TILE16) {
    if (n % 2 || rows == 0 || cols > std::numeric_limits<size_t>::max() / rows || rows * cols != n / 2)
      return 1;
  } else if (codec == XKSV_CODEC_PARALLEL32) {
    if (n % 2 || !rows || rows > 16 || !cols || cols > std::numeric_limits<size_t>::max() / rows ||
        rows * cols != n / 2)
      return 1;
  } else {
    return 1;
  }
  try {
    const std::vector<uint16_t> w = load_words(data, n);
    std::vector<uint8_t> v;
    const bool ok = codec == XKSV_CODEC_TILE16 ? pack_serial(w.data(), rows, cols, v)
                                               : pack_parallel(w.data(), rows, cols, v);
    if (!ok) return 1;
    *out = copy_out(v, out_size);
    return *out ? 0 : 1;
  } catch (...) {
    return 1;
  }
}

void xksv_host_free(void* p) { std::free(p); }

int xksv_host_pack_tensor(const void* data, size_t nbytes, size_t rows, size_t cols, int codec,
                          int threads, uint64_t dst_base, void** payload, size_t* payload_size,
                          xksv_slab** table, size_t* nslabs) {
  if (!payload || !payload_size || !table || !nslabs || (nbytes && !data)) return 1;
  if (codec != XKSV_CODEC_TILE16 && codec != XKSV_CODEC_PARALLEL32) return 1;
  if (!rows || !cols || rows > std::numeric_limits<size_t>::max() / cols ||
      rows * cols * 2 != nbytes)
    return 1;
  try {
    // slab geometry of src/compile.cpp:449-457, 471-479 (1 MiB slabs of whole
    // rows, at most 16 rows; cols <= 524288)
    constexpr uint64_t chunk = 1 << 20;
    if (cols > chunk / 2) return 1;
    const uint64_t rows_per = std::min<uint64_t>(16, chunk / (cols * 2));
    const size_t ns = (rows + rows_per - 1) / rows_per;
    std::vector<std::vector<uint8_t>> enc(ns);
    std::vector<int> kind(ns);
    const uint16_t* w = static_cast<const uint16_t*>(data);
    std::atomic<size_t> next{0};
    std::atomic<bool> fail{false};
    auto work = [&]() {
      std::vector<uint8_t> v;
      for (size_t i; (i = next.fetch_add(1)) < ns;) {
        const size_t r0 = i * rows_per, nr = std::min<size_t>(rows_per, rows - r0);
        const uint16_t* src = w + r0 * cols;
        const bool ok = codec == XKSV_CODEC_TILE16 ? pack_serial(src, nr, cols, v)
                                                   : pack_parallel(src, nr, cols, v);
        if (!ok) {
          fail = true;
          return;
        }
        // keep the encoding only when it is smaller (src/compile.cpp:268-275)
        if (v.size() < nr * cols * 2) {
          enc[i] = v;
          kind[i] = codec;
        } else {
          enc[i].assign(reinterpret_cast<const uint8_t*>(src),
                        reinterpret_cast<const uint8_t*>(src) + nr * cols * 2);
          kind[i] = XKSV_CODEC_RAW;
        }
      }
    };
    int nt = threads > 0 ? threads : int(std::max(1u, std::thread::hardware_concurrency()));
    nt = int(std::min<size_t>(size_t(nt), ns));
    std::vector<std::thread> pool;
    for (int k = 1; k < nt; ++k) pool.emplace_back(work);
    work();
    for (auto& th : pool) th.join();
    if (fail) return 1;
    size_t total = 0;
    for (auto& e : enc) total += e.size();
    auto* pay = static_cast<uint8_t*>(std::malloc(total ? total : 1));
    auto* tab = static_cast<xksv_slab*>(std::malloc(sizeof(xksv_slab) * ns));
    if (!pay || !tab) {
      std::free(pay);
      std::free(tab);
      return 1;
    }
    size_t pos = 0;
    for (size_t i = 0; i < ns; ++i) {
      const size_t r0 = i * rows_per, nr = std::min<size_t>(rows_per, rows - r0);
      std::memcpy(pay + pos, enc[i].data(), enc[i].size());
      tab[i].src_offset = pos;
      tab[i].src_size = enc[i].size();
      tab[i].rows = nr;
      tab[i].cols = cols;
      tab[i].dst_offset = dst_base + r0 * cols * 2;
      tab[i].x_offset = 0;
      tab[i].codec = uint32_t(kind[i]);
      tab[i].flags = 0;
      pos += enc[i].size();
    }
    *payload = pay;
    *payload_size = total;
    *table = tab;
    *nslabs = ns;
    return 0;
  } catch (...) {
    return 1;
  }
}

}  // extern "C"
