/*
 * xksv_oracle.c -- TEST INFRASTRUCTURE ONLY.
 *
 * A plain-C restatement of the XKS VectorForge CPU slab codec, used as the
 * parity checker for the CUDA decoder in this repository.  Only tests/,
 * __graft_entry__.smoke() and bench.py's cpu_baseline leg may load it; the
 * product library never links or calls it.
 *
 * Every function cites the reference file:line whose behaviour it restates
 * (paths are relative to the reference project root).  The restatement is
 * pinned by tests/test_oracle.py against golden vectors produced by the
 * reference library itself (tests/golden/make_golden.py) and, when the
 * reference is compiled here (oracle/_ref), against it on random inputs.
 *
 * Wire formats (docs/format.md:15-30):
 *   serial slab   : u64 count | u64 bit_count | u8 lengths[256] | u8 sm[count]
 *                   | u8 exponent_bits[ceil(bit_count/8)]   (little-endian)
 *   parallel slab : "XKSP2\0\0\0" | u64 rows | u64 cols | u64 chunks
 *                   | u64 seg_len[chunks] | serial segments
 * Elements are stored in 16x16 tile order (src/layout.cpp:32-50).
 */
#include "xksv_oracle.h"

#include <stdlib.h>
#include <string.h>

#define HDR 272u

static uint64_t rd64(const uint8_t* p) {
  uint64_t v = 0;
  for (int i = 0; i < 8; ++i) v |= (uint64_t)p[i] << (8 * i);
  return v;
}
static void wr64(uint8_t* p, uint64_t v) {
  for (int i = 0; i < 8; ++i) p[i] = (uint8_t)(v >> (8 * i));
}

/* ---------------------------------------------------------------- layout --
 * Row-major <-> 16x16 tile order.  src/layout.cpp:32-50 (transform): tiles are
 * visited row-block by row-block, left to right; inside a tile, rows in
 * order; edge tiles are narrower / shorter and hold only real elements.
 * inverse=0 is tile(), inverse=1 is untile().                                */
static void transform(const uint16_t* in, uint16_t* out, size_t rows, size_t cols,
                      int inverse) {
  size_t packed = 0;
  for (size_t r = 0; r < rows; r += 16) {
    size_t nr = rows - r < 16 ? rows - r : 16;
    for (size_t c = 0; c < cols; c += 16) {
      size_t nc = cols - c < 16 ? cols - c : 16;
      for (size_t i = 0; i < nr; ++i) {
        size_t orig = (r + i) * cols + c;
        if (inverse)
          memcpy(out + orig, in + packed, nc * 2);
        else
          memcpy(out + packed, in + orig, nc * 2);
        packed += nc;
      }
    }
  }
}

void oracle_tile(const uint16_t* in, uint16_t* out, size_t rows, size_t cols) {
  transform(in, out, rows, cols, 0);
}
void oracle_untile(const uint16_t* in, uint16_t* out, size_t rows, size_t cols) {
  transform(in, out, rows, cols, 1);
}

/* ------------------------------------------------------------- canonical --
 * src/codec.cpp:11-29.  Symbols with a non-zero length are ordered by
 * (length, symbol); the first code is all zeros; every later code is the
 * previous one plus one (binary, carry to the left) followed by zeros up to
 * its length.  A carry out of the leftmost bit means the lengths are
 * oversubscribed and the codebook is rejected.
 * Codes are held as bit strings (one byte per bit, MSB first) because the
 * format allows lengths up to 255.                                           */
typedef struct {
  uint8_t len[256];
  uint8_t bits[256][256]; /* bits[s][0..len-1] */
} codebook;

static int canonical(const uint8_t* lengths, codebook* cb) {
  int order[256], n = 0;
  for (int s = 0; s < 256; ++s)
    if (lengths[s]) order[n++] = s;
  /* insertion sort by (length, symbol) */
  for (int i = 1; i < n; ++i) {
    int v = order[i], j = i - 1;
    while (j >= 0 && (lengths[order[j]] > lengths[v] ||
                      (lengths[order[j]] == lengths[v] && order[j] > v))) {
      order[j + 1] = order[j];
      --j;
    }
    order[j + 1] = v;
  }
  memset(cb->len, 0, sizeof cb->len);
  uint8_t code[256];
  int clen = 0;
  for (int k = 0; k < n; ++k) {
    int s = order[k], L = lengths[s];
    if (clen == 0) {
      memset(code, 0, (size_t)L);
    } else {
      int i = clen - 1;
      while (i >= 0 && code[i] == 1) code[i--] = 0;
      if (i < 0) return -1; /* oversubscribed (codec.cpp:24) */
      code[i] = 1;
      memset(code + clen, 0, (size_t)(L - clen));
    }
    clen = L;
    cb->len[s] = (uint8_t)L;
    memcpy(cb->bits[s], code, (size_t)L);
  }
  return 0;
}

/* ---------------------------------------------------------------- decode --
 * src/codec.cpp:59-74 (decode_bf16).  A binary tree is grown from the
 * canonical codes; each element walks it one MSB-first bit at a time.
 * Errors, each returning -1: bad section sizes (:60), prefix conflicts
 * (:65-67), running out of bits (:69), a bit with no child (:69), and bits
 * left over after `count` symbols (:72).
 * The word is (sm & 0x80) << 8 | symbol << 7 | (sm & 0x7f)  (:70).          */
typedef struct {
  int child[2];
  int symbol;
} tnode;

static int decode_block(const uint8_t* lengths, const uint8_t* sm, uint64_t count,
                        const uint8_t* ebits, uint64_t nbits, uint16_t* out) {
  codebook* cb = (codebook*)malloc(sizeof(codebook));
  if (!cb) return -1;
  if (canonical(lengths, cb)) {
    free(cb);
    return -1;
  }
  size_t cap = 1 + 256 * 256;
  tnode* tree = (tnode*)malloc(cap * sizeof(tnode));
  if (!tree) {
    free(cb);
    return -1;
  }
  size_t nodes = 1;
  tree[0].child[0] = tree[0].child[1] = -1;
  tree[0].symbol = -1;
  int rc = 0;
  for (int s = 0; s < 256 && !rc; ++s) {
    if (!cb->len[s]) continue;
    int n = 0;
    for (int i = 0; i < cb->len[s]; ++i) {
      if (tree[n].symbol != -1) {
        rc = -1;
        break;
      }
      int b = cb->bits[s][i];
      int nx = tree[n].child[b];
      if (nx < 0) {
        nx = (int)nodes++;
        tree[nx].child[0] = tree[nx].child[1] = -1;
        tree[nx].symbol = -1;
        tree[n].child[b] = nx;
      }
      n = nx;
    }
    if (rc) break;
    if (tree[n].symbol != -1 || tree[n].child[0] != -1 || tree[n].child[1] != -1)
      rc = -1;
    else
      tree[n].symbol = s;
  }
  uint64_t pos = 0;
  for (uint64_t k = 0; k < count && !rc; ++k) {
    int n = 0;
    while (tree[n].symbol < 0) {
      if (pos >= nbits) {
        rc = -1;
        break;
      }
      int b = (ebits[pos / 8] >> (7 - (pos % 8))) & 1;
      ++pos;
      n = tree[n].child[b];
      if (n < 0) {
        rc = -1;
        break;
      }
    }
    if (rc) break;
    uint8_t v = sm[k];
    out[k] = (uint16_t)(((v & 0x80u) << 8) | ((unsigned)tree[n].symbol << 7) | (v & 0x7fu));
  }
  if (!rc && pos != nbits) rc = -1;
  free(tree);
  free(cb);
  return rc;
}

/* Writes words little-endian into a malloc'd buffer (c_api.cpp:12-14, 37). */
static int emit_words(const uint16_t* w, size_t n, void** out, size_t* out_size) {
  uint8_t* b = (uint8_t*)malloc(n ? n * 2 : 1);
  if (!b) return -1;
  for (size_t i = 0; i < n; ++i) {
    b[2 * i] = (uint8_t)(w[i] & 255);
    b[2 * i + 1] = (uint8_t)(w[i] >> 8);
  }
  *out = b;
  *out_size = n * 2;
  return 0;
}

/* src/c_api.cpp:29-40 (xksv_unpack). */
int oracle_unpack(const void* data, size_t n, size_t rows, size_t cols, void** out,
                  size_t* out_size) {
  const uint8_t* p = (const uint8_t*)data;
  if (n < HDR || !rows || cols > SIZE_MAX / rows) return -1;
  uint64_t count = rd64(p), bits = rd64(p + 8);
  if (count != (uint64_t)rows * cols || count > n - HDR ||
      bits / 8 + (bits % 8 != 0) != n - HDR - count)
    return -1;
  uint16_t* packed = (uint16_t*)malloc(count ? count * 2 : 2);
  uint16_t* words = (uint16_t*)malloc(count ? count * 2 : 2);
  int rc = -1;
  if (packed && words &&
      decode_block(p + 16, p + HDR, count, p + HDR + count, bits, packed) == 0) {
    oracle_untile(packed, words, rows, cols);
    rc = emit_words(words, count, out, out_size);
  }
  free(packed);
  free(words);
  return rc;
}

/* src/c_api.cpp:66-85 (xksv_unpack_parallel). */
int oracle_unpack_parallel(const void* data, size_t n, void** out, size_t* out_size) {
  const uint8_t* p = (const uint8_t*)data;
  if (n < 32 || memcmp(p, "XKSP2\0\0\0", 8)) return -1;
  uint64_t rows = rd64(p + 8), cols = rd64(p + 16), chunks = rd64(p + 24);
  if (!rows || rows > 16 || !cols || !chunks || chunks > 32 || cols > SIZE_MAX / rows ||
      chunks > rows * cols || rows * cols > n || rows * cols > SIZE_MAX / 32 ||
      n < 32 + 8 * chunks)
    return -1;
  uint64_t total = rows * cols;
  uint16_t* packed = (uint16_t*)malloc(total * 2);
  uint16_t* words = (uint16_t*)malloc(total * 2);
  int rc = 0;
  if (!packed || !words) rc = -1;
  size_t pos = 32 + 8 * chunks;
  for (uint64_t i = 0; i < chunks && !rc; ++i) {
    uint64_t length = rd64(p + 32 + 8 * i);
    if (length < HDR || length > n - pos) {
      rc = -1;
      break;
    }
    uint64_t cnt = rd64(p + pos), bits = rd64(p + pos + 8);
    uint64_t start = total * i / chunks, end = total * (i + 1) / chunks;
    if (cnt != end - start || cnt > length - HDR ||
        bits / 8 + (bits % 8 != 0) != length - HDR - cnt) {
      rc = -1;
      break;
    }
    if (decode_block(p + pos + 16, p + pos + HDR, cnt, p + pos + HDR + cnt, bits,
                     packed + start))
      rc = -1;
    pos += length;
  }
  if (!rc && pos != n) rc = -1;
  if (!rc) {
    oracle_untile(packed, words, rows, cols);
    rc = emit_words(words, total, out, out_size);
  }
  free(packed);
  free(words);
  return rc;
}

/* ---------------------------------------------------------------- encode --
 * src/codec.cpp:32-58 (encode_bf16).  Exponent byte (w >> 7) & 255 is
 * Huffman coded; leaves are created in symbol order for every non-zero
 * frequency; the two smallest (frequency, node index) pairs are merged
 * repeatedly (std::priority_queue with std::greater, so ties break on the
 * lower node index); a leaf's length is max(depth, 1) and depth > 255 is an
 * error.  The sign and mantissa go to one raw byte ((w >> 8) & 0x80) | (w &
 * 0x7f); code bits are appended MSB first.                                   */
typedef struct {
  uint64_t freq;
  int symbol, left, right;
} hnode;
typedef struct {
  uint64_t f;
  int i;
} hitem;

static int hless(hitem a, hitem b) { return a.f < b.f || (a.f == b.f && a.i < b.i); }
static void hpush(hitem* h, int* n, hitem v) {
  int k = (*n)++;
  h[k] = v;
  while (k > 0) {
    int p = (k - 1) / 2;
    if (!hless(h[k], h[p])) break;
    hitem t = h[k];
    h[k] = h[p];
    h[p] = t;
    k = p;
  }
}
static hitem hpop(hitem* h, int* n) {
  hitem top = h[0];
  h[0] = h[--(*n)];
  int k = 0;
  for (;;) {
    int l = 2 * k + 1, r = l + 1, m = k;
    if (l < *n && hless(h[l], h[m])) m = l;
    if (r < *n && hless(h[r], h[m])) m = r;
    if (m == k) break;
    hitem t = h[k];
    h[k] = h[m];
    h[m] = t;
    k = m;
  }
  return top;
}

/* Appends one encoded block for `words` to buf (which has room), returning
 * the number of bytes written or -1. */
static long long encode_block(const uint16_t* words, uint64_t count, uint8_t* buf) {
  uint64_t freq[256] = {0};
  for (uint64_t i = 0; i < count; ++i) ++freq[(words[i] >> 7) & 255];
  hnode nodes[512];
  hitem heap[512];
  int nn = 0, hn = 0;
  for (int s = 0; s < 256; ++s)
    if (freq[s]) {
      nodes[nn] = (hnode){freq[s], s, -1, -1};
      hpush(heap, &hn, (hitem){freq[s], nn});
      ++nn;
    }
  while (hn > 1) {
    hitem a = hpop(heap, &hn), b = hpop(heap, &hn);
    if (a.f > UINT64_MAX - b.f) return -1;
    nodes[nn] = (hnode){a.f + b.f, -1, a.i, b.i};
    hpush(heap, &hn, (hitem){a.f + b.f, nn});
    ++nn;
  }
  uint8_t lengths[256] = {0};
  if (hn == 1) {
    int stack[512], depth[512], sp = 0;
    stack[sp] = heap[0].i;
    depth[sp++] = 0;
    while (sp) {
      --sp;
      int i = stack[sp], d = depth[sp];
      if (nodes[i].symbol >= 0) {
        if (d > 255) return -1;
        lengths[nodes[i].symbol] = (uint8_t)(d > 1 ? d : 1);
      } else {
        stack[sp] = nodes[i].left;
        depth[sp++] = d + 1;
        stack[sp] = nodes[i].right;
        depth[sp++] = d + 1;
      }
    }
  }
  codebook* cb = (codebook*)malloc(sizeof(codebook));
  if (!cb || canonical(lengths, cb)) {
    free(cb);
    return -1;
  }
  uint64_t bits = 0;
  for (uint64_t i = 0; i < count; ++i) bits += cb->len[(words[i] >> 7) & 255];
  uint64_t ebytes = bits / 8 + (bits % 8 != 0);
  wr64(buf, count);
  wr64(buf + 8, bits);
  memcpy(buf + 16, lengths, 256);
  uint8_t* sm = buf + HDR;
  uint8_t* e = sm + count;
  memset(e, 0, ebytes);
  uint64_t pos = 0;
  for (uint64_t i = 0; i < count; ++i) {
    uint16_t w = words[i];
    sm[i] = (uint8_t)(((w >> 8) & 0x80) | (w & 0x7f));
    int s = (w >> 7) & 255;
    for (int k = 0; k < cb->len[s]; ++k, ++pos)
      if (cb->bits[s][k]) e[pos / 8] |= (uint8_t)(0x80u >> (pos % 8));
  }
  free(cb);
  return (long long)(HDR + count + ebytes);
}

/* Worst case per block: header + count + ceil(count * 255 / 8). */
static size_t block_bound(uint64_t count) { return HDR + count + (count * 255 + 7) / 8; }

static uint16_t* load_words(const void* data, size_t n) {
  const uint8_t* p = (const uint8_t*)data;
  uint16_t* w = (uint16_t*)malloc(n ? n : 2);
  if (!w) return NULL;
  for (size_t i = 0; i < n / 2; ++i) w[i] = (uint16_t)(p[2 * i] | (p[2 * i + 1] << 8));
  return w;
}

/* src/c_api.cpp:18-28 (xksv_pack). */
int oracle_pack(const void* data, size_t n, size_t rows, size_t cols, void** out,
                size_t* out_size) {
  if (n % 2 || rows == 0 || cols > SIZE_MAX / rows || rows * cols != n / 2) return -1;
  uint16_t* w = load_words(data, n);
  uint16_t* t = (uint16_t*)malloc(n ? n : 2);
  uint8_t* buf = (uint8_t*)malloc(block_bound(n / 2));
  int rc = -1;
  if (w && t && buf) {
    oracle_tile(w, t, rows, cols);
    long long sz = encode_block(t, n / 2, buf);
    if (sz >= 0) {
      *out = buf;
      *out_size = (size_t)sz;
      buf = NULL;
      rc = 0;
    }
  }
  free(w);
  free(t);
  free(buf);
  return rc;
}

/* src/c_api.cpp:44-65 (xksv_pack_parallel): min(32, n) contiguous substreams
 * of the tiled slab, substream i covering [n*i/chunks, n*(i+1)/chunks).      */
int oracle_pack_parallel(const void* data, size_t n, size_t rows, size_t cols, void** out,
                         size_t* out_size) {
  if (n % 2 || !rows || rows > 16 || !cols || cols > SIZE_MAX / rows ||
      rows * cols != n / 2 || rows * cols > SIZE_MAX / 32)
    return -1;
  uint64_t total = n / 2;
  uint64_t chunks = total < 32 ? total : 32;
  uint16_t* w = load_words(data, n);
  uint16_t* t = (uint16_t*)malloc(n);
  size_t cap = 32 + 8 * chunks;
  for (uint64_t i = 0; i < chunks; ++i)
    cap += block_bound(total * (i + 1) / chunks - total * i / chunks);
  uint8_t* buf = (uint8_t*)malloc(cap);
  int rc = -1;
  if (w && t && buf) {
    oracle_tile(w, t, rows, cols);
    memcpy(buf, "XKSP2\0\0\0", 8);
    wr64(buf + 8, rows);
    wr64(buf + 16, cols);
    wr64(buf + 24, chunks);
    size_t pos = 32 + 8 * chunks;
    rc = 0;
    for (uint64_t i = 0; i < chunks; ++i) {
      uint64_t s = total * i / chunks, e = total * (i + 1) / chunks;
      long long sz = encode_block(t + s, e - s, buf + pos);
      if (sz < 0) {
        rc = -1;
        break;
      }
      wr64(buf + 32 + 8 * i, (uint64_t)sz);
      pos += (size_t)sz;
    }
    if (!rc) {
      *out = buf;
      *out_size = pos;
      buf = NULL;
    }
  }
  free(w);
  free(t);
  free(buf);
  return rc;
}

void oracle_free(void* p) { free(p); }

/* Decodes one slab of either kind (codec 1 = serial, 2 = parallel) straight
 * into a caller buffer of rows*cols*2 bytes; used by the CPU baseline timer. */
int oracle_decode_into(const void* data, size_t n, size_t rows, size_t cols, int codec,
                       void* dst) {
  void* out = NULL;
  size_t sz = 0;
  int rc = codec == 2 ? oracle_unpack_parallel(data, n, &out, &sz)
                      : oracle_unpack(data, n, rows, cols, &out, &sz);
  if (rc) return rc;
  if (sz != rows * cols * 2) rc = -1;
  else memcpy(dst, out, sz);
  free(out);
  return rc;
}
