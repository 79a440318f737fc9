// rkv_kvc.cpp -- the KVC on-disk format for pooled sequences (prefix
// persistence), after rsLLM's plan in docs/03-HLD.md:242-282:
//
//   file name:  SHA1 of the token ids (little-endian u32) in hex + ".kvc"
//   header (48 bytes, little-endian):
//     "KVC" | version u8 (1) | quant_bits u32 (8: E4M3FN) | reason u32
//     (COLD / CONTINUED / EVICT / SHUTDOWN) | token_count u64 | ctx_size u64 |
//     created_at u64 (unix seconds) | payload_bytes u64 | reserved u32 (0)
//   body:
//     rendered_text: length u32 + bytes (human-readable, for debugging)
//     engine payload: magic u32 0x34565344 ("DSV4") | version u32 (1) |
//       vocab_size u32 | n_layers u32 | head_dim u32 (576 stored lanes) |
//       page_tokens u32 (64) | n_pages u32 | token_ids u32[token_count] |
//       for each layer, for each page of the sequence: the page as stored in
//       the pool (codes | scales | RoPE, 43008 bytes); rows at or beyond
//       token_count are written as zeros.
//
// The plan lists 44 bytes of header fields under a 48-byte header; the four
// bytes after payload_bytes are written as zero.  The rendered text carries a
// length prefix so that a reader can find the engine payload.
//
// Pages move through a bounded staging area (pack / unpack kernels into a
// device buffer, one copy to or from pinned host memory per chunk).
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>
#include <string.h>
#include <time.h>

#include <string>
#include <vector>

#include "rkv_common.cuh"
#include "rkv_host.h"

namespace rkv {
namespace {

// ---- SHA-1 (FIPS 180-4) ---------------------------------------------------
struct Sha1 {
  uint32_t h[5] = {0x67452301u, 0xEFCDAB89u, 0x98BADCFEu, 0x10325476u, 0xC3D2E1F0u};
  uint8_t block[64];
  size_t used = 0;
  uint64_t total = 0;

  static uint32_t rol(uint32_t x, int n) { return (x << n) | (x >> (32 - n)); }

  void compress(const uint8_t* b) {
    uint32_t w[80];
    for (int t = 0; t < 16; ++t)
      w[t] = (uint32_t)b[4 * t] << 24 | (uint32_t)b[4 * t + 1] << 16 | (uint32_t)b[4 * t + 2] << 8 | b[4 * t + 3];
    for (int t = 16; t < 80; ++t) w[t] = rol(w[t - 3] ^ w[t - 8] ^ w[t - 14] ^ w[t - 16], 1);
    uint32_t a = h[0], bb = h[1], c = h[2], d = h[3], e = h[4];
    for (int t = 0; t < 80; ++t) {
      uint32_t f, k;
      if (t < 20) {
        f = (bb & c) | (~bb & d);
        k = 0x5A827999u;
      } else if (t < 40) {
        f = bb ^ c ^ d;
        k = 0x6ED9EBA1u;
      } else if (t < 60) {
        f = (bb & c) | (bb & d) | (c & d);
        k = 0x8F1BBCDCu;
      } else {
        f = bb ^ c ^ d;
        k = 0xCA62C1D6u;
      }
      const uint32_t tmp = rol(a, 5) + f + e + k + w[t];
      e = d;
      d = c;
      c = rol(bb, 30);
      bb = a;
      a = tmp;
    }
    h[0] += a;
    h[1] += bb;
    h[2] += c;
    h[3] += d;
    h[4] += e;
  }

  void update(const uint8_t* p, size_t n) {
    total += n;
    while (n > 0) {
      const size_t take = n < 64 - used ? n : 64 - used;
      memcpy(block + used, p, take);
      used += take;
      p += take;
      n -= take;
      if (used == 64) {
        compress(block);
        used = 0;
      }
    }
  }

  void hex(char out[41]) {
    const uint64_t bits = total * 8;
    const uint8_t one = 0x80, zero = 0;
    update(&one, 1);
    while (used != 56) update(&zero, 1);
    uint8_t len[8];
    for (int i = 0; i < 8; ++i) len[i] = (uint8_t)(bits >> (56 - 8 * i));
    update(len, 8);
    for (int i = 0; i < 5; ++i) snprintf(out + 8 * i, 9, "%08x", h[i]);
  }
};

void name_of(const int32_t* ids, int64_t n, char out[46]) {
  Sha1 s;
  for (int64_t i = 0; i < n; ++i) {
    const uint32_t v = (uint32_t)ids[i];
    const uint8_t le[4] = {(uint8_t)v, (uint8_t)(v >> 8), (uint8_t)(v >> 16), (uint8_t)(v >> 24)};
    s.update(le, 4);
  }
  s.hex(out);
  memcpy(out + 40, ".kvc", 5);
}

constexpr uint32_t kPayloadMagic = 0x34565344u;  // "DSV4"
constexpr int64_t kStageBudget = 64ll << 20;

void put32(std::vector<uint8_t>& v, uint32_t x) {
  for (int i = 0; i < 4; ++i) v.push_back((uint8_t)(x >> (8 * i)));
}
void put64(std::vector<uint8_t>& v, uint64_t x) {
  for (int i = 0; i < 8; ++i) v.push_back((uint8_t)(x >> (8 * i)));
}
uint32_t get32(const uint8_t* p) { return (uint32_t)p[0] | (uint32_t)p[1] << 8 | (uint32_t)p[2] << 16 | (uint32_t)p[3] << 24; }
uint64_t get64(const uint8_t* p) { return (uint64_t)get32(p) | (uint64_t)get32(p + 4) << 32; }

// Staging buffers for page chunks, released on scope exit.
struct Staging {
  void* dev = nullptr;
  void* host = nullptr;
  int32_t* dpages = nullptr;
  ~Staging() {
    if (dev) cudaFree(dev);
    if (host) cudaFreeHost(host);
    if (dpages) cudaFree(dpages);
  }
  cudaError_t alloc(int64_t bytes, int64_t n_pages) {
    cudaError_t e = cudaMalloc(&dev, (size_t)bytes);
    if (e == cudaSuccess) e = cudaMallocHost(&host, (size_t)bytes);
    if (e == cudaSuccess) e = cudaMalloc(&dpages, (size_t)(n_pages > 0 ? n_pages : 1) * 4);
    return e;
  }
};

struct File {
  FILE* f = nullptr;
  ~File() {
    if (f) fclose(f);
  }
};

rkv_status parse_header(const uint8_t* b, rkv_kvc_header* out, const char* what) {
  if (memcmp(b, "KVC", 3) != 0) return fail(RKV_ERR_INVALID_ARGUMENT, "%s: not a KVC file (bad magic)", what);
  out->version = b[3];
  out->quant_bits = get32(b + 4);
  out->reason = get32(b + 8);
  out->reserved = get32(b + 44);
  out->token_count = get64(b + 12);
  out->ctx_size = get64(b + 20);
  out->created_at = get64(b + 28);
  out->payload_bytes = get64(b + 36);
  if (out->version != 1) return fail(RKV_ERR_INVALID_ARGUMENT, "%s: unsupported KVC version %u", what, out->version);
  if (out->quant_bits != 8)
    return fail(RKV_ERR_INVALID_ARGUMENT, "%s: KVC written with %u-bit KV, this pool stores 8-bit E4M3FN", what,
                out->quant_bits);
  return RKV_OK;
}

}  // namespace
}  // namespace rkv

extern "C" {

rkv_status rkv_kvc_name(const int32_t* token_ids, int64_t n_tokens, char out[46]) {
  using namespace rkv;
  if (!out || n_tokens < 0 || (n_tokens > 0 && !token_ids))
    return fail(RKV_ERR_INVALID_ARGUMENT, "rkv_kvc_name: token_ids (n > 0) and out are required");
  name_of(token_ids, n_tokens, out);
  clear_error();
  return RKV_OK;
}

rkv_status rkv_kvc_read_header(const char* path, rkv_kvc_header* out) {
  using namespace rkv;
  if (!path || !out) return fail(RKV_ERR_INVALID_ARGUMENT, "rkv_kvc_read_header: path and out are required");
  File fh;
  fh.f = fopen(path, "rb");
  if (!fh.f) return fail(RKV_ERR_INVALID_ARGUMENT, "rkv_kvc_read_header: cannot open %s", path);
  uint8_t b[RKV_KVC_HEADER_BYTES];
  if (fread(b, 1, sizeof b, fh.f) != sizeof b)
    return fail(RKV_ERR_INVALID_ARGUMENT, "rkv_kvc_read_header: %s is shorter than a header", path);
  rkv_status st = parse_header(b, out, "rkv_kvc_read_header");
  if (st == RKV_OK) clear_error();
  return st;
}

rkv_status rkv_kvc_save(rkv_pool* pool, int64_t seq, const int32_t* token_ids, int64_t n_tokens, uint32_t reason,
                        uint32_t vocab_size, const char* text, int64_t text_len, const char* dir, char* path_out,
                        int64_t path_cap, rkv_stream_t stream) {
  using namespace rkv;
  const char* what = "rkv_kvc_save";
  if (!pool || !dir || n_tokens <= 0 || !token_ids || text_len < 0 || (text_len > 0 && !text) ||
      text_len > UINT32_MAX || n_tokens > UINT32_MAX)
    return fail(RKV_ERR_INVALID_ARGUMENT, "%s: pool, dir, token_ids (n > 0) are required", what);
  if (pool_device(pool) < 0) return fail(RKV_ERR_INVALID_ARGUMENT, "%s: a plan-only pool holds no KV bytes", what);
  if (reason > RKV_KVC_SHUTDOWN) return fail(RKV_ERR_INVALID_ARGUMENT, "%s: unknown reason %u", what, reason);
  int64_t len = 0, n_seq_pages = 0;
  rkv_status st = rkv_seq_info(pool, seq, &len, &n_seq_pages);
  if (st != RKV_OK) return st;
  if (len < n_tokens)
    return fail_shape("n_tokens", len, n_tokens, "%s: sequence %lld holds %lld tokens, %lld requested", what,
                      (long long)seq, (long long)len, (long long)n_tokens);
  std::vector<int32_t> table((size_t)n_seq_pages);
  st = rkv_seq_page_table(pool, seq, table.data(), n_seq_pages);
  if (st != RKV_OK) return st;
  const int64_t n_pages = (n_tokens + kPageTokens - 1) / kPageTokens;
  rkv_pool_view view;
  rkv_pool_get_view(pool, &view);
  cudaSetDevice(pool_device(pool));

  std::string path = std::string(dir) + "/";
  char name[46];
  name_of(token_ids, n_tokens, name);
  path += name;
  if (path_out && path_cap < (int64_t)path.size() + 1)
    return fail(RKV_ERR_INVALID_ARGUMENT, "%s: path_out needs %zu bytes", what, path.size() + 1);

  const uint64_t body_fixed = 4 + (uint64_t)text_len + 7 * 4 + 4 * (uint64_t)n_tokens;
  const uint64_t page_bytes = (uint64_t)view.n_layers * n_pages * kPageBytes;
  std::vector<uint8_t> head;
  head.insert(head.end(), {'K', 'V', 'C', 1});
  put32(head, 8);
  put32(head, reason);
  put64(head, (uint64_t)n_tokens);
  put64(head, (uint64_t)n_pages * kPageTokens);
  put64(head, (uint64_t)time(nullptr));
  put64(head, body_fixed + page_bytes);
  put32(head, 0);
  put32(head, (uint32_t)text_len);
  head.insert(head.end(), text, text + text_len);
  put32(head, kPayloadMagic);
  put32(head, 1);
  put32(head, vocab_size);
  put32(head, (uint32_t)view.n_layers);
  put32(head, (uint32_t)(kLatent + kRope));
  put32(head, (uint32_t)kPageTokens);
  put32(head, (uint32_t)n_pages);
  for (int64_t i = 0; i < n_tokens; ++i) put32(head, (uint32_t)token_ids[i]);

  const int64_t chunk = n_pages * kPageBytes <= kStageBudget ? n_pages : kStageBudget / kPageBytes;
  Staging sg;
  cudaError_t e = sg.alloc(chunk * kPageBytes, n_pages);
  if (e == cudaSuccess)
    e = cudaMemcpyAsync(sg.dpages, table.data(), (size_t)n_pages * 4, cudaMemcpyHostToDevice, (cudaStream_t)stream);
  if (e != cudaSuccess) return fail(RKV_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  File fh;
  const std::string tmp = path + ".part";
  fh.f = fopen(tmp.c_str(), "wb");
  if (!fh.f) return fail(RKV_ERR_INVALID_ARGUMENT, "%s: cannot create %s", what, tmp.c_str());
  if (fwrite(head.data(), 1, head.size(), fh.f) != head.size())
    return fail(RKV_ERR_INVALID_ARGUMENT, "%s: write to %s failed", what, tmp.c_str());
  const int tail_rows = (int)(n_tokens - (n_pages - 1) * kPageTokens);  // valid rows of the last page
  for (int32_t l = 0; l < view.n_layers; ++l) {
    for (int64_t p0 = 0; p0 < n_pages; p0 += chunk) {
      const int64_t np = n_pages - p0 < chunk ? n_pages - p0 : chunk;
      st = rkv_pack_pages(&view, l, 1, sg.dpages + p0, np, sg.dev, pool_status_word(pool), stream);
      if (st != RKV_OK) return st;
      e = cudaMemcpyAsync(sg.host, sg.dev, (size_t)(np * kPageBytes), cudaMemcpyDeviceToHost, (cudaStream_t)stream);
      if (e == cudaSuccess) e = cudaStreamSynchronize((cudaStream_t)stream);
      if (e != cudaSuccess) return fail(RKV_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
      if (p0 + np == n_pages && tail_rows < kPageTokens) {  // rows of no token of this sequence
        uint8_t* last = static_cast<uint8_t*>(sg.host) + (np - 1) * kPageBytes;
        memset(last + codes_off(tail_rows), 0, (size_t)(kPageTokens - tail_rows) * kLatent);
        memset(last + scales_off(tail_rows), 0, (size_t)(kPageTokens - tail_rows) * kBlocks * 4);
        memset(last + rope_off(tail_rows), 0, (size_t)(kPageTokens - tail_rows) * kRope * 2);
      }
      if (fwrite(sg.host, 1, (size_t)(np * kPageBytes), fh.f) != (size_t)(np * kPageBytes))
        return fail(RKV_ERR_INVALID_ARGUMENT, "%s: write to %s failed", what, tmp.c_str());
    }
  }
  uint32_t bits = 0;
  rkv_pool_device_status(pool, &bits);
  if (bits) return fail(rkv_status_from_bits(bits), "%s: the sequence's page table names a page outside the pool", what);
  const bool closed = fclose(fh.f) == 0;
  fh.f = nullptr;
  if (!closed || rename(tmp.c_str(), path.c_str()) != 0)
    return fail(RKV_ERR_INVALID_ARGUMENT, "%s: cannot finish %s", what, path.c_str());
  if (path_out) memcpy(path_out, path.c_str(), path.size() + 1);
  clear_error();
  return RKV_OK;
}

rkv_status rkv_kvc_load(rkv_pool* pool, const char* path, int32_t* token_ids_out, int64_t cap, int64_t* n_tokens_out,
                        int64_t* seq_out, int32_t insert_prefix, rkv_stream_t stream) {
  using namespace rkv;
  const char* what = "rkv_kvc_load";
  if (!pool || !path || !seq_out) return fail(RKV_ERR_INVALID_ARGUMENT, "%s: pool, path and seq_out are required", what);
  if (pool_device(pool) < 0) return fail(RKV_ERR_INVALID_ARGUMENT, "%s: a plan-only pool holds no KV bytes", what);
  File fh;
  fh.f = fopen(path, "rb");
  if (!fh.f) return fail(RKV_ERR_INVALID_ARGUMENT, "%s: cannot open %s", what, path);
  uint8_t hb[RKV_KVC_HEADER_BYTES];
  rkv_kvc_header h;
  if (fread(hb, 1, sizeof hb, fh.f) != sizeof hb) return fail(RKV_ERR_INVALID_ARGUMENT, "%s: truncated header", what);
  rkv_status st = parse_header(hb, &h, what);
  if (st != RKV_OK) return st;
  uint8_t w[4];
  if (fread(w, 1, 4, fh.f) != 4) return fail(RKV_ERR_INVALID_ARGUMENT, "%s: truncated body", what);
  if (fseek(fh.f, (long)get32(w), SEEK_CUR) != 0) return fail(RKV_ERR_INVALID_ARGUMENT, "%s: truncated text", what);
  uint8_t ph[28];
  if (fread(ph, 1, sizeof ph, fh.f) != sizeof ph) return fail(RKV_ERR_INVALID_ARGUMENT, "%s: truncated payload", what);
  rkv_pool_view view;
  rkv_pool_get_view(pool, &view);
  const uint32_t n_layers = get32(ph + 12), head_dim = get32(ph + 16), page_tokens = get32(ph + 20),
                 n_pages = get32(ph + 24);
  if (get32(ph) != kPayloadMagic || get32(ph + 4) != 1)
    return fail(RKV_ERR_INVALID_ARGUMENT, "%s: unknown engine payload", what);
  const int64_t n_tokens = (int64_t)h.token_count;
  if ((int32_t)n_layers != view.n_layers || head_dim != (uint32_t)(kLatent + kRope) ||
      page_tokens != (uint32_t)kPageTokens || (int64_t)n_pages != (n_tokens + kPageTokens - 1) / kPageTokens ||
      n_tokens <= 0)
    return fail(RKV_ERR_SHAPE_MISMATCH, "%s: file holds %u layers of %u-lane rows in %u-token pages, pool has %d layers",
                what, n_layers, head_dim, page_tokens, view.n_layers);
  std::vector<int32_t> tokens((size_t)n_tokens);
  std::vector<uint8_t> tb((size_t)n_tokens * 4);
  if (fread(tb.data(), 1, tb.size(), fh.f) != tb.size())
    return fail(RKV_ERR_INVALID_ARGUMENT, "%s: truncated token ids", what);
  for (int64_t i = 0; i < n_tokens; ++i) tokens[(size_t)i] = (int32_t)get32(tb.data() + 4 * i);
  if (n_tokens_out) *n_tokens_out = n_tokens;
  if (token_ids_out && cap < n_tokens)
    return fail(RKV_ERR_SHAPE_MISMATCH, "%s: token_ids_out holds %lld ids, the file %lld", what, (long long)cap,
                (long long)n_tokens);

  cudaSetDevice(pool_device(pool));
  int64_t seq = -1;
  st = rkv_seq_create(pool, &seq);
  if (st != RKV_OK) return st;
  st = rkv_seq_reserve(pool, 1, &seq, &n_tokens, nullptr, stream);
  if (st != RKV_OK) {
    rkv_seq_free(pool, seq);
    return st;
  }
  std::vector<int32_t> table((size_t)n_pages);
  rkv_seq_page_table(pool, seq, table.data(), n_pages);
  const int64_t chunk = (int64_t)n_pages * kPageBytes <= kStageBudget ? n_pages : kStageBudget / kPageBytes;
  Staging sg;
  cudaError_t e = sg.alloc(chunk * kPageBytes, n_pages);
  if (e == cudaSuccess)
    e = cudaMemcpyAsync(sg.dpages, table.data(), (size_t)n_pages * 4, cudaMemcpyHostToDevice, (cudaStream_t)stream);
  for (int32_t l = 0; e == cudaSuccess && l < view.n_layers; ++l) {
    for (int64_t p0 = 0; p0 < n_pages; p0 += chunk) {
      const int64_t np = n_pages - p0 < chunk ? (int64_t)n_pages - p0 : chunk;
      if (fread(sg.host, 1, (size_t)(np * kPageBytes), fh.f) != (size_t)(np * kPageBytes)) {
        rkv_seq_free(pool, seq);
        return fail(RKV_ERR_INVALID_ARGUMENT, "%s: truncated page data", what);
      }
      e = cudaMemcpyAsync(sg.dev, sg.host, (size_t)(np * kPageBytes), cudaMemcpyHostToDevice, (cudaStream_t)stream);
      if (e != cudaSuccess) break;
      st = rkv_unpack_pages(&view, l, 1, sg.dpages + p0, np, sg.dev, pool_status_word(pool), stream);
      if (st != RKV_OK) {
        rkv_seq_free(pool, seq);
        return st;
      }
      e = cudaStreamSynchronize((cudaStream_t)stream);  // the pinned buffer is reused for the next chunk
      if (e != cudaSuccess) break;
    }
  }
  if (e != cudaSuccess) {
    rkv_seq_free(pool, seq);
    return fail(RKV_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  }
  if (insert_prefix) {
    st = rkv_prefix_insert(pool, tokens.data(), n_tokens, seq);
    if (st != RKV_OK) return st;
  }
  if (token_ids_out) memcpy(token_ids_out, tokens.data(), (size_t)n_tokens * 4);
  *seq_out = seq;
  clear_error();
  return RKV_OK;
}

}  // extern "C"
