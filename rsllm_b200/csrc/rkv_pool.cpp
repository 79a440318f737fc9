// rkv_pool.cpp -- host side of the paged KV pool: page allocator, per-sequence
// page tables, radix prefix store, copy-on-write, LRU eviction, compaction.
//
// rsLLM has no paged pool yet.  Its plan (docs/03-HLD.md:363-376):
//   8.1 paged KV: a block table per session, free-list allocation, blocks
//       freed when a session ends or is evicted, shared-prefix blocks
//       refcounted across sessions;
//   8.2 radix-tree prefix cache: a node is a token span plus its block ids;
//       insertion splits or adds nodes; lookup returns the longest common
//       prefix and its reusable blocks; LRU eviction.
// This file implements that plan with deterministic rules (so a CPU model can
// check it exactly):
//   * allocation takes the lowest-numbered free page;
//   * appending into a partially filled last page that another owner shares
//     first copies it to a fresh page (copy-on-write);
//   * eviction drops, in increasing (last use, kind, id) order, released
//     sequences and radix leaves until the requested number of pages is free;
//   * compaction moves the highest live page into the lowest hole until every
//     live page is below the live-page count, and rewrites every page table.
// The pool is single-owner (like rsLLM's `&mut` caches): calls on one pool
// must not overlap.  Device work (page copies, table remaps) is enqueued on
// the caller's stream through the kernels of rkv_pages.cu.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <cstring>
#include <map>
#include <set>
#include <tuple>
#include <unordered_map>
#include <vector>

#include "../../include/rsllm_kv_cuda.h"
#include "rkv_host.h"

namespace {

constexpr int64_t kPageTokens = RKV_PAGE_TOKENS;

// Free pages as a two-level bitmap (bit = free): lowest free page in a few
// word scans for millions of pages.
class FreeMap {
 public:
  void reset(int64_t n) {
    n_ = n;
    words_.assign((size_t)((n + 63) / 64), 0ull);
    summary_.assign((words_.size() + 63) / 64, 0ull);
    count_ = 0;
    for (int64_t p = 0; p < n; ++p) set_free(p);
  }
  void set_free(int64_t p) {
    uint64_t& w = words_[(size_t)(p >> 6)];
    if (!(w >> (p & 63) & 1ull)) ++count_;
    w |= 1ull << (p & 63);
    summary_[(size_t)(p >> 12)] |= 1ull << ((p >> 6) & 63);
  }
  void set_used(int64_t p) {
    uint64_t& w = words_[(size_t)(p >> 6)];
    if (w >> (p & 63) & 1ull) --count_;
    w &= ~(1ull << (p & 63));
    if (w == 0) summary_[(size_t)(p >> 12)] &= ~(1ull << ((p >> 6) & 63));
  }
  bool is_free(int64_t p) const { return words_[(size_t)(p >> 6)] >> (p & 63) & 1ull; }
  int64_t lowest() const {
    for (size_t s = 0; s < summary_.size(); ++s) {
      if (!summary_[s]) continue;
      const size_t wi = s * 64 + (size_t)__builtin_ctzll(summary_[s]);
      return (int64_t)(wi * 64 + (size_t)__builtin_ctzll(words_[wi]));
    }
    return -1;
  }
  int64_t count() const { return count_; }
  // one past the highest used page (0 if none)
  int64_t high_water() const {
    for (int64_t wi = (int64_t)words_.size() - 1; wi >= 0; --wi) {
      const int64_t valid = std::min<int64_t>(64, n_ - wi * 64);
      const uint64_t mask = valid == 64 ? ~0ull : ((1ull << valid) - 1ull);
      const uint64_t used = ~words_[(size_t)wi] & mask;
      if (used) return wi * 64 + 64 - __builtin_clzll(used);
    }
    return 0;
  }

 private:
  int64_t n_ = 0, count_ = 0;
  std::vector<uint64_t> words_, summary_;
};

struct Seq {
  std::vector<int32_t> pages;  // page of token t is pages[t / 64]
  int64_t len = 0;
  uint64_t last_use = 0;
  bool released = false;
};

// Radix node: tokens [start, start + span) of every sequence through it, and
// the pages holding page indices [start / 64, ceil((start + span) / 64)).  A
// page straddling a node boundary is listed by both nodes; the deeper node's
// copy holds the longer valid prefix.
struct Node {
  int32_t parent = -1;
  int64_t start = 0;
  std::vector<int32_t> tokens;
  std::vector<int32_t> pages;
  std::map<int32_t, int32_t> children;  // first token -> node
  uint64_t last_use = 0;
  bool alive = false;
};

enum Kind { kSeqKind = 0, kNodeKind = 1 };

}  // namespace

struct rkv_pool {
  int device = 0;
  int64_t n_pages = 0;
  int32_t n_layers = 0;
  void* storage = nullptr;
  bool owns_storage = false;
  int32_t* d_moves = nullptr;  // [2][n_pages] src, dst
  int32_t* d_remap = nullptr;  // [n_pages]
  uint32_t* d_status = nullptr;
  std::vector<uint32_t> ref;
  FreeMap free;
  std::unordered_map<int64_t, Seq> seqs;
  int64_t next_seq = 1;
  std::vector<Node> nodes;  // nodes[0] = root
  std::vector<int32_t> free_nodes;
  uint64_t tick = 0;
  std::vector<int32_t> last_remap;
  std::vector<int32_t> pending_src, pending_dst;  // copy-on-write copies not yet enqueued
  std::vector<int32_t> planned_src, planned_dst;  // plan-only pools: moves handed to the caller

  rkv_pool_view view() const { return rkv_pool_view{storage, n_pages, n_layers, 0}; }

  int32_t alloc_page() {
    const int64_t p = free.lowest();
    if (p < 0) return -1;
    free.set_used(p);
    ref[(size_t)p] = 1;
    return (int32_t)p;
  }
  void incref(int32_t p) { ++ref[(size_t)p]; }
  // returns true when the page became free
  bool decref(int32_t p) {
    if (--ref[(size_t)p] == 0) {
      free.set_free(p);
      return true;
    }
    return false;
  }

  int32_t new_node() {
    int32_t id;
    if (!free_nodes.empty()) {
      id = free_nodes.back();
      free_nodes.pop_back();
      nodes[(size_t)id] = Node();
    } else {
      id = (int32_t)nodes.size();
      nodes.emplace_back();
    }
    nodes[(size_t)id].alive = true;
    return id;
  }
};

namespace {

using rkv::fail;

rkv_status enqueue_copies(rkv_pool* P, const std::vector<int32_t>& src, const std::vector<int32_t>& dst,
                          rkv_stream_t stream) {
  if (src.empty()) return RKV_OK;
  if (P->device < 0) {  // plan-only pool: the caller moves the pages (rkv_pool_take_moves)
    P->planned_src.insert(P->planned_src.end(), src.begin(), src.end());
    P->planned_dst.insert(P->planned_dst.end(), dst.begin(), dst.end());
    return RKV_OK;
  }
  const size_t n = src.size();
  cudaError_t e = cudaSetDevice(P->device);
  if (e == cudaSuccess) e = cudaMemcpyAsync(P->d_moves, src.data(), n * 4, cudaMemcpyHostToDevice, (cudaStream_t)stream);
  if (e == cudaSuccess)
    e = cudaMemcpyAsync(P->d_moves + P->n_pages, dst.data(), n * 4, cudaMemcpyHostToDevice, (cudaStream_t)stream);
  if (e != cudaSuccess) return fail(RKV_ERR_CUDA, "page copy upload: %s", cudaGetErrorString(e));
  // pageable sources: the copies above have consumed the host vectors on return
  const rkv_pool_view v = P->view();
  return rkv_copy_pages(&v, P->d_moves, P->d_moves + P->n_pages, (int64_t)n, P->d_status, stream);
}

Seq* find_seq(rkv_pool* P, int64_t id) {
  auto it = P->seqs.find(id);
  return it == P->seqs.end() ? nullptr : &it->second;
}

// Plans copy-on-write of the partially filled last page of `s` if shared and
// the new pages for `n` more tokens; returns false (and changes nothing) when
// the pool lacks pages.
bool reserve(rkv_pool* P, Seq& s, int64_t n, int32_t* slots) {
  const int64_t L = s.len;
  const bool cow = (L % kPageTokens) != 0 && P->ref[(size_t)s.pages[(size_t)(L / kPageTokens)]] > 1;
  const int64_t have = (L + kPageTokens - 1) / kPageTokens;
  const int64_t want = (L + n + kPageTokens - 1) / kPageTokens;
  if (P->free.count() < (cow ? 1 : 0) + (want - have)) return false;
  if (cow) {
    const int32_t old = s.pages[(size_t)(L / kPageTokens)];
    const int32_t fresh = P->alloc_page();
    P->pending_src.push_back(old);
    P->pending_dst.push_back(fresh);
    P->decref(old);  // still shared: never reaches zero here
    s.pages[(size_t)(L / kPageTokens)] = fresh;
  }
  for (int64_t i = have; i < want; ++i) s.pages.push_back(P->alloc_page());
  if (slots)
    for (int64_t t = L; t < L + n; ++t)
      slots[t - L] = (int32_t)(s.pages[(size_t)(t / kPageTokens)] * kPageTokens + t % kPageTokens);
  s.len = L + n;
  s.last_use = ++P->tick;
  return true;
}

void drop_seq_pages(rkv_pool* P, Seq& s, int64_t* freed) {
  for (int32_t p : s.pages)
    if (P->decref(p) && freed) ++*freed;
  s.pages.clear();
}

int64_t page_begin(int64_t tok) { return tok / kPageTokens; }
int64_t page_end(int64_t tok) { return (tok + kPageTokens - 1) / kPageTokens; }

// Splits node `id` at span offset `off` (0 < off < span); returns the upper
// part (the former node id keeps the lower part and gains it as only child).
int32_t split_node(rkv_pool* P, int32_t id, int64_t off) {
  const int32_t low_id = id;
  const int32_t up_id = P->new_node();  // may reallocate nodes: index afresh below
  Node& low = P->nodes[(size_t)low_id];
  Node& up = P->nodes[(size_t)up_id];
  const int64_t s = low.start, m = low.start + off;
  const int64_t pb = page_begin(s);
  up.parent = low_id;
  up.start = m;
  up.tokens.assign(low.tokens.begin() + off, low.tokens.end());
  up.children = std::move(low.children);
  up.last_use = low.last_use;
  for (auto& kv : up.children) P->nodes[(size_t)kv.second].parent = up_id;
  // upper: page indices [page_begin(m), end) taken from the node's list
  up.pages.assign(low.pages.begin() + (page_begin(m) - pb), low.pages.end());
  low.tokens.resize((size_t)off);
  low.pages.resize((size_t)(page_end(m) - pb));
  low.children.clear();
  low.children[up.tokens[0]] = up_id;
  if (m % kPageTokens != 0) P->incref(up.pages[0]);  // the straddling page is now listed twice
  return up_id;
}

void remove_leaf(rkv_pool* P, int32_t id, int64_t* freed) {
  Node& n = P->nodes[(size_t)id];
  for (int32_t p : n.pages)
    if (P->decref(p) && freed) ++*freed;
  Node& par = P->nodes[(size_t)n.parent];
  par.children.erase(n.tokens[0]);
  n = Node();
  P->free_nodes.push_back(id);
}

}  // namespace

namespace rkv {
int pool_device(const rkv_pool* pool) { return pool->device; }
uint32_t* pool_status_word(rkv_pool* pool) { return pool->d_status; }
}  // namespace rkv

extern "C" {

rkv_status rkv_pool_create(const rkv_pool_desc* desc, rkv_pool** out) {
  using namespace rkv;
  if (!desc || !out) return fail(RKV_ERR_INVALID_ARGUMENT, "rkv_pool_create: desc and out are required");
  *out = nullptr;
  if (desc->n_pages <= 0 || desc->n_layers <= 0 || desc->n_pages > (int64_t)(INT32_MAX / kPageTokens))
    return fail(RKV_ERR_SHAPE_MISMATCH, "rkv_pool_create: need 0 < n_pages <= %d and n_layers > 0",
                (int)(INT32_MAX / kPageTokens));
  if (desc->storage && ((uintptr_t)desc->storage & 255))
    return fail(RKV_ERR_INVALID_ARGUMENT, "rkv_pool_create: storage must be 256-byte aligned");
  rkv_pool* P = new rkv_pool();
  P->device = desc->device;
  P->n_pages = desc->n_pages;
  P->n_layers = desc->n_layers;
  P->ref.assign((size_t)P->n_pages, 0u);
  P->free.reset(P->n_pages);
  P->nodes.emplace_back();
  P->nodes[0].alive = true;
  if (P->device == RKV_PLAN_ONLY) {
    if (desc->storage) {
      delete P;
      return fail(RKV_ERR_INVALID_ARGUMENT, "rkv_pool_create: a plan-only pool takes no storage");
    }
    *out = P;
    clear_error();
    return RKV_OK;
  }
  if (P->device < 0) {
    delete P;
    return fail(RKV_ERR_INVALID_ARGUMENT, "rkv_pool_create: device %d", desc->device);
  }
  cudaError_t e = cudaSetDevice(P->device);
  if (e == cudaSuccess && desc->storage) {
    P->storage = desc->storage;
  } else if (e == cudaSuccess) {
    e = cudaMalloc(&P->storage, (size_t)rkv_pool_bytes(P->n_pages, P->n_layers));
    P->owns_storage = e == cudaSuccess;
  }
  if (e == cudaSuccess) e = cudaMalloc(&P->d_moves, (size_t)P->n_pages * 2 * 4);
  if (e == cudaSuccess) e = cudaMalloc(&P->d_remap, (size_t)P->n_pages * 4);
  if (e == cudaSuccess) e = cudaMalloc(&P->d_status, 4);
  if (e == cudaSuccess) e = cudaMemset(P->d_status, 0, 4);
  if (e != cudaSuccess) {
    rkv_pool_destroy(P);
    return fail(RKV_ERR_CUDA, "rkv_pool_create: %s", cudaGetErrorString(e));
  }
  *out = P;
  clear_error();
  return RKV_OK;
}

void rkv_pool_destroy(rkv_pool* P) {
  if (!P) return;
  if (P->device < 0) {
    delete P;
    return;
  }
  cudaSetDevice(P->device);
  if (P->owns_storage) cudaFree(P->storage);
  cudaFree(P->d_moves);
  cudaFree(P->d_remap);
  cudaFree(P->d_status);
  delete P;
}

rkv_status rkv_pool_get_view(const rkv_pool* P, rkv_pool_view* out) {
  if (!P || !out) return rkv::fail(RKV_ERR_INVALID_ARGUMENT, "rkv_pool_get_view: pool and out are required");
  *out = P->view();
  return RKV_OK;
}

rkv_status rkv_pool_get_stats(const rkv_pool* P, rkv_pool_stats* out) {
  if (!P || !out) return rkv::fail(RKV_ERR_INVALID_ARGUMENT, "rkv_pool_get_stats: pool and out are required");
  out->free_pages = P->free.count();
  out->live_pages = P->n_pages - P->free.count();
  out->sequences = (int64_t)P->seqs.size();
  int64_t nodes = 0;
  for (size_t i = 1; i < P->nodes.size(); ++i) nodes += P->nodes[i].alive ? 1 : 0;
  out->prefix_nodes = nodes;
  out->tick = (int64_t)P->tick;
  out->high_water = P->free.high_water();
  return RKV_OK;
}

rkv_status rkv_page_refcount(const rkv_pool* P, int32_t* out, int64_t cap) {
  if (!P || !out || cap < P->n_pages) return rkv::fail(RKV_ERR_INVALID_ARGUMENT, "rkv_page_refcount: out[n_pages] required");
  for (int64_t p = 0; p < P->n_pages; ++p) out[p] = (int32_t)P->ref[(size_t)p];
  return RKV_OK;
}

rkv_status rkv_seq_create(rkv_pool* P, int64_t* seq) {
  if (!P || !seq) return rkv::fail(RKV_ERR_INVALID_ARGUMENT, "rkv_seq_create: pool and seq are required");
  const int64_t id = P->next_seq++;
  Seq& s = P->seqs[id];
  s.last_use = ++P->tick;
  *seq = id;
  return RKV_OK;
}

rkv_status rkv_seq_fork(rkv_pool* P, int64_t parent, int64_t n_tokens, int64_t* child) {
  using namespace rkv;
  if (!P || !child) return fail(RKV_ERR_INVALID_ARGUMENT, "rkv_seq_fork: pool and child are required");
  Seq* s = find_seq(P, parent);
  if (!s) return fail_index("seq", parent, -1, "rkv_seq_fork: no sequence %lld", (long long)parent);
  if (n_tokens < 0 || n_tokens > s->len)
    return fail_index("n_tokens", n_tokens, s->len + 1, "rkv_seq_fork: %lld tokens of a %lld-token sequence",
                      (long long)n_tokens, (long long)s->len);
  std::vector<int32_t> pages(s->pages.begin(), s->pages.begin() + page_end(n_tokens));
  for (int32_t p : pages) P->incref(p);
  s->last_use = ++P->tick;
  const int64_t id = P->next_seq++;
  Seq& c = P->seqs[id];
  c.pages = std::move(pages);
  c.len = n_tokens;
  c.last_use = ++P->tick;
  *child = id;
  clear_error();
  return RKV_OK;
}

rkv_status rkv_seq_reserve(rkv_pool* P, int64_t n_seqs, const int64_t* seqs, const int64_t* n_tokens, int32_t* slots,
                           rkv_stream_t stream) {
  using namespace rkv;
  if (!P || n_seqs < 0 || (n_seqs > 0 && (!seqs || !n_tokens)))
    return fail(RKV_ERR_INVALID_ARGUMENT, "rkv_seq_reserve: pool, seqs and n_tokens are required");
  // validate everything and count pages first: the call is all-or-nothing
  int64_t need = 0;
  std::unordered_map<int64_t, int64_t> seen;
  for (int64_t i = 0; i < n_seqs; ++i) {
    Seq* s = find_seq(P, seqs[i]);
    if (!s) return fail_index("seq", seqs[i], -1, "rkv_seq_reserve: no sequence %lld", (long long)seqs[i]);
    if (n_tokens[i] < 0) return fail_shape("n_tokens", 0, n_tokens[i], "rkv_seq_reserve: negative token count");
    if (!seen.emplace(seqs[i], i).second)
      return fail(RKV_ERR_INVALID_ARGUMENT, "rkv_seq_reserve: sequence %lld listed twice", (long long)seqs[i]);
    const int64_t L = s->len;
    const bool cow = L % kPageTokens != 0 && P->ref[(size_t)s->pages[(size_t)(L / kPageTokens)]] > 1;
    need += (cow ? 1 : 0) + page_end(L + n_tokens[i]) - page_end(L);
  }
  if (need > P->free.count())
    return fail_full((int64_t)P->n_pages * kPageTokens, "rkv_seq_reserve: %lld pages needed, %lld free", (long long)need,
                     (long long)P->free.count());
  int64_t off = 0;
  for (int64_t i = 0; i < n_seqs; ++i) {
    reserve(P, *find_seq(P, seqs[i]), n_tokens[i], slots ? slots + off : nullptr);
    off += n_tokens[i];
  }
  std::vector<int32_t> src, dst;
  src.swap(P->pending_src);
  dst.swap(P->pending_dst);
  rkv_status st = enqueue_copies(P, src, dst, stream);
  if (st == RKV_OK) clear_error();
  return st;
}

rkv_status rkv_seq_release(rkv_pool* P, int64_t seq) {
  if (!P) return rkv::fail(RKV_ERR_INVALID_ARGUMENT, "rkv_seq_release: pool is required");
  Seq* s = find_seq(P, seq);
  if (!s) return rkv::fail_index("seq", seq, -1, "rkv_seq_release: no sequence %lld", (long long)seq);
  s->released = true;
  return RKV_OK;
}

rkv_status rkv_seq_touch(rkv_pool* P, int64_t seq) {
  if (!P) return rkv::fail(RKV_ERR_INVALID_ARGUMENT, "rkv_seq_touch: pool is required");
  Seq* s = find_seq(P, seq);
  if (!s) return rkv::fail_index("seq", seq, -1, "rkv_seq_touch: no sequence %lld", (long long)seq);
  s->last_use = ++P->tick;
  return RKV_OK;
}

rkv_status rkv_seq_free(rkv_pool* P, int64_t seq) {
  if (!P) return rkv::fail(RKV_ERR_INVALID_ARGUMENT, "rkv_seq_free: pool is required");
  auto it = P->seqs.find(seq);
  if (it == P->seqs.end()) return rkv::fail_index("seq", seq, -1, "rkv_seq_free: no sequence %lld", (long long)seq);
  drop_seq_pages(P, it->second, nullptr);
  P->seqs.erase(it);
  return RKV_OK;
}

rkv_status rkv_seq_info(const rkv_pool* P, int64_t seq, int64_t* len, int64_t* n_pages) {
  if (!P) return rkv::fail(RKV_ERR_INVALID_ARGUMENT, "rkv_seq_info: pool is required");
  auto it = P->seqs.find(seq);
  if (it == P->seqs.end()) return rkv::fail_index("seq", seq, -1, "rkv_seq_info: no sequence %lld", (long long)seq);
  if (len) *len = it->second.len;
  if (n_pages) *n_pages = (int64_t)it->second.pages.size();
  return RKV_OK;
}

rkv_status rkv_seq_page_table(const rkv_pool* P, int64_t seq, int32_t* out, int64_t cap) {
  if (!P) return rkv::fail(RKV_ERR_INVALID_ARGUMENT, "rkv_seq_page_table: pool is required");
  auto it = P->seqs.find(seq);
  if (it == P->seqs.end())
    return rkv::fail_index("seq", seq, -1, "rkv_seq_page_table: no sequence %lld", (long long)seq);
  const std::vector<int32_t>& pg = it->second.pages;
  if (pg.empty()) return RKV_OK;
  if (!out || cap < (int64_t)pg.size())
    return rkv::fail_shape("out", (int64_t)pg.size(), out ? cap : 0, "rkv_seq_page_table: need room for %lld pages",
                           (long long)pg.size());
  std::copy(pg.begin(), pg.end(), out);
  return RKV_OK;
}

rkv_status rkv_prefix_insert(rkv_pool* P, const int32_t* tokens, int64_t n, int64_t seq) {
  using namespace rkv;
  if (!P || (n > 0 && !tokens)) return fail(RKV_ERR_INVALID_ARGUMENT, "rkv_prefix_insert: pool and tokens are required");
  Seq* s = find_seq(P, seq);
  if (!s) return fail_index("seq", seq, -1, "rkv_prefix_insert: no sequence %lld", (long long)seq);
  if (n < 0 || n > s->len)
    return fail_index("n_tokens", n, s->len + 1, "rkv_prefix_insert: %lld tokens of a %lld-token sequence",
                      (long long)n, (long long)s->len);
  const uint64_t now = ++P->tick;
  int32_t cur = 0;
  int64_t pos = 0;
  P->nodes[0].last_use = now;
  while (pos < n) {
    auto it = P->nodes[(size_t)cur].children.find(tokens[pos]);
    if (it == P->nodes[(size_t)cur].children.end()) {
      // new leaf for tokens [pos, n)
      const int32_t id = P->new_node();
      Node& leaf = P->nodes[(size_t)id];
      leaf.parent = cur;
      leaf.start = pos;
      leaf.tokens.assign(tokens + pos, tokens + n);
      leaf.pages.assign(s->pages.begin() + page_begin(pos), s->pages.begin() + page_end(n));
      for (int32_t p : leaf.pages) P->incref(p);
      leaf.last_use = now;
      P->nodes[(size_t)cur].children[tokens[pos]] = id;
      pos = n;
      break;
    }
    const int32_t child = it->second;
    const Node& c = P->nodes[(size_t)child];
    int64_t j = 0;
    const int64_t span = (int64_t)c.tokens.size();
    while (j < span && pos + j < n && c.tokens[(size_t)j] == tokens[pos + j]) ++j;
    if (j < span && pos + j < n) {
      split_node(P, child, j);  // diverges inside the node: the lower part becomes the shared prefix
    }
    P->nodes[(size_t)child].last_use = now;
    cur = child;
    pos += j;
    if (j < span) break;  // the prefix ends inside this node (or was split there and continues below)
  }
  if (pos < n) {
    // split case: continue with a new leaf under the (lower) split node
    const int32_t id = P->new_node();
    Node& leaf = P->nodes[(size_t)id];
    leaf.parent = cur;
    leaf.start = pos;
    leaf.tokens.assign(tokens + pos, tokens + n);
    leaf.pages.assign(s->pages.begin() + page_begin(pos), s->pages.begin() + page_end(n));
    for (int32_t p : leaf.pages) P->incref(p);
    leaf.last_use = now;
    P->nodes[(size_t)cur].children[tokens[pos]] = id;
  }
  s->last_use = now;
  clear_error();
  return RKV_OK;
}

rkv_status rkv_prefix_match(rkv_pool* P, const int32_t* tokens, int64_t n, int64_t* matched, int64_t* seq_out) {
  using namespace rkv;
  if (!P || !matched || !seq_out || (n > 0 && !tokens))
    return fail(RKV_ERR_INVALID_ARGUMENT, "rkv_prefix_match: pool, tokens, matched and seq_out are required");
  const uint64_t now = ++P->tick;
  std::vector<int32_t> pages;
  int32_t cur = 0;
  int64_t pos = 0;
  while (pos < n) {
    auto it = P->nodes[(size_t)cur].children.find(tokens[pos]);
    if (it == P->nodes[(size_t)cur].children.end()) break;
    Node& c = P->nodes[(size_t)it->second];
    int64_t j = 0;
    const int64_t span = (int64_t)c.tokens.size();
    while (j < span && pos + j < n && c.tokens[(size_t)j] == tokens[pos + j]) ++j;
    // pages for indices [page_begin(pos), page_end(pos + j)) from this node;
    // a straddling first page replaces the shallower node's copy
    const int64_t pb = page_begin(c.start);
    for (int64_t p = page_begin(pos); p < page_end(pos + j); ++p) {
      const int32_t pg = c.pages[(size_t)(p - pb)];
      if (p < (int64_t)pages.size()) pages[(size_t)p] = pg;
      else pages.push_back(pg);
    }
    c.last_use = now;
    cur = it->second;
    pos += j;
    if (j < span) break;
  }
  const int64_t id = P->next_seq++;
  Seq& s = P->seqs[id];
  s.pages.assign(pages.begin(), pages.begin() + page_end(pos));
  for (int32_t p : s.pages) P->incref(p);
  s.len = pos;
  s.last_use = now;
  *matched = pos;
  *seq_out = id;
  clear_error();
  return RKV_OK;
}

rkv_status rkv_pool_evict(rkv_pool* P, int64_t target_pages, int64_t* freed_out) {
  using namespace rkv;
  if (!P) return fail(RKV_ERR_INVALID_ARGUMENT, "rkv_pool_evict: pool is required");
  std::set<std::tuple<uint64_t, int, int64_t>> lru;  // (last use, kind, id)
  for (auto& kv : P->seqs)
    if (kv.second.released) lru.emplace(kv.second.last_use, (int)kSeqKind, kv.first);
  for (size_t i = 1; i < P->nodes.size(); ++i)
    if (P->nodes[i].alive && P->nodes[i].children.empty()) lru.emplace(P->nodes[i].last_use, (int)kNodeKind, (int64_t)i);
  int64_t freed = 0;
  while (freed < target_pages && !lru.empty()) {
    const auto [use, kind, id] = *lru.begin();
    lru.erase(lru.begin());
    if (kind == kSeqKind) {
      auto it = P->seqs.find(id);
      drop_seq_pages(P, it->second, &freed);
      P->seqs.erase(it);
    } else {
      const int32_t parent = P->nodes[(size_t)id].parent;
      remove_leaf(P, (int32_t)id, &freed);
      if (parent != 0 && P->nodes[(size_t)parent].children.empty())
        lru.emplace(P->nodes[(size_t)parent].last_use, (int)kNodeKind, (int64_t)parent);
    }
  }
  if (freed_out) *freed_out = freed;
  clear_error();
  return RKV_OK;
}

rkv_status rkv_pool_compact(rkv_pool* P, int32_t* d_tables, int64_t n_entries, int64_t* moved_out,
                            rkv_stream_t stream) {
  using namespace rkv;
  if (!P) return fail(RKV_ERR_INVALID_ARGUMENT, "rkv_pool_compact: pool is required");
  const int64_t live = P->n_pages - P->free.count();
  std::vector<int32_t> src, dst;
  int64_t hole = 0, top = P->n_pages - 1;
  while (true) {
    while (hole < live && !P->free.is_free(hole)) ++hole;
    while (top >= live && P->free.is_free(top)) --top;
    if (hole >= live || top < live) break;
    src.push_back((int32_t)top);
    dst.push_back((int32_t)hole);
    ++hole;
    --top;
  }
  std::vector<int32_t>& remap = P->last_remap;
  remap.resize((size_t)P->n_pages);
  for (int64_t p = 0; p < P->n_pages; ++p) remap[(size_t)p] = (int32_t)p;
  for (size_t i = 0; i < src.size(); ++i) {
    remap[(size_t)src[i]] = dst[i];
    P->ref[(size_t)dst[i]] = P->ref[(size_t)src[i]];
    P->ref[(size_t)src[i]] = 0;
    P->free.set_used(dst[i]);
    P->free.set_free(src[i]);
  }
  for (auto& kv : P->seqs)
    for (int32_t& p : kv.second.pages) p = remap[(size_t)p];
  for (Node& nd : P->nodes)
    for (int32_t& p : nd.pages) p = remap[(size_t)p];
  rkv_status st = enqueue_copies(P, src, dst, stream);
  if (st != RKV_OK) return st;
  if (d_tables && n_entries > 0 && !src.empty() && P->device >= 0) {
    cudaError_t e = cudaMemcpyAsync(P->d_remap, remap.data(), (size_t)P->n_pages * 4, cudaMemcpyHostToDevice,
                                    (cudaStream_t)stream);
    if (e != cudaSuccess) return fail(RKV_ERR_CUDA, "rkv_pool_compact: remap upload: %s", cudaGetErrorString(e));
    st = rkv_remap_pages(d_tables, n_entries, P->d_remap, P->n_pages, P->d_status, stream);
    if (st != RKV_OK) return st;
  }
  if (moved_out) *moved_out = (int64_t)src.size();
  clear_error();
  return RKV_OK;
}

rkv_status rkv_pool_last_remap(const rkv_pool* P, int32_t* out, int64_t cap) {
  if (!P || !out || cap < P->n_pages) return rkv::fail(RKV_ERR_INVALID_ARGUMENT, "rkv_pool_last_remap: out[n_pages] required");
  if (P->last_remap.empty())
    for (int64_t p = 0; p < P->n_pages; ++p) out[p] = (int32_t)p;
  else
    std::copy(P->last_remap.begin(), P->last_remap.end(), out);
  return RKV_OK;
}

rkv_status rkv_pool_take_moves(rkv_pool* P, int32_t* src, int32_t* dst, int64_t cap, int64_t* n) {
  if (!P || !n) return rkv::fail(RKV_ERR_INVALID_ARGUMENT, "rkv_pool_take_moves: pool and n are required");
  const int64_t m = (int64_t)P->planned_src.size();
  *n = m;
  if (m == 0 || (!src && !dst)) return RKV_OK;  // count query
  if (!src || !dst || cap < m)
    return rkv::fail_shape("src/dst", m, cap, "rkv_pool_take_moves: need room for %lld moves", (long long)m);
  std::copy(P->planned_src.begin(), P->planned_src.end(), src);
  std::copy(P->planned_dst.begin(), P->planned_dst.end(), dst);
  P->planned_src.clear();
  P->planned_dst.clear();
  return RKV_OK;
}

rkv_status rkv_pool_device_status(rkv_pool* P, uint32_t* bits) {
  if (!P || !bits) return rkv::fail(RKV_ERR_INVALID_ARGUMENT, "rkv_pool_device_status: pool and bits are required");
  if (P->device < 0) {
    *bits = 0;
    return RKV_OK;
  }
  cudaError_t e = cudaSetDevice(P->device);
  if (e == cudaSuccess) e = cudaMemcpy(bits, P->d_status, 4, cudaMemcpyDeviceToHost);
  if (e == cudaSuccess) e = cudaMemset(P->d_status, 0, 4);
  if (e != cudaSuccess) return rkv::fail(RKV_ERR_CUDA, "rkv_pool_device_status: %s", cudaGetErrorString(e));
  return RKV_OK;
}

}  // extern "C"
