// rkv_noalloc.cu -- the page moves of a compaction applied without
// allocating any memory.
//
// rkv_pool_compact keeps its move lists and remap table in device memory the
// pool allocates when it is created.  Some callers cannot call cudaMalloc: an
// engine that reserves all of its device memory at start-up and hands it out
// through its own allocator, or the owner of a plan-only pool that moves the
// pages itself with whatever memory it already has.
// rkv_apply_page_moves_static takes the move list in host memory, stages it in
// a fixed array that lives in this library (a file-scope __device__ array,
// present on every GPU that loads the library until the process exits), and
// from there copies the pages and rewrites a device page table.  Nothing is
// allocated: no cudaMalloc, cudaFree or allocating library call.
//
// The staging array is shared by every call on a device and keeps the last
// call's contents; each call overwrites the entries it uses, so nothing needs
// clearing, but two calls whose work overlaps on the GPU (different streams,
// or the same device from several threads) race on it -- order them.
#include <algorithm>

#include <atomic>
#include <mutex>

#include "rkv_common.cuh"
#include "rkv_host.h"

namespace rkv {

constexpr int64_t kStaticMaxMoves = RKV_STATIC_MAX_MOVES;

// [0, kStaticMaxMoves): move sources, ascending; [kStaticMaxMoves, 2x): their
// destinations.  2 MB.
static __device__ __align__(256) int32_t g_move_scratch[2 * kStaticMaxMoves];

constexpr int kMaxDevices = 64;
static std::atomic<int32_t*> g_scratch_addr[kMaxDevices];  // device address of g_move_scratch, per device

// Host-side room to sort a copy of the destinations (the duplicate check),
// fixed like the device array so that validation allocates nothing either;
// calls from several host threads take turns on it.
static int32_t g_dst_sorted[kStaticMaxMoves];
static std::mutex g_dst_sorted_mutex;

// Page-table rewrite against the staged move list: an entry equal to some
// src[i] becomes dst[i] (binary search of the ascending sources).
__global__ void remap_by_moves_kernel(int32_t* __restrict__ table, int64_t n, const int32_t* __restrict__ src,
                                      const int32_t* __restrict__ dst, int64_t n_moves, int64_t n_pages,
                                      uint32_t* __restrict__ status) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int32_t p = table[i];
    if (p < 0) continue;
    if (p >= n_pages) {
      set_status(status, RKV_ERR_INDEX_OUT_OF_RANGE);
      continue;
    }
    int64_t lo = 0, hi = n_moves;
    while (lo < hi) {
      const int64_t mid = (lo + hi) >> 1;
      if (__ldg(src + mid) < p) lo = mid + 1;
      else hi = mid;
    }
    if (lo < n_moves && __ldg(src + lo) == p) table[i] = __ldg(dst + lo);
  }
}

}  // namespace rkv

extern "C" rkv_status rkv_apply_page_moves_static(const rkv_pool_view* pool, const int32_t* src, const int32_t* dst,
                                                  int64_t n_moves, int32_t* d_tables, int64_t n_entries,
                                                  uint32_t* d_status, rkv_stream_t stream) {
  using namespace rkv;
  rkv_status st = check_pool(pool, "rkv_apply_page_moves_static");
  if (st != RKV_OK) return st;
  if (n_moves < 0 || n_entries < 0) return fail(RKV_ERR_SHAPE_MISMATCH, "rkv_apply_page_moves_static: negative sizes");
  if (n_moves > kStaticMaxMoves)
    return fail_shape("n_moves", kStaticMaxMoves, n_moves,
                      "rkv_apply_page_moves_static: %lld moves exceed the %lld this entry point stages",
                      (long long)n_moves, (long long)kStaticMaxMoves);
  if (n_moves == 0) {
    clear_error();
    return RKV_OK;
  }
  if (!src || !dst) return fail(RKV_ERR_INVALID_ARGUMENT, "rkv_apply_page_moves_static: src and dst are required");
  for (int64_t i = 0; i < n_moves; ++i) {
    if (i > 0 && src[i] <= src[i - 1])
      return fail(RKV_ERR_INVALID_ARGUMENT, "rkv_apply_page_moves_static: src must be strictly ascending");
    if (src[i] < 0 || src[i] >= pool->n_pages || dst[i] < 0 || dst[i] >= pool->n_pages) {
      const bool bad_src = src[i] < 0 || src[i] >= pool->n_pages;
      return fail_index(bad_src ? "src" : "dst", bad_src ? src[i] : dst[i], pool->n_pages,
                        "rkv_apply_page_moves_static: move %lld outside the pool", (long long)i);
    }
  }
  for (int64_t i = 0; i < n_moves; ++i) {  // destinations must not be sources (copies run in parallel)
    const int32_t* hit = std::lower_bound(src, src + n_moves, dst[i]);
    if (hit != src + n_moves && *hit == dst[i])
      return fail(RKV_ERR_INVALID_ARGUMENT, "rkv_apply_page_moves_static: page %d is both a source and a destination",
                  dst[i]);
  }
  {  // no two moves may write one page: the copies run in parallel, and the
     // table rewrite would map two live pages onto it
    std::lock_guard<std::mutex> lock(g_dst_sorted_mutex);
    std::copy(dst, dst + n_moves, g_dst_sorted);
    std::sort(g_dst_sorted, g_dst_sorted + n_moves);
    const int32_t* dup = std::adjacent_find(g_dst_sorted, g_dst_sorted + n_moves);
    if (dup != g_dst_sorted + n_moves)
      return fail(RKV_ERR_INVALID_ARGUMENT, "rkv_apply_page_moves_static: page %d is the destination of two moves",
                  *dup);
  }
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(RKV_ERR_CUDA, "rkv_apply_page_moves_static: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices) return fail(RKV_ERR_INVALID_ARGUMENT, "rkv_apply_page_moves_static: device %d", dev);
  // Once per device, with that device current: the device address of the
  // staging array (the symbol itself is only a host-side stand-in).
  if (!g_scratch_addr[dev].load(std::memory_order_acquire)) {
    void* ptr = nullptr;
    e = cudaGetSymbolAddress(&ptr, g_move_scratch);
    if (e != cudaSuccess || !ptr)
      return fail(RKV_ERR_CUDA, "rkv_apply_page_moves_static: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
    g_scratch_addr[dev].store(static_cast<int32_t*>(ptr), std::memory_order_release);
  }
  int32_t* s_src = g_scratch_addr[dev].load(std::memory_order_acquire);
  int32_t* s_dst = s_src + kStaticMaxMoves;
  e = cudaMemcpyAsync(s_src, src, (size_t)n_moves * 4, cudaMemcpyHostToDevice, (cudaStream_t)stream);
  if (e == cudaSuccess)
    e = cudaMemcpyAsync(s_dst, dst, (size_t)n_moves * 4, cudaMemcpyHostToDevice, (cudaStream_t)stream);
  if (e != cudaSuccess) return fail(RKV_ERR_CUDA, "rkv_apply_page_moves_static: staging: %s", cudaGetErrorString(e));
  st = rkv_copy_pages(pool, s_src, s_dst, n_moves, d_status, stream);
  if (st != RKV_OK || !d_tables || n_entries == 0) return st;
  const int64_t blocks = (n_entries + 255) / 256;
  remap_by_moves_kernel<<<(unsigned)(blocks < 148 * 16 ? blocks : 148 * 16), 256, 0, (cudaStream_t)stream>>>(
      d_tables, n_entries, s_src, s_dst, n_moves, pool->n_pages, d_status);
  return check_launch("rkv_apply_page_moves_static");
}
