// rkv_pages.cu -- whole-page moves for copy-on-write and compaction, and the
// page-table rewrite that follows a compaction.
//
// rsLLM has no paged pool yet; its plan (docs/03-HLD.md:363-376) is refcounted
// shared prefix blocks, a free list, radix-tree prefix reuse and LRU eviction.
// The host side (rkv_pool.cpp) decides which pages move; these kernels move
// the bytes: one 256-thread CTA per (page pair, layer), 43008 B = 2688
// 16-byte vectors, all loads of a thread issued before its stores.
#include "rkv_common.cuh"
#include "rkv_host.h"

namespace rkv {

constexpr int kCopyThreads = 256;
constexpr int kVecPerPage = kPageBytes / 16;                                 // 2688
constexpr int kVecPerThread = (kVecPerPage + kCopyThreads - 1) / kCopyThreads;  // 11

__global__ void __launch_bounds__(kCopyThreads)
copy_pages_kernel(rkv_pool_view pool, const int32_t* __restrict__ src, const int32_t* __restrict__ dst,
                  uint32_t* __restrict__ status) {
  const int64_t i = blockIdx.x;
  const int layer = blockIdx.y;
  const int32_t s = __ldg(src + i), d = __ldg(dst + i);
  if (s < 0 || s >= pool.n_pages || d < 0 || d >= pool.n_pages) {
    if (threadIdx.x == 0 && layer == 0) set_status(status, RKV_ERR_INDEX_OUT_OF_RANGE);
    return;
  }
  const uint4* sp = reinterpret_cast<const uint4*>(page_base(pool, layer, s));
  uint4* dp = reinterpret_cast<uint4*>(page_base(pool, layer, d));
  uint4 v[kVecPerThread];
#pragma unroll
  for (int j = 0; j < kVecPerThread; ++j) {
    const int e = threadIdx.x + j * kCopyThreads;
    if (e < kVecPerPage) v[j] = ld_stream16(sp + e);
  }
#pragma unroll
  for (int j = 0; j < kVecPerThread; ++j) {
    const int e = threadIdx.x + j * kCopyThreads;
    if (e < kVecPerPage) st_stream16(dp + e, v[j]);
  }
}

__global__ void remap_pages_kernel(int32_t* __restrict__ table, int64_t n, const int32_t* __restrict__ remap,
                                   int64_t n_pages, uint32_t* __restrict__ status) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int32_t p = table[i];
    if (p < 0) continue;
    if (p >= n_pages) {
      set_status(status, RKV_ERR_INDEX_OUT_OF_RANGE);
      continue;
    }
    table[i] = __ldg(remap + p);
  }
}

}  // namespace rkv

extern "C" rkv_status rkv_copy_pages(const rkv_pool_view* pool, const int32_t* src, const int32_t* dst, int64_t n,
                                     uint32_t* d_status, rkv_stream_t stream) {
  using namespace rkv;
  rkv_status st = check_pool(pool, "rkv_copy_pages");
  if (st != RKV_OK) return st;
  if (n < 0) return fail_shape("n", 0, n, "rkv_copy_pages: n < 0");
  if (n == 0) {
    clear_error();
    return RKV_OK;
  }
  if (!src || !dst) return fail(RKV_ERR_INVALID_ARGUMENT, "rkv_copy_pages: src and dst are required");
  if (n > INT32_MAX || pool->n_layers > 65535) return fail(RKV_ERR_SHAPE_MISMATCH, "rkv_copy_pages: too many pages");
  dim3 grid((unsigned)n, (unsigned)pool->n_layers);
  copy_pages_kernel<<<grid, kCopyThreads, 0, (cudaStream_t)stream>>>(*pool, src, dst, d_status);
  return check_launch("rkv_copy_pages");
}

extern "C" rkv_status rkv_remap_pages(int32_t* page_table, int64_t n_entries, const int32_t* remap, int64_t n_pages,
                                      uint32_t* d_status, rkv_stream_t stream) {
  using namespace rkv;
  if (n_entries < 0 || n_pages < 0) return fail(RKV_ERR_SHAPE_MISMATCH, "rkv_remap_pages: negative sizes");
  if (n_entries == 0) {
    clear_error();
    return RKV_OK;
  }
  if (!page_table || !remap) return fail(RKV_ERR_INVALID_ARGUMENT, "rkv_remap_pages: page_table and remap are required");
  const int64_t blocks = (n_entries + 255) / 256;
  remap_pages_kernel<<<(unsigned)(blocks < 148 * 16 ? blocks : 148 * 16), 256, 0, (cudaStream_t)stream>>>(
      page_table, n_entries, remap, n_pages, d_status);
  return check_launch("rkv_remap_pages");
}

// ---- contiguous staging of a page list (swap to host memory, disk format) ---
// pack: dst[l][i] = page pages[i] of layer layer0 + l; unpack: the reverse.
// One CTA per (page, layer), as copy_pages_kernel.
namespace rkv {

template <bool kPack>
__global__ void __launch_bounds__(kCopyThreads)
stage_pages_kernel(rkv_pool_view pool, int layer0, const int32_t* __restrict__ pages, int64_t n,
                   uint8_t* __restrict__ buf, uint32_t* __restrict__ status) {
  const int64_t i = blockIdx.x;
  const int l = blockIdx.y;
  const int32_t pg = __ldg(pages + i);
  if (pg < 0 || pg >= pool.n_pages) {
    if (threadIdx.x == 0 && l == 0) set_status(status, RKV_ERR_INDEX_OUT_OF_RANGE);
    return;
  }
  uint4* pp = reinterpret_cast<uint4*>(page_base(pool, layer0 + l, pg));
  uint4* bp = reinterpret_cast<uint4*>(buf + ((int64_t)l * n + i) * kPageBytes);
  const uint4* sp = kPack ? pp : bp;
  uint4* dp = kPack ? bp : pp;
  uint4 v[kVecPerThread];
#pragma unroll
  for (int j = 0; j < kVecPerThread; ++j) {
    const int e = threadIdx.x + j * kCopyThreads;
    if (e < kVecPerPage) v[j] = ld_stream16(sp + e);
  }
#pragma unroll
  for (int j = 0; j < kVecPerThread; ++j) {
    const int e = threadIdx.x + j * kCopyThreads;
    if (e < kVecPerPage) st_stream16(dp + e, v[j]);
  }
}

static rkv_status stage_pages(bool pack, const rkv_pool_view* pool, int32_t layer0, int32_t n_layers,
                              const int32_t* pages, int64_t n, void* buf, uint32_t* d_status, rkv_stream_t stream,
                              const char* what) {
  rkv_status st = check_pool(pool, what);
  if (st != RKV_OK) return st;
  if (layer0 < 0 || n_layers < 0 || (int64_t)layer0 + n_layers > pool->n_layers)
    return fail_layer(layer0 < 0 || n_layers < 0 ? layer0 : (int64_t)layer0 + n_layers - 1, pool->n_layers,
                      "%s: layers [%d, %d) outside pool of %d layers", what, layer0, layer0 + n_layers,
                      pool->n_layers);
  if (n < 0 || n > INT32_MAX || n_layers > 65535) return fail(RKV_ERR_SHAPE_MISMATCH, "%s: bad page count", what);
  if (n == 0 || n_layers == 0) {
    clear_error();
    return RKV_OK;
  }
  if (!pages || !buf || !aligned(buf, 16))
    return fail(RKV_ERR_INVALID_ARGUMENT, "%s: pages and a 16-byte aligned buffer are required", what);
  dim3 grid((unsigned)n, (unsigned)n_layers);
  if (pack)
    stage_pages_kernel<true><<<grid, kCopyThreads, 0, (cudaStream_t)stream>>>(*pool, layer0, pages, n,
                                                                              static_cast<uint8_t*>(buf), d_status);
  else
    stage_pages_kernel<false><<<grid, kCopyThreads, 0, (cudaStream_t)stream>>>(*pool, layer0, pages, n,
                                                                               static_cast<uint8_t*>(buf), d_status);
  return check_launch(what);
}

}  // namespace rkv

extern "C" rkv_status rkv_pack_pages(const rkv_pool_view* pool, int32_t layer0, int32_t n_layers, const int32_t* pages,
                                     int64_t n, void* dst, uint32_t* d_status, rkv_stream_t stream) {
  return rkv::stage_pages(true, pool, layer0, n_layers, pages, n, dst, d_status, stream, "rkv_pack_pages");
}

extern "C" rkv_status rkv_unpack_pages(const rkv_pool_view* pool, int32_t layer0, int32_t n_layers,
                                       const int32_t* pages, int64_t n, const void* src, uint32_t* d_status,
                                       rkv_stream_t stream) {
  return rkv::stage_pages(false, pool, layer0, n_layers, pages, n, const_cast<void*>(src), d_status, stream,
                          "rkv_unpack_pages");
}
