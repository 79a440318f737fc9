// rkv_indexer.cu -- the indexer's scoring of compressed rows against a query,
// feeding the top-k selection: IndexerPool::select_top_k
// (crates/rsllm-kvcache/src/dsv4/indexer.rs:169-236) for a batch of queries.
//
// score[c] = sum_h relu(dot(row_c, q_h)) * w_h over 64 heads of 128 lanes.
// rsLLM accumulates every dot lane by lane and the score head by head in f32,
// each product and sum rounded on its own; the kernel does exactly that (an
// f32 dot product on tensor cores or with fused multiply-adds would round
// differently), so the scores -- and therefore the selected indices -- are
// bit-exact.
//
// Shape: the scoring is a (rows x heads) product with K = 128 lanes, so the
// kernel is tiled like a register-blocked f32 GEMM, with a separately rounded
// multiply and add (__fmul_rn / __fadd_rn, which the compiler never fuses) in
// place of each fused multiply-add, and the lanes visited in ascending order
// for every (row, head) pair.  One CTA of 128 threads takes 128 rows of one
// query: the rows (64 KB) and the query (32 KB) pass through shared memory in
// four chunks of 32 lanes, double-buffered with cp.async (55 KB per CTA, so
// three CTAs share an SM); each thread owns an 8-row x 8-head tile of dot
// products, so one 16-byte shared load feeds 32 products (a thread holding
// one row and looping over heads needs one load per 4 products, which leaves
// the kernel bound by shared-memory wavefronts near 0.6 of the FP32 rate).  Finally the 128 x 64 dot products go through
// shared memory once more, and each thread applies ReLU and the weighted sum
// to one row, head by head in head order.
// The work is 8192 multiplies and 8192 adds per (query, row): CUDA-core
// bound, not HBM bound.  (Packed f32x2 arithmetic was measured slower here:
// on this part it does not raise the FP32 rate.)
#include <atomic>

#include "rkv_common.cuh"
#include "rkv_host.h"

namespace rkv {

constexpr int kIdxHeads = 64;
constexpr int kIdxDim = 128;
constexpr int kIdxRows = 128;  // rows (threads) per CTA

constexpr int kIdxChunk = 32;                  // lanes per staged chunk
constexpr int kIdxChunks = kIdxDim / kIdxChunk;
constexpr int kIdxStride = kIdxChunk + 4;      // padded shared row of a chunk, floats
constexpr int kIdxBuf = (kIdxRows + kIdxHeads) * kIdxStride;  // one chunk buffer, floats
constexpr int kIdxDotStride = kIdxHeads + 4;   // the dot-product tile's row, floats
constexpr int kIdxSmem = (2 * kIdxBuf + kIdxHeads) * 4;
static_assert(kIdxRows * kIdxDotStride <= 2 * kIdxBuf, "dot tile fits in the chunk buffers");

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  const uint32_t d = (uint32_t)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(d), "l"(gmem) : "memory");
}

// Copies lanes [32 ch, 32 ch + 32) of the CTA's rows and of the query into a
// chunk buffer as one cp.async group: a warp copies 4 rows x 128 bytes per
// step (coalesced reads, conflict-free shared stores); rows past the visible
// end are left alone (the buffer's zeroed rows stay zero).
__device__ __forceinline__ void stage_chunk(float* buf, const float* rg, const float* qg, int n_rows, int ch,
                                            int tid) {
  constexpr int kVec = kIdxChunk / 4;
  float* s_kv = buf;
  float* s_q = buf + kIdxRows * kIdxStride;
#pragma unroll 4
  for (int v = tid; v < kIdxRows * kVec; v += kIdxRows) {
    const int r = v / kVec, c = 4 * (v % kVec);
    if (r < n_rows) cp_async16(s_kv + r * kIdxStride + c, rg + (int64_t)r * kIdxDim + ch * kIdxChunk + c);
  }
#pragma unroll 4
  for (int v = tid; v < kIdxHeads * kVec; v += kIdxRows) {
    const int h = v / kVec, c = 4 * (v % kVec);
    cp_async16(s_q + h * kIdxStride + c, qg + h * kIdxDim + ch * kIdxChunk + c);
  }
  asm volatile("cp.async.commit_group;" ::: "memory");
}

// The thread tile over one staged chunk: rows warp*32 + rt + 4a and heads
// ht + 8b (a, b < 8); at a fixed a (b) the warp reads 4 (8) consecutive
// padded rows, which fall in distinct banks, the other lanes reading the
// same addresses.  The lanes are added in ascending order, as rsLLM's dot
// adds them.
__device__ __forceinline__ void dot_chunk(float (&d)[8][8], const float* buf, int warp, int rt, int ht) {
  const float* kvb = buf + (warp * 32 + rt) * kIdxStride;
  const float* qb = buf + kIdxRows * kIdxStride + ht * kIdxStride;
#pragma unroll 1
  for (int i = 0; i < kIdxChunk; i += 4) {
    float4 kr[8], qh[8];
#pragma unroll
    for (int a = 0; a < 8; ++a) kr[a] = *reinterpret_cast<const float4*>(kvb + 4 * a * kIdxStride + i);
#pragma unroll
    for (int b = 0; b < 8; ++b) qh[b] = *reinterpret_cast<const float4*>(qb + 8 * b * kIdxStride + i);
#pragma unroll
    for (int a = 0; a < 8; ++a)
#pragma unroll
      for (int b = 0; b < 8; ++b) d[a][b] = __fadd_rn(d[a][b], __fmul_rn(kr[a].x, qh[b].x));
#pragma unroll
    for (int a = 0; a < 8; ++a)
#pragma unroll
      for (int b = 0; b < 8; ++b) d[a][b] = __fadd_rn(d[a][b], __fmul_rn(kr[a].y, qh[b].y));
#pragma unroll
    for (int a = 0; a < 8; ++a)
#pragma unroll
      for (int b = 0; b < 8; ++b) d[a][b] = __fadd_rn(d[a][b], __fmul_rn(kr[a].z, qh[b].z));
#pragma unroll
    for (int a = 0; a < 8; ++a)
#pragma unroll
      for (int b = 0; b < 8; ++b) d[a][b] = __fadd_rn(d[a][b], __fmul_rn(kr[a].w, qh[b].w));
  }
}

__global__ void __launch_bounds__(kIdxRows, 3)
indexer_score_kernel(const float* __restrict__ rows, const int64_t* __restrict__ row_start,
                     const int32_t* __restrict__ seq_rows, int64_t n_seq, const float* __restrict__ q,
                     const float* __restrict__ w, const int32_t* __restrict__ seq_of_query,
                     const int32_t* __restrict__ n_visible, int32_t blocks_per_q, float* __restrict__ scores,
                     int64_t ld, uint32_t* __restrict__ status) {
  extern __shared__ __align__(16) float smem[];
  float* buf0 = smem;
  float* buf1 = smem + kIdxBuf;
  float* s_w = smem + 2 * kIdxBuf;  // [kIdxHeads]
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int tid = threadIdx.x;
  const int64_t qi = blockIdx.x / blocks_per_q;
  const int rb = (int)(blockIdx.x % blocks_per_q);
  const int s = __ldg(seq_of_query + qi), nv = __ldg(n_visible + qi);
  if (s < 0 || (int64_t)s >= n_seq || nv < 0 || nv > __ldg(seq_rows + s)) {
    if (rb == 0 && tid == 0) set_status(status, RKV_ERR_INDEX_OUT_OF_RANGE);
    return;
  }
  const int r0 = rb * kIdxRows;
  if (r0 >= nv) return;
  const int n_rows = nv - r0 < kIdxRows ? nv - r0 : kIdxRows;
  const float* rg = rows + (__ldg(row_start + s) + r0) * kIdxDim;
  const float* qg = q + qi * (kIdxHeads * kIdxDim);

  // rows past the visible end read as zero in both buffers
  for (int v = tid; v < (kIdxRows - n_rows) * (kIdxChunk / 4); v += kIdxRows) {
    const int r = n_rows + v / (kIdxChunk / 4), c = 4 * (v % (kIdxChunk / 4));
    *reinterpret_cast<float4*>(buf0 + r * kIdxStride + c) = make_float4(0.f, 0.f, 0.f, 0.f);
    *reinterpret_cast<float4*>(buf1 + r * kIdxStride + c) = make_float4(0.f, 0.f, 0.f, 0.f);
  }
  stage_chunk(buf0, rg, qg, n_rows, 0, tid);
  stage_chunk(buf1, rg, qg, n_rows, 1, tid);
  if (tid < kIdxHeads) s_w[tid] = __ldg(w + qi * kIdxHeads + tid);

  const int warp = tid >> 5, lane = tid & 31, rt = lane & 3, ht = lane >> 2;
  float d[8][8];
#pragma unroll
  for (int a = 0; a < 8; ++a)
#pragma unroll
    for (int b = 0; b < 8; ++b) d[a][b] = 0.0f;
  // two buffers: chunk ch + 2 is copied while chunk ch + 1 is multiplied
  static_assert(kIdxChunks == 4, "the pipeline below covers four chunks");
  asm volatile("cp.async.wait_group 1;" ::: "memory");
  __syncthreads();
  dot_chunk(d, buf0, warp, rt, ht);
  __syncthreads();  // buffer 0 is free
  stage_chunk(buf0, rg, qg, n_rows, 2, tid);
  asm volatile("cp.async.wait_group 1;" ::: "memory");
  __syncthreads();
  dot_chunk(d, buf1, warp, rt, ht);
  __syncthreads();  // buffer 1 is free
  stage_chunk(buf1, rg, qg, n_rows, 3, tid);
  asm volatile("cp.async.wait_group 1;" ::: "memory");
  __syncthreads();
  dot_chunk(d, buf0, warp, rt, ht);
  asm volatile("cp.async.wait_group 0;" ::: "memory");
  __syncthreads();
  dot_chunk(d, buf1, warp, rt, ht);
  __syncthreads();  // every thread is done reading the buffers

  float* s_dot = smem;  // [kIdxRows][kIdxDotStride]
#pragma unroll
  for (int a = 0; a < 8; ++a)
#pragma unroll
    for (int b = 0; b < 8; ++b) s_dot[(warp * 32 + rt + 4 * a) * kIdxDotStride + ht + 8 * b] = d[a][b];
  __syncthreads();
  if (tid >= n_rows) return;
  // ReLU and the weighted sum head by head, in head order
  const float4* dr = reinterpret_cast<const float4*>(s_dot + tid * kIdxDotStride);
  float acc = 0.0f;
#pragma unroll 4
  for (int h = 0; h < kIdxHeads; h += 4) {
    const float4 d4 = dr[h / 4];
    if (d4.x > 0.0f) acc = __fadd_rn(acc, __fmul_rn(d4.x, s_w[h]));
    if (d4.y > 0.0f) acc = __fadd_rn(acc, __fmul_rn(d4.y, s_w[h + 1]));
    if (d4.z > 0.0f) acc = __fadd_rn(acc, __fmul_rn(d4.z, s_w[h + 2]));
    if (d4.w > 0.0f) acc = __fadd_rn(acc, __fmul_rn(d4.w, s_w[h + 3]));
  }
  scores[qi * ld + r0 + tid] = acc;
}

}  // namespace rkv

extern "C" rkv_status rkv_indexer_scores_f32(const float* rows, const int64_t* row_start, const int32_t* seq_rows,
                                             int64_t n_seq, const float* q, const float* w,
                                             const int32_t* seq_of_query, const int32_t* n_visible, int32_t n_q,
                                             int32_t max_visible, float* scores, int64_t ld, uint32_t* d_status,
                                             rkv_stream_t stream) {
  using namespace rkv;
  if (n_q < 0 || max_visible < 0 || n_seq < 0)
    return fail(RKV_ERR_SHAPE_MISMATCH, "rkv_indexer_scores_f32: negative sizes");
  if (ld < max_visible)
    return fail_shape("ld", max_visible, ld, "rkv_indexer_scores_f32: ld %lld < max_visible %d", (long long)ld,
                      max_visible);
  if (n_q == 0 || max_visible == 0) {
    clear_error();
    return RKV_OK;
  }
  if (!rows || !aligned(rows, 16) || !q || !aligned(q, 16) || !w || !row_start || !seq_rows || !seq_of_query ||
      !n_visible || !scores || !d_status)
    return fail(RKV_ERR_INVALID_ARGUMENT,
                "rkv_indexer_scores_f32: rows, q (16-byte aligned), w, row_start, seq_rows, seq_of_query, "
                "n_visible, scores and d_status are required");
  // the shared-memory opt-in is per device
  static std::atomic<bool> attr_set[kMaxDevicesCached];
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= kMaxDevicesCached || !attr_set[dev].load(std::memory_order_acquire)) {
    cudaError_t e = cudaFuncSetAttribute(indexer_score_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kIdxSmem);
    if (e != cudaSuccess) return fail(RKV_ERR_CUDA, "rkv_indexer_scores_f32: %s", cudaGetErrorString(e));
    if (dev >= 0 && dev < kMaxDevicesCached) attr_set[dev].store(true, std::memory_order_release);
  }
  const int64_t per_q = (max_visible + kIdxRows - 1) / kIdxRows;
  const int64_t blocks = per_q * n_q;
  if (blocks > (int64_t)INT32_MAX) return fail(RKV_ERR_SHAPE_MISMATCH, "rkv_indexer_scores_f32: grid too large");
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)blocks);
  cfg.blockDim = dim3(kIdxRows);
  cfg.dynamicSmemBytes = kIdxSmem;
  cfg.stream = (cudaStream_t)stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, indexer_score_kernel, rows, row_start, seq_rows, n_seq, q, w,
                                     seq_of_query, n_visible, (int32_t)per_q, scores, ld, d_status);
  if (e != cudaSuccess) return fail(RKV_ERR_CUDA, "rkv_indexer_scores_f32: launch failed: %s", cudaGetErrorString(e));
  return check_launch("rkv_indexer_scores_f32");
}

extern "C" rkv_status rkv_indexer_topk_f32(const float* rows, const int64_t* row_start, const int32_t* seq_rows,
                                           int64_t n_seq, const float* q, const float* w,
                                           const int32_t* seq_of_query, const int32_t* n_visible, int32_t n_q,
                                           int32_t max_visible, int32_t k, float* scores, int64_t ld,
                                           int32_t* out_idx, uint32_t* d_status, rkv_stream_t stream) {
  rkv_status st = rkv_indexer_scores_f32(rows, row_start, seq_rows, n_seq, q, w, seq_of_query, n_visible, n_q,
                                         max_visible, scores, ld, d_status, stream);
  if (st != RKV_OK) return st;
  return rkv_topk_select_f32(scores, ld, n_q, n_visible, max_visible, k, out_idx, stream);
}
