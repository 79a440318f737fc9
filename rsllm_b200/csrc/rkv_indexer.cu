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
// kernel is tiled like a register-blocked f32 GEMM, every fused multiply-add
// replaced by a rounded product and a rounded add, and the lanes visited in
// ascending order for every (row, head) pair.  One CTA of 128 threads takes
// 128 rows of one query: the rows (64 KB) pass through shared memory in four
// chunks of 32 lanes, double-buffered with cp.async; the query (32 KB) is
// stored transposed (lane-major) once per CTA; 70 KB per CTA, so three CTAs
// share an SM.  Each thread owns an 8-row x 8-head tile of dot products held
// as packed f32x2 pairs of heads, so each instruction does two heads' work:
// the product is fma.rn.f32x2 with a -0.0 addend -- exactly the rounded
// product -- and the sum add.rn.f32x2.  (A thread holding one row and
// looping over heads needs one shared load per 4 products and stays bound by
// shared-memory wavefronts near 0.6 of the scalar FP32 rate; the scalar
// register-tiled form reached 0.78 of it.)  Finally the 128 x 64 dot
// products go through shared memory once more, and each thread applies ReLU
// and the weighted sum to one row, head by head in head order.
// The work is 8192 multiplies and 8192 adds per (query, row): CUDA-core
// bound, not HBM bound.
#include <atomic>

#include "rkv_common.cuh"
#include "rkv_host.h"

namespace rkv {

constexpr int kIdxHeads = 64;
constexpr int kIdxDim = 128;
constexpr int kIdxRows = 128;  // rows (threads) per CTA

constexpr int kIdxChunk = 32;                  // lanes per staged chunk of rows
constexpr int kIdxChunks = kIdxDim / kIdxChunk;
constexpr int kIdxStride = kIdxChunk + 4;      // padded shared row of a chunk, floats
constexpr int kIdxBuf = kIdxRows * kIdxStride;  // one chunk buffer, floats
constexpr int kIdxQtStride = kIdxHeads + 4;    // the transposed query's row (one lane), floats
constexpr int kIdxDotStride = kIdxHeads + 4;   // the dot-product tile's row, floats
constexpr int kIdxSmem = (2 * kIdxBuf + kIdxDim * kIdxQtStride + kIdxHeads) * 4;
static_assert(kIdxRows * kIdxDotStride <= kIdxDim * kIdxQtStride, "dot tile fits in the query tile");

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  const uint32_t d = (uint32_t)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(d), "l"(gmem) : "memory");
}

// One product of rsLLM's dot for two heads: fma.rn(a, b, -0.0) is the
// correctly rounded product a * b (adding -0.0 changes no value and keeps the
// sign of a zero product).  `nz` holds -0.0 in both halves and arrives as a
// kernel argument: with a literal -0.0 the compiler may turn the fused
// multiply-add back into a multiply and contract that into the following add.
__device__ __forceinline__ unsigned long long prod2(unsigned long long a, unsigned long long b,
                                                    unsigned long long nz) {
  unsigned long long r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(nz));
  return r;
}
__device__ __forceinline__ unsigned long long dup2(float x) {
  const unsigned long long b = __float_as_uint(x);
  return (b << 32) | b;
}
constexpr unsigned long long kNegZero2 = 0x8000000080000000ull;

// Copies lanes [32 ch, 32 ch + 32) of the CTA's rows into a chunk buffer as
// one cp.async group: a warp copies 4 rows x 128 bytes per step (coalesced
// reads, conflict-free shared stores); rows past the visible end are left
// alone (the buffers' zeroed rows stay zero).
__device__ __forceinline__ void stage_chunk(float* buf, const float* rg, int n_rows, int ch, int tid) {
  constexpr int kVec = kIdxChunk / 4;
#pragma unroll 4
  for (int v = tid; v < kIdxRows * kVec; v += kIdxRows) {
    const int r = v / kVec, c = 4 * (v % kVec);
    if (r < n_rows) cp_async16(buf + r * kIdxStride + c, rg + (int64_t)r * kIdxDim + ch * kIdxChunk + c);
  }
  asm volatile("cp.async.commit_group;" ::: "memory");
}

// The thread tile over one staged chunk: rows warp*32 + rt + 4a (a < 8) and
// heads 4ht + j, 32 + 4ht + j (j < 4) as four packed pairs.  At a fixed a the
// warp reads 4 consecutive padded rows, which fall in distinct banks; the
// query pairs of one lane are 128 contiguous bytes across the warp.  The
// lanes are added in ascending order, as rsLLM's dot adds them.
__device__ __forceinline__ void dot_chunk(unsigned long long (&d)[8][4], const float* buf, const float* s_qt,
                                          int ch, int warp, int rt, int ht, unsigned long long nz) {
  const float* kvb = buf + (warp * 32 + rt) * kIdxStride;
  const float* qb = s_qt + ch * kIdxChunk * kIdxQtStride + 4 * ht;
#pragma unroll 1
  for (int i = 0; i < kIdxChunk; i += 4) {
    float4 kr[8];
#pragma unroll
    for (int a = 0; a < 8; ++a) kr[a] = *reinterpret_cast<const float4*>(kvb + 4 * a * kIdxStride + i);
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const ulonglong2 q01 = *reinterpret_cast<const ulonglong2*>(qb + (i + c) * kIdxQtStride);
      const ulonglong2 q23 = *reinterpret_cast<const ulonglong2*>(qb + (i + c) * kIdxQtStride + 32);
#pragma unroll
      for (int a = 0; a < 8; ++a) {
        const float x = c == 0 ? kr[a].x : c == 1 ? kr[a].y : c == 2 ? kr[a].z : kr[a].w;
        const unsigned long long k2 = dup2(x);
        d[a][0] = add_f32x2(d[a][0], prod2(k2, q01.x, nz));
        d[a][1] = add_f32x2(d[a][1], prod2(k2, q01.y, nz));
        d[a][2] = add_f32x2(d[a][2], prod2(k2, q23.x, nz));
        d[a][3] = add_f32x2(d[a][3], prod2(k2, q23.y, nz));
      }
    }
  }
}

__global__ void __launch_bounds__(kIdxRows, 3)
indexer_score_kernel(const float* __restrict__ rows, const int64_t* __restrict__ row_start,
                     const int32_t* __restrict__ seq_rows, int64_t n_seq, const float* __restrict__ q,
                     const float* __restrict__ w, const int32_t* __restrict__ seq_of_query,
                     const int32_t* __restrict__ n_visible, int32_t blocks_per_q, float* __restrict__ scores,
                     int64_t ld, unsigned long long nz, uint32_t* __restrict__ status) {
  extern __shared__ __align__(16) float smem[];
  float* buf0 = smem;
  float* buf1 = smem + kIdxBuf;
  float* s_qt = smem + 2 * kIdxBuf;                 // [kIdxDim][kIdxQtStride]: s_qt[i][h] = q[h][i]
  float* s_w = s_qt + kIdxDim * kIdxQtStride;       // [kIdxHeads]
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

  // rows past the visible end read as zero in both buffers
  for (int v = tid; v < (kIdxRows - n_rows) * (kIdxChunk / 4); v += kIdxRows) {
    const int r = n_rows + v / (kIdxChunk / 4), c = 4 * (v % (kIdxChunk / 4));
    *reinterpret_cast<float4*>(buf0 + r * kIdxStride + c) = make_float4(0.f, 0.f, 0.f, 0.f);
    *reinterpret_cast<float4*>(buf1 + r * kIdxStride + c) = make_float4(0.f, 0.f, 0.f, 0.f);
  }
  stage_chunk(buf0, rg, n_rows, 0, tid);
  stage_chunk(buf1, rg, n_rows, 1, tid);
  // the query, transposed while the first row chunks are in flight: a warp
  // reads lanes 4c..4c+3 of 32 consecutive heads and stores them as four
  // conflict-free rows of s_qt
  const float4* qg = reinterpret_cast<const float4*>(q + qi * (kIdxHeads * kIdxDim));
#pragma unroll 4
  for (int v = tid; v < kIdxHeads * kIdxDim / 4; v += kIdxRows) {
    const int h = v % kIdxHeads, c = 4 * (v / kIdxHeads);
    const float4 t = __ldg(qg + h * (kIdxDim / 4) + c / 4);
    s_qt[(c + 0) * kIdxQtStride + h] = t.x;
    s_qt[(c + 1) * kIdxQtStride + h] = t.y;
    s_qt[(c + 2) * kIdxQtStride + h] = t.z;
    s_qt[(c + 3) * kIdxQtStride + h] = t.w;
  }
  if (tid < kIdxHeads) s_w[tid] = __ldg(w + qi * kIdxHeads + tid);

  const int warp = tid >> 5, lane = tid & 31, rt = lane & 3, ht = lane >> 2;
  unsigned long long d[8][4];
#pragma unroll
  for (int a = 0; a < 8; ++a)
#pragma unroll
    for (int p = 0; p < 4; ++p) d[a][p] = 0ull;
  // two buffers: chunk ch + 2 is copied while chunk ch + 1 is multiplied
  static_assert(kIdxChunks == 4, "the pipeline below covers four chunks");
  asm volatile("cp.async.wait_group 1;" ::: "memory");
  __syncthreads();
  dot_chunk(d, buf0, s_qt, 0, warp, rt, ht, nz);
  __syncthreads();  // buffer 0 is free
  stage_chunk(buf0, rg, n_rows, 2, tid);
  asm volatile("cp.async.wait_group 1;" ::: "memory");
  __syncthreads();
  dot_chunk(d, buf1, s_qt, 1, warp, rt, ht, nz);
  __syncthreads();  // buffer 1 is free
  stage_chunk(buf1, rg, n_rows, 3, tid);
  asm volatile("cp.async.wait_group 1;" ::: "memory");
  __syncthreads();
  dot_chunk(d, buf0, s_qt, 2, warp, rt, ht, nz);
  asm volatile("cp.async.wait_group 0;" ::: "memory");
  __syncthreads();
  dot_chunk(d, buf1, s_qt, 3, warp, rt, ht, nz);
  __syncthreads();  // every thread is done reading the query tile

  float* s_dot = s_qt;  // [kIdxRows][kIdxDotStride]
#pragma unroll
  for (int a = 0; a < 8; ++a) {
    float* dr = s_dot + (warp * 32 + rt + 4 * a) * kIdxDotStride + 4 * ht;
    *reinterpret_cast<ulonglong2*>(dr) = make_ulonglong2(d[a][0], d[a][1]);
    *reinterpret_cast<ulonglong2*>(dr + 32) = make_ulonglong2(d[a][2], d[a][3]);
  }
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
                                     seq_of_query, n_visible, (int32_t)per_q, scores, ld, kNegZero2, d_status);
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
