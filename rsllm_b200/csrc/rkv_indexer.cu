// rkv_indexer.cu -- the indexer's scoring of compressed rows against a query,
// feeding the top-k selection: IndexerPool::select_top_k
// (crates/rsllm-kvcache/src/dsv4/indexer.rs:169-236) for a batch of queries.
//
// score[c] = sum_h relu(dot(row_c, q_h)) * w_h over 64 heads of 128 lanes.
// rsLLM accumulates every dot lane by lane and the score head by head in f32,
// each product and sum rounded on its own; the kernel does exactly that (an
// f32 dot product on tensor cores or with fused multiply-adds would round
// differently), so the scores -- and therefore the selected indices -- are
// bit-exact.  (Packed mul.rn.f32x2 / add.rn.f32x2 pairs are not used: in a
// loop ptxas was measured to contract them into fused multiply-adds on this
// B200, which changes the rounding.)  Layout: one CTA of 128 threads per
// (query, 128 rows); the query (32 KB) and its weights are staged in shared
// memory and read as broadcast 16-byte loads; each thread holds its row in 128
// registers and runs four head chains at a time (four independent add chains
// hide the add latency).
// The work is 8192 multiplies and 8192 adds per (query, row): CUDA-core
// bound, not HBM bound.
#include "rkv_common.cuh"
#include "rkv_host.h"

namespace rkv {

constexpr int kIdxHeads = 64;
constexpr int kIdxDim = 128;
constexpr int kIdxRows = 128;  // rows (threads) per CTA

__global__ void __launch_bounds__(kIdxRows, 3)
indexer_score_kernel(const float* __restrict__ rows, const int64_t* __restrict__ row_start,
                     const int32_t* __restrict__ seq_rows, int64_t n_seq, const float* __restrict__ q,
                     const float* __restrict__ w, const int32_t* __restrict__ seq_of_query,
                     const int32_t* __restrict__ n_visible, int32_t blocks_per_q, float* __restrict__ scores,
                     int64_t ld, uint32_t* __restrict__ status) {
  __shared__ __align__(16) float s_q[kIdxHeads * kIdxDim];
  __shared__ float s_w[kIdxHeads];
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
  const float4* qg = reinterpret_cast<const float4*>(q + qi * (kIdxHeads * kIdxDim));
#pragma unroll 4
  for (int v = tid; v < kIdxHeads * kIdxDim / 4; v += kIdxRows) reinterpret_cast<float4*>(s_q)[v] = __ldg(qg + v);
  if (tid < kIdxHeads) s_w[tid] = __ldg(w + qi * kIdxHeads + tid);
  __syncthreads();
  const int r = r0 + tid;
  if (r >= nv) return;

  const float4* rg = reinterpret_cast<const float4*>(rows + (__ldg(row_start + s) + r) * kIdxDim);
  float kv[kIdxDim];
#pragma unroll
  for (int v = 0; v < kIdxDim / 4; ++v) {
    const float4 t = __ldg(rg + v);
    kv[4 * v] = t.x;
    kv[4 * v + 1] = t.y;
    kv[4 * v + 2] = t.z;
    kv[4 * v + 3] = t.w;
  }
  float acc = 0.0f;
#pragma unroll 1
  for (int h = 0; h < kIdxHeads; h += 4) {
    const float* qh = s_q + h * kIdxDim;
    float d[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
    for (int i = 0; i < kIdxDim; i += 4) {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float4 qv = *reinterpret_cast<const float4*>(qh + j * kIdxDim + i);
        d[j] = __fadd_rn(d[j], __fmul_rn(kv[i], qv.x));
        d[j] = __fadd_rn(d[j], __fmul_rn(kv[i + 1], qv.y));
        d[j] = __fadd_rn(d[j], __fmul_rn(kv[i + 2], qv.z));
        d[j] = __fadd_rn(d[j], __fmul_rn(kv[i + 3], qv.w));
      }
    }
#pragma unroll
    for (int j = 0; j < 4; ++j)
      if (d[j] > 0.0f) acc = __fadd_rn(acc, __fmul_rn(d[j], s_w[h + j]));
  }
  scores[qi * ld + r] = acc;
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
  const int64_t per_q = (max_visible + kIdxRows - 1) / kIdxRows;
  const int64_t blocks = per_q * n_q;
  if (blocks > (int64_t)INT32_MAX) return fail(RKV_ERR_SHAPE_MISMATCH, "rkv_indexer_scores_f32: grid too large");
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)blocks);
  cfg.blockDim = dim3(kIdxRows);
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
