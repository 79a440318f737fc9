// rkv_gather.cu -- paged gather + dequant (dense, per sequence) and sparse
// gather + dequant (top-k selected rows) to bf16 [*, 576].
//
// A stored row is read as 512 B of codes (16 B per lane), the lane's block
// scale (4 B; lanes 4j..4j+3 share block j) and 128 B of bf16 RoPE (16 B on
// each lane of one 8-lane group); it is written as 1 KB of decoded latent
// (one 256-bit store per lane, 1 KB contiguous per warp) plus the RoPE part.
// A warp moves kRows rows at a time with every load issued before any
// decode.  Output rows must be 32-byte aligned (1152 B rows keep that).
//
// Decode: (sign * e4m3fn_value(code)) * 2^e rounded to bf16, the value the
// reference forms at crates/rsllm-backend-cpu/src/ops/dsv4_quant.rs:359;
// exact, see rkv_common.cuh.
#include "rkv_common.cuh"
#include "rkv_host.h"

namespace rkv {

// A batch of kRows rows as one warp holds it: for every row, lane l has codes
// 16l..16l+15 (16 B) and the scale of their block (l/4); for RoPE, lane l has
// 16 B of row l/8 of the batch (8 lanes per 128 B RoPE part).
constexpr int kRows = 4;

struct RowBatch {
  uint4 codes[kRows];
  float scale[kRows];
  uint4 rope;
};

__device__ __forceinline__ void load_latent(const uint8_t* pg, int off, int lane, uint4& codes, float& scale) {
  codes = ld_stream16(pg + codes_off(off) + lane * 16);
  scale = __ldg(reinterpret_cast<const float*>(pg + scales_off(off)) + (lane >> 2));
}

__device__ __forceinline__ void store_latent(uint8_t* out_row, const uint4& codes, float scale, int lane) {
  uint4 o0, o1;
  dequant16(codes, decode_scale(scale), o0, o1);
  st_stream32(out_row + lane * 32, o0, o1);  // 1 KB per warp, one instruction
}

constexpr int kGatherWarps = 8;  // one 256-thread CTA per (sequence, page)

// grid = (pages of the longest sequence, n_seq).  Warp w handles rows
// w + 8i of the page, kRows at a time (two batches cover 64 rows).
__global__ void __launch_bounds__(kGatherWarps * 32, 6)
gather_dequant_kernel(rkv_pool_view pool, int layer, const int32_t* __restrict__ page_table, int64_t pt_stride,
                      const int32_t* __restrict__ cu_seqlens, uint16_t* __restrict__ out,
                      uint32_t* __restrict__ status) {
  const int s = blockIdx.y;
  const int p = blockIdx.x;
  const int start = __ldg(cu_seqlens + s);
  const int len = __ldg(cu_seqlens + s + 1) - start;
  const int t0 = p * kPageTokens;
  if (t0 >= len) return;
  const int nrows = min(kPageTokens, len - t0);
  const int32_t page = __ldg(page_table + (int64_t)s * pt_stride + p);
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  uint8_t* out_page = reinterpret_cast<uint8_t*>(out + ((int64_t)start + t0) * kRowDim);
  const uint4 z = make_uint4(0, 0, 0, 0);
  if (page < 0 || page >= pool.n_pages) {
    if (threadIdx.x == 0) set_status(status, RKV_ERR_INDEX_OUT_OF_RANGE);
    for (int row = w; row < nrows; row += kGatherWarps) {
      uint8_t* o = out_page + (int64_t)row * (kRowDim * 2);
      st_stream32(o + lane * 32, z, z);
      if (lane < 8) st_stream16(o + 1024 + lane * 16, z);
    }
    return;
  }
  const uint8_t* pg = page_base(pool, layer, page);
  const int rl = lane >> 3;  // the batch row whose RoPE part this lane moves
#pragma unroll
  for (int base = 0; base < kPageTokens; base += kGatherWarps * kRows) {
    RowBatch b;
#pragma unroll
    for (int i = 0; i < kRows; ++i) {
      const int row = base + w + i * kGatherWarps;
      if (row < nrows) load_latent(pg, row, lane, b.codes[i], b.scale[i]);
    }
    const int rrow = base + w + rl * kGatherWarps;
    if (rrow < nrows) b.rope = ld_stream16(pg + rope_off(rrow) + (lane & 7) * 16);
#pragma unroll
    for (int i = 0; i < kRows; ++i) {
      const int row = base + w + i * kGatherWarps;
      if (row < nrows) store_latent(out_page + (int64_t)row * (kRowDim * 2), b.codes[i], b.scale[i], lane);
    }
    if (rrow < nrows) st_stream16(out_page + (int64_t)rrow * (kRowDim * 2) + 1024 + (lane & 7) * 16, b.rope);
  }
}

constexpr int kSparseWarps = 8;
constexpr int kSparseRows = 8;  // selections per warp, resolved by lanes 0..7

// One warp per kSparseRows consecutive selections of out[n_q][k].  Lanes
// 0..7 resolve index -> sequence -> page in parallel and broadcast; the rows
// are then moved kRows at a time.
__global__ void __launch_bounds__(kSparseWarps * 32, 5)
sparse_gather_dequant_kernel(rkv_pool_view pool, int layer, const int32_t* __restrict__ page_table,
                             int64_t pt_stride, const int32_t* __restrict__ seq_of_query,
                             const int32_t* __restrict__ seq_lens, const int32_t* __restrict__ idx, int64_t n_sel,
                             int k, uint16_t* __restrict__ out, uint32_t* __restrict__ status) {
  const unsigned FULL = 0xffffffffu;
  const int lane = threadIdx.x & 31;
  const int64_t g0 = ((int64_t)blockIdx.x * kSparseWarps + (threadIdx.x >> 5)) * kSparseRows;
  if (g0 >= n_sel) return;
  // lane i < kSparseRows: where selection g0 + i lives (page = -2: past the
  // end of the output, -1: write zeros)
  int32_t my_page = -2, my_off = 0;
  if (lane < kSparseRows && g0 + lane < n_sel) {
    const int64_t g = g0 + lane;
    const int32_t t = __ldg(idx + g);
    const int32_t s = __ldg(seq_of_query + g / k);
    my_page = -1;
    if (t >= 0) {
      if (t < __ldg(seq_lens + s)) {
        const int32_t pgid = __ldg(page_table + (int64_t)s * pt_stride + (t >> 6));
        if (pgid >= 0 && pgid < pool.n_pages) {
          my_page = pgid;
          my_off = t & 63;
        } else {
          set_status(status, RKV_ERR_INDEX_OUT_OF_RANGE);
        }
      } else {
        set_status(status, RKV_ERR_INDEX_OUT_OF_RANGE);
      }
    }
  }
  const int rl = lane >> 3;
  const uint4 z = make_uint4(0, 0, 0, 0);
#pragma unroll
  for (int base = 0; base < kSparseRows; base += kRows) {
    int32_t page[kRows], off[kRows];
#pragma unroll
    for (int i = 0; i < kRows; ++i) {
      page[i] = __shfl_sync(FULL, my_page, base + i);
      off[i] = __shfl_sync(FULL, my_off, base + i);
    }
    RowBatch b;
#pragma unroll
    for (int i = 0; i < kRows; ++i)
      if (page[i] >= 0) load_latent(page_base(pool, layer, page[i]), off[i], lane, b.codes[i], b.scale[i]);
    // RoPE of batch row rl (register-indexed selects, no local memory)
    int32_t rpage = page[0], roff = off[0];
#pragma unroll
    for (int i = 1; i < kRows; ++i)
      if (rl == i) {
        rpage = page[i];
        roff = off[i];
      }
    if (rpage >= 0) b.rope = ld_stream16(page_base(pool, layer, rpage) + rope_off(roff) + (lane & 7) * 16);
#pragma unroll
    for (int i = 0; i < kRows; ++i) {
      uint8_t* orow = reinterpret_cast<uint8_t*>(out + (g0 + base + i) * kRowDim);
      if (page[i] >= 0) store_latent(orow, b.codes[i], b.scale[i], lane);
      else if (page[i] == -1) st_stream32(orow + lane * 32, z, z);
    }
    uint8_t* rrow = reinterpret_cast<uint8_t*>(out + (g0 + base + rl) * kRowDim) + 1024 + (lane & 7) * 16;
    if (rpage >= 0) st_stream16(rrow, b.rope);
    else if (rpage == -1) st_stream16(rrow, z);
  }
}

}  // namespace rkv

extern "C" rkv_status rkv_gather_dequant_bf16(const rkv_pool_view* pool, int32_t layer, const int32_t* page_table,
                                              int64_t pt_stride, const int32_t* cu_seqlens, int32_t n_seq,
                                              int32_t max_seq_len, uint16_t* out, uint32_t* d_status,
                                              rkv_stream_t stream) {
  using namespace rkv;
  rkv_status st = check_pool(pool, "rkv_gather_dequant_bf16");
  if (st != RKV_OK) return st;
  if (layer < 0 || layer >= pool->n_layers)
    return fail_layer(layer, pool->n_layers, "rkv_gather_dequant_bf16: layer %d outside pool of %d layers", layer,
                      pool->n_layers);
  if (n_seq < 0 || max_seq_len < 0)
    return fail_shape(n_seq < 0 ? "n_seq" : "max_seq_len", 0, n_seq < 0 ? n_seq : max_seq_len,
                      "rkv_gather_dequant_bf16: negative sizes");
  if (n_seq == 0 || max_seq_len == 0) {
    clear_error();
    return RKV_OK;
  }
  const int64_t pages = (max_seq_len + kPageTokens - 1) / kPageTokens;
  if (pt_stride < pages)
    return fail_shape("pt_stride", pages, pt_stride, "rkv_gather_dequant_bf16: pt_stride %lld < %lld pages",
                      (long long)pt_stride, (long long)pages);
  if (n_seq > 65535)
    return fail_shape("n_seq", 65535, n_seq, "rkv_gather_dequant_bf16: at most 65535 sequences per call");
  if (!page_table || !cu_seqlens || !out || !aligned(out, 32))
    return fail(RKV_ERR_INVALID_ARGUMENT, "rkv_gather_dequant_bf16: page_table, cu_seqlens and a 32-byte aligned out are required");
  dim3 grid((unsigned)pages, (unsigned)n_seq);
  gather_dequant_kernel<<<grid, kGatherWarps * 32, 0, (cudaStream_t)stream>>>(*pool, layer, page_table, pt_stride,
                                                                            cu_seqlens, out, d_status);
  return check_launch("rkv_gather_dequant_bf16");
}

extern "C" rkv_status rkv_sparse_gather_dequant_bf16(const rkv_pool_view* pool, int32_t layer,
                                                     const int32_t* page_table, int64_t pt_stride,
                                                     const int32_t* seq_of_query, const int32_t* seq_lens,
                                                     const int32_t* idx, int32_t n_q, int32_t k, uint16_t* out,
                                                     uint32_t* d_status, rkv_stream_t stream) {
  using namespace rkv;
  rkv_status st = check_pool(pool, "rkv_sparse_gather_dequant_bf16");
  if (st != RKV_OK) return st;
  if (layer < 0 || layer >= pool->n_layers)
    return fail_layer(layer, pool->n_layers, "rkv_sparse_gather_dequant_bf16: layer %d outside pool of %d layers",
                      layer, pool->n_layers);
  if (n_q < 0 || k < 0)
    return fail_shape(n_q < 0 ? "n_q" : "k", 0, n_q < 0 ? n_q : k, "rkv_sparse_gather_dequant_bf16: negative sizes");
  const int64_t n_sel = (int64_t)n_q * k;
  if (n_sel == 0) {
    clear_error();
    return RKV_OK;
  }
  if (!page_table || !seq_of_query || !seq_lens || !idx || !out || !aligned(out, 32))
    return fail(RKV_ERR_INVALID_ARGUMENT,
                "rkv_sparse_gather_dequant_bf16: page_table, seq_of_query, seq_lens, idx and a 32-byte aligned out are required");
  const int64_t per_cta = (int64_t)kSparseWarps * kSparseRows;
  const int64_t grid = (n_sel + per_cta - 1) / per_cta;
  if (grid > INT32_MAX) return fail_shape("idx", INT32_MAX, n_sel, "rkv_sparse_gather_dequant_bf16: too many rows");
  sparse_gather_dequant_kernel<<<(unsigned)grid, kSparseWarps * 32, 0, (cudaStream_t)stream>>>(
      *pool, layer, page_table, pt_stride, seq_of_query, seq_lens, idx, n_sel, k, out, d_status);
  return check_launch("rkv_sparse_gather_dequant_bf16");
}
