// rkv_gather.cu -- paged gather + dequant (dense, per sequence) and sparse
// gather + dequant (top-k selected rows) to bf16 [*, 576].
//
// Both read a stored row as 512 B of codes (16 B per lane), the lane's block
// scale (4 B, lanes 4j..4j+3 share block j) and, on lanes 0..7, 16 B of the
// bf16 RoPE part; they write 1152 B per row (32 B of decoded latent per lane
// plus the RoPE part).  Loads for several rows are issued before any decode
// so each warp keeps several KB in flight.
//
// Decode: (sign * e4m3fn_value(code)) * 2^e rounded to bf16, the value the
// reference forms at crates/rsllm-backend-cpu/src/ops/dsv4_quant.rs:359;
// exact, see rkv_common.cuh.
#include "rkv_common.cuh"
#include "rkv_host.h"

namespace rkv {

struct RowLoad {
  uint4 codes;
  float scale;
  uint4 rope;
};

__device__ __forceinline__ RowLoad load_row(const uint8_t* pg, int off, int lane) {
  RowLoad r;
  r.codes = ld_stream16(pg + codes_off(off) + lane * 16);
  r.scale = __ldg(reinterpret_cast<const float*>(pg + scales_off(off)) + (lane >> 2));
  r.rope = make_uint4(0, 0, 0, 0);
  if (lane < 8) r.rope = ld_stream16(pg + rope_off(off) + lane * 16);
  return r;
}

__device__ __forceinline__ void store_row(uint8_t* out_row, const RowLoad& r, int lane) {
  uint4 o0, o1;
  dequant16(r.codes, decode_scale(r.scale), o0, o1);
  st_stream16(out_row + lane * 32, o0);
  st_stream16(out_row + lane * 32 + 16, o1);
  if (lane < 8) st_stream16(out_row + 1024 + lane * 16, r.rope);
}

__device__ __forceinline__ void zero_row(uint8_t* out_row, int lane) {
  const uint4 z = make_uint4(0, 0, 0, 0);
  st_stream16(out_row + lane * 32, z);
  st_stream16(out_row + lane * 32 + 16, z);
  if (lane < 8) st_stream16(out_row + 1024 + lane * 16, z);
}

constexpr int kGatherWarps = 8;  // one 256-thread CTA per (sequence, page)
constexpr int kRowsInFlight = 4;  // rows each warp loads before decoding

// grid = (pages per longest sequence, n_seq).  Warp w handles rows
// w, w+8, ..., w+56 of the page, kRowsInFlight at a time.
__global__ void __launch_bounds__(kGatherWarps * 32)
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
  if (page < 0 || page >= pool.n_pages) {
    if (threadIdx.x == 0) set_status(status, RKV_ERR_INDEX_OUT_OF_RANGE);
    for (int row = w; row < nrows; row += kGatherWarps) zero_row(out_page + (int64_t)row * (kRowDim * 2), lane);
    return;
  }
  const uint8_t* pg = page_base(pool, layer, page);
#pragma unroll
  for (int base = 0; base < kPageTokens; base += kGatherWarps * kRowsInFlight) {
    RowLoad ld[kRowsInFlight];
#pragma unroll
    for (int i = 0; i < kRowsInFlight; ++i) {
      const int row = base + w + i * kGatherWarps;
      if (row < nrows) ld[i] = load_row(pg, row, lane);
    }
#pragma unroll
    for (int i = 0; i < kRowsInFlight; ++i) {
      const int row = base + w + i * kGatherWarps;
      if (row < nrows) store_row(out_page + (int64_t)row * (kRowDim * 2), ld[i], lane);
    }
  }
}

constexpr int kSparseWarps = 8;
constexpr int kSparseRowsPerWarp = 4;

// One warp per kSparseRowsPerWarp consecutive selections of out[n_q][k].
__global__ void __launch_bounds__(kSparseWarps * 32)
sparse_gather_dequant_kernel(rkv_pool_view pool, int layer, const int32_t* __restrict__ page_table,
                             int64_t pt_stride, const int32_t* __restrict__ seq_of_query,
                             const int32_t* __restrict__ seq_lens, const int32_t* __restrict__ idx, int64_t n_sel,
                             int k, uint16_t* __restrict__ out, uint32_t* __restrict__ status) {
  const int lane = threadIdx.x & 31;
  const int64_t g0 = ((int64_t)blockIdx.x * kSparseWarps + (threadIdx.x >> 5)) * kSparseRowsPerWarp;
  if (g0 >= n_sel) return;
  int64_t page[kSparseRowsPerWarp];
  int off[kSparseRowsPerWarp];
#pragma unroll
  for (int i = 0; i < kSparseRowsPerWarp; ++i) {
    const int64_t g = g0 + i;
    page[i] = -2;  // -2: past the end, -1: write zeros
    off[i] = 0;
    if (g < n_sel) {
      const int32_t t = __ldg(idx + g);
      const int32_t s = __ldg(seq_of_query + g / k);
      page[i] = -1;
      if (t >= 0) {
        if (t < __ldg(seq_lens + s)) {
          const int32_t pgid = __ldg(page_table + (int64_t)s * pt_stride + (t >> 6));
          if (pgid >= 0 && pgid < pool.n_pages) {
            page[i] = pgid;
            off[i] = t & 63;
          } else if (lane == 0) {
            set_status(status, RKV_ERR_INDEX_OUT_OF_RANGE);
          }
        } else if (lane == 0) {
          set_status(status, RKV_ERR_INDEX_OUT_OF_RANGE);
        }
      }
    }
  }
  RowLoad ld[kSparseRowsPerWarp];
#pragma unroll
  for (int i = 0; i < kSparseRowsPerWarp; ++i)
    if (page[i] >= 0) ld[i] = load_row(page_base(pool, layer, page[i]), off[i], lane);
#pragma unroll
  for (int i = 0; i < kSparseRowsPerWarp; ++i) {
    uint8_t* orow = reinterpret_cast<uint8_t*>(out + (g0 + i) * kRowDim);
    if (page[i] >= 0) store_row(orow, ld[i], lane);
    else if (page[i] == -1) zero_row(orow, lane);
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
    return fail(RKV_ERR_INVALID_LAYER, "rkv_gather_dequant_bf16: layer %d outside pool of %d layers", layer,
                pool->n_layers);
  if (n_seq < 0 || max_seq_len < 0) return fail(RKV_ERR_SHAPE_MISMATCH, "rkv_gather_dequant_bf16: negative sizes");
  if (n_seq == 0 || max_seq_len == 0) {
    clear_error();
    return RKV_OK;
  }
  const int64_t pages = (max_seq_len + kPageTokens - 1) / kPageTokens;
  if (pt_stride < pages)
    return fail(RKV_ERR_SHAPE_MISMATCH, "rkv_gather_dequant_bf16: pt_stride %lld < %lld pages", (long long)pt_stride,
                (long long)pages);
  if (n_seq > 65535) return fail(RKV_ERR_SHAPE_MISMATCH, "rkv_gather_dequant_bf16: at most 65535 sequences per call");
  if (!page_table || !cu_seqlens || !out || !aligned(out, 16))
    return fail(RKV_ERR_INVALID_ARGUMENT, "rkv_gather_dequant_bf16: page_table, cu_seqlens and a 16-byte aligned out are required");
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
    return fail(RKV_ERR_INVALID_LAYER, "rkv_sparse_gather_dequant_bf16: layer %d outside pool of %d layers", layer,
                pool->n_layers);
  if (n_q < 0 || k < 0) return fail(RKV_ERR_SHAPE_MISMATCH, "rkv_sparse_gather_dequant_bf16: negative sizes");
  const int64_t n_sel = (int64_t)n_q * k;
  if (n_sel == 0) {
    clear_error();
    return RKV_OK;
  }
  if (!page_table || !seq_of_query || !seq_lens || !idx || !out || !aligned(out, 16))
    return fail(RKV_ERR_INVALID_ARGUMENT,
                "rkv_sparse_gather_dequant_bf16: page_table, seq_of_query, seq_lens, idx and a 16-byte aligned out are required");
  const int64_t per_cta = (int64_t)kSparseWarps * kSparseRowsPerWarp;
  const int64_t grid = (n_sel + per_cta - 1) / per_cta;
  if (grid > INT32_MAX) return fail(RKV_ERR_SHAPE_MISMATCH, "rkv_sparse_gather_dequant_bf16: too many rows");
  sparse_gather_dequant_kernel<<<(unsigned)grid, kSparseWarps * 32, 0, (cudaStream_t)stream>>>(
      *pool, layer, page_table, pt_stride, seq_of_query, seq_lens, idx, n_sel, k, out, d_status);
  return check_launch("rkv_sparse_gather_dequant_bf16");
}
