// rkv_append.cu -- quantize-on-append of bf16 KV rows into the paged pool.
//
// One warp per row (576 bf16 = 1152 B in, 672 B out).  Lane l loads 16 B of
// each latent half (lanes 8j..8j+7 cover 64-lane block j of that half) and,
// for l < 8, 16 B of the RoPE part; all loads are issued before any math.
// The block amax is a 3-step xor-shuffle inside each 8-lane group on the bf16
// magnitude bits (integer max, so NaN/inf are caught by the same value).
// Codes go out as one 256 B coalesced run per half, the 8 block scales as one
// 32 B sector, the RoPE part as 128 B.
//
// Semantics: crates/rsllm-backend-cpu/src/ops/dsv4_quant.rs:316-362 applied
// per row (see rkv_common.cuh), row placement of crates/rsllm-kvcache/src/
// dsv4/swa.rs:73-94 generalised to a slot mapping.
#include "rkv_common.cuh"
#include "rkv_host.h"

namespace rkv {

constexpr int kAppendWarps = 8;  // rows per 256-thread CTA

__global__ void __launch_bounds__(kAppendWarps * 32)
append_quant_kernel(rkv_pool_view pool, int layer0, uint32_t n_tokens, uint32_t n_rows,
                    const uint16_t* __restrict__ rows, const int32_t* __restrict__ slots,
                    uint32_t* __restrict__ status) {
  const unsigned FULL = 0xffffffffu;
  const int lane = threadIdx.x & 31;
  const uint32_t r = blockIdx.x * kAppendWarps + (threadIdx.x >> 5);
  if (r >= n_rows) return;
  const uint32_t li = r / n_tokens;
  const uint32_t t = r - li * n_tokens;
  const int32_t slot = __ldg(slots + t);
  if (slot < 0) return;  // padding token
  const int64_t page = slot >> 6;
  const int off = slot & 63;
  if (page >= pool.n_pages) {
    if (lane == 0) set_status(status, RKV_ERR_INDEX_OUT_OF_RANGE);
    return;
  }

  const uint8_t* src = reinterpret_cast<const uint8_t*>(rows) + (size_t)r * (kRowDim * 2);
  const uint4 a = ld_stream16(src + lane * 16);
  const uint4 b = ld_stream16(src + 512 + lane * 16);
  uint4 rp = make_uint4(0, 0, 0, 0);
  if (lane < 8) rp = ld_stream16(src + 1024 + lane * 16);

  uint32_t ma = absmax_bits8(a), mb = absmax_bits8(b);
#pragma unroll
  for (int o = 1; o < 8; o <<= 1) {
    ma = max(ma, __shfl_xor_sync(FULL, ma, o));
    mb = max(mb, __shfl_xor_sync(FULL, mb, o));
  }
  // A non-finite latent lane rejects the whole row before anything is written.
  if (__any_sync(FULL, (ma >= 0x7f80u) | (mb >= 0x7f80u))) {
    if (lane == 0) set_status(status, RKV_ERR_NON_FINITE_INPUT);
    return;
  }
  const int ea = scale_exponent_bf16amax(__uint_as_float(ma << 16));
  const int eb = scale_exponent_bf16amax(__uint_as_float(mb << 16));
  const uint2 ca = quant8(a, __uint_as_float((uint32_t)(127 - ea) << 23));
  const uint2 cb = quant8(b, __uint_as_float((uint32_t)(127 - eb) << 23));

  uint8_t* pg = page_base(pool, layer0 + (int)li, page);
  st_stream8(pg + codes_off(off) + lane * 8, ca);
  st_stream8(pg + codes_off(off) + 256 + lane * 8, cb);
  // Lane j < 8 stores the scale of block j: blocks 0..3 live on lanes
  // 0,8,16,24 of the first half, blocks 4..7 on the same lanes of the second.
  const float sa = __shfl_sync(FULL, __uint_as_float((uint32_t)(ea + 127) << 23), (lane & 3) * 8);
  const float sb = __shfl_sync(FULL, __uint_as_float((uint32_t)(eb + 127) << 23), (lane & 3) * 8);
  if (lane < 8) {
    reinterpret_cast<float*>(pg + scales_off(off))[lane] = lane < 4 ? sa : sb;
    st_stream16(pg + rope_off(off) + lane * 16, rp);
  }
}

// Exhaustive-check helper: the same per-lane conversion on raw f32 values.
__global__ void e4m3_code_range_kernel(uint32_t first, int64_t n, uint8_t* __restrict__ out) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    float x = __uint_as_float(first + (uint32_t)i);
    float t = __fadd_rn(fminf(fmaxf(x, -448.0f), 448.0f), 0.0f);
    out[i] = (uint8_t)(cvt_e4m3x2(t, 0.0f) & 0xffu);
  }
}

}  // namespace rkv

extern "C" rkv_status rkv_append_quant_bf16(const rkv_pool_view* pool, int32_t layer0, int32_t n_layers_in,
                                            const uint16_t* rows, int64_t n_tokens, const int32_t* slot_mapping,
                                            uint32_t* d_status, rkv_stream_t stream) {
  using namespace rkv;
  rkv_status st = check_pool(pool, "rkv_append_quant_bf16");
  if (st != RKV_OK) return st;
  if (layer0 < 0 || n_layers_in < 0 || (int64_t)layer0 + n_layers_in > pool->n_layers)
    return fail(RKV_ERR_INVALID_LAYER, "rkv_append_quant_bf16: layers [%d, %d) outside pool of %d layers", layer0,
                layer0 + n_layers_in, pool->n_layers);
  if (n_tokens < 0) return fail(RKV_ERR_SHAPE_MISMATCH, "rkv_append_quant_bf16: n_tokens < 0");
  const int64_t n_rows = n_tokens * (int64_t)n_layers_in;
  if (n_rows == 0) {
    clear_error();
    return RKV_OK;
  }
  if (n_rows > (int64_t)INT32_MAX) return fail(RKV_ERR_SHAPE_MISMATCH, "rkv_append_quant_bf16: too many rows in one call");
  if (!rows || !aligned(rows, 16) || !slot_mapping || !aligned(slot_mapping, 4))
    return fail(RKV_ERR_INVALID_ARGUMENT, "rkv_append_quant_bf16: rows (16-byte aligned) and slot_mapping are required");
  const unsigned grid = (unsigned)((n_rows + kAppendWarps - 1) / kAppendWarps);
  append_quant_kernel<<<grid, kAppendWarps * 32, 0, (cudaStream_t)stream>>>(
      *pool, layer0, (uint32_t)n_tokens, (uint32_t)n_rows, rows, slot_mapping, d_status);
  return check_launch("rkv_append_quant_bf16");
}

extern "C" rkv_status rkv_e4m3fn_code_range(uint32_t first_bits, int64_t n, uint8_t* out, rkv_stream_t stream) {
  using namespace rkv;
  if (n < 0 || (n > 0 && !out)) return fail(RKV_ERR_INVALID_ARGUMENT, "rkv_e4m3fn_code_range: bad output");
  if (n > 0x100000000LL - (int64_t)first_bits) return fail(RKV_ERR_SHAPE_MISMATCH, "rkv_e4m3fn_code_range: range wraps");
  if (n == 0) return RKV_OK;
  e4m3_code_range_kernel<<<148 * 8, 256, 0, (cudaStream_t)stream>>>(first_bits, n, out);
  return check_launch("rkv_e4m3fn_code_range");
}
