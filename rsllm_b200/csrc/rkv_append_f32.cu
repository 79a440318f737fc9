// rkv_append_f32.cu -- quantize-on-append of f32 KV rows (rsLLM's own row
// type) into the paged pool, bit-exact with rsLLM's CPU round trip.
//
// rsLLM computes the block exponent as ceil(log2f(max(amax, 1e-4) / 448)) with
// glibc log2f (crates/rsllm-backend-cpu/src/ops/dsv4_quant.rs:346-355).  For
// bf16 amax the quotient is never close to a power of two above it and the
// integer rule of rkv_common.cuh suffices; for arbitrary f32 amax, log2f of a
// value just above 2^E rounds down to E in most binades, so the exponent is E
// there, not E + 1.  The library therefore probes the host's log2f once per
// process and keeps, per binade of y = amax / 448, the smallest mantissa at
// which log2f(y) exceeds E (the threshold table); the kernel computes y with
// the same IEEE division and compares its mantissa with the table entry.
// The table is exposed (rkv_scale_threshold_table) so that it can be checked
// against the reference's log2f over every f32 in range.
//
// The RoPE lanes are stored as bf16 (round to nearest even): the stored row
// format holds bf16 RoPE, and the gathered bf16 rows equal rsLLM's f32 round
// trip rounded to bf16 in every lane.
#include <math.h>

#include <mutex>

#include "rkv_common.cuh"
#include "rkv_host.h"

namespace rkv {

struct ThresholdTable {
  uint32_t m[256];  // by biased exponent of y: exponent + 1 iff mantissa >= m
};

static ThresholdTable g_table;
static std::once_flag g_table_once;

static void build_table() {
  for (int eb = 0; eb < 256; ++eb) g_table.m[eb] = 0x800000u;  // never reached: exponent stays E
  for (int eb = 1; eb < 255; ++eb) {
    const float E = (float)(eb - 127);
    uint32_t lo = 1, hi = 0x7fffffu;  // smallest mantissa with log2f(y) > E
    auto above = [&](uint32_t m) {
      const uint32_t bits = ((uint32_t)eb << 23) | m;
      float y;
      memcpy(&y, &bits, 4);
      return log2f(y) > E;
    };
    if (!above(hi)) continue;
    while (lo < hi) {
      const uint32_t mid = lo + (hi - lo) / 2;
      if (above(mid)) hi = mid;
      else lo = mid + 1;
    }
    g_table.m[eb] = lo;
  }
}

static const ThresholdTable& table() {
  std::call_once(g_table_once, build_table);
  return g_table;
}

constexpr int kF32Warps = 8;

__device__ __forceinline__ int scale_exponent_f32(uint32_t amax_bits, const ThresholdTable& tab) {
  const float amax = fmaxf(__uint_as_float(amax_bits), 1.0e-4f);
  const uint32_t y = __float_as_uint(__fdiv_rn(amax, 448.0f));
  const uint32_t eb = y >> 23;
  return (int)eb - 127 + ((y & 0x7fffffu) >= tab.m[eb] ? 1 : 0);
}

// One f32 row as a warp holds it: lane l has latent lanes 16l..16l+15 (64 B,
// two 256-bit loads; block l/4); lanes 0..7 hold 32 B of the RoPE part.
struct RowF32 {
  uint32_t a[8], b[8];
  uint32_t rope[8];
  int32_t slot;
};

__device__ __forceinline__ void load_row_f32(const uint8_t* rows, const int32_t* __restrict__ slots, uint32_t r,
                                             uint32_t n_tokens, int lane, RowF32& x) {
  const uint8_t* src = rows + (size_t)r * (kRowDim * 4);
  ld_stream32(src + lane * 64, x.a);
  ld_stream32(src + lane * 64 + 32, x.b);
  if (lane < 8) ld_stream32(src + 2048 + lane * 32, x.rope);
  x.slot = __ldg(slots + r % n_tokens);
}

__device__ __forceinline__ uint32_t quant_pair_f32(uint32_t lo, uint32_t hi, unsigned long long inv2) {
  const unsigned long long v = ((unsigned long long)hi << 32) | lo;
  const unsigned long long t = add_f32x2(mul_f32x2(v, inv2), 0ull);
  return cvt_e4m3x2(__uint_as_float((uint32_t)t), __uint_as_float((uint32_t)(t >> 32)));
}

// Two f32 -> bf16x2, round to nearest even; a NaN keeps its sign and top
// payload bits with the quiet bit set (the rule of the host's conversion),
// not the canonical NaN the instruction writes.
__device__ __forceinline__ uint32_t bf16x2_rn(uint32_t lo, uint32_t hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(__uint_as_float(hi)), "f"(__uint_as_float(lo)));
  if ((lo & 0x7fffffffu) > 0x7f800000u) r = (r & 0xffff0000u) | (lo >> 16) | 0x40u;
  if ((hi & 0x7fffffffu) > 0x7f800000u) r = (r & 0x0000ffffu) | ((hi & 0xffff0000u) | 0x400000u);
  return r;
}

__device__ __forceinline__ void append_row_f32(const rkv_pool_view& pool, int layer, const RowF32& x,
                                               const ThresholdTable& tab, uint32_t* status, int lane) {
  const unsigned FULL = 0xffffffffu;
  if (x.slot < 0) return;
  const int64_t page = x.slot >> 6;
  const int off = x.slot & 63;
  uint32_t m = 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) m = max(m, max(x.a[i] & 0x7fffffffu, x.b[i] & 0x7fffffffu));
  m = max(m, __shfl_xor_sync(FULL, m, 1));
  m = max(m, __shfl_xor_sync(FULL, m, 2));
  if (page >= pool.n_pages) {
    if (lane == 0) set_status(status, RKV_ERR_INDEX_OUT_OF_RANGE);
    return;
  }
  if (__any_sync(FULL, m >= 0x7f800000u)) {  // a non-finite latent lane rejects the row before any write
    if (lane == 0) set_status(status, RKV_ERR_NON_FINITE_INPUT);
    return;
  }
  const int e = scale_exponent_f32(m, tab);
  const uint32_t invb = (uint32_t)(127 - e) << 23;
  const unsigned long long inv2 = ((unsigned long long)invb << 32) | invb;
  uint32_t c[8];
#pragma unroll
  for (int i = 0; i < 4; ++i) c[i] = quant_pair_f32(x.a[2 * i], x.a[2 * i + 1], inv2);
#pragma unroll
  for (int i = 0; i < 4; ++i) c[4 + i] = quant_pair_f32(x.b[2 * i], x.b[2 * i + 1], inv2);
  uint8_t* pg = page_base(pool, layer, page);
  st_stream16(pg + codes_off(off) + lane * 16,
              make_uint4(c[0] | (c[1] << 16), c[2] | (c[3] << 16), c[4] | (c[5] << 16), c[6] | (c[7] << 16)));
  const float sc = __shfl_sync(FULL, __uint_as_float((uint32_t)(e + 127) << 23), (lane & 7) * 4);
  if (lane < 8) {
    reinterpret_cast<float*>(pg + scales_off(off))[lane] = sc;
    st_stream16(pg + rope_off(off) + lane * 16,
                make_uint4(bf16x2_rn(x.rope[0], x.rope[1]), bf16x2_rn(x.rope[2], x.rope[3]),
                           bf16x2_rn(x.rope[4], x.rope[5]), bf16x2_rn(x.rope[6], x.rope[7])));
  }
}

// Persistent grid, one row per warp at a time with the next row prefetched,
// launched with programmatic dependent launch (as the bf16 kernel).
__global__ void __launch_bounds__(kF32Warps * 32)
append_quant_f32_kernel(rkv_pool_view pool, int layer0, uint32_t n_tokens, uint32_t n_rows,
                        const float* __restrict__ rows, const int32_t* __restrict__ slots,
                        uint32_t* __restrict__ status, const ThresholdTable tab) {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int lane = threadIdx.x & 31;
  const uint32_t stride = gridDim.x * kF32Warps;
  uint32_t r = blockIdx.x * kF32Warps + (threadIdx.x >> 5);
  if (r >= n_rows) return;
  const uint8_t* rows8 = reinterpret_cast<const uint8_t*>(rows);
  RowF32 cur, nxt;
  load_row_f32(rows8, slots, r, n_tokens, lane, cur);
  for (; r < n_rows; r += stride) {
    const uint32_t rn = r + stride;
    if (rn < n_rows) load_row_f32(rows8, slots, rn, n_tokens, lane, nxt);
    append_row_f32(pool, layer0 + (int)(r / n_tokens), cur, tab, status, lane);
    cur = nxt;
  }
}

}  // namespace rkv

extern "C" void rkv_scale_threshold_table(uint32_t* out) {
  const rkv::ThresholdTable& t = rkv::table();
  for (int i = 0; i < 256; ++i) out[i] = t.m[i];
}

extern "C" rkv_status rkv_append_quant_f32(const rkv_pool_view* pool, int32_t layer0, int32_t n_layers_in,
                                           const float* rows, int64_t n_tokens, const int32_t* slot_mapping,
                                           uint32_t* d_status, rkv_stream_t stream) {
  using namespace rkv;
  rkv_status st = check_pool(pool, "rkv_append_quant_f32");
  if (st != RKV_OK) return st;
  if (layer0 < 0 || n_layers_in < 0 || (int64_t)layer0 + n_layers_in > pool->n_layers)
    return fail(RKV_ERR_INVALID_LAYER, "rkv_append_quant_f32: layers [%d, %d) outside pool of %d layers", layer0,
                layer0 + n_layers_in, pool->n_layers);
  if (n_tokens < 0) return fail(RKV_ERR_SHAPE_MISMATCH, "rkv_append_quant_f32: n_tokens < 0");
  const int64_t n_rows = n_tokens * (int64_t)n_layers_in;
  if (n_rows == 0) {
    clear_error();
    return RKV_OK;
  }
  if (n_rows > (int64_t)INT32_MAX) return fail(RKV_ERR_SHAPE_MISMATCH, "rkv_append_quant_f32: too many rows in one call");
  if (!rows || !aligned(rows, 32) || !slot_mapping || !aligned(slot_mapping, 4))
    return fail(RKV_ERR_INVALID_ARGUMENT, "rkv_append_quant_f32: rows (32-byte aligned) and slot_mapping are required");
  const ThresholdTable& tab = table();
  static int resident = 0;
  if (resident == 0) {
    int dev = 0, sms = 0, per_sm = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, append_quant_f32_kernel, kF32Warps * 32, 0);
    resident = (sms > 0 && per_sm > 0) ? sms * per_sm : 148 * 4;
  }
  const int64_t need = (n_rows + kF32Warps - 1) / kF32Warps;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(need < resident ? need : resident));
  cfg.blockDim = dim3(kF32Warps * 32);
  cfg.stream = (cudaStream_t)stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const rkv_pool_view v = *pool;
  cudaError_t e = cudaLaunchKernelEx(&cfg, append_quant_f32_kernel, v, (int)layer0, (uint32_t)n_tokens,
                                     (uint32_t)n_rows, rows, slot_mapping, d_status, tab);
  if (e != cudaSuccess) return fail(RKV_ERR_CUDA, "rkv_append_quant_f32: launch failed: %s", cudaGetErrorString(e));
  return check_launch("rkv_append_quant_f32");
}
