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

#include <atomic>
#include <mutex>

#include "rkv_common.cuh"
#include "rkv_f32row.cuh"
#include "rkv_host.h"

namespace rkv {

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

const ThresholdTable& f32_threshold_table() {
  std::call_once(g_table_once, build_table);
  return g_table;
}

// Persistent grid, one row per warp at a time with the next row prefetched,
// launched with programmatic dependent launch (as the bf16 kernel).
__global__ void __launch_bounds__(kF32Warps * 32)
append_quant_f32_kernel(rkv_pool_view pool, int layer0, uint32_t n_tokens, uint32_t n_rows,
                        const float* __restrict__ rows, const int32_t* __restrict__ slots,
                        uint32_t* __restrict__ status, const ThresholdTable tab, unsigned long long nz2) {
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
    append_row_f32(pool, layer0 + (int)(r / n_tokens), cur, tab, status, lane, nz2);
    cur = nxt;
  }
}

}  // namespace rkv

extern "C" void rkv_scale_threshold_table(uint32_t* out) {
  const rkv::ThresholdTable& t = rkv::f32_threshold_table();
  for (int i = 0; i < 256; ++i) out[i] = t.m[i];
}

extern "C" rkv_status rkv_append_quant_f32(const rkv_pool_view* pool, int32_t layer0, int32_t n_layers_in,
                                           const float* rows, int64_t n_tokens, const int32_t* slot_mapping,
                                           uint32_t* d_status, rkv_stream_t stream) {
  using namespace rkv;
  rkv_status st = check_pool(pool, "rkv_append_quant_f32");
  if (st != RKV_OK) return st;
  if (layer0 < 0 || n_layers_in < 0 || (int64_t)layer0 + n_layers_in > pool->n_layers)
    return fail_layer(layer0 < 0 || n_layers_in < 0 ? layer0 : (int64_t)layer0 + n_layers_in - 1, pool->n_layers,
                      "rkv_append_quant_f32: layers [%d, %d) outside pool of %d layers", layer0,
                      layer0 + n_layers_in, pool->n_layers);
  if (n_tokens < 0) return fail_shape("n_tokens", 0, n_tokens, "rkv_append_quant_f32: n_tokens < 0");
  const int64_t n_rows = n_tokens * (int64_t)n_layers_in;
  if (n_rows == 0) {
    clear_error();
    return RKV_OK;
  }
  if (n_rows > (int64_t)INT32_MAX)
    return fail_shape("rows", INT32_MAX, n_rows, "rkv_append_quant_f32: too many rows in one call");
  if (!rows || !aligned(rows, 32) || !slot_mapping || !aligned(slot_mapping, 4))
    return fail(RKV_ERR_INVALID_ARGUMENT, "rkv_append_quant_f32: rows (32-byte aligned) and slot_mapping are required");
  const ThresholdTable& tab = f32_threshold_table();
  static std::atomic<int> resident_of[kMaxDevicesCached];  // one wave of this kernel, per device
  int dev = 0;
  cudaGetDevice(&dev);
  int resident = (dev >= 0 && dev < kMaxDevicesCached) ? resident_of[dev].load(std::memory_order_relaxed) : 0;
  if (resident == 0) {
    int sms = 0, per_sm = 0;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, append_quant_f32_kernel, kF32Warps * 32, 0);
    resident = (sms > 0 && per_sm > 0) ? sms * per_sm : 148 * 4;
    if (dev >= 0 && dev < kMaxDevicesCached) resident_of[dev].store(resident, std::memory_order_relaxed);
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
                                     (uint32_t)n_rows, rows, slot_mapping, d_status, tab,
                                     0x8000000080000000ull);  // -0.0 in both halves, for quant_pair_f32
  if (e != cudaSuccess) return fail(RKV_ERR_CUDA, "rkv_append_quant_f32: launch failed: %s", cudaGetErrorString(e));
  return check_launch("rkv_append_quant_f32");
}
