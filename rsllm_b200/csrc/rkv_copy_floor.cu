// rkv_copy_floor.cu -- the memory-traffic floor of the decode append, for
// measurement.
//
// rkv_copy_floor_bf16 moves exactly the bytes rkv_append_quant_bf16_ex moves
// with RKV_APPEND_INPUTS_READY -- per row 1152 B read (32 B of latent per
// lane, 4 B of RoPE per lane, the slot) and 672 B written to the row's pool
// slot (a 512 B code run, 32 B of scales, 128 B of RoPE) -- with the same
// persistent grid of 256-thread CTAs, the same two rows per warp loaded before
// griddepcontrol.wait and the same programmatic dependent launch, but stores
// bytes it already holds instead of computing the codes and scales.  Timing
// it in the same graph as the append shows how close the append runs to a
// plain copy of its own traffic.  The rows it writes are not valid FP8 rows:
// it is for benchmarks on pools whose contents no longer matter.
#include <atomic>

#include "rkv_common.cuh"
#include "rkv_host.h"

namespace rkv {

constexpr int kFloorWarps = 8;  // 256-thread CTAs, as the append
constexpr int kFloorRows = 2;   // rows per warp loaded ahead, as the early append

__device__ __forceinline__ void floor_load(const uint8_t* rows8, const int32_t* slots, uint32_t r,
                                           uint32_t n_tokens, int lane, uint32_t (&lat)[8], uint32_t& rope,
                                           int32_t& slot) {
  const uint8_t* row = rows8 + (size_t)r * (kRowDim * 2);
  ld_stream32(row + lane * 32, lat);
  rope = ld_stream4(row + 1024 + lane * 4);
  slot = __ldg(slots + r % n_tokens);
}

__device__ __forceinline__ void floor_store(const rkv_pool_view& pool, int layer, int32_t slot,
                                            const uint32_t (&lat)[8], uint32_t rope, int lane) {
  if (slot < 0) return;
  const int64_t page = slot >> 6;
  if (page >= pool.n_pages) return;
  const int off = slot & 63;
  uint8_t* pg = page_base(pool, layer, page);
  st_stream16(pg + codes_off(off) + lane * 16, make_uint4(lat[0], lat[1], lat[2], lat[3]));
  if (lane < 8) reinterpret_cast<uint32_t*>(pg + scales_off(off))[lane] = lat[4];
  st_stream4(pg + rope_off(off) + lane * 4, rope);
}

__global__ void __launch_bounds__(kFloorWarps * 32, 5)
copy_floor_kernel(rkv_pool_view pool, int layer0, uint32_t n_tokens, uint32_t n_rows,
                  const uint16_t* __restrict__ rows, const int32_t* __restrict__ slots) {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const int lane = threadIdx.x & 31;
  const uint32_t stride = gridDim.x * kFloorWarps;
  const uint32_t r0 = blockIdx.x * kFloorWarps + (threadIdx.x >> 5);
  const uint8_t* rows8 = reinterpret_cast<const uint8_t*>(rows);
  uint32_t lat[kFloorRows][8];
  uint32_t rope[kFloorRows];
  int32_t slot[kFloorRows];
#pragma unroll
  for (int i = 0; i < kFloorRows; ++i) {
    rope[i] = 0;
    slot[i] = -1;
    if (r0 + i * stride < n_rows) floor_load(rows8, slots, r0 + i * stride, n_tokens, lane, lat[i], rope[i], slot[i]);
  }
  asm volatile("griddepcontrol.wait;" ::: "memory");
  for (uint32_t r = r0; r < n_rows; r += kFloorRows * stride) {
#pragma unroll
    for (int i = 0; i < kFloorRows; ++i) {
      const uint32_t ri = r + i * stride;
      if (ri < n_rows) {
        floor_store(pool, layer0 + (int)(ri / n_tokens), slot[i], lat[i], rope[i], lane);
        const uint32_t rn = ri + kFloorRows * stride;
        if (rn < n_rows) floor_load(rows8, slots, rn, n_tokens, lane, lat[i], rope[i], slot[i]);
      }
    }
  }
}

static std::atomic<int> g_resident_floor[kMaxDevicesCached];

}  // namespace rkv

extern "C" rkv_status rkv_copy_floor_bf16(const rkv_pool_view* pool, int32_t layer0, int32_t n_layers_in,
                                          const uint16_t* rows, int64_t n_tokens, const int32_t* slot_mapping,
                                          rkv_stream_t stream) {
  using namespace rkv;
  const char* what = "rkv_copy_floor_bf16";
  rkv_status st = check_pool(pool, what);
  if (st != RKV_OK) return st;
  if (layer0 < 0 || n_layers_in < 0 || (int64_t)layer0 + n_layers_in > pool->n_layers)
    return fail_layer(layer0 < 0 || n_layers_in < 0 ? layer0 : (int64_t)layer0 + n_layers_in - 1, pool->n_layers,
                      "%s: layers [%d, %d) outside pool of %d layers", what, layer0, layer0 + n_layers_in,
                      pool->n_layers);
  if (n_tokens < 0) return fail_shape("n_tokens", 0, n_tokens, "%s: n_tokens < 0", what);
  const int64_t n_rows = n_tokens * (int64_t)n_layers_in;
  if (n_rows == 0) {
    clear_error();
    return RKV_OK;
  }
  if (n_rows > (int64_t)INT32_MAX) return fail_shape("rows", INT32_MAX, n_rows, "%s: too many rows in one call", what);
  if (!rows || !aligned(rows, 32) || !slot_mapping || !aligned(slot_mapping, 4))
    return fail(RKV_ERR_INVALID_ARGUMENT, "%s: rows (32-byte aligned) and slot_mapping are required", what);
  int dev = 0;
  cudaGetDevice(&dev);
  int resident = (dev >= 0 && dev < kMaxDevicesCached) ? g_resident_floor[dev].load(std::memory_order_relaxed) : 0;
  if (resident == 0) {
    int sms = 0, per_sm = 0;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, copy_floor_kernel, kFloorWarps * 32, 0);
    resident = (sms > 0 && per_sm > 0) ? sms * per_sm : 148 * 4;
    if (dev >= 0 && dev < kMaxDevicesCached) g_resident_floor[dev].store(resident, std::memory_order_relaxed);
  }
  const int64_t need = (n_rows + kFloorWarps - 1) / kFloorWarps;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(need < resident ? need : resident));
  cfg.blockDim = dim3(kFloorWarps * 32);
  cfg.stream = (cudaStream_t)stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  rkv_pool_view view = *pool;
  cudaError_t e = cudaLaunchKernelEx(&cfg, copy_floor_kernel, view, (int)layer0, (uint32_t)n_tokens, (uint32_t)n_rows,
                                     rows, slot_mapping);
  if (e != cudaSuccess) return fail(RKV_ERR_CUDA, "%s: launch failed: %s", what, cudaGetErrorString(e));
  return check_launch(what);
}
