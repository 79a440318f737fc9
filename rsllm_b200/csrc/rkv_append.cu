// rkv_append.cu -- quantize-on-append of bf16 KV rows into the paged pool.
//
// A persistent grid (at most one wave of 256-thread CTAs) in which each warp
// moves one row (576 bf16 = 1152 B in, 672 B out) at a time and prefetches
// its next row before quantising the current one.  Lane l loads 32 B of
// latent (lanes 16l..16l+15, inside 64-lane block l/4) with one 256-bit load;
// lanes 0..7 also 16 B of RoPE.  The block amax is an integer max over the
// bf16 magnitude bits (NaN and inf show up as >= 0x7f80) reduced over the 4
// lanes of the block; the power-of-two scale exponent comes from the amax
// bits; the lanes are scaled with packed f32x2 multiplies and converted two at
// a time to E4M3 with saturating RNE.  Codes go out as one 512 B run per row,
// the 8 block scales as one 32 B sector, the RoPE part as 128 B.
//
// Semantics: crates/rsllm-backend-cpu/src/ops/dsv4_quant.rs:316-362 applied
// per row (see rkv_common.cuh), row placement of crates/rsllm-kvcache/src/
// dsv4/swa.rs:73-94 generalised to a slot mapping.
#include <atomic>

#include "rkv_common.cuh"
#include "rkv_host.h"

namespace rkv {

static inline rkv_pool_view pool_copy(const rkv_pool_view& p) { return p; }

constexpr int kAppendWarps = 8;  // 256-thread CTAs
constexpr unsigned long long kNegZero2 = 0x8000000080000000ull;  // -0.0 in both halves, a kernel argument

// Quantise and store one row a warp holds: lane l has latent lanes
// 16l..16l+15 in lat (inside 64-lane block l/4), lanes 0..7 hold 16 B each of
// the RoPE part.  Every lane sees the same slot, so the branches are uniform.
__device__ __forceinline__ void append_row(const rkv_pool_view& pool, int layer, int32_t slot,
                                           const uint32_t (&lat)[8], const uint4& rope, uint32_t* status,
                                           int lane, unsigned long long nz2) {
  const unsigned FULL = 0xffffffffu;
  if (slot < 0) return;  // padding token
  const int64_t page = slot >> 6;
  const int off = slot & 63;
  uint32_t m = absmax_bits16(lat);
  m = max(m, __shfl_xor_sync(FULL, m, 1));
  m = max(m, __shfl_xor_sync(FULL, m, 2));
  if (page >= pool.n_pages) {
    if (lane == 0) set_status(status, RKV_ERR_INDEX_OUT_OF_RANGE);
    return;
  }
  if (__any_sync(FULL, m >= 0x7f80u)) {  // a non-finite latent lane rejects the row before any write
    if (lane == 0) set_status(status, RKV_ERR_NON_FINITE_INPUT);
    return;
  }
  const int e = scale_exponent_bf16bits(m);
  const uint4 codes = quant16(lat, __uint_as_float((uint32_t)(127 - e) << 23), nz2);
  uint8_t* pg = page_base(pool, layer, page);
  st_stream16(pg + codes_off(off) + lane * 16, codes);
  // lane j < 8 stores the scale of block j, held by lane 4j, and 16 B of RoPE
  const float sc = __shfl_sync(FULL, __uint_as_float((uint32_t)(e + 127) << 23), (lane & 7) * 4);
  if (lane < 8) {
    reinterpret_cast<float*>(pg + scales_off(off))[lane] = sc;
    st_stream16(pg + rope_off(off) + lane * 16, rope);
  }
}

// Persistent grid (at most one wave): warp w handles rows w, w + W, ...
// (W = warps in the grid) and issues the loads of its next row -- 32 B of
// latent per lane (one 256-bit load), 16 B of RoPE on lanes 0..7 and the
// slot index -- before it quantises the current one, so two rows per warp
// are in flight.  Launched with Programmatic Dependent Launch: the CTAs of
// the next launch become resident while this one drains and wait
// (griddepcontrol.wait) for it before touching memory.
__global__ void __launch_bounds__(kAppendWarps * 32)
append_quant_kernel(rkv_pool_view pool, int layer0, uint32_t n_tokens, uint32_t n_rows,
                    const uint16_t* __restrict__ rows, const int32_t* __restrict__ slots,
                    uint32_t* __restrict__ status, unsigned long long nz2) {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int lane = threadIdx.x & 31;
  const uint32_t stride = gridDim.x * kAppendWarps;
  uint32_t r = blockIdx.x * kAppendWarps + (threadIdx.x >> 5);
  if (r >= n_rows) return;
  const uint8_t* rows8 = reinterpret_cast<const uint8_t*>(rows);
  uint32_t lat[8], nlat[8];
  uint4 rope = make_uint4(0, 0, 0, 0), nrope = rope;
  int32_t slot, nslot = -1;
  ld_stream32(rows8 + (size_t)r * (kRowDim * 2) + lane * 32, lat);
  if (lane < 8) rope = ld_stream16(rows8 + (size_t)r * (kRowDim * 2) + 1024 + lane * 16);
  slot = __ldg(slots + r % n_tokens);
  for (; r < n_rows; r += stride) {
    const uint32_t rn = r + stride;
    if (rn < n_rows) {
      ld_stream32(rows8 + (size_t)rn * (kRowDim * 2) + lane * 32, nlat);
      if (lane < 8) nrope = ld_stream16(rows8 + (size_t)rn * (kRowDim * 2) + 1024 + lane * 16);
      nslot = __ldg(slots + rn % n_tokens);
    }
    append_row(pool, layer0 + (int)(r / n_tokens), slot, lat, rope, status, lane, nz2);
#pragma unroll
    for (int j = 0; j < 8; ++j) lat[j] = nlat[j];
    rope = nrope;
    slot = nslot;
  }
}

// The same append for callers whose inputs are ready before the previous
// kernel on the stream ends (RKV_APPEND_INPUTS_READY): each warp loads its
// first two rows -- 32 B of latent and 4 B of RoPE per lane, and the slot --
// BEFORE griddepcontrol.wait, so those reads overlap the previous kernel's
// drain; every store stays after the wait.  Rows are taken two at a time
// (r, r + W, then r + 2W, r + 3W, ...), each buffer refilled right after its
// row is stored.  46 registers: five 256-thread CTAs per SM.
constexpr int kEarlyRows = 2;

__device__ __forceinline__ void append_row_rope4(const rkv_pool_view& pool, int layer, int32_t slot,
                                                 const uint32_t (&lat)[8], uint32_t rope, uint32_t* status,
                                                 int lane, unsigned long long nz2) {
  const unsigned FULL = 0xffffffffu;
  if (slot < 0) return;  // padding token
  const int64_t page = slot >> 6;
  const int off = slot & 63;
  uint32_t m = absmax_bits16(lat);
  m = max(m, __shfl_xor_sync(FULL, m, 1));
  m = max(m, __shfl_xor_sync(FULL, m, 2));
  if (page >= pool.n_pages) {
    if (lane == 0) set_status(status, RKV_ERR_INDEX_OUT_OF_RANGE);
    return;
  }
  if (__any_sync(FULL, m >= 0x7f80u)) {  // a non-finite latent lane rejects the row before any write
    if (lane == 0) set_status(status, RKV_ERR_NON_FINITE_INPUT);
    return;
  }
  const int e = scale_exponent_bf16bits(m);
  const uint4 codes = quant16(lat, __uint_as_float((uint32_t)(127 - e) << 23), nz2);
  uint8_t* pg = page_base(pool, layer, page);
  st_stream16(pg + codes_off(off) + lane * 16, codes);
  const float sc = __shfl_sync(FULL, __uint_as_float((uint32_t)(e + 127) << 23), (lane & 7) * 4);
  if (lane < 8) reinterpret_cast<float*>(pg + scales_off(off))[lane] = sc;
  st_stream4(pg + rope_off(off) + lane * 4, rope);
}

__device__ __forceinline__ void load_row_rope4(const uint8_t* rows8, const int32_t* slots, uint32_t r,
                                               uint32_t n_tokens, int lane, uint32_t (&lat)[8], uint32_t& rope,
                                               int32_t& slot) {
  const uint8_t* row = rows8 + (size_t)r * (kRowDim * 2);
  ld_stream32(row + lane * 32, lat);
  rope = ld_stream4(row + 1024 + lane * 4);
  slot = __ldg(slots + r % n_tokens);
}

__global__ void __launch_bounds__(kAppendWarps * 32, 5)
append_quant_early_kernel(rkv_pool_view pool, int layer0, uint32_t n_tokens, uint32_t n_rows,
                          const uint16_t* __restrict__ rows, const int32_t* __restrict__ slots,
                          uint32_t* __restrict__ status, unsigned long long nz2) {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const int lane = threadIdx.x & 31;
  const uint32_t stride = gridDim.x * kAppendWarps;
  const uint32_t r0 = blockIdx.x * kAppendWarps + (threadIdx.x >> 5);
  const uint8_t* rows8 = reinterpret_cast<const uint8_t*>(rows);
  uint32_t lat[kEarlyRows][8];
  uint32_t rope[kEarlyRows];
  int32_t slot[kEarlyRows];
#pragma unroll
  for (int i = 0; i < kEarlyRows; ++i) {
    rope[i] = 0;
    slot[i] = -1;
    if (r0 + i * stride < n_rows) load_row_rope4(rows8, slots, r0 + i * stride, n_tokens, lane, lat[i], rope[i], slot[i]);
  }
  asm volatile("griddepcontrol.wait;" ::: "memory");
  for (uint32_t r = r0; r < n_rows; r += kEarlyRows * stride) {
#pragma unroll
    for (int i = 0; i < kEarlyRows; ++i) {
      const uint32_t ri = r + i * stride;
      if (ri < n_rows) {
        append_row_rope4(pool, layer0 + (int)(ri / n_tokens), slot[i], lat[i], rope[i], status, lane, nz2);
        const uint32_t rn = ri + kEarlyRows * stride;
        if (rn < n_rows) load_row_rope4(rows8, slots, rn, n_tokens, lane, lat[i], rope[i], slot[i]);
      }
    }
  }
}

// Exhaustive-check helper: the append kernels' lane conversion (the product
// with the inverse scale, here 1.0, as fma.rn.f32x2 with the run-time -0.0
// pair, -0.0 folded to +0.0 by add.rn.f32x2 of +0.0, saturating RNE) applied
// to raw f32 values that are already divided by their block scale.
__global__ void e4m3_code_range_kernel(uint32_t first, int64_t n, uint8_t* __restrict__ out,
                                       unsigned long long nz2) {
  const unsigned long long one2 = 0x3f8000003f800000ull;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const unsigned long long x = first + (uint32_t)i;  // lane 0 = x, lane 1 = +0.0
    const unsigned long long t = add_f32x2(fma_f32x2(x, one2, nz2), 0ull);
    out[i] = (uint8_t)(cvt_e4m3x2(__uint_as_float((uint32_t)t), 0.0f) & 0xffu);
  }
}

}  // namespace rkv

namespace rkv {

// CTAs of `kernel` one wave holds on the current device (cached per device).
template <typename Kernel>
static int resident_ctas(Kernel kernel, std::atomic<int> (&cache)[kMaxDevicesCached]) {
  int dev = 0;
  cudaGetDevice(&dev);
  int resident = (dev >= 0 && dev < kMaxDevicesCached) ? cache[dev].load(std::memory_order_relaxed) : 0;
  if (resident == 0) {
    int sms = 0, per_sm = 0;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, kAppendWarps * 32, 0);
    resident = (sms > 0 && per_sm > 0) ? sms * per_sm : 148 * 4;
    if (dev >= 0 && dev < kMaxDevicesCached) cache[dev].store(resident, std::memory_order_relaxed);
  }
  return resident;
}

static std::atomic<int> g_resident_append[kMaxDevicesCached];
static std::atomic<int> g_resident_append_early[kMaxDevicesCached];

static rkv_status append_bf16(const rkv_pool_view* pool, int32_t layer0, int32_t n_layers_in, const uint16_t* rows,
                              int64_t n_tokens, const int32_t* slot_mapping, uint32_t flags, uint32_t* d_status,
                              rkv_stream_t stream, const char* what) {
  rkv_status st = check_pool(pool, what);
  if (st != RKV_OK) return st;
  if (flags & ~RKV_APPEND_INPUTS_READY) return fail(RKV_ERR_INVALID_ARGUMENT, "%s: unknown flags 0x%x", what, flags);
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
  if (n_rows > (int64_t)INT32_MAX)
    return fail_shape("rows", INT32_MAX, n_rows, "%s: too many rows in one call", what);
  if (!rows || !aligned(rows, 32) || !slot_mapping || !aligned(slot_mapping, 4))
    return fail(RKV_ERR_INVALID_ARGUMENT, "%s: rows (32-byte aligned) and slot_mapping are required", what);
  const bool early = (flags & RKV_APPEND_INPUTS_READY) != 0;
  const int resident = early ? resident_ctas(append_quant_early_kernel, g_resident_append_early)
                             : resident_ctas(append_quant_kernel, g_resident_append);
  const int64_t need = (n_rows + kAppendWarps - 1) / kAppendWarps;
  const unsigned grid = (unsigned)(need < resident ? need : resident);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kAppendWarps * 32);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = (cudaStream_t)stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = early ? cudaLaunchKernelEx(&cfg, append_quant_early_kernel, pool_copy(*pool), (int)layer0,
                                             (uint32_t)n_tokens, (uint32_t)n_rows, rows, slot_mapping, d_status,
                                             kNegZero2)
                        : cudaLaunchKernelEx(&cfg, append_quant_kernel, pool_copy(*pool), (int)layer0,
                                             (uint32_t)n_tokens, (uint32_t)n_rows, rows, slot_mapping, d_status,
                                             kNegZero2);
  if (e != cudaSuccess) return fail(RKV_ERR_CUDA, "%s: launch failed: %s", what, cudaGetErrorString(e));
  return check_launch(what);
}

}  // namespace rkv

extern "C" rkv_status rkv_append_quant_bf16(const rkv_pool_view* pool, int32_t layer0, int32_t n_layers_in,
                                            const uint16_t* rows, int64_t n_tokens, const int32_t* slot_mapping,
                                            uint32_t* d_status, rkv_stream_t stream) {
  return rkv::append_bf16(pool, layer0, n_layers_in, rows, n_tokens, slot_mapping, 0u, d_status, stream,
                          "rkv_append_quant_bf16");
}

extern "C" rkv_status rkv_append_quant_bf16_ex(const rkv_pool_view* pool, int32_t layer0, int32_t n_layers_in,
                                               const uint16_t* rows, int64_t n_tokens, const int32_t* slot_mapping,
                                               uint32_t flags, uint32_t* d_status, rkv_stream_t stream) {
  return rkv::append_bf16(pool, layer0, n_layers_in, rows, n_tokens, slot_mapping, flags, d_status, stream,
                          "rkv_append_quant_bf16_ex");
}

extern "C" rkv_status rkv_e4m3fn_code_range(uint32_t first_bits, int64_t n, uint8_t* out, rkv_stream_t stream) {
  using namespace rkv;
  if (n < 0 || (n > 0 && !out)) return fail(RKV_ERR_INVALID_ARGUMENT, "rkv_e4m3fn_code_range: bad output");
  if (n > 0x100000000LL - (int64_t)first_bits) return fail(RKV_ERR_SHAPE_MISMATCH, "rkv_e4m3fn_code_range: range wraps");
  if (n == 0) return RKV_OK;
  e4m3_code_range_kernel<<<148 * 8, 256, 0, (cudaStream_t)stream>>>(first_bits, n, out, kNegZero2);
  return check_launch("rkv_e4m3fn_code_range");
}
