// rkv_f32row.cuh -- quantisation of one f32 row (rsLLM's own row type) into
// the pool's stored form, shared by the f32 append and the compressor emit.
//
// The block exponent is ceil(log2f(max(amax, 1e-4) / 448)) as the reference
// evaluates it (crates/rsllm-backend-cpu/src/ops/dsv4_quant.rs:346-355), via a
// per-binade threshold table built once per process from the host's log2f:
// for y = RN(amax / 448) with biased exponent b and mantissa m, the exponent
// is (b - 127) + (m >= table[b]).  RoPE lanes are stored rounded to bf16.
#pragma once
#include "rkv_common.cuh"

namespace rkv {

struct ThresholdTable {
  uint32_t m[256];  // by biased exponent of y: exponent + 1 iff mantissa >= m
};

// The host-built table (rkv_append_f32.cu).
const ThresholdTable& f32_threshold_table();

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

// Two f32 lanes -> two codes with quant_pair's arithmetic: the product as
// fma.rn.f32x2 with the run-time -0.0 pair nz2 (exactly the rounded product),
// then add.rn.f32x2 of +0.0 (a zero of either sign becomes +0.0).
__device__ __forceinline__ uint32_t quant_pair_f32(uint32_t lo, uint32_t hi, unsigned long long inv2,
                                                   unsigned long long nz2) {
  const unsigned long long v = ((unsigned long long)hi << 32) | lo;
  const unsigned long long t = add_f32x2(fma_f32x2(v, inv2, nz2), 0ull);
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
                                               const ThresholdTable& tab, uint32_t* status, int lane,
                                               unsigned long long nz2) {
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
  for (int i = 0; i < 4; ++i) c[i] = quant_pair_f32(x.a[2 * i], x.a[2 * i + 1], inv2, nz2);
#pragma unroll
  for (int i = 0; i < 4; ++i) c[4 + i] = quant_pair_f32(x.b[2 * i], x.b[2 * i + 1], inv2, nz2);
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

}  // namespace rkv
