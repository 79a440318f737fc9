// rkv_common.cuh -- layout constants and the device-side FP8 E4M3FN codec
// shared by every kernel of the KV-cache path.
//
// Codec semantics follow rsLLM's CPU round trip
// (crates/rsllm-backend-cpu/src/ops/dsv4_quant.rs:316-362):
//   per 64-lane block: amax = max|v| (floored at 1e-4), e = ceil(log2(amax/448)),
//   scale = 2^e, code = sign(v/scale < 0) | RNE-saturating E4M3 index of
//   |clamp(v/scale, +-448)|; the stored scale is the f32 2^e.  Dequant is
//   (sign * e4m3_value(code)) * 2^e, which is exact in f32 and in bf16.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/rsllm_kv_cuda.h"

namespace rkv {

constexpr int kPageTokens = RKV_PAGE_TOKENS;   // 64 token rows per page
constexpr int kLatent = RKV_LATENT_DIM;        // 512 FP8 lanes per row
constexpr int kRope = RKV_ROPE_DIM;            // 64 bf16 lanes per row
constexpr int kRowDim = RKV_ROW_DIM;           // 576 bf16 lanes per input row
constexpr int kBlock = RKV_BLOCK;              // 64 lanes share one scale
constexpr int kBlocks = kLatent / kBlock;      // 8 scales per row
constexpr int kCodesBytes = kPageTokens * kLatent;            // 32768
constexpr int kScalesBytes = kPageTokens * kBlocks * 4;       // 2048
constexpr int kRopeBytes = kPageTokens * kRope * 2;           // 8192
constexpr int kPageBytes = kCodesBytes + kScalesBytes + kRopeBytes;  // 43008
static_assert(kPageBytes == RKV_PAGE_BYTES, "page layout");

// Byte offsets of token row `off` inside a page (structure of arrays).
__host__ __device__ __forceinline__ int64_t codes_off(int off) { return (int64_t)off * kLatent; }
__host__ __device__ __forceinline__ int64_t scales_off(int off) { return kCodesBytes + (int64_t)off * kBlocks * 4; }
__host__ __device__ __forceinline__ int64_t rope_off(int off) { return kCodesBytes + kScalesBytes + (int64_t)off * kRope * 2; }

__device__ __forceinline__ uint8_t* page_base(const rkv_pool_view& p, int layer, int64_t page) {
  return static_cast<uint8_t*>(p.base) + ((int64_t)layer * p.n_pages + page) * (int64_t)kPageBytes;
}

__device__ __forceinline__ void set_status(uint32_t* st, int code) {
  if (st) atomicOr(st, 1u << code);
}

// ---- encode ---------------------------------------------------------------

// Two f32 -> two E4M3 bytes (lo in bits 0..7), round to nearest even with
// saturation to +-448.  PTX puts the conversion of the first source operand
// in the upper byte.
__device__ __forceinline__ uint32_t cvt_e4m3x2(float lo, float hi) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
  return r;
}

// Block scale exponent e = ceil(log2(y)), y = RN(max(amax,1e-4) / 448), for a
// block amax that is a bf16 value.  y is a positive normal f32, so ceil(log2)
// is its unbiased exponent plus one unless y is an exact power of two.  For
// bf16 amax this equals the reference's ceil(log2f(y)): y = (m/7) * 2^j with
// an 8-bit m, which is either an exact power of two or at least 1/224 away
// from one (verified over every bf16 value by the GPU parity tests).
__device__ __forceinline__ int scale_exponent_bf16amax(float amax) {
  amax = fmaxf(amax, 1.0e-4f);
  float y = __fdiv_rn(amax, 448.0f);
  uint32_t b = __float_as_uint(y);
  int e = (int)((b >> 23) & 0xffu) - 127;
  return e + ((b & 0x7fffffu) != 0u ? 1 : 0);
}

// One quantised lane pair: t = v * 2^-e (equal to v / 2^e, both correctly
// rounded), clamp to +-448, fold -0.0 into +0.0 (the reference's sign is
// `x < 0`), convert.
__device__ __forceinline__ float quant_lane(float v, float inv_scale) {
  float t = __fmul_rn(v, inv_scale);
  t = fminf(fmaxf(t, -448.0f), 448.0f);
  return __fadd_rn(t, 0.0f);
}

// bf16 pair (packed u32, lo lane in bits 0..15) -> f32 lanes.
__device__ __forceinline__ float bf16lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }

// 8 bf16 lanes (one uint4) -> 8 codes (uint2), with the block's inverse scale.
__device__ __forceinline__ uint2 quant8(const uint4& v, float inv) {
  uint32_t c0 = cvt_e4m3x2(quant_lane(bf16lo(v.x), inv), quant_lane(bf16hi(v.x), inv));
  uint32_t c1 = cvt_e4m3x2(quant_lane(bf16lo(v.y), inv), quant_lane(bf16hi(v.y), inv));
  uint32_t c2 = cvt_e4m3x2(quant_lane(bf16lo(v.z), inv), quant_lane(bf16hi(v.z), inv));
  uint32_t c3 = cvt_e4m3x2(quant_lane(bf16lo(v.w), inv), quant_lane(bf16hi(v.w), inv));
  return make_uint2(c0 | (c1 << 16), c2 | (c3 << 16));
}

// Largest |bf16| magnitude bits in a uint4 of 8 lanes (0x7f80 and above means
// inf or NaN).
__device__ __forceinline__ uint32_t absmax_bits8(const uint4& v) {
  uint32_t m = __vmaxu2(__vmaxu2(v.x & 0x7fff7fffu, v.y & 0x7fff7fffu),
                        __vmaxu2(v.z & 0x7fff7fffu, v.w & 0x7fff7fffu));
  return max(m & 0xffffu, m >> 16);
}

// ---- decode ---------------------------------------------------------------

// Two E4M3 bytes -> f16x2 (exact: every E4M3 value is an f16 normal or zero).
__device__ __forceinline__ uint32_t cvt_f16x2_from_e4m3x2(uint32_t two_codes) {
  uint32_t r;
  asm("{\n\t.reg .b16 c;\n\tcvt.u16.u32 c, %1;\n\tcvt.rn.f16x2.e4m3x2 %0, c;\n\t}" : "=r"(r) : "r"(two_codes));
  return r;
}

__device__ __forceinline__ uint32_t mul_bf16x2(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}

// Per-block multiplier(s) for decode.  Re-reading an f16 E4M3 value's bits as
// bf16 (exponent field moved down by three bits) gives value * 2^-112, so the
// bf16 product with 2^(112+e) is value * 2^e -- exact, or +-inf on overflow,
// exactly as the reference's f32 product rounded to bf16.  2^(112+e) is a bf16
// normal for e <= 15; larger exponents split into 2^112 * 2^e.
struct DecodeScale {
  uint32_t m1, m2;
  bool two;
};
__device__ __forceinline__ DecodeScale decode_scale(float scale) {
  int eb = (int)((__float_as_uint(scale) >> 23) & 0xffu);  // e + 127
  DecodeScale d;
  if (eb <= 142) {
    uint32_t h = (uint32_t)(eb + 112) << 7;
    d.m1 = h | (h << 16);
    d.m2 = 0u;
    d.two = false;
  } else {
    uint32_t h1 = 239u << 7, h2 = (uint32_t)eb << 7;
    d.m1 = h1 | (h1 << 16);
    d.m2 = h2 | (h2 << 16);
    d.two = true;
  }
  return d;
}

__device__ __forceinline__ uint32_t dequant2(uint32_t two_codes, const DecodeScale& d) {
  uint32_t h = cvt_f16x2_from_e4m3x2(two_codes);
  uint32_t y = (h & 0x80008000u) | ((h >> 3) & 0x0fff0fffu);
  y = mul_bf16x2(y, d.m1);
  if (d.two) y = mul_bf16x2(y, d.m2);
  return y;
}

// 16 codes (uint4) -> 16 bf16 lanes (two uint4).
__device__ __forceinline__ void dequant16(const uint4& c, const DecodeScale& d, uint4& o0, uint4& o1) {
  o0.x = dequant2(c.x & 0xffffu, d);
  o0.y = dequant2(c.x >> 16, d);
  o0.z = dequant2(c.y & 0xffffu, d);
  o0.w = dequant2(c.y >> 16, d);
  o1.x = dequant2(c.z & 0xffffu, d);
  o1.y = dequant2(c.z >> 16, d);
  o1.z = dequant2(c.w & 0xffffu, d);
  o1.w = dequant2(c.w >> 16, d);
}

// ---- cache-policy loads and stores ----------------------------------------
// Streaming data is touched once: keep it out of L1 so the page tables and
// indices stay cached there.
__device__ __forceinline__ uint4 ld_stream16(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
  return v;
}
__device__ __forceinline__ void st_stream16(void* p, const uint4& v) {
  asm volatile("st.global.L1::no_allocate.v4.u32 [%0], {%1,%2,%3,%4};"
               :: "l"(p), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w) : "memory");
}
__device__ __forceinline__ void st_stream8(void* p, const uint2& v) {
  asm volatile("st.global.L1::no_allocate.v2.u32 [%0], {%1,%2};" :: "l"(p), "r"(v.x), "r"(v.y) : "memory");
}

}  // namespace rkv
