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

// Block scale exponent e = ceil(log2f(max(amax, 1e-4) / 448)) for a block
// amax that is a bf16 value, from its bits.  With amax = (m/128) * 2^E
// (m the 8-bit significand, 128..255): amax/448 = (m/7) * 2^(E-13) and
// m/7 lies in (16, 36.5), so e = E - 8 + (m > 224): the quotient is a power
// of two only at m = 224 and otherwise at least 1/224 away from one, so the
// reference's f32 division and glibc log2f land on the same integer
// (checked on the GPU for every finite bf16 amax against the CPU oracle).
// Every amax below 1e-4 (the reference's floor) gives e = -22.
__device__ __forceinline__ int scale_exponent_bf16bits(uint32_t amax_bits) {
  if (amax_bits < 0x38D2u) return -22;  // bf16 0x38D2 = 1.0014e-4 is the first value >= 1e-4f
  const int E = (int)(amax_bits >> 7) - 127;
  return E - 8 + ((amax_bits & 0x7fu) > 96u ? 1 : 0);
}

// Packed f32x2 arithmetic (sm_100): lo lane in bits 0..31.
__device__ __forceinline__ unsigned long long add_f32x2(unsigned long long a, unsigned long long b) {
  unsigned long long r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}

// One bf16 pair -> two E4M3 codes (bits 0..15): t = v * 2^-e exactly as the
// reference's v / 2^e (both correctly rounded), -0.0 folded into +0.0 (the
// reference's sign is `x < 0`), then RNE with saturation.  For bf16 inputs
// |t| <= 448 always holds, so the reference's clamp is the identity.  Two
// packed instructions for the arithmetic: the product as
// fma.rn.f32x2(v, inv, nz) with nz = -0.0 in both
// halves, passed in at run time -- exactly the rounded product, sign included
// -- then add.rn.f32x2 of +0.0, which turns a zero of either sign into +0.0
// and leaves every other value as it is.  An add cannot be fused into an fma,
// so the product is rounded before the add (a multiply followed by that add
// can be contracted into one fused multiply-add, which keeps the sign of a
// product that underflows to zero; so can an fma whose -0.0 addend the
// compiler sees).
__device__ __forceinline__ unsigned long long fma_f32x2(unsigned long long a, unsigned long long b,
                                                        unsigned long long c) {
  unsigned long long r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}
__device__ __forceinline__ uint32_t quant_pair(uint32_t w, unsigned long long inv2, unsigned long long nz2) {
  const unsigned long long v = ((unsigned long long)(w & 0xffff0000u) << 32) | (unsigned long long)(w << 16);
  const unsigned long long t = add_f32x2(fma_f32x2(v, inv2, nz2), 0ull);
  return cvt_e4m3x2(__uint_as_float((uint32_t)t), __uint_as_float((uint32_t)(t >> 32)));
}

// ---- decode ---------------------------------------------------------------

// Two E4M3 bytes -> f16x2 (exact: every E4M3 value is an f16 normal or zero).
__device__ __forceinline__ uint32_t cvt_f16x2_from_e4m3x2(uint32_t two_codes) {
  uint32_t r;
  asm("{\n\t.reg .b16 c;\n\tcvt.u16.u32 c, %1;\n\tcvt.rn.f16x2.e4m3x2 %0, c;\n\t}" : "=r"(r) : "r"(two_codes));
  return r;
}

// Four E4M3 bytes -> two f16x2 words (codes 0-1 in lo, 2-3 in hi): the word
// is split into its two 16-bit halves instead of shifting the upper pair down.
__device__ __forceinline__ void cvt_f16x2x2_from_e4m3x4(uint32_t four_codes, uint32_t& lo, uint32_t& hi) {
  asm("{\n\t.reg .b16 a, b;\n\tmov.b32 {a, b}, %2;\n\tcvt.rn.f16x2.e4m3x2 %0, a;\n\tcvt.rn.f16x2.e4m3x2 %1, b;\n\t}"
      : "=r"(lo), "=r"(hi)
      : "r"(four_codes));
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

// Two f16x2 words of E4M3 values -> bf16x2 times the block scale (dequant2's
// second half).
__device__ __forceinline__ uint32_t rebias_scale2(uint32_t h, const DecodeScale& d) {
  uint32_t y = (h & 0x80008000u) | ((h >> 3) & 0x0fff0fffu);
  y = mul_bf16x2(y, d.m1);
  if (d.two) y = mul_bf16x2(y, d.m2);
  return y;
}

// 16 codes (uint4) -> 16 bf16 lanes (two uint4).
__device__ __forceinline__ void dequant16(const uint4& c, const DecodeScale& d, uint4& o0, uint4& o1) {
  uint32_t h[8];
  cvt_f16x2x2_from_e4m3x4(c.x, h[0], h[1]);
  cvt_f16x2x2_from_e4m3x4(c.y, h[2], h[3]);
  cvt_f16x2x2_from_e4m3x4(c.z, h[4], h[5]);
  cvt_f16x2x2_from_e4m3x4(c.w, h[6], h[7]);
  o0 = make_uint4(rebias_scale2(h[0], d), rebias_scale2(h[1], d), rebias_scale2(h[2], d), rebias_scale2(h[3], d));
  o1 = make_uint4(rebias_scale2(h[4], d), rebias_scale2(h[5], d), rebias_scale2(h[6], d), rebias_scale2(h[7], d));
}

// 16 bf16 lanes (8 words) -> 16 codes (uint4); nz2: -0.0 in both halves, a
// run-time value (see quant_pair).
__device__ __forceinline__ uint4 quant16(const uint32_t (&w)[8], float inv, unsigned long long nz2) {
  const unsigned long long inv2 = ((unsigned long long)__float_as_uint(inv) << 32) | __float_as_uint(inv);
  uint32_t c[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) c[i] = quant_pair(w[i], inv2, nz2);
  return make_uint4(c[0] | (c[1] << 16), c[2] | (c[3] << 16), c[4] | (c[5] << 16), c[6] | (c[7] << 16));
}

// Largest |bf16| magnitude bits over 16 lanes (>= 0x7f80: inf or NaN present).
__device__ __forceinline__ uint32_t absmax_bits16(const uint32_t (&w)[8]) {
  uint32_t m = 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) m = __vmaxu2(m, w[i] & 0x7fff7fffu);
  return max(m & 0xffffu, m >> 16);
}

// ---- cache-policy loads and stores ----------------------------------------
// 256-bit accesses (sm_100): one instruction moves 32 B per lane, a whole
// 1 KB latent row per warp.
__device__ __forceinline__ void ld_stream32(const void* p, uint32_t (&v)[8]) {
  asm volatile("ld.global.nc.L1::no_allocate.L2::evict_first.v8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7])
               : "l"(p));
}
__device__ __forceinline__ void st_stream32(void* p, const uint4& a, const uint4& b) {
  asm volatile("st.global.L1::no_allocate.v8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};"
               :: "l"(p), "r"(a.x), "r"(a.y), "r"(a.z), "r"(a.w), "r"(b.x), "r"(b.y), "r"(b.z), "r"(b.w)
               : "memory");
}
// 256-bit load through L1 (data several lanes of a warp share, e.g. a row's
// scales).
__device__ __forceinline__ void ld_cached32(const void* p, uint32_t (&v)[8]) {
  asm volatile("ld.global.nc.v8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7])
               : "l"(p));
}
// Streaming data is touched once: keep it out of L1 so the page tables and
// indices stay cached there.
__device__ __forceinline__ uint4 ld_stream16(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
  return v;
}
__device__ __forceinline__ uint32_t ld_stream4(const void* p) {
  uint32_t v;
  asm volatile("ld.global.nc.L1::no_allocate.u32 %0, [%1];" : "=r"(v) : "l"(p));
  return v;
}
__device__ __forceinline__ void st_stream4(void* p, uint32_t v) {
  asm volatile("st.global.L1::no_allocate.u32 [%0], %1;" :: "l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void st_stream16(void* p, const uint4& v) {
  asm volatile("st.global.L1::no_allocate.v4.u32 [%0], {%1,%2,%3,%4};"
               :: "l"(p), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w) : "memory");
}

}  // namespace rkv
