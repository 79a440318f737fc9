// rkv_compress.cu -- the compressor's emission step on the GPU: per-dimension
// softmax aggregate of a window of token rows, RMSNorm, YaRN RoPE of the 64
// tail lanes, and FP8 quantize-on-append of the emitted row into the pool,
// bit-exact with rsLLM's CPU path.
//
// rsLLM (crates/rsllm-models/src/dsv4/compressor.rs:264-357) adds the APE bias
// to the score row, hands (kv, score) to CompressedKvPool::accumulate_wide
// (crates/rsllm-kvcache/src/dsv4/compressed.rs:310-417), which stores the row
// in its window state and, every ratio tokens, aggregates the window per
// dimension (:481-554); the emitted row is RMS-normalised with an f64 sum of
// squares, its 64 tail lanes are rotated (crates/rsllm-backend-cpu/src/ops/
// rope.rs:128-172 at position pos + 1 - ratio) and it is FP8-quantized
// (dsv4_quant.rs:316-362).  Here a batch of tokens is one launch: each warp
// takes one emitting token and reads the window's rows straight from this
// call's input or, for positions of earlier calls, from a per-state ring of
// the last coff * ratio rows; a second launch then writes the ring.
//
// Bit-exactness.  Every f32/f64 operation is rsLLM's, in its order, with
// explicit round-to-nearest intrinsics (no contraction).  rsLLM's exp is the
// host libm's expf, which is not correctly rounded: for about 1e-4 of inputs
// it returns the neighbour of the correctly rounded value.  The kernel
// evaluates exp in double precision (Tang's table-driven method: 2^(k/256)
// from a 256-entry table times a cubic in the reduced argument, |r| <= ln2/512,
// relative error about 2^-42), rounds to f32, and wherever the double lies
// within 2^-7 f32 ulp of a rounding midpoint (about 1% of inputs, the only
// place a libm within 0.51 ulp can round differently) looks x up in a table of
// the inputs where the host's expf differs from that rounding.  The host
// builds the table once per process by evaluating the identical double
// algorithm (same IEEE operations) over every f32 in [-150, 0]; it is correct
// by construction for inputs inside the band, and an exhaustive test checks
// that no input outside the band differs.  RoPE cos/sin come from a host table
// computed with the host's libm as rope.rs does.
#include <math.h>
#include <stdio.h>
#include <string.h>

#include <algorithm>
#include <mutex>
#include <thread>
#include <vector>

#include "rkv_common.cuh"
#include "rkv_f32row.cuh"
#include "rkv_host.h"

namespace rkv {

// ---- exp: double evaluation shared by host and device --------------------------

constexpr int kExpTableBits = 8;                       // 2^(j/256)
constexpr uint32_t kExpMaxKey = 0x43160000u;           // |x| bits of 150.0f
constexpr int kExpBucketShift = 14;
constexpr int kExpBuckets = (int)(kExpMaxKey >> kExpBucketShift) + 2;
constexpr int kExpMaxEntries = 1 << 18;
constexpr uint32_t kExpBand = 1u << 22;               // 2^-7 f32 ulp, in units of the 29 dropped bits

struct ExpConsts {
  double inv_step;  // 256 / ln 2
  double step_hi;   // ln 2 / 256, 21 significant bits (k * step_hi is exact)
  double step_lo;   // ln 2 / 256 - step_hi
  double c2, c3;    // 1/2, 1/6
};

__host__ __device__ __forceinline__ double d_mul(double a, double b) {
#ifdef __CUDA_ARCH__
  return __dmul_rn(a, b);
#else
  return a * b;
#endif
}
__host__ __device__ __forceinline__ double d_add(double a, double b) {
#ifdef __CUDA_ARCH__
  return __dadd_rn(a, b);
#else
  return a + b;
#endif
}
__host__ __device__ __forceinline__ double d_sub(double a, double b) {
#ifdef __CUDA_ARCH__
  return __dsub_rn(a, b);
#else
  return a - b;
#endif
}
__host__ __device__ __forceinline__ uint64_t d_bits(double d) {
#ifdef __CUDA_ARCH__
  return (uint64_t)__double_as_longlong(d);
#else
  uint64_t b;
  memcpy(&b, &d, 8);
  return b;
#endif
}
__host__ __device__ __forceinline__ double d_from_bits(uint64_t b) {
#ifdef __CUDA_ARCH__
  return __longlong_as_double((long long)b);
#else
  double d;
  memcpy(&d, &b, 8);
  return d;
#endif
}

// exp(x) in double for x in [-150, 0]; the same IEEE operations on both sides.
__host__ __device__ __forceinline__ double exp_core(float xf, const ExpConsts& K, const double* T) {
  const double x = (double)xf;
  const double shift = 6755399441055744.0;  // 1.5 * 2^52: adding it rounds to an integer
  const double k = d_sub(d_add(d_mul(x, K.inv_step), shift), shift);
  const double r = d_sub(d_sub(x, d_mul(k, K.step_hi)), d_mul(k, K.step_lo));
  double p = d_add(d_mul(K.c3, r), K.c2);
  p = d_add(d_mul(p, r), 1.0);
  p = d_add(d_mul(p, r), 1.0);
  const long long ki = (long long)k;
  const double y = d_mul(T[ki & ((1 << kExpTableBits) - 1)], p);
  const double scale = d_from_bits((uint64_t)((ki >> kExpTableBits) + 1023) << 52);
  return d_mul(y, scale);
}

// True where the rounding of d to f32 may differ from the host's expf.
__host__ __device__ __forceinline__ bool exp_in_band(double d) {
  if (d < 1.1754943508222875e-38) return true;  // f32 subnormal results: always looked up
  const int64_t low = (int64_t)(d_bits(d) & ((1ull << 29) - 1)) - (1ll << 28);
  return (low < 0 ? -low : low) <= (int64_t)kExpBand;
}

// ---- host table ------------------------------------------------------------------

struct ExpHost {
  ExpConsts K;
  double T[1 << kExpTableBits];
  std::vector<uint32_t> entries;  // |x| bits ascending; bit 31: host expf = rounded + 1 ulp (else - 1)
  std::vector<uint32_t> buckets;  // first entry of each key >> kExpBucketShift
  bool ok = false;
  char err[160] = {0};
};

static ExpHost g_exp;
static std::once_flag g_exp_once;

static float bits_to_float(uint32_t b) {
  float f;
  memcpy(&f, &b, 4);
  return f;
}
static uint32_t float_to_bits(float f) {
  uint32_t b;
  memcpy(&b, &f, 4);
  return b;
}

static void build_exp_host() {
  ExpHost& E = g_exp;
  const long double ln2 = 0.693147180559945309417232121458176568L;
  E.K.inv_step = (double)(256.0L / ln2);
  const double step = (double)(ln2 / 256.0L);
  E.K.step_hi = d_from_bits(d_bits(step) & ~((1ull << 32) - 1));
  E.K.step_lo = (double)(ln2 / 256.0L - (long double)E.K.step_hi);
  E.K.c2 = 0.5;
  E.K.c3 = 1.0 / 6.0;
  for (int j = 0; j < (1 << kExpTableBits); ++j) E.T[j] = (double)exp2l((long double)j / 256.0L);

  unsigned nt = std::thread::hardware_concurrency();
  nt = nt < 1 ? 1 : (nt > 64 ? 64 : nt);
  std::vector<std::vector<uint32_t>> part(nt);
  std::vector<int> bad(nt, 0);
  std::vector<std::thread> th;
  for (unsigned t = 0; t < nt; ++t)
    th.emplace_back([&, t] {
      const uint64_t n = kExpMaxKey;  // keys 1 .. kExpMaxKey
      const uint32_t a = 1 + (uint32_t)(n * t / nt), b = 1 + (uint32_t)(n * (t + 1) / nt);
      for (uint32_t key = a; key < b; ++key) {
        const float x = bits_to_float(key | 0x80000000u);
        const double d = exp_core(x, E.K, E.T);
        if (!exp_in_band(d)) continue;
        const uint32_t f = float_to_bits((float)d), g = float_to_bits(expf(x));
        if (f == g) continue;
        if (g != f + 1 && g + 1 != f) {
          bad[t] = 1;
          continue;
        }
        part[t].push_back(key | (g > f ? 0x80000000u : 0u));
      }
    });
  for (auto& x : th) x.join();
  size_t total = 0;
  for (unsigned t = 0; t < nt; ++t) {
    if (bad[t]) {
      snprintf(E.err, sizeof E.err, "host expf differs from the double evaluation by more than one ulp");
      return;
    }
    total += part[t].size();
  }
  if (total > (size_t)kExpMaxEntries) {
    snprintf(E.err, sizeof E.err, "expf correction table has %zu entries (capacity %d)", total, kExpMaxEntries);
    return;
  }
  E.entries.reserve(total);
  for (unsigned t = 0; t < nt; ++t) E.entries.insert(E.entries.end(), part[t].begin(), part[t].end());
  E.buckets.assign(kExpBuckets + 1, 0);
  size_t e = 0;
  for (int b = 0; b <= kExpBuckets; ++b) {
    while (e < E.entries.size() && ((E.entries[e] & 0x7fffffffu) >> kExpBucketShift) < (uint32_t)b) ++e;
    E.buckets[b] = (uint32_t)e;
  }
  E.ok = true;
}

static const ExpHost* exp_host() {
  std::call_once(g_exp_once, build_exp_host);
  return g_exp.ok ? &g_exp : nullptr;
}

// Host-side lookup: the value the kernel produces.
static float expf_table_host(float x, const ExpHost& E) {
  if (x != x) return x;
  if (!(x >= -150.0f)) return 0.0f;
  if (x > 0.0f) return (float)exp((double)x);  // outside the aggregate's domain
  const double d = exp_core(x, E.K, E.T);
  uint32_t f = float_to_bits((float)d);
  if (exp_in_band(d)) {
    const uint32_t key = float_to_bits(x) & 0x7fffffffu;
    const uint32_t b = key >> kExpBucketShift;
    for (uint32_t i = E.buckets[b]; i < E.buckets[b + 1]; ++i)
      if ((E.entries[i] & 0x7fffffffu) == key) {
        f = (E.entries[i] >> 31) ? f + 1 : f - 1;
        break;
      }
  }
  return bits_to_float(f);
}

// ---- device copies of the table ------------------------------------------------

static __device__ double g_exp_T[1 << kExpTableBits];
static __device__ uint32_t g_exp_buckets[kExpBuckets + 1];
static __device__ uint32_t g_exp_entries[kExpMaxEntries];

constexpr int kMaxDevices = 64;
static bool g_exp_uploaded[kMaxDevices];
static std::mutex g_exp_mu;

static rkv_status prepare_device(const char* what) {
  const ExpHost* E = exp_host();
  if (!E) return fail(RKV_ERR_INVALID_ARGUMENT, "%s: %s", what, g_exp.err);
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(RKV_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices) return fail(RKV_ERR_INVALID_ARGUMENT, "%s: device %d", what, dev);
  std::lock_guard<std::mutex> lock(g_exp_mu);
  if (g_exp_uploaded[dev]) return RKV_OK;
  e = cudaMemcpyToSymbol(g_exp_T, E->T, sizeof E->T);
  if (e == cudaSuccess) e = cudaMemcpyToSymbol(g_exp_buckets, E->buckets.data(), E->buckets.size() * 4);
  if (e == cudaSuccess && !E->entries.empty())
    e = cudaMemcpyToSymbol(g_exp_entries, E->entries.data(), E->entries.size() * 4);
  if (e != cudaSuccess) return fail(RKV_ERR_CUDA, "%s: uploading the expf table: %s", what, cudaGetErrorString(e));
  g_exp_uploaded[dev] = true;
  return RKV_OK;
}

// expf as the host's libm rounds it, for the x = score - max of the aggregate
// (x <= 0 or NaN).
__device__ __forceinline__ float expf_host_rounding(float x, const ExpConsts& K) {
  if (!(x >= -150.0f)) return x != x ? x : 0.0f;
  if (x > 0.0f) return __double2float_rn(exp((double)x));  // outside the aggregate's domain
  const double d = exp_core(x, K, g_exp_T);
  uint32_t f = __float_as_uint(__double2float_rn(d));
  if (exp_in_band(d)) {
    const uint32_t key = __float_as_uint(x) & 0x7fffffffu;
    const uint32_t b = key >> kExpBucketShift;
    const uint32_t e1 = g_exp_buckets[b + 1];
    for (uint32_t i = g_exp_buckets[b]; i < e1; ++i) {
      const uint32_t v = g_exp_entries[i];
      if ((v & 0x7fffffffu) == key) {
        f = (v >> 31) ? f + 1 : f - 1;
        break;
      }
    }
  }
  return __uint_as_float(f);
}

__global__ void expf_map_kernel(const float* __restrict__ x, float* __restrict__ out, int64_t n, ExpConsts K) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    out[i] = expf_host_rounding(x[i], K);
}

// ---- RoPE table (host) ------------------------------------------------------------

// cos/sin * mscale of the 32 pairs at position pos, rope.rs:128-172 with the
// compressed-layer parameters of compressor.rs:372-397 (n_rot 64, freq_base
// 160000, freq_scale 1/16, ext_factor 1, beta_fast 32, beta_slow 1,
// n_ctx_orig 65536).  Plain f32 operations in rsLLM's order.
static void rope_coeffs(uint32_t pos, float* out) {
  const float pi = 3.14159265358979323846f;
  const float freq_base = 160000.0f, freq_scale = 1.0f / 16.0f, ext_factor = 1.0f;
  const float beta_fast = 32.0f, beta_slow = 1.0f;
  const int n_rot = 64;
  const float attn_factor = 1.0f / (1.0f + 0.1f * logf(1.0f / freq_scale));
  const float theta_scale = powf(freq_base, -2.0f / (float)n_rot);
  auto corr_dim = [&](float beta) {
    return ((float)n_rot * logf((float)65536 / (beta * 2.0f * pi))) / (2.0f * logf(freq_base));
  };
  const float lo = fmaxf(floorf(corr_dim(beta_fast)), 0.0f);
  const float hi = fminf(ceilf(corr_dim(beta_slow)), (float)(n_rot - 1));
  float theta_extrap = (float)pos;
  for (int i = 0; i < n_rot; i += 2) {
    const float theta_interp = freq_scale * theta_extrap;
    float y = ((float)(i / 2) - lo) / fmaxf(hi - lo, 0.001f);
    y = y < 0.0f ? 0.0f : (y > 1.0f ? 1.0f : y);
    const float ramp_mix = (1.0f - y) * ext_factor;
    const float theta = theta_interp * (1.0f - ramp_mix) + theta_extrap * ramp_mix;
    float mscale = attn_factor;
    mscale *= 1.0f + 0.1f * logf(1.0f / freq_scale);
    out[i] = cosf(theta) * mscale;
    out[i + 1] = (1.0f * sinf(theta)) * mscale;
    theta_extrap *= theta_scale;
  }
}

// ---- kernels ---------------------------------------------------------------------

constexpr int kCmpWarps = 8;
constexpr int kCmpMaxSources = 128;  // coff * ratio <= 128
constexpr int kRowF = kRowDim;       // 576 lanes per compressed row
constexpr int kDimIters = kRowF / 32;  // 18 dims per lane

struct CmpArgs {
  rkv_pool_view pool;
  int layer, ratio, coff, cr, width;
  float* states;
  int64_t n_states, n_tok, rope_rows;
  const float* kv;
  const float* score;
  const int32_t* pos;
  const int32_t* state_of;
  const int32_t* emit_slot;
  const float* ape;
  const float* norm;
  const float* rope;
  uint32_t* status;
};

// Where the row of position q (q <= pos of token t, same state s) lives:
// >= 0: input token index; -1: the state's ring; -2: before the sequence start.
__device__ __forceinline__ int source_of(const CmpArgs& a, int64_t t, int p, int s, int q) {
  if (q < 0) return -2;
  const int64_t u = t - (int64_t)(p - q);
  if (u >= 0 && __ldg(a.state_of + u) == s && __ldg(a.pos + u) == q) return (int)u;
  return -1;
}

struct SrcPtr {
  const float* kv;     // column 0 of the row (nullptr: kv 0, score -inf)
  const float* sc;
  const float* ape;    // APE row to add to the score (input rows only), or nullptr
};

__device__ __forceinline__ SrcPtr source_ptr(const CmpArgs& a, int code, int s, int q) {
  SrcPtr r{nullptr, nullptr, nullptr};
  if (code == -2) return r;
  if (code >= 0) {
    r.kv = a.kv + (int64_t)code * a.width;
    r.sc = a.score + (int64_t)code * a.width;
    r.ape = a.ape ? a.ape + (int64_t)(q % a.ratio) * a.width : nullptr;
  } else {
    const float* st = a.states + (int64_t)s * 2 * a.cr * a.width;
    r.kv = st + (int64_t)(q % a.cr) * a.width;
    r.sc = st + (int64_t)(a.cr + q % a.cr) * a.width;
  }
  return r;
}

__device__ __forceinline__ void load_src(const SrcPtr& p, int col, float& kv, float& sc) {
  if (!p.kv) {
    kv = 0.0f;
    sc = -INFINITY;
    return;
  }
  kv = __ldg(p.kv + col);
  sc = __ldg(p.sc + col);
  if (p.ape) sc = __fadd_rn(sc, __ldg(p.ape + col));
}

// One warp per emitting token.
__global__ void __launch_bounds__(kCmpWarps * 32)
compress_emit_kernel(const CmpArgs a, const ThresholdTable tab, const ExpConsts K) {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  __shared__ float s_row[kCmpWarps][kRowF];
  __shared__ int s_src[kCmpWarps][kCmpMaxSources];
  const unsigned FULL = 0xffffffffu;
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  float* row = s_row[w];
  int* src = s_src[w];
  const int64_t stride = (int64_t)gridDim.x * kCmpWarps;
  for (int64_t t = (int64_t)blockIdx.x * kCmpWarps + w; t < a.n_tok; t += stride) {
    const int p = __ldg(a.pos + t), s = __ldg(a.state_of + t), slot = __ldg(a.emit_slot + t);
    if (p < 0 || s < 0 || (int64_t)s >= a.n_states) {
      if (lane == 0) set_status(a.status, RKV_ERR_INDEX_OUT_OF_RANGE);
      continue;
    }
    if ((p + 1) % a.ratio != 0 || slot < 0) continue;
    const int k = (p + 1) / a.ratio - 1;
    if ((int64_t)k >= a.rope_rows) {
      if (lane == 0) set_status(a.status, RKV_ERR_INDEX_OUT_OF_RANGE);
      continue;
    }
    // Sources: coff 2: r < ratio the previous window (p lanes), then the
    // current one (c lanes); coff 1: the current window.
    const int q0 = p + 1 - a.cr;
    for (int r = lane; r < a.cr; r += 32) src[r] = source_of(a, t, p, s, q0 + r);
    __syncwarp();

    if (a.coff == 2) {
      // ratio 4: eight sources, pointers kept in registers.
      SrcPtr sp[4], sc[4];
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        sp[r] = source_ptr(a, src[r], s, q0 + r);
        sc[r] = source_ptr(a, src[4 + r], s, q0 + 4 + r);
      }
#pragma unroll 1
      for (int i = 0; i < kDimIters; ++i) {
        const int j = lane + 32 * i;
        float kp[4], spv[4], kc[4], scv[4];
#pragma unroll
        for (int r = 0; r < 4; ++r) {
          load_src(sp[r], j, kp[r], spv[r]);
          load_src(sc[r], kRowF + j, kc[r], scv[r]);
        }
        float m = -INFINITY;
#pragma unroll
        for (int r = 0; r < 4; ++r) {
          if (spv[r] > m) m = spv[r];
          if (scv[r] > m) m = scv[r];
        }
        float out = 0.0f;
        if (!(m <= -INFINITY)) {
          float den = 0.0f, num = 0.0f;
#pragma unroll
          for (int r = 0; r < 4; ++r) {
            const float wp = expf_host_rounding(__fsub_rn(spv[r], m), K);
            const float wc = expf_host_rounding(__fsub_rn(scv[r], m), K);
            den = __fadd_rn(den, __fadd_rn(wp, wc));
            num = __fadd_rn(num, __fadd_rn(__fmul_rn(wp, kp[r]), __fmul_rn(wc, kc[r])));
          }
          out = den > 0.0f ? __fdiv_rn(num, den) : 0.0f;
        }
        row[j] = out;
      }
    } else {
#pragma unroll 1
      for (int i = 0; i < kDimIters; ++i) {
        const int j = lane + 32 * i;
        float m = -INFINITY;
#pragma unroll 4
        for (int r = 0; r < a.cr; ++r) {
          float kv, sv;
          load_src(source_ptr(a, src[r], s, q0 + r), j, kv, sv);
          if (sv > m) m = sv;
        }
        float out = 0.0f;
        if (!(m <= -INFINITY)) {
          float den = 0.0f, num = 0.0f;
#pragma unroll 4
          for (int r = 0; r < a.cr; ++r) {
            float kv, sv;
            load_src(source_ptr(a, src[r], s, q0 + r), j, kv, sv);
            const float wgt = expf_host_rounding(__fsub_rn(sv, m), K);
            den = __fadd_rn(den, wgt);
            num = __fadd_rn(num, __fmul_rn(wgt, kv));
          }
          out = den > 0.0f ? __fdiv_rn(num, den) : 0.0f;
        }
        row[j] = out;
      }
    }
    __syncwarp();

    // RMSNorm: sequential f64 sum of squares (compressor.rs:292-296).
    float rms = 0.0f;
    if (lane == 0) {
      double ss = 0.0;
#pragma unroll 8
      for (int j = 0; j < kRowF; ++j) {
        const double v = (double)row[j];
        ss = __dadd_rn(ss, __dmul_rn(v, v));
      }
      const float mean = __double2float_rn(__ddiv_rn(ss, (double)kRowF));
      rms = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, 1e-6f)));
    }
    rms = __shfl_sync(FULL, rms, 0);
#pragma unroll
    for (int i = 0; i < kDimIters; ++i) {
      const int j = lane + 32 * i;
      row[j] = __fmul_rn(__fmul_rn(row[j], rms), __ldg(a.norm + j));
    }
    __syncwarp();

    // RoPE of the tail pairs (rope.rs:163-168), lane = pair.
    {
      const float c = __ldg(a.rope + (int64_t)k * 64 + 2 * lane);
      const float sn = __ldg(a.rope + (int64_t)k * 64 + 2 * lane + 1);
      const float x0 = row[kLatent + 2 * lane], x1 = row[kLatent + 2 * lane + 1];
      row[kLatent + 2 * lane] = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, sn));
      row[kLatent + 2 * lane + 1] = __fadd_rn(__fmul_rn(x0, sn), __fmul_rn(x1, c));
    }
    __syncwarp();

    // Quantize-on-append (dsv4_quant.rs:316-362) into the emit slot.
    RowF32 x;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      x.a[i] = __float_as_uint(row[16 * lane + i]);
      x.b[i] = __float_as_uint(row[16 * lane + 8 + i]);
      x.rope[i] = 0u;
    }
    if (lane < 8) {
#pragma unroll
      for (int i = 0; i < 8; ++i) x.rope[i] = __float_as_uint(row[kLatent + 8 * lane + i]);
    }
    x.slot = slot;
    append_row_f32(a.pool, a.layer, x, tab, a.status, lane);
    __syncwarp();
  }
}

// The ring keeps the last coff * ratio rows of every state: a token is
// written when no later token of its state is within coff * ratio of it.
__global__ void __launch_bounds__(256) compress_ring_kernel(const CmpArgs a) {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int lane = threadIdx.x & 31;
  const int64_t stride = (int64_t)gridDim.x * 8;
  for (int64_t t = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5); t < a.n_tok; t += stride) {
    const int p = __ldg(a.pos + t), s = __ldg(a.state_of + t);
    if (p < 0 || s < 0 || (int64_t)s >= a.n_states) continue;
    if (t + a.cr < a.n_tok && __ldg(a.state_of + t + a.cr) == s) continue;
    float* st = a.states + (int64_t)s * 2 * a.cr * a.width;
    const float4* kv = reinterpret_cast<const float4*>(a.kv + t * a.width);
    const float4* sc = reinterpret_cast<const float4*>(a.score + t * a.width);
    const float4* ape = a.ape ? reinterpret_cast<const float4*>(a.ape + (int64_t)(p % a.ratio) * a.width) : nullptr;
    float4* dk = reinterpret_cast<float4*>(st + (int64_t)(p % a.cr) * a.width);
    float4* ds = reinterpret_cast<float4*>(st + (int64_t)(a.cr + p % a.cr) * a.width);
    for (int v = lane; v < a.width / 4; v += 32) {
      dk[v] = __ldg(kv + v);
      float4 x = __ldg(sc + v);
      if (ape) {
        const float4 b = __ldg(ape + v);
        x = make_float4(__fadd_rn(x.x, b.x), __fadd_rn(x.y, b.y), __fadd_rn(x.z, b.z), __fadd_rn(x.w, b.w));
      }
      ds[v] = x;
    }
  }
}

static int coff_of(int ratio) { return ratio == 4 ? 2 : 1; }

}  // namespace rkv

extern "C" int64_t rkv_compress_state_bytes(int32_t ratio) {
  if (ratio <= 0 || ratio > rkv::kCmpMaxSources) return -1;
  const int coff = rkv::coff_of(ratio);
  return (int64_t)2 * coff * ratio * coff * rkv::kRowF * 4;
}

extern "C" rkv_status rkv_compress_rope_table(int32_t ratio, int64_t n_rows, float* out) {
  using namespace rkv;
  if (ratio <= 0 || n_rows < 0 || (n_rows > 0 && (int64_t)(n_rows - 1) * ratio > (int64_t)UINT32_MAX))
    return fail(RKV_ERR_SHAPE_MISMATCH, "rkv_compress_rope_table: ratio %d, %lld rows", ratio, (long long)n_rows);
  if (n_rows > 0 && !out) return fail(RKV_ERR_INVALID_ARGUMENT, "rkv_compress_rope_table: out is required");
  for (int64_t k = 0; k < n_rows; ++k) rope_coeffs((uint32_t)(k * ratio), out + k * 64);
  clear_error();
  return RKV_OK;
}

extern "C" rkv_status rkv_compress_prepare(void) {
  rkv_status st = rkv::prepare_device("rkv_compress_prepare");
  if (st == RKV_OK) rkv::clear_error();
  return st;
}

extern "C" int64_t rkv_compress_expf_table_size(void) {
  const rkv::ExpHost* E = rkv::exp_host();
  return E ? (int64_t)E->entries.size() : -1;
}

extern "C" rkv_status rkv_compress_expf(const float* x, float* out, int64_t n, int32_t host, rkv_stream_t stream) {
  using namespace rkv;
  if (n < 0) return fail(RKV_ERR_SHAPE_MISMATCH, "rkv_compress_expf: n < 0");
  if (n > 0 && (!x || !out)) return fail(RKV_ERR_INVALID_ARGUMENT, "rkv_compress_expf: x and out are required");
  const ExpHost* E = exp_host();
  if (!E) return fail(RKV_ERR_INVALID_ARGUMENT, "rkv_compress_expf: %s", g_exp.err);
  if (host) {
    unsigned nt = std::thread::hardware_concurrency();
    nt = n < (1 << 20) ? 1 : (nt < 1 ? 1 : (nt > 64 ? 64 : nt));
    std::vector<std::thread> th;
    for (unsigned t = 0; t < nt; ++t)
      th.emplace_back([&, t] {
        for (int64_t i = n * t / nt, e = n * (t + 1) / nt; i < e; ++i) out[i] = expf_table_host(x[i], *E);
      });
    for (auto& w : th) w.join();
    clear_error();
    return RKV_OK;
  }
  rkv_status st = prepare_device("rkv_compress_expf");
  if (st != RKV_OK) return st;
  if (n == 0) {
    clear_error();
    return RKV_OK;
  }
  const int64_t blocks = (n + 255) / 256;
  expf_map_kernel<<<(unsigned)(blocks < 148 * 16 ? blocks : 148 * 16), 256, 0, (cudaStream_t)stream>>>(x, out, n,
                                                                                                      E->K);
  return check_launch("rkv_compress_expf");
}

extern "C" rkv_status rkv_compress_append(const rkv_pool_view* pool, int32_t layer, int32_t ratio, float* states,
                                          int64_t n_states, const float* kv, const float* score, int64_t n_tok,
                                          const int32_t* pos, const int32_t* state_of_token,
                                          const int32_t* emit_slot, const float* ape, const float* norm,
                                          const float* rope_table, int64_t rope_rows, uint32_t* d_status,
                                          rkv_stream_t stream) {
  using namespace rkv;
  rkv_status st = check_pool(pool, "rkv_compress_append");
  if (st != RKV_OK) return st;
  if (layer < 0 || layer >= pool->n_layers)
    return fail(RKV_ERR_INVALID_LAYER, "rkv_compress_append: layer %d outside pool of %d layers", layer,
                pool->n_layers);
  if (ratio <= 0 || ratio > kCmpMaxSources)
    return fail(RKV_ERR_SHAPE_MISMATCH, "rkv_compress_append: ratio %d outside [1, %d]", ratio, kCmpMaxSources);
  if (n_tok < 0 || n_states < 0 || rope_rows < 0)
    return fail(RKV_ERR_SHAPE_MISMATCH, "rkv_compress_append: negative sizes");
  if (n_tok > (int64_t)INT32_MAX) return fail(RKV_ERR_SHAPE_MISMATCH, "rkv_compress_append: too many tokens");
  if (n_tok == 0) {
    clear_error();
    return RKV_OK;
  }
  if (!states || !aligned(states, 16) || !kv || !aligned(kv, 16) || !score || !aligned(score, 16) || !pos ||
      !state_of_token || !emit_slot || !norm || !rope_table || (ape && !aligned(ape, 16)) || !d_status)
    return fail(RKV_ERR_INVALID_ARGUMENT,
                "rkv_compress_append: states, kv, score, ape (16-byte aligned), pos, state_of_token, emit_slot, "
                "norm, rope_table and d_status are required");
  st = prepare_device("rkv_compress_append");
  if (st != RKV_OK) return st;
  CmpArgs a;
  a.pool = *pool;
  a.layer = layer;
  a.ratio = ratio;
  a.coff = coff_of(ratio);
  a.cr = a.coff * ratio;
  a.width = a.coff * kRowF;
  a.states = states;
  a.n_states = n_states;
  a.n_tok = n_tok;
  a.rope_rows = rope_rows;
  a.kv = kv;
  a.score = score;
  a.pos = pos;
  a.state_of = state_of_token;
  a.emit_slot = emit_slot;
  a.ape = ape;
  a.norm = norm;
  a.rope = rope_table;
  a.status = d_status;
  const ThresholdTable& tab = f32_threshold_table();
  const ExpConsts K = exp_host()->K;

  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t need = (n_tok + kCmpWarps - 1) / kCmpWarps;
  const int64_t cap = (int64_t)sms * 8;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(need < cap ? need : cap));
  cfg.blockDim = dim3(kCmpWarps * 32);
  cfg.stream = (cudaStream_t)stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, compress_emit_kernel, a, tab, K);
  if (e != cudaSuccess) return fail(RKV_ERR_CUDA, "rkv_compress_append: launch failed: %s", cudaGetErrorString(e));
  const int64_t need2 = (n_tok + 7) / 8;
  cfg.gridDim = dim3((unsigned)(need2 < cap ? need2 : cap));
  cfg.blockDim = dim3(256);
  e = cudaLaunchKernelEx(&cfg, compress_ring_kernel, a);
  if (e != cudaSuccess) return fail(RKV_ERR_CUDA, "rkv_compress_append: launch failed: %s", cudaGetErrorString(e));
  return check_launch("rkv_compress_append");
}
