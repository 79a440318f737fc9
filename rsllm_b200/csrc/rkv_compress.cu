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
// (dsv4_quant.rs:316-362).  Here a batch of tokens is two launches: the
// aggregate kernel (one CTA of 576 threads per emission, one output dimension
// per thread) reads the window's rows straight from this call's input or, for
// positions of earlier calls, from a per-state ring of the last coff * ratio
// rows, and leaves each aggregate row in a workspace; the finishing kernel
// (one warp per row: the in-order f64 sum of squares, RMSNorm, RoPE,
// quantize-on-append) also writes the rings for the next call.
//
// Bit-exactness.  Every f32/f64 operation is rsLLM's, in its order, with
// explicit round-to-nearest intrinsics (no contraction).  rsLLM's exp is the
// host libm's expf, which is not correctly rounded: for about 1e-4 of inputs
// it returns the neighbour of the correctly rounded value.  The kernel
// evaluates exp in double precision (Tang's table-driven method: 2^(k/256)
// from a 256-entry table times a cubic in the reduced argument, |r| <= ln2/512,
// relative error about 2^-42) and rounds it to f32.  Only where that double
// lies within a narrow band around an f32 rounding midpoint can the libm round
// the other way; there the kernel looks x up in a hash table of the inputs
// where the host's expf differs from that rounding.  The host builds the table
// once per process by evaluating the identical double algorithm (the same IEEE
// operations) over every f32 in [-150, 0] and calling its expf wherever the
// double lies within 2^-5 ulp of a midpoint; the band is the largest distance
// at which it found a difference (2^-9.25 ulp for glibc 2.39, so about 0.4% of
// inputs are looked up).  An exhaustive test checks every input.  RoPE cos/sin
// come from a host table computed with the host's libm as rope.rs does.
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

constexpr int kExpTableBits = 8;                 // 2^(j/256)
constexpr uint32_t kExpMaxKey = 0x43160000u;     // |x| bits of 150.0f
constexpr int kExpHashBits = 19;                 // 2 MB open-addressing table, load factor ~0.2
constexpr uint32_t kExpScanWindow = 1u << 24;    // 2^-5 ulp, in units of the 29 dropped bits

struct ExpConsts {
  float inv_step_f;  // 256 / ln 2 rounded to f32
  double step_hi;   // ln 2 / 256, 21 significant bits (k * step_hi is exact)
  double step_lo;   // ln 2 / 256 - step_hi
  double c2, c3;    // 1/2, 1/6
  int64_t band;     // |dropped bits - 2^28| at or below which x is looked up
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

__host__ __device__ __forceinline__ float f_mul(float a, float b) {
#ifdef __CUDA_ARCH__
  return __fmul_rn(a, b);
#else
  return a * b;
#endif
}

// exp(x) in double for x in [-150, 0]; the same IEEE operations on both sides.
// k = rint(x * 256/ln2) is taken in f32 (any integer near the quotient
// serves: r stays within 1.01 * ln2/512); the scaling by 2^(k/256) adds to the
// exponent field (exact: every result is a normal double).
__host__ __device__ __forceinline__ double exp_core(float xf, const ExpConsts& K, const double* T) {
  const double x = (double)xf;
  const float kf = rintf(f_mul(xf, K.inv_step_f));
  const double k = (double)kf;
  const double r = d_sub(d_sub(x, d_mul(k, K.step_hi)), d_mul(k, K.step_lo));
  double p = d_add(d_mul(K.c3, r), K.c2);
  p = d_add(d_mul(p, r), 1.0);
  p = d_add(d_mul(p, r), 1.0);
  const int ki = (int)kf;
  const double y = d_mul(T[ki & ((1 << kExpTableBits) - 1)], p);
  return d_from_bits(d_bits(y) + ((uint64_t)(int64_t)(ki >> kExpTableBits) << 52));
}

// True where the rounding of d to f32 may differ from the host's expf.
__host__ __device__ __forceinline__ bool exp_in_band(double d, int64_t band) {
  if (d < 1.1754943508222875e-38) return true;  // f32 subnormal results: always looked up
  const int64_t low = (int64_t)(d_bits(d) & ((1ull << 29) - 1)) - (1ll << 28);
  return (low < 0 ? -low : low) <= band;
}

__host__ __device__ __forceinline__ uint32_t exp_hash(uint32_t key) {
  return (key * 0x9E3779B1u) >> (32 - kExpHashBits);
}

// ---- host table ------------------------------------------------------------------

struct ExpHost {
  ExpConsts K;
  double T[1 << kExpTableBits];
  std::vector<uint32_t> hash;  // |x| bits | (bit 31: host expf = rounded + 1 ulp, else - 1); 0 = empty
  int64_t n_entries = 0;
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
  E.K.inv_step_f = (float)(256.0L / ln2);
  const double step = (double)(ln2 / 256.0L);
  E.K.step_hi = d_from_bits(d_bits(step) & ~((1ull << 32) - 1));
  E.K.step_lo = (double)(ln2 / 256.0L - (long double)E.K.step_hi);
  E.K.c2 = 0.5;
  E.K.c3 = 1.0 / 6.0;
  E.K.band = kExpScanWindow;
  for (int j = 0; j < (1 << kExpTableBits); ++j) E.T[j] = (double)exp2l((long double)j / 256.0L);

  unsigned nt = std::thread::hardware_concurrency();
  nt = nt < 1 ? 1 : (nt > 64 ? 64 : nt);
  std::vector<std::vector<uint32_t>> part(nt);
  std::vector<int64_t> far(nt, 0);
  std::vector<int> bad(nt, 0);
  std::vector<std::thread> th;
  for (unsigned t = 0; t < nt; ++t)
    th.emplace_back([&, t] {
      const uint64_t n = kExpMaxKey;  // keys 1 .. kExpMaxKey
      const uint32_t a = 1 + (uint32_t)(n * t / nt), b = 1 + (uint32_t)(n * (t + 1) / nt);
      for (uint32_t key = a; key < b; ++key) {
        const float x = bits_to_float(key | 0x80000000u);
        const double d = exp_core(x, E.K, E.T);
        if (!exp_in_band(d, kExpScanWindow)) continue;
        const uint32_t f = float_to_bits((float)d), g = float_to_bits(expf(x));
        if (f == g) continue;
        if (g != f + 1 && g + 1 != f) {
          bad[t] = 1;
          continue;
        }
        if (d >= 1.1754943508222875e-38) {
          const int64_t low = (int64_t)(d_bits(d) & ((1ull << 29) - 1)) - (1ll << 28);
          far[t] = std::max(far[t], low < 0 ? -low : low);
        }
        part[t].push_back(key | (g > f ? 0x80000000u : 0u));
      }
    });
  for (auto& x : th) x.join();
  int64_t band = 1;
  for (unsigned t = 0; t < nt; ++t) {
    if (bad[t]) {
      snprintf(E.err, sizeof E.err, "host expf differs from the double evaluation by more than one ulp");
      return;
    }
    band = std::max(band, far[t]);
    E.n_entries += (int64_t)part[t].size();
  }
  if (band > (int64_t)kExpScanWindow / 2) {
    snprintf(E.err, sizeof E.err, "host expf rounds differently %.4f ulp from a midpoint",
             (double)band / (double)(1 << 29));
    return;
  }
  if (E.n_entries > (1 << kExpHashBits) / 2) {
    snprintf(E.err, sizeof E.err, "expf correction table has %lld entries", (long long)E.n_entries);
    return;
  }
  E.K.band = band;
  E.hash.assign((size_t)1 << kExpHashBits, 0u);
  const uint32_t mask = (1u << kExpHashBits) - 1;
  for (unsigned t = 0; t < nt; ++t)
    for (uint32_t v : part[t]) {
      uint32_t h = exp_hash(v & 0x7fffffffu);
      while (E.hash[h]) h = (h + 1) & mask;
      E.hash[h] = v;
    }
  E.ok = true;
}

static const ExpHost* exp_host() {
  std::call_once(g_exp_once, build_exp_host);
  return g_exp.ok ? &g_exp : nullptr;
}

// The correction for an in-band x: +1, -1 or 0 ulp (table probe).
__host__ __device__ __forceinline__ int exp_correction(uint32_t key, const uint32_t* hash) {
  const uint32_t mask = (1u << kExpHashBits) - 1;
  for (uint32_t h = exp_hash(key);; h = (h + 1) & mask) {
    const uint32_t v = hash[h];
    if (v == 0) return 0;
    if ((v & 0x7fffffffu) == key) return (v >> 31) ? 1 : -1;
  }
}

// Host-side evaluation: the value the kernel produces.
static float expf_table_host(float x, const ExpHost& E) {
  if (x != x) return x;
  if (!(x >= -150.0f)) return 0.0f;
  const double d = exp_core(x, E.K, E.T);
  uint32_t f = float_to_bits((float)d);
  if (exp_in_band(d, E.K.band)) f += exp_correction(float_to_bits(x) & 0x7fffffffu, E.hash.data());
  return bits_to_float(f);
}

// ---- device copies of the table ------------------------------------------------

static __device__ double g_exp_T[1 << kExpTableBits];
static __device__ uint32_t g_exp_hash[1 << kExpHashBits];
// Stand-ins for the rows of positions before a sequence's start (kv 0,
// score -inf) and for "no APE" (adding +0.0 to a score changes at most the
// sign of a zero, which no exp or comparison downstream can see).
static __device__ float g_zero_row[2 * kRowDim];
static __device__ float g_neginf_row[2 * kRowDim];

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
  if (e == cudaSuccess) e = cudaMemcpyToSymbol(g_exp_hash, E->hash.data(), E->hash.size() * 4);
  if (e == cudaSuccess) {
    std::vector<float> ninf(2 * kRowDim, -INFINITY);
    e = cudaMemcpyToSymbol(g_neginf_row, ninf.data(), ninf.size() * 4);
  }
  if (e != cudaSuccess) return fail(RKV_ERR_CUDA, "%s: uploading the expf table: %s", what, cudaGetErrorString(e));
  g_exp_uploaded[dev] = true;
  return RKV_OK;
}

// expf as the host's libm rounds it, in two steps so that a warp's table
// probes can be gathered: exp_first gives the rounded double and whether x is
// in the band; exp_fix applies the table.
struct ExpVal {
  float f;
  bool probe;
};

// Branch-free so that a thread's exps interleave: x below -150 gives 0, NaN
// gives NaN (x > 0 is outside the domain: the aggregate's x = score - max).
__device__ __forceinline__ ExpVal exp_first(float x, const ExpConsts& K, const double* T) {
  const bool in_range = x >= -150.0f;
  const double d = exp_core(in_range ? x : 0.0f, K, T);
  const float f = __double2float_rn(d);
  return {in_range ? f : (x != x ? x : 0.0f), in_range && exp_in_band(d, K.band)};
}

__device__ __forceinline__ float exp_fix(float x, float f) {
  return __uint_as_float(__float_as_uint(f) + exp_correction(__float_as_uint(x) & 0x7fffffffu, g_exp_hash));
}

// The 2 KB table of 2^(j/256), staged in shared memory by each CTA.
__device__ __forceinline__ void load_exp_table(double* s_T) {
  for (int i = threadIdx.x; i < (1 << kExpTableBits); i += blockDim.x) s_T[i] = g_exp_T[i];
  __syncthreads();
}

__global__ void expf_map_kernel(const float* __restrict__ x, float* __restrict__ out, int64_t n, ExpConsts K) {
  __shared__ double s_T[1 << kExpTableBits];
  load_exp_table(s_T);
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const ExpVal v = exp_first(x[i], K, s_T);
    out[i] = v.probe ? exp_fix(x[i], v.f) : v.f;
  }
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

constexpr int kCmpMaxSources = 128;  // coff * ratio <= 128
constexpr int kRowF = kRowDim;       // 576 lanes per compressed row
constexpr int kAggThreads = kRowF;   // aggregate: one thread per output dimension
constexpr int kFinWarps = 8;         // finish: one warp per emitted row

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
  const float* kv;   // column 0 of the row
  const float* sc;
  const float* ape;  // APE row added to the score (zeros for ring rows and when there is no APE)
};

__device__ __forceinline__ SrcPtr source_ptr(const CmpArgs& a, int code, int s, int q) {
  SrcPtr r{g_zero_row, g_neginf_row, g_zero_row};
  if (code >= 0) {
    r.kv = a.kv + (int64_t)code * a.width;
    r.sc = a.score + (int64_t)code * a.width;
    if (a.ape) r.ape = a.ape + (int64_t)(q % a.ratio) * a.width;
  } else if (code == -1) {
    const float* st = a.states + (int64_t)s * 2 * a.cr * a.width;
    r.kv = st + (int64_t)(q % a.cr) * a.width;
    r.sc = st + (int64_t)(a.cr + q % a.cr) * a.width;
  }
  return r;
}

__device__ __forceinline__ void load_src(const SrcPtr& p, int col, float& kv, float& sc) {
  kv = __ldg(p.kv + col);
  sc = __fadd_rn(__ldg(p.sc + col), __ldg(p.ape + col));
}

// Applies the table to the lanes of x[] whose bit is set in `probes`: the
// first probes of all of them are issued together, then the rare collisions
// are walked.
template <int N>
__device__ __forceinline__ void exp_fix_n(const float (&x)[N], float (&f)[N], uint32_t probes) {
  const uint32_t mask = (1u << kExpHashBits) - 1;
  uint32_t h[N], v[N];
#pragma unroll
  for (int r = 0; r < N; ++r) {
    h[r] = exp_hash(__float_as_uint(x[r]) & 0x7fffffffu);
    v[r] = (probes >> r) & 1u ? g_exp_hash[h[r]] : 0u;
  }
#pragma unroll
  for (int r = 0; r < N; ++r) {
    if (!((probes >> r) & 1u)) continue;
    const uint32_t key = __float_as_uint(x[r]) & 0x7fffffffu;
    while (v[r] != 0u && (v[r] & 0x7fffffffu) != key) {
      h[r] = (h[r] + 1) & mask;
      v[r] = g_exp_hash[h[r]];
    }
    if (v[r] != 0u) f[r] = __uint_as_float(__float_as_uint(f[r]) + ((v[r] >> 31) ? 1u : 0xffffffffu));
  }
}

// Stage 1 of an emission: the per-dimension softmax aggregate of the window
// (compressed.rs:481-554), one thread per output dimension (576 threads).
// Each CTA takes groups of `ratio` consecutive tokens (a group inside one
// sequence's run holds exactly one emitting token), lists the emitting ones,
// reserves workspace rows for them with one atomic and writes each aggregate
// row (f32 [576]) and its (slot, compressed row) pair there.
__global__ void __launch_bounds__(kAggThreads, 2)
compress_aggregate_kernel(const CmpArgs a, const ExpConsts K, float* __restrict__ ws_rows,
                          int2* __restrict__ ws_meta, int* __restrict__ ws_count, int64_t ws_cap) {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  __shared__ double s_T[1 << kExpTableBits];
  __shared__ SrcPtr s_ptr[kCmpMaxSources];  // the window's source rows, resolved once per emission
  __shared__ int s_list[kCmpMaxSources][4];
  __shared__ int s_count, s_base;
  load_exp_table(s_T);
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int tid = threadIdx.x, j = tid;
  const int64_t n_groups = (a.n_tok + a.ratio - 1) / a.ratio;
  for (int64_t g = blockIdx.x; g < n_groups; g += gridDim.x) {
    if (tid == 0) s_count = 0;
    __syncthreads();
    if (tid < a.ratio) {
      const int64_t t = g * a.ratio + tid;
      if (t < a.n_tok) {
        const int p = __ldg(a.pos + t), s = __ldg(a.state_of + t), slot = __ldg(a.emit_slot + t);
        if (p < 0 || s < 0 || (int64_t)s >= a.n_states) {
          set_status(a.status, RKV_ERR_INDEX_OUT_OF_RANGE);
        } else if ((p + 1) % a.ratio == 0 && slot >= 0) {
          if ((int64_t)((p + 1) / a.ratio - 1) >= a.rope_rows) {
            set_status(a.status, RKV_ERR_INDEX_OUT_OF_RANGE);
          } else {
            const int i = atomicAdd(&s_count, 1);
            s_list[i][0] = tid;
            s_list[i][1] = p;
            s_list[i][2] = s;
            s_list[i][3] = slot;
          }
        }
      }
    }
    __syncthreads();
    const int n = s_count;
    if (n == 0) continue;
    if (tid == 0) s_base = atomicAdd(ws_count, n);
    __syncthreads();
    const int64_t base = s_base;
    for (int e = 0; e < n; ++e) {
      const int64_t t = g * a.ratio + s_list[e][0];
      const int p = s_list[e][1], s = s_list[e][2];
      const bool room = base + e < ws_cap;
      // Sources: coff 2: r < ratio the previous window (p lanes), then the
      // current one (c lanes); coff 1: the current window.
      const int q0 = p + 1 - a.cr;
      if (tid < a.cr) s_ptr[tid] = source_ptr(a, source_of(a, t, p, s, q0 + tid), s, q0 + tid);
      __syncthreads();
      float out = 0.0f;
      if (a.coff == 2) {
        float kp[4], kc[4], x[8], w[8];
#pragma unroll
        for (int r = 0; r < 4; ++r) {
          load_src(s_ptr[r], j, kp[r], x[2 * r]);
          load_src(s_ptr[4 + r], kRowF + j, kc[r], x[2 * r + 1]);
        }
        float m = -INFINITY;
#pragma unroll
        for (int r = 0; r < 8; ++r)
          if (x[r] > m) m = x[r];  // order p0, c0, p1, c1, ...: the reference's comparison sequence
        if (!(m <= -INFINITY)) {
          uint32_t probes = 0;
#pragma unroll
          for (int r = 0; r < 8; ++r) {
            x[r] = __fsub_rn(x[r], m);
            const ExpVal ev = exp_first(x[r], K, s_T);
            w[r] = ev.f;
            probes |= (uint32_t)ev.probe << r;
          }
          if (probes) exp_fix_n<8>(x, w, probes);
          float den = 0.0f, num = 0.0f;
#pragma unroll
          for (int r = 0; r < 4; ++r) {
            den = __fadd_rn(den, __fadd_rn(w[2 * r], w[2 * r + 1]));
            num = __fadd_rn(num, __fadd_rn(__fmul_rn(w[2 * r], kp[r]), __fmul_rn(w[2 * r + 1], kc[r])));
          }
          out = den > 0.0f ? __fdiv_rn(num, den) : 0.0f;
        }
      } else {
        float m = -INFINITY;
#pragma unroll 8
        for (int r = 0; r < a.cr; ++r) {
          float kv, sv;
          load_src(s_ptr[r], j, kv, sv);
          if (sv > m) m = sv;
        }
        if (!(m <= -INFINITY)) {
          float den = 0.0f, num = 0.0f;
#pragma unroll 1
          for (int r0 = 0; r0 < a.cr; r0 += 8) {
            float x[8], w[8], kv[8];
            uint32_t probes = 0;
#pragma unroll
            for (int r = 0; r < 8; ++r) {
              float sv = -INFINITY;
              kv[r] = 0.0f;
              if (r0 + r < a.cr) load_src(s_ptr[r0 + r], j, kv[r], sv);
              x[r] = __fsub_rn(sv, m);
            }
#pragma unroll
            for (int r = 0; r < 8; ++r) {
              const ExpVal ev = exp_first(x[r], K, s_T);
              w[r] = ev.f;
              probes |= (uint32_t)ev.probe << r;
            }
            if (probes) exp_fix_n<8>(x, w, probes);
#pragma unroll
            for (int r = 0; r < 8; ++r) {
              if (r0 + r < a.cr) {
                den = __fadd_rn(den, w[r]);
                num = __fadd_rn(num, __fmul_rn(w[r], kv[r]));
              }
            }
          }
          out = den > 0.0f ? __fdiv_rn(num, den) : 0.0f;
        }
      }
      if (room) {
        ws_rows[(base + e) * kRowF + j] = out;
        if (tid == 0) ws_meta[base + e] = make_int2(s_list[e][3], (p + 1) / a.ratio - 1);
      } else if (tid == 0) {
        set_status(a.status, RKV_ERR_SHAPE_MISMATCH);  // workspace smaller than the call's emissions
      }
      __syncthreads();  // s_ptr is rewritten for the next emission
    }
  }
}

// The ring keeps the last coff * ratio rows of every state: a token is
// written when no later token of its state is within coff * ratio of it.
// Warps [w0, w0 + n_warps) of the finishing grid do this after the aggregate
// has read the rings.
__device__ __forceinline__ void write_rings(const CmpArgs& a, int64_t w0, int64_t n_warps) {
  const int lane = threadIdx.x & 31;
  for (int64_t t = w0; t < a.n_tok; t += n_warps) {
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

// Stage 2: one warp per aggregated row: RMSNorm with the f64 sum of squares
// added in order by one lane (compressor.rs:292-296), the YaRN rotation of the
// tail pairs (rope.rs:163-168) and the quantize-on-append into the slot
// (dsv4_quant.rs:316-362).  Many warps per SM keep the sequential sums of
// different rows running side by side.
__global__ void __launch_bounds__(kFinWarps * 32)
compress_finish_kernel(const CmpArgs a, const ThresholdTable tab, const float* __restrict__ ws_rows,
                       const int2* __restrict__ ws_meta, const int* __restrict__ ws_count, int64_t ws_cap,
                       int fin_blocks) {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  __shared__ double s_sq[kFinWarps][kRowF];
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const unsigned FULL = 0xffffffffu;
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  if ((int)blockIdx.x >= fin_blocks) {  // the ring writers
    write_rings(a, (int64_t)(blockIdx.x - fin_blocks) * kFinWarps + w, (int64_t)(gridDim.x - fin_blocks) * kFinWarps);
    return;
  }
  double* sq = s_sq[w];
  float* row = reinterpret_cast<float*>(sq);  // reused for the finished row after the sum
  const int64_t count = min((int64_t)*ws_count, ws_cap);
  for (int64_t e = (int64_t)blockIdx.x * kFinWarps + w; e < count; e += (int64_t)fin_blocks * kFinWarps) {
    const int2 meta = ws_meta[e];
    float v[kRowF / 32];
#pragma unroll
    for (int i = 0; i < kRowF / 32; ++i) {
      v[i] = ws_rows[e * kRowF + lane + 32 * i];
      const double d = (double)v[i];
      sq[lane + 32 * i] = __dmul_rn(d, d);
    }
    __syncwarp();
    float rms = 0.0f;
    if (lane == 0) {
      double ss = 0.0;
#pragma unroll 16
      for (int i = 0; i < kRowF; ++i) ss = __dadd_rn(ss, sq[i]);
      const float mean = __double2float_rn(__ddiv_rn(ss, (double)kRowF));
      rms = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, 1e-6f)));
    }
    rms = __shfl_sync(FULL, rms, 0);
    __syncwarp();  // the sum has read sq; row[] overwrites it
#pragma unroll
    for (int i = 0; i < kRowF / 32; ++i)
      row[lane + 32 * i] = __fmul_rn(__fmul_rn(v[i], rms), __ldg(a.norm + lane + 32 * i));
    __syncwarp();
    {
      const float c = __ldg(a.rope + (int64_t)meta.y * 64 + 2 * lane);
      const float sn = __ldg(a.rope + (int64_t)meta.y * 64 + 2 * lane + 1);
      const float x0 = row[kLatent + 2 * lane], x1 = row[kLatent + 2 * lane + 1];
      row[kLatent + 2 * lane] = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, sn));
      row[kLatent + 2 * lane + 1] = __fadd_rn(__fmul_rn(x0, sn), __fmul_rn(x1, c));
    }
    __syncwarp();
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
    x.slot = meta.x;
    append_row_f32(a.pool, a.layer, x, tab, a.status, lane);
    __syncwarp();
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
  return E ? E->n_entries : -1;
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

namespace rkv {

// Workspace of one rkv_compress_append call: the emission count, then per
// emission its (slot, compressed row) pair and its aggregate row.  A state's
// run of L tokens emits at most L / ratio + 1 rows.
static int64_t ws_cap_of(int32_t ratio, int64_t n_tok, int64_t n_states) {
  return n_tok / ratio + (n_tok < n_states ? n_tok : n_states) + 1;
}
static int64_t ws_meta_off() { return 256; }
static int64_t ws_rows_off(int64_t cap) { return (ws_meta_off() + cap * 8 + 255) / 256 * 256; }

}  // namespace rkv

extern "C" int64_t rkv_compress_workspace_bytes(int32_t ratio, int64_t n_tok, int64_t n_states) {
  if (ratio <= 0 || n_tok < 0 || n_states < 0) return -1;
  const int64_t cap = rkv::ws_cap_of(ratio, n_tok, n_states);
  return rkv::ws_rows_off(cap) + cap * rkv::kRowF * 4;
}

extern "C" rkv_status rkv_compress_append(const rkv_pool_view* pool, int32_t layer, int32_t ratio, float* states,
                                          int64_t n_states, const float* kv, const float* score, int64_t n_tok,
                                          const int32_t* pos, const int32_t* state_of_token,
                                          const int32_t* emit_slot, const float* ape, const float* norm,
                                          const float* rope_table, int64_t rope_rows, void* workspace,
                                          int64_t workspace_bytes, uint32_t* d_status, rkv_stream_t stream) {
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
      !state_of_token || !emit_slot || !norm || !rope_table || (ape && !aligned(ape, 16)) || !d_status ||
      !workspace || !aligned(workspace, 256))
    return fail(RKV_ERR_INVALID_ARGUMENT,
                "rkv_compress_append: states, kv, score, ape (16-byte aligned), pos, state_of_token, emit_slot, "
                "norm, rope_table, workspace (256-byte aligned) and d_status are required");
  const int64_t cap = ws_cap_of(ratio, n_tok, n_states);
  if (workspace_bytes < rkv_compress_workspace_bytes(ratio, n_tok, n_states))
    return fail(RKV_ERR_SHAPE_MISMATCH, "rkv_compress_append: workspace of %lld bytes, %lld needed",
                (long long)workspace_bytes, (long long)rkv_compress_workspace_bytes(ratio, n_tok, n_states));
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
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  int* ws_count = reinterpret_cast<int*>(ws);
  int2* ws_meta = reinterpret_cast<int2*>(ws + ws_meta_off());
  float* ws_rows = reinterpret_cast<float*>(ws + ws_rows_off(cap));

  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  cudaError_t e = cudaMemsetAsync(ws_count, 0, 4, (cudaStream_t)stream);
  if (e != cudaSuccess) return fail(RKV_ERR_CUDA, "rkv_compress_append: %s", cudaGetErrorString(e));
  cudaLaunchConfig_t cfg = {};
  cfg.stream = (cudaStream_t)stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  // 1. aggregate: one CTA per token group, two resident per SM
  const int64_t groups = (n_tok + ratio - 1) / ratio;
  const int64_t agg_cap = (int64_t)sms * 2;
  cfg.gridDim = dim3((unsigned)(groups < agg_cap ? groups : agg_cap));
  cfg.blockDim = dim3(kAggThreads);
  e = cudaLaunchKernelEx(&cfg, compress_aggregate_kernel, a, K, ws_rows, ws_meta, ws_count, cap);
  if (e != cudaSuccess) return fail(RKV_ERR_CUDA, "rkv_compress_append: launch failed: %s", cudaGetErrorString(e));
  // 2. finish (one warp per emitted row, at most cap of them) and, in the
  // same grid, the rings for the next call (after the aggregate has read them)
  const int64_t fin_need = (cap + kFinWarps - 1) / kFinWarps, fin_cap = (int64_t)sms * 6;
  const int64_t fin_blocks = fin_need < fin_cap ? fin_need : fin_cap;
  const int64_t ring_need = (n_tok + kFinWarps - 1) / kFinWarps, ring_cap = (int64_t)sms * 2;
  cfg.gridDim = dim3((unsigned)(fin_blocks + (ring_need < ring_cap ? ring_need : ring_cap)));
  cfg.blockDim = dim3(kFinWarps * 32);
  e = cudaLaunchKernelEx(&cfg, compress_finish_kernel, a, tab, (const float*)ws_rows, (const int2*)ws_meta,
                         (const int*)ws_count, cap, (int)fin_blocks);
  if (e != cudaSuccess) return fail(RKV_ERR_CUDA, "rkv_compress_append: launch failed: %s", cudaGetErrorString(e));
  return check_launch("rkv_compress_append");
}
