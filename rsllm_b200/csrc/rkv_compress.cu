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
// emission kernel (one CTA of 576 threads per emission, one output dimension
// per thread) reads the window's rows straight from this call's input or, for
// positions of earlier calls, from a per-state ring of the last coff * ratio
// rows, aggregates, normalises, rotates and quantizes the row into its pool
// slot, and writes the ring rows that no emission of the call still needs;
// the ring kernel writes the rest once every emission has read the rings.
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
// inputs are looked up).  An exhaustive test checks every input.  The f64
// sum of squares of RMSNorm is a tree sum whose mean is used wherever the
// in-order sum provably rounds to the same f32; otherwise (about 1 row in
// 2^16) one thread adds the squares in order.  RoPE cos/sin come from a host
// table computed with the host's libm as rope.rs does.
#include <math.h>
#include <cmath>
#include <stdio.h>
#include <string.h>

#include <algorithm>
#include <atomic>
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
  double inv_step;     // 256 / ln 2
  double magic;        // 1.5 * 2^52: fma(x, inv_step, magic) rounds x * inv_step to an integer
  double neg_step_hi;  // -(ln 2 / 256), 21 significant bits
  double neg_step_lo;  // -(ln 2 / 256 - step_hi)
  double c2, c3;       // 1/2, 1/6
  int32_t band;        // |dropped bits - 2^28| at or below which x is looked up
};

__host__ __device__ __forceinline__ double d_fma(double a, double b, double c) {
#ifdef __CUDA_ARCH__
  return __fma_rn(a, b, c);
#else
  return std::fma(a, b, c);
#endif
}
__host__ __device__ __forceinline__ double d_mul(double a, double b) {
#ifdef __CUDA_ARCH__
  return __dmul_rn(a, b);
#else
  return a * b;
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


// exp(x) in double for x in [-150, 0]; the same IEEE operations on both sides
// (fused multiply-adds are single correctly rounded operations on both).
// k = round(x * 256/ln2) comes from the magic-constant addition, whose low
// word is k itself; r = x - k ln2/256 in two steps (|r| <= ln2/512); the
// scaling by 2^(k/256) adds to the exponent field (exact: every result is a
// normal double).
__host__ __device__ __forceinline__ double exp_core(float xf, const ExpConsts& K, const double* T) {
  const double x = (double)xf;
  const double t = d_fma(x, K.inv_step, K.magic);
  const double k = d_sub(t, K.magic);
  const int ki = (int)(uint32_t)d_bits(t);
  const double r = d_fma(k, K.neg_step_lo, d_fma(k, K.neg_step_hi, x));
  const double p = d_fma(d_fma(d_fma(K.c3, r, K.c2), r, 1.0), r, 1.0);
  const double y = d_mul(T[ki & ((1 << kExpTableBits) - 1)], p);
#ifdef __CUDA_ARCH__
  return __hiloint2double(__double2hiint(y) + ((ki >> kExpTableBits) << 20), __double2loint(y));
#else
  return d_from_bits(d_bits(y) + ((uint64_t)(int64_t)(ki >> kExpTableBits) << 52));
#endif
}

// Distance of the 29 bits that the rounding to f32 drops from their midpoint.
__host__ __device__ __forceinline__ int32_t exp_mid_dist(double d) {
  const int32_t low = (int32_t)((uint32_t)d_bits(d) & ((1u << 29) - 1)) - (1 << 28);
  return low < 0 ? -low : low;
}

// True where the rounding of d to f32 (f) may differ from the host's expf:
// near a rounding midpoint, or f32 results at or below the smallest normal.
__host__ __device__ __forceinline__ bool exp_in_band(double d, uint32_t f_bits, int32_t band) {
  return f_bits <= 0x00800000u || exp_mid_dist(d) <= band;
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
  E.K.inv_step = (double)(256.0L / ln2);
  E.K.magic = 6755399441055744.0;
  const double step = (double)(ln2 / 256.0L);
  const double step_hi = d_from_bits(d_bits(step) & ~((1ull << 32) - 1));
  E.K.neg_step_hi = -step_hi;
  E.K.neg_step_lo = -(double)(ln2 / 256.0L - (long double)step_hi);
  E.K.c2 = 0.5;
  E.K.c3 = 1.0 / 6.0;
  E.K.band = (int32_t)kExpScanWindow;
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
        const uint32_t f = float_to_bits((float)d);
        if (!exp_in_band(d, f, (int32_t)kExpScanWindow)) continue;
        const uint32_t g = float_to_bits(expf(x));
        if (f == g) continue;
        if (g != f + 1 && g + 1 != f) {
          bad[t] = 1;
          continue;
        }
        if (f > 0x00800000u) far[t] = std::max(far[t], (int64_t)exp_mid_dist(d));
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
  E.K.band = (int32_t)band;
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
  if (exp_in_band(d, f, E.K.band)) f += exp_correction(float_to_bits(x) & 0x7fffffffu, E.hash.data());
  return bits_to_float(f);
}

// ---- device copies of the table ------------------------------------------------

static __device__ double g_exp_T[1 << kExpTableBits];
static __device__ uint32_t g_exp_hash[1 << kExpHashBits];
// Stand-ins for the rows of positions before a sequence's start (kv 0,
// score -inf) and for "no APE" (adding +0.0 to a score changes at most the
// sign of a zero, which no exp or comparison downstream can see).
static __device__ __align__(16) float g_zero_row[2 * kRowDim];
static __device__ __align__(16) float g_neginf_row[2 * kRowDim];

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
  return {in_range ? f : (x != x ? x : 0.0f), in_range && exp_in_band(d, __float_as_uint(f), K.band)};
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
constexpr int kRingWarps = 8;        // ring kernel: warps per CTA

struct CmpArgs {
  rkv_pool_view pool;
  int layer, ratio, coff, cr, width;
  int hd;                 // lanes of a compressed row: 576 (attention pool) or 128 (indexer pool)
  float* out_rows;        // indexer pool: f32 [n_out_rows][128] emitted rows
  int64_t n_out_rows;
  uint32_t flags;         // RKV_COMPRESS_INPUTS_READY, RKV_COMPRESS_ONE_TOKEN_PER_STATE
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
  const float* ape;  // APE row added to the score (zeros before the sequence start and when there is no APE)
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
    if (a.ape) r.ape = a.ape + (int64_t)(q % a.ratio) * a.width;
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

// exp of x[0..7] (x <= 0, -inf or NaN) as the host's expf rounds it.  When
// all eight lie in [-87, 0] (no f32 subnormal results, no range or NaN
// handling) the band test is the only check.  A per-lane branch, no warp
// vote: callers may be divergent (dimensions whose scores are all -inf skip
// the exps).
__device__ __forceinline__ void exp8(float (&x)[8], float (&w)[8], const ExpConsts& K, const double* T) {
  bool fast = true;
#pragma unroll
  for (int r = 0; r < 8; ++r) fast = fast && x[r] >= -87.0f;
  uint32_t probes = 0;
  if (fast) {
    const uint32_t lo_edge = (1u << 28) - (uint32_t)K.band, width = 2u * (uint32_t)K.band;
#pragma unroll
    for (int r = 0; r < 8; ++r) {
      const double d = exp_core(x[r], K, T);
      w[r] = __double2float_rn(d);
      const uint32_t low = (uint32_t)__double2loint(d) & ((1u << 29) - 1);
      probes |= (uint32_t)(low - lo_edge <= width) << r;
    }
  } else {
#pragma unroll
    for (int r = 0; r < 8; ++r) {
      const ExpVal ev = exp_first(x[r], K, T);
      w[r] = ev.f;
      probes |= (uint32_t)ev.probe << r;
    }
  }
  if (probes) exp_fix_n<8>(x, w, probes);
}

// The per-dimension softmax aggregate of one emission's window
// (compressed.rs:481-554) for output dimension j, from the window's source
// rows listed in s_ptr (p lanes of the previous window, then c lanes of the
// current one for coff 2).
__device__ __forceinline__ float aggregate_dim(const CmpArgs& a, const ExpConsts& K, const double* s_T,
                                               const SrcPtr* s_ptr, int j) {
  float out = 0.0f;
  if (a.coff == 2) {
    float kp[4], kc[4], x[8], w[8];
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      load_src(s_ptr[r], j, kp[r], x[2 * r]);
      load_src(s_ptr[4 + r], a.hd + j, kc[r], x[2 * r + 1]);
    }
    float m = -INFINITY;
#pragma unroll
    for (int r = 0; r < 8; ++r)
      if (x[r] > m) m = x[r];  // order p0, c0, p1, c1, ...: the reference's comparison sequence
    if (!(m <= -INFINITY)) {
#pragma unroll
      for (int r = 0; r < 8; ++r) x[r] = __fsub_rn(x[r], m);
      exp8(x, w, K, s_T);
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
#pragma unroll
        for (int r = 0; r < 8; ++r) {
          float sv = -INFINITY;
          kv[r] = 0.0f;
          if (r0 + r < a.cr) load_src(s_ptr[r0 + r], j, kv[r], sv);
          x[r] = __fsub_rn(sv, m);
        }
        exp8(x, w, K, s_T);
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
  return out;
}

// The ring keeps the last coff * ratio rows of every state: token t (of
// state s) writes its kv row and its score row at pos % (coff * ratio) when
// no later token of its state is within coff * ratio of it.  The score is kept
// without the APE row, which is added when the row is read (the same rounded
// sum rsLLM stores: APE is a per-layer constant).
__device__ __forceinline__ bool ring_written(const CmpArgs& a, int64_t t, int s) {
  return !(t + a.cr < a.n_tok && __ldg(a.state_of + t + a.cr) == s);
}

// Whether that write may happen while this call's emissions still read the
// ring.  It overwrites position pos - coff*ratio.  For the first token of a
// state's run every emission of the run reads only later positions; from the
// (coff*ratio)-th token of the run on, the overwritten position lies inside
// this call, where the emissions read the input rows.  Other ring writes (the
// 2nd .. (coff*ratio)-th token of a run that is also among its last coff*ratio
// tokens) wait for the ring kernel.
__device__ __forceinline__ bool ring_write_now(const CmpArgs& a, int64_t t, int s) {
  return t == 0 || __ldg(a.state_of + t - 1) != s || (t >= a.cr && __ldg(a.state_of + t - a.cr) == s);
}

// Copies token t's ring rows (kv, and the score as it came, without APE),
// threads [i, i + n) of the caller.
__device__ __forceinline__ void copy_ring_rows(const CmpArgs& a, int64_t t, int p, int s, int i, int n) {
  float4* st = reinterpret_cast<float4*>(a.states + (int64_t)s * 2 * a.cr * a.width);
  const float4* kv = reinterpret_cast<const float4*>(a.kv + t * a.width);
  const float4* sc = reinterpret_cast<const float4*>(a.score + t * a.width);
  const int n4 = a.width / 4;
  float4* dk = st + (int64_t)(p % a.cr) * n4;
  float4* ds = st + (int64_t)(a.cr + p % a.cr) * n4;
  for (int v = i; v < 2 * n4; v += n) {
    if (v < n4)
      dk[v] = __ldg(kv + v);
    else
      ds[v - n4] = __ldg(sc + (v - n4));
  }
}

constexpr int kEmitWarps = kAggThreads / 32;  // 18
// The in-order f64 sum of squares is replaced by a tree sum unless the mean
// lies within this many units of the 29 bits that its rounding to f32 drops
// from a rounding midpoint: both sums are within 585 * 2^-53 of the exact sum
// of the 576 non-negative squares (a tree of depth 10, and 575 roundings in
// order), and the tree's mean (a product with the rounded 1/576) and the
// reference's quotient differ by 3 more roundings, so the two means are
// within 2^9.3 such units of each other and round alike outside the margin.
constexpr int32_t kSumMargin = 1 << 11;

// Barriers over the threads that work on one emission: the whole CTA
// (compress_emit_kernel) or named barrier 1 over the consumer warps
// (compress_emit_staged_kernel).
template <bool kNamed>
__device__ __forceinline__ void emit_bar() {
  if (kNamed)
    asm volatile("bar.sync 1, %0;" ::"n"(kAggThreads) : "memory");
  else
    __syncthreads();
}
template <bool kNamed>
__device__ __forceinline__ bool emit_bar_or(bool v) {
  if (!kNamed) return __syncthreads_or(v) != 0;
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %1, 0;\n\tbar.red.or.pred q, 1, %2, p;\n\tselp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)v), "n"(kAggThreads)
      : "memory");
  return r != 0;
}

struct EmitScratch {
  double* sq;    // [576]
  double* part;  // [18]
  uint32_t* amax;  // [18]
  double* ss;    // [1]
};

// The rest of an emission once thread j (of 576) holds the aggregate `out` of
// dimension j: RMSNorm (compressor.rs:292-296: the f64 sum of squares, its
// mean rounded to f32, 1/sqrt(mean + 1e-6), (v * rms) * w), the YaRN rotation
// of the tail pairs (rope.rs:163-168; c, sn: this thread's pair coefficients)
// and the quantize-on-append of the row (dsv4_quant.rs:316-362) into `slot`.
template <bool kNamed>
__device__ __forceinline__ void emit_finish(const CmpArgs& a, const ThresholdTable& tab, const EmitScratch& sc,
                                            float out, float wn, float c, float sn, int slot) {
  const unsigned FULL = 0xffffffffu;
  const int j = threadIdx.x, lane = j & 31, w = j >> 5;
  const double dv = (double)out;
  const double sq = __dmul_rn(dv, dv);
  sc.sq[j] = sq;
  double ws = sq;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ws = __dadd_rn(ws, __shfl_xor_sync(FULL, ws, o));
  if (lane == 0) sc.part[w] = ws;
  emit_bar<kNamed>();
  double ss = lane < kEmitWarps ? sc.part[lane] : 0.0;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss = __dadd_rn(ss, __shfl_xor_sync(FULL, ss, o));
  double qd = __dmul_rn(ss, 1.0 / (double)kRowF);
  if (!(qd >= 0x1p-125 && qd < 0x1p127) || exp_mid_dist(qd) <= kSumMargin) {  // uniform over the emission's threads
    if (j == 0) {
      double s2 = 0.0;
#pragma unroll 16
      for (int i = 0; i < kRowF; ++i) s2 = __dadd_rn(s2, sc.sq[i]);
      *sc.ss = s2;
    }
    emit_bar<kNamed>();
    qd = __ddiv_rn(*sc.ss, (double)kRowF);
  }
  const float mean = __double2float_rn(qd);
  const float rms = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, 1e-6f)));
  float v = __fmul_rn(__fmul_rn(out, rms), wn);
  if (w >= kLatent / 32) {  // RoPE pairs (j, j ^ 1), warp-uniform
    const float other = __shfl_xor_sync(FULL, v, 1);
    v = (j & 1) ? __fadd_rn(__fmul_rn(other, sn), __fmul_rn(v, c)) : __fsub_rn(__fmul_rn(v, c), __fmul_rn(other, sn));
  }

  // quantize-on-append: block maxima, then one byte per latent lane
  const uint32_t vb = __float_as_uint(v);
  const uint32_t mag = j < kLatent ? (vb & 0x7fffffffu) : 0u;
  const uint32_t wmax = __reduce_max_sync(FULL, mag);
  if (lane == 0) sc.amax[w] = wmax;
  if (emit_bar_or<kNamed>(mag >= 0x7f800000u)) {  // a non-finite latent lane rejects the row
    if (j == 0) set_status(a.status, RKV_ERR_NON_FINITE_INPUT);
    return;
  }
  uint8_t* pg = page_base(a.pool, a.layer, slot >> 6);
  const int off = slot & 63;
  if (j < kLatent) {
    const int blk = j >> 6;
    const int e = scale_exponent_f32(max(sc.amax[2 * blk], sc.amax[2 * blk + 1]), tab);
    uint32_t tq = __float_as_uint(__fmul_rn(v, __uint_as_float((uint32_t)(127 - e) << 23)));
    tq = (tq & 0x7fffffffu) ? tq : 0u;  // the reference's sign is x < 0
    const float hi = __uint_as_float(__shfl_down_sync(FULL, tq, 1));
    const uint32_t c2 = cvt_e4m3x2(__uint_as_float(tq), hi);  // lanes j, j + 1 (even j)
    const uint32_t c4 = c2 | (__shfl_down_sync(FULL, c2, 2) << 16);
    if ((j & 3) == 0) *reinterpret_cast<uint32_t*>(pg + codes_off(off) + j) = c4;
    if ((j & 63) == 0) reinterpret_cast<uint32_t*>(pg + scales_off(off))[blk] = (uint32_t)(e + 127) << 23;
  } else {
    const uint32_t hi = __shfl_down_sync(FULL, vb, 1);
    const uint32_t r2 = bf16x2_rn(vb, hi);
    if ((j & 1) == 0) *reinterpret_cast<uint32_t*>(pg + rope_off(off) + 2 * (j - kLatent)) = r2;
  }
}

// One emission per CTA iteration, one thread per output dimension: the
// aggregate, RMSNorm (compressor.rs:292-296: the f64 sum of squares, its mean
// rounded to f32, 1/sqrt(mean + 1e-6), (v * rms) * w), the YaRN rotation of
// the tail pairs (rope.rs:163-168) and the quantize-on-append of the row
// (dsv4_quant.rs:316-362) straight into its pool slot.  CTAs take groups of
// `ratio` consecutive tokens; the ring rows of the group's tokens are written
// here when ring_write_now allows it.
__global__ void __launch_bounds__(kAggThreads, 2)
compress_emit_kernel(const CmpArgs a, const ExpConsts K, const ThresholdTable tab) {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  __shared__ double s_T[1 << kExpTableBits];
  __shared__ SrcPtr s_ptr[kCmpMaxSources];  // the window's source rows, resolved once per emission
  __shared__ int4 s_tok[kCmpMaxSources];    // pos, state, slot of the group's tokens
  __shared__ uint32_t s_bal[2][kCmpMaxSources / 32];  // emitting / ring-writing tokens of the group
  __shared__ double s_sq[kRowF];
  __shared__ double s_part[kEmitWarps];
  __shared__ uint32_t s_amax[kEmitWarps];
  __shared__ double s_ss;
  const EmitScratch scr{s_sq, s_part, s_amax, &s_ss};
  load_exp_table(s_T);
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const unsigned FULL = 0xffffffffu;
  const int tid = threadIdx.x, j = tid, lane = tid & 31, w = tid >> 5;
  const float wn = __ldg(a.norm + j);
  const int n_bal = (a.ratio + 31) >> 5;
  const int64_t n_groups = (a.n_tok + a.ratio - 1) / a.ratio;
  for (int64_t g = blockIdx.x; g < n_groups; g += gridDim.x) {
    __syncthreads();  // the previous group's s_tok and s_bal are consumed
    if (w < n_bal) {
      const int64_t t = g * a.ratio + tid;
      bool em = false, rg = false;
      if (tid < a.ratio && t < a.n_tok) {
        const int p = __ldg(a.pos + t), s = __ldg(a.state_of + t), slot = __ldg(a.emit_slot + t);
        if (p < 0 || s < 0 || (int64_t)s >= a.n_states) {
          set_status(a.status, RKV_ERR_INDEX_OUT_OF_RANGE);
        } else {
          if ((p + 1) % a.ratio == 0 && slot >= 0) {
            if ((int64_t)((p + 1) / a.ratio - 1) >= a.rope_rows || (int64_t)(slot >> 6) >= a.pool.n_pages)
              set_status(a.status, RKV_ERR_INDEX_OUT_OF_RANGE);
            else
              em = true;
          }
          rg = ring_written(a, t, s) && ring_write_now(a, t, s);
          if ((a.flags & RKV_COMPRESS_ONE_TOKEN_PER_STATE) && ring_written(a, t, s) && !ring_write_now(a, t, s))
            set_status(a.status, RKV_ERR_INVALID_ARGUMENT);
          s_tok[tid] = make_int4(p, s, slot, 0);
        }
      }
      const uint32_t be = __ballot_sync(FULL, em), br = __ballot_sync(FULL, rg);
      if (lane == 0) {
        s_bal[0][w] = be;
        s_bal[1][w] = br;
      }
    }
    __syncthreads();
    for (int b = 0; b < n_bal; ++b) {
      for (uint32_t bits = s_bal[0][b]; bits; bits &= bits - 1) {
        const int tl = 32 * b + __ffs(bits) - 1;
        const int64_t t = g * a.ratio + tl;
        const int4 tk = s_tok[tl];
        const int p = tk.x, s = tk.y, slot = tk.z;
        // Sources: coff 2: r < ratio the previous window (p lanes), then the
        // current one (c lanes); coff 1: the current window.
        const int q0 = p + 1 - a.cr;
        if (tid < a.cr) s_ptr[tid] = source_ptr(a, source_of(a, t, p, s, q0 + tid), s, q0 + tid);
        __syncthreads();
        const float out = aggregate_dim(a, K, s_T, s_ptr, j);

        float c = 0.0f, sn = 0.0f;
        if (j >= kLatent) {
          const float* cs = a.rope + (int64_t)((p + 1) / a.ratio - 1) * 64 + ((j - kLatent) & ~1);
          c = __ldg(cs);
          sn = __ldg(cs + 1);
        }
        emit_finish<false>(a, tab, scr, out, wn, c, sn, slot);
      }
    }
    for (int b = 0; b < n_bal; ++b) {
      for (uint32_t bits = s_bal[1][b]; bits; bits &= bits - 1) {
        const int tl = 32 * b + __ffs(bits) - 1;
        copy_ring_rows(a, g * a.ratio + tl, s_tok[tl].x, s_tok[tl].y, tid, kAggThreads);
      }
    }
  }
}

// The ring writes that the emission kernels left (ring_write_now false), after
// every emission of the call has read the rings: each warp tests 32 tokens
// (one per lane) and copies the deferred ones together.
__global__ void __launch_bounds__(kRingWarps * 32)
compress_ring_kernel(const CmpArgs a) {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const unsigned FULL = 0xffffffffu;
  const int lane = threadIdx.x & 31;
  const int64_t n_warps = (int64_t)gridDim.x * kRingWarps;
  for (int64_t t0 = ((int64_t)blockIdx.x * kRingWarps + (threadIdx.x >> 5)) * 32; t0 < a.n_tok; t0 += n_warps * 32) {
    const int64_t t = t0 + lane;
    int p = -1, s = -1;
    bool deferred = false;
    if (t < a.n_tok) {
      p = __ldg(a.pos + t);
      s = __ldg(a.state_of + t);
      deferred = p >= 0 && s >= 0 && (int64_t)s < a.n_states && ring_written(a, t, s) && !ring_write_now(a, t, s);
    }
    for (uint32_t bits = __ballot_sync(FULL, deferred); bits; bits &= bits - 1) {
      const int L = __ffs(bits) - 1;
      copy_ring_rows(a, t0 + L, __shfl_sync(FULL, p, L), __shfl_sync(FULL, s, L), lane, 32);
    }
  }
}

// ---- the indexer pool's emission (128-lane rows) ------------------------------------
//
// rsLLM runs the same compressor step on its indexer pool (attention.rs:405-429,
// compressor_decode_one with head_dim 128): the aggregate, then RMSNorm and the
// rotation of the last 64 lanes, then a Hadamard + FP4 QAT of the row
// (compressor.rs:343-348) that this library does not restate.  The rows go to
// an f32 row buffer (the rows rkv_indexer_scores_f32 reads) instead of the FP8
// pool.  One CTA of 128 threads per token group, one output dimension per
// thread, the window rows resolved and read as in compress_emit_kernel.

constexpr int kIdxDim = 128;
constexpr int kIdxWarps = kIdxDim / 32;

__global__ void __launch_bounds__(kIdxDim)
indexer_emit_kernel(const CmpArgs a, const ExpConsts K) {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  __shared__ double s_T[1 << kExpTableBits];
  __shared__ SrcPtr s_ptr[kCmpMaxSources];
  __shared__ int4 s_tok[kCmpMaxSources];
  __shared__ uint32_t s_bal[2][kCmpMaxSources / 32];
  __shared__ double s_sq[kIdxDim];
  __shared__ double s_part[kIdxWarps];
  __shared__ double s_ss;
  load_exp_table(s_T);
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const unsigned FULL = 0xffffffffu;
  const int tid = threadIdx.x, j = tid, lane = tid & 31, w = tid >> 5;
  const float wn = __ldg(a.norm + j);
  const int n_bal = (a.ratio + 31) >> 5;
  const int64_t n_groups = (a.n_tok + a.ratio - 1) / a.ratio;
  for (int64_t g = blockIdx.x; g < n_groups; g += gridDim.x) {
    __syncthreads();  // the previous group's s_tok and s_bal are consumed
    if (w < n_bal) {
      const int64_t t = g * a.ratio + tid;
      bool em = false, rg = false;
      if (tid < a.ratio && t < a.n_tok) {
        const int p = __ldg(a.pos + t), s = __ldg(a.state_of + t), row = __ldg(a.emit_slot + t);
        if (p < 0 || s < 0 || (int64_t)s >= a.n_states) {
          set_status(a.status, RKV_ERR_INDEX_OUT_OF_RANGE);
        } else {
          if ((p + 1) % a.ratio == 0 && row >= 0) {
            if ((int64_t)((p + 1) / a.ratio - 1) >= a.rope_rows || (int64_t)row >= a.n_out_rows)
              set_status(a.status, RKV_ERR_INDEX_OUT_OF_RANGE);
            else
              em = true;
          }
          rg = ring_written(a, t, s) && ring_write_now(a, t, s);
          if ((a.flags & RKV_COMPRESS_ONE_TOKEN_PER_STATE) && ring_written(a, t, s) && !ring_write_now(a, t, s))
            set_status(a.status, RKV_ERR_INVALID_ARGUMENT);
          s_tok[tid] = make_int4(p, s, row, 0);
        }
      }
      const uint32_t be = __ballot_sync(FULL, em), br = __ballot_sync(FULL, rg);
      if (lane == 0) {
        s_bal[0][w] = be;
        s_bal[1][w] = br;
      }
    }
    __syncthreads();
    for (int b = 0; b < n_bal; ++b) {
      for (uint32_t bits = s_bal[0][b]; bits; bits &= bits - 1) {
        const int tl = 32 * b + __ffs(bits) - 1;
        const int64_t t = g * a.ratio + tl;
        const int4 tk = s_tok[tl];
        const int p = tk.x, s = tk.y, row = tk.z;
        const int q0 = p + 1 - a.cr;
        if (tid < a.cr) s_ptr[tid] = source_ptr(a, source_of(a, t, p, s, q0 + tid), s, q0 + tid);
        __syncthreads();
        const float out = aggregate_dim(a, K, s_T, s_ptr, j);
        // RMSNorm (compressor.rs:292-296): the f64 sum of squares as a tree,
        // or in rsLLM's order where the two could round to different means
        // (see kSumMargin; the 128-lane sums are even closer), then the mean
        // rounded to f32, 1/sqrt(mean + 1e-6) and (v * rms) * w
        const double dv = (double)out;
        const double sq = __dmul_rn(dv, dv);
        s_sq[j] = sq;
        double ws = sq;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ws = __dadd_rn(ws, __shfl_xor_sync(FULL, ws, o));
        if (lane == 0) s_part[w] = ws;
        __syncthreads();
        double ss = lane < kIdxWarps ? s_part[lane] : 0.0;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ss = __dadd_rn(ss, __shfl_xor_sync(FULL, ss, o));
        double qd = __dmul_rn(ss, 1.0 / (double)kIdxDim);  // exact: a power of two
        if (!(qd >= 0x1p-125 && qd < 0x1p127) || exp_mid_dist(qd) <= kSumMargin) {  // uniform over the CTA
          if (j == 0) {
            double s2 = 0.0;
#pragma unroll 16
            for (int i = 0; i < kIdxDim; ++i) s2 = __dadd_rn(s2, s_sq[i]);
            s_ss = s2;
          }
          __syncthreads();
          qd = __ddiv_rn(s_ss, (double)kIdxDim);
        }
        const float mean = __double2float_rn(qd);
        const float rms = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, 1e-6f)));
        float v = __fmul_rn(__fmul_rn(out, rms), wn);
        if (w >= (kIdxDim - 64) / 32) {  // the 64 tail lanes: RoPE pairs (j, j ^ 1), warp-uniform
          const float* cs = a.rope + (int64_t)((p + 1) / a.ratio - 1) * 64 + ((j - (kIdxDim - 64)) & ~1);
          const float c = __ldg(cs), sn = __ldg(cs + 1);
          const float other = __shfl_xor_sync(FULL, v, 1);
          v = (j & 1) ? __fadd_rn(__fmul_rn(other, sn), __fmul_rn(v, c))
                      : __fsub_rn(__fmul_rn(v, c), __fmul_rn(other, sn));
        }
        a.out_rows[(int64_t)row * kIdxDim + j] = v;
        __syncthreads();  // s_ptr, s_sq and s_part are reused by the next emission
      }
    }
    for (int b = 0; b < n_bal; ++b) {
      for (uint32_t bits = s_bal[1][b]; bits; bits &= bits - 1) {
        const int tl = 32 * b + __ffs(bits) - 1;
        copy_ring_rows(a, g * a.ratio + tl, s_tok[tl].x, s_tok[tl].y, tid, kIdxDim);
      }
    }
  }
}

// ---- staged emission kernel (windows of at most 8 source rows) -------------------
//
// A producer warp walks the CTA's token groups one emission ahead of the 18
// consumer warps: it loads the group's token metadata in one round trip,
// resolves each emission's eight source rows with warp shuffles, and brings the
// half-rows the aggregate reads (2 x 8 x 2304 B) into a shared-memory stage
// with bulk asynchronous copies completing on the stage's mbarrier; it also
// writes the group's ring rows where ring_write_now allows it.  Two stages:
// the consumers aggregate, normalise and quantize one emission while the next
// one's rows arrive.  Every wait is bounded (1 s); a timeout sets
// RKV_ERR_CUDA in the status word and ends the CTA.

constexpr int kStageRows = 8;                          // coff * ratio <= 8
constexpr uint32_t kHalfBytes = kRowF * 4;             // one staged half-row (576 f32)
constexpr int kConsumers = kAggThreads;                // 18 warps, one output dimension per thread
constexpr int kStagedThreads = kConsumers + 32;        // + the producer warp
constexpr uint64_t kStageTimeoutNs = 1000000000ull;

struct StageDesc {
  int kind;  // 1: an emission (its rows arrive on the stage's mbarrier), 2: ring rows only, 0: done
  int p, slot, krow;
  uint32_t ape_mask;  // sources that are real rows (their score gets the APE row)
  int n_ring;         // ring rows to write after the emission (the group's last item carries them)
  int pad[2];
  int ring_t[kStageRows], ring_p[kStageRows], ring_s[kStageRows];
};
static_assert(sizeof(StageDesc) == 128, "stage descriptor layout");

// Dynamic shared memory of the staged kernel.
constexpr uint32_t kStKv = 0;                                         // f32 [2][8][576]
constexpr uint32_t kStSc = kStKv + 2 * kStageRows * kHalfBytes;       // f32 [2][8][576]
constexpr uint32_t kStT = kStSc + 2 * kStageRows * kHalfBytes;        // f64 [256]
constexpr uint32_t kStSq = kStT + (1u << kExpTableBits) * 8;          // f64 [576]
constexpr uint32_t kStPart = kStSq + kRowF * 8;                       // f64 [18]
constexpr uint32_t kStAmax = kStPart + 160;                           // u32 [18]
constexpr uint32_t kStDesc = kStAmax + 80;                            // StageDesc [2]
constexpr uint32_t kStBar = kStDesc + 2 * sizeof(StageDesc);          // full[2], empty[2]
constexpr uint32_t kStMisc = kStBar + 32;                             // f64 sum, abort flag
constexpr uint32_t kStRingBar = kStMisc + 16;                         // ring staging barrier
constexpr uint32_t kStagedSmem = kStRingBar + 16;                     // two CTAs per SM
// One CTA per SM also keeps the APE table (f32 [ratio][width], at most 4608)
// and stages a group's ring rows (at most ratio tokens x 2 x width f32 =
// 36,864 B for every ratio <= 8) so that the producer moves them with bulk
// copies while the consumers compute.
constexpr uint32_t kStApe = kStagedSmem;
constexpr uint32_t kStRing = (kStApe + kStageRows * kHalfBytes + 127) & ~127u;
constexpr uint32_t kRingStageBytes = kStageRows * 2 * kHalfBytes;
constexpr uint32_t kStagedSmem1 = kStRing + kRingStageBytes;

__device__ __forceinline__ uint64_t st_now_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ bool st_mbar_test(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait for the phase of the given parity; false on timeout or abort.
__device__ __noinline__ bool st_mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag) {
  if (st_mbar_test(bar, parity)) return true;
  const uint64_t t0 = st_now_ns();
  while (!st_mbar_test(bar, parity)) {
    if (*abort_flag) return false;
    if (st_now_ns() - t0 > kStageTimeoutNs) return false;
  }
  return true;
}
// Barrier 1 over the consumer warps, AND of a predicate.
__device__ __forceinline__ bool st_bar_and(bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %1, 0;\n\tbar.red.and.pred q, 1, %2, p;\n\tselp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)v), "n"(kConsumers)
      : "memory");
  return r != 0;
}
__device__ __forceinline__ void st_bar() { asm volatile("bar.sync 1, %0;" ::"n"(kConsumers) : "memory"); }
__device__ __forceinline__ void st_arrive_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ void st_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
// Global -> own shared memory bulk copy (no multicast), completing on bar.
__device__ __forceinline__ void st_bulk_load(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile("cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
               "l"(src), "r"(bytes), "r"(bar)
               : "memory");
}
__device__ __forceinline__ uint32_t st_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
// Own shared memory -> global bulk copy, in this thread's bulk async-group.
__device__ __forceinline__ void st_bulk_store(void* dst, uint32_t src, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst), "r"(src), "r"(bytes)
               : "memory");
}

// The aggregate of output dimension j from one stage: kvs / scs hold the
// window's source half-rows [8][576] (for coff 2: sources 0..3 the previous
// window's p lanes, 4..7 the current window's c lanes).  Source r reads APE
// row r % ratio (q0 = pos + 1 - coff*ratio is a multiple of ratio).
// kApeShared: the APE table was staged in shared memory (s_ape); otherwise
// it is read from global memory.
template <bool kApeShared>
__device__ __forceinline__ float aggregate_staged(const CmpArgs& a, const ExpConsts& K, const double* s_T,
                                                  const float* kvs, const float* scs, const float* s_ape,
                                                  uint32_t ape_mask, int j) {
  auto ape_at = [&](int i) { return kApeShared ? s_ape[i] : __ldg(a.ape + i); };
  // The kv values stay in shared memory until the sums: fewer live registers.
  float out = 0.0f;
  if (a.coff == 2) {
    float x[8], w[8];
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      x[2 * r] = scs[r * kRowF + j];
      x[2 * r + 1] = scs[(4 + r) * kRowF + j];
    }
    if (ape_mask) {
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        if ((ape_mask >> r) & 1u) x[2 * r] = __fadd_rn(x[2 * r], ape_at(r * a.width + j));
        if ((ape_mask >> (4 + r)) & 1u) x[2 * r + 1] = __fadd_rn(x[2 * r + 1], ape_at(r * a.width + kRowF + j));
      }
    }
    float m = -INFINITY;
#pragma unroll
    for (int r = 0; r < 8; ++r)
      if (x[r] > m) m = x[r];  // order p0, c0, p1, c1, ...: the reference's comparison sequence
    if (!(m <= -INFINITY)) {
#pragma unroll
      for (int r = 0; r < 8; ++r) x[r] = __fsub_rn(x[r], m);
      exp8(x, w, K, s_T);
      float den = 0.0f, num = 0.0f;
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        den = __fadd_rn(den, __fadd_rn(w[2 * r], w[2 * r + 1]));
        num = __fadd_rn(num, __fadd_rn(__fmul_rn(w[2 * r], kvs[r * kRowF + j]),
                                       __fmul_rn(w[2 * r + 1], kvs[(4 + r) * kRowF + j])));
      }
      out = den > 0.0f ? __fdiv_rn(num, den) : 0.0f;
    }
  } else {
    float x[8], w[8];
#pragma unroll
    for (int r = 0; r < 8; ++r) {
      x[r] = -INFINITY;
      if (r < a.cr) {
        x[r] = scs[r * kRowF + j];
        if ((ape_mask >> r) & 1u) x[r] = __fadd_rn(x[r], ape_at(r * a.width + j));
      }
    }
    float m = -INFINITY;
#pragma unroll
    for (int r = 0; r < 8; ++r)
      if (x[r] > m) m = x[r];
    if (!(m <= -INFINITY)) {
#pragma unroll
      for (int r = 0; r < 8; ++r) x[r] = r < a.cr ? __fsub_rn(x[r], m) : 0.0f;  // padding: unused
      exp8(x, w, K, s_T);
      float den = 0.0f, num = 0.0f;
#pragma unroll
      for (int r = 0; r < 8; ++r) {
        if (r < a.cr) {
          den = __fadd_rn(den, w[r]);
          num = __fadd_rn(num, __fmul_rn(w[r], kvs[r * kRowF + j]));
        }
      }
      out = den > 0.0f ? __fdiv_rn(num, den) : 0.0f;
    }
  }
  return out;
}

// Thread j of 576 copies its share of the ring rows listed in the stage
// descriptor (token kv and score rows, one float4 at a time, four in flight).
__device__ __forceinline__ void copy_ring_staged(const CmpArgs& a, const StageDesc* d, int n_ring, int j) {
  const int n4 = a.width / 4, per = 2 * n4, total = n_ring * per;
  for (int base = j; base < total; base += 4 * kAggThreads) {
    float4 v[4];
    float4* dst[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int i = base + k * kAggThreads;
      dst[k] = nullptr;
      if (i < total) {
        const int e = i / per, x = i - e * per;
        const int64_t t = d->ring_t[e];
        const int p = d->ring_p[e], s = d->ring_s[e];
        float4* st = reinterpret_cast<float4*>(a.states + (int64_t)s * 2 * a.cr * a.width);
        if (x < n4) {
          v[k] = __ldg(reinterpret_cast<const float4*>(a.kv) + t * n4 + x);
          dst[k] = st + (int64_t)(p % a.cr) * n4 + x;
        } else {
          v[k] = __ldg(reinterpret_cast<const float4*>(a.score) + t * n4 + (x - n4));
          dst[k] = st + (int64_t)(a.cr + p % a.cr) * n4 + (x - n4);
        }
      }
    }
#pragma unroll
    for (int k = 0; k < 4; ++k)
      if (dst[k]) *dst[k] = v[k];
  }
}

// kMinBlocks 2: two CTAs per SM (48 registers, some spilled) for calls with
// more token groups than SMs; 1: one CTA per SM with no spills, the shorter
// latency for decode-sized calls.
template <int kMinBlocks>
__global__ void __launch_bounds__(kStagedThreads, kMinBlocks)
compress_emit_staged_kernel(const CmpArgs a, const ExpConsts K, const ThresholdTable tab) {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  extern __shared__ __align__(16) uint8_t st_smem[];
  float* s_kv = reinterpret_cast<float*>(st_smem + kStKv);
  float* s_sc = reinterpret_cast<float*>(st_smem + kStSc);
  double* s_T = reinterpret_cast<double*>(st_smem + kStT);
  StageDesc* s_desc = reinterpret_cast<StageDesc*>(st_smem + kStDesc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(st_smem + kStMisc + 8);
  const EmitScratch scr{reinterpret_cast<double*>(st_smem + kStSq), reinterpret_cast<double*>(st_smem + kStPart),
                        reinterpret_cast<uint32_t*>(st_smem + kStAmax), reinterpret_cast<double*>(st_smem + kStMisc)};
  const uint32_t bar_full = st_u32(st_smem + kStBar), bar_empty = bar_full + 16;  // [2] each, 8 B apart
  const unsigned FULL = 0xffffffffu;
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  for (int i = tid; i < (1 << kExpTableBits); i += kStagedThreads) s_T[i] = g_exp_T[i];
  if (tid == 0) {
    for (int b = 0; b < 4; ++b)
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(bar_full + 8 * b) : "memory");
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(st_u32(st_smem + kStRingBar)) : "memory");
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  // With RKV_COMPRESS_INPUTS_READY the token metadata, the APE, norm and RoPE
  // tables are complete before the previous kernel on the stream ends: the
  // producer reads them and resolves the first window's sources, and the
  // consumers stage the APE table, before waiting for that kernel (the
  // producer waits before its first copy of a kv / score / ring row, and the
  // consumers touch no other global memory before its copies arrive).
  const bool early = (a.flags & RKV_COMPRESS_INPUTS_READY) != 0;
  if (!early) asm volatile("griddepcontrol.wait;" ::: "memory");

  if (w == kConsumers / 32) {
    // ---- producer warp ----
    const int cr = a.cr, ratio = a.ratio, n_meta = 2 * cr + ratio;  // n_meta <= 24
    const int64_t n_groups = (a.n_tok + ratio - 1) / ratio;
    uint32_t it = 0, ring_phase = 0;
    bool ok = true, waited = !early;
    for (int64_t g = blockIdx.x; g < n_groups && ok; g += gridDim.x) {
      // tokens t0 - cr .. t0 + ratio + cr - 1 around the group, one per lane
      const int64_t t0 = g * ratio, tm = t0 - cr + lane;
      int mp = -1, ms = -1, mslot = -1;
      if (lane < n_meta && tm >= 0 && tm < a.n_tok) {
        mp = __ldg(a.pos + tm);
        ms = __ldg(a.state_of + tm);
        mslot = __ldg(a.emit_slot + tm);
      }
      const bool in_group = lane >= cr && lane < cr + ratio && tm < a.n_tok;
      const bool valid = mp >= 0 && ms >= 0 && (int64_t)ms < a.n_states;
      if (in_group && !valid) set_status(a.status, RKV_ERR_INDEX_OUT_OF_RANGE);
      const int s_prev = __shfl_sync(FULL, ms, (lane - 1) & 31);
      const int s_back = __shfl_sync(FULL, ms, (lane - cr) & 31);
      const int s_fwd = __shfl_sync(FULL, ms, (lane + cr) & 31);
      bool em = false;
      if (in_group && valid && (mp + 1) % ratio == 0 && mslot >= 0) {
        if ((int64_t)((mp + 1) / ratio - 1) >= a.rope_rows || (int64_t)(mslot >> 6) >= a.pool.n_pages)
          set_status(a.status, RKV_ERR_INDEX_OUT_OF_RANGE);
        else
          em = true;
      }
      // ring_written and ring_write_now from the neighbouring lanes
      const bool rg = in_group && valid && s_fwd != ms && (s_prev != ms || s_back == ms);
      // a ring write left for the ring kernel, which RKV_COMPRESS_ONE_TOKEN_PER_STATE does not launch
      if ((a.flags & RKV_COMPRESS_ONE_TOKEN_PER_STATE) && in_group && valid && s_fwd != ms && s_prev == ms &&
          s_back != ms)
        set_status(a.status, RKV_ERR_INVALID_ARGUMENT);
      const uint32_t emask = __ballot_sync(FULL, em), rmask = __ballot_sync(FULL, rg);
      // one CTA per SM: the producer writes the ring rows itself (below)
      const int n_ring = kMinBlocks == 1 ? 0 : __popc(rmask);
      // items: one per emission, the last one carrying the ring rows; or one
      // ring-only item
      uint32_t items = emask ? emask : (n_ring ? (rmask & (0u - rmask)) : 0u);
      for (; items; items &= items - 1) {
        const int L = __ffs(items) - 1;
        const bool emission = emask != 0, last = (items & (items - 1)) == 0;
        const uint32_t buf = it & 1;
        if (it >= 2) {
          bool got = true;
          if (lane == 0) got = st_mbar_wait(bar_empty + 8 * buf, ((it >> 1) - 1) & 1, abort_flag);
          if (!__shfl_sync(FULL, (int)got, 0)) {
            ok = false;
            break;
          }
        }
        StageDesc* d = s_desc + buf;
        const int nr = last ? n_ring : 0;
        if (nr && rg) {  // nr == 0 when the producer writes the ring rows
          const int e = __popc(rmask & ((1u << lane) - 1));
          d->ring_t[e] = (int)(t0 - cr + lane);
          d->ring_p[e] = mp;
          d->ring_s[e] = ms;
        }
        const uint32_t full = bar_full + 8 * buf;
        if (!emission) {
          if (early && !waited) {  // the consumers copy this call's kv / score rows into the ring
            asm volatile("griddepcontrol.wait;" ::: "memory");
            waited = true;
          }
          __syncwarp();
          if (lane == 0) {
            d->kind = 2;
            d->n_ring = nr;
            st_arrive(full);
          }
          ++it;
          continue;
        }
        const int p = __shfl_sync(FULL, mp, L), s = __shfl_sync(FULL, ms, L), slot = __shfl_sync(FULL, mslot, L);
        const int64_t t = t0 - cr + L;
        // source r = lane: position q = p + 1 - cr + r, input token u = t - cr + 1 + r
        const int r = lane, q = p + 1 - cr + r;
        const int lu = r < cr ? L - cr + 1 + r : L;
        const int su = __shfl_sync(FULL, ms, lu), pu = __shfl_sync(FULL, mp, lu);
        const int col = (a.coff == 2 && r >= ratio) ? kRowF : 0;
        const float* skv = g_zero_row + col;
        const float* ssc = g_neginf_row + col;
        if (q >= 0 && su == s && pu == q) {
          const int64_t u = t - cr + 1 + r;
          skv = a.kv + u * a.width + col;
          ssc = a.score + u * a.width + col;
        } else if (q >= 0) {
          const float* st = a.states + (int64_t)s * 2 * cr * a.width;
          skv = st + (int64_t)(q % cr) * a.width + col;
          ssc = st + (int64_t)(cr + q % cr) * a.width + col;
        }
        const uint32_t apem = __ballot_sync(FULL, r < cr && q >= 0 && a.ape != nullptr);
        __syncwarp();
        if (lane == 0) {
          d->kind = 1;
          d->p = p;
          d->slot = slot;
          d->krow = (p + 1) / ratio - 1;
          d->ape_mask = apem;
          d->n_ring = nr;
          st_arrive_tx(full, 2u * cr * kHalfBytes);
        }
        __syncwarp();
        if (early && !waited) {  // the rows may come from the previous kernel
          asm volatile("griddepcontrol.wait;" ::: "memory");
          waited = true;
        }
        if (r < cr) {
          st_bulk_load(st_u32(s_kv + (buf * kStageRows + r) * kRowF), skv, kHalfBytes, full);
          st_bulk_load(st_u32(s_sc + (buf * kStageRows + r) * kRowF), ssc, kHalfBytes, full);
        }
        ++it;
      }
      if (kMinBlocks == 1 && ok && rmask) {
        // this group's ring rows (all safe to write now): bulk loads into the
        // staging buffer, then bulk stores into the ring slots, while the
        // consumers compute the group's emissions
        if (early && !waited) {
          asm volatile("griddepcontrol.wait;" ::: "memory");
          waited = true;
        }
        asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");  // earlier stores have read the buffer
        __syncwarp();
        const uint32_t rbar = st_u32(st_smem + kStRingBar), row_bytes = (uint32_t)a.width * 4u;
        if (lane == 0) st_arrive_tx(rbar, (uint32_t)__popc(rmask) * 2u * row_bytes);
        __syncwarp();
        const uint32_t sbuf = st_u32(st_smem + kStRing) + (uint32_t)__popc(rmask & ((1u << lane) - 1u)) * 2u * row_bytes;
        const int64_t t = t0 - cr + lane;
        if (rg) {
          st_bulk_load(sbuf, a.kv + t * a.width, row_bytes, rbar);
          st_bulk_load(sbuf + row_bytes, a.score + t * a.width, row_bytes, rbar);
        }
        bool got = true;
        if (lane == 0) got = st_mbar_wait(rbar, ring_phase & 1u, abort_flag);
        if (!__shfl_sync(FULL, (int)got, 0)) {
          ok = false;
          break;
        }
        ++ring_phase;
        if (rg) {
          float* st = a.states + (int64_t)ms * 2 * cr * a.width;
          st_bulk_store(st + (int64_t)(mp % cr) * a.width, sbuf, row_bytes);
          st_bulk_store(st + (int64_t)(cr + mp % cr) * a.width, sbuf + row_bytes, row_bytes);
          asm volatile("cp.async.bulk.commit_group;" ::: "memory");
        }
      }
    }
    if (ok) {  // the end marker
      const uint32_t buf = it & 1;
      bool got = true;
      if (it >= 2 && lane == 0) got = st_mbar_wait(bar_empty + 8 * buf, ((it >> 1) - 1) & 1, abort_flag);
      ok = __shfl_sync(FULL, (int)got, 0) != 0;
      if (ok && lane == 0) {
        s_desc[buf].kind = 0;
        st_arrive(bar_full + 8 * buf);
      }
    }
    if (!ok && lane == 0) {
      *abort_flag = 1;
      set_status(a.status, RKV_ERR_CUDA);
      // copies this CTA issued may still be in flight: wait for them (bounded)
      // before the CTA's shared memory goes away
      for (uint32_t i = it >= 2 ? it - 2 : 0; i < it; ++i) {
        const uint32_t bar = bar_full + 8 * (i & 1), par = (i >> 1) & 1;
        const uint64_t t0 = st_now_ns();
        while (!st_mbar_test(bar, par) && st_now_ns() - t0 < kStageTimeoutNs) {
        }
      }
      if (kMinBlocks == 1) {  // and the ring rows of an unfinished group
        const uint64_t t0 = st_now_ns();
        while (!st_mbar_test(st_u32(st_smem + kStRingBar), ring_phase & 1u) && st_now_ns() - t0 < kStageTimeoutNs) {
        }
      }
    }
    // a CTA with nothing to copy still waits: this grid then completes only after
    // the previous one, so later kernels' waits cover every grid before it
    if (early && !waited) asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");  // this lane's ring stores are done
    return;
  }

  // ---- consumer warps: thread j owns output dimension j ----
  const int j = tid;
  const float wn = __ldg(a.norm + j);
  // one CTA per SM (decode): the APE table into shared memory while the
  // first stage is on its way (the stage-ready barrier below orders these
  // writes before the reads)
  float* s_ape = reinterpret_cast<float*>(st_smem + kStApe);
  if (kMinBlocks == 1 && a.ape)
    for (int i = j; i < a.ratio * a.width; i += kConsumers) s_ape[i] = __ldg(a.ape + i);
  for (uint32_t it = 0;; ++it) {
    const uint32_t buf = it & 1;
    bool got = true;
    if (j == 0) got = st_mbar_wait(bar_full + 8 * buf, (it >> 1) & 1, abort_flag);
    if (!st_bar_and(got)) {
      if (j == 0) {
        *abort_flag = 1;
        set_status(a.status, RKV_ERR_CUDA);
      }
      break;
    }
    const StageDesc* d = s_desc + buf;
    const int kind = d->kind, n_ring = d->n_ring;
    if (kind == 0) break;
    if (kind == 1) {
      const int slot = d->slot;
      const uint32_t ape_mask = d->ape_mask;
      float c = 0.0f, sn = 0.0f;
      if (j >= kLatent) {
        const float* cs = a.rope + (int64_t)d->krow * 64 + ((j - kLatent) & ~1);
        c = __ldg(cs);
        sn = __ldg(cs + 1);
      }
      const float out = aggregate_staged<kMinBlocks == 1>(a, K, s_T, s_kv + buf * kStageRows * kRowF,
                                         s_sc + buf * kStageRows * kRowF, s_ape, ape_mask, j);
      emit_finish<true>(a, tab, scr, out, wn, c, sn, slot);
    }
    if (n_ring) {
      copy_ring_staged(a, d, n_ring, j);
      st_bar();  // every thread has read the descriptor
    }
    // the stage (rows, descriptor) is free once every thread is past its
    // reads: the emission's barriers, or the one above
    if (j == 0) st_arrive(bar_empty + 8 * buf);
  }
}

// Test hook for the bounded waits: thread 0 waits, with the staged kernel's
// st_mbar_wait, for a phase of an mbarrier that nothing arrives on.  The wait
// gives up after kStageTimeoutNs, the kernel records RKV_ERR_CUDA in the
// status word and returns -- the path every staged-kernel wait takes when its
// producer or consumers stop -- and the context stays usable.
__global__ void wait_probe_kernel(uint32_t* status) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(st_u32(&bar)) : "memory");
    abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  if (threadIdx.x == 0 && !st_mbar_wait(st_u32(&bar), 0, &abort_flag)) set_status(status, RKV_ERR_CUDA);
}

static int coff_of(int ratio) { return ratio == 4 ? 2 : 1; }

// The staged kernels' shared-memory opt-in, once per device.
static std::atomic<bool> g_staged_smem[kMaxDevices];

static rkv_status staged_smem_opt_in(int dev) {
  if (dev < 0 || dev >= kMaxDevices) return fail(RKV_ERR_INVALID_ARGUMENT, "rkv_compress_append: device %d", dev);
  if (g_staged_smem[dev].load(std::memory_order_acquire)) return RKV_OK;
  cudaError_t e = cudaFuncSetAttribute(compress_emit_staged_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)kStagedSmem1);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(compress_emit_staged_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)kStagedSmem);
  if (e != cudaSuccess) return fail(RKV_ERR_CUDA, "rkv_compress_append: %s", cudaGetErrorString(e));
  g_staged_smem[dev].store(true, std::memory_order_release);
  return RKV_OK;
}

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

extern "C" rkv_status rkv_compress_wait_probe(uint32_t* d_status, rkv_stream_t stream) {
  using namespace rkv;
  if (!d_status) return fail(RKV_ERR_INVALID_ARGUMENT, "rkv_compress_wait_probe: d_status is required");
  wait_probe_kernel<<<1, 32, 0, (cudaStream_t)stream>>>(d_status);
  return check_launch("rkv_compress_wait_probe");
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
static rkv_status compress_append(const rkv_pool_view* pool, int32_t layer, int32_t ratio, float* states,
                                  int64_t n_states, const float* kv, const float* score, int64_t n_tok,
                                  const int32_t* pos, const int32_t* state_of_token, const int32_t* emit_slot,
                                  const float* ape, const float* norm, const float* rope_table, int64_t rope_rows,
                                  uint32_t flags, uint32_t* d_status, rkv_stream_t stream) {
  if (flags & ~(RKV_COMPRESS_INPUTS_READY | RKV_COMPRESS_ONE_TOKEN_PER_STATE))
    return fail(RKV_ERR_INVALID_ARGUMENT, "rkv_compress_append_ex: unknown flags 0x%x", flags);
  rkv_status st = check_pool(pool, "rkv_compress_append");
  if (st != RKV_OK) return st;
  if (layer < 0 || layer >= pool->n_layers)
    return fail_layer(layer, pool->n_layers, "rkv_compress_append: layer %d outside pool of %d layers", layer,
                      pool->n_layers);
  if (ratio <= 0 || ratio > kCmpMaxSources)
    return fail_shape("ratio", kCmpMaxSources, ratio, "rkv_compress_append: ratio %d outside [1, %d]", ratio,
                      kCmpMaxSources);
  if (n_tok < 0 || n_states < 0 || rope_rows < 0)
    return fail(RKV_ERR_SHAPE_MISMATCH, "rkv_compress_append: negative sizes");
  if (n_tok > (int64_t)INT32_MAX)
    return fail_shape("n_tokens", INT32_MAX, n_tok, "rkv_compress_append: too many tokens");
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
  a.hd = kRowF;
  a.out_rows = nullptr;
  a.n_out_rows = 0;
  a.flags = flags;
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
  cudaLaunchConfig_t cfg = {};
  cfg.stream = (cudaStream_t)stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  // 1. emissions and the ring writes that may happen alongside them: one CTA
  // per token group, two resident per SM; windows of up to 8 rows go through
  // the staged kernel
  const int64_t groups = (n_tok + ratio - 1) / ratio;
  const int64_t emit_cap = (int64_t)sms * 2;
  cfg.gridDim = dim3((unsigned)(groups < emit_cap ? groups : emit_cap));
  cudaError_t e;
  if (a.cr <= kStageRows) {
    st = staged_smem_opt_in(dev);
    if (st != RKV_OK) return st;
    cfg.blockDim = dim3(kStagedThreads);
    if (groups <= sms) {
      cfg.dynamicSmemBytes = kStagedSmem1;
      e = cudaLaunchKernelEx(&cfg, compress_emit_staged_kernel<1>, a, K, tab);
    } else {
      cfg.dynamicSmemBytes = kStagedSmem;
      e = cudaLaunchKernelEx(&cfg, compress_emit_staged_kernel<2>, a, K, tab);
    }
    cfg.dynamicSmemBytes = 0;
  } else {
    cfg.blockDim = dim3(kAggThreads);
    e = cudaLaunchKernelEx(&cfg, compress_emit_kernel, a, K, tab);
  }
  if (e != cudaSuccess) return fail(RKV_ERR_CUDA, "rkv_compress_append: launch failed: %s", cudaGetErrorString(e));
  // 2. the remaining ring writes, after every emission has read the rings
  // (none when every state has at most one token in the call)
  if (!(flags & RKV_COMPRESS_ONE_TOKEN_PER_STATE)) {
    const int64_t ring_need = (n_tok + 32 * kRingWarps - 1) / (32 * kRingWarps), ring_cap = (int64_t)sms * 2;
    cfg.gridDim = dim3((unsigned)(ring_need < ring_cap ? ring_need : ring_cap));
    cfg.blockDim = dim3(kRingWarps * 32);
    e = cudaLaunchKernelEx(&cfg, compress_ring_kernel, a);
    if (e != cudaSuccess) return fail(RKV_ERR_CUDA, "rkv_compress_append: launch failed: %s", cudaGetErrorString(e));
  }
  return check_launch("rkv_compress_append");
}
}  // namespace rkv

extern "C" rkv_status rkv_compress_append(const rkv_pool_view* pool, int32_t layer, int32_t ratio, float* states,
                                          int64_t n_states, const float* kv, const float* score, int64_t n_tok,
                                          const int32_t* pos, const int32_t* state_of_token,
                                          const int32_t* emit_slot, const float* ape, const float* norm,
                                          const float* rope_table, int64_t rope_rows, uint32_t* d_status,
                                          rkv_stream_t stream) {
  return rkv::compress_append(pool, layer, ratio, states, n_states, kv, score, n_tok, pos, state_of_token, emit_slot,
                              ape, norm, rope_table, rope_rows, 0u, d_status, stream);
}

extern "C" rkv_status rkv_compress_append_ex(const rkv_pool_view* pool, int32_t layer, int32_t ratio, float* states,
                                             int64_t n_states, const float* kv, const float* score, int64_t n_tok,
                                             const int32_t* pos, const int32_t* state_of_token,
                                             const int32_t* emit_slot, const float* ape, const float* norm,
                                             const float* rope_table, int64_t rope_rows, uint32_t flags,
                                             uint32_t* d_status, rkv_stream_t stream) {
  return rkv::compress_append(pool, layer, ratio, states, n_states, kv, score, n_tok, pos, state_of_token, emit_slot,
                              ape, norm, rope_table, rope_rows, flags, d_status, stream);
}

extern "C" int64_t rkv_indexer_compress_state_bytes(int32_t ratio) {
  if (ratio <= 0 || ratio > rkv::kCmpMaxSources) return -1;
  const int coff = rkv::coff_of(ratio);
  if (coff * ratio > rkv::kCmpMaxSources) return -1;
  return (int64_t)2 * coff * ratio * coff * rkv::kIdxDim * 4;
}

extern "C" rkv_status rkv_indexer_compress_append(int32_t ratio, float* states, int64_t n_states, const float* kv,
                                                  const float* score, int64_t n_tok, const int32_t* pos,
                                                  const int32_t* state_of_token, const int32_t* emit_row,
                                                  const float* ape, const float* norm, const float* rope_table,
                                                  int64_t rope_rows, float* out_rows, int64_t n_out_rows,
                                                  uint32_t* d_status, rkv_stream_t stream) {
  using namespace rkv;
  const char* what = "rkv_indexer_compress_append";
  if (ratio <= 0 || coff_of(ratio) * ratio > kCmpMaxSources)
    return fail_shape("ratio", kCmpMaxSources, ratio, "%s: ratio %d outside [1, %d]", what, ratio, kCmpMaxSources);
  if (n_tok < 0 || n_states < 0 || rope_rows < 0 || n_out_rows < 0)
    return fail(RKV_ERR_SHAPE_MISMATCH, "%s: negative sizes", what);
  if (n_tok > (int64_t)INT32_MAX) return fail_shape("n_tokens", INT32_MAX, n_tok, "%s: too many tokens", what);
  if (n_tok == 0) {
    clear_error();
    return RKV_OK;
  }
  if (!states || !aligned(states, 16) || !kv || !aligned(kv, 16) || !score || !aligned(score, 16) || !pos ||
      !state_of_token || !emit_row || !norm || !rope_table || (ape && !aligned(ape, 16)) || !out_rows ||
      !d_status)
    return fail(RKV_ERR_INVALID_ARGUMENT,
                "%s: states, kv, score, ape (16-byte aligned), pos, state_of_token, emit_row, norm, rope_table, "
                "out_rows and d_status are required", what);
  rkv_status st = prepare_device(what);
  if (st != RKV_OK) return st;
  CmpArgs a = {};
  a.ratio = ratio;
  a.coff = coff_of(ratio);
  a.cr = a.coff * ratio;
  a.width = a.coff * kIdxDim;
  a.hd = kIdxDim;
  a.out_rows = out_rows;
  a.n_out_rows = n_out_rows;
  a.states = states;
  a.n_states = n_states;
  a.n_tok = n_tok;
  a.rope_rows = rope_rows;
  a.kv = kv;
  a.score = score;
  a.pos = pos;
  a.state_of = state_of_token;
  a.emit_slot = emit_row;
  a.ape = ape;
  a.norm = norm;
  a.rope = rope_table;
  a.status = d_status;
  const ExpConsts K = exp_host()->K;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  cudaLaunchConfig_t cfg = {};
  cfg.stream = (cudaStream_t)stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  // 1. emissions (one 128-thread CTA per token group, many per SM) and the
  // ring writes allowed alongside them; 2. the deferred ring writes
  const int64_t groups = (n_tok + ratio - 1) / ratio;
  const int64_t emit_cap = (int64_t)sms * 8;
  cfg.gridDim = dim3((unsigned)(groups < emit_cap ? groups : emit_cap));
  cfg.blockDim = dim3(kIdxDim);
  cudaError_t e = cudaLaunchKernelEx(&cfg, indexer_emit_kernel, a, K);
  if (e != cudaSuccess) return fail(RKV_ERR_CUDA, "%s: launch failed: %s", what, cudaGetErrorString(e));
  const int64_t ring_need = (n_tok + 32 * kRingWarps - 1) / (32 * kRingWarps), ring_cap = (int64_t)sms * 2;
  cfg.gridDim = dim3((unsigned)(ring_need < ring_cap ? ring_need : ring_cap));
  cfg.blockDim = dim3(kRingWarps * 32);
  e = cudaLaunchKernelEx(&cfg, compress_ring_kernel, a);
  if (e != cudaSuccess) return fail(RKV_ERR_CUDA, "%s: launch failed: %s", what, cudaGetErrorString(e));
  return check_launch(what);
}
