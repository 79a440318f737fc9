// rkv_topk.cu -- indexer top-k selection over f32 scores.
//
// Output contract = crates/rsllm-kvcache/src/dsv4/indexer.rs:218-236 (the
// repeated strict-`>` best scan): descending score, ties to the lowest index,
// NaN / -inf never selected, index 0 repeated when too few candidates beat
// -inf.  The scan is O(k*n); this kernel produces the same list in one pass
// over the scores in the common case.
//
// One 512-thread CTA per query, two per SM.  Scores map to order-preserving u32 keys
// (0 = cannot win; -0.0 folded into +0.0 because `>` ties them), so "key >= t"
// is "score >= float(t)".
//  * n <= 8192: every key goes to the shared-memory candidate buffer.
//  * Otherwise a 2048-key sample (16 contiguous chunks of 128) gives a
//    threshold t, the sample's r-th largest key, with r set from the sampling
//    error so that effective_k to ~1.7 effective_k scores are expected at or
//    above it; a separate light kernel (128-thread CTAs, the sample in
//    registers) picks every query's t before the selection kernel runs, so
//    the selection streams its row from the start.  One pass over the
//    scores appends every score >= t to the candidate buffer (8192 entries,
//    warp-aggregated).  If that set holds at least effective_k and fits, it
//    contains the exact top-k (the k-th largest score is >= t, whatever t
//    is), ties included.
//  * Otherwise (a skewed sample, or fewer than effective_k scores beat -inf)
//    an exact radix selection runs: 11 + 11 + 10-bit histogram passes until
//    the keys at or above the selected bin fit, then a collection pass; keys
//    equal to a fully resolved threshold are taken lowest index first.
// The candidates (key << 32 | ~index) are cut to the keys >= the
// effective_k-th largest by one more radix selection in shared memory,
// bitonic-sorted (register stages for strides below 64) and the first
// effective_k indices written.
#include "rkv_common.cuh"
#include "rkv_host.h"

namespace rkv {

constexpr int kTopkThreads = 512;  // two CTAs per SM, 64 registers per thread
constexpr int kTopkWarps = kTopkThreads / 32;
constexpr int kTopkMaxK = 4096;
constexpr int kCandCap = 8192;
constexpr int kCutCap = 2048;           // cut + bitonic path (sorts at most 2048)
constexpr int kBucketBins = 2048;
constexpr uint32_t kBucketMax = 32;     // bucket sort: largest bucket sorted by one thread
constexpr int kSortedCap = kTopkMaxK + kBucketMax;
constexpr int kSampleChunk = 128;                         // keys per chunk: one float4 per lane
constexpr int kSampleChunks = 16;
constexpr int kSample = kSampleChunks * kSampleChunk;     // 2048
#ifndef RKV_TOPK_PREFETCH_ROUNDS
#define RKV_TOPK_PREFETCH_ROUNDS 2
#endif
constexpr int kPrefetchRounds = RKV_TOPK_PREFETCH_ROUNDS;  // collection rounds prefetched ahead

struct TopkSmem {
  uint32_t hist[2048];
  unsigned long long cand[kCandCap];
  unsigned long long cut[kSortedCap];  // cut output (<= 2048) or bucket-sorted output (<= k + 32)
  uint32_t keep[kBucketBins / 32];
  uint32_t warp_sums[32];
  uint32_t sel_bin, sel_above, n_cand, flag, kept_end;
};

__device__ __forceinline__ uint32_t topk_key(float s) {
  if (!(s > -INFINITY)) return 0u;
  const uint32_t b = __float_as_uint(s == 0.0f ? 0.0f : s);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

__device__ __forceinline__ unsigned long long composite(uint32_t key, uint32_t idx) {
  return ((unsigned long long)key << 32) | (unsigned long long)(0xffffffffu - idx);
}

// Calls f(key, index) for every visible score of the row, block-strided.
template <class F>
__device__ __forceinline__ void for_each_key(const float* __restrict__ row, int n, int vec, F&& f) {
  if (vec) {
    const float4* r4 = reinterpret_cast<const float4*>(row);
    const int n4 = n >> 2;
    for (int i = threadIdx.x; i < n4; i += kTopkThreads) {
      const float4 v = __ldg(r4 + i);
      f(topk_key(v.x), 4 * i);
      f(topk_key(v.y), 4 * i + 1);
      f(topk_key(v.z), 4 * i + 2);
      f(topk_key(v.w), 4 * i + 3);
    }
    for (int i = (n4 << 2) + threadIdx.x; i < n; i += kTopkThreads) f(topk_key(__ldg(row + i)), i);
  } else {
    for (int i = threadIdx.x; i < n; i += kTopkThreads) f(topk_key(__ldg(row + i)), i);
  }
}

// Finds the bin b (of nbins <= 2048) with above(b) < rank <= above(b) +
// hist[b], above(b) = sum of hist over bins > b, with NT threads: thread t
// owns the 2048/NT bins counted down from nbins-1-t*(2048/NT).  Result in
// *sel_bin / *sel_above (valid after a barrier).
template <int NT>
__device__ void select_bin_t(const uint32_t* hist, uint32_t* warp_sums, int nbins, uint32_t rank, uint32_t* sel_bin,
                             uint32_t* sel_above) {
  constexpr int kPer = 2048 / NT, kWarps = NT / 32;
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  const int top = nbins - 1 - tid * kPer;
  uint32_t h[kPer], v = 0;
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    h[j] = top - j >= 0 ? hist[top - j] : 0u;
    v += h[j];
  }
  uint32_t incl = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t y = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += y;
  }
  if (lane == 31) warp_sums[w] = incl;
  __syncthreads();
  if (w == 0) {
    uint32_t x = lane < kWarps ? warp_sums[lane] : 0u, xi = x;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t y = __shfl_up_sync(0xffffffffu, xi, o);
      if (lane >= o) xi += y;
    }
    if (lane < kWarps) warp_sums[lane] = xi - x;  // exclusive
  }
  __syncthreads();
  uint32_t above = warp_sums[w] + incl - v;
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    if (top - j >= 0 && above < rank && rank <= above + h[j]) {
      *sel_bin = (uint32_t)(top - j);
      *sel_above = above;
    }
    above += h[j];
  }
}

__device__ __forceinline__ void select_bin(TopkSmem& sm, int nbins, uint32_t rank) {
  select_bin_t<kTopkThreads>(sm.hist, sm.warp_sums, nbins, rank, &sm.sel_bin, &sm.sel_above);
}

// Exclusive block scan of a 0/1 flag; returns the position, total in *total.
__device__ __forceinline__ uint32_t block_scan_flag(TopkSmem& sm, bool flag, uint32_t* total) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const unsigned bal = __ballot_sync(0xffffffffu, flag);
  const uint32_t in_warp = __popc(bal & ((1u << lane) - 1u));
  __syncthreads();  // warp_sums may still be read by the previous round
  if (lane == 0) sm.warp_sums[w] = __popc(bal);
  __syncthreads();
  uint32_t before = 0, all = 0;
  for (int i = 0; i < kTopkWarps; ++i) {
    const uint32_t c = sm.warp_sums[i];
    before += i < w ? c : 0u;
    all += c;
  }
  *total = all;
  return before + in_warp;
}

__device__ __forceinline__ float key_to_float(uint32_t key) {
  return __uint_as_float((key & 0x80000000u) ? (key & 0x7fffffffu) : ~key);
}

// Radix selection over `count` keys in shared memory (key(i) reads the
// i-th): the lower bound of the narrowest bin (11, then 11, then 10 bits)
// holding the rank-th largest key (rank >= 1), stopping once the keys at or
// above the bin number at most `fit`; after three passes the bound is the
// rank-th largest key itself.  *n_at_least = keys >= the returned bound.
template <class KeyAt>
__device__ uint32_t smem_select(TopkSmem& sm, int count, uint32_t rank, uint32_t fit, uint32_t* n_at_least,
                                KeyAt key) {
  const int tid = threadIdx.x;
  uint32_t prefix = 0u, pmask = 0u, above_total = 0u, in_bin = (uint32_t)count;
  for (int pass = 0; pass < 3; ++pass) {
    const int shift = pass == 0 ? 21 : (pass == 1 ? 10 : 0);
    const uint32_t dmask = pass == 2 ? 0x3ffu : 0x7ffu;
    for (int b = tid; b < 2048; b += kTopkThreads) sm.hist[b] = 0u;
    __syncthreads();
    for (int i = tid; i < count; i += kTopkThreads) {
      const uint32_t x = key(i);
      if ((x & pmask) == prefix) atomicAdd(&sm.hist[(x >> shift) & dmask], 1u);
    }
    __syncthreads();
    select_bin(sm, (int)dmask + 1, rank);
    __syncthreads();
    const uint32_t b = sm.sel_bin, above = sm.sel_above;
    in_bin = sm.hist[b];
    __syncthreads();
    rank -= above;
    above_total += above;
    prefix |= b << shift;
    pmask |= dmask << shift;
    if (above_total + in_bin <= fit) break;
  }
  *n_at_least = above_total + in_bin;
  return prefix;
}

// The sample rank: expected scores at or above the sample's rank-th largest
// key are rank * n / kSample, with a relative spread of about 1/sqrt(rank).
// rank = q + 3.5 sqrt(q) + 2 (q = kk * kSample / n) keeps the count >= kk in
// all but ~0.1% of rows and far under the 8192-entry buffer for k <= 2048.
__device__ __forceinline__ uint32_t sample_rank(int kk, int n) {
  const float q = (float)kk * (float)kSample / (float)n;
  const uint32_t rank = (uint32_t)ceilf(q + 3.5f * sqrtf(q) + 2.0f);
  return max(1u, min(rank, (uint32_t)kSample));
}

// Start of sample chunk c (of kSampleChunks, 128 consecutive scores each,
// spread evenly over the row; 4-aligned when the row is vectorised).
__device__ __forceinline__ int64_t sample_chunk_start(int c, int n, int vec) {
  int64_t c0 = (int64_t)c * (n - kSampleChunk) / (kSampleChunks - 1);
  return vec ? (c0 & ~(int64_t)3) : c0;
}

// The rank-th largest of the kSample sample keys, PER of them in each of
// the NT threads' registers, to its top 16 bits (the lower bound of the
// 2^16-key bin that holds it), by a bitwise search from the top bit down: bit
// b is set when at least `rank` sample keys are >= the prefix with it set.
// One count (a warp reduction and a barrier) per bit, no shared-memory
// atomics.  16 bits keep the sign, exponent and 7 mantissa bits of the score:
// the bin adds well under 1% to the expected count at or above it.  Returns
// 0 when fewer than `rank` sample keys can win (key 0).
template <int NT, int PER>
__device__ uint32_t sample_kth_largest(const uint32_t (&keys)[PER], uint32_t rank, uint32_t (*part)[NT / 32]) {
  static_assert(NT * PER == kSample, "sample size");
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  auto count_ge = [&](uint32_t x, int slot) {
    uint32_t c = 0;
#pragma unroll
    for (int j = 0; j < PER; ++j) c += keys[j] >= x ? 1u : 0u;
    c = __reduce_add_sync(0xffffffffu, c);
    if (lane == 0) part[slot][w] = c;
    __syncthreads();
    uint32_t all = 0;
#pragma unroll
    for (int i = 0; i < NT / 32; ++i) all += part[slot][i];
    return all;
  };
  if (count_ge(1u, 1) < rank) return 0u;  // slot 1; bit 31 uses slot 0, bit 30 slot 1, ...
  uint32_t prefix = 0u;
#pragma unroll 1
  for (int bit = 31; bit >= 16; --bit) {
    const uint32_t cand = prefix | (1u << bit);
    if (count_ge(cand, (bit & 1) ^ 1) >= rank) prefix = cand;  // two slots: a slot is rewritten two counts later
  }
  return prefix;
}

// Per query with more than kCandCap visible scores: the collection threshold
// (the sample's rank-th largest key, 0 when the sample cannot supply one)
// written to out[q * k] -- the first entry of the query's own output row,
// which topk_select_kernel reads before it writes any output.  One 128-thread
// CTA per query, 16 sample keys per thread in registers; many CTAs per SM, so
// a layer's queries take their latency-bound sample phases in about one wave
// instead of inside the streaming kernel.
constexpr int kThrThreads = 128;
constexpr int kThrPerThread = kSample / kThrThreads;  // 16

__global__ void __launch_bounds__(kThrThreads)
topk_threshold_kernel(const float* __restrict__ scores, int64_t ld, const int32_t* __restrict__ n_visible, int k,
                      int32_t* __restrict__ out, int vec) {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  __shared__ uint32_t part[2][kThrThreads / 32];
  const int q = blockIdx.x;
  const int n = max(0, __ldg(n_visible + q));
  const int kk = min(k, n);
  if (n <= kCandCap || kk == 0) return;
  const float* row = scores + (int64_t)q * ld;
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  uint32_t skeys[kThrPerThread];
  constexpr int kChunksPerWarp = kSampleChunks / (kThrThreads / 32);  // 4
#pragma unroll
  for (int c = 0; c < kChunksPerWarp; ++c) {
    const int64_t c0 = sample_chunk_start(w * kChunksPerWarp + c, n, vec);
    if (vec) {
      const float4 v = __ldg(reinterpret_cast<const float4*>(row + c0) + lane);
      skeys[4 * c] = topk_key(v.x), skeys[4 * c + 1] = topk_key(v.y);
      skeys[4 * c + 2] = topk_key(v.z), skeys[4 * c + 3] = topk_key(v.w);
    } else {
#pragma unroll
      for (int j = 0; j < 4; ++j) skeys[4 * c + j] = topk_key(__ldg(row + c0 + lane * 4 + j));
    }
  }
  const uint32_t t = sample_kth_largest<kThrThreads, kThrPerThread>(skeys, sample_rank(kk, n), part);
  if (threadIdx.x == 0) out[(int64_t)q * k] = (int32_t)t;
}

// One compare-exchange stage of a descending bitonic sort on the 64-element
// segment a warp holds in registers (e0 = element base + lane, e1 = element
// base + lane + 32), for merge size kSize and stride kStride < 64.
template <uint32_t kSize, uint32_t kStride>
__device__ __forceinline__ void reg_stage(unsigned long long& e0, unsigned long long& e1, uint32_t base, int lane) {
  if (kStride == 32) {
    const bool desc = ((base + lane) & kSize) == 0;
    if ((e0 < e1) == desc) {
      const unsigned long long t = e0;
      e0 = e1;
      e1 = t;
    }
    return;
  }
  const bool lower = (lane & kStride) == 0;
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    unsigned long long& e = h ? e1 : e0;
    const unsigned long long p = __shfl_xor_sync(0xffffffffu, e, kStride);
    const bool desc = (((base + lane + 32 * h) & ~kStride) & kSize) == 0;
    const bool take_max = lower == desc;
    e = take_max ? (e > p ? e : p) : (e < p ? e : p);
  }
}

template <uint32_t kSize, uint32_t kStride>
__device__ __forceinline__ void reg_stages_down(unsigned long long& e0, unsigned long long& e1, uint32_t base,
                                                int lane) {
  reg_stage<kSize, kStride>(e0, e1, base, lane);
  if constexpr (kStride > 1) reg_stages_down<kSize, kStride / 2>(e0, e1, base, lane);
}

template <uint32_t kSize>
__device__ __forceinline__ void reg_sort64(unsigned long long& e0, unsigned long long& e1, uint32_t base, int lane) {
  if constexpr (kSize > 2) reg_sort64<kSize / 2>(e0, e1, base, lane);
  reg_stages_down<kSize, kSize / 2>(e0, e1, base, lane);
}

template <uint32_t P, uint32_t kSize>
__device__ __forceinline__ void merge_level(unsigned long long* a) {
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
#pragma unroll
  for (uint32_t stride = kSize >> 1; stride >= 64; stride >>= 1) {
    for (uint32_t t = tid; t < (P >> 1); t += kTopkThreads) {
      const uint32_t lo = 2 * t - (t & (stride - 1)), hi = lo + stride;
      const bool desc = (lo & kSize) == 0;
      const unsigned long long x = a[lo], y = a[hi];
      if ((x < y) == desc) {
        a[lo] = y;
        a[hi] = x;
      }
    }
    __syncthreads();
  }
  for (uint32_t seg = w; seg < (P >> 6); seg += kTopkWarps) {
    unsigned long long e0 = a[seg * 64 + lane], e1 = a[seg * 64 + lane + 32];
    reg_stages_down<kSize, 32>(e0, e1, seg * 64, lane);
    a[seg * 64 + lane] = e0;
    a[seg * 64 + lane + 32] = e1;
  }
  __syncthreads();
  if constexpr (kSize < P) merge_level<P, kSize * 2>(a);
}

// Descending bitonic sort of a[0..P) by the whole block, P a power of two in
// [64, 8192], fully unrolled: strides >= 64 go through shared memory with a
// barrier, the six strides below 64 run on 64-element segments in registers
// (warp shuffles); a sort of 2048 needs 20 block barriers instead of 66.
template <uint32_t P>
__device__ void bitonic_sort_desc_t(unsigned long long* a) {
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  for (uint32_t seg = w; seg < (P >> 6); seg += kTopkWarps) {
    unsigned long long e0 = a[seg * 64 + lane], e1 = a[seg * 64 + lane + 32];
    reg_sort64<64>(e0, e1, seg * 64, lane);
    a[seg * 64 + lane] = e0;
    a[seg * 64 + lane + 32] = e1;
  }
  __syncthreads();
  if constexpr (P > 64) merge_level<P, 128>(a);
}

__device__ void bitonic_sort_desc(unsigned long long* a, uint32_t P) {
  switch (P) {
    case 64: bitonic_sort_desc_t<64>(a); break;
    case 128: bitonic_sort_desc_t<128>(a); break;
    case 256: bitonic_sort_desc_t<256>(a); break;
    case 512: bitonic_sort_desc_t<512>(a); break;
    case 1024: bitonic_sort_desc_t<1024>(a); break;
    case 2048: bitonic_sort_desc_t<2048>(a); break;
    case 4096: bitonic_sort_desc_t<4096>(a); break;
    default: bitonic_sort_desc_t<8192>(a); break;
  }
}

// Appends every score >= thr to the candidate buffer as its (key, ~index)
// composite, warp by warp; sm.n_cand counts all matches (even past the cap).  Per round a warp
// tests 1024 consecutive scores: each lane issues all of its loads (four
// 256-bit loads when the row is 32-byte aligned, eight 128-bit loads when
// 16-byte aligned; every load instruction covers 1 KB contiguous across the
// warp) before testing them into a 32-bit mask, so 128 B per thread are in
// flight.  A warp scan of the mask counts places the matches; a match's score
// is taken from the registers that loaded it (no second read of the row).
// kVec: 2 = 32-byte aligned row, 1 = 16-byte aligned, 0 = scalar.
template <int kVec>
__device__ __forceinline__ void collect_at_least(TopkSmem& sm, const float* __restrict__ row, int n, float thr) {
  const unsigned FULL = 0xffffffffu;
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  constexpr int kWarpChunk = 1024;
  const int n_chunks = kVec ? (n / kWarpChunk) : 0;
  // uniform trip count for the warp-wide scan: every warp runs the same rounds
  for (int c0 = 0; c0 < n_chunks; c0 += kTopkWarps) {
    const int chunk = c0 + w;
    const float* base = row + (size_t)chunk * kWarpChunk;
    // the warp's chunk kPrefetchRounds rounds ahead into L2 (one 128-byte
    // line per lane; the first rounds were prefetched while the sample was
    // selected), so that the rounds' loads hit L2 instead of paying HBM latency
    if (chunk + kPrefetchRounds * kTopkWarps < n_chunks)
      asm volatile("prefetch.global.L2 [%0];" ::"l"(base + (size_t)kPrefetchRounds * kTopkWarps * kWarpChunk +
                                                         lane * 32));
    uint32_t m = 0;
    uint32_t u2[4][8], u1[8][4];
    if (chunk < n_chunks) {
      if (kVec == 2) {
#pragma unroll
        for (int q = 0; q < 4; ++q)
          asm volatile("ld.global.nc.L1::no_allocate.v8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                       : "=r"(u2[q][0]), "=r"(u2[q][1]), "=r"(u2[q][2]), "=r"(u2[q][3]), "=r"(u2[q][4]),
                         "=r"(u2[q][5]), "=r"(u2[q][6]), "=r"(u2[q][7])
                       : "l"(base + q * 256 + lane * 8));
#pragma unroll
        for (int q = 0; q < 4; ++q)
#pragma unroll
          for (int j = 0; j < 8; ++j) m |= (__uint_as_float(u2[q][j]) >= thr ? 1u : 0u) << (q * 8 + j);
      } else {
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          const float4 v = __ldg(reinterpret_cast<const float4*>(base + q * 128) + lane);
          u1[q][0] = __float_as_uint(v.x), u1[q][1] = __float_as_uint(v.y);
          u1[q][2] = __float_as_uint(v.z), u1[q][3] = __float_as_uint(v.w);
        }
#pragma unroll
        for (int q = 0; q < 8; ++q)
#pragma unroll
          for (int j = 0; j < 4; ++j) m |= (__uint_as_float(u1[q][j]) >= thr ? 1u : 0u) << (q * 4 + j);
      }
    }
    const uint32_t c = __popc(m);
    if (!__any_sync(FULL, c != 0u)) continue;
    uint32_t incl = c;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t y = __shfl_up_sync(FULL, incl, o);
      if (lane >= o) incl += y;
    }
    uint32_t pos = 0;
    if (lane == 31) pos = atomicAdd(&sm.n_cand, incl);
    pos = __shfl_sync(FULL, pos, 31) + incl - c;
    while (m) {
      const int b = __ffs(m) - 1;
      m &= m - 1;
      // bit b of lane `lane`: piece b/8 (b/4) of the lane, element b%8 (b%4);
      // its score is picked from the registers that loaded it
      const int off = kVec == 2 ? (b >> 3) * 256 + lane * 8 + (b & 7) : (b >> 2) * 128 + lane * 4 + (b & 3);
      // element b of the 32 loaded values by a 5-level select tree (31
      // selects on the bits of b; static register indices throughout)
      uint32_t t16[16], t8[8], t4[4], t2[2];
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const uint32_t e0 = kVec == 2 ? u2[(2 * i) >> 3][(2 * i) & 7] : u1[(2 * i) >> 2][(2 * i) & 3];
        const uint32_t e1 = kVec == 2 ? u2[(2 * i + 1) >> 3][(2 * i + 1) & 7] : u1[(2 * i + 1) >> 2][(2 * i + 1) & 3];
        t16[i] = (b & 1) ? e1 : e0;
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) t8[i] = (b & 2) ? t16[2 * i + 1] : t16[2 * i];
#pragma unroll
      for (int i = 0; i < 4; ++i) t4[i] = (b & 4) ? t8[2 * i + 1] : t8[2 * i];
#pragma unroll
      for (int i = 0; i < 2; ++i) t2[i] = (b & 8) ? t4[2 * i + 1] : t4[2 * i];
      const uint32_t bits = (b & 16) ? t2[1] : t2[0];
      if (pos < (uint32_t)kCandCap)
        sm.cand[pos] = composite(topk_key(__uint_as_float(bits)), (uint32_t)(chunk * kWarpChunk + off));
      ++pos;
    }
  }
  for (int i = n_chunks * kWarpChunk + threadIdx.x; i < n; i += kTopkThreads) {
    const float v = __ldg(row + i);
    if (v >= thr) {
      const uint32_t pos = atomicAdd(&sm.n_cand, 1u);
      if (pos < (uint32_t)kCandCap) sm.cand[pos] = composite(topk_key(v), (uint32_t)i);
    }
  }
}

// Exact ordering of the top `need` candidates a[0..m) by bucket sort: 2048
// buckets split the candidates' key range evenly (descending), a histogram
// and a block scan place each bucket, the buckets that start before `need`
// are scattered to out (need + kBucketMax entries), and every kept element
// goes to sorted[its bucket start + the number of its bucket mates above it]
// on the full (key, ~index) composite, so sorted[0..need) is exactly ordered.
// sorted may alias a.  Returns false (nothing written to sorted) when such a
// bucket holds more than kBucketMax entries (heavy ties); the caller then
// sorts another way.
__device__ bool bucket_sort_top(TopkSmem& sm, const unsigned long long* __restrict__ a, uint32_t m, uint32_t need,
                                unsigned long long* __restrict__ out, unsigned long long* __restrict__ sorted) {
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  uint32_t mn = 0xffffffffu, mx = 0u;
  for (uint32_t i = tid; i < m; i += kTopkThreads) {
    const uint32_t k = (uint32_t)(a[i] >> 32);
    mn = min(mn, k);
    mx = max(mx, k);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    mn = min(mn, __shfl_xor_sync(0xffffffffu, mn, o));
    mx = max(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  }
  __syncthreads();  // warp_sums may still be read by an earlier phase
  if (lane == 0) {
    sm.warp_sums[w] = mn;
    sm.warp_sums[16 + w] = mx;
  }
  for (int b = tid; b < kBucketBins; b += kTopkThreads) sm.hist[b] = 0u;
  if (tid < kBucketBins / 32) sm.keep[tid] = 0u;
  if (tid == 0) {
    sm.flag = 0u;
    sm.kept_end = 0u;
  }
  __syncthreads();
  mn = 0xffffffffu;
  mx = 0u;
  for (int i = 0; i < kTopkWarps; ++i) {
    mn = min(mn, sm.warp_sums[i]);
    mx = max(mx, sm.warp_sums[16 + i]);
  }
  const uint32_t range = mx - mn;
  int shift = 0;
  while ((range >> shift) >= (uint32_t)kBucketBins) ++shift;
  for (uint32_t i = tid; i < m; i += kTopkThreads)
    atomicAdd(&sm.hist[kBucketBins - 1 - (((uint32_t)(a[i] >> 32) - mn) >> shift)], 1u);
  __syncthreads();
  // exclusive scan of the bucket counts; thread t owns buckets B*t .. B*t+B-1
  constexpr int B = kBucketBins / kTopkThreads;
  uint32_t c[B], tot = 0;
#pragma unroll
  for (int j = 0; j < B; ++j) {
    c[j] = sm.hist[tid * B + j];
    tot += c[j];
  }
  uint32_t incl = tot;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t y = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += y;
  }
  __syncthreads();
  if (lane == 31) sm.warp_sums[w] = incl;
  __syncthreads();
  uint32_t start = incl - tot;
  for (int i = 0; i < w; ++i) start += sm.warp_sums[i];
#pragma unroll
  for (int j = 0; j < B; ++j) {
    const int b = tid * B + j;
    if (start < need) {
      atomicOr(&sm.keep[b >> 5], 1u << (b & 31));
      if (c[j] > kBucketMax) sm.flag = 1u;
      if (start + c[j] >= need) sm.kept_end = start + c[j];  // the bucket holding position need - 1
    }
    sm.hist[b] = start;
    start += c[j];
  }
  __syncthreads();
  if (sm.flag) return false;
  for (uint32_t i = tid; i < m; i += kTopkThreads) {
    const unsigned long long v = a[i];
    const int b = kBucketBins - 1 - (int)((((uint32_t)(v >> 32)) - mn) >> shift);
    const uint32_t p = atomicAdd(&sm.hist[b], 1u);
    if (sm.keep[b >> 5] >> (b & 31) & 1u) out[p] = v;
  }
  __syncthreads();
  // hist[b] now holds the end of bucket b (the start of bucket b + 1).  Each
  // kept element's final place is its bucket's start plus the number of
  // bucket mates above it (composites are distinct); written to `sorted`.
  const uint32_t kept_end = sm.kept_end;
  for (uint32_t p = tid; p < kept_end; p += kTopkThreads) {
    const unsigned long long x = out[p];
    const int b = kBucketBins - 1 - (int)((((uint32_t)(x >> 32)) - mn) >> shift);
    const uint32_t s0 = b ? sm.hist[b - 1] : 0u, e = sm.hist[b];
    uint32_t r = 0;
    for (uint32_t q = s0; q < e; ++q) r += out[q] > x ? 1u : 0u;
    sorted[s0 + r] = x;
  }
  __syncthreads();
  return true;
}


__global__ void __launch_bounds__(kTopkThreads, 2)
topk_select_kernel(const float* __restrict__ scores, int64_t ld, const int32_t* __restrict__ n_visible, int k,
                   int32_t* __restrict__ out, int vec) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  TopkSmem& sm = *reinterpret_cast<TopkSmem*>(smem_raw);
  const int tid = threadIdx.x;
  const int q = blockIdx.x;
  const float* row = scores + (int64_t)q * ld;
  const int n = max(0, __ldg(n_visible + q));
  const int kk = min(k, n);
  int32_t* o = out + (int64_t)q * k;
  // The scores are complete before topk_threshold_kernel (launched without
  // programmatic overlap) starts, so the first collection rounds go into L2
  // before waiting for its thresholds.
  if (vec && n > kCandCap) {
    const int w_ = tid >> 5;
    for (int rr = 0; rr < kPrefetchRounds; ++rr) {
      const int64_t chunk = (int64_t)rr * kTopkWarps + w_;
      if ((chunk + 1) * 1024 <= n)
        asm volatile("prefetch.global.L2 [%0];" ::"l"(row + chunk * 1024 + (tid & 31) * 32));
    }
  }
  asm volatile("griddepcontrol.wait;" ::: "memory");
  // the threshold topk_threshold_kernel left in this row's first entry
  const uint32_t t = (n > kCandCap && kk > 0) ? (uint32_t)o[0] : 0u;
  __syncthreads();  // every thread has read o[0] before any output is written
  for (int i = kk + tid; i < k; i += kTopkThreads) o[i] = -1;
  if (kk == 0) return;

  uint32_t nsel = (uint32_t)kk;  // entries of the sorted candidates to emit; the rest of kk are 0
  bool done = false;
  if (tid == 0) sm.n_cand = 0u;
  __syncthreads();
  if (n <= kCandCap) {
    // every key that can win fits the buffer
    for (int i = tid; i < n; i += kTopkThreads) {
      const uint32_t x = topk_key(__ldg(row + i));
      if (x != 0u) sm.cand[atomicAdd(&sm.n_cand, 1u)] = composite(x, (uint32_t)i);
    }
    __syncthreads();
    nsel = min(sm.n_cand, (uint32_t)kk);
    done = true;
  } else if (t != 0u) {
    const float thr = key_to_float(t);
    if (vec == 2) collect_at_least<2>(sm, row, n, thr);
    else if (vec == 1) collect_at_least<1>(sm, row, n, thr);
    else collect_at_least<0>(sm, row, n, thr);
    __syncthreads();
    const uint32_t got = sm.n_cand;
    done = got >= (uint32_t)kk && got <= (uint32_t)kCandCap;
    __syncthreads();
  }

  if (!done) {
    uint32_t prefix = 0u, pmask = 0u, remaining = (uint32_t)kk, n_real = 0u;
    bool resolved = false, quirk = false;
    for (int pass = 0; pass < 3; ++pass) {
      const int shift = pass == 0 ? 21 : (pass == 1 ? 10 : 0);
      const uint32_t dmask = pass == 2 ? 0x3ffu : 0x7ffu;
      for (int b = tid; b < 2048; b += kTopkThreads) sm.hist[b] = 0u;
      __syncthreads();
      for_each_key(row, n, vec, [&](uint32_t x, int) {
        if ((x & pmask) == prefix) atomicAdd(&sm.hist[(x >> shift) & dmask], 1u);
      });
      __syncthreads();
      if (pass == 0) {
        // Real keys are >= 0x00800000 (top digit >= 4): bin 0 holds only keys
        // that cannot win.
        n_real = (uint32_t)n - sm.hist[0];
        if (n_real < (uint32_t)kk) {
          quirk = true;
          break;
        }
      }
      select_bin(sm, (int)dmask + 1, remaining);
      __syncthreads();
      const uint32_t b = sm.sel_bin, above = sm.sel_above, in_bin = sm.hist[b];
      __syncthreads();
      remaining -= above;
      prefix |= b << shift;
      pmask |= dmask << shift;
      if (pass == 2) {
        resolved = true;
        break;
      }
      // Keys >= the bin's lower bound: above the bin (< kk of them) + the bin.
      if ((uint32_t)kk - remaining + in_bin <= (uint32_t)kCandCap) break;
    }

    if (tid == 0) sm.n_cand = 0u;
    __syncthreads();
    if (quirk) {
      for_each_key(row, n, vec, [&](uint32_t x, int i) {
        if (x != 0u) sm.cand[atomicAdd(&sm.n_cand, 1u)] = composite(x, (uint32_t)i);
      });
    } else if (!resolved) {
      for_each_key(row, n, vec, [&](uint32_t x, int i) {
        if (x >= prefix) sm.cand[atomicAdd(&sm.n_cand, 1u)] = composite(x, (uint32_t)i);
      });
    } else {
      // Threshold key T = prefix: every key > T, plus the `remaining`
      // lowest-index keys equal to T.
      const uint32_t T = prefix;
      uint32_t taken = 0u;
      for (int base = 0; base < n; base += kTopkThreads) {
        const int i = base + tid;
        const uint32_t x = i < n ? topk_key(__ldg(row + i)) : 0u;
        if (x > T) sm.cand[atomicAdd(&sm.n_cand, 1u)] = composite(x, (uint32_t)i);
        uint32_t total;
        const uint32_t pos = block_scan_flag(sm, x == T, &total);
        if (x == T && taken + pos < remaining) sm.cand[atomicAdd(&sm.n_cand, 1u)] = composite(x, (uint32_t)i);
        taken += total;
      }
    }

    __syncthreads();
    if (quirk) nsel = n_real;
  }
  __syncthreads();
  unsigned long long* cand = sm.cand;
  uint32_t m = min(sm.n_cand, (uint32_t)kCandCap);
  if (nsel > 0u && bucket_sort_top(sm, cand, m, nsel, sm.cut, cand)) {
    for (uint32_t i = tid; i < (uint32_t)kk; i += kTopkThreads)
      o[i] = i < nsel ? (int32_t)(0xffffffffu - (uint32_t)(cand[i] & 0xffffffffull)) : 0;
    return;
  }
  if (m > (uint32_t)kCutCap && nsel <= (uint32_t)kCutCap) {
    // Cut the candidates to the keys >= the nsel-th largest key (its ties
    // kept, the sort orders them by index): normally exactly nsel entries.
    uint32_t n_ge;
    const uint32_t kth =
        smem_select(sm, (int)m, nsel, (uint32_t)kCutCap, &n_ge, [&](int i) { return (uint32_t)(cand[i] >> 32); });
    if (n_ge <= (uint32_t)kCutCap) {
      if (tid == 0) sm.n_cand = 0u;
      __syncthreads();
      for (uint32_t i = tid; i < m; i += kTopkThreads) {
        const unsigned long long c = cand[i];
        if ((uint32_t)(c >> 32) >= kth) sm.cut[atomicAdd(&sm.n_cand, 1u)] = c;
      }
      __syncthreads();
      cand = sm.cut;
      m = n_ge;
    }
  }
  uint32_t P = 64u;
  while (P < m) P <<= 1;
  for (uint32_t i = m + tid; i < P; i += kTopkThreads) cand[i] = 0ull;
  __syncthreads();
  bitonic_sort_desc(cand, P);
  for (uint32_t i = tid; i < (uint32_t)kk; i += kTopkThreads)
    o[i] = i < nsel ? (int32_t)(0xffffffffu - (uint32_t)(cand[i] & 0xffffffffull)) : 0;
}

}  // namespace rkv

extern "C" rkv_status rkv_topk_select_f32(const float* scores, int64_t ld, int32_t n_q, const int32_t* n_visible,
                                          int32_t n_keys_max, int32_t k, int32_t* out_idx, rkv_stream_t stream) {
  using namespace rkv;
  if (n_q < 0 || k < 0 || ld < 0 || n_keys_max < 0)
    return fail(RKV_ERR_SHAPE_MISMATCH, "rkv_topk_select_f32: negative sizes");
  if (k > kTopkMaxK) return fail_shape("k", kTopkMaxK, k, "rkv_topk_select_f32: k %d > %d", k, kTopkMaxK);
  if (n_keys_max > ld) return fail_shape("n_keys_max", ld, n_keys_max, "rkv_topk_select_f32: n_keys_max > ld");
  if (n_q == 0 || k == 0) {
    clear_error();
    return RKV_OK;
  }
  if (!scores || !n_visible || !out_idx || !aligned(scores, 4))
    return fail(RKV_ERR_INVALID_ARGUMENT, "rkv_topk_select_f32: scores, n_visible and out_idx are required");
  const int vec = (aligned(scores, 32) && ld % 8 == 0) ? 2 : ((aligned(scores, 16) && ld % 4 == 0) ? 1 : 0);
  static_assert(sizeof(TopkSmem) <= 227 * 1024, "shared memory");
  const int smem = (int)sizeof(TopkSmem);
  cudaError_t e = cudaFuncSetAttribute(topk_select_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return fail(RKV_ERR_CUDA, "rkv_topk_select_f32: %s", cudaGetErrorString(e));
  // thresholds of the long rows first (into each row's first output entry),
  // then the selection, launched to overlap the threshold kernel's tail
  if (n_keys_max > kCandCap)
    topk_threshold_kernel<<<(unsigned)n_q, kThrThreads, 0, (cudaStream_t)stream>>>(scores, ld, n_visible, k, out_idx,
                                                                                   vec);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)n_q);
  cfg.blockDim = dim3(kTopkThreads);
  cfg.dynamicSmemBytes = (size_t)smem;
  cfg.stream = (cudaStream_t)stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = n_keys_max > kCandCap ? 1 : 0;
  e = cudaLaunchKernelEx(&cfg, topk_select_kernel, scores, ld, n_visible, (int)k, out_idx, vec);
  if (e != cudaSuccess) return fail(RKV_ERR_CUDA, "rkv_topk_select_f32: launch failed: %s", cudaGetErrorString(e));
  return check_launch("rkv_topk_select_f32");
}
