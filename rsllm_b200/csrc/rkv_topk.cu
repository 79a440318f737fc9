// rkv_topk.cu -- indexer top-k selection over f32 scores.
//
// Output contract = crates/rsllm-kvcache/src/dsv4/indexer.rs:218-236 (the
// repeated strict-`>` best scan): descending score, ties to the lowest index,
// NaN / -inf never selected, index 0 repeated when too few candidates beat
// -inf.  The scan is O(k*n); this kernel produces the same list in one pass
// over the scores in the common case.
//
// One 1024-thread CTA per query.  Scores map to order-preserving u32 keys
// (0 = cannot win; -0.0 folded into +0.0 because `>` ties them), so "key >= t"
// is "score >= float(t)".
//  * n <= 8192: every key goes to the shared-memory candidate buffer.
//  * Otherwise a 4096-key sample (32 contiguous chunks of 128) gives a
//    threshold t, the sample's r-th largest key with r chosen so that about
//    1.5 * effective_k scores are expected at or above it.  One pass over the
//    scores appends every score >= t to the candidate buffer (8192 entries,
//    warp-aggregated).  If that set holds at least effective_k and fits, it
//    contains the exact top-k (the k-th largest score is >= t), ties included.
//  * Otherwise (a skewed sample, or fewer than effective_k scores beat -inf)
//    an exact radix selection runs: 11 + 11 + 10-bit histogram passes until
//    the keys at or above the selected bin fit, then a collection pass; keys
//    equal to a fully resolved threshold are taken lowest index first.
// The candidates (key << 32 | ~index) are bitonic-sorted in shared memory and
// the first effective_k indices written.
#include "rkv_common.cuh"
#include "rkv_host.h"

namespace rkv {

constexpr int kTopkThreads = 1024;
constexpr int kTopkMaxK = 4096;
constexpr int kCandCap = 8192;
constexpr int kSampleChunk = 128;                            // keys per chunk: one float4 per lane
constexpr int kSample = (kTopkThreads / 32) * kSampleChunk;  // 4096, one chunk per warp

struct TopkSmem {
  uint32_t hist[2048];
  unsigned long long cand[kCandCap];
  uint32_t sample[kSample];
  uint32_t warp_sums[32];
  uint32_t sel_bin, sel_above, n_cand;
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

// Finds the bin b (of nbins) with above(b) < rank <= above(b) + hist[b],
// above(b) = sum of hist over bins > b.  Thread t owns bins nbins-1-2t and
// nbins-2-2t.  Result in sm.sel_bin / sm.sel_above (valid after a barrier).
__device__ void select_bin(TopkSmem& sm, int nbins, uint32_t rank) {
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  const int b0 = nbins - 1 - 2 * tid, b1 = b0 - 1;
  const uint32_t h0 = b0 >= 0 ? sm.hist[b0] : 0u, h1 = b1 >= 0 ? sm.hist[b1] : 0u;
  uint32_t v = h0 + h1, incl = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t y = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += y;
  }
  if (lane == 31) sm.warp_sums[w] = incl;
  __syncthreads();
  if (w == 0) {
    uint32_t s = sm.warp_sums[lane], si = s;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t y = __shfl_up_sync(0xffffffffu, si, o);
      if (lane >= o) si += y;
    }
    sm.warp_sums[lane] = si - s;  // exclusive
  }
  __syncthreads();
  const uint32_t above0 = sm.warp_sums[w] + incl - v;
  if (b0 >= 0 && above0 < rank && rank <= above0 + h0) {
    sm.sel_bin = (uint32_t)b0;
    sm.sel_above = above0;
  }
  const uint32_t above1 = above0 + h0;
  if (b1 >= 0 && above1 < rank && rank <= above1 + h1) {
    sm.sel_bin = (uint32_t)b1;
    sm.sel_above = above1;
  }
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
  for (int i = 0; i < kTopkThreads / 32; ++i) {
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

// The rank-th largest of `count` keys held in shared memory (rank >= 1), or 0
// when fewer than `rank` of them can win.  Three histogram passes (11, 11, 10
// bits); key(i) reads the i-th key.
template <class KeyAt>
__device__ uint32_t smem_select(TopkSmem& sm, int count, uint32_t rank, KeyAt key) {
  const int tid = threadIdx.x;
  uint32_t prefix = 0u, pmask = 0u;
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
    if (pass == 0 && (uint32_t)count - sm.hist[0] < rank) return 0u;  // bin 0 holds only keys that cannot win
    select_bin(sm, (int)dmask + 1, rank);
    __syncthreads();
    const uint32_t b = sm.sel_bin, above = sm.sel_above;
    __syncthreads();
    rank -= above;
    prefix |= b << shift;
    pmask |= dmask << shift;
  }
  return prefix;
}

// One compare-exchange stage of a descending bitonic sort on the 64-element
// segment a warp holds in registers (e0 = element base + lane, e1 = element
// base + lane + 32), for merge size `size` and stride < 64.
__device__ __forceinline__ void reg_stage(unsigned long long& e0, unsigned long long& e1, uint32_t base,
                                          uint32_t size, uint32_t stride, int lane) {
  if (stride == 32) {
    const bool desc = ((base + lane) & size) == 0;
    if ((e0 < e1) == desc) {
      const unsigned long long t = e0;
      e0 = e1;
      e1 = t;
    }
    return;
  }
  const bool lower = (lane & stride) == 0;
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    unsigned long long& e = h ? e1 : e0;
    const unsigned long long p = __shfl_xor_sync(0xffffffffu, e, stride);
    const uint32_t i_lo = (base + lane + 32 * h) & ~stride;
    const bool desc = (i_lo & size) == 0;
    const bool take_max = lower == desc;
    e = take_max ? (e > p ? e : p) : (e < p ? e : p);
  }
}

// Descending bitonic sort of a[0..P), P a power of two in [64, 8192], by the
// whole block: strides >= 64 go through shared memory with a barrier, the
// six strides below 64 run on 64-element segments in registers (warp
// shuffles), so a sort of 2048 needs 15 block barriers instead of 66.
__device__ void bitonic_sort_desc(unsigned long long* a, uint32_t P) {
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  const uint32_t nseg = P >> 6;
  for (uint32_t seg = w; seg < nseg; seg += kTopkThreads / 32) {
    unsigned long long e0 = a[seg * 64 + lane], e1 = a[seg * 64 + lane + 32];
    for (uint32_t size = 2; size <= 64; size <<= 1)
      for (uint32_t stride = size >> 1; stride > 0; stride >>= 1) reg_stage(e0, e1, seg * 64, size, stride, lane);
    a[seg * 64 + lane] = e0;
    a[seg * 64 + lane + 32] = e1;
  }
  __syncthreads();
  for (uint32_t size = 128; size <= P; size <<= 1) {
    for (uint32_t stride = size >> 1; stride >= 64; stride >>= 1) {
      for (uint32_t t = tid; t < (P >> 1); t += kTopkThreads) {
        const uint32_t lo = 2 * t - (t & (stride - 1)), hi = lo + stride;
        const bool desc = (lo & size) == 0;
        const unsigned long long x = a[lo], y = a[hi];
        if ((x < y) == desc) {
          a[lo] = y;
          a[hi] = x;
        }
      }
      __syncthreads();
    }
    for (uint32_t seg = w; seg < nseg; seg += kTopkThreads / 32) {
      unsigned long long e0 = a[seg * 64 + lane], e1 = a[seg * 64 + lane + 32];
      for (uint32_t stride = 32; stride > 0; stride >>= 1) reg_stage(e0, e1, seg * 64, size, stride, lane);
      a[seg * 64 + lane] = e0;
      a[seg * 64 + lane + 32] = e1;
    }
    __syncthreads();
  }
}

// Appends (key, index) of every score >= thr to the candidate buffer, warp
// by warp; sm.n_cand counts all matches (even past the cap).  kVec: 2 = the
// row is 32-byte aligned (256-bit loads), 1 = 16-byte aligned, 0 = scalar.
template <int kVec>
__device__ __forceinline__ void collect_at_least(TopkSmem& sm, const float* __restrict__ row, int n, float thr) {
  const unsigned FULL = 0xffffffffu;
  const int lane = threadIdx.x & 31;
  const int tid = threadIdx.x;
  // 8 consecutive scores per lane per round
  const int n8 = kVec ? (n >> 3) : 0;
  for (int base = 0; base < n8; base += kTopkThreads) {  // uniform trip count for the warp-wide scan
    const int c8 = base + tid;
    float v[8];
    if (c8 < n8) {
      if (kVec == 2) {
        uint32_t w[8];
        ld_stream32(row + (size_t)c8 * 8, w);
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] = __uint_as_float(w[j]);
      } else {
        const float4 a = __ldg(reinterpret_cast<const float4*>(row) + 2 * c8);
        const float4 b = __ldg(reinterpret_cast<const float4*>(row) + 2 * c8 + 1);
        v[0] = a.x, v[1] = a.y, v[2] = a.z, v[3] = a.w, v[4] = b.x, v[5] = b.y, v[6] = b.z, v[7] = b.w;
      }
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = -INFINITY;
    }
    uint32_t c = 0;
#pragma unroll
    for (int j = 0; j < 8; ++j) c += v[j] >= thr ? 1u : 0u;
    uint32_t incl = c;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t y = __shfl_up_sync(FULL, incl, o);
      if (lane >= o) incl += y;
    }
    const uint32_t tot = __shfl_sync(FULL, incl, 31);
    if (tot) {
      uint32_t pos = 0;
      if (lane == 31) pos = atomicAdd(&sm.n_cand, tot);
      pos = __shfl_sync(FULL, pos, 31) + incl - c;
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (v[j] >= thr) {
          if (pos < (uint32_t)kCandCap) sm.cand[pos] = composite(topk_key(v[j]), (uint32_t)(c8 * 8 + j));
          ++pos;
        }
    }
  }
  for (int i = n8 * 8 + tid; i < n; i += kTopkThreads) {
    const float v = __ldg(row + i);
    if (v >= thr) {
      const uint32_t pos = atomicAdd(&sm.n_cand, 1u);
      if (pos < (uint32_t)kCandCap) sm.cand[pos] = composite(topk_key(v), (uint32_t)i);
    }
  }
}

__global__ void __launch_bounds__(kTopkThreads)
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
  } else {
    // sample of kSample keys: chunk w of 128 consecutive scores
    const int w = tid >> 5, lane = tid & 31;
    int64_t c0 = (int64_t)w * (n - kSampleChunk) / (kTopkThreads / 32 - 1);
    if (vec) c0 &= ~(int64_t)3;
    if (vec) {
      const float4 v = __ldg(reinterpret_cast<const float4*>(row + c0) + lane);
      sm.sample[w * kSampleChunk + lane * 4 + 0] = topk_key(v.x);
      sm.sample[w * kSampleChunk + lane * 4 + 1] = topk_key(v.y);
      sm.sample[w * kSampleChunk + lane * 4 + 2] = topk_key(v.z);
      sm.sample[w * kSampleChunk + lane * 4 + 3] = topk_key(v.w);
    } else {
      for (int j = 0; j < 4; ++j) sm.sample[w * kSampleChunk + lane * 4 + j] = topk_key(__ldg(row + c0 + lane * 4 + j));
    }
    __syncthreads();
    // about 1.5 * kk scores expected at or above the threshold
    const double want = 1.5 * (double)kk;
    uint32_t rank = (uint32_t)(want * kSample / (double)n + 0.5);
    rank = max(1u, min(rank, (uint32_t)kSample));
    const uint32_t t = smem_select(sm, kSample, rank, [&](int i) { return sm.sample[i]; });
    if (t != 0u) {
      if (tid == 0) sm.n_cand = 0u;
      __syncthreads();
      const float thr = key_to_float(t);
      if (vec == 2) collect_at_least<2>(sm, row, n, thr);
      else if (vec == 1) collect_at_least<1>(sm, row, n, thr);
      else collect_at_least<0>(sm, row, n, thr);
      __syncthreads();
      const uint32_t got = sm.n_cand;
      done = got >= (uint32_t)kk && got <= (uint32_t)kCandCap;
      __syncthreads();
    }
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
  if (m > 2048u && nsel <= 2048u) {
    // Cut the candidates to the keys >= the nsel-th largest key (all of its
    // ties kept, the sort orders them by index): normally exactly nsel.
    const uint32_t kth = smem_select(sm, (int)m, nsel, [&](int i) { return (uint32_t)(cand[i] >> 32); });
    unsigned long long* dst = reinterpret_cast<unsigned long long*>(sm.sample);  // 2048 entries
    if (tid == 0) sm.n_cand = 0u;
    __syncthreads();
    for (uint32_t i = tid; i < m; i += kTopkThreads) {
      const unsigned long long c = cand[i];
      if ((uint32_t)(c >> 32) >= kth) {
        const uint32_t pos = atomicAdd(&sm.n_cand, 1u);
        if (pos < 2048u) dst[pos] = c;
      }
    }
    __syncthreads();
    if (sm.n_cand <= 2048u) {
      cand = dst;
      m = sm.n_cand;
    }
    __syncthreads();
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
  if (k > kTopkMaxK) return fail(RKV_ERR_SHAPE_MISMATCH, "rkv_topk_select_f32: k %d > %d", k, kTopkMaxK);
  if (n_keys_max > ld) return fail(RKV_ERR_SHAPE_MISMATCH, "rkv_topk_select_f32: n_keys_max > ld");
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
  topk_select_kernel<<<(unsigned)n_q, kTopkThreads, smem, (cudaStream_t)stream>>>(scores, ld, n_visible, k, out_idx,
                                                                                 vec);
  return check_launch("rkv_topk_select_f32");
}
