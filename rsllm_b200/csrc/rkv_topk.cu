// rkv_topk.cu -- indexer top-k selection over f32 scores.
//
// Output contract = crates/rsllm-kvcache/src/dsv4/indexer.rs:218-236 (the
// repeated strict-`>` best scan): descending score, ties to the lowest index,
// NaN / -inf never selected, index 0 repeated when too few candidates beat
// -inf.  The scan is O(k*n); this kernel computes the same list by radix
// selection.
//
// One 1024-thread CTA per query.  Scores map to order-preserving u32 keys
// (0 = cannot win; -0.0 folded into +0.0 because `>` ties them).  Pass 1
// histograms the top 11 key bits over the query's scores; the bin holding
// rank effective_k (counted from the top) is found by a block suffix scan.
// When every key at or above that bin fits the 8192-entry candidate buffer
// (the usual case: ~3k entries for N(0,1) scores with k=2048 of 131072) one
// more pass collects them; otherwise the bin is refined by the next 11 and
// then 10 bits.  If all 32 bits are resolved with too many equal keys, the
// lowest-index equal keys are taken in index order with a block scan.  The
// candidates (key << 32 | ~index) are bitonic-sorted in shared memory and the
// first effective_k written out.  Scores are read from global memory; the
// second read of a query's 512 KB mostly hits L2.
#include "rkv_common.cuh"
#include "rkv_host.h"

namespace rkv {

constexpr int kTopkThreads = 1024;
constexpr int kTopkMaxK = 4096;
constexpr int kCandCap = 8192;

struct TopkSmem {
  uint32_t hist[2048];
  unsigned long long cand[kCandCap];
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
__device__ __forceinline__ void for_each_key(const float* __restrict__ row, int n, bool vec, F&& f) {
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

__global__ void __launch_bounds__(kTopkThreads)
topk_select_kernel(const float* __restrict__ scores, int64_t ld, const int32_t* __restrict__ n_visible, int k,
                   int32_t* __restrict__ out, bool vec) {
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
  const uint32_t m = sm.n_cand;
  uint32_t P = 1u;
  while (P < m) P <<= 1;
  for (uint32_t i = m + tid; i < P; i += kTopkThreads) sm.cand[i] = 0ull;
  __syncthreads();
  for (uint32_t size = 2; size <= P; size <<= 1) {
    for (uint32_t stride = size >> 1; stride > 0; stride >>= 1) {
      for (uint32_t t = tid; t < (P >> 1); t += kTopkThreads) {
        const uint32_t lo = 2 * t - (t & (stride - 1)), hi = lo + stride;
        const bool desc = (lo & size) == 0;
        const unsigned long long a = sm.cand[lo], c = sm.cand[hi];
        if ((a < c) == desc) {
          sm.cand[lo] = c;
          sm.cand[hi] = a;
        }
      }
      __syncthreads();
    }
  }
  const uint32_t nsel = quirk ? n_real : (uint32_t)kk;
  for (uint32_t i = tid; i < (uint32_t)kk; i += kTopkThreads)
    o[i] = i < nsel ? (int32_t)(0xffffffffu - (uint32_t)(sm.cand[i] & 0xffffffffull)) : 0;
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
  const bool vec = aligned(scores, 16) && (ld % 4) == 0;
  static_assert(sizeof(TopkSmem) <= 227 * 1024, "shared memory");
  const int smem = (int)sizeof(TopkSmem);
  cudaError_t e = cudaFuncSetAttribute(topk_select_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return fail(RKV_ERR_CUDA, "rkv_topk_select_f32: %s", cudaGetErrorString(e));
  topk_select_kernel<<<(unsigned)n_q, kTopkThreads, smem, (cudaStream_t)stream>>>(scores, ld, n_visible, k, out_idx,
                                                                                 vec);
  return check_launch("rkv_topk_select_f32");
}
