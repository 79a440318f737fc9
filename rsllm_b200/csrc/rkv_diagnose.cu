// rkv_diagnose.cu -- the data of an error a kernel detected.
//
// The kernels report a bad slot, page id, position or a non-finite row as a
// bit in a device status word and skip the row, so the hot path carries no
// per-row bookkeeping.  When a caller sees such a bit, these calls re-run the
// kernel's checks on the host, over copies of the same inputs, in the
// kernel's row order, and fill an rkv_err_info with the first failing row and
// the fields of rsLLM's error variant (IndexOutOfRange { what, idx, len },
// crates/rsllm-kvcache/src/lib.rs:28-70; NonFiniteInput(what),
// crates/rsllm-backend-cpu/src/error.rs:33).  They are for the error path:
// synchronous on `stream`, with host copies of the inputs.
#include <stdio.h>

#include <vector>

#include "rkv_common.cuh"
#include "rkv_host.h"

namespace rkv {

static rkv_status copy_back(void* dst, const void* src, size_t bytes, rkv_stream_t stream, const char* what) {
  if (bytes == 0) return RKV_OK;
  cudaError_t e = cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, (cudaStream_t)stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize((cudaStream_t)stream);
  if (e != cudaSuccess) return fail(RKV_ERR_CUDA, "%s: reading the inputs back: %s", what, cudaGetErrorString(e));
  return RKV_OK;
}

static rkv_status report(rkv_err_info* out, const rkv_err_info& info, const char* msg_fmt, long long a,
                         long long b, long long c) {
  if (out) *out = info;
  if (info.status == RKV_OK) {
    clear_error();
    return RKV_OK;
  }
  return fail_info(info, msg_fmt, a, b, c);
}

static void set_what(rkv_err_info& e, const char* what) { snprintf(e.what, sizeof(e.what), "%s", what); }

}  // namespace rkv

extern "C" rkv_status rkv_append_diagnose_bf16(const rkv_pool_view* pool, int32_t layer0, int32_t n_layers_in,
                                               const uint16_t* rows, int64_t n_tokens, const int32_t* slot_mapping,
                                               rkv_err_info* out, rkv_stream_t stream) {
  using namespace rkv;
  const char* what = "rkv_append_diagnose_bf16";
  rkv_status st = check_pool(pool, what);
  if (st != RKV_OK) return st;
  if (n_layers_in < 0 || n_tokens < 0) return fail_shape("n_tokens", 0, n_tokens, "%s: negative sizes", what);
  if (n_tokens > 0 && (!rows || !slot_mapping))
    return fail(RKV_ERR_INVALID_ARGUMENT, "%s: rows and slot_mapping are required", what);
  std::vector<int32_t> slots((size_t)n_tokens);
  st = copy_back(slots.data(), slot_mapping, slots.size() * 4, stream, what);
  if (st != RKV_OK) return st;
  const int64_t n_slots = pool->n_pages * kPageTokens;
  const int64_t chunk = 1 << 16;  // rows read back at a time
  std::vector<uint16_t> buf;
  rkv_err_info info = blank_info(RKV_OK);
  for (int64_t i = 0; i < n_layers_in && info.status == RKV_OK; ++i) {
    for (int64_t t0 = 0; t0 < n_tokens && info.status == RKV_OK; t0 += chunk) {
      const int64_t t1 = t0 + chunk < n_tokens ? t0 + chunk : n_tokens;
      buf.resize((size_t)((t1 - t0) * kRowDim));
      st = copy_back(buf.data(), rows + (i * n_tokens + t0) * kRowDim, buf.size() * 2, stream, what);
      if (st != RKV_OK) return st;
      for (int64_t t = t0; t < t1; ++t) {
        const int32_t slot = slots[(size_t)t];
        if (slot < 0) continue;  // padding token
        if (slot >= n_slots) {   // the kernel checks the slot first
          info = blank_info(RKV_ERR_INDEX_OUT_OF_RANGE);
          set_what(info, "slot_mapping");
          info.idx = slot;
          info.len = n_slots;
          info.row = i * n_tokens + t;
          break;
        }
        const uint16_t* row = buf.data() + (t - t0) * kRowDim;
        for (int l = 0; l < kLatent; ++l)
          if ((row[l] & 0x7fffu) >= 0x7f80u) {  // inf or NaN in a latent lane
            info = blank_info(RKV_ERR_NON_FINITE_INPUT);
            set_what(info, "rows");
            info.idx = l;
            info.row = i * n_tokens + t;
            break;
          }
        if (info.status != RKV_OK) break;
      }
    }
  }
  (void)layer0;
  return report(out, info, "rkv_append_diagnose_bf16: first failing row %lld (index %lld, bound %lld)",
                (long long)info.row, (long long)info.idx, (long long)info.len);
}

extern "C" rkv_status rkv_gather_diagnose(const rkv_pool_view* pool, const int32_t* page_table, int64_t pt_stride,
                                          const int32_t* cu_seqlens, int32_t n_seq, rkv_err_info* out,
                                          rkv_stream_t stream) {
  using namespace rkv;
  const char* what = "rkv_gather_diagnose";
  rkv_status st = check_pool(pool, what);
  if (st != RKV_OK) return st;
  if (n_seq < 0 || pt_stride < 0) return fail_shape("n_seq", 0, n_seq, "%s: negative sizes", what);
  if (n_seq > 0 && (!page_table || !cu_seqlens))
    return fail(RKV_ERR_INVALID_ARGUMENT, "%s: page_table and cu_seqlens are required", what);
  std::vector<int32_t> cu((size_t)n_seq + 1, 0), pt((size_t)(n_seq * pt_stride));
  st = copy_back(cu.data(), cu_seqlens, cu.size() * 4, stream, what);
  if (st == RKV_OK) st = copy_back(pt.data(), page_table, pt.size() * 4, stream, what);
  if (st != RKV_OK) return st;
  rkv_err_info info = blank_info(RKV_OK);
  for (int32_t s = 0; s < n_seq && info.status == RKV_OK; ++s) {
    const int64_t len = (int64_t)cu[(size_t)s + 1] - cu[(size_t)s];
    for (int64_t p = 0; p * kPageTokens < len; ++p) {
      const int32_t page = p < pt_stride ? pt[(size_t)(s * pt_stride + p)] : -1;
      if (page < 0 || page >= pool->n_pages) {
        info = blank_info(RKV_ERR_INDEX_OUT_OF_RANGE);
        set_what(info, "page_table");
        info.idx = page;
        info.len = pool->n_pages;
        info.row = (int64_t)cu[(size_t)s] + p * kPageTokens;
        break;
      }
    }
  }
  return report(out, info, "rkv_gather_diagnose: first failing output row %lld (page %lld of %lld)",
                (long long)info.row, (long long)info.idx, (long long)info.len);
}

extern "C" rkv_status rkv_sparse_gather_diagnose(const rkv_pool_view* pool, const int32_t* page_table,
                                                 int64_t pt_stride, const int32_t* seq_of_query,
                                                 const int32_t* seq_lens, int32_t n_seq, const int32_t* idx,
                                                 int32_t n_q, int32_t k, rkv_err_info* out, rkv_stream_t stream) {
  using namespace rkv;
  const char* what = "rkv_sparse_gather_diagnose";
  rkv_status st = check_pool(pool, what);
  if (st != RKV_OK) return st;
  if (n_seq < 0 || n_q < 0 || k < 0 || pt_stride < 0)
    return fail_shape("n_q", 0, n_q, "%s: negative sizes", what);
  if ((n_q > 0 && (!seq_of_query || (k > 0 && !idx))) || (n_seq > 0 && (!seq_lens || !page_table)))
    return fail(RKV_ERR_INVALID_ARGUMENT, "%s: page_table, seq_of_query, seq_lens and idx are required", what);
  std::vector<int32_t> sq((size_t)n_q), sl((size_t)n_seq), ix((size_t)n_q * k), pt((size_t)(n_seq * pt_stride));
  st = copy_back(sq.data(), seq_of_query, sq.size() * 4, stream, what);
  if (st == RKV_OK) st = copy_back(sl.data(), seq_lens, sl.size() * 4, stream, what);
  if (st == RKV_OK) st = copy_back(ix.data(), idx, ix.size() * 4, stream, what);
  if (st == RKV_OK) st = copy_back(pt.data(), page_table, pt.size() * 4, stream, what);
  if (st != RKV_OK) return st;
  rkv_err_info info = blank_info(RKV_OK);
  for (int64_t g = 0; g < (int64_t)n_q * k; ++g) {
    const int32_t t = ix[(size_t)g];
    if (t < 0) continue;  // a zero row, not an error
    const int32_t s = sq[(size_t)(g / k)];
    if (s < 0 || s >= n_seq) {
      info = blank_info(RKV_ERR_INDEX_OUT_OF_RANGE);
      set_what(info, "seq_of_query");
      info.idx = s;
      info.len = n_seq;
      info.row = g;
      break;
    }
    if (t >= sl[(size_t)s]) {
      info = blank_info(RKV_ERR_INDEX_OUT_OF_RANGE);
      set_what(info, "idx");
      info.idx = t;
      info.len = sl[(size_t)s];
      info.row = g;
      break;
    }
    const int64_t p = t / kPageTokens;
    const int32_t page = p < pt_stride ? pt[(size_t)(s * pt_stride + p)] : -1;
    if (page < 0 || page >= pool->n_pages) {
      info = blank_info(RKV_ERR_INDEX_OUT_OF_RANGE);
      set_what(info, "page_table");
      info.idx = page;
      info.len = pool->n_pages;
      info.row = g;
      break;
    }
  }
  return report(out, info, "rkv_sparse_gather_diagnose: first failing selection %lld (index %lld, bound %lld)",
                (long long)info.row, (long long)info.idx, (long long)info.len);
}
