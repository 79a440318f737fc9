// rkv_abi.cu -- library-wide C-ABI utilities: version, last-error message,
// status-word decoding, pool sizing.
#include <stdarg.h>
#include <stdio.h>

#include "rkv_common.cuh"
#include "rkv_host.h"

namespace rkv {

static thread_local char g_last_error[512] = {0};

rkv_status fail(rkv_status st, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return st;
}

void clear_error() { g_last_error[0] = 0; }

rkv_status check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(RKV_ERR_CUDA, "%s: launch failed: %s", what, cudaGetErrorString(e));
  clear_error();
  return RKV_OK;
}

rkv_status check_pool(const rkv_pool_view* p, const char* what) {
  if (!p) return fail(RKV_ERR_INVALID_ARGUMENT, "%s: pool view is NULL", what);
  if (!p->base || !aligned(p->base, 256))
    return fail(RKV_ERR_INVALID_ARGUMENT, "%s: pool base must be a non-null 256-byte aligned device pointer", what);
  if (p->n_pages <= 0 || p->n_layers <= 0 || p->reserved != 0)
    return fail(RKV_ERR_INVALID_ARGUMENT, "%s: pool needs n_pages > 0, n_layers > 0, reserved == 0", what);
  if (p->n_pages > (int64_t)(INT32_MAX / kPageTokens))
    return fail(RKV_ERR_INVALID_ARGUMENT, "%s: n_pages * 64 must fit in int32 slots", what);
  return RKV_OK;
}

}  // namespace rkv

extern "C" {

const char* rkv_version(void) { return "0.1.0"; }

const char* rkv_last_error(void) { return rkv::g_last_error; }

rkv_status rkv_status_from_bits(uint32_t bits) {
  static const rkv_status order[] = {RKV_ERR_INVALID_ARGUMENT, RKV_ERR_INVALID_LAYER,  RKV_ERR_SHAPE_MISMATCH,
                                     RKV_ERR_INDEX_OUT_OF_RANGE, RKV_ERR_POOL_FULL, RKV_ERR_NON_FINITE_INPUT};
  for (rkv_status s : order)
    if (bits & (1u << s)) return s;
  return bits ? RKV_ERR_CUDA : RKV_OK;
}

int64_t rkv_pool_bytes(int64_t n_pages, int32_t n_layers) {
  if (n_pages < 0 || n_layers < 0) return -1;
  return n_pages * (int64_t)n_layers * (int64_t)RKV_PAGE_BYTES;
}

}  // extern "C"
