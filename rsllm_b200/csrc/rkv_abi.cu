// rkv_abi.cu -- library-wide C-ABI utilities: version, last-error message,
// status-word decoding, pool sizing.
#include <stdarg.h>
#include <stdio.h>

#include "rkv_common.cuh"
#include "rkv_host.h"

namespace rkv {

static thread_local char g_last_error[512] = {0};
static thread_local rkv_err_info g_last_info = {RKV_OK, 0, {0}, -1, -1, -1, -1, -1, -1, -1};

rkv_err_info blank_info(rkv_status st) {
  rkv_err_info e = {st, 0, {0}, -1, -1, -1, -1, -1, -1, -1};
  return e;
}

static void set_what(rkv_err_info& e, const char* what) {
  snprintf(e.what, sizeof(e.what), "%s", what ? what : "");
}

static rkv_status record(const rkv_err_info& info, const char* fmt, va_list ap) {
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  g_last_info = info;
  return info.status;
}

rkv_status fail(rkv_status st, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  record(blank_info(st), fmt, ap);
  va_end(ap);
  return st;
}

rkv_status fail_shape(const char* what, int64_t expected, int64_t actual, const char* fmt, ...) {
  rkv_err_info e = blank_info(RKV_ERR_SHAPE_MISMATCH);
  set_what(e, what);
  e.expected = expected;
  e.actual = actual;
  va_list ap;
  va_start(ap, fmt);
  record(e, fmt, ap);
  va_end(ap);
  return e.status;
}

rkv_status fail_index(const char* what, int64_t idx, int64_t len, const char* fmt, ...) {
  rkv_err_info e = blank_info(RKV_ERR_INDEX_OUT_OF_RANGE);
  set_what(e, what);
  e.idx = idx;
  e.len = len;
  va_list ap;
  va_start(ap, fmt);
  record(e, fmt, ap);
  va_end(ap);
  return e.status;
}

rkv_status fail_layer(int64_t idx, int64_t max, const char* fmt, ...) {
  rkv_err_info e = blank_info(RKV_ERR_INVALID_LAYER);
  set_what(e, "layer");
  e.idx = idx;
  e.max = max;
  va_list ap;
  va_start(ap, fmt);
  record(e, fmt, ap);
  va_end(ap);
  return e.status;
}

rkv_status fail_full(int64_t cap, const char* fmt, ...) {
  rkv_err_info e = blank_info(RKV_ERR_POOL_FULL);
  set_what(e, "pool");
  e.cap = cap;
  va_list ap;
  va_start(ap, fmt);
  record(e, fmt, ap);
  va_end(ap);
  return e.status;
}

rkv_status fail_info(const rkv_err_info& info, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  record(info, fmt, ap);
  va_end(ap);
  return info.status;
}

void clear_error() {
  g_last_error[0] = 0;
  g_last_info = blank_info(RKV_OK);
}

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

rkv_status rkv_last_error_info(rkv_err_info* out) {
  if (!out) return RKV_ERR_INVALID_ARGUMENT;
  *out = rkv::g_last_info;
  return RKV_OK;
}

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
