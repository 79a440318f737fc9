// rkv_host.h -- host-side helpers shared by the C-ABI entry points:
// argument validation, the per-thread last-error message, launch checks.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/rsllm_kv_cuda.h"

namespace rkv {

// Records a printf-style message as this thread's last error; returns `st`.
// The error data (rkv_last_error_info) carries only the status.
rkv_status fail(rkv_status st, const char* fmt, ...);

// The same, with the data of rsLLM's error variant (rkv_err_info):
// ShapeMismatch { what, expected, actual }, IndexOutOfRange { what, idx, len },
// InvalidLayer { idx, max }, CompressedPoolFull { cap } (token rows).
rkv_status fail_shape(const char* what, int64_t expected, int64_t actual, const char* fmt, ...);
rkv_status fail_index(const char* what, int64_t idx, int64_t len, const char* fmt, ...);
rkv_status fail_layer(int64_t idx, int64_t max, const char* fmt, ...);
rkv_status fail_full(int64_t cap, const char* fmt, ...);
// Records a device-detected error found by a diagnosis: `info` and a message.
rkv_status fail_info(const rkv_err_info& info, const char* fmt, ...);
// An rkv_err_info with status `st` and every field "does not apply".
rkv_err_info blank_info(rkv_status st);

// Clears this thread's last error (a call that succeeds leaves "" behind).
void clear_error();

// Maps a pending launch error (cudaGetLastError) to RKV_ERR_CUDA.
rkv_status check_launch(const char* what);

// Per-device caches of launch parameters cover devices [0, kMaxDevicesCached).
constexpr int kMaxDevicesCached = 64;

inline bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; }

// Validates a pool view: non-null 256-byte aligned base, positive sizes.
rkv_status check_pool(const rkv_pool_view* p, const char* what);

// Internal accessors of a pool handle (rkv_pool.cpp): its device (RKV_PLAN_ONLY
// for a plan-only pool) and its device status word.
int pool_device(const rkv_pool* pool);
uint32_t* pool_status_word(rkv_pool* pool);

}  // namespace rkv
