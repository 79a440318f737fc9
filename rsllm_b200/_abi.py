"""ctypes bindings of ``include/rsllm_kv_cuda.h`` (the C ABI of the library).

Loading fails loudly: there is no CPU fallback for any entry point.
"""
from __future__ import annotations

import ctypes
from ctypes import POINTER, Structure, c_char_p, c_float, c_int32, c_int64, c_uint8, c_uint16, c_uint32, c_uint64, c_void_p
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "librsllm_kv_cuda.so"
HEADER = Path(__file__).resolve().parent.parent / "include" / "rsllm_kv_cuda.h"

RKV_OK = 0
RKV_ERR_SHAPE_MISMATCH = 1
RKV_ERR_INDEX_OUT_OF_RANGE = 2
RKV_ERR_INVALID_LAYER = 3
RKV_ERR_POOL_FULL = 4
RKV_ERR_NON_FINITE_INPUT = 5
RKV_ERR_INVALID_ARGUMENT = 6
RKV_ERR_CUDA = 7

PAGE_TOKENS = 64
LATENT_DIM = 512
ROPE_DIM = 64
ROW_DIM = 576
BLOCK = 64
PAGE_BYTES = 43008


class PoolView(Structure):
    """``rkv_pool_view``: device base pointer, pages per layer, layers."""

    _fields_ = [("base", c_void_p), ("n_pages", c_int64), ("n_layers", c_int32), ("reserved", c_int32)]


class PoolDesc(Structure):
    """``rkv_pool_desc``."""

    _fields_ = [("n_pages", c_int64), ("n_layers", c_int32), ("device", c_int32), ("storage", c_void_p)]


class ErrInfo(Structure):
    """rkv_err_info: the fields of rsLLM's error variants."""

    _fields_ = [("status", c_int32), ("reserved", c_int32), ("what", ctypes.c_char * 48), ("idx", c_int64),
                ("len", c_int64), ("expected", c_int64), ("actual", c_int64), ("max", c_int64), ("cap", c_int64),
                ("row", c_int64)]

    def as_dict(self) -> dict:
        d = {f: getattr(self, f) for f, _ in self._fields_ if f != "reserved"}
        d["what"] = self.what.decode("utf-8", "replace")
        return d


class PoolStats(Structure):
    """``rkv_pool_stats``."""

    _fields_ = [("free_pages", c_int64), ("live_pages", c_int64), ("sequences", c_int64), ("prefix_nodes", c_int64),
                ("tick", c_int64), ("high_water", c_int64)]


class KvcHeader(Structure):
    """``rkv_kvc_header``."""

    _fields_ = [("version", c_uint32), ("quant_bits", c_uint32), ("reason", c_uint32), ("reserved", c_uint32),
                ("token_count", c_uint64), ("ctx_size", c_uint64), ("created_at", c_uint64),
                ("payload_bytes", c_uint64)]


KVC_COLD, KVC_CONTINUED, KVC_EVICT, KVC_SHUTDOWN = 0, 1, 2, 3
KVC_HEADER_BYTES = 48

PLAN_ONLY = -1

_P = POINTER
_u8p, _u16p, _u32p, _i32p, _f32p = c_void_p, c_void_p, c_void_p, c_void_p, c_void_p

# name -> (restype, argtypes); every function the header declares.
SIGNATURES = {
    "rkv_version": (c_char_p, []),
    "rkv_last_error": (c_char_p, []),
    "rkv_last_error_info": (c_int32, [c_void_p]),
    "rkv_append_diagnose_bf16": (c_int32, [_P(PoolView), c_int32, c_int32, _u16p, c_int64, _i32p, c_void_p,
                                           c_void_p]),
    "rkv_gather_diagnose": (c_int32, [_P(PoolView), _i32p, c_int64, _i32p, c_int32, c_void_p, c_void_p]),
    "rkv_sparse_gather_diagnose": (c_int32, [_P(PoolView), _i32p, c_int64, _i32p, _i32p, c_int32, _i32p, c_int32,
                                             c_int32, c_void_p, c_void_p]),
    "rkv_status_from_bits": (c_int32, [c_uint32]),
    "rkv_pool_bytes": (c_int64, [c_int64, c_int32]),
    "rkv_append_quant_bf16": (c_int32, [_P(PoolView), c_int32, c_int32, _u16p, c_int64, _i32p, _u32p, c_void_p]),
    "rkv_append_quant_bf16_ex": (c_int32, [_P(PoolView), c_int32, c_int32, _u16p, c_int64, _i32p, c_uint32, _u32p,
                                           c_void_p]),
    "rkv_copy_floor_bf16": (c_int32, [_P(PoolView), c_int32, c_int32, _u16p, c_int64, _i32p, c_void_p]),
    "rkv_append_quant_f32": (c_int32, [_P(PoolView), c_int32, c_int32, _f32p, c_int64, _i32p, _u32p, c_void_p]),
    "rkv_scale_threshold_table": (None, [_u32p]),
    "rkv_gather_dequant_bf16": (c_int32, [_P(PoolView), c_int32, _i32p, c_int64, _i32p, c_int32, c_int32, _u16p,
                                          _u32p, c_void_p]),
    "rkv_topk_select_f32": (c_int32, [_f32p, c_int64, c_int32, _i32p, c_int32, c_int32, _i32p, c_void_p]),
    "rkv_sparse_gather_dequant_bf16": (c_int32, [_P(PoolView), c_int32, _i32p, c_int64, _i32p, _i32p, _i32p,
                                                 c_int32, c_int32, _u16p, _u32p, c_void_p]),
    "rkv_copy_pages": (c_int32, [_P(PoolView), _i32p, _i32p, c_int64, _u32p, c_void_p]),
    "rkv_remap_pages": (c_int32, [_i32p, c_int64, _i32p, c_int64, _u32p, c_void_p]),
    "rkv_e4m3fn_code_range": (c_int32, [c_uint32, c_int64, _u8p, c_void_p]),
    "rkv_pack_pages": (c_int32, [_P(PoolView), c_int32, c_int32, _i32p, c_int64, c_void_p, _u32p, c_void_p]),
    "rkv_unpack_pages": (c_int32, [_P(PoolView), c_int32, c_int32, _i32p, c_int64, c_void_p, _u32p, c_void_p]),
    "rkv_kvc_name": (c_int32, [_i32p, c_int64, c_char_p]),
    "rkv_kvc_read_header": (c_int32, [c_char_p, _P(KvcHeader)]),
    "rkv_kvc_save": (c_int32, [c_void_p, c_int64, _i32p, c_int64, c_uint32, c_uint32, c_char_p, c_int64, c_char_p,
                               c_char_p, c_int64, c_void_p]),
    "rkv_kvc_load": (c_int32, [c_void_p, c_char_p, _i32p, c_int64, _P(c_int64), _P(c_int64), c_int32, c_void_p]),
    "rkv_mla_decode_workspace_bytes": (c_int64, [c_int32, c_int32]),
    "rkv_mla_decode_fp8": (c_int32, [_P(PoolView), c_int32, _i32p, c_int64, _i32p, _i32p, _u16p, c_int32, _i32p,
                                     c_int32, _f32p, c_float, c_int32, c_void_p, _f32p, _u32p, c_void_p]),
    "rkv_compress_state_bytes": (c_int64, [c_int32]),
    "rkv_compress_append_ex": (c_int32, [_P(PoolView), c_int32, c_int32, _f32p, c_int64, _f32p, _f32p, c_int64,
                                         _i32p, _i32p, _i32p, _f32p, _f32p, _f32p, c_int64, c_uint32, _u32p,
                                         c_void_p]),
    "rkv_indexer_compress_state_bytes": (c_int64, [c_int32]),
    "rkv_indexer_compress_append": (c_int32, [c_int32, _f32p, c_int64, _f32p, _f32p, c_int64, _i32p, _i32p, _i32p,
                                              _f32p, _f32p, _f32p, c_int64, _f32p, c_int64, _u32p, c_void_p]),
    "rkv_compress_rope_table": (c_int32, [c_int32, c_int64, _f32p]),
    "rkv_compress_prepare": (c_int32, []),
    "rkv_compress_wait_probe": (c_int32, [_u32p, c_void_p]),
    "rkv_compress_append": (c_int32, [_P(PoolView), c_int32, c_int32, _f32p, c_int64, _f32p, _f32p, c_int64, _i32p,
                                      _i32p, _i32p, _f32p, _f32p, _f32p, c_int64, _u32p, c_void_p]),
    "rkv_compress_expf": (c_int32, [_f32p, _f32p, c_int64, c_int32, c_void_p]),
    "rkv_compress_expf_table_size": (c_int64, []),
    "rkv_indexer_scores_f32": (c_int32, [_f32p, c_void_p, _i32p, c_int64, _f32p, _f32p, _i32p, _i32p, c_int32,
                                         c_int32, _f32p, c_int64, _u32p, c_void_p]),
    "rkv_indexer_topk_f32": (c_int32, [_f32p, c_void_p, _i32p, c_int64, _f32p, _f32p, _i32p, _i32p, c_int32,
                                       c_int32, c_int32, _f32p, c_int64, _i32p, _u32p, c_void_p]),
    "rkv_pool_create": (c_int32, [_P(PoolDesc), _P(c_void_p)]),
    "rkv_pool_destroy": (None, [c_void_p]),
    "rkv_pool_get_view": (c_int32, [c_void_p, _P(PoolView)]),
    "rkv_pool_get_stats": (c_int32, [c_void_p, _P(PoolStats)]),
    "rkv_page_refcount": (c_int32, [c_void_p, _i32p, c_int64]),
    "rkv_seq_create": (c_int32, [c_void_p, _P(c_int64)]),
    "rkv_seq_fork": (c_int32, [c_void_p, c_int64, c_int64, _P(c_int64)]),
    "rkv_seq_reserve": (c_int32, [c_void_p, c_int64, c_void_p, c_void_p, _i32p, c_void_p]),
    "rkv_seq_release": (c_int32, [c_void_p, c_int64]),
    "rkv_seq_touch": (c_int32, [c_void_p, c_int64]),
    "rkv_seq_free": (c_int32, [c_void_p, c_int64]),
    "rkv_seq_info": (c_int32, [c_void_p, c_int64, _P(c_int64), _P(c_int64)]),
    "rkv_seq_page_table": (c_int32, [c_void_p, c_int64, _i32p, c_int64]),
    "rkv_prefix_insert": (c_int32, [c_void_p, _i32p, c_int64, c_int64]),
    "rkv_prefix_match": (c_int32, [c_void_p, _i32p, c_int64, _P(c_int64), _P(c_int64)]),
    "rkv_pool_evict": (c_int32, [c_void_p, c_int64, _P(c_int64)]),
    "rkv_pool_compact": (c_int32, [c_void_p, _i32p, c_int64, _P(c_int64), c_void_p]),
    "rkv_pool_last_remap": (c_int32, [c_void_p, _i32p, c_int64]),
    "rkv_pool_take_moves": (c_int32, [c_void_p, _i32p, _i32p, c_int64, _P(c_int64)]),
    "rkv_pool_device_status": (c_int32, [c_void_p, _P(c_uint32)]),
    "rkv_apply_page_moves_static": (c_int32, [_P(PoolView), _i32p, _i32p, c_int64, _i32p, c_int64, _u32p,
                                              c_void_p]),
}
STATIC_MAX_MOVES = 262144
APPEND_INPUTS_READY = 1
COMPRESS_INPUTS_READY = 1
COMPRESS_ONE_TOKEN_PER_STATE = 2

_lib = None


def load() -> ctypes.CDLL:
    """Loads the CUDA library (building it first if sources are newer)."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        from . import build

        build.build()
    if not LIB_PATH.exists():
        raise ImportError(f"rsllm_b200: CUDA library missing at {LIB_PATH}")
    lib = ctypes.CDLL(str(LIB_PATH))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def last_error() -> str:
    return load().rkv_last_error().decode("utf-8", "replace")


def last_error_info() -> dict:
    """rkv_last_error_info as a dict (fields that do not apply are -1)."""
    info = ErrInfo()
    load().rkv_last_error_info(ctypes.byref(info))
    return info.as_dict()


def header_functions() -> list[str]:
    """Names of the functions the public header declares (parsed from it)."""
    import re

    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"^\s*RKV_API\s+[^;()]*?\b(rkv_[a-z0-9_]+)\s*\(", text, flags=re.M)))
