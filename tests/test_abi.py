"""The C-ABI library loads, exports every function include/rsllm_kv_cuda.h
declares, and rejects bad arguments on the host before any launch (no GPU is
touched here)."""
import ctypes
import re
from ctypes import byref, c_void_p

import pytest

from rsllm_b200 import _abi


def test_every_header_function_is_exported():
    lib = _abi.load()
    names = _abi.header_functions()
    assert len(names) >= 11
    for name in names:
        assert hasattr(lib, name), name
        assert name in _abi.SIGNATURES, f"{name} has no ctypes signature"
    assert set(_abi.SIGNATURES) == set(names)


def test_header_constants_match_bindings():
    text = _abi.HEADER.read_text()
    consts = dict(re.findall(r"#define (RKV_[A-Z_]+) (\d+)", text))
    assert int(consts["RKV_PAGE_BYTES"]) == _abi.PAGE_BYTES == 64 * 512 + 64 * 8 * 4 + 64 * 64 * 2
    for name in ("RKV_ERR_SHAPE_MISMATCH", "RKV_ERR_INDEX_OUT_OF_RANGE", "RKV_ERR_INVALID_LAYER", "RKV_ERR_POOL_FULL",
                 "RKV_ERR_NON_FINITE_INPUT", "RKV_ERR_INVALID_ARGUMENT", "RKV_ERR_CUDA"):
        assert int(consts[name]) == getattr(_abi, name)


def test_status_bits_priority_and_sizes():
    lib = _abi.load()
    assert lib.rkv_status_from_bits(0) == 0
    assert lib.rkv_status_from_bits(1 << _abi.RKV_ERR_NON_FINITE_INPUT) == _abi.RKV_ERR_NON_FINITE_INPUT
    both = (1 << _abi.RKV_ERR_NON_FINITE_INPUT) | (1 << _abi.RKV_ERR_INDEX_OUT_OF_RANGE)
    assert lib.rkv_status_from_bits(both) == _abi.RKV_ERR_INDEX_OUT_OF_RANGE
    assert lib.rkv_pool_bytes(1 << 20, 1) == (1 << 20) * 43008
    assert lib.rkv_version().decode().count(".") == 2


def test_host_validation_without_device():
    lib = _abi.load()
    null = c_void_p(0)
    # NULL pool view
    assert lib.rkv_append_quant_bf16(None, 0, 1, null, 1, null, null, null) == _abi.RKV_ERR_INVALID_ARGUMENT
    assert "pool view is NULL" in _abi.last_error()
    # misaligned base
    v = _abi.PoolView(0x1001, 4, 2, 0)
    assert lib.rkv_gather_dequant_bf16(byref(v), 0, null, 1, null, 1, 64, null, null, null) == \
        _abi.RKV_ERR_INVALID_ARGUMENT
    # layer outside the pool: InvalidLayer, as ThreeTierKvCache::append_layer
    v = _abi.PoolView(0x100000, 4, 2, 0)
    assert lib.rkv_append_quant_bf16(byref(v), 1, 2, null, 1, null, null, null) == _abi.RKV_ERR_INVALID_LAYER
    assert lib.rkv_gather_dequant_bf16(byref(v), 2, null, 1, null, 1, 64, null, null, null) == \
        _abi.RKV_ERR_INVALID_LAYER
    assert lib.rkv_sparse_gather_dequant_bf16(byref(v), -1, null, 1, null, null, null, 1, 1, null, null, null) == \
        _abi.RKV_ERR_INVALID_LAYER
    # shape errors
    assert lib.rkv_topk_select_f32(null, 8, 1, null, 8, 5000, null, null) == _abi.RKV_ERR_SHAPE_MISMATCH
    assert lib.rkv_topk_select_f32(null, 8, 1, null, 16, 4, null, null) == _abi.RKV_ERR_SHAPE_MISMATCH
    assert lib.rkv_gather_dequant_bf16(byref(v), 0, null, 1, null, 1, 65, null, null, null) == \
        _abi.RKV_ERR_SHAPE_MISMATCH  # pt_stride 1 < 2 pages
    # empty work is a no-op success
    assert lib.rkv_append_quant_bf16(byref(v), 0, 2, null, 0, null, null, null) == 0
    assert lib.rkv_sparse_gather_dequant_bf16(byref(v), 0, null, 1, null, null, null, 0, 8, null, null, null) == 0


def test_python_layer_fails_loudly_without_cuda(monkeypatch):
    import torch

    import rsllm_b200

    if torch.cuda.is_available():
        pytest.skip("a CUDA device is present")
    with pytest.raises(rsllm_b200.CudaError):
        rsllm_b200.PagedKvPool(4, 1)
    with pytest.raises(rsllm_b200.CudaError):
        rsllm_b200.CudaBackend()
