"""The data of rsLLM's error variants at the C boundary (rkv_last_error_info):
host-validated errors fill ShapeMismatch { what, expected, actual },
IndexOutOfRange { what, idx, len }, InvalidLayer { idx, max } and
CompressedPoolFull { cap } (crates/rsllm-kvcache/src/lib.rs:28-70), and a
call that succeeds clears them.  These checks run before any CUDA call, so
they need no GPU (the pool view points nowhere)."""
from ctypes import byref, c_int64, c_void_p

import numpy as np
import pytest

import rsllm_b200 as rk
from rsllm_b200 import _abi
from rsllm_b200.prefix_pool import PrefixKvPool

NULL = c_void_p(0)


@pytest.fixture(scope="module")
def lib():
    return _abi.load()


def fake_view(n_pages=4, n_layers=2):
    return _abi.PoolView(256, n_pages, n_layers, 0)  # never dereferenced: validation fails first


def test_invalid_layer_carries_idx_and_max(lib):
    v = fake_view(n_layers=2)
    rc = lib.rkv_append_quant_bf16(byref(v), 1, 2, c_void_p(256), 8, c_void_p(256), NULL, NULL)
    assert rc == _abi.RKV_ERR_INVALID_LAYER
    info = _abi.last_error_info()
    assert info["status"] == rc and info["what"] == "layer" and info["idx"] == 2 and info["max"] == 2
    assert info["expected"] == -1 and info["cap"] == -1 and info["row"] == -1
    rc = lib.rkv_gather_dequant_bf16(byref(v), -1, c_void_p(256), 1, c_void_p(256), 1, 64, c_void_p(256), NULL, NULL)
    assert rc == _abi.RKV_ERR_INVALID_LAYER and _abi.last_error_info()["idx"] == -1


def test_shape_mismatch_carries_expected_and_actual(lib):
    v = fake_view()
    rc = lib.rkv_append_quant_bf16(byref(v), 0, 1, c_void_p(256), -3, c_void_p(256), NULL, NULL)
    assert rc == _abi.RKV_ERR_SHAPE_MISMATCH
    info = _abi.last_error_info()
    assert (info["what"], info["expected"], info["actual"]) == ("n_tokens", 0, -3)
    # a page table 2 pages wide cannot hold 200-token sequences (4 pages)
    rc = lib.rkv_gather_dequant_bf16(byref(v), 0, c_void_p(256), 2, c_void_p(256), 1, 200, c_void_p(256), NULL, NULL)
    assert rc == _abi.RKV_ERR_SHAPE_MISMATCH
    info = _abi.last_error_info()
    assert (info["what"], info["expected"], info["actual"]) == ("pt_stride", 4, 2)
    rc = lib.rkv_topk_select_f32(c_void_p(256), 8192, 1, c_void_p(256), 8192, 5000, c_void_p(256), NULL)
    info = _abi.last_error_info()
    assert rc == _abi.RKV_ERR_SHAPE_MISMATCH and (info["what"], info["expected"], info["actual"]) == ("k", 4096, 5000)


def test_pool_errors_carry_their_data_and_success_clears_them(lib):
    pool = PrefixKvPool(4, 1, device=None)  # plan-only: host allocator, no device memory
    s = pool.create_sequence()
    with pytest.raises(rk.IndexOutOfRange) as e:
        pool.reserve([s + 99], [1])
    assert e.value.what == "seq" and e.value.idx == s + 99
    with pytest.raises(rk.PoolFull) as e:
        pool.reserve([s], [5 * 64])
    assert e.value.cap == 4 * 64 and e.value.status == _abi.RKV_ERR_POOL_FULL
    with pytest.raises(rk.ShapeMismatch) as e:
        pool.reserve([s], [-1])
    assert (e.value.what, e.value.expected, e.value.actual) == ("n_tokens", 0, -1)
    pool.reserve([s], [70])
    assert _abi.last_error_info()["status"] == 0 and _abi.last_error() == ""
    with pytest.raises(rk.IndexOutOfRange) as e:
        pool.fork(s, 71)
    assert (e.value.what, e.value.idx, e.value.len) == ("n_tokens", 71, 71)


def test_static_moves_outside_the_pool_name_the_page(lib):
    v = fake_view(n_pages=8)
    src = np.array([1, 2], np.int32)
    dst = np.array([5, 9], np.int32)
    rc = lib.rkv_apply_page_moves_static(byref(v), c_void_p(src.ctypes.data), c_void_p(dst.ctypes.data), 2, NULL,
                                         0, NULL, NULL)
    info = _abi.last_error_info()
    assert rc == _abi.RKV_ERR_INDEX_OUT_OF_RANGE and (info["what"], info["idx"], info["len"]) == ("dst", 9, 8)


def test_copy_floor_validates_like_the_append(lib):
    """rkv_copy_floor_bf16 (the append's traffic for measurement) rejects the
    same bad arguments as the append, with the same error data, before any
    device work."""
    v = fake_view(n_layers=2)
    rc = lib.rkv_copy_floor_bf16(byref(v), 1, 2, c_void_p(256), 8, c_void_p(256), NULL)
    info = _abi.last_error_info()
    assert rc == _abi.RKV_ERR_INVALID_LAYER and info["idx"] == 2 and info["max"] == 2
    rc = lib.rkv_copy_floor_bf16(byref(v), 0, 1, c_void_p(256), -3, c_void_p(256), NULL)
    info = _abi.last_error_info()
    assert rc == _abi.RKV_ERR_SHAPE_MISMATCH and (info["what"], info["expected"], info["actual"]) == ("n_tokens", 0, -3)
    rc = lib.rkv_copy_floor_bf16(byref(v), 0, 1, c_void_p(8), 4, c_void_p(256), NULL)  # rows not 32-byte aligned
    assert rc == _abi.RKV_ERR_INVALID_ARGUMENT
    assert lib.rkv_copy_floor_bf16(byref(v), 0, 1, c_void_p(256), 0, c_void_p(256), NULL) == _abi.RKV_OK
