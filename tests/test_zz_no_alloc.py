"""The allocation-free page-move entry point (rkv_apply_page_moves_static)
against the pool's own compaction (rkv_pool_compact), through the C ABI.

Callers that cannot allocate device memory -- an engine that reserves all of
its device memory at start-up, or the owner of a plan-only pool moving pages
with memory it already has -- apply a compaction's moves through this entry
point, which stages them in a fixed array inside the library instead of
memory the pool allocated.  Two compactions in a row: after each, the pool
bytes and the device page table must equal those the pool's own compaction
produced from the same starting bytes (the moves are exact copies, so the
tolerance is zero).  This file sorts last so that a failure here comes after
every other test has run.
"""
from ctypes import byref, c_void_p

import numpy as np
import pytest
import torch

import rsllm_b200 as rk
from rsllm_b200 import _abi, synth
from rsllm_b200.prefix_pool import PrefixKvPool

pytestmark = pytest.mark.gpu


def test_static_moves_match_pool_compaction_twice(cuda):
    lib = _abi.load()
    rng = np.random.default_rng(11)
    n_pages, n_layers = 2048, 2
    pool = PrefixKvPool(n_pages, n_layers, device=0)
    pool.kv.storage.random_(0, 256)
    twin = torch.empty_like(pool.kv.storage)  # second copy of the pool bytes for the static path
    twin_view = _abi.PoolView(twin.data_ptr(), n_pages, n_layers, 0)
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    seqs = []
    for round_ in range(2):
        # grow and shrink the pool so the compaction has holes to fill
        for i in range(12):
            s = pool.create_sequence()
            n = int(rng.integers(200, 6000))
            slots = pool.reserve([s], [n])
            rows = synth.kv_rows(n_layers * n, seed=100 * round_ + i, device=cuda).view(n_layers, n, 576)
            pool.kv.append_layer(0, rows.contiguous(), torch.from_numpy(slots).to(cuda))
            seqs.append(s)
        for s in list(seqs):
            if rng.random() < 0.4:
                pool.free(s)
                seqs.remove(s)
        pool.kv.check("append")
        tabs = [pool.page_table(s) for s in seqs]
        stride = max(len(t) for t in tabs)
        pt = np.full((len(seqs), stride), -1, np.int32)
        for i, t in enumerate(tabs):
            pt[i, :len(t)] = t
        d_pt = torch.from_numpy(pt).to(cuda)
        d_pt_twin = d_pt.clone()
        twin.copy_(pool.kv.storage)
        torch.cuda.synchronize()

        moved = pool.compact(device_tables=d_pt)  # the pool's own compaction
        remap = pool.last_remap()
        src = np.nonzero(remap != np.arange(n_pages, dtype=np.int32))[0].astype(np.int32)
        dst = remap[src].astype(np.int32)
        assert src.size == moved > 0
        rc = lib.rkv_apply_page_moves_static(byref(twin_view), c_void_p(src.ctypes.data), c_void_p(dst.ctypes.data),
                                             src.size, c_void_p(d_pt_twin.data_ptr()), d_pt_twin.numel(),
                                             c_void_p(status.data_ptr()), c_void_p(torch.cuda.current_stream().cuda_stream))
        assert rc == 0, _abi.last_error()
        torch.cuda.synchronize()
        assert int(status.item()) == 0 and pool.device_status() == 0
        assert torch.equal(d_pt_twin, d_pt), f"round {round_}: page tables differ"
        assert torch.equal(twin, pool.kv.storage), f"round {round_}: pool bytes differ"
        # what the compaction promised: every live page below the live count
        st = pool.stats()
        assert st["high_water"] == st["live_pages"]


def test_static_moves_rejects_too_many_and_bad_lists(cuda):
    lib = _abi.load()
    buf = torch.empty(rk.pool_bytes(8, 1), dtype=torch.uint8, device=cuda)
    view = _abi.PoolView(buf.data_ptr(), 8, 1, 0)
    null = c_void_p(0)
    big = np.arange(_abi.STATIC_MAX_MOVES + 1, dtype=np.int32)
    rc = lib.rkv_apply_page_moves_static(byref(view), c_void_p(big.ctypes.data), c_void_p(big.ctypes.data),
                                         big.size, null, 0, null, null)
    assert rc == _abi.RKV_ERR_SHAPE_MISMATCH and "exceed" in _abi.last_error()
    src = np.array([5, 3], np.int32)
    dst = np.array([0, 1], np.int32)
    assert lib.rkv_apply_page_moves_static(byref(view), c_void_p(src.ctypes.data), c_void_p(dst.ctypes.data), 2,
                                           null, 0, null, null) == _abi.RKV_ERR_INVALID_ARGUMENT
    src = np.array([3, 5], np.int32)
    dst = np.array([5, 1], np.int32)  # 5 is a source and a destination
    assert lib.rkv_apply_page_moves_static(byref(view), c_void_p(src.ctypes.data), c_void_p(dst.ctypes.data), 2,
                                           null, 0, null, null) == _abi.RKV_ERR_INVALID_ARGUMENT
    src = np.array([3, 9], np.int32)
    assert lib.rkv_apply_page_moves_static(byref(view), c_void_p(src.ctypes.data), c_void_p(dst.ctypes.data), 2,
                                           null, 0, null, null) == _abi.RKV_ERR_INDEX_OUT_OF_RANGE
    src = np.array([1, 2, 3], np.int32)
    dst = np.array([6, 7, 6], np.int32)  # two moves write page 6
    assert lib.rkv_apply_page_moves_static(byref(view), c_void_p(src.ctypes.data), c_void_p(dst.ctypes.data), 3,
                                           null, 0, null, null) == _abi.RKV_ERR_INVALID_ARGUMENT
    assert "two moves" in _abi.last_error()


def _moves(rng, n_pages: int, n: int):
    """n moves with ascending distinct sources and distinct destinations
    outside the sources."""
    pages = rng.permutation(n_pages)[:2 * n].astype(np.int32)
    return np.sort(pages[:n]), pages[n:].copy()


def test_static_moves_large_then_small_and_without_tables(cuda):
    """A long move list, then short ones on the same stream (the staging
    array's leftover entries from the long list must never be read), one of
    them with no page table: pool bytes and tables equal those of
    rkv_copy_pages + rkv_remap_pages applied to a twin of the pool."""
    lib = _abi.load()
    rng = np.random.default_rng(5)
    n_pages, n_layers = 4096, 2
    mine = torch.empty(rk.pool_bytes(n_pages, n_layers), dtype=torch.uint8, device=cuda).random_(0, 256)
    twin = rk.PagedKvPool(n_pages, n_layers, device=cuda, storage=mine.clone())
    view = _abi.PoolView(mine.data_ptr(), n_pages, n_layers, 0)
    table = torch.from_numpy(rng.integers(-1, n_pages, 6000).astype(np.int32)).to(cuda)
    table_twin = table.clone()
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    stream = torch.cuda.current_stream()
    for n, with_table in ((1800, True), (7, True), (5, False)):
        src, dst = _moves(rng, n_pages, n)
        rc = lib.rkv_apply_page_moves_static(byref(view), c_void_p(src.ctypes.data), c_void_p(dst.ctypes.data), n,
                                             c_void_p(table.data_ptr() if with_table else 0),
                                             table.numel() if with_table else 0, c_void_p(status.data_ptr()),
                                             c_void_p(stream.cuda_stream))
        assert rc == 0, _abi.last_error()
        twin.copy_pages(torch.from_numpy(src).to(cuda), torch.from_numpy(dst).to(cuda))
        if with_table:
            remap = np.arange(n_pages, dtype=np.int32)
            remap[src] = dst
            rk.remap_pages(table_twin, torch.from_numpy(remap).to(cuda))
        torch.cuda.synchronize()
        twin.check("twin moves")
        assert int(status.item()) == 0
        assert torch.equal(table, table_twin), f"{n} moves: page tables differ"
        assert torch.equal(mine, twin.storage), f"{n} moves: pool bytes differ"
