"""GPU checks of the device-backed prefix pool: copy-on-write copies happen on
the device before the new rows land (a branch reads its parent's rows, then
its own), and compaction moves pages without changing any row a surviving
sequence reads; every row is bit-exact against the CPU oracle."""
import numpy as np
import pytest
import torch

import oracle
import rsllm_b200 as rk
from rsllm_b200 import synth
from rsllm_b200.prefix_pool import PrefixKvPool

pytestmark = pytest.mark.gpu


def u16(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def expected_rows(rows: np.ndarray) -> np.ndarray:
    """Oracle round trip of bf16 rows: quantise, dequantise."""
    codes, scales, rope, st = oracle.quantize_rows_bf16(rows)
    assert np.all(st == 0)
    return oracle.dequant_rows_bf16(codes, scales, rope)


def gather(pool: PrefixKvPool, seqs, layer=0) -> list[np.ndarray]:
    tabs = [pool.page_table(s) for s in seqs]
    lens = [pool.seq_len(s) for s in seqs]
    stride = max(1, max(len(t) for t in tabs))
    pt = np.full((len(seqs), stride), -1, np.int32)
    for i, t in enumerate(tabs):
        pt[i, :len(t)] = t
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    dev = pool.kv.device
    out = u16(pool.kv.rows(layer, torch.from_numpy(pt).to(dev), torch.from_numpy(cu).to(dev), max(lens)))
    pool.kv.check("gather")
    return [out[cu[i]:cu[i + 1]] for i in range(len(seqs))]


def append(pool: PrefixKvPool, seqs, ns, rows_by_seq, seed):
    """Reserves ns[i] tokens for seqs[i] and appends fresh rows into them."""
    slots = pool.reserve(seqs, ns)
    total = int(sum(ns))
    rows = u16(synth.kv_rows(pool.n_layers * total, seed=seed)).reshape(pool.n_layers, total, 576)
    dev = pool.kv.device
    pool.kv.append_layer(0, torch.from_numpy(rows.view(np.int16)).view(torch.bfloat16).to(dev),
                         torch.from_numpy(slots).to(dev))
    pool.kv.check("append")
    o = 0
    for s, n in zip(seqs, ns):
        rows_by_seq.setdefault(s, [np.zeros((0, 576), np.uint16) for _ in range(pool.n_layers)])
        for layer in range(pool.n_layers):
            rows_by_seq[s][layer] = np.concatenate([rows_by_seq[s][layer], rows[layer, o:o + n]])
        o += n


def test_copy_on_write_on_device(cuda):
    pool = PrefixKvPool(64, 2, device=0)
    pool.kv.storage.zero_()
    rows = {}
    parent = pool.create_sequence()
    append(pool, [parent], [200], rows, seed=1)
    child = pool.fork(parent, 150)  # shares pages 0..2; page 2 is partial
    rows[child] = [r[:150] for r in rows[parent]]
    append(pool, [child], [100], rows, seed=2)   # child copies page 2 first
    append(pool, [parent], [30], rows, seed=3)   # parent's page 3 is its own
    assert pool.page_table(child)[:2].tolist() == pool.page_table(parent)[:2].tolist()
    assert pool.page_table(child)[2] != pool.page_table(parent)[2]
    for layer in (0, 1):
        got = gather(pool, [parent, child], layer)
        for s, g in zip([parent, child], got):
            assert np.array_equal(g, expected_rows(rows[s][layer])), (s, layer)
    assert pool.device_status() == 0


def test_prefix_store_branches_and_compaction(cuda):
    """Config 5 in miniature on the device: a shared prefix (8192 + 37
    tokens) in the radix store, branches matching it and appending, LRU
    eviction of 30% of the used pages, compaction with a device page table
    remapped in place -- every surviving row unchanged."""
    n_pages = 1024
    pool = PrefixKvPool(n_pages, 1, device=0)
    pool.kv.storage.zero_()
    rows = {}
    rng = np.random.default_rng(6)
    residents = []
    for i in range(6):
        s = pool.create_sequence()
        append(pool, [s], [int(rng.integers(1024, 4096))], rows, seed=10 + i)
        residents.append(s)
    for s in residents[:4]:
        pool.release(s)
    prefix = list(range(8192 + 37))
    owner = pool.create_sequence()
    append(pool, [owner], [len(prefix)], rows, seed=20)
    pool.insert_prefix(prefix, owner)
    branches = []
    for i in range(8):
        m, b = pool.match_prefix(prefix)
        assert m == len(prefix)
        rows[b] = [rows[owner][0][:m]]
        branches.append(b)
    pool.free(owner)
    append(pool, branches, [2048] * len(branches), rows, seed=30)
    survivors = [s for s in residents[4:]] + branches
    before = gather(pool, survivors)
    for s, g in zip(survivors, before):
        assert np.array_equal(g, expected_rows(rows[s][0]))
    used = pool.stats()["live_pages"]
    freed = pool.evict(int(0.3 * used))
    assert freed >= int(0.3 * used) or pool.stats()["sequences"] == len(survivors)
    # device copy of the survivors' page tables, remapped by the compaction
    tabs = [pool.page_table(s) for s in survivors]
    stride = max(len(t) for t in tabs)
    pt = np.full((len(survivors), stride), -1, np.int32)
    for i, t in enumerate(tabs):
        pt[i, :len(t)] = t
    d_pt = torch.from_numpy(pt).to(pool.kv.device)
    moved = pool.compact(device_tables=d_pt)
    torch.cuda.synchronize()
    assert moved > 0
    st = pool.stats()
    assert st["high_water"] == st["live_pages"]
    remap = pool.last_remap()
    assert np.array_equal(d_pt.cpu().numpy(), np.where(pt >= 0, remap[np.maximum(pt, 0)], pt))
    for i, s in enumerate(survivors):
        assert pool.page_table(s).tolist() == d_pt[i, :len(tabs[i])].cpu().tolist()
    after = gather(pool, survivors)
    for b, a in zip(before, after):
        assert np.array_equal(b, a)
    assert pool.device_status() == 0
