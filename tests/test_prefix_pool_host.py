"""The C++ pool's host rules (page allocator, page tables, radix prefix store,
copy-on-write, LRU eviction, compaction) against the independent Python model
in oracle/prefix_model.py, decision by decision, on a plan-only pool (no GPU):
every return value, page table, refcount, statistic and page move must match.
"""
import random

import numpy as np
import pytest

import rsllm_b200 as rk
from oracle.prefix_model import OutOfRange, PoolFull, PrefixModel
from rsllm_b200.prefix_pool import PrefixKvPool


def compare(pool: PrefixKvPool, model: PrefixModel, live: dict):
    assert pool.stats() == model.stats()
    assert np.array_equal(pool.refcounts(), np.array(model.ref, np.int32))
    for s in live:
        assert pool.page_table(s).tolist() == model.page_table(s), s
        assert pool.seq_len(s) == model.seqs[s].len
    src, dst = pool.take_moves()
    assert list(zip(src.tolist(), dst.tolist())) == model.take_moves()


def run_ops(seed: int, n_pages: int, n_ops: int, vocab: int):
    rng = random.Random(seed)
    pool = PrefixKvPool(n_pages, 1, device=None)
    model = PrefixModel(n_pages)
    toks: dict[int, list[int]] = {}  # token ids of every live sequence

    def both(fn_pool, fn_model):
        try:
            a = fn_pool()
            ea = None
        except rk.KvError as e:
            a, ea = None, type(e)
        try:
            b = fn_model()
            eb = None
        except (PoolFull, OutOfRange) as e:
            b, eb = None, type(e)
        want = {PoolFull: rk.PoolFull, OutOfRange: rk.IndexOutOfRange, None: None}[eb]
        assert ea is want, (ea, eb)
        return a, b

    for step in range(n_ops):
        op = rng.choices(["create", "reserve", "fork", "insert", "match", "release", "touch", "free", "evict",
                          "compact"], weights=[6, 20, 8, 8, 8, 5, 3, 3, 3, 2])[0]
        seqs = sorted(toks)
        if op == "create" or not seqs:
            a, b = both(pool.create_sequence, model.create)
            assert a == b
            toks[a] = []
        elif op == "reserve":
            k = rng.randint(1, min(4, len(seqs)))
            chosen = rng.sample(seqs, k)
            ns = [rng.choice([0, 1, 5, 63, 64, 65, 130, 200]) for _ in chosen]
            a, b = both(lambda: pool.reserve(chosen, ns), lambda: model.reserve(chosen, ns))
            if a is not None:
                assert a.tolist() == b
                for s, n in zip(chosen, ns):
                    toks[s] += [rng.randrange(vocab) for _ in range(n)]
        elif op == "fork":
            s = rng.choice(seqs)
            n = rng.randint(0, len(toks[s]))
            a, b = both(lambda: pool.fork(s, n), lambda: model.fork(s, n))
            assert a == b
            toks[a] = toks[s][:n]
        elif op == "insert":
            s = rng.choice(seqs)
            n = rng.randint(0, len(toks[s]))
            both(lambda: pool.insert_prefix(toks[s][:n], s), lambda: model.insert(toks[s][:n], s))
        elif op == "match":
            s = rng.choice(seqs)
            n = rng.randint(0, len(toks[s]))
            q = toks[s][:n] + [rng.randrange(vocab) for _ in range(rng.randint(0, 70))]
            a, b = both(lambda: pool.match_prefix(q), lambda: model.match(q))
            assert a == b
            toks[a[1]] = q[:a[0]]
        elif op == "release":
            s = rng.choice(seqs)
            both(lambda: pool.release(s), lambda: model.release(s))
        elif op == "touch":
            s = rng.choice(seqs)
            both(lambda: pool.touch(s), lambda: model.touch(s))
        elif op == "free":
            s = rng.choice(seqs)
            both(lambda: pool.free(s), lambda: model.free(s))
            del toks[s]
        elif op == "evict":
            t = rng.randint(1, max(1, n_pages // 3))
            a, b = both(lambda: pool.evict(t), lambda: model.evict(t))
            assert a == b
            for s in list(toks):
                if s not in model.seqs:
                    del toks[s]
        else:
            a, b = both(pool.compact, model.compact)
            assert a == sum(1 for i, r in enumerate(b) if r != i)
            assert pool.last_remap().tolist() == b
        compare(pool, model, toks)
    pool.close()


@pytest.mark.parametrize("seed", range(12))
def test_random_operations_match_model(seed):
    run_ops(seed, n_pages=[48, 96, 256][seed % 3], n_ops=400, vocab=[2, 3, 50][seed % 3])


def test_unknown_sequence_and_bad_lengths():
    pool = PrefixKvPool(8, 1, device=None)
    s = pool.create_sequence()
    pool.reserve([s], [10])
    with pytest.raises(rk.IndexOutOfRange):
        pool.fork(s, 11)
    with pytest.raises(rk.IndexOutOfRange):
        pool.fork(99, 0)
    with pytest.raises(rk.IndexOutOfRange):
        pool.insert_prefix(list(range(11)), s)
    with pytest.raises(rk.PoolFull):
        pool.reserve([s], [8 * 64])
    assert pool.seq_len(s) == 10  # all-or-nothing
    with pytest.raises(rk.InvalidArgument):
        pool.reserve([s, s], [1, 1])


def test_config5_shape_small():
    """Config 5 in miniature: a shared prefix of 8192 + r tokens in the radix
    store, branches that match it (sharing its partial last page), copy it on
    write and append 2048 tokens each, then LRU eviction of 30% of the used
    pages and compaction -- C++ and model agree on every page."""
    r = 37
    prefix = list(range(8192 + r))
    n_pages = 4096
    pool = PrefixKvPool(n_pages, 1, device=None)
    model = PrefixModel(n_pages)
    rng = random.Random(6)
    for impl in (pool, model):  # background residents, released with LRU stamps
        pass
    bg = []
    for i in range(12):
        a = pool.create_sequence()
        b = model.create()
        assert a == b
        n = rng.randint(1024, 8192)
        assert pool.reserve([a], [n]).tolist() == model.reserve([b], [n])
        bg.append(a)
    for s in bg:
        pool.release(s)
        model.release(s)
    owner = pool.create_sequence()
    assert owner == model.create()
    assert pool.reserve([owner], [len(prefix)]).tolist() == model.reserve([owner], [len(prefix)])
    pool.insert_prefix(prefix, owner)
    model.insert(prefix, owner)
    pool.free(owner)
    model.free(owner)
    branches = []
    for i in range(16):
        a = pool.match_prefix(prefix)
        b = model.match(prefix)
        assert a == b and a[0] == len(prefix)
        branches.append(a[1])
    ns = [2048] * len(branches)
    assert pool.reserve(branches, ns).tolist() == model.reserve(branches, ns)
    src, dst = pool.take_moves()
    mv = model.take_moves()
    assert list(zip(src.tolist(), dst.tolist())) == mv
    assert len(mv) == 16  # every branch copied the shared partial page
    used = pool.stats()["live_pages"]
    t = int(0.3 * used)
    assert pool.evict(t) == model.evict(t)
    assert pool.compact() == sum(1 for i, x in enumerate(model.compact()) if x != i)
    compare(pool, model, {s: None for s in branches})
    st = pool.stats()
    assert st["high_water"] == st["live_pages"]
