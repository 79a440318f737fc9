"""Compressor emission on the GPU (rkv_compress_append through CompressorBank)
against the oracle's restatement of rsLLM's streaming state machine: the pool
bytes of every emitted row (FP8 codes, scales, bf16 RoPE lanes) are identical
after every call, across prefill chunks, decode steps, states in any order,
ratios 4 (two lanes), 128, 16, 8, 3, 2 and 1, with and without the APE bias, masked
(-inf) and NaN score lanes; errors land in the status word as the oracle's."""
import numpy as np
import pytest
import torch

import compress_cases as cc
import rsllm_b200 as rk

pytestmark = pytest.mark.gpu

SLOTS_PER_STATE = 256


def _run(cuda, orc, ratio, calls, with_ape=True, seed=0, n_states=None, order=None, specials=False):
    rng = np.random.default_rng(seed)
    n_states = n_states or max(len(c) for c in calls)
    coff = 2 if ratio == 4 else 1
    width = coff * 576
    n_pages = n_states * SLOTS_PER_STATE // 64
    pool = rk.PagedKvPool(n_pages, 2, device=cuda)
    pool.storage.zero_()
    bank = rk.CompressorBank(ratio, n_states, device=cuda, max_positions=SLOTS_PER_STATE * ratio)
    ref = orc.new_pool(n_pages, 2)
    ref_states = orc.compress_states(n_states, ratio)
    ape = rng.standard_normal((ratio, width)).astype(np.float32) if with_ape else None
    norm = rng.uniform(0.5, 1.5, 576).astype(np.float32)
    cur = [0] * n_states
    for ci, counts in enumerate(calls):
        states = list(range(len(counts)))
        if order == "reversed" or (order == "alternate" and ci % 2):
            states = states[::-1]
        kv_l, sc_l, pos_l, st_l, slot_l = [], [], [], [], []
        for s in states:
            n = counts[s]
            if n == 0:
                continue
            kv = rng.standard_normal((n, width)).astype(np.float32)
            sc = (rng.standard_normal((n, width)) * 3).astype(np.float32)
            if specials:
                sc[:, 5] = -np.inf            # a lane no token ever scores: aggregate 0
                sc[:, 700 % width] = -np.inf
                sc[rng.random(n) < 0.3, 17] = np.nan
                sc[:, 33] = 80.0 * rng.standard_normal(n)  # far-apart scores: exp underflows to 0
            p = np.arange(cur[s], cur[s] + n)
            cur[s] += n
            kv_l.append(kv)
            sc_l.append(sc)
            pos_l.append(p)
            st_l.append(np.full(n, s))
            slot_l.append(np.where((p + 1) % ratio == 0, s * SLOTS_PER_STATE + (p + 1) // ratio - 1, -1))
        kv, sc = np.concatenate(kv_l), np.concatenate(sc_l)
        pos = np.concatenate(pos_l).astype(np.int32)
        st = np.concatenate(st_l).astype(np.int32)
        slot = np.concatenate(slot_l).astype(np.int32)
        T = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda)
        bank.append(pool, 1, T(kv), T(sc), T(pos), T(st), T(slot), T(norm), None if ape is None else T(ape))
        bits = pool.take_status()
        want_bits = orc.compress_append(ref, n_pages, 2, 1, ratio, ref_states, kv, sc, pos, st, slot, ape, norm)
        assert bits == want_bits, (ci, bits, want_bits)
        got = pool.storage.cpu().numpy()
        if not np.array_equal(got, ref):
            bad = np.nonzero(got != ref)[0]
            raise AssertionError(f"call {ci}: {bad.size} bytes differ, first at {bad[:8]}")
    return pool


@pytest.mark.parametrize("with_ape", [True, False])
def test_ratio4_prefill_then_decode(cuda, orc, with_ape):
    calls = [[37, 8, 1, 0, 13]] + [[1, 1, 1, 1, 1]] * 9 + [[3, 0, 9, 4, 2]] + [[1, 1, 1, 1, 1]] * 4
    _run(cuda, orc, 4, calls, with_ape=with_ape, seed=1, order="alternate")


def test_ratio128_prefill_then_decode(cuda, orc):
    calls = [[300, 127, 1]] + [[1, 1, 1]] * 3 + [[129, 2, 200]] + [[1, 1, 1]] * 2
    _run(cuda, orc, 128, calls, seed=2, order="reversed")


@pytest.mark.parametrize("ratio", [1, 2, 3, 8, 16])
def test_other_ratios(cuda, orc, ratio):
    """Staged windows with padding (1, 2, 3), a full eight-row staged window
    (8) and the first window too long to stage (16: the generic kernel)."""
    _run(cuda, orc, ratio, [[9, 4, 1]] + [[1, 1, 1]] * 5 + [[6, 0, 3]], seed=3 + ratio)


@pytest.mark.parametrize("ratio", [4, 2])
def test_decode_sized_calls_with_multi_token_runs(cuda, orc, ratio):
    """Small calls (at most n_states tokens) in which some states get two or
    three tokens, so part of their ring rows must wait for the call's
    emissions."""
    calls = [[5, 3, 1, 2]] + [[2, 2, 0, 1], [1, 3, 2, 1], [2, 1, 1, 2]] * 4
    _run(cuda, orc, ratio, calls, n_states=8, seed=11 + ratio)


def test_masked_nan_and_underflowing_scores(cuda, orc):
    _run(cuda, orc, 4, [[40, 17, 64]] + [[1, 1, 1]] * 6, seed=7, specials=True)
    _run(cuda, orc, 128, [[256, 130]] + [[1, 1]] * 2, seed=8, specials=True)


def test_many_states_one_call(cuda, orc):
    _run(cuda, orc, 4, [[1024] * 48], seed=9)


def test_non_finite_row_is_rejected(cuda, orc):
    """An emitted row with an infinite latent lane: NON_FINITE_INPUT, not
    written (the oracle stores nothing for it either)."""
    ratio, width = 4, 1152
    pool = rk.PagedKvPool(8, 1, device=cuda)
    pool.storage.zero_()
    bank = rk.CompressorBank(ratio, 1, device=cuda, max_positions=64)
    kv = torch.zeros((4, width), device=cuda)
    kv[:, 600] = float("inf")  # c lane of dim 24
    sc = torch.zeros((4, width), device=cuda)
    pos = torch.arange(4, dtype=torch.int32, device=cuda)
    st = torch.zeros(4, dtype=torch.int32, device=cuda)
    slot = torch.full((4,), 5, dtype=torch.int32, device=cuda)
    bank.append(pool, 0, kv, sc, pos, st, slot, torch.ones(576, device=cuda))
    with pytest.raises(rk.NonFiniteInput):
        pool.check("append")
    assert int(pool.storage.sum().item()) == 0


def test_index_errors(cuda):
    pool = rk.PagedKvPool(2, 1, device=cuda)
    bank = rk.CompressorBank(4, 2, device=cuda, max_positions=8)  # RoPE rows for k = 0, 1, 2
    kv = torch.randn((12, 1152), device=cuda)
    sc = torch.randn((12, 1152), device=cuda)
    norm = torch.ones(576, device=cuda)
    pos = torch.arange(12, dtype=torch.int32, device=cuda)
    st = torch.zeros(12, dtype=torch.int32, device=cuda)
    ok = torch.zeros(12, dtype=torch.int32, device=cuda)
    bank.append(pool, 0, kv, sc, pos, st, ok, norm)
    assert pool.take_status() == 0
    far = torch.full((12,), 64 * 2, dtype=torch.int32, device=cuda)  # page 2 of a 2-page pool
    bank.append(pool, 0, kv[:4], sc[:4], pos[:4] + 12, st[:4], far[:4], norm)  # emits k = 3: no RoPE row
    with pytest.raises(rk.IndexOutOfRange):
        pool.check("rope rows")
    bank2 = rk.CompressorBank(4, 1, device=cuda, max_positions=64)
    bank2.append(pool, 0, kv[:4], sc[:4], pos[:4], st[:4], far[:4], norm)
    with pytest.raises(rk.IndexOutOfRange):
        pool.check("slot")
    bad_state = torch.full((4,), 3, dtype=torch.int32, device=cuda)
    bank2.append(pool, 0, kv[:4], sc[:4], pos[:4], bad_state, ok[:4], norm)
    with pytest.raises(rk.IndexOutOfRange):
        pool.check("state")
    with pytest.raises(rk.ShapeMismatch):
        bank2.append(pool, 0, kv[:4, :576].contiguous(), sc[:4, :576].contiguous(), pos[:4], st[:4], ok[:4], norm)
    with pytest.raises(rk.InvalidLayer):
        bank2.append(pool, 1, kv[:4], sc[:4], pos[:4], st[:4], ok[:4], norm)


def test_device_expf_matches_libm(cuda, orc):
    rng = np.random.default_rng(5)
    top = int(np.float32(150.0).view(np.uint32))
    keys = rng.integers(0, top + 1, 1 << 26, dtype=np.uint32)
    x = (keys | np.uint32(0x80000000)).view(np.float32)
    got = rk.compress_expf(torch.from_numpy(x).to(cuda)).cpu().numpy()
    want = orc.expf(x)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    sp = np.array([0.0, -0.0, -np.inf, -151.0, -1e30], np.float32)
    assert np.array_equal(rk.compress_expf(torch.from_numpy(sp).to(cuda)).cpu().numpy(), orc.expf(sp))


@pytest.mark.parametrize("ratio", [4, 2, 128])
def test_rms_mean_at_an_f32_midpoint(cuda, orc, ratio):
    """An emitted row whose RMSNorm mean the kernels' tree sum would round to
    the other f32 (tests/compress_cases.py), with a lane whose FP8 code tells
    the two means apart: the kernels must redo the sum in rsLLM's order.  One
    finite score per dimension makes the aggregate the row itself.  Ratio 4
    (two lanes) and 2 run the staged kernel, 128 the generic one."""
    width = (2 if ratio == 4 else 1) * 576
    row = cc.sensitive_row(orc.quantize_rows_f32)
    kv = np.zeros((ratio, width), np.float32)
    sc = np.full((ratio, width), -np.inf, np.float32)
    kv[0, width - 576:] = row  # the current window's lanes (the c lanes for ratio 4)
    sc[0, width - 576:] = 0.0
    pos = np.arange(ratio, dtype=np.int32)
    st = np.zeros(ratio, np.int32)
    slot = np.where(pos == ratio - 1, 5, -1).astype(np.int32)
    norm = np.ones(576, np.float32)
    n_pages = 4
    pool = rk.PagedKvPool(n_pages, 2, device=cuda)
    pool.storage.zero_()
    bank = rk.CompressorBank(ratio, 1, device=cuda, max_positions=4 * ratio)
    ref = orc.new_pool(n_pages, 2)
    T = lambda a: torch.from_numpy(a).to(cuda)
    bank.append(pool, 1, T(kv), T(sc), T(pos), T(st), T(slot), T(norm))
    assert pool.take_status() == 0
    assert orc.compress_append(ref, n_pages, 2, 1, ratio, orc.compress_states(1, ratio), kv, sc, pos, st, slot,
                               None, norm) == 0
    got = pool.storage.cpu().numpy()
    assert np.array_equal(got, ref)
    assert got.any()  # the row was written


def test_stalled_wait_ends_in_a_status(cuda):
    """The compressor kernels' bounded wait (rkv_compress_wait_probe): a wait on
    a barrier that nothing arrives on gives up after about a second, leaves
    RKV_ERR_CUDA in the status word instead of hanging, and the context keeps
    working afterwards."""
    import time

    from rsllm_b200 import _abi

    lib = _abi.load()
    st = torch.zeros(1, dtype=torch.int32, device=cuda)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    assert lib.rkv_compress_wait_probe(st.data_ptr(), None) == 0
    torch.cuda.synchronize()
    dt = time.perf_counter() - t0
    assert int(st.item()) == 1 << _abi.RKV_ERR_CUDA
    assert 0.5 < dt < 30.0
    x = torch.arange(1024, dtype=torch.float32, device=cuda)
    assert float(x.sum().item()) == 1023 * 1024 / 2


@pytest.mark.parametrize("ratio", [4, 2, 128])
def test_decode_steps_with_launch_flags(cuda, orc, ratio):
    """Decode steps through rkv_compress_append_ex with
    RKV_COMPRESS_INPUTS_READY | RKV_COMPRESS_ONE_TOKEN_PER_STATE, queued back to
    back on one stream over two pool layers (each call's metadata read while
    the previous call's kernel still runs; one launch per call): the pool
    bytes equal the oracle's after a prefill and every decode step."""
    rng = np.random.default_rng(40 + ratio)
    n_states, coff = 6, (2 if ratio == 4 else 1)
    width = coff * 576
    n_pages = n_states * SLOTS_PER_STATE // 64
    pool = rk.PagedKvPool(n_pages, 2, device=cuda)
    pool.storage.zero_()
    banks = [rk.CompressorBank(ratio, n_states, device=cuda, max_positions=SLOTS_PER_STATE * ratio) for _ in range(2)]
    ref = orc.new_pool(n_pages, 2)
    ref_states = [orc.compress_states(n_states, ratio) for _ in range(2)]
    ape = [rng.standard_normal((ratio, width)).astype(np.float32) for _ in range(2)]
    norm = rng.uniform(0.5, 1.5, 576).astype(np.float32)
    T = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda)  # noqa: E731
    prefill = 3 * ratio + 1
    stream = torch.cuda.Stream(device=cuda)
    calls = []
    for step in range(1 + 2 * ratio + 3):
        n = prefill if step == 0 else 1
        p0 = 0 if step == 0 else prefill + step - 1
        pos = np.tile(np.arange(p0, p0 + n), n_states).astype(np.int32)
        st = np.repeat(np.arange(n_states), n).astype(np.int32)
        slot = np.where((pos + 1) % ratio == 0, st * SLOTS_PER_STATE + (pos + 1) // ratio - 1, -1).astype(np.int32)
        for layer in range(2):
            kv = rng.standard_normal((n * n_states, width)).astype(np.float32)
            sc = (rng.standard_normal((n * n_states, width)) * 3).astype(np.float32)
            calls.append((layer, kv, sc, pos, st, slot, step > 0))
    dev_calls = [(layer, T(kv), T(sc), T(pos), T(st), T(slot), flags) for layer, kv, sc, pos, st, slot, flags in calls]
    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        for layer, kv, sc, pos, st, slot, decode in dev_calls:
            banks[layer].append(pool, layer, kv, sc, pos, st, slot, T(norm), T(ape[layer]), stream=stream,
                                inputs_ready=decode, one_token_per_state=decode)
    assert pool.take_status(stream) == 0
    for layer, kv, sc, pos, st, slot, _ in calls:
        assert orc.compress_append(ref, n_pages, 2, layer, ratio, ref_states[layer], kv, sc, pos, st, slot,
                                   ape[layer], norm) == 0
    got = pool.storage.cpu().numpy()
    assert np.array_equal(got, ref), f"{int((got != ref).sum())} bytes differ"


def test_one_token_flag_reports_a_repeated_state(cuda):
    """Two tokens of one state in a call made with
    RKV_COMPRESS_ONE_TOKEN_PER_STATE: the deferred ring write is reported as
    INVALID_ARGUMENT in the status word."""
    pool = rk.PagedKvPool(4, 1, device=cuda)
    bank = rk.CompressorBank(4, 2, device=cuda, max_positions=64)
    kv = torch.randn((3, 1152), device=cuda)
    sc = torch.randn((3, 1152), device=cuda)
    pos = torch.tensor([0, 1, 0], dtype=torch.int32, device=cuda)
    st = torch.tensor([0, 0, 1], dtype=torch.int32, device=cuda)
    slot = torch.full((3,), -1, dtype=torch.int32, device=cuda)
    bank.append(pool, 0, kv, sc, pos, st, slot, torch.ones(576, device=cuda), one_token_per_state=True)
    assert pool.take_status() == 1 << rk.InvalidArgument.status
