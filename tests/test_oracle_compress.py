"""Compressor emission on the CPU (no GPU): the oracle's restatement of
rsLLM's window state machine, aggregate, RMSNorm and YaRN RoPE is pinned by
the reference's own known-answer tests (tests/golden/kat_reference.json); the
product's host-side pieces -- the RoPE coefficient table and the expf
rounding the kernel uses -- are checked against the oracle, the latter over
every f32 in the aggregate's domain."""
import json
import math
from pathlib import Path

import numpy as np
import pytest

import compress_cases as cc
import oracle
import rsllm_b200 as rk

KAT = json.loads((Path(__file__).parent / "golden" / "kat_reference.json").read_text())


def _f(v):
    return -np.inf if v == "-inf" else float(v)


@pytest.mark.parametrize("case", KAT["compressor"]["cases"], ids=lambda c: c["name"])
def test_window_state_machine_kats(case):
    c = oracle.Compressor(case["ratio"], case["head_dim"])
    feed = c.accumulate if case["wide"] else c.accumulate_narrow
    fin = dict((a, n) for a, n in case.get("finish_prefill", []))
    rows, emit_at, t = [], [], 0
    for kv, score, rep in case["tokens"]:
        for _ in range(rep):
            r = feed(np.array([_f(v) for v in kv], np.float32), np.array([_f(v) for v in score], np.float32))
            if r is not None:
                rows.append(r)
                emit_at.append(t)
            if t in fin:
                c.finish_prefill(fin[t])
            t += 1
    if "emit_at" in case:
        assert emit_at == case["emit_at"]
    if case.get("expect_rows") is not None:
        assert len(rows) == len(case["expect_rows"])
        for got, want in zip(rows, case["expect_rows"]):
            assert np.allclose(got, np.array(want, np.float32), atol=case["tol"], rtol=0), (got, want)
        for lane in case.get("exact_zero_lanes", []):
            assert rows[0][lane] == 0.0
    if "count_after" in case:
        assert int(c.count[0]) == case["count_after"]
        for n, want in case["finish_prefill_counts"]:
            c.finish_prefill(n)
            assert int(c.count[0]) == want


def test_rms_norm_kat():
    k = KAT["compressor"]["rms_norm"]
    c = oracle.Compressor(k["ratio"], k["head_dim"])
    kv = np.full(k["head_dim"], k["kv"], np.float32)
    sc = np.full(k["head_dim"], k["score"], np.float32)
    for pos in range(k["emit_pos"]):
        assert c.accumulate_narrow(kv, sc) is None, pos
    row = c.accumulate_narrow(kv, sc)
    assert row is not None
    oracle.compressor_postprocess(row, np.full(k["head_dim"], k["norm"], np.float32), k["emit_pos"] + 1 - k["ratio"])
    assert np.allclose(row[:k["prefix_lanes"]], k["expect"], atol=k["tol"], rtol=0)


def test_ape_layout_matches_reference_column_read():
    k = KAT["compressor"]["ape_layout"]
    ape = np.arange(k["width"] * k["ratio"], dtype=np.float32).reshape(k["ratio"], k["width"])
    for pos_mod, want in k["columns"]:
        assert ape[pos_mod].tolist() == want  # rkv_compress_append reads ape + (pos % ratio) * width


def _rope_x(expr, n):
    i = np.arange(n, dtype=np.float32)
    return {"i + 1": i + 1, "sin(i * 0.3 - 1)": np.sin(i * np.float32(0.3) - np.float32(1)),
            "cos(i * 0.27 + 0.4)": np.cos(i * np.float32(0.27) + np.float32(0.4)),
            "1": np.ones(n, np.float32)}[expr].astype(np.float32)


@pytest.mark.parametrize("case", KAT["rope"]["cases"], ids=lambda c: c["name"])
def test_rope_kats(case):
    hd, nr = case["head_dim"], case["n_rot"]
    kw = dict(freq_scale=case.get("freq_scale", 1.0), ext_factor=case.get("ext_factor", 0.0))
    x = _rope_x(case["x"], hd).copy()
    orig = x.copy()
    oracle.rope_yarn_tail(x, 1, hd, nr, case["pos"], **kw)
    chk = case["check"]
    if chk == "identity":
        assert np.allclose(x, orig, atol=case["tol"], rtol=0)
    elif chk == "pair_norm":
        n_nope = hd - nr
        assert np.allclose(x[:n_nope], orig[:n_nope], atol=1e-6, rtol=0)
        for i in range(n_nope, hd, 2):
            assert abs(math.hypot(x[i], x[i + 1]) - math.hypot(orig[i], orig[i + 1])) < case["tol"]
    elif chk == "inverse":
        oracle.rope_yarn_tail(x, 1, hd, nr, case["pos"], inverse=True, **kw)
        assert np.allclose(x, orig, atol=case["tol"], rtol=0)
    else:
        assert np.isfinite(x).all()


def test_rope_table_matches_oracle_rotation():
    """The product's host table holds (cos, sin) * mscale of every pair; the
    oracle's rotation of a (1, 0) pair yields exactly (c, s)."""
    for ratio in (4, 128, 1):
        rows = 300
        table = rk.compress_rope_table(ratio, rows)
        ks = list(range(rows)) if ratio != 1 else list(range(0, rows, 7))
        for k in ks:
            x = np.zeros(576, np.float32)
            x[512::2] = 1.0
            oracle.compress_rope(x, k * ratio)
            want = x[512:].reshape(32, 2)
            assert np.array_equal(table[k].view(np.uint32), want.view(np.uint32)), (ratio, k)


def test_rope_table_large_positions_bit_exact():
    table = rk.compress_rope_table(4, 1 << 16)
    rng = np.random.default_rng(3)
    for k in rng.integers(0, 1 << 16, 64):
        x = np.zeros(576, np.float32)
        x[512::2] = 1.0
        oracle.compress_rope(x, int(k) * 4)
        assert np.array_equal(table[k].view(np.uint32), x[512:].reshape(32, 2).view(np.uint32)), k


def test_expf_rounding_matches_libm_on_every_input():
    """Every f32 x in [-150, 0] (and the specials): the kernel's expf (double
    evaluation + correction table, evaluated on the host with the same IEEE
    operations) equals the host libm's expf bit for bit."""
    assert rk.compress_expf_table_size() > 0
    top = int(np.float32(150.0).view(np.uint32))
    chunk = 1 << 25
    for lo in range(0, top + 1, chunk):
        keys = np.arange(lo, min(lo + chunk, top + 1), dtype=np.uint32)
        x = (keys | np.uint32(0x80000000)).view(np.float32)
        got = rk.compress_expf(x)
        want = oracle.expf(x)
        bad = np.nonzero(got.view(np.uint32) != want.view(np.uint32))[0]
        assert bad.size == 0, f"x = {x[bad[:5]]}: {got[bad[:5]]} vs {want[bad[:5]]}"
    sp = np.array([0.0, -np.inf, -151.0, -1e30, np.float32(-0.0)], np.float32)
    assert np.array_equal(rk.compress_expf(sp), oracle.expf(sp))
    assert np.isnan(rk.compress_expf(np.array([np.nan], np.float32)))[0]


def test_batch_driver_matches_primitives():
    """oracle.compress_append (the batched C driver) equals the window state
    machine + post-process + quantize primitives composed token by token."""
    rng = np.random.default_rng(11)
    for ratio in (4, 128, 2):
        coff = 2 if ratio == 4 else 1
        width = coff * 576
        n_states, n_pages = 3, 24
        lens = [2 * ratio + 3, ratio, 5 * ratio - 1]
        pool = oracle.new_pool(n_pages, 1)
        states = oracle.compress_states(n_states, ratio)
        kv = rng.standard_normal((sum(lens), width)).astype(np.float32)
        score = (rng.standard_normal((sum(lens), width)) * 2).astype(np.float32)
        ape = rng.standard_normal((ratio, width)).astype(np.float32)
        norm = rng.uniform(0.5, 1.5, 576).astype(np.float32)
        pos = np.concatenate([np.arange(n) for n in lens]).astype(np.int32)
        state_of = np.concatenate([np.full(n, s) for s, n in enumerate(lens)]).astype(np.int32)
        slot = np.arange(sum(lens), dtype=np.int32)
        st = oracle.compress_append(pool, n_pages, 1, 0, ratio, states, kv, score, pos, state_of, slot, ape, norm)
        assert st == 0
        want = oracle.new_pool(n_pages, 1)
        comps = [oracle.Compressor(ratio) for _ in range(n_states)]
        rows, slots = [], []
        for t in range(sum(lens)):
            r = comps[state_of[t]].accumulate(kv[t], score[t] + ape[pos[t] % ratio])
            if r is not None:
                oracle.compressor_postprocess(r, norm, int(pos[t]) + 1 - ratio)
                rows.append(r)
                slots.append(slot[t])
        assert oracle.append_rows(want, n_pages, 1, 0, np.array(rows, np.float32)[None], np.array(slots)) == 0
        assert np.array_equal(pool, want), ratio


def test_midpoint_row_needs_the_in_order_sum():
    """The constructed row (tests/compress_cases.py): the in-order f64 sum of
    squares and the emission kernels' tree sum give f32 means on either side
    of a rounding midpoint, the tree's mean lies inside the kernels' 2^11-unit
    band (so they redo the sum in order), and the oracle's RMSNorm uses the
    in-order mean."""
    for off in (20, 56, 120):
        row = cc.midpoint_row(off)
        qs, qt = cc.means(row)
        assert np.float32(qs) != np.float32(qt)
        assert cc.mid_distance(qt) <= 1 << 11
        x = row.copy()
        oracle.compressor_postprocess(x, np.ones(576, np.float32), 0)
        rms = np.float32(1.0) / np.sqrt(np.float32(qs) + np.float32(1e-6), dtype=np.float32)
        assert np.array_equal(x[:512], (row[:512] * rms).astype(np.float32))
    # the GPU test's row: one lane's FP8 code tells the two means apart
    row = cc.sensitive_row(oracle.quantize_rows_f32)
    qs, qt = cc.means(row)
    assert np.float32(qs) != np.float32(qt) and cc.mid_distance(qt) <= 1 << 11


def test_indexer_batch_driver_matches_primitives():
    """oracle.indexer_compress_append (the indexer pool's 128-lane step, rows
    out as f32 before the FP4 QAT) equals the same window state machine +
    RMSNorm + RoPE primitives composed token by token on 128-lane rows."""
    rng = np.random.default_rng(12)
    for ratio in (4, 128, 2, 1):
        coff = 2 if ratio == 4 else 1
        width = coff * 128
        n_states = 3
        lens = [2 * ratio + 3, ratio, 5 * ratio - 1]
        states = oracle.indexer_compress_states(n_states, ratio)
        kv = rng.standard_normal((sum(lens), width)).astype(np.float32)
        score = (rng.standard_normal((sum(lens), width)) * 2).astype(np.float32)
        ape = rng.standard_normal((ratio, width)).astype(np.float32)
        norm = rng.uniform(0.5, 1.5, 128).astype(np.float32)
        pos = np.concatenate([np.arange(n) for n in lens]).astype(np.int32)
        state_of = np.concatenate([np.full(n, s) for s, n in enumerate(lens)]).astype(np.int32)
        emit_row = np.arange(sum(lens), dtype=np.int32)[::-1].copy()
        out = np.full((sum(lens), 128), 7.0, np.float32)
        st = oracle.indexer_compress_append(out, ratio, states, kv, score, pos, state_of, emit_row, ape, norm)
        assert st == 0
        want = np.full_like(out, 7.0)
        comps = [oracle.Compressor(ratio, head_dim=128) for _ in range(n_states)]
        for t in range(sum(lens)):
            r = comps[state_of[t]].accumulate(kv[t], score[t] + ape[pos[t] % ratio])
            if r is not None:
                oracle.compressor_postprocess(r, norm, int(pos[t]) + 1 - ratio)
                want[emit_row[t]] = r
        assert np.array_equal(out.view(np.uint32), want.view(np.uint32)), ratio
    # an emit row past the buffer: INDEX_OUT_OF_RANGE, nothing written
    states = oracle.indexer_compress_states(1, 1)
    out = np.zeros((2, 128), np.float32)
    st = oracle.indexer_compress_append(out, 1, states, np.ones((1, 128), np.float32), np.zeros((1, 128), np.float32),
                                        np.zeros(1, np.int32), np.zeros(1, np.int32), np.array([2], np.int32), None,
                                        np.ones(128, np.float32))
    assert st == 1 << oracle.INDEX_OUT_OF_RANGE and not out.any()
