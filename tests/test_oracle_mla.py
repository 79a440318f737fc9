"""The oracle's MLA decode attention (the f32 restatement of
attention.rs:493-663 over pooled rows) against an independent float64
statement of the same rule: dense and sparse key sets, sinks, the repeated-0
and out-of-range index entries, empty sequences."""
import numpy as np
import pytest

import mla_cases as mc


@pytest.mark.parametrize("mode", ["dense", "sparse", "sparse_sinks"])
def test_oracle_matches_float64(orc, mode):
    lens = [150, 70, 0, 64]
    case = mc.build(orc, lens, seed=3)
    q, sq = mc.queries(8, len(lens), seed=4)
    idx = mc.index_lists(case["lens"], sq, 96, seed=5) if mode != "dense" else None
    sinks = np.random.default_rng(6).standard_normal(64).astype(np.float32) if mode == "sparse_sinks" else None
    scale = 1.0 / 24.0
    got, st = orc.mla_decode(case["pool"], case["n_pages"], case["n_layers"], case["layer"], case["pt"],
                             case["lens"], sq, q, idx, sinks, scale)
    assert st == 0
    want = mc.attention_f64(orc, case, q, sq, idx, sinks, scale)
    vs = mc.value_scale(orc, case, sq)
    err = np.abs(got - want).max(axis=(1, 2)) / vs
    assert np.all(err < 1e-5), err
    # a query of the empty sequence: zeros without a sink, zeros with one too
    assert np.all(got[2] == 0) and np.all(got[6] == 0)


def test_oracle_bad_page_is_skipped(orc):
    case = mc.build(orc, [100], seed=7)
    case["pt"][0, 1] = case["n_pages"] + 5  # rows 64..99 on a page outside the pool
    q, sq = mc.queries(1, 1, seed=8)
    got, st = orc.mla_decode(case["pool"], case["n_pages"], case["n_layers"], case["layer"], case["pt"],
                             case["lens"], sq, q, None, None, 0.05)
    assert st == 1 << orc.INDEX_OUT_OF_RANGE
    only = dict(case, lens=np.array([64], np.int32))
    want, _ = orc.mla_decode(only["pool"], only["n_pages"], only["n_layers"], only["layer"], only["pt"],
                             only["lens"], sq, q, None, None, 0.05)
    assert np.array_equal(got, want)
