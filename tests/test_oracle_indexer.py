"""Indexer scoring on the CPU (no GPU): the oracle's restatement of
IndexerPool::select_top_k's scoring (indexer.rs:198-216) against the
reference's own test pools (tests/golden/kat_reference.json), and against a
lane-by-lane float32 restatement in numpy for random rows."""
import json
from pathlib import Path

import numpy as np
import pytest

import oracle

KAT = json.loads((Path(__file__).parent / "golden" / "kat_reference.json").read_text())["indexer_scoring"]


@pytest.mark.parametrize("case", KAT["cases"], ids=lambda c: c["name"])
def test_reference_pools(case):
    n = len(case["row_values"])
    rows = np.repeat(np.array(case["row_values"], np.float32)[:, None], 128, axis=1).reshape(max(n, 0), 128)
    q = np.full((1, 64, 128), case["q"], np.float32)
    w = np.full((1, 64), case["w"], np.float32)
    scores, st = oracle.indexer_scores(rows if n else np.zeros((1, 128), np.float32), np.array([0]), np.array([n]),
                                       q, w, np.array([0]), np.array([n]), max(n, 1))
    assert st == 0
    assert scores[0, :n].tolist() == case["expect_scores"]
    sel = oracle.select_top_k(scores[0, :n], case["k"])
    if "expect_sorted" in case:
        assert sorted(sel.tolist()) == case["expect_sorted"]
    if "expect_len" in case:
        assert len(sel) == case["expect_len"]


def test_scale_factor():
    sf = KAT["scale_factor"]
    v = np.float32(1.0) / np.sqrt(np.float32(64 * 128))
    assert abs(float(v) - sf["approx"]) < sf["tol"]


def _score_np(row, q, w):
    s = np.float32(0.0)
    for h in range(64):
        dot = np.float32(0.0)
        for i in range(128):
            dot = np.float32(dot + np.float32(row[i] * q[h, i]))
        if dot > 0:
            s = np.float32(s + np.float32(dot * w[h]))
    return s


def test_oracle_matches_lane_by_lane_float32():
    rng = np.random.default_rng(3)
    rows = rng.standard_normal((6, 128)).astype(np.float32)
    q = rng.standard_normal((2, 64, 128)).astype(np.float32)
    w = (rng.standard_normal((2, 64)) / np.sqrt(8192)).astype(np.float32)
    scores, st = oracle.indexer_scores(rows, np.array([0, 2]), np.array([2, 4]), q, w, np.array([1, 0]),
                                       np.array([4, 1]), 4)
    assert st == 0
    assert scores[0].tolist() == [_score_np(rows[2 + c], q[0], w[0]) for c in range(4)]
    assert scores[1, 0] == _score_np(rows[0], q[1], w[1]) and np.isneginf(scores[1, 1:]).all()
    _, st = oracle.indexer_scores(rows, np.array([0]), np.array([6]), q[:1], w[:1], np.array([0]), np.array([7]), 8)
    assert st == 1 << oracle.INDEX_OUT_OF_RANGE
