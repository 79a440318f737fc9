"""Indexer scoring + top-k on the GPU (rkv_indexer_scores_f32 /
rkv_indexer_topk_f32) against the oracle: every score bit-exact (rsLLM's
lane-by-lane f32 dots, ReLU, head-by-head weighted sum), the selection equal
to the reference rule on those scores; ragged sequences, causal n_visible
(including 0 and a partial last block), non-positive dots, NaN lanes, and the
out-of-range errors."""
import numpy as np
import pytest
import torch

import rsllm_b200 as rk

pytestmark = pytest.mark.gpu


def _case(rng, seq_rows, queries, scale=1.0):
    n_rows = int(sum(seq_rows))
    rows = (rng.standard_normal((max(n_rows, 1), 128)) * scale).astype(np.float32)
    row_start = np.concatenate([[0], np.cumsum(seq_rows)[:-1]]).astype(np.int64)
    seq_of_query = np.array([s for s, _ in queries], np.int32)
    n_visible = np.array([v for _, v in queries], np.int32)
    n_q = len(queries)
    q = rng.standard_normal((n_q, 64, 128)).astype(np.float32)
    w = (rng.standard_normal((n_q, 64)) / np.sqrt(8192)).astype(np.float32)
    return rows, row_start, np.array(seq_rows, np.int32), q, w, seq_of_query, n_visible


def _check(cuda, orc, args, k):
    rows, row_start, seq_rows, q, w, sq, nv = args
    T = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda)
    max_vis = max(int(nv.max()), 1)
    got = rk.indexer_scores(T(rows), T(row_start), T(seq_rows), T(q), T(w), T(sq), T(nv), max_vis).cpu().numpy()
    want, st = orc.indexer_scores(rows, row_start, seq_rows, q, w, sq, nv, got.shape[1])
    assert st == 0
    for i, v in enumerate(nv):
        assert np.array_equal(got[i, :v].view(np.uint32), want[i, :v].view(np.uint32)), i
    idx = rk.indexer_select_top_k(T(rows), T(row_start), T(seq_rows), T(q), T(w), T(sq), T(nv), max_vis, k)
    want_idx = orc.topk_batch(want, nv, k)
    assert np.array_equal(idx.cpu().numpy(), want_idx)


def test_ragged_sequences_and_causal_visibility(cuda, orc):
    rng = np.random.default_rng(1)
    seq_rows = [1000, 37, 4097, 0, 129]
    queries = [(0, 1000), (0, 500), (1, 37), (2, 4097), (2, 1), (2, 128), (2, 129), (3, 0), (4, 129), (1, 0)]
    _check(cuda, orc, _case(rng, seq_rows, queries), 512)


def test_nonpositive_dots_tie_to_lowest_index(cuda, orc):
    rng = np.random.default_rng(2)
    args = list(_case(rng, [300], [(0, 300), (0, 77)]))
    args[3][:] = -np.abs(args[3])          # q < 0 ...
    args[0][:150] = np.abs(args[0][:150])  # ... rows 0-149 > 0: every dot < 0, score 0
    _check(cuda, orc, args, 64)


def test_nan_lanes_and_large_values(cuda, orc):
    rng = np.random.default_rng(3)
    args = list(_case(rng, [640, 333], [(0, 640), (1, 333), (1, 200)], scale=1e18))
    args[0][5, 17] = np.nan
    args[0][700, :] = np.inf
    _check(cuda, orc, args, 100)


def test_decode_batch_at_scale(cuda, orc):
    rng = np.random.default_rng(4)
    n_seq, n_rows = 8, 8192
    _check(cuda, orc, _case(rng, [n_rows] * n_seq, [(s, n_rows - 13 * s) for s in range(n_seq)]), 512)


def test_index_errors(cuda):
    rng = np.random.default_rng(5)
    rows, row_start, seq_rows, q, w, sq, nv = _case(rng, [100, 50], [(0, 100), (1, 50)])
    T = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda)
    with pytest.raises(rk.IndexOutOfRange):
        rk.indexer_scores(T(rows), T(row_start), T(seq_rows), T(q), T(w), T(np.array([0, 2], np.int32)), T(nv), 100)
    with pytest.raises(rk.IndexOutOfRange):
        rk.indexer_scores(T(rows), T(row_start), T(seq_rows), T(q), T(w), T(sq), T(np.array([101, 50], np.int32)),
                          101)
    with pytest.raises(rk.ShapeMismatch):
        rk.indexer_scores(T(rows[:, :64]), T(row_start), T(seq_rows), T(q), T(w), T(sq), T(nv), 100)
