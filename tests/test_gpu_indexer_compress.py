"""The indexer pool's compressor emission on the GPU
(rkv_indexer_compress_append through IndexerCompressorBank) against the
oracle's restatement of rsLLM's streaming state machine on 128-lane rows
(attention.rs:405-429 -> compressor.rs:264-330): every emitted f32 row is
bit-identical after every call, across prefill chunks, decode steps, ratios
4 (two lanes), 128, 16, 2 and 1, with and without the APE bias, masked and
NaN score lanes.  Then the device chain the indexer runs: emitted rows ->
rkv_indexer_topk_f32 (scores + top-k) against the oracle's scoring
(indexer.rs:198-216) and the reference's selection on the oracle's rows."""
import numpy as np
import pytest
import torch

import rsllm_b200 as rk

pytestmark = pytest.mark.gpu

ROWS_PER_STATE = 256


def _run(cuda, orc, ratio, calls, with_ape=True, seed=0, specials=False, rows_per_state=ROWS_PER_STATE):
    rng = np.random.default_rng(seed)
    n_states = max(len(c) for c in calls)
    coff = 2 if ratio == 4 else 1
    width = coff * 128
    n_rows = n_states * rows_per_state
    bank = rk.IndexerCompressorBank(ratio, n_states, device=cuda, max_positions=rows_per_state * ratio)
    out = torch.full((n_rows, 128), 3.0, dtype=torch.float32, device=cuda)
    ref = np.full((n_rows, 128), 3.0, np.float32)
    ref_states = orc.indexer_compress_states(n_states, ratio)
    ape = rng.standard_normal((ratio, width)).astype(np.float32) if with_ape else None
    norm = rng.uniform(0.5, 1.5, 128).astype(np.float32)
    cur = [0] * n_states
    T = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda)  # noqa: E731
    for ci, counts in enumerate(calls):
        kv_l, sc_l, pos_l, st_l, row_l = [], [], [], [], []
        for s, n in enumerate(counts):
            if n == 0:
                continue
            kv = rng.standard_normal((n, width)).astype(np.float32)
            sc = (rng.standard_normal((n, width)) * 3).astype(np.float32)
            if specials:
                sc[:, 5] = -np.inf
                sc[rng.random(n) < 0.3, 17] = np.nan
                sc[:, 33] = 80.0 * rng.standard_normal(n)
            p = np.arange(cur[s], cur[s] + n)
            cur[s] += n
            kv_l.append(kv)
            sc_l.append(sc)
            pos_l.append(p)
            st_l.append(np.full(n, s))
            row_l.append(np.where((p + 1) % ratio == 0, s * rows_per_state + (p + 1) // ratio - 1, -1))
        kv, sc = np.concatenate(kv_l), np.concatenate(sc_l)
        pos = np.concatenate(pos_l).astype(np.int32)
        st = np.concatenate(st_l).astype(np.int32)
        row = np.concatenate(row_l).astype(np.int32)
        bank.append(out, T(kv), T(sc), T(pos), T(st), T(row), T(norm), None if ape is None else T(ape))
        bits = bank.take_status()
        want_bits = orc.indexer_compress_append(ref, ratio, ref_states, kv, sc, pos, st, row, ape, norm)
        assert bits == want_bits, (ci, bits, want_bits)
        got = out.cpu().numpy()
        bad = np.nonzero(got.view(np.uint32) != ref.view(np.uint32))
        assert bad[0].size == 0, f"call {ci}: {bad[0].size} lanes differ, first rows {bad[0][:4]} lanes {bad[1][:4]}"
    return out, ref, cur


@pytest.mark.parametrize("with_ape", [True, False])
def test_ratio4_prefill_then_decode(cuda, orc, with_ape):
    calls = [[37, 8, 1, 0, 13]] + [[1, 1, 1, 1, 1]] * 9 + [[3, 0, 9, 4, 2]] + [[1, 1, 1, 1, 1]] * 4
    _run(cuda, orc, 4, calls, with_ape=with_ape, seed=1)


@pytest.mark.parametrize("ratio", [1, 2, 16, 128])
def test_other_ratios(cuda, orc, ratio):
    _run(cuda, orc, ratio, [[3 * ratio + 1, 4, 1]] + [[1, 1, 1]] * 5 + [[ratio + 2, 0, 3]], seed=3 + ratio)


def test_masked_nan_and_underflowing_scores(cuda, orc):
    _run(cuda, orc, 4, [[40, 17, 64]] + [[1, 1, 1]] * 6, seed=7, specials=True)


def test_emitted_rows_feed_scoring_and_top_k(cuda, orc):
    """Prefill of 4 sequences (ratio 4) on the device, then the indexer's
    scoring and top-k over the emitted rows: indices equal the oracle's
    scoring + the reference's selection on the oracle's rows."""
    n_seq, per, k = 4, 4096, 512
    n_rows = per // 4
    # each sequence's emitted rows are one contiguous span of the buffer:
    # the packed row layout the scoring reads (row_start = s * n_rows)
    out, ref, cur = _run(cuda, orc, 4, [[per] * n_seq], seed=21, rows_per_state=n_rows)
    rng = np.random.default_rng(22)
    q = rng.standard_normal((n_seq, 64, 128)).astype(np.float32)
    w = (rng.standard_normal((n_seq, 64)) / 90.0).astype(np.float32)
    seq_rows = np.full(n_seq, n_rows, np.int32)
    nv = np.array([n_rows, n_rows - 1, 700, 1], np.int32)
    T = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda)  # noqa: E731
    rows_buf, ref_buf = out, ref
    row_start = (np.arange(n_seq) * n_rows).astype(np.int64)
    sq = np.arange(n_seq, dtype=np.int32)
    idx = rk.indexer_select_top_k(rows_buf, T(row_start), T(seq_rows), T(q), T(w), T(sq), T(nv), n_rows, k)
    scores, st = orc.indexer_scores(ref_buf, row_start, seq_rows, q, w, sq, nv, n_rows)
    assert st == 0
    want = np.full((n_seq, k), -1, np.int32)
    for i in range(n_seq):
        sel = orc.select_top_k(scores[i, :nv[i]], k)
        want[i, :sel.size] = sel
    assert np.array_equal(idx.cpu().numpy(), want)
