"""GPU MLA decode attention over the FP8 pages (rkv_mla_decode_fp8, tcgen05)
against the oracle's restatement of attention.rs:493-663 and a float64
statement of it, on the same pooled rows and bf16 queries.

Tolerance: the kernel rounds each softmax weight exp2(x - m) to bf16 before
the tensor-core product (relative error <= 2^-9 per weight, the same rounded
weights in numerator and denominator); logits, sums and the output are f32.
A weighted mean with weights perturbed by at most 2^-9 moves by at most
2 * 2^-9 of the largest |value| it averages, so every output lane must be
within 2^-8 of the sequence's largest |latent| of the float64 result; the
mean error is also required to be 16x smaller than that bound."""
import numpy as np
import pytest
import torch

import mla_cases as mc
import rsllm_b200 as rk

pytestmark = pytest.mark.gpu

TOL = 2.0 ** -8


def run_gpu(case, q, sq, idx, sinks, scale, n_splits, cuda):
    pool = rk.PagedKvPool(case["n_pages"], case["n_layers"], device=cuda)
    pool.storage.copy_(torch.from_numpy(case["pool"]).to(cuda))
    qt = torch.from_numpy(q.view(np.int16)).view(torch.bfloat16).to(cuda)
    out = pool.mla_decode(case["layer"], qt, torch.from_numpy(case["pt"]).to(cuda),
                          torch.from_numpy(case["lens"]).to(cuda), torch.from_numpy(sq).to(cuda),
                          None if idx is None else torch.from_numpy(idx).to(cuda),
                          None if sinks is None else torch.from_numpy(sinks).to(cuda), scale, n_splits)
    pool.check("mla_decode")
    return out.cpu().numpy()


def check(orc, case, q, sq, idx, sinks, scale, got, label):
    ref, st = orc.mla_decode(case["pool"], case["n_pages"], case["n_layers"], case["layer"], case["pt"],
                             case["lens"], sq, q, idx, sinks, scale)
    assert st == 0
    f64 = mc.attention_f64(orc, case, q, sq, idx, sinks, scale)
    vs = mc.value_scale(orc, case, sq)[:, None, None]
    e_gpu = np.abs(got - f64) / vs
    e_orc = np.abs(ref - f64) / vs
    print(f"\n{label}: max err / max|v| gpu {e_gpu.max():.3e} (mean {e_gpu.mean():.3e}), "
          f"oracle {e_orc.max():.3e}")
    assert np.all(np.isfinite(got))
    assert e_gpu.max() <= TOL, f"{label}: max error {e_gpu.max()} at {np.unravel_index(e_gpu.argmax(), got.shape)}"
    assert e_gpu.mean() <= TOL / 16


@pytest.mark.parametrize("n_splits", [1, 3])
def test_dense(cuda, orc, n_splits):
    lens = [700, 64, 1, 0, 130]
    case = mc.build(orc, lens, seed=11)
    q, sq = mc.queries(10, len(lens), seed=12)
    got = run_gpu(case, q, sq, None, None, 1 / 24.0, n_splits, cuda)
    check(orc, case, q, sq, None, None, 1 / 24.0, got, f"dense splits={n_splits}")
    assert np.all(got[3] == 0) and np.all(got[8] == 0)  # the empty sequence


def test_dense_sinks_and_sharp_softmax(cuda, orc):
    lens = [1000, 333]
    case = mc.build(orc, lens, seed=13)
    q, sq = mc.queries(4, len(lens), seed=14, scale=4.0)  # large logits: exercises the rescale of O
    sinks = (np.random.default_rng(15).standard_normal(64) * 3).astype(np.float32)
    got = run_gpu(case, q, sq, None, sinks, 1 / 24.0, 1, cuda)
    check(orc, case, q, sq, None, sinks, 1 / 24.0, got, "dense sinks sharp")


@pytest.mark.parametrize("k", [96, 2048])
def test_sparse(cuda, orc, k):
    lens = [4096, 100, 0, 3000]
    case = mc.build(orc, lens, seed=16)
    q, sq = mc.queries(8, len(lens), seed=17)
    idx = mc.index_lists(case["lens"], sq, k, seed=18)
    sinks = np.random.default_rng(19).standard_normal(64).astype(np.float32)
    got = run_gpu(case, q, sq, idx, sinks, 1 / 24.0, 1, cuda)
    check(orc, case, q, sq, idx, sinks, 1 / 24.0, got, f"sparse k={k}")


def test_sparse_from_topk(cuda, orc):
    """The indexer's own output as the mask: top-k of scores where fewer than
    k keys beat -inf, so the list ends in repeated 0s."""
    lens = [500, 2000]
    case = mc.build(orc, lens, seed=20)
    q, sq = mc.queries(4, len(lens), seed=21)
    rng = np.random.default_rng(22)
    k = 256
    scores = rng.standard_normal((4, 2000)).astype(np.float32)
    scores[0, 100:] = -np.inf
    n_vis = np.array([lens[s] for s in sq], np.int32)
    idx = orc.topk_batch(scores, n_vis, k)
    assert (idx[0] == 0).sum() > 1
    got = run_gpu(case, q, sq, idx, None, 1 / 24.0, 1, cuda)
    check(orc, case, q, sq, idx, None, 1 / 24.0, got, "sparse top-k")


@pytest.mark.parametrize("where", ["first_entry", "mid_tile_upper_half", "later_tile", "none"])
def test_sparse_first_zero_only(cuda, orc, where):
    """Only an index list's first 0 is a key; later 0s repeat the top-k fill
    value and are dropped.  The first 0 sits at different rows and tiles
    (including rows 32-63 of a tile and the list's first entry) with more 0s
    before and after tile boundaries; the oracle applies the same rule."""
    lens = [3000, 900]
    case = mc.build(orc, lens, seed=30)
    q, sq = mc.queries(4, len(lens), seed=31)
    k = 320  # five 64-key tiles
    rng = np.random.default_rng(32)
    idx = np.empty((4, k), np.int32)
    for i, s in enumerate(sq):
        row = rng.permutation(np.arange(1, lens[s]))[:k].astype(np.int32)
        first = {"first_entry": 0, "mid_tile_upper_half": 64 + 40, "later_tile": 3 * 64 + 5, "none": None}[where]
        if first is not None:
            row[first] = 0
            for extra in (first + 1, first + 33, first + 70, k - 1):
                if extra < k:
                    row[extra] = 0
        idx[i] = row
    got = run_gpu(case, q, sq, idx, None, 1 / 24.0, 1, cuda)
    check(orc, case, q, sq, idx, None, 1 / 24.0, got, f"sparse first zero {where}")


def test_single_key_returns_its_row_exactly(cuda, orc):
    """With one key the softmax weight is exactly 1, so each head's output is
    that key's latent dequantised to bf16: checked bit for bit against the
    oracle's dequantisation, over every finite E4M3 code and block scales from
    2^-21 (the quantiser's floor) to 2^15 (the two-multiply range), which
    covers the loaders' conversion and the epilogue's column order."""
    n = 64
    page = 43008
    pool = orc.new_pool(n, 1).reshape(n, page)
    codes = (np.arange(n * 512) % 256).astype(np.uint8)
    codes[(codes & 0x7F) == 0x7F] -= 1  # no NaN codes: the quantiser never writes them
    pool[:, :512] = codes.reshape(n, 512)
    exps = (np.arange(n * 8) % 37 - 21).astype(np.int32)  # e = -21 .. 15
    scales = np.ldexp(np.ones(n * 8, np.float32), exps).astype(np.float32)
    pool[:, 64 * 512:64 * 512 + 32] = scales.view(np.uint8).reshape(n, 32)
    rope = np.random.default_rng(30).standard_normal((n, 64))
    pool[:, 64 * 544:64 * 544 + 128] = mc.bf16_bits(rope).view(np.uint8).reshape(n, 128)
    case = dict(pool=pool.reshape(-1), n_pages=n, n_layers=1, layer=0,
                pt=np.arange(n, dtype=np.int32)[:, None], lens=np.ones(n, np.int32))
    q, sq = mc.queries(n, n, seed=31)
    got = run_gpu(case, q, sq, None, None, 1 / 24.0, 1, cuda)
    rows, st = orc.gather_rows(case["pool"], n, 1, 0, case["pt"], np.arange(n + 1, dtype=np.int32))
    assert st == 0
    want = (rows[:, :512].astype(np.uint32) << 16).view(np.float32)  # bf16 -> f32
    # equal as values: the tensor core's f32 sum turns the -0.0 of code 0x80 into +0.0
    assert np.array_equal(got, np.broadcast_to(want[:, None, :], got.shape))
