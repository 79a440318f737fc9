"""GPU parity of the indexer top-k selection against the oracle (which is
itself pinned to rsLLM's repeated best-scan, indexer.rs:218-236): exact index
lists, in order, for N(0,1) scores at the config-4 key count with causal
masking, heavy ties, all-equal scores, NaN / -inf (the repeated index-0 pick),
k above the visible count, and unaligned rows."""
import zlib

import numpy as np
import pytest
import torch

import rsllm_b200 as rk
from rsllm_b200 import synth

pytestmark = pytest.mark.gpu


def run(scores: np.ndarray, n_visible: np.ndarray, k: int, cuda, ld_pad: int = 0):
    n_q, n = scores.shape
    buf = np.zeros((n_q, n + ld_pad), np.float32)
    buf[:, :n] = scores
    s = torch.from_numpy(buf).to(cuda)
    nv = torch.from_numpy(n_visible.astype(np.int32)).to(cuda)
    out = rk.select_top_k(s, nv, k, n_keys_max=n)
    torch.cuda.synchronize()
    return out.cpu().numpy()


def check(orc, scores, n_visible, k, got, scan=False):
    want = orc.topk_batch(scores, n_visible, k, scan=scan)
    bad = np.argwhere(got != want)
    assert bad.shape[0] == 0, f"first mismatch at (q, i) = {bad[0].tolist()}: got {got[tuple(bad[0])]} " \
                              f"want {want[tuple(bad[0])]}"


def test_config4_shape_causal(cuda, orc):
    """64 queries over 131072 keys (the last 64 positions, causal), k = 2048."""
    n, n_q, k = 131072, 64, 2048
    s = synth.scores(n_q, n, seed=5).numpy()
    n_visible = (n - n_q + 1 + np.arange(n_q)).astype(np.int32)
    check(orc, s, n_visible, k, run(s, n_visible, k, cuda))


@pytest.mark.parametrize("case", ["ties", "all_equal", "specials", "few_real", "small", "unaligned", "k_above_n",
                                  "neg_zero"])
def test_edge_cases(cuda, orc, case):
    rng = np.random.default_rng(zlib.crc32(case.encode()))
    n_q, n, k = 8, 20000, 2048
    ld_pad = 0
    if case == "ties":
        s = rng.integers(-5, 6, (n_q, n)).astype(np.float32)
    elif case == "all_equal":
        s = np.full((n_q, n), 1.5, np.float32)
    elif case == "specials":
        s = rng.standard_normal((n_q, n)).astype(np.float32)
        m = rng.random((n_q, n))
        s[m < 0.2] = -np.inf
        s[(m >= 0.2) & (m < 0.3)] = np.nan
        s[(m >= 0.3) & (m < 0.31)] = np.inf
    elif case == "few_real":  # fewer candidates than k beat -inf: index 0 repeats
        s = np.full((n_q, n), -np.inf, np.float32)
        s[:, ::50] = rng.standard_normal((n_q, (n + 49) // 50)).astype(np.float32)
        s[1, :] = np.nan
        s[2, :] = -np.inf
    elif case == "small":
        n, k = 5, 3
        s = rng.standard_normal((n_q, n)).astype(np.float32)
    elif case == "unaligned":
        n = 4099
        s = rng.standard_normal((n_q, n)).astype(np.float32)
        ld_pad = 2  # ld = 4101: not a multiple of 4, scalar-load path
    elif case == "k_above_n":
        n, k = 1000, 2048
        s = rng.standard_normal((n_q, n)).astype(np.float32)
    else:  # neg_zero: -0.0 and +0.0 tie, lowest index first
        s = np.where(rng.random((n_q, n)) < 0.5, np.float32(-0.0), np.float32(0.0)).astype(np.float32)
        s[:, :10] = 1.0
    n_visible = rng.integers(max(1, n // 2), n + 1, n_q).astype(np.int32)
    n_visible[0] = n
    if case != "small":
        n_visible[-1] = 0  # nothing visible -> all -1
    got = run(s, n_visible, k, cuda, ld_pad)
    check(orc, s, n_visible, k, got)
    if case in ("small", "few_real"):  # also against the reference's own scan
        check(orc, s, n_visible, k, got, scan=True)


def test_large_bin_refinement(cuda, orc):
    """Scores packed into one narrow range force the second and third radix
    passes (more than 8192 keys share the top 11 bits)."""
    rng = np.random.default_rng(4)
    n_q, n, k = 4, 65536, 4096
    s = (1.0 + rng.random((n_q, n)) * 1e-3).astype(np.float32)
    s[1] = (1.0 + rng.integers(0, 16, n) * 2.0 ** -23).astype(np.float32)  # only 16 distinct values
    n_visible = np.full(n_q, n, np.int32)
    check(orc, s, n_visible, k, run(s, n_visible, k, cuda))


@pytest.mark.parametrize("k", [4096, 2048, 512, 1])
def test_sampled_threshold_near_the_buffer_size(cuda, orc, k):
    """Rows just above the 8192-key buffer take the sampled-threshold path
    (a 2048-key sample); with k up to the maximum the sample rank and the
    expected candidate count are at their largest.  Also rows sorted
    ascending and rows whose large scores all sit in one region, which the
    evenly spread sample chunks must still bound."""
    rng = np.random.default_rng(100 + k)
    lens = np.array([8193, 8200, 8320, 9000, 12000, 16384, 20000, 24576], np.int32)
    n = int(lens.max())
    s = rng.standard_normal((3 * lens.size, n)).astype(np.float32)
    for i in range(lens.size):
        s[lens.size + i, :lens[i]] = np.sort(s[lens.size + i, :lens[i]])
        r = s[2 * lens.size + i]
        r[:lens[i]] = -np.abs(r[:lens[i]])
        lo = int(lens[i]) // 3
        r[lo:lo + 3000] = np.abs(r[lo:lo + 3000]) + 1.0
    n_visible = np.tile(lens, 3)
    check(orc, s, n_visible, k, run(s, n_visible, k, cuda))
