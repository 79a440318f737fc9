"""Generates tests/golden/fixtures.npz with the CPU oracle (oracle/).

Contents (all seeded, regenerate with `python tests/golden/make_fixtures.py`):
  rows      bf16 bits [64, 576]: 48 N(0,1) rows with 1% x20 outliers + 16 edge rows
  codes     u8  [64, 512]   stored E4M3 codes
  scales    f32 [64, 8]     stored power-of-two block scales
  rope      u16 [64, 64]    stored bf16 RoPE lanes
  dequant   u16 [64, 576]   bf16 read-back
  scores    f32 [8, 3000]   top-k scores (N(0,1), ties, -0.0, NaN, -inf)
  n_visible i32 [8]
  topk      i32 [8, 256]    selected indices (descending score, lowest index on ties, -1 past effective_k)
"""
import sys
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

import oracle  # noqa: E402
from rsllm_b200 import synth  # noqa: E402


def edge_rows() -> np.ndarray:
    r = np.zeros((16, 576), np.uint16)
    r[1, :512] = 0x8000                                   # -0.0
    r[2, :512] = 0x0001                                   # smallest subnormal
    r[3, :512] = 0x8001                                   # -smallest subnormal
    r[4, :512] = 0x7F7F                                   # bf16 max: decodes to +inf
    r[5, :512] = 0xFF7F                                   # -bf16 max: -inf
    r[6, :512] = np.arange(512, dtype=np.uint16) * 63     # magnitudes across the range
    r[7, :512] = 0x3F80
    r[7, 0] = 0x447A                                      # 1000 among 1.0s
    r[8, :512] = (np.arange(512) % 2 * 0x8000 + 0x3A83).astype(np.uint16)
    r[9, :512] = 0x38D1                                   # just below the 1e-4 amax floor
    r[10, :512] = 0x38D2                                  # just above it
    r[11, :512] = 0x7F00                                  # exponent 120
    r[12, :512] = 0x4360                                  # 224.0: amax/448 exactly 2^-1
    r[13, :512] = 0x4361                                  # 225.0
    r[14, :256] = 0x3F80
    r[14, 256:512] = 0xBF80
    r[15, :512] = np.arange(512, dtype=np.uint16) % 128 + 0x3C00
    r[:, 512:] = np.arange(64, dtype=np.uint16) * 1021
    return r


def main():
    rows = np.concatenate([synth.kv_rows(48, seed=2024).view(torch.int16).numpy().view(np.uint16), edge_rows()])
    codes, scales, rope, st = oracle.quantize_rows_bf16(rows)
    assert np.all(st == 0)
    dequant = oracle.dequant_rows_bf16(codes, scales, rope)
    rng = np.random.default_rng(2025)
    scores = rng.standard_normal((8, 3000)).astype(np.float32)
    scores[1] = rng.integers(-3, 4, 3000).astype(np.float32)
    scores[2, rng.random(3000) < 0.3] = -0.0
    scores[3, rng.random(3000) < 0.5] = np.nan
    scores[4, :] = -np.inf
    scores[4, ::40] = 1.0
    scores[5, rng.random(3000) < 0.2] = -np.inf
    n_visible = np.array([3000, 2999, 1500, 3000, 3000, 100, 7, 0], np.int32)
    topk = oracle.topk_batch(scores, n_visible, 256, scan=True)
    np.savez_compressed(Path(__file__).parent / "fixtures.npz", rows=rows, codes=codes, scales=scales, rope=rope,
                        dequant=dequant, scores=scores, n_visible=n_visible, topk=topk)


if __name__ == "__main__":
    main()
