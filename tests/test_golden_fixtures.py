"""The committed golden fixtures (tests/golden/fixtures.npz, made by
tests/golden/make_fixtures.py with the CPU oracle): the oracle still
reproduces them (CPU), and the CUDA path reproduces them byte for byte (GPU)
-- stored codes, scales and RoPE lanes, bf16 read-back, top-k indices."""
from pathlib import Path

import numpy as np
import pytest
import torch

FIX = np.load(Path(__file__).parent / "golden" / "fixtures.npz")


def test_oracle_reproduces_fixtures(orc):
    codes, scales, rope, st = orc.quantize_rows_bf16(FIX["rows"])
    assert np.all(st == 0)
    assert np.array_equal(codes, FIX["codes"]) and np.array_equal(scales, FIX["scales"])
    assert np.array_equal(rope, FIX["rope"])
    assert np.array_equal(orc.dequant_rows_bf16(codes, scales, rope), FIX["dequant"])
    assert np.array_equal(orc.topk_batch(FIX["scores"], FIX["n_visible"], 256, scan=False), FIX["topk"])


@pytest.mark.gpu
def test_cuda_reproduces_fixtures(cuda):
    import rsllm_b200 as rk

    rows = FIX["rows"]
    n = rows.shape[0]
    pool = rk.PagedKvPool(1, 1, device=cuda)
    pool.storage.zero_()
    slots = torch.arange(n, dtype=torch.int32, device=cuda).flip(0).contiguous()  # reversed slots
    pool.append_layer(0, torch.from_numpy(rows.view(np.int16)).view(torch.bfloat16).to(cuda), slots)
    pool.check("append")
    page = pool.storage.cpu().numpy()
    order = np.arange(n)[::-1]
    codes = page[:32768].reshape(64, 512)[order]
    scales = page[32768:34816].view(np.float32).reshape(64, 8)[order]
    rope = page[34816:].view(np.uint16).reshape(64, 64)[order]
    assert np.array_equal(codes, FIX["codes"])
    assert np.array_equal(scales, FIX["scales"])
    assert np.array_equal(rope, FIX["rope"])
    out = pool.rows(0, torch.zeros((1, 1), dtype=torch.int32, device=cuda),
                    torch.tensor([0, n], dtype=torch.int32, device=cuda), n)
    pool.check("gather")
    got = out.cpu().view(torch.int16).numpy().view(np.uint16)
    assert np.array_equal(got[order], FIX["dequant"])
    idx = rk.select_top_k(torch.from_numpy(FIX["scores"]).to(cuda), torch.from_numpy(FIX["n_visible"]).to(cuda), 256)
    torch.cuda.synchronize()
    assert np.array_equal(idx.cpu().numpy(), FIX["topk"])
