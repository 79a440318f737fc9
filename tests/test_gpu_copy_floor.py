"""GPU: rkv_copy_floor_bf16, the append's traffic without the codec (the
measurement reference bench.py times beside the append).  Checks that it
touches exactly the bytes of each row's slot that the append writes, with the
byte mapping its header documents, and skips padding slots."""
import numpy as np
import pytest
import torch

import rsllm_b200 as rk
from rsllm_b200._abi import PAGE_BYTES

pytestmark = pytest.mark.gpu

CODES = 64 * 512          # code run of a page
SCALES = CODES + 64 * 32  # start of the RoPE region


def test_copy_floor_moves_the_append_bytes():
    dev = torch.device("cuda:0")
    n_pages, n_layers, n_tok = 16, 2, 300
    pool = rk.PagedKvPool(n_pages, n_layers, device=dev)
    pool.storage.fill_(0xA5)
    g = torch.Generator(device="cpu").manual_seed(7)
    rows = torch.randint(-30000, 30000, (n_layers, n_tok, 576), generator=g, dtype=torch.int16)
    slots = torch.randperm(n_pages * 64, generator=g)[:n_tok].to(torch.int32)
    slots[::17] = -1  # padding tokens
    pool.copy_floor_layer(0, rows.view(torch.bfloat16).to(dev), slots.to(dev))
    torch.cuda.synchronize()
    got = pool.storage.cpu().numpy().reshape(n_layers, n_pages, PAGE_BYTES)
    rb = rows.numpy().view(np.uint8).reshape(n_layers, n_tok, 1152)
    want = np.full_like(got, 0xA5)
    for layer in range(n_layers):
        for t in range(n_tok):
            s = int(slots[t])
            if s < 0:
                continue
            page, off = divmod(s, 64)
            row = rb[layer, t]
            codes = want[layer, page, off * 512:(off + 1) * 512].reshape(32, 16)
            codes[:] = row[:1024].reshape(32, 32)[:, :16]
            scales = want[layer, page, CODES + off * 32:CODES + off * 32 + 32].reshape(8, 4)
            scales[:] = row[:256].reshape(8, 32)[:, 16:20]
            want[layer, page, SCALES + off * 128:SCALES + off * 128 + 128] = row[1024:1152]
    assert np.array_equal(got, want)
