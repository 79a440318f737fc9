"""GPU parity of the FP8 codec: the device encoder against the oracle for every
f32 lane value up to |512| (both signs), the block exponent for every bf16
block amax, and the device decoder for every finite code under scales from
2^-22 to 2^120.  Bit-exact."""
import numpy as np
import pytest
import torch

import rsllm_b200 as rk
from rsllm_b200 import PAGE_BYTES

pytestmark = pytest.mark.gpu


def u16(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def test_device_encoder_every_f32_up_to_512(cuda, orc):
    hi = 0x44000000  # 512.0: everything above saturates like 448 < x <= 512
    chunk = 1 << 27
    for sign in (0, 0x80000000):
        for first in range(0, hi + 1, chunk):
            n = min(chunk, hi + 1 - first)
            got = rk.e4m3fn_code_range(sign + first, n, device=cuda).cpu().numpy()
            want = orc.e4m3fn_code_range(sign + first, n)
            bad = np.nonzero(got != want)[0]
            assert bad.size == 0, f"code mismatch at f32 bits 0x{sign + first + int(bad[0]):08x}"
    # the largest finite values and a stride through the saturating range (the
    # append path never converts a value above 448; this pins saturation)
    tail = [0x7F7FFFFF, 0xFF7FFFFF]
    for b in tail + list(range(hi, 0x7F800000, 0x100001)) + list(range(0x80000000 + hi, 0xFF800000, 0x100001)):
        got = int(rk.e4m3fn_code_range(b, 1, device=cuda).item())
        assert got == int(orc.e4m3fn_code_range(b, 1)[0]), hex(b)


def test_block_exponent_every_bf16_amax(cuda, orc):
    """Every finite bf16 magnitude is a block amax once; the stored page bytes
    (codes, scales, rope) equal the oracle's."""
    rng = np.random.default_rng(5)
    amax_bits = np.arange(0, 0x7F80, dtype=np.uint32)
    n_blocks = amax_bits.size
    n_rows = (n_blocks + 7) // 8
    rows = np.zeros((n_rows, 576), np.uint16)
    flat = np.zeros((n_rows * 8, 64), np.uint16)
    amax = (amax_bits << 16).view(np.float32)
    frac = rng.uniform(-1, 1, (n_blocks, 64)).astype(np.float32)
    vals = (amax[:, None] * frac).astype(np.float32)
    vb = (vals.view(np.uint32) + 0x7FFF + ((vals.view(np.uint32) >> 16) & 1)) >> 16  # RNE to bf16
    vb = vb.astype(np.uint16)
    mag = vb & 0x7FFF
    vb = np.where(mag > (amax_bits[:, None] & 0x7FFF), (vb & 0x8000) | amax_bits[:, None].astype(np.uint16), vb)
    vb[:, 0] = amax_bits.astype(np.uint16) | np.where(rng.random(n_blocks) < 0.5, 0x8000, 0).astype(np.uint16)
    flat[:n_blocks] = vb
    rows[:, :512] = flat.reshape(n_rows, 512)
    rows[:, 512:] = rng.integers(0, 0x7F80, (n_rows, 64), dtype=np.uint16)

    n_pages = (n_rows + 63) // 64
    slots = rng.permutation(n_pages * 64)[:n_rows].astype(np.int32)
    pool = rk.PagedKvPool(n_pages, 1, device=cuda)
    pool.storage.zero_()
    rows_t = torch.from_numpy(rows.view(np.int16)).view(torch.bfloat16).to(cuda)
    pool.append_layer(0, rows_t, torch.from_numpy(slots).to(cuda))
    pool.check("append")
    ref = orc.new_pool(n_pages, 1)
    assert orc.append_rows(ref, n_pages, 1, 0, rows, slots) == 0
    got = pool.storage.cpu().numpy()
    bad = np.nonzero(got != ref)[0]
    assert bad.size == 0, f"pool bytes differ first at byte {int(bad[0])} (page {int(bad[0]) // PAGE_BYTES})"


def test_device_decoder_every_code_and_scale(cuda, orc):
    """A page filled with every finite code under per-block scales 2^e,
    e in [-22, 120], gathered back, equals the oracle decode."""
    codes = np.tile(np.array([c for c in range(256) if c not in (0x7F, 0xFF)], np.uint8), 200)[: 64 * 512]
    codes = codes.reshape(64, 512)
    exps = np.concatenate([np.arange(-22, 121), np.arange(-22, 121), np.arange(-22, 121), np.arange(-22, 105)])
    exps = exps[: 64 * 8].reshape(64, 8)
    scales = (2.0 ** exps).astype(np.float32)
    rope = np.random.default_rng(3).integers(0, 0xFFFF, (64, 64), dtype=np.uint16)
    page = np.concatenate([codes.reshape(-1), scales.reshape(-1).view(np.uint8), rope.reshape(-1).view(np.uint8)])
    assert page.size == PAGE_BYTES
    pool = rk.PagedKvPool(1, 1, device=cuda)
    pool.storage.copy_(torch.from_numpy(page))
    pt = torch.zeros((1, 1), dtype=torch.int32, device=cuda)
    cu = torch.tensor([0, 64], dtype=torch.int32, device=cuda)
    out = pool.rows(0, pt, cu, 64)
    pool.check("gather")
    want = orc.dequant_rows_bf16(codes, scales, rope)
    got = u16(out)
    bad = np.argwhere(got != want)
    assert bad.shape[0] == 0, f"decode mismatch at row/lane {bad[0].tolist()}: got 0x{got[tuple(bad[0])]:04x} " \
                              f"want 0x{want[tuple(bad[0])]:04x}"
