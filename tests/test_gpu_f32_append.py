"""GPU parity of the f32-row append (rkv_append_quant_f32) against the oracle:
the pool bytes equal the oracle's stored form of the same f32 rows, and the
gathered bf16 rows equal rsLLM's own f32 round trip
(fp8_kv_quantize_row_inplace, dsv4_quant.rs:316-362) rounded to bf16 -- on
rows whose block maxima sit at the log2f threshold of every binade, on N(0,1)
rows over several layers, and with padding, out-of-range and non-finite rows."""
import numpy as np
import pytest
import torch

import rsllm_b200 as rk
from test_oracle_f32 import f32_rows_at_thresholds, product_table, reference_roundtrip_f32

pytestmark = pytest.mark.gpu


def u16(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def i32(a, dev) -> torch.Tensor:
    return torch.as_tensor(np.ascontiguousarray(a, np.int32)).to(dev)


def gather_all(pool, n_tok: int, pages: np.ndarray, dev) -> np.ndarray:
    pt = pages.reshape(1, -1).astype(np.int32)
    cu = np.array([0, n_tok], np.int32)
    out = u16(pool.rows(0, i32(pt, dev), i32(cu, dev), n_tok))
    pool.check("gather")
    return out


def test_thresholds_every_binade(cuda, orc):
    rows = f32_rows_at_thresholds(product_table(), seed=1)
    n_tok = rows.shape[0]
    n_pages = (n_tok + 63) // 64
    perm = np.random.default_rng(2).permutation(n_pages).astype(np.int32)
    slots = (perm[np.arange(n_tok) // 64] * 64 + np.arange(n_tok) % 64).astype(np.int32)
    pool = rk.PagedKvPool(n_pages, 1, device=cuda)
    pool.storage.zero_()
    pool.append_layer(0, torch.from_numpy(rows).to(cuda), i32(slots, cuda))
    pool.check("append")
    ref = orc.new_pool(n_pages, 1)
    assert orc.append_rows(ref, n_pages, 1, 0, rows, slots) == 0
    got = pool.storage.cpu().numpy()
    bad = np.nonzero(got != ref)[0]
    assert bad.size == 0, f"{bad.size} pool bytes differ, first at byte {int(bad[0])}"
    assert np.array_equal(gather_all(pool, n_tok, perm, cuda), reference_roundtrip_f32(orc, rows))


def test_multilayer_normal_rows_with_padding(cuda, orc):
    n_pages, n_layers, n_tok = 12, 4, 700
    rng = np.random.default_rng(5)
    rows = rng.standard_normal((3, n_tok, 576)).astype(np.float32)
    rows[:, :, :512] *= np.exp(rng.uniform(-12, 12, (3, n_tok, 8))).repeat(64, axis=2).astype(np.float32)
    slots = rng.permutation(n_pages * 64)[:n_tok].astype(np.int32)
    slots[rng.random(n_tok) < 0.1] = -1
    pool = rk.PagedKvPool(n_pages, n_layers, device=cuda)
    pool.storage.zero_()
    pool.append_layer(1, torch.from_numpy(rows).to(cuda), i32(slots, cuda))
    pool.check("append")
    ref = orc.new_pool(n_pages, n_layers)
    assert orc.append_rows(ref, n_pages, n_layers, 1, rows, slots) == 0
    assert np.array_equal(pool.storage.cpu().numpy(), ref)


def test_bad_rows_write_nothing(cuda, orc):
    n_pages, n_tok = 2, 70
    rng = np.random.default_rng(9)
    rows = rng.standard_normal((n_tok, 576)).astype(np.float32)
    rows[3, 17] = np.nan
    rows[4, 500] = -np.inf
    rows[5, 540] = np.inf      # RoPE lane: stored
    rows[6, 520] = np.nan      # RoPE lane: stored as a quiet NaN
    slots = np.arange(n_tok, dtype=np.int32)
    slots[10] = n_pages * 64   # out of range
    pool = rk.PagedKvPool(n_pages, 1, device=cuda)
    pool.storage.zero_()
    pool.append_layer(0, torch.from_numpy(rows).to(cuda), i32(slots, cuda))
    bits = pool.take_status()
    ref = orc.new_pool(n_pages, 1)
    want = orc.append_rows(ref, n_pages, 1, 0, rows, slots)
    assert bits == want == (1 << rk._abi.RKV_ERR_NON_FINITE_INPUT) | (1 << rk._abi.RKV_ERR_INDEX_OUT_OF_RANGE)
    assert np.array_equal(pool.storage.cpu().numpy(), ref)
    pool.append_layer(0, torch.from_numpy(rows[:3]).to(cuda), i32(slots[:3], cuda))
    pool.check("clean append")
    with pytest.raises(rk.NonFiniteInput):
        pool.append_layer(0, torch.from_numpy(rows[3:4]).to(cuda), i32(slots[3:4], cuda))
        pool.check("append")


@pytest.mark.parametrize("dtype,inputs_ready", [("f32", False), ("bf16", False), ("bf16", True)])
def test_tiny_lanes_next_to_huge_amax(cuda, orc, dtype, inputs_ready):
    """Lanes so small next to their block's amax that v / 2^e underflows: the
    reference's f32 division gives -0.0 or +0.0 and the code is 0x00 either
    way (sign = x < 0); subnormal and tiny negative quotients keep 0x80 where
    they round to a zero magnitude of a negative value."""
    rng = np.random.default_rng(9)
    n_tok = 128
    rows = rng.standard_normal((n_tok, 576)).astype(np.float32)
    big = np.float32(3.0e38) if dtype == "f32" else np.float32(1.0e38)
    for b in range(8):
        blk = rows[:, 64 * b:64 * b + 64]
        blk[:, 0] = big * (1 if b % 2 else -1)
        blk[:, 1:9] = np.array([-1e-30, 1e-30, -1e-38, -1e-40, -1e-45, -3e-7, 2e-9, -2e-9], np.float32)
        blk[:, 9:17] *= np.float32(1e-20)
    if dtype == "bf16":
        b16 = (rows.view(np.uint32) >> 16).astype(np.uint16)  # truncation keeps every class of value
        rows_t = torch.from_numpy(b16.view(np.int16)).view(torch.bfloat16)
        ref_rows = b16
    else:
        rows_t = torch.from_numpy(rows)
        ref_rows = rows
    slots = np.arange(n_tok, dtype=np.int32)
    pool = rk.PagedKvPool(2, 1, device=cuda)
    pool.storage.zero_()
    pool.append_layer(0, rows_t.to(cuda), i32(slots, cuda), inputs_ready=inputs_ready)
    pool.check("append")
    ref = orc.new_pool(2, 1)
    assert orc.append_rows(ref, 2, 1, 0, ref_rows, slots) == 0
    got = pool.storage.cpu().numpy()
    bad = np.nonzero(got != ref)[0]
    assert bad.size == 0, f"{bad.size} pool bytes differ, first at byte {int(bad[0])}: {got[bad[:4]]} vs {ref[bad[:4]]}"
