"""GPU parity of the KV-cache path against the CPU oracle: quantize-on-append,
paged gather, sparse gather and page moves, bit-exact on the bytes of the pool
and on every bf16 output lane; plus the error behaviour (status bits and the
rsLLM-named exceptions) on bad slots, bad page ids, non-finite rows and bad
layers."""
import numpy as np
import pytest
import torch

import rsllm_b200 as rk
from rsllm_b200 import synth

pytestmark = pytest.mark.gpu


def u16(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def bf16_dev(a: np.ndarray, dev) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(torch.bfloat16).to(dev)


def i32(a, dev) -> torch.Tensor:
    return torch.as_tensor(np.ascontiguousarray(a, np.int32)).to(dev)


def f32_to_bf16(x: np.ndarray) -> np.ndarray:
    b = x.astype(np.float32).view(np.uint32)
    return ((b + 0x7FFF + ((b >> 16) & 1)) >> 16).astype(np.uint16)


def reference_roundtrip(orc, rows: np.ndarray) -> np.ndarray:
    """rsLLM's f32 round trip (fp8_kv_quantize_row_inplace(row, 576, 64)) of
    each bf16 row, rounded to bf16; the rope lanes pass through."""
    out = np.empty_like(rows)
    for i in range(rows.shape[0]):
        x = (rows[i].astype(np.uint32) << 16).view(np.float32).copy()
        assert orc.quantize_row_inplace(x, 576, 64) == orc.OK
        out[i] = f32_to_bf16(x)
        out[i, 512:] = rows[i, 512:]
    return out


def test_config1_roundtrip(cuda, orc):
    """Config 1: 1 layer, 4096 tokens, 64-token pages in a seeded random
    physical order; append, gather back; pool bytes and bf16 output equal
    the oracle, and the output equals rsLLM's own f32 round trip."""
    n_tok, n_pages = 4096, 64
    rows = u16(synth.kv_rows(n_tok, seed=1))
    perm = synth.permutation(n_pages, seed=2).numpy()
    slots = (perm[np.arange(n_tok) // 64] * 64 + np.arange(n_tok) % 64).astype(np.int32)
    pool = rk.PagedKvPool(n_pages, 1, device=cuda)
    pool.storage.zero_()
    pool.append_layer(0, bf16_dev(rows, cuda), i32(slots, cuda))
    pool.check("append")
    ref = orc.new_pool(n_pages, 1)
    assert orc.append_rows(ref, n_pages, 1, 0, rows, slots) == 0
    assert np.array_equal(pool.storage.cpu().numpy(), ref)

    pt = perm.reshape(1, -1).astype(np.int32)
    cu = np.array([0, n_tok], np.int32)
    out = u16(pool.rows(0, i32(pt, cuda), i32(cu, cuda), n_tok))
    pool.check("gather")
    want, st = orc.gather_rows(ref, n_pages, 1, 0, pt, cu)
    assert st == 0
    assert np.array_equal(out, want)
    assert np.array_equal(out, reference_roundtrip(orc, rows))


def test_multilayer_append_shared_slots_and_padding(cuda, orc):
    n_pages, n_layers, n_tok = 9, 5, 300
    rng = np.random.default_rng(1)
    rows = u16(synth.kv_rows(3 * n_tok, seed=3)).reshape(3, n_tok, 576)
    slots = rng.permutation(n_pages * 64)[:n_tok].astype(np.int32)
    slots[rng.random(n_tok) < 0.1] = -1  # padding tokens are skipped
    pool = rk.PagedKvPool(n_pages, n_layers, device=cuda)
    pool.storage.zero_()
    pool.append_layer(1, bf16_dev(rows, cuda), i32(slots, cuda))
    pool.check("append")
    ref = orc.new_pool(n_pages, n_layers)
    assert orc.append_rows(ref, n_pages, n_layers, 1, rows, slots) == 0
    assert np.array_equal(pool.storage.cpu().numpy(), ref)


def test_append_rejects_bad_rows_without_writing(cuda, orc):
    n_pages = 2
    rows = u16(synth.kv_rows(6, seed=4))
    rows[1, 100] = 0x7FC0  # NaN latent -> NonFiniteInput, row skipped
    rows[2, 511] = 0xFF80  # -inf latent
    rows[3, 530] = 0x7F80  # inf rope: stored as is
    slots = np.array([0, 1, 2, 3, n_pages * 64, 5], np.int32)  # slot 128 is out of range
    pool = rk.PagedKvPool(n_pages, 1, device=cuda)
    pool.storage.zero_()
    pool.append_layer(0, bf16_dev(rows, cuda), i32(slots, cuda))
    bits = pool.take_status()
    assert bits == (1 << rk.IndexOutOfRange.status) | (1 << rk.NonFiniteInput.status)
    ref = orc.new_pool(n_pages, 1)
    st = orc.append_rows(ref, n_pages, 1, 0, rows, slots)
    assert st == bits
    assert np.array_equal(pool.storage.cpu().numpy(), ref)
    # the rsLLM-named error surfaces through check()
    pool.append_layer(0, bf16_dev(rows[1:2], cuda), i32([7], cuda))
    with pytest.raises(rk.NonFiniteInput):
        pool.check("append")


def test_append_host_errors(cuda):
    pool = rk.PagedKvPool(2, 3, device=cuda)
    rows = synth.kv_rows(4, seed=5).to(cuda)
    slots = torch.arange(4, dtype=torch.int32, device=cuda)
    with pytest.raises(rk.InvalidLayer):
        pool.append_layer(3, rows, slots)
    with pytest.raises(rk.InvalidLayer):
        pool.append_layer(2, rows.unsqueeze(0).expand(2, 4, 576).contiguous(), slots)
    with pytest.raises(rk.ShapeMismatch):
        pool.append_layer(0, rows[:, :512].contiguous(), slots)
    with pytest.raises(rk.ShapeMismatch):
        pool.append_layer(0, rows, slots[:3])
    with pytest.raises(rk.ShapeMismatch):  # bf16 and f32 rows only
        pool.append_layer(0, rows.half(), slots)


def build_paged(orc, cuda, lens, n_layers=2, seed=7):
    """Sequences of the given lengths appended into a shared pool with a
    seeded random physical page order; returns everything both sides need."""
    rng = np.random.default_rng(seed)
    pages_per = [(n + 63) // 64 for n in lens]
    n_pages = max(1, sum(pages_per))
    stride = max(1, max(pages_per))
    perm = rng.permutation(n_pages).astype(np.int32)
    pt = np.full((len(lens), stride), -1, np.int32)
    c = 0
    for s, p in enumerate(pages_per):
        pt[s, :p] = perm[c:c + p]
        c += p
    tot = int(sum(lens))
    rows = u16(synth.kv_rows(n_layers * max(tot, 1), seed=seed)).reshape(n_layers, max(tot, 1), 576)[:, :tot]
    rows = np.ascontiguousarray(rows)
    slots = np.concatenate([pt[s, np.arange(n) // 64] * 64 + np.arange(n) % 64 for s, n in enumerate(lens)]) \
        if tot else np.zeros(0, np.int32)
    slots = slots.astype(np.int32)
    pool = rk.PagedKvPool(n_pages, n_layers, device=cuda)
    pool.storage.zero_()
    ref = orc.new_pool(n_pages, n_layers)
    if tot:
        pool.append_layer(0, bf16_dev(rows, cuda), i32(slots, cuda))
        pool.check("append")
        assert orc.append_rows(ref, n_pages, n_layers, 0, rows, slots) == 0
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    return pool, ref, n_pages, pt, cu


def test_gather_ragged_and_empty_sequences(cuda, orc):
    lens = [1, 64, 65, 0, 130, 7, 1000, 63]
    pool, ref, n_pages, pt, cu = build_paged(orc, cuda, lens)
    for layer in (0, 1):
        out = u16(pool.rows(layer, i32(pt, cuda), i32(cu, cuda), max(lens)))
        pool.check("gather")
        want, st = orc.gather_rows(ref, n_pages, 2, layer, pt, cu)
        assert st == 0
        assert np.array_equal(out, want)


def test_gather_bad_page_id_zero_fills(cuda, orc):
    lens = [200, 100]
    pool, ref, n_pages, pt, cu = build_paged(orc, cuda, lens)
    pt = pt.copy()
    pt[0, 1] = n_pages + 5  # corrupt entry
    out = u16(pool.rows(0, i32(pt, cuda), i32(cu, cuda), 200))
    with pytest.raises(rk.IndexOutOfRange):
        pool.check("gather")
    want, st = orc.gather_rows(ref, n_pages, 2, 0, pt, cu)
    assert st == 1 << rk.IndexOutOfRange.status
    assert np.array_equal(out, want)
    assert np.all(out[64:128] == 0)
    with pytest.raises(rk.InvalidLayer):
        pool.rows(2, i32(pt, cuda), i32(cu, cuda), 200)


def test_sparse_gather(cuda, orc):
    lens = [700, 1, 300, 129]
    pool, ref, n_pages, pt, cu = build_paged(orc, cuda, lens, seed=9)
    rng = np.random.default_rng(2)
    n_q, k = 37, 50
    seq_of_query = rng.integers(0, len(lens), n_q).astype(np.int32)
    idx = np.stack([rng.integers(0, lens[s], k) for s in seq_of_query]).astype(np.int32)
    idx[rng.random(idx.shape) < 0.05] = -1  # unused selections -> zero rows
    seq_lens = np.array(lens, np.int32)
    out = u16(pool.sparse_rows(1, i32(pt, cuda), i32(seq_of_query, cuda), i32(seq_lens, cuda), i32(idx, cuda)))
    pool.check("sparse")
    want, st = orc.sparse_gather_rows(ref, n_pages, 2, 1, pt, seq_of_query, seq_lens, idx)
    assert st == 0
    assert np.array_equal(out, want)
    # a position past the sequence end: IndexOutOfRange and a zero row
    idx[3, 4] = lens[seq_of_query[3]]
    out = u16(pool.sparse_rows(1, i32(pt, cuda), i32(seq_of_query, cuda), i32(seq_lens, cuda), i32(idx, cuda)))
    with pytest.raises(rk.IndexOutOfRange):
        pool.check("sparse")
    want, st = orc.sparse_gather_rows(ref, n_pages, 2, 1, pt, seq_of_query, seq_lens, idx)
    assert st == 1 << rk.IndexOutOfRange.status
    assert np.array_equal(out, want) and np.all(out[3, 4] == 0)


def test_copy_pages_and_remap(cuda, orc):
    lens = [640, 320]
    pool, ref, n_pages, pt, cu = build_paged(orc, cuda, lens, n_layers=3, seed=11)
    # grow the pool view to have free pages above the used ones
    big = rk.PagedKvPool(n_pages + 8, 3, device=cuda)
    big.storage.zero_()
    for layer in range(3):
        src = pool.storage.view(3, n_pages, -1)[layer]
        big.storage.view(3, n_pages + 8, -1)[layer, :n_pages].copy_(src)
    ref_big = np.zeros((3, n_pages + 8, rk.PAGE_BYTES), np.uint8)
    ref_big[:, :n_pages] = ref.reshape(3, n_pages, -1)
    ref_big = ref_big.reshape(-1)
    src = np.array([0, 3, 7, 10], np.int32)
    dst = np.array([n_pages + 1, n_pages + 0, n_pages + 7, n_pages + 3], np.int32)
    big.copy_pages(i32(src, cuda), i32(dst, cuda))
    big.check("copy")
    orc.copy_pages(ref_big, n_pages + 8, 3, src, dst)
    assert np.array_equal(big.storage.cpu().numpy(), ref_big)
    # remap the table onto the copies; the gather is unchanged
    remap = np.arange(n_pages + 8, dtype=np.int32)
    remap[src] = dst
    pt_d = i32(pt, cuda)
    before = u16(big.rows(2, pt_d, i32(cu, cuda), 640))
    rk.remap_pages(pt_d, i32(remap, cuda))
    assert np.array_equal(pt_d.cpu().numpy(), np.where(pt >= 0, remap[np.maximum(pt, 0)], pt))
    after = u16(big.rows(2, pt_d, i32(cu, cuda), 640))
    big.check("gather")
    assert np.array_equal(before, after)
