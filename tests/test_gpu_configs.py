"""Bit-exact parity with the CPU oracle at the benchmark configurations' full
sizes, through the same launch shapes the benchmark times:

* config 2: decode steps of 256 sequences x 61 layers, every step ONE append
  launch of 15,616 rows (several passes of the persistent grid), slots from
  the seeded lengths U[1024, 32768] and a seeded page permutation, a new page
  whenever a sequence crosses a page boundary -- every byte of the 61-layer
  pool against the oracle's ``fp8_kv_quantize_row_inplace`` + append
  (dsv4_quant.rs:316-362, three_tier.rs:187-202);
* config 3: one layer of 64 sequences x 32,768 rows appended through a random
  page permutation and gathered back in one launch -- every pool byte and
  every bf16 lane of the 2,097,152 gathered rows (swa.rs:131-149 read order);
* config 4: one layer of 32 sequences x 131,072 rows; 2048 queries (the last
  64 positions of each sequence, causal) select their top 2048 of seeded
  N(0,1) scores on the GPU (every index in order against indexer.rs:218-236),
  and the sparse gather of those 4,194,304 rows is compared lane for lane
  (attention.rs:549-560).

Rows are generated on the GPU (seeded) and copied to the host for the
oracle, so both sides see the same bytes."""
import numpy as np
import pytest
import torch

import rsllm_b200 as rk
from rsllm_b200 import synth

pytestmark = pytest.mark.gpu

N_LAYERS = 61


def u16(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def i32(a, dev) -> torch.Tensor:
    return torch.as_tensor(np.ascontiguousarray(a, np.int32)).to(dev)


def same_bytes(storage: torch.Tensor, ref: np.ndarray, chunk: int = 1 << 28) -> int:
    """-1 if the device bytes equal ``ref``, else the first differing offset
    (compared in chunks, so no second host copy of a multi-GB pool)."""
    assert storage.numel() == ref.size
    for c0 in range(0, ref.size, chunk):
        got = storage[c0:c0 + chunk].cpu().numpy()
        want = ref[c0:c0 + chunk]
        if not np.array_equal(got, want):
            return c0 + int(np.flatnonzero(got != want)[0])
    return -1


def fill(pool: rk.PagedKvPool, ref: np.ndarray, orc, pt: np.ndarray, ctx: int, per_chunk: int, seed: int):
    """Appends ctx rows of every sequence of page table ``pt`` into layer 0 of
    both pools, ``per_chunk`` sequences per launch."""
    n_seq = pt.shape[0]
    tok = np.arange(ctx)
    for c in range(0, n_seq, per_chunk):
        rows = synth.kv_rows(per_chunk * ctx, seed=seed + c, device=pool.device)
        slots = (pt[c:c + per_chunk][:, tok // 64] * 64 + tok % 64).reshape(-1).astype(np.int32)
        pool.append_layer(0, rows, i32(slots, pool.device))
        st = orc.append_rows(ref, pool.n_pages, 1, 0, u16(rows), slots, n_threads=orc.threads())
        assert st == 0
        del rows
    pool.check("fill")


@pytest.mark.parametrize("inputs_ready", [False, True], ids=["wait_first", "inputs_ready"])
def test_config2_decode_steps(cuda, orc, inputs_ready):
    """Both launch forms of the append: loads after the wait on the previous
    kernel, and loads before it (RKV_APPEND_INPUTS_READY), the steps queued
    back to back on one stream so each launch overlaps the one before."""
    n_seq, n_steps = 256, 3
    slots, n_pages, lens = synth.decode_slots(n_seq, n_steps, seed=3)
    pos = lens[None, :] + np.arange(n_steps)[:, None]
    assert (pos % 64 == 0).any(), "no sequence crosses into a new page in these steps"
    pool = rk.PagedKvPool(n_pages, N_LAYERS, device=cuda)
    pool.storage.zero_()
    ref = orc.new_pool(n_pages, N_LAYERS)
    rows = [synth.kv_rows(N_LAYERS * n_seq, seed=3000 + j, device=cuda).view(N_LAYERS, n_seq, 576)
            for j in range(n_steps)]
    d_slots = [i32(slots[j], cuda) for j in range(n_steps)]
    torch.cuda.synchronize()
    for j in range(n_steps):
        pool.append_layer(0, rows[j], d_slots[j], inputs_ready=inputs_ready)
    for j in range(n_steps):
        st = orc.append_rows(ref, n_pages, N_LAYERS, 0, u16(rows[j]), slots[j], n_threads=orc.threads())
        assert st == 0
    pool.check("config 2 append")
    bad = same_bytes(pool.storage, ref)
    assert bad < 0, f"pool bytes differ from the oracle at byte {bad}"


def test_config3_layer_gather(cuda, orc):
    n_seq, ctx = 64, 32768
    pp = ctx // 64
    n_pages = n_seq * pp
    pt = synth.permutation(n_pages, seed=4).numpy().reshape(n_seq, pp)
    pool = rk.PagedKvPool(n_pages, 1, device=cuda)
    pool.storage.zero_()
    ref = orc.new_pool(n_pages, 1)
    fill(pool, ref, orc, pt, ctx, per_chunk=8, seed=400)
    bad = same_bytes(pool.storage, ref)
    assert bad < 0, f"config 3 pool bytes differ from the oracle at byte {bad}"

    cu = (np.arange(n_seq + 1) * ctx).astype(np.int32)
    out = pool.rows(0, i32(pt, cuda), i32(cu, cuda), ctx)     # the whole layer in one launch
    pool.check("config 3 gather")
    per = 8
    for c in range(0, n_seq, per):
        want, st = orc.gather_rows(ref, n_pages, 1, 0, pt[c:c + per], cu[:per + 1], n_threads=orc.threads())
        assert st == 0
        got = u16(out[c * ctx:(c + per) * ctx])
        assert np.array_equal(got, want), f"gather differs in sequences {c}..{c + per - 1}"


def test_config4_topk_and_sparse_gather(cuda, orc):
    n_seq, ctx, n_qpos, k = 32, 131072, 64, 2048
    pp = ctx // 64
    n_pages = n_seq * pp
    n_q = n_seq * n_qpos
    pt = synth.permutation(n_pages, seed=6).numpy().reshape(n_seq, pp)
    pool = rk.PagedKvPool(n_pages, 1, device=cuda)
    pool.storage.zero_()
    ref = orc.new_pool(n_pages, 1)
    fill(pool, ref, orc, pt, ctx, per_chunk=4, seed=600)
    bad = same_bytes(pool.storage, ref)
    assert bad < 0, f"config 4 pool bytes differ from the oracle at byte {bad}"

    # query i of sequence s sits at position ctx - n_qpos + i and sees keys 0..pos
    n_visible = np.tile(ctx - n_qpos + 1 + np.arange(n_qpos), n_seq).astype(np.int32)
    seq_of_query = np.repeat(np.arange(n_seq), n_qpos).astype(np.int32)
    scores = synth.scores(n_q, ctx, seed=5, device=cuda)
    idx = rk.select_top_k(scores, i32(n_visible, cuda), k)
    want_idx = orc.topk_batch(scores.cpu().numpy(), n_visible, k, n_threads=orc.threads())
    got_idx = idx.cpu().numpy()
    assert np.array_equal(got_idx, want_idx), "top-k indices differ from the oracle"
    del scores

    seq_lens = np.full(n_seq, ctx, np.int32)
    out = pool.sparse_rows(0, i32(pt, cuda), i32(seq_of_query, cuda), i32(seq_lens, cuda), idx)
    pool.check("config 4 sparse gather")
    per = 128
    for c in range(0, n_q, per):
        want, st = orc.sparse_gather_rows(ref, n_pages, 1, 0, pt, seq_of_query[c:c + per], seq_lens,
                                          want_idx[c:c + per], n_threads=orc.threads())
        assert st == 0
        assert np.array_equal(u16(out[c:c + per]), want), f"sparse gather differs in queries {c}..{c + per - 1}"
