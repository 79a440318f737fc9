"""Device-detected errors and their data: a planted bad slot, NaN row, bad
page id or out-of-range position sets the status bit on the device, and the
diagnose calls name the first failing row in the kernel's order with the
fields of rsLLM's IndexOutOfRange { what, idx, len } / NonFiniteInput(what)
(crates/rsllm-kvcache/src/lib.rs:28-70, crates/rsllm-backend-cpu/src/error.rs:33).
The failures are planted in the inputs on the host side; no kernel faults."""
import numpy as np
import pytest
import torch

import rsllm_b200 as rk
from rsllm_b200 import synth

pytestmark = pytest.mark.gpu


def test_append_names_the_first_bad_row(cuda):
    n_pages, n_tok = 4, 40
    pool = rk.PagedKvPool(n_pages, 3, device=cuda)
    rows = synth.kv_rows(2 * n_tok, seed=9).view(2, n_tok, 576).clone()
    slots = torch.arange(n_tok, dtype=torch.int32)
    slots[11] = n_pages * 64 + 5           # bad slot: every layer's token 11
    rows[0, 17, 300] = float("nan")        # layer 0, token 17: NaN latent lane
    rows[1, 3, 540] = float("inf")         # RoPE lane: stored as is, not an error
    rows_d, slots_d = rows.to(cuda), slots.to(cuda)
    pool.append_layer(1, rows_d, slots_d)
    bits = pool.take_status()
    assert bits == (1 << rk.IndexOutOfRange.status) | (1 << rk.NonFiniteInput.status)
    info = pool.diagnose_append(1, rows_d, slots_d)
    assert info["status"] == rk.IndexOutOfRange.status
    assert (info["what"], info["idx"], info["len"], info["row"]) == ("slot_mapping", n_pages * 64 + 5, n_pages * 64, 11)
    with pytest.raises(rk.IndexOutOfRange) as e:
        rk.raise_for_info(info, "append")
    assert e.value.row == 11
    # without the bad slot the NaN row is the first failure
    slots_d[11] = 11
    info = pool.diagnose_append(1, rows_d, slots_d)
    assert (info["status"], info["what"], info["idx"], info["row"]) == (rk.NonFiniteInput.status, "rows", 300, 17)
    rows_d[0, 17, 300] = 0.0
    info = pool.diagnose_append(1, rows_d, slots_d)
    assert info["status"] == 0 and info["row"] == -1


def test_gather_names_the_bad_page(cuda):
    pool = rk.PagedKvPool(8, 1, device=cuda)
    pool.storage.zero_()
    pt = torch.tensor([[0, 1, 2], [3, 9, 4]], dtype=torch.int32, device=cuda)   # page 9 is outside the pool
    cu = torch.tensor([0, 150, 330], dtype=torch.int32, device=cuda)
    pool.rows(0, pt, cu, 180, total=330)
    assert pool.take_status() == 1 << rk.IndexOutOfRange.status
    info = pool.diagnose_rows(pt, cu)
    assert (info["status"], info["what"], info["idx"], info["len"], info["row"]) == \
        (rk.IndexOutOfRange.status, "page_table", 9, 8, 150 + 64)


def test_sparse_gather_names_the_bad_selection(cuda):
    pool = rk.PagedKvPool(8, 1, device=cuda)
    pool.storage.zero_()
    pt = torch.tensor([[0, 1], [2, 3]], dtype=torch.int32, device=cuda)
    seq_lens = torch.tensor([100, 128], dtype=torch.int32, device=cuda)
    sq = torch.tensor([0, 1], dtype=torch.int32, device=cuda)
    idx = torch.tensor([[5, -1, 99], [127, 0, 3]], dtype=torch.int32, device=cuda)
    pool.sparse_rows(0, pt, sq, seq_lens, idx)
    assert pool.take_status() == 0
    assert pool.diagnose_sparse_rows(pt, sq, seq_lens, idx)["status"] == 0
    idx[0, 2] = 100                         # position == seq_len of sequence 0
    pool.sparse_rows(0, pt, sq, seq_lens, idx)
    assert pool.take_status() == 1 << rk.IndexOutOfRange.status
    info = pool.diagnose_sparse_rows(pt, sq, seq_lens, idx)
    assert (info["what"], info["idx"], info["len"], info["row"]) == ("idx", 100, 100, 2)
