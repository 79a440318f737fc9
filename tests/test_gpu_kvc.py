"""KVC save / load on the GPU: a pooled sequence written with rkv_kvc_save is
read back by the independent test reader (header, token ids, every page of
every layer equal to the oracle's pool bytes, rows past the sequence zero),
loaded into a second pool through rkv_kvc_load (gathered rows bit-exact,
prefix registered in the radix store), and rejected where rsLLM's rules
reject it (no room: PoolFull; another layer count: ShapeMismatch)."""
import numpy as np
import pytest
import torch

import rsllm_b200 as rk
from rsllm_b200 import synth
from rsllm_b200.prefix_pool import PrefixKvPool, kvc_name

import kvc_reader

pytestmark = pytest.mark.gpu


def u16(t):
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def filled_pool(orc, cuda, n_tok=150, n_layers=3, n_pages=16, seed=0):
    pool = PrefixKvPool(n_pages, n_layers, device=cuda)
    pool.kv.storage.zero_()
    seq = pool.create_sequence()
    slots = pool.reserve([seq], [n_tok])
    rows = u16(synth.kv_rows(n_layers * n_tok, seed=seed)).reshape(n_layers, n_tok, 576)
    pool.kv.append_layer(0, torch.from_numpy(rows.view(np.int16)).view(torch.bfloat16).to(cuda),
                         torch.from_numpy(slots).to(cuda))
    pool.kv.check("append")
    ref = orc.new_pool(n_pages, n_layers)
    assert orc.append_rows(ref, n_pages, n_layers, 0, rows, slots) == 0
    return pool, seq, rows, ref


def gather_seq(pool, seq, n_tok, layer, cuda):
    pt = torch.from_numpy(pool.page_table(seq).reshape(1, -1)).to(cuda)
    cu = torch.tensor([0, n_tok], dtype=torch.int32, device=cuda)
    out = pool.kv.rows(layer, pt, cu, n_tok)
    pool.kv.check("gather")
    return u16(out)


def test_save_read_load_round_trip(cuda, orc, tmp_path):
    n_tok, n_layers, n_pages = 150, 3, 16
    pool, seq, rows, ref = filled_pool(orc, cuda, n_tok, n_layers, n_pages)
    tokens = (np.arange(n_tok) * 31 + 7).astype(np.int32)
    path = pool.save_kvc(seq, tokens, str(tmp_path), reason=2, vocab_size=129280, text=b"hello")
    assert path.endswith("/" + kvc_name(tokens))
    f = kvc_reader.read(path)
    assert (f["magic"], f["version"], f["quant_bits"], f["reason"], f["token_count"], f["ctx_size"]) == \
        (b"KVC", 1, 8, 2, n_tok, 192)
    assert f["text"] == b"hello" and f["trailing"] == 0 and f["payload_bytes"] == f["body_bytes"]
    assert (f["payload_magic"], f["payload_version"], f["vocab_size"], f["n_layers"], f["head_dim"],
            f["page_tokens"], f["n_pages"]) == (0x34565344, 1, 129280, n_layers, 576, 64, 3)
    assert np.array_equal(f["tokens"], tokens)
    pt = pool.page_table(seq)
    ref_pages = ref.reshape(n_layers, n_pages, kvc_reader.PAGE_BYTES)
    for layer in range(n_layers):
        for i, page in enumerate(pt):
            want = ref_pages[layer, page].copy()
            if i == len(pt) - 1:  # rows 22..63 of the last page belong to no token: zero in the file
                tail = n_tok - 64 * i
                want[tail * 512:64 * 512] = 0
                want[32768 + tail * 32:32768 + 2048] = 0
                want[34816 + tail * 128:] = 0
            assert np.array_equal(f["pages"][layer, i], want), (layer, i)

    pool2 = PrefixKvPool(32, n_layers, device=cuda)
    pool2.kv.storage.fill_(0x55)  # stale bytes elsewhere in the pool do not matter
    pool2.reserve([pool2.create_sequence()], [100])  # take two pages first: the loaded pages land elsewhere
    s2, toks = pool2.load_kvc(path)
    assert np.array_equal(toks, tokens) and pool2.seq_len(s2) == n_tok
    for layer in range(n_layers):
        assert np.array_equal(gather_seq(pool2, s2, n_tok, layer, cuda), gather_seq(pool, seq, n_tok, layer, cuda))
    matched, s3 = pool2.match_prefix(tokens)
    assert matched == n_tok


def test_load_errors(cuda, orc, tmp_path):
    pool, seq, rows, ref = filled_pool(orc, cuda, n_tok=150, n_layers=3, n_pages=16)
    tokens = np.arange(150, dtype=np.int32)
    path = pool.save_kvc(seq, tokens, str(tmp_path))
    with pytest.raises(rk.PoolFull):
        PrefixKvPool(2, 3, device=cuda).load_kvc(path)  # three pages needed
    with pytest.raises(rk.ShapeMismatch):
        PrefixKvPool(16, 2, device=cuda).load_kvc(path)
    with pytest.raises(rk.ShapeMismatch):
        pool.save_kvc(seq, np.arange(151, dtype=np.int32), str(tmp_path))  # longer than the sequence
