"""Shared inputs of the MLA decode attention tests: a pool of seeded rows in
a random physical page order, bf16 queries, index lists with the sparse-mask
corner cases, and an independent float64 statement of the attention
(attention.rs:493-663) over the exactly dequantised rows."""
import numpy as np
import torch

from rsllm_b200 import synth

HEADS, QK, V = 64, 576, 512


def bf16_bits(x: np.ndarray) -> np.ndarray:
    return torch.from_numpy(np.ascontiguousarray(x, np.float32)).to(torch.bfloat16).view(torch.int16).numpy().view(
        np.uint16)


def build(orc, lens, n_layers=2, layer=1, seed=0):
    """Rows for sequences of the given lengths appended (by the oracle) into a
    pool with a seeded random page order.  Returns a dict of numpy arrays."""
    rng = np.random.default_rng(seed)
    pages_per = [(n + 63) // 64 for n in lens]
    n_pages = max(1, sum(pages_per)) + 3
    stride = max(1, max(pages_per))
    perm = rng.permutation(n_pages).astype(np.int32)
    pt = np.full((len(lens), stride), -1, np.int32)
    slots, k = [], 0
    for s, n in enumerate(lens):
        pt[s, :pages_per[s]] = perm[k:k + pages_per[s]]
        k += pages_per[s]
        t = np.arange(n)
        slots.append(pt[s, t // 64] * 64 + t % 64)
    slots = np.concatenate(slots).astype(np.int32) if slots else np.zeros(0, np.int32)
    rows = synth.kv_rows(max(1, slots.size), seed=seed + 1).view(torch.int16).numpy().view(np.uint16)[:slots.size]
    pool = orc.new_pool(n_pages, n_layers)
    if slots.size:
        assert orc.append_rows(pool, n_pages, n_layers, layer, rows.reshape(1, -1, 576), slots) == 0
    return dict(pool=pool, n_pages=n_pages, n_layers=n_layers, layer=layer, pt=pt,
                lens=np.array(lens, np.int32), rows=rows, slots=slots)


def queries(n_q, n_seq, seed=1, scale=1.0):
    rng = np.random.default_rng(seed)
    q = bf16_bits(rng.standard_normal((n_q, HEADS, QK)) * scale)
    seq_of_query = (np.arange(n_q) % max(1, n_seq)).astype(np.int32)
    return q, seq_of_query


def index_lists(lens, seq_of_query, k, seed=2):
    """Per query k positions: distinct valid positions, then the corner cases
    -- out-of-range and negative entries (ignored) and, for odd queries, the
    repeated 0 the top-k selection fills with."""
    rng = np.random.default_rng(seed)
    idx = np.empty((seq_of_query.size, k), np.int32)
    for i, s in enumerate(seq_of_query):
        n = int(lens[s])
        take = min(n, k)
        row = rng.permutation(n)[:take] if n else np.zeros(0, np.int64)
        fill = np.zeros(k - take, np.int64)
        if i % 2 == 0 and k - take > 0:
            fill = rng.choice([-1, n, n + 100], k - take)
        idx[i] = np.concatenate([row, fill]).astype(np.int32)
        if i % 3 == 1 and take > 4:  # a few stray entries in the middle
            idx[i, 2] = -5
            idx[i, 3] = n + 7
    return idx


def dequant_rows_f64(orc, case, seq):
    """The sequence's rows [len, 576] exactly as stored (bf16 gather of the
    oracle is exact), in float64."""
    n = int(case["lens"][seq])
    if n == 0:
        return np.zeros((0, QK))
    cu = np.array([0, n], np.int32)
    out, st = orc.gather_rows(case["pool"], case["n_pages"], case["n_layers"], case["layer"],
                              case["pt"][seq:seq + 1], cu)
    assert st == 0
    return (out.astype(np.uint32) << 16).view(np.float32).astype(np.float64)


def attention_f64(orc, case, q, seq_of_query, idx, sinks, scale):
    """float64 attention: the same key sets and guards as the reference."""
    out = np.zeros((q.shape[0], HEADS, V))
    qf = (q.astype(np.uint32) << 16).view(np.float32).astype(np.float64)
    cache = {}
    for i, s in enumerate(seq_of_query):
        if s not in cache:
            cache[s] = dequant_rows_f64(orc, case, s)
        rows = cache[s]
        n = rows.shape[0]
        if idx is None:
            keys = np.arange(n)
        else:
            keys = np.unique(idx[i][(idx[i] >= 0) & (idx[i] < n)])
        kr = rows[keys]
        logits = qf[i] @ kr.T * scale  # [64, n_keys]
        for h in range(HEADS):
            sink = -np.inf if sinks is None else float(sinks[h])
            m = max([sink] + list(logits[h])) if keys.size else sink
            if not np.isfinite(m):
                continue
            e = np.exp(logits[h] - m)
            den = e.sum() + (np.exp(sink - m) if np.isfinite(sink) else 0.0)
            if den == 0 or not np.isfinite(den):
                continue
            out[i, h] = (e / den) @ kr[:, :V]
    return out


def value_scale(orc, case, seq_of_query):
    """Per query the largest |latent| over its sequence (the error scale)."""
    sc = np.zeros(seq_of_query.size)
    for i, s in enumerate(seq_of_query):
        r = dequant_rows_f64(orc, case, s)
        sc[i] = np.abs(r[:, :V]).max() if r.size else 1.0
    return sc
