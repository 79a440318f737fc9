"""TEST INFRASTRUCTURE ONLY: Python access to the CPU oracle (rkv_oracle.c).

The oracle is a plain-C restatement of rsLLM's KV-cache hot path on the CPU
(see the header of rkv_oracle.c for the reference file:line of each function
and how it is pinned).  Only tests/, __graft_entry__.smoke() and bench.py's
cpu_baseline / reference legs use it, as the checker and as the timed CPU
baseline; the rsllm_b200 package never imports it.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from ctypes import c_float, c_int, c_int32, c_int64, c_uint8, c_uint16, c_uint32, c_void_p
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "librkv_oracle.so"

PAGE_TOKENS, LATENT, ROPE, ROW_DIM, BLOCK = 64, 512, 64, 576, 64
PAGE_BYTES = 43008
OK, SHAPE_MISMATCH, INDEX_OUT_OF_RANGE, INVALID_LAYER, POOL_FULL, NON_FINITE_INPUT = 0, 1, 2, 3, 4, 5

_lib = None


def build() -> Path:
    """Compiles the oracle with its Makefile (gcc, no fast-math)."""
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB_PATH


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is not None:
        return _lib
    src = HERE / "rkv_oracle.c"
    if not LIB_PATH.exists() or (src.exists() and src.stat().st_mtime > LIB_PATH.stat().st_mtime):
        build()
    L = ctypes.CDLL(str(LIB_PATH))
    P = c_void_p
    sig = {
        "rkvo_page_bytes": (c_int, []),
        "rkvo_f32_to_bf16": (c_uint16, [c_float]),
        "rkvo_e4m3fn_value": (c_float, [c_uint32]),
        "rkvo_e4m3fn_dequant": (c_float, [c_float]),
        "rkvo_e4m3fn_code": (c_uint8, [c_float]),
        "rkvo_e4m3fn_code_range": (None, [c_uint32, ctypes.c_uint64, P, c_int]),
        "rkvo_libm_ldexpf": (c_float, [c_float, c_int]),
        "rkvo_scale_exponent": (c_int, [c_float]),
        "rkvo_fp8_kv_quantize_row_inplace": (c_int, [P, c_int64, c_int64, c_int64]),
        "rkvo_quantize_row_bf16": (c_int, [P, c_int64, c_int64, P, P, P]),
        "rkvo_dequant_row_bf16": (None, [P, P, P, c_int64, c_int64, P]),
        "rkvo_fp8_e4m3_to_f32": (c_float, [c_uint8]),
        "rkvo_f32_to_fp8_e4m3": (c_uint8, [c_float]),
        "rkvo_select_top_k_scan": (c_int64, [P, c_int64, c_int64, P]),
        "rkvo_select_top_k_sorted": (c_int64, [P, c_int64, c_int64, P]),
        "rkvo_topk_batch": (None, [P, c_int64, c_int32, P, c_int32, P, c_int, c_int]),
        "rkvo_quantize_row_f32": (c_int, [P, c_int64, c_int64, P, P, P]),
        "rkvo_threshold_mismatches": (ctypes.c_uint64, [P, c_int, c_int, c_int, P]),
        "rkvo_append_rows": (c_uint32, [P, c_int64, c_int32, c_int32, c_int32, P, c_int, c_int64, P, c_int]),
        "rkvo_gather_rows": (c_uint32, [P, c_int64, c_int32, c_int32, P, c_int64, P, c_int32, P, c_int]),
        "rkvo_sparse_gather_rows": (c_uint32, [P, c_int64, c_int32, c_int32, P, c_int64, P, P, P, c_int32, c_int32,
                                               P, c_int]),
        "rkvo_copy_pages": (None, [P, c_int64, c_int32, P, P, c_int64]),
        "rkvo_mla_decode": (c_uint32, [P, c_int64, c_int32, c_int32, P, c_int64, P, P, P, c_int32, P, c_int32, P,
                                       c_float, P, c_int]),
        "rkvo_per_dim_softmax_aggregate": (None, [P, P, c_int64, c_int64, c_int64, c_int64, P]),
        "rkvo_compressor_accumulate": (c_int, [P, P, P, c_int64, c_int64, P, P, P]),
        "rkvo_compressor_finish_prefill": (None, [P, P, P, c_int64, c_int64, c_int64]),
        "rkvo_rope_yarn_tail": (None, [P, c_uint32, c_uint32, c_uint32, c_uint32, ctypes.c_uint64, c_float, c_float,
                                       c_float, c_float, c_float, c_float, c_int]),
        "rkvo_compressor_postprocess": (None, [P, c_int64, P, c_uint32]),
        "rkvo_compress_rope": (None, [P, c_int64, c_uint32]),
        "rkvo_compress_append": (c_uint32, [P, c_int64, c_int32, c_int32, c_int32, P, P, P, c_int64, P, P, c_int64,
                                            P, P, P, P, P, c_int]),
        "rkvo_expf_batch": (None, [P, P, c_int64, c_int]),
        "rkvo_indexer_compress_append": (c_uint32, [P, c_int64, c_int32, P, P, P, c_int64, P, P, c_int64, P, P, P,
                                                    P, P, c_int]),
        "rkvo_indexer_score_row": (c_float, [P, P, P]),
        "rkvo_indexer_scores": (c_uint32, [P, P, P, c_int64, P, P, P, P, c_int32, P, c_int64, c_int]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    _lib = L
    return L


def _p(a: np.ndarray) -> c_void_p:
    assert a.flags["C_CONTIGUOUS"], "oracle arrays must be C-contiguous"
    return c_void_p(a.ctypes.data)


def threads() -> int:
    return max(1, len(os.sched_getaffinity(0)))


# ---- codec ----------------------------------------------------------------

def quantize_row_inplace(x: np.ndarray, head_dim: int, n_rot: int) -> int:
    """dsv4_quant.rs:316-362 on a float32 row, in place; returns the status."""
    assert x.dtype == np.float32
    return lib().rkvo_fp8_kv_quantize_row_inplace(_p(x), x.size, head_dim, n_rot)


def quantize_rows_bf16(rows: np.ndarray):
    """bf16 rows (uint16 [n, 576]) -> (codes u8 [n,512], scales f32 [n,8], rope u16 [n,64], status i32 [n])."""
    rows = np.ascontiguousarray(rows, dtype=np.uint16).reshape(-1, ROW_DIM)
    n = rows.shape[0]
    codes = np.zeros((n, LATENT), np.uint8)
    scales = np.zeros((n, LATENT // BLOCK), np.float32)
    rope = np.zeros((n, ROPE), np.uint16)
    st = np.zeros(n, np.int32)
    L = lib()
    for i in range(n):
        st[i] = L.rkvo_quantize_row_bf16(_p(rows[i]), ROW_DIM, ROPE, _p(codes[i]), _p(scales[i]), _p(rope[i]))
    return codes, scales, rope, st


def quantize_rows_f32(rows: np.ndarray):
    """f32 rows [n, 576] -> (codes, scales, rope bf16 bits, status), the stored
    form of the reference's f32 round trip."""
    rows = np.ascontiguousarray(rows, dtype=np.float32).reshape(-1, ROW_DIM)
    n = rows.shape[0]
    codes = np.zeros((n, LATENT), np.uint8)
    scales = np.zeros((n, LATENT // BLOCK), np.float32)
    rope = np.zeros((n, ROPE), np.uint16)
    st = np.zeros(n, np.int32)
    L = lib()
    for i in range(n):
        st[i] = L.rkvo_quantize_row_f32(_p(rows[i]), ROW_DIM, ROPE, _p(codes[i]), _p(scales[i]), _p(rope[i]))
    return codes, scales, rope, st


def threshold_mismatches(table: np.ndarray, eb_lo: int, eb_hi: int, n_threads: int | None = None):
    """(count, first bad y bits) of a scale-exponent threshold table against
    ceilf(log2f(y)) over every y with biased exponent in [eb_lo, eb_hi]."""
    t = np.ascontiguousarray(table, np.uint32)
    assert t.shape == (256,)
    first = np.zeros(1, np.uint32)
    n = lib().rkvo_threshold_mismatches(_p(t), eb_lo, eb_hi, n_threads or threads(), _p(first))
    return int(n), int(first[0])


def dequant_rows_bf16(codes: np.ndarray, scales: np.ndarray, rope: np.ndarray) -> np.ndarray:
    codes = np.ascontiguousarray(codes, np.uint8).reshape(-1, LATENT)
    scales = np.ascontiguousarray(scales, np.float32).reshape(-1, LATENT // BLOCK)
    rope = np.ascontiguousarray(rope, np.uint16).reshape(-1, ROPE)
    out = np.zeros((codes.shape[0], ROW_DIM), np.uint16)
    L = lib()
    for i in range(codes.shape[0]):
        L.rkvo_dequant_row_bf16(_p(codes[i]), _p(scales[i]), _p(rope[i]), LATENT, ROPE, _p(out[i]))
    return out


def e4m3fn_code_range(first_bits: int, n: int, n_threads: int | None = None) -> np.ndarray:
    out = np.empty(n, np.uint8)
    lib().rkvo_e4m3fn_code_range(first_bits, n, _p(out), n_threads or threads())
    return out


# ---- top-k ----------------------------------------------------------------

def select_top_k(scores: np.ndarray, top_k: int, scan: bool = True) -> np.ndarray:
    """indexer.rs:218-236 on one score vector; returns the effective_k indices."""
    s = np.ascontiguousarray(scores, np.float32)
    out = np.empty(max(0, min(top_k, s.size)), np.int32)
    fn = lib().rkvo_select_top_k_scan if scan else lib().rkvo_select_top_k_sorted
    got = fn(_p(s), s.size, top_k, _p(out))
    return out[:got]


def topk_batch(scores: np.ndarray, n_visible: np.ndarray, k: int, scan: bool = False,
               n_threads: int | None = None) -> np.ndarray:
    s = np.ascontiguousarray(scores, np.float32)
    nv = np.ascontiguousarray(n_visible, np.int32)
    out = np.empty((s.shape[0], k), np.int32)
    lib().rkvo_topk_batch(_p(s), s.shape[1], s.shape[0], _p(nv), k, _p(out), int(scan), n_threads or threads())
    return out


# ---- paged pool model -----------------------------------------------------

def new_pool(n_pages: int, n_layers: int) -> np.ndarray:
    return np.zeros(n_layers * n_pages * PAGE_BYTES, np.uint8)


def append_rows(pool: np.ndarray, n_pages: int, n_layers: int, layer0: int, rows: np.ndarray,
                slots: np.ndarray, n_threads: int = 1) -> int:
    """rows: bf16 bits (uint16) or float32 ``[n_layers_in, n_tokens, 576]``."""
    is_f32 = rows.dtype == np.float32
    rows = np.ascontiguousarray(rows, np.float32 if is_f32 else np.uint16)
    n_layers_in = rows.shape[0] if rows.ndim == 3 else 1
    n_tokens = rows.shape[-2]
    slots = np.ascontiguousarray(slots, np.int32)
    if rows.shape[-1] != ROW_DIM or slots.shape != (n_tokens,):
        raise ValueError(f"append_rows: rows [layers, n_tokens, 576] with slots [n_tokens], got {rows.shape} "
                         f"and {slots.shape}")
    return lib().rkvo_append_rows(_p(pool), n_pages, n_layers, layer0, n_layers_in, _p(rows), int(is_f32), n_tokens,
                                  _p(slots), n_threads)


def gather_rows(pool: np.ndarray, n_pages: int, n_layers: int, layer: int, page_table: np.ndarray,
                cu_seqlens: np.ndarray, n_threads: int = 1):
    pt = np.ascontiguousarray(page_table, np.int32)
    cu = np.ascontiguousarray(cu_seqlens, np.int32)
    out = np.zeros((int(cu[-1]), ROW_DIM), np.uint16)
    st = lib().rkvo_gather_rows(_p(pool), n_pages, n_layers, layer, _p(pt), pt.shape[1], _p(cu), cu.size - 1,
                                _p(out), n_threads)
    return out, st


def sparse_gather_rows(pool: np.ndarray, n_pages: int, n_layers: int, layer: int, page_table: np.ndarray,
                       seq_of_query: np.ndarray, seq_lens: np.ndarray, idx: np.ndarray, n_threads: int = 1):
    pt = np.ascontiguousarray(page_table, np.int32)
    sq = np.ascontiguousarray(seq_of_query, np.int32)
    sl = np.ascontiguousarray(seq_lens, np.int32)
    ix = np.ascontiguousarray(idx, np.int32)
    n_q, k = ix.shape
    out = np.zeros((n_q, k, ROW_DIM), np.uint16)
    st = lib().rkvo_sparse_gather_rows(_p(pool), n_pages, n_layers, layer, _p(pt), pt.shape[1], _p(sq), _p(sl),
                                       _p(ix), n_q, k, _p(out), n_threads)
    return out, st


def copy_pages(pool: np.ndarray, n_pages: int, n_layers: int, src: np.ndarray, dst: np.ndarray) -> None:
    s = np.ascontiguousarray(src, np.int32)
    d = np.ascontiguousarray(dst, np.int32)
    lib().rkvo_copy_pages(_p(pool), n_pages, n_layers, _p(s), _p(d), s.size)


# ---- MLA decode attention ------------------------------------------------------

def mla_decode(pool: np.ndarray, n_pages: int, n_layers: int, layer: int, page_table: np.ndarray,
               seq_lens: np.ndarray, seq_of_query: np.ndarray, q: np.ndarray, idx: np.ndarray | None,
               sinks: np.ndarray | None, scale: float, n_threads: int | None = None):
    """attention.rs:493-663 over pooled rows: q bf16 bits [n_q, 64, 576];
    idx int32 [n_q, k] (sparse) or None (every row); returns (out f32
    [n_q, 64, 512], status bits)."""
    pt = np.ascontiguousarray(page_table, np.int32)
    sl = np.ascontiguousarray(seq_lens, np.int32)
    sq = np.ascontiguousarray(seq_of_query, np.int32)
    q = np.ascontiguousarray(q, np.uint16)
    n_q = q.shape[0]
    assert q.shape == (n_q, 64, 576) and sq.shape == (n_q,)
    out = np.zeros((n_q, 64, 512), np.float32)
    if idx is not None:
        idx = np.ascontiguousarray(idx, np.int32)
        assert idx.shape[0] == n_q
        k, ip = idx.shape[1], _p(idx)
    else:
        k, ip = 0, None
    sk = None if sinks is None else np.ascontiguousarray(sinks, np.float32)
    st = lib().rkvo_mla_decode(_p(pool), n_pages, n_layers, layer, _p(pt), pt.shape[1], _p(sl), _p(sq), _p(q), n_q,
                               ip, k, None if sk is None else _p(sk), float(scale), _p(out),
                               n_threads or threads())
    return out, st


# ---- compressor emission -----------------------------------------------------------

class Compressor:
    """One reference compressor window state (compressed.rs:76-120 layout):
    kv and score [coff*ratio, coff*head_dim], initial kv 0 / score -inf."""

    def __init__(self, ratio: int, head_dim: int = ROW_DIM):
        self.ratio, self.head_dim = ratio, head_dim
        self.coff = 2 if ratio == 4 else 1
        self.width = self.coff * head_dim
        self.kv = np.zeros((self.coff * ratio, self.width), np.float32)
        self.score = np.full((self.coff * ratio, self.width), -np.inf, np.float32)
        self.count = np.zeros(1, np.uint32)

    def accumulate(self, kv: np.ndarray, score: np.ndarray) -> np.ndarray | None:
        """accumulate_wide: the aggregate row when the window is full, else None."""
        kv = np.ascontiguousarray(kv, np.float32)
        score = np.ascontiguousarray(score, np.float32)
        assert kv.shape == (self.width,) and score.shape == (self.width,)
        out = np.zeros(self.head_dim, np.float32)
        got = lib().rkvo_compressor_accumulate(_p(self.kv), _p(self.score), _p(self.count), self.ratio,
                                               self.head_dim, _p(kv), _p(score), _p(out))
        return out if got else None

    def accumulate_narrow(self, kv: np.ndarray, score: np.ndarray) -> np.ndarray | None:
        """accumulate (compressed.rs's head_dim-wide entry): the row replicated
        into every lane."""
        return self.accumulate(np.tile(np.asarray(kv, np.float32), self.coff),
                               np.tile(np.asarray(score, np.float32), self.coff))

    def finish_prefill(self, n_tokens: int) -> None:
        lib().rkvo_compressor_finish_prefill(_p(self.kv), _p(self.score), _p(self.count), self.ratio, self.head_dim,
                                             n_tokens)


def rope_yarn_tail(x: np.ndarray, n_head: int, head_dim: int, n_rot: int, pos: int, n_ctx_orig: int = 65536,
                   freq_base: float = 10000.0, freq_scale: float = 1.0, ext_factor: float = 0.0,
                   attn_factor: float = 1.0, beta_fast: float = 32.0, beta_slow: float = 1.0,
                   inverse: bool = False) -> None:
    """rope.rs:128-172 in place on x float32 [n_head * head_dim]."""
    assert x.dtype == np.float32 and x.flags["C_CONTIGUOUS"] and x.size == n_head * head_dim
    lib().rkvo_rope_yarn_tail(_p(x), n_head, head_dim, n_rot, pos, n_ctx_orig, freq_base, freq_scale, ext_factor,
                              attn_factor, beta_fast, beta_slow, int(inverse))


def compressor_postprocess(row: np.ndarray, norm: np.ndarray, comp_pos: int) -> None:
    """compressor.rs:284-330 in place: RMSNorm then the compressed-layer RoPE."""
    assert row.dtype == np.float32 and row.flags["C_CONTIGUOUS"]
    norm = np.ascontiguousarray(norm, np.float32)
    assert norm.shape == row.shape
    lib().rkvo_compressor_postprocess(_p(row), row.size, _p(norm), comp_pos)


def compress_rope(row: np.ndarray, comp_pos: int) -> None:
    """The compressed-layer YaRN rotation of the last 64 lanes, in place."""
    assert row.dtype == np.float32 and row.flags["C_CONTIGUOUS"]
    lib().rkvo_compress_rope(_p(row), row.size, comp_pos)


def compress_states(n_states: int, ratio: int):
    """Reference-layout states for compress_append: (kv, score, count)."""
    coff = 2 if ratio == 4 else 1
    shape = (n_states, coff * ratio, coff * ROW_DIM)
    return np.zeros(shape, np.float32), np.full(shape, -np.inf, np.float32), np.zeros(n_states, np.uint32)


def compress_append(pool: np.ndarray, n_pages: int, n_layers: int, layer: int, ratio: int, states,
                    kv: np.ndarray, score: np.ndarray, pos: np.ndarray, state_of: np.ndarray,
                    emit_slot: np.ndarray, ape: np.ndarray | None, norm: np.ndarray,
                    n_threads: int | None = None) -> int:
    """The compressor step of rkvo_compress_append (token order, reference
    state machine); returns the status bits."""
    skv, ssc, cnt = states
    kv = np.ascontiguousarray(kv, np.float32)
    score = np.ascontiguousarray(score, np.float32)
    pos = np.ascontiguousarray(pos, np.int32)
    state_of = np.ascontiguousarray(state_of, np.int32)
    emit_slot = np.ascontiguousarray(emit_slot, np.int32)
    norm = np.ascontiguousarray(norm, np.float32)
    ape = None if ape is None else np.ascontiguousarray(ape, np.float32)
    n_tok = kv.shape[0]
    return lib().rkvo_compress_append(_p(pool), n_pages, n_layers, layer, ratio, _p(skv), _p(ssc), _p(cnt),
                                      skv.shape[0], _p(kv), _p(score), n_tok, _p(pos), _p(state_of),
                                      _p(emit_slot), None if ape is None else _p(ape), _p(norm),
                                      n_threads or threads())


def indexer_compress_states(n_states: int, ratio: int, head_dim: int = 128):
    """Reference-layout states of the indexer compressor: (kv, score, count)."""
    coff = 2 if ratio == 4 else 1
    shape = (n_states, coff * ratio, coff * head_dim)
    return np.zeros(shape, np.float32), np.full(shape, -np.inf, np.float32), np.zeros(n_states, np.uint32)


def indexer_compress_append(out_rows: np.ndarray, ratio: int, states, kv: np.ndarray, score: np.ndarray,
                            pos: np.ndarray, state_of: np.ndarray, emit_row: np.ndarray, ape: np.ndarray | None,
                            norm: np.ndarray, n_threads: int | None = None) -> int:
    """The indexer pool's compressor step (128-lane rows) in token order over
    the reference state machine; emitted rows (after RMSNorm and RoPE, before
    the FP4 QAT) go to out_rows f32 [n_out_rows, 128]; returns status bits."""
    skv, ssc, cnt = states
    assert out_rows.dtype == np.float32 and out_rows.flags["C_CONTIGUOUS"] and out_rows.shape[1:] == (128,)
    kv = np.ascontiguousarray(kv, np.float32)
    score = np.ascontiguousarray(score, np.float32)
    pos = np.ascontiguousarray(pos, np.int32)
    state_of = np.ascontiguousarray(state_of, np.int32)
    emit_row = np.ascontiguousarray(emit_row, np.int32)
    norm = np.ascontiguousarray(norm, np.float32)
    ape = None if ape is None else np.ascontiguousarray(ape, np.float32)
    return lib().rkvo_indexer_compress_append(_p(out_rows), out_rows.shape[0], ratio, _p(skv), _p(ssc), _p(cnt),
                                              skv.shape[0], _p(kv), _p(score), kv.shape[0], _p(pos), _p(state_of),
                                              _p(emit_row), None if ape is None else _p(ape), _p(norm),
                                              n_threads or threads())


def expf(x: np.ndarray, n_threads: int | None = None) -> np.ndarray:
    """The host libm's expf over an array."""
    x = np.ascontiguousarray(x, np.float32)
    out = np.empty_like(x)
    lib().rkvo_expf_batch(_p(x), _p(out), x.size, n_threads or threads())
    return out


# ---- indexer scoring -------------------------------------------------------------

def indexer_scores(rows: np.ndarray, row_start: np.ndarray, seq_rows: np.ndarray, q: np.ndarray, w: np.ndarray,
                   seq_of_query: np.ndarray, n_visible: np.ndarray, ld: int, n_threads: int | None = None):
    """indexer.rs:198-216 for a batch of queries: rows f32 [*, 128]; q f32
    [n_q, 64, 128]; w f32 [n_q, 64]; returns (scores f32 [n_q, ld] with
    -inf past n_visible, status bits)."""
    rows = np.ascontiguousarray(rows, np.float32)
    rs = np.ascontiguousarray(row_start, np.int64)
    sr = np.ascontiguousarray(seq_rows, np.int32)
    q = np.ascontiguousarray(q, np.float32)
    w = np.ascontiguousarray(w, np.float32)
    sq = np.ascontiguousarray(seq_of_query, np.int32)
    nv = np.ascontiguousarray(n_visible, np.int32)
    n_q = q.shape[0]
    out = np.full((n_q, ld), -np.inf, np.float32)
    st = lib().rkvo_indexer_scores(_p(rows), _p(rs), _p(sr), rs.size, _p(q), _p(w), _p(sq), _p(nv), n_q, _p(out), ld,
                                   n_threads or threads())
    return out, st
