"""Compressor emission on the GPU, mirroring rsLLM's compressed-pool append path.

rsLLM's compressor (crates/rsllm-models/src/dsv4/compressor.rs:223-362) turns
every token into a (kv, score) row pair of ``width = coff * head_dim`` lanes,
adds the APE bias to the score, and hands both to
``CompressedKvPool::accumulate_wide`` (crates/rsllm-kvcache/src/dsv4/
compressed.rs:310-343), which keeps a window state and, every ``ratio``
tokens, emits one per-dimension softmax aggregate (:360-417, :481-554).  The
emitted row is RMS-normalised, its 64 tail lanes are YaRN-rotated and it is
FP8-quantized (compressor.rs:284-357).

``CompressorBank`` holds the window states of many (sequence, layer)
compressors of one ratio on the device and runs that whole step for a batch of
tokens in one call (``rkv_compress_append``), writing each emitted row into a
``PagedKvPool`` slot in the stored FP8 format.  Rows are 576 lanes here (512
latent + 64 RoPE, the pool's row format); ratio 4 uses two lanes per token
(coff 2) as rsLLM does.  Results are bit-exact with rsLLM's f32/f64
arithmetic, including the host libm's expf and cos/sin.
"""
from __future__ import annotations

from ctypes import byref

import numpy as np
import torch

from . import _abi
from ._abi import ROW_DIM
from .kvcache import PagedKvPool, ShapeMismatch, _need, _ptr, _stream, check

__all__ = ["CompressorBank", "IndexerCompressorBank", "compress_rope_table", "compress_expf",
           "compress_expf_table_size"]

INDEXER_HEAD_DIM = 128  # rsLLM's DSV4_N_INDEXER_HEAD_DIM


def compress_rope_table(ratio: int, n_rows: int) -> np.ndarray:
    """cos/sin * mscale of the 32 RoPE pairs of compressed rows 0 .. n_rows-1
    (position k * ratio): f32 [n_rows, 32, 2], computed on the host with its
    libm as rope.rs:128-172 does with compress_rope_params."""
    out = np.empty((n_rows, 32, 2), dtype=np.float32)
    check(_abi.load().rkv_compress_rope_table(ratio, n_rows, out.ctypes.data), "compress_rope_table")
    return out


def compress_expf(x: torch.Tensor | np.ndarray) -> torch.Tensor | np.ndarray:
    """The kernel's expf (the host libm's rounding) over f32 values: on the
    device for a CUDA tensor, on the host for a numpy array."""
    lib = _abi.load()
    if isinstance(x, np.ndarray):
        x = np.ascontiguousarray(x, dtype=np.float32)
        out = np.empty_like(x)
        check(lib.rkv_compress_expf(x.ctypes.data, out.ctypes.data, x.size, 1, None), "compress_expf")
        return out
    _need(x, torch.float32, "x", x.device)
    out = torch.empty_like(x)
    check(lib.rkv_compress_expf(_ptr(x), _ptr(out), x.numel(), 0, _stream(None)), "compress_expf")
    return out


def compress_expf_table_size() -> int:
    """Entries of this process's expf correction table."""
    return int(_abi.load().rkv_compress_expf_table_size())


class CompressorBank:
    """Window states of ``n_states`` compressors of one ratio (one per
    sequence and layer, indexed by the caller), resident on one device.

    ``max_positions`` bounds the token positions the bank serves: the RoPE
    table holds the rows of compressed positions below it."""

    def __init__(self, ratio: int, n_states: int, device: int | str | torch.device | None = None,
                 max_positions: int = 1 << 17):
        if ratio <= 0 or ratio > 128:
            raise ShapeMismatch(f"CompressorBank: ratio {ratio} outside [1, 128]")
        self.lib = _abi.load()
        dev = torch.device("cuda", device) if isinstance(device, int) else \
            torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        if dev.index is None:
            dev = torch.device("cuda", torch.cuda.current_device())
        self.device = dev
        self.ratio = ratio
        self.coff = 2 if ratio == 4 else 1
        self.width = self.coff * ROW_DIM
        self.n_states = n_states
        nbytes = int(self.lib.rkv_compress_state_bytes(ratio))
        self.states = torch.zeros((n_states, nbytes // 4), dtype=torch.float32, device=self.device)
        rows = max_positions // ratio + 1
        self.rope = torch.from_numpy(compress_rope_table(ratio, rows)).to(self.device)
        with torch.cuda.device(self.device):
            check(self.lib.rkv_compress_prepare(), "CompressorBank")

    def append(self, pool: PagedKvPool, layer: int, kv: torch.Tensor, score: torch.Tensor, pos: torch.Tensor,
               state_of_token: torch.Tensor, emit_slot: torch.Tensor, norm: torch.Tensor,
               ape: torch.Tensor | None = None, stream: torch.cuda.Stream | None = None,
               inputs_ready: bool = False, one_token_per_state: bool = False) -> None:
        """One compressor step for ``n_tok`` tokens (``rkv_compress_append``):
        kv, score f32 [n_tok, width]; pos, state_of_token, emit_slot int32
        [n_tok]; norm f32 [576]; ape f32 [ratio, width] or None (the same on
        every call: the states keep scores without it).  Tokens of one
        state are consecutive entries at consecutive positions.  A token with
        (pos + 1) % ratio == 0 writes its emitted row at ``emit_slot`` (< 0:
        dropped).  Device-side errors land in ``pool.status``.
        ``inputs_ready``: pos / state_of_token / emit_slot / ape / norm are not
        written by a kernel that may still be running on the stream
        (RKV_COMPRESS_INPUTS_READY); ``one_token_per_state``: no state has two
        tokens in this call, e.g. a decode step
        (RKV_COMPRESS_ONE_TOKEN_PER_STATE, one launch instead of two)."""
        for t, n in ((kv, "kv"), (score, "score"), (norm, "norm")):
            _need(t, torch.float32, n, self.device)
        for t, n in ((pos, "pos"), (state_of_token, "state_of_token"), (emit_slot, "emit_slot")):
            _need(t, torch.int32, n, self.device)
        n_tok = kv.shape[0] if kv.dim() == 2 else -1
        if kv.dim() != 2 or kv.shape[1] != self.width or score.shape != kv.shape or \
                pos.shape != (n_tok,) or state_of_token.shape != (n_tok,) or emit_slot.shape != (n_tok,) or \
                norm.shape != (ROW_DIM,):
            raise ShapeMismatch(f"CompressorBank.append: kv/score [n_tok, {self.width}], pos/state_of_token/"
                                f"emit_slot [n_tok], norm [{ROW_DIM}]")
        if ape is not None:
            _need(ape, torch.float32, "ape", self.device)
            if ape.shape != (self.ratio, self.width):
                raise ShapeMismatch(f"CompressorBank.append: ape must be [{self.ratio}, {self.width}]")
        flags = (_abi.COMPRESS_INPUTS_READY if inputs_ready else 0) | \
            (_abi.COMPRESS_ONE_TOKEN_PER_STATE if one_token_per_state else 0)
        if not flags:
            check(self.lib.rkv_compress_append(byref(pool.view), layer, self.ratio, _ptr(self.states), self.n_states,
                                               _ptr(kv), _ptr(score), n_tok, _ptr(pos), _ptr(state_of_token),
                                               _ptr(emit_slot), _ptr(ape), _ptr(norm), _ptr(self.rope),
                                               self.rope.shape[0], _ptr(pool.status), _stream(stream)),
                  "CompressorBank.append")
            return
        check(self.lib.rkv_compress_append_ex(byref(pool.view), layer, self.ratio, _ptr(self.states), self.n_states,
                                              _ptr(kv), _ptr(score), n_tok, _ptr(pos), _ptr(state_of_token),
                                              _ptr(emit_slot), _ptr(ape), _ptr(norm), _ptr(self.rope),
                                              self.rope.shape[0], flags, _ptr(pool.status), _stream(stream)),
              "CompressorBank.append")


class IndexerCompressorBank:
    """Window states of the indexer pool's compressors (128-lane rows; rsLLM
    runs compressor_decode_one on its indexer pool too, attention.rs:405-429).
    ``append`` aggregates, RMS-normalises and rotates each emitted row like
    ``CompressorBank`` and writes it as f32 into a row buffer (the rows
    ``indexer_scores`` reads), stopping before rsLLM's Hadamard + FP4 QAT of
    the indexer row (compressor.rs:343-348), which this library does not
    restate."""

    def __init__(self, ratio: int, n_states: int, device: int | str | torch.device | None = None,
                 max_positions: int = 1 << 17):
        coff = 2 if ratio == 4 else 1
        if ratio <= 0 or coff * ratio > 128:
            raise ShapeMismatch(f"IndexerCompressorBank: ratio {ratio} outside [1, 128]")
        self.lib = _abi.load()
        dev = torch.device("cuda", device) if isinstance(device, int) else \
            torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        if dev.index is None:
            dev = torch.device("cuda", torch.cuda.current_device())
        self.device = dev
        self.ratio, self.coff = ratio, coff
        self.width = coff * INDEXER_HEAD_DIM
        self.n_states = n_states
        nbytes = int(self.lib.rkv_indexer_compress_state_bytes(ratio))
        self.states = torch.zeros((n_states, nbytes // 4), dtype=torch.float32, device=self.device)
        rows = max_positions // ratio + 1
        self.rope = torch.from_numpy(compress_rope_table(ratio, rows)).to(self.device)
        self.status = torch.zeros(1, dtype=torch.int32, device=self.device)
        with torch.cuda.device(self.device):
            check(self.lib.rkv_compress_prepare(), "IndexerCompressorBank")

    def append(self, out_rows: torch.Tensor, kv: torch.Tensor, score: torch.Tensor, pos: torch.Tensor,
               state_of_token: torch.Tensor, emit_row: torch.Tensor, norm: torch.Tensor,
               ape: torch.Tensor | None = None, stream: torch.cuda.Stream | None = None) -> None:
        """One indexer compressor step for ``n_tok`` tokens
        (``rkv_indexer_compress_append``): kv, score f32 [n_tok, width]; pos,
        state_of_token, emit_row int32 [n_tok]; norm f32 [128]; ape f32
        [ratio, width] or None; a token with (pos + 1) % ratio == 0 writes its
        row to ``out_rows[emit_row]`` (f32 [n_rows, 128]; < 0: dropped).
        Device-side errors land in ``self.status``."""
        for t, n in ((kv, "kv"), (score, "score"), (norm, "norm"), (out_rows, "out_rows")):
            _need(t, torch.float32, n, self.device)
        for t, n in ((pos, "pos"), (state_of_token, "state_of_token"), (emit_row, "emit_row")):
            _need(t, torch.int32, n, self.device)
        n_tok = kv.shape[0] if kv.dim() == 2 else -1
        if kv.dim() != 2 or kv.shape[1] != self.width or score.shape != kv.shape or \
                pos.shape != (n_tok,) or state_of_token.shape != (n_tok,) or emit_row.shape != (n_tok,) or \
                norm.shape != (INDEXER_HEAD_DIM,) or out_rows.dim() != 2 or out_rows.shape[1] != INDEXER_HEAD_DIM:
            raise ShapeMismatch(f"IndexerCompressorBank.append: kv/score [n_tok, {self.width}], pos/state_of_token/"
                                f"emit_row [n_tok], norm [128], out_rows [n_rows, 128]")
        if ape is not None:
            _need(ape, torch.float32, "ape", self.device)
            if ape.shape != (self.ratio, self.width):
                raise ShapeMismatch(f"IndexerCompressorBank.append: ape must be [{self.ratio}, {self.width}]")
        check(self.lib.rkv_indexer_compress_append(self.ratio, _ptr(self.states), self.n_states, _ptr(kv),
                                                   _ptr(score), n_tok, _ptr(pos), _ptr(state_of_token),
                                                   _ptr(emit_row), _ptr(ape), _ptr(norm), _ptr(self.rope),
                                                   self.rope.shape[0], _ptr(out_rows), out_rows.shape[0],
                                                   _ptr(self.status), _stream(stream)),
              "IndexerCompressorBank.append")

    def take_status(self, stream: torch.cuda.Stream | None = None) -> int:
        """Synchronises, returns and clears the device status bits."""
        (stream or torch.cuda.current_stream()).synchronize()
        bits = int(self.status.item()) & 0xFFFFFFFF
        self.status.zero_()
        return bits
