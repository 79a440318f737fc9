"""Paged KV pool with sequences, a radix prefix store, copy-on-write, LRU
eviction and compaction -- the Python face of the ``rkv_pool`` C ABI.

rsLLM plans this as its paged KV cache and radix-tree prefix cache
(docs/03-HLD.md:363-376); the rules are in include/rsllm_kv_cuda.h.  A pool
made with ``device=None`` is plan-only: it holds no device memory and
returns the page moves it decides (``take_moves``) for the caller to apply.
"""
from __future__ import annotations

import ctypes
from ctypes import byref, c_int64, c_uint32, c_void_p

import numpy as np
import torch

from . import _abi
from .kvcache import PagedKvPool, check, _stream


def _i32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.int32)


def _ptr(a: np.ndarray) -> c_void_p:
    return c_void_p(a.ctypes.data if a.size else 0)


class PrefixKvPool:
    """A pool of ``n_pages`` 64-token pages per layer (``n_layers`` layers).

    ``kv`` (device pools only) is the ``PagedKvPool`` over the same memory,
    for appends and reads; ``reserve`` hands out the slots to append into."""

    def __init__(self, n_pages: int, n_layers: int = 1, device: int | str | torch.device | None = 0):
        self.lib = _abi.load()
        self.n_pages = int(n_pages)
        self.n_layers = int(n_layers)
        self.kv = None
        storage = None
        dev_index = _abi.PLAN_ONLY
        if device is not None:
            self.kv = PagedKvPool(n_pages, n_layers, device=device if not isinstance(device, int) else
                                  torch.device("cuda", device))
            storage = self.kv.storage
            dev_index = self.kv.device.index
        desc = _abi.PoolDesc(self.n_pages, self.n_layers, dev_index, c_void_p(storage.data_ptr() if storage is not None
                                                                               else 0))
        h = c_void_p()
        check(self.lib.rkv_pool_create(byref(desc), byref(h)))
        self._h = h

    def close(self) -> None:
        if getattr(self, "_h", None):
            self.lib.rkv_pool_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # -- sequences ----------------------------------------------------------
    def create_sequence(self) -> int:
        v = c_int64()
        check(self.lib.rkv_seq_create(self._h, byref(v)))
        return v.value

    def fork(self, parent: int, n_tokens: int) -> int:
        v = c_int64()
        check(self.lib.rkv_seq_fork(self._h, parent, n_tokens, byref(v)))
        return v.value

    def reserve(self, seqs, n_tokens, stream: torch.cuda.Stream | None = None,
                out: np.ndarray | None = None) -> np.ndarray:
        """Slots (int32, sequence after sequence) for n_tokens[i] more tokens
        of each seqs[i]; copy-on-write copies go on ``stream``.  ``out`` (a
        contiguous int32 array of sum(n_tokens) entries, e.g. a view of a
        pinned host tensor) receives the slots instead of a new array."""
        from .kvcache import ShapeMismatch

        s = np.ascontiguousarray(np.atleast_1d(seqs), dtype=np.int64)
        n = np.ascontiguousarray(np.atleast_1d(n_tokens), dtype=np.int64)
        if s.shape != n.shape:
            raise ShapeMismatch("reserve: seqs and n_tokens differ in length")
        total = int(n[n > 0].sum())  # a negative count is the C call's ShapeMismatch
        if out is None:
            slots = np.empty(total, np.int32)
        elif out.dtype != np.int32 or not out.flags["C_CONTIGUOUS"] or out.size != total:
            raise ShapeMismatch(f"reserve: out must be a contiguous int32 array of {total} entries")
        else:
            slots = out
        st = c_void_p(0) if self.kv is None else _stream(stream)
        check(self.lib.rkv_seq_reserve(self._h, s.size, _ptr(s), _ptr(n), _ptr(slots), st))
        return slots

    def release(self, seq: int) -> None:
        check(self.lib.rkv_seq_release(self._h, seq))

    def touch(self, seq: int) -> None:
        check(self.lib.rkv_seq_touch(self._h, seq))

    def free(self, seq: int) -> None:
        check(self.lib.rkv_seq_free(self._h, seq))

    def seq_len(self, seq: int) -> int:
        v, p = c_int64(), c_int64()
        check(self.lib.rkv_seq_info(self._h, seq, byref(v), byref(p)))
        return v.value

    def page_table(self, seq: int) -> np.ndarray:
        v, p = c_int64(), c_int64()
        check(self.lib.rkv_seq_info(self._h, seq, byref(v), byref(p)))
        out = np.empty(p.value, np.int32)
        check(self.lib.rkv_seq_page_table(self._h, seq, _ptr(out), out.size))
        return out

    # -- radix prefix store -------------------------------------------------
    def insert_prefix(self, tokens, seq: int) -> None:
        t = _i32(tokens)
        check(self.lib.rkv_prefix_insert(self._h, _ptr(t), t.size, seq))

    def match_prefix(self, tokens) -> tuple[int, int]:
        """(matched tokens, new sequence sharing them)."""
        t = _i32(tokens)
        m, s = c_int64(), c_int64()
        check(self.lib.rkv_prefix_match(self._h, _ptr(t), t.size, byref(m), byref(s)))
        return m.value, s.value

    # -- eviction and compaction ---------------------------------------------
    def evict(self, target_pages: int) -> int:
        v = c_int64()
        check(self.lib.rkv_pool_evict(self._h, target_pages, byref(v)))
        return v.value

    def compact(self, device_tables: torch.Tensor | None = None, stream: torch.cuda.Stream | None = None) -> int:
        """Moves live pages down; optionally remaps an int32 device table."""
        v = c_int64()
        if device_tables is not None:
            if self.kv is None or device_tables.dtype != torch.int32 or not device_tables.is_contiguous():
                from .kvcache import ShapeMismatch

                raise ShapeMismatch("compact: device_tables must be a contiguous int32 tensor of a device pool")
            ptr, n = c_void_p(device_tables.data_ptr()), device_tables.numel()
        else:
            ptr, n = c_void_p(0), 0
        st = c_void_p(0) if self.kv is None else _stream(stream)
        check(self.lib.rkv_pool_compact(self._h, ptr, n, byref(v), st))
        return v.value

    def last_remap(self) -> np.ndarray:
        out = np.empty(self.n_pages, np.int32)
        check(self.lib.rkv_pool_last_remap(self._h, _ptr(out), out.size))
        return out

    def take_moves(self) -> tuple[np.ndarray, np.ndarray]:
        """Plan-only pools: (src, dst) page moves decided since the last call."""
        n = c_int64()
        check(self.lib.rkv_pool_take_moves(self._h, c_void_p(0), c_void_p(0), 0, byref(n)))
        src = np.empty(n.value, np.int32)
        dst = np.empty(n.value, np.int32)
        if n.value:
            check(self.lib.rkv_pool_take_moves(self._h, _ptr(src), _ptr(dst), n.value, byref(n)))
        return src, dst

    def stats(self) -> dict:
        st = _abi.PoolStats()
        check(self.lib.rkv_pool_get_stats(self._h, byref(st)))
        return {f: getattr(st, f) for f, _ in _abi.PoolStats._fields_}

    def refcounts(self) -> np.ndarray:
        out = np.empty(self.n_pages, np.int32)
        check(self.lib.rkv_page_refcount(self._h, _ptr(out), out.size))
        return out

    def device_status(self) -> int:
        b = c_uint32()
        check(self.lib.rkv_pool_device_status(self._h, byref(b)))
        return b.value

    # -- KVC files (prefix persistence) -----------------------------------------
    def save_kvc(self, seq: int, tokens, directory: str, reason: int = _abi.KVC_COLD, vocab_size: int = 0,
                 text: bytes = b"", stream: torch.cuda.Stream | None = None) -> str:
        """Writes the first ``len(tokens)`` tokens of ``seq`` (every layer) to
        ``<directory>/<SHA1(tokens)>.kvc``; returns the path (see
        ``rkv_kvc_save``)."""
        t = _i32(tokens)
        out = ctypes.create_string_buffer(len(directory.encode()) + 64)
        check(self.lib.rkv_kvc_save(self._h, seq, _ptr(t), t.size, reason, vocab_size, text, len(text),
                                    directory.encode(), out, len(out), _stream(stream)))
        return out.value.decode()

    def load_kvc(self, path: str, insert_prefix: bool = True,
                 stream: torch.cuda.Stream | None = None) -> tuple[int, np.ndarray]:
        """Loads a KVC file into a new sequence; returns (sequence, tokens)."""
        h = read_kvc_header(path)
        tokens = np.empty(h["token_count"], np.int32)
        n, seq = c_int64(), c_int64()
        check(self.lib.rkv_kvc_load(self._h, path.encode(), _ptr(tokens), tokens.size, byref(n), byref(seq),
                                    int(insert_prefix), _stream(stream)))
        return seq.value, tokens


def kvc_name(tokens) -> str:
    """File name of a token sequence: SHA1 of the ids as little-endian u32."""
    t = _i32(tokens)
    out = ctypes.create_string_buffer(46)
    check(_abi.load().rkv_kvc_name(_ptr(t), t.size, out))
    return out.value.decode()


def read_kvc_header(path: str) -> dict:
    h = _abi.KvcHeader()
    check(_abi.load().rkv_kvc_read_header(path.encode(), byref(h)))
    return {f: getattr(h, f) for f, _ in _abi.KvcHeader._fields_}
