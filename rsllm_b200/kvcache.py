"""Host-side API of the B200 KV-cache path, mirroring rsLLM's interfaces.

Names and error behaviour follow rsLLM (paths within the rsLLM tree):

* errors: ``ShapeMismatch`` / ``IndexOutOfRange`` / ``InvalidLayer`` /
  ``PoolFull`` (= ``CompressedPoolFull``) of crates/rsllm-kvcache/src/lib.rs:28-70
  and ``NonFiniteInput`` of crates/rsllm-backend-cpu/src/error.rs:33;
* ``CudaBackend`` is the ``rsllm_cal::Backend`` marker trait
  (crates/rsllm-cal/src/lib.rs:84-90) with ``fp8_kv_cache = True``;
* ``PagedKvPool.append_layer`` = ``ThreeTierKvCache::append_layer``
  (three_tier.rs:187) fused with ``fp8_kv_quantize_row_inplace``
  (dsv4_quant.rs:316); ``PagedKvPool.rows`` = ``RawSwaRing::rows`` /
  ``CompressedKvPool::rows`` over a page table; ``select_top_k`` =
  ``IndexerPool::select_top_k``'s selection (indexer.rs:218-236).

Every call goes to the CUDA library; torch only provides device memory and
streams.  There is no CPU fallback.
"""
from __future__ import annotations

from ctypes import byref, c_void_p
from dataclasses import dataclass

import torch

from . import _abi
from ._abi import PAGE_BYTES, PAGE_TOKENS, ROW_DIM


class KvError(RuntimeError):
    """A failed call.  ``info`` holds rkv_last_error_info's fields, the data
    of rsLLM's error variant: ``what``, ``idx``, ``len`` (IndexOutOfRange),
    ``expected``, ``actual`` (ShapeMismatch), ``max`` (InvalidLayer), ``cap``
    (CompressedPoolFull) and ``row`` (device-detected errors, from the
    diagnose calls); -1 where a field does not apply."""

    status = -1

    def __init__(self, msg: str = "", info: dict | None = None):
        super().__init__(msg)
        self.info = dict(info or {})

    def __getattr__(self, name):
        info = self.__dict__.get("info", {})
        if name in info:
            return info[name]
        raise AttributeError(name)


class ShapeMismatch(KvError):
    status = _abi.RKV_ERR_SHAPE_MISMATCH


class IndexOutOfRange(KvError):
    status = _abi.RKV_ERR_INDEX_OUT_OF_RANGE


class InvalidLayer(KvError):
    status = _abi.RKV_ERR_INVALID_LAYER


class PoolFull(KvError):
    status = _abi.RKV_ERR_POOL_FULL


class NonFiniteInput(KvError):
    status = _abi.RKV_ERR_NON_FINITE_INPUT


class InvalidArgument(KvError):
    status = _abi.RKV_ERR_INVALID_ARGUMENT


class CudaError(KvError):
    status = _abi.RKV_ERR_CUDA


ERRORS = {c.status: c for c in (ShapeMismatch, IndexOutOfRange, InvalidLayer, PoolFull, NonFiniteInput,
                                InvalidArgument, CudaError)}


def check(rc: int, what: str = "") -> None:
    """Raises the rsLLM-named error for a non-zero status, with its data."""
    if rc != 0:
        msg = _abi.last_error() or what
        raise ERRORS.get(rc, KvError)(msg, _abi.last_error_info())


def raise_for_info(info: dict, what: str = "") -> None:
    """Raises the error a diagnose call found (nothing if status is 0)."""
    rc = int(info.get("status", 0))
    if rc != 0:
        raise ERRORS.get(rc, KvError)(f"{what}: {_abi.last_error()}" if what else _abi.last_error(), info)


def raise_status_bits(bits: int, what: str) -> None:
    """Raises for a device status word (OR of 1 << status over failed rows)."""
    bits &= 0xFFFFFFFF
    if bits:
        rc = _abi.load().rkv_status_from_bits(bits)
        raise ERRORS.get(rc, KvError)(f"{what}: device status bits 0x{bits:x}")


def _stream(stream: torch.cuda.Stream | None) -> c_void_p:
    s = stream if stream is not None else torch.cuda.current_stream()
    return c_void_p(s.cuda_stream)


def _ptr(t: torch.Tensor | None) -> c_void_p:
    return c_void_p(t.data_ptr() if t is not None else 0)


def _need(t: torch.Tensor, dtype: torch.dtype, name: str, device: torch.device) -> None:
    if not isinstance(t, torch.Tensor) or t.dtype != dtype:
        raise ShapeMismatch(f"{name}: expected a {dtype} tensor")
    if t.device != device:
        raise ShapeMismatch(f"{name}: expected a tensor on {device}, got {t.device}")
    if not t.is_contiguous():
        raise ShapeMismatch(f"{name}: expected a contiguous tensor")


@dataclass(frozen=True)
class BackendCapability:
    """rsllm_cal::BackendCapability (crates/rsllm-cal/src/lib.rs:62-75)."""

    backend: str = "cuda"
    arch: str = "sm_100a"
    q4k_matmul: bool = False
    q2k_matmul: bool = False
    iq2xxs_matmul: bool = False
    fp8_kv_cache: bool = True


class CudaBackend:
    """rsllm_cal::Backend for the B200 path: kind() and capability()."""

    def __init__(self, device: int | str | torch.device = 0):
        if not torch.cuda.is_available():
            raise CudaError("CudaBackend: no CUDA device")
        self.device = torch.device("cuda", torch.device(device).index if not isinstance(device, int) else device)
        self.lib = _abi.load()

    def kind(self) -> str:
        return "cuda"

    def capability(self) -> BackendCapability:
        return BackendCapability()


class PagedKvPool:
    """A paged FP8 KV pool on one GPU: ``n_layers`` regions of ``n_pages``
    pages, 64 token rows per page (see ``include/rsllm_kv_cuda.h``)."""

    def __init__(self, n_pages: int, n_layers: int = 1, device: int | str | torch.device | None = None,
                 storage: torch.Tensor | None = None):
        if n_pages <= 0 or n_layers <= 0:
            raise ShapeMismatch("PagedKvPool: n_pages and n_layers must be positive")
        if not torch.cuda.is_available():
            raise CudaError("PagedKvPool: no CUDA device")
        self.lib = _abi.load()
        dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        if dev.type != "cuda":
            raise CudaError("PagedKvPool: device must be a CUDA device")
        if dev.index is None:
            dev = torch.device("cuda", torch.cuda.current_device())
        self.device = dev
        self.n_pages = int(n_pages)
        self.n_layers = int(n_layers)
        nbytes = self.n_layers * self.n_pages * PAGE_BYTES
        if storage is None:
            storage = torch.empty(nbytes, dtype=torch.uint8, device=dev)
        elif storage.numel() * storage.element_size() < nbytes or storage.device != dev:
            raise ShapeMismatch("PagedKvPool: storage too small or on another device")
        self.storage = storage
        self.status = torch.zeros(1, dtype=torch.int32, device=dev)
        self.view = _abi.PoolView(storage.data_ptr(), self.n_pages, self.n_layers, 0)

    # -- status -------------------------------------------------------------
    def take_status(self, stream: torch.cuda.Stream | None = None) -> int:
        """Synchronises, returns and clears the per-row device status bits."""
        (stream or torch.cuda.current_stream()).synchronize()
        bits = int(self.status.item()) & 0xFFFFFFFF
        self.status.zero_()
        return bits

    def check(self, what: str = "PagedKvPool", stream: torch.cuda.Stream | None = None) -> None:
        raise_status_bits(self.take_status(stream), what)

    # -- quantize-on-append ---------------------------------------------------
    def append_layer(self, layer0: int, rows: torch.Tensor, slot_mapping: torch.Tensor,
                     stream: torch.cuda.Stream | None = None, inputs_ready: bool = False) -> None:
        """Quantise bf16 or f32 rows ``[n_layers_in, n_tokens, 576]`` (or
        ``[n_tokens, 576]`` for one layer) into the slots ``slot_mapping``
        (int32 ``[n_tokens]``, shared by the layers; negative = skip).  f32
        rows take the reference's log2f exponent and store RoPE as bf16.
        ``inputs_ready`` (bf16 rows): no kernel that may still be running on
        the stream writes ``rows`` or ``slot_mapping``, so the append may read
        them while the previous kernel drains (RKV_APPEND_INPUTS_READY)."""
        f32 = rows.dtype == torch.float32
        _need(rows, torch.float32 if f32 else torch.bfloat16, "rows", self.device)
        _need(slot_mapping, torch.int32, "slot_mapping", self.device)
        if rows.dim() == 2:
            rows = rows.unsqueeze(0)
        if rows.dim() != 3 or rows.shape[-1] != ROW_DIM:
            raise ShapeMismatch(f"append_layer: rows must be [..., {ROW_DIM}], got {tuple(rows.shape)}")
        if slot_mapping.dim() != 1 or slot_mapping.shape[0] != rows.shape[1]:
            raise ShapeMismatch("append_layer: slot_mapping must be [n_tokens]")
        if inputs_ready and not f32:
            check(self.lib.rkv_append_quant_bf16_ex(byref(self.view), layer0, rows.shape[0], _ptr(rows), rows.shape[1],
                                                    _ptr(slot_mapping), _abi.APPEND_INPUTS_READY, _ptr(self.status),
                                                    _stream(stream)))
            return
        fn = self.lib.rkv_append_quant_f32 if f32 else self.lib.rkv_append_quant_bf16
        check(fn(byref(self.view), layer0, rows.shape[0], _ptr(rows), rows.shape[1], _ptr(slot_mapping),
                 _ptr(self.status), _stream(stream)))

    def copy_floor_layer(self, layer0: int, rows: torch.Tensor, slot_mapping: torch.Tensor,
                         stream: torch.cuda.Stream | None = None) -> None:
        """Measurement reference (rkv_copy_floor_bf16): moves the bytes
        ``append_layer(..., inputs_ready=True)`` moves, with the same launch,
        but without the codec -- the rows it leaves in the slots are NOT valid
        FP8 rows.  For timing the append against a plain copy of its traffic
        on a pool whose contents no longer matter."""
        _need(rows, torch.bfloat16, "rows", self.device)
        _need(slot_mapping, torch.int32, "slot_mapping", self.device)
        if rows.dim() == 2:
            rows = rows.unsqueeze(0)
        if rows.dim() != 3 or rows.shape[-1] != ROW_DIM or slot_mapping.dim() != 1 \
                or slot_mapping.shape[0] != rows.shape[1]:
            raise ShapeMismatch("copy_floor_layer: rows [..., n_tokens, 576] and slot_mapping [n_tokens] required")
        check(self.lib.rkv_copy_floor_bf16(byref(self.view), layer0, rows.shape[0], _ptr(rows), rows.shape[1],
                                           _ptr(slot_mapping), _stream(stream)))

    # -- data of device-detected errors -------------------------------------------
    def diagnose_append(self, layer0: int, rows: torch.Tensor, slot_mapping: torch.Tensor,
                        stream: torch.cuda.Stream | None = None) -> dict:
        """The first row of an append (same arguments) that the kernel
        rejects, as rkv_append_diagnose_bf16 finds it: a dict of
        rkv_err_info's fields, status 0 when every row passes."""
        if rows.dim() == 2:
            rows = rows.unsqueeze(0)
        info = _abi.ErrInfo()
        self.lib.rkv_append_diagnose_bf16(byref(self.view), layer0, rows.shape[0], _ptr(rows), rows.shape[1],
                                          _ptr(slot_mapping), byref(info), _stream(stream))
        return info.as_dict()

    def diagnose_rows(self, page_table: torch.Tensor, cu_seqlens: torch.Tensor,
                      stream: torch.cuda.Stream | None = None) -> dict:
        """The first bad page of a gather (rkv_gather_diagnose)."""
        info = _abi.ErrInfo()
        self.lib.rkv_gather_diagnose(byref(self.view), _ptr(page_table), page_table.shape[1], _ptr(cu_seqlens),
                                     page_table.shape[0], byref(info), _stream(stream))
        return info.as_dict()

    def diagnose_sparse_rows(self, page_table: torch.Tensor, seq_of_query: torch.Tensor, seq_lens: torch.Tensor,
                             idx: torch.Tensor, stream: torch.cuda.Stream | None = None) -> dict:
        """The first bad selection of a sparse gather (rkv_sparse_gather_diagnose)."""
        info = _abi.ErrInfo()
        self.lib.rkv_sparse_gather_diagnose(byref(self.view), _ptr(page_table), page_table.shape[1],
                                            _ptr(seq_of_query), _ptr(seq_lens), seq_lens.shape[0], _ptr(idx),
                                            idx.shape[0], idx.shape[1], byref(info), _stream(stream))
        return info.as_dict()

    # -- reads ----------------------------------------------------------------
    def rows(self, layer: int, page_table: torch.Tensor, cu_seqlens: torch.Tensor, max_seq_len: int,
             out: torch.Tensor | None = None, stream: torch.cuda.Stream | None = None,
             total: int | None = None) -> torch.Tensor:
        """Chronological bf16 rows of every sequence (``[total, 576]``):
        row t of sequence s at ``out[cu_seqlens[s] + t]``.  Pass ``out`` or
        ``total`` (= cu_seqlens[-1]) to keep the call asynchronous; without
        either the call reads cu_seqlens[-1] back from the device (a stream
        synchronisation) to size the output."""
        _need(page_table, torch.int32, "page_table", self.device)
        _need(cu_seqlens, torch.int32, "cu_seqlens", self.device)
        if page_table.dim() != 2 or cu_seqlens.dim() != 1 or cu_seqlens.shape[0] != page_table.shape[0] + 1:
            raise ShapeMismatch("rows: page_table [n_seq, stride] and cu_seqlens [n_seq+1] required")
        if out is None:
            if total is None:
                total = int(cu_seqlens[-1].item())
            out = torch.empty((total, ROW_DIM), dtype=torch.bfloat16, device=self.device)
        _need(out, torch.bfloat16, "out", self.device)
        check(self.lib.rkv_gather_dequant_bf16(byref(self.view), layer, _ptr(page_table), page_table.shape[1],
                                               _ptr(cu_seqlens), page_table.shape[0], int(max_seq_len), _ptr(out),
                                               _ptr(self.status), _stream(stream)))
        return out

    def sparse_rows(self, layer: int, page_table: torch.Tensor, seq_of_query: torch.Tensor, seq_lens: torch.Tensor,
                    idx: torch.Tensor, out: torch.Tensor | None = None,
                    stream: torch.cuda.Stream | None = None) -> torch.Tensor:
        """bf16 rows of the selected token positions ``idx`` [n_q, k]."""
        for t, n in ((page_table, "page_table"), (seq_of_query, "seq_of_query"), (seq_lens, "seq_lens"),
                     (idx, "idx")):
            _need(t, torch.int32, n, self.device)
        if idx.dim() != 2 or seq_of_query.shape != (idx.shape[0],) or page_table.dim() != 2:
            raise ShapeMismatch("sparse_rows: idx [n_q, k], seq_of_query [n_q], page_table [n_seq, stride]")
        if out is None:
            out = torch.empty((idx.shape[0], idx.shape[1], ROW_DIM), dtype=torch.bfloat16, device=self.device)
        _need(out, torch.bfloat16, "out", self.device)
        check(self.lib.rkv_sparse_gather_dequant_bf16(byref(self.view), layer, _ptr(page_table), page_table.shape[1],
                                                      _ptr(seq_of_query), _ptr(seq_lens), _ptr(idx), idx.shape[0],
                                                      idx.shape[1], _ptr(out), _ptr(self.status), _stream(stream)))
        return out

    # -- attention read -------------------------------------------------------
    def mla_decode(self, layer: int, q: torch.Tensor, page_table: torch.Tensor, seq_lens: torch.Tensor,
                   seq_of_query: torch.Tensor, idx: torch.Tensor | None = None, sinks: torch.Tensor | None = None,
                   softmax_scale: float | None = None, n_splits: int = 1, out: torch.Tensor | None = None,
                   workspace: torch.Tensor | None = None, stream: torch.cuda.Stream | None = None) -> torch.Tensor:
        """MLA decode attention over the FP8 pages (see ``rkv_mla_decode_fp8``):
        q bf16 [n_q, 64, 576] -> f32 [n_q, 64, 512]; every row of the query's
        sequence (idx None) or the rows ``idx`` [n_q, k] selects.  The scale
        defaults to 1/sqrt(576), as attention.rs:337 takes 1/sqrt(head_dim)."""
        _need(q, torch.bfloat16, "q", self.device)
        for t, n in ((page_table, "page_table"), (seq_lens, "seq_lens"), (seq_of_query, "seq_of_query")):
            _need(t, torch.int32, n, self.device)
        if q.dim() != 3 or q.shape[1:] != (64, ROW_DIM) or seq_of_query.shape != (q.shape[0],) or \
                page_table.dim() != 2:
            raise ShapeMismatch("mla_decode: q [n_q, 64, 576], seq_of_query [n_q], page_table [n_seq, stride]")
        n_q = q.shape[0]
        k = 0
        if idx is not None:
            _need(idx, torch.int32, "idx", self.device)
            if idx.dim() != 2 or idx.shape[0] != n_q:
                raise ShapeMismatch("mla_decode: idx must be [n_q, k]")
            k = idx.shape[1]
        if sinks is not None:
            _need(sinks, torch.float32, "sinks", self.device)
            if sinks.shape != (64,):
                raise ShapeMismatch("mla_decode: sinks must be [64]")
        if out is None:
            out = torch.empty((n_q, 64, 512), dtype=torch.float32, device=self.device)
        _need(out, torch.float32, "out", self.device)
        ws = None
        nbytes = self.lib.rkv_mla_decode_workspace_bytes(n_q, n_splits)
        if nbytes > 0:
            if workspace is not None and workspace.is_cuda and workspace.numel() * workspace.element_size() >= nbytes:
                ws = workspace
            else:
                ws = torch.empty(nbytes // 4, dtype=torch.float32, device=self.device)
        scale = softmax_scale if softmax_scale is not None else 1.0 / ROW_DIM ** 0.5
        check(self.lib.rkv_mla_decode_fp8(byref(self.view), layer, _ptr(page_table), page_table.shape[1],
                                          _ptr(seq_lens), _ptr(seq_of_query), _ptr(q), n_q, _ptr(idx), k,
                                          _ptr(sinks), float(scale), n_splits, _ptr(ws), _ptr(out),
                                          _ptr(self.status), _stream(stream)))
        return out

    # -- page moves -----------------------------------------------------------
    def copy_pages(self, src: torch.Tensor, dst: torch.Tensor, stream: torch.cuda.Stream | None = None) -> None:
        """Every layer: page dst[i] <- page src[i] (disjoint sets)."""
        _need(src, torch.int32, "src", self.device)
        _need(dst, torch.int32, "dst", self.device)
        if src.shape != dst.shape or src.dim() != 1:
            raise ShapeMismatch("copy_pages: src and dst must be equal-length vectors")
        check(self.lib.rkv_copy_pages(byref(self.view), _ptr(src), _ptr(dst), src.shape[0], _ptr(self.status),
                                      _stream(stream)))


def select_top_k(scores: torch.Tensor, n_visible: torch.Tensor, k: int, out: torch.Tensor | None = None,
                 n_keys_max: int | None = None, stream: torch.cuda.Stream | None = None) -> torch.Tensor:
    """Top-k selection per query row (see ``rkv_topk_select_f32``):
    ``out[q, :effective_k]`` in descending score, ties to the lowest index;
    ``-1`` past effective_k."""
    lib = _abi.load()
    dev = scores.device
    _need(scores, torch.float32, "scores", dev)
    _need(n_visible, torch.int32, "n_visible", dev)
    if scores.dim() != 2 or n_visible.shape != (scores.shape[0],):
        raise ShapeMismatch("select_top_k: scores [n_q, n_keys] and n_visible [n_q] required")
    if out is None:
        out = torch.empty((scores.shape[0], k), dtype=torch.int32, device=dev)
    _need(out, torch.int32, "out", dev)
    nk = scores.shape[1] if n_keys_max is None else n_keys_max
    check(lib.rkv_topk_select_f32(_ptr(scores), scores.shape[1], scores.shape[0], _ptr(n_visible), nk, k, _ptr(out),
                                  _stream(stream)))
    return out


def _indexer_args(rows, row_start, seq_rows, q, w, seq_of_query, n_visible):
    dev = q.device
    for t, n in ((rows, "rows"), (q, "q"), (w, "w")):
        _need(t, torch.float32, n, dev)
    _need(row_start, torch.int64, "row_start", dev)
    for t, n in ((seq_rows, "seq_rows"), (seq_of_query, "seq_of_query"), (n_visible, "n_visible")):
        _need(t, torch.int32, n, dev)
    n_q = q.shape[0] if q.dim() == 3 else -1
    if rows.dim() != 2 or rows.shape[1] != 128 or q.shape[1:] != (64, 128) or w.shape != (n_q, 64) or \
            seq_of_query.shape != (n_q,) or n_visible.shape != (n_q,) or row_start.shape != seq_rows.shape:
        raise ShapeMismatch("indexer: rows [*, 128], q [n_q, 64, 128], w [n_q, 64], seq_of_query / n_visible "
                            "[n_q], row_start / seq_rows [n_seq]")
    return dev, n_q


def indexer_scores(rows: torch.Tensor, row_start: torch.Tensor, seq_rows: torch.Tensor, q: torch.Tensor,
                   w: torch.Tensor, seq_of_query: torch.Tensor, n_visible: torch.Tensor, max_visible: int,
                   out: torch.Tensor | None = None, status: torch.Tensor | None = None,
                   stream: torch.cuda.Stream | None = None) -> torch.Tensor:
    """Indexer scores (``rkv_indexer_scores_f32``, the scoring of
    IndexerPool::select_top_k, indexer.rs:198-216): f32 [n_q, ld], entries
    [0, n_visible[q]) written.  Device errors go to ``status`` (int32 [1]);
    without one the call synchronises and raises."""
    lib = _abi.load()
    dev, n_q = _indexer_args(rows, row_start, seq_rows, q, w, seq_of_query, n_visible)
    if out is None:
        out = torch.empty((n_q, (max_visible + 3) // 4 * 4), dtype=torch.float32, device=dev)
    _need(out, torch.float32, "out", dev)
    st = status if status is not None else torch.zeros(1, dtype=torch.int32, device=dev)
    check(lib.rkv_indexer_scores_f32(_ptr(rows), _ptr(row_start), _ptr(seq_rows), row_start.shape[0], _ptr(q),
                                     _ptr(w), _ptr(seq_of_query), _ptr(n_visible), n_q, max_visible, _ptr(out),
                                     out.shape[1], _ptr(st), _stream(stream)), "indexer_scores")
    if status is None:
        raise_status_bits(int(st.item()), "indexer_scores")
    return out


def indexer_select_top_k(rows: torch.Tensor, row_start: torch.Tensor, seq_rows: torch.Tensor, q: torch.Tensor,
                         w: torch.Tensor, seq_of_query: torch.Tensor, n_visible: torch.Tensor, max_visible: int,
                         k: int, scores: torch.Tensor | None = None, out: torch.Tensor | None = None,
                         status: torch.Tensor | None = None, stream: torch.cuda.Stream | None = None) -> torch.Tensor:
    """IndexerPool::select_top_k for a batch of queries
    (``rkv_indexer_topk_f32``): int32 [n_q, k], the first min(k, n_visible)
    entries in the reference's order, -1 after."""
    lib = _abi.load()
    dev, n_q = _indexer_args(rows, row_start, seq_rows, q, w, seq_of_query, n_visible)
    if scores is None:
        scores = torch.empty((n_q, (max_visible + 3) // 4 * 4), dtype=torch.float32, device=dev)
    if out is None:
        out = torch.empty((n_q, k), dtype=torch.int32, device=dev)
    _need(scores, torch.float32, "scores", dev)
    _need(out, torch.int32, "out", dev)
    st = status if status is not None else torch.zeros(1, dtype=torch.int32, device=dev)
    check(lib.rkv_indexer_topk_f32(_ptr(rows), _ptr(row_start), _ptr(seq_rows), row_start.shape[0], _ptr(q), _ptr(w),
                                   _ptr(seq_of_query), _ptr(n_visible), n_q, max_visible, k, _ptr(scores),
                                   scores.shape[1], _ptr(out), _ptr(st), _stream(stream)), "indexer_select_top_k")
    if status is None:
        raise_status_bits(int(st.item()), "indexer_select_top_k")
    return out


def remap_pages(page_table: torch.Tensor, remap: torch.Tensor, status: torch.Tensor | None = None,
                stream: torch.cuda.Stream | None = None) -> None:
    """In place: every entry >= 0 becomes remap[entry]."""
    lib = _abi.load()
    dev = page_table.device
    _need(page_table, torch.int32, "page_table", dev)
    _need(remap, torch.int32, "remap", dev)
    check(lib.rkv_remap_pages(_ptr(page_table), page_table.numel(), _ptr(remap), remap.numel(), _ptr(status),
                              _stream(stream)))


def e4m3fn_code_range(first_bits: int, n: int, device: torch.device | str = "cuda") -> torch.Tensor:
    """Device codes for the f32 values with bit patterns first_bits + i."""
    lib = _abi.load()
    out = torch.empty(n, dtype=torch.uint8, device=device)
    check(lib.rkv_e4m3fn_code_range(first_bits, n, _ptr(out), _stream(None)))
    return out


def pool_bytes(n_pages: int, n_layers: int) -> int:
    return int(_abi.load().rkv_pool_bytes(n_pages, n_layers))


__all__ = [
    "KvError", "raise_for_info", "ShapeMismatch", "IndexOutOfRange", "InvalidLayer", "PoolFull", "NonFiniteInput", "InvalidArgument",
    "CudaError", "BackendCapability", "CudaBackend", "PagedKvPool", "select_top_k", "indexer_scores",
    "indexer_select_top_k", "remap_pages",
    "e4m3fn_code_range", "pool_bytes", "PAGE_TOKENS", "PAGE_BYTES", "ROW_DIM",
]
