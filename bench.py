#!/usr/bin/env python
"""Benchmark of the B200 KV-cache hot path (rsLLM's FP8 KV cache).

Headline workload (``config.workload``): the decode-step batched append of
the benchmark's config 2 -- 256 sequences with current lengths uniform in
[1024, 32768], 61 layers, one new bf16 row (512 latent + 64 rope) per sequence
per layer per step, quantised to FP8 E4M3FN into a paged pool of 64-token
pages with a seeded random page table; a new page whenever a sequence crosses
a page boundary.  One step = one launch over all 256 x 61 rows; the K timed
steps are one CUDA-graph replay.

metric/unit: algorithmic HBM bytes moved per second (GB/s) -- per row 1152 B
of bf16 read + 672 B of FP8 row written, plus the 4-byte slot index per
sequence per step; ``tokens_per_s`` (sequence-steps appended per second) is
reported beside it.  Extra keys measure the other configurations of the same
path on the same GPU: ``phases.gather`` (config 3: 64 x 32768 tokens x 61
layers gathered + dequantised), ``phases.topk`` and ``phases.sparse_gather``
(config 4: 32 x 64 queries over 131072 keys, k = 2048, 61 layers).

Multi-GPU: one process per GPU (torchrun), each rank owns its own pool and
runs the whole per-GPU workload (weak scaling); no collective in the timed
region.  ``--impl reference`` times the CPU restatement of rsLLM's path (the
oracle; rsLLM itself is Rust and cannot be built here) on the host cores.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time
from ctypes import byref, c_void_p
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

N_SEQ_APPEND = 256
N_LAYERS = 61
LEN_RANGE = (1024, 32768)
ROW_IN = 576 * 2           # bf16 row read
ROW_OUT = 512 + 8 * 4 + 64 * 2  # stored row written (672 B)
APPEND_ROW_BYTES = ROW_IN + ROW_OUT
GATHER_ROW_BYTES = ROW_OUT + ROW_IN  # stored row read + bf16 row written
L2_BYTES = 126 * 2**20
GB = 1e9

# DRAM bytes (read + write) per row from ncu captures of each kernel
# (profiles/append_quant_c2.md, gather_dequant_c3_small.md,
# sparse_gather_c4_small.md).  The append's figure is the mean over four
# consecutive launches captured without cache control, so each launch carries
# the previous launch's page writes draining from L2: 17,992,896 B read +
# 8,830,016 B written per 15,616-row launch.
NCU_TRAFFIC_PER_ROW = {"append": (17992896 + 8830016) / 15616, "gather": (176206080 + 248001536) / 262144,
                       "sparse_gather": (335133696 + 548617728) / 524288}


# ---------------------------------------------------------------------------
# plumbing
# ---------------------------------------------------------------------------

def peaks() -> tuple[float, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    try:
        return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


class Dist:
    """One process per GPU (torchrun env vars); NCCL between GPUs, gloo when
    no GPU is present (the CPU tests of the multi-rank path).  Only used
    outside timed regions: barriers, the max over ranks of a time, every
    rank's time, and the AND over ranks of a parity check."""

    def __init__(self, backend: str | None = None):
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        self.pg = None
        self.dev = torch.device("cpu")
        if self.world > 1:
            import datetime

            import torch.distributed as dist

            backend = backend or ("nccl" if torch.cuda.is_available() else "gloo")
            timeout = datetime.timedelta(seconds=300)
            if backend == "nccl":
                torch.cuda.set_device(self.local)
                self.dev = torch.device("cuda", self.local)
                dist.init_process_group("nccl", timeout=timeout, device_id=self.dev)
            else:
                dist.init_process_group(backend, timeout=timeout)
            self.pg = dist

    def barrier(self):
        if self.pg:
            self.pg.barrier()
        if torch.cuda.is_available():
            torch.cuda.synchronize()

    def max(self, x: float) -> float:
        if not self.pg:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=self.dev)
        self.pg.all_reduce(t, op=self.pg.ReduceOp.MAX)
        return float(t.item())

    def all(self, x: float) -> list[float]:
        """x of every rank, in rank order."""
        if not self.pg:
            return [x]
        t = torch.tensor([x], dtype=torch.float64, device=self.dev)
        out = [torch.zeros_like(t) for _ in range(self.world)]
        self.pg.all_gather(out, t)
        return [float(o.item()) for o in out]

    def all_true(self, ok: bool | None) -> bool | None:
        """AND over ranks (None -- not checked -- on any rank gives None)."""
        v = -1.0 if ok is None else float(bool(ok))
        vals = self.all(v)
        return None if min(vals) < 0 else all(v > 0 for v in vals)

    def close(self):
        if self.pg:
            self.pg.barrier()
            self.pg.destroy_process_group()


class ClockSampler:
    """nvidia-smi samples (200 ms) of this GPU's clocks and throttle reasons."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,utilization.gpu,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: torch.device):
        self.rows: list[list[str]] = []
        self.proc = None
        try:
            uuid = str(torch.cuda.get_device_properties(device).uuid)
            ident = uuid if uuid.startswith("GPU-") else f"GPU-{uuid}"
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={ident}", f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append([c.strip() for c in line.split(",")])

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"], "samples": 0}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.thread.join(timeout=2)
        sm, mx, reasons, loaded = [], [], set(), 0
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in self.rows:
            try:
                cur, top, util = float(r[0]), float(r[1]), float(r[3])
            except (ValueError, IndexError):
                continue
            mx.append(top)
            if util >= 50:
                loaded += 1
                sm.append(cur)
                for n, v in zip(names, r[5:9]):
                    if v.strip().lower() == "active":
                        reasons.add(n)
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(self.rows), "samples_under_load": loaded}


# cycles of torch's sleep kernel queued ahead of a timed region (about 1 ms at
# 1.9 GHz): the host enqueues the timed work while the GPU still sleeps, so the
# start event is followed at once by the first timed kernel and the host's
# launch latency (a graph launch, the first eager launches) stays outside
LAUNCH_COVER_CYCLES = 2_000_000


def events_time(fn, stream: torch.cuda.Stream) -> float:
    """Milliseconds of fn() on `stream`, by CUDA events recorded on it."""
    a = torch.cuda.Event(enable_timing=True)
    b = torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        torch.cuda._sleep(LAUNCH_COVER_CYCLES)
    a.record(stream)
    fn()
    b.record(stream)
    b.synchronize()
    return a.elapsed_time(b)


def flush_l2(dev):
    buf = torch.empty(2 * L2_BYTES, dtype=torch.uint8, device=dev)
    buf.fill_(1)
    del buf


def same_bytes(storage: torch.Tensor, ref: np.ndarray, chunk: int = 1 << 28) -> bool:
    """Device bytes == host bytes, compared in chunks (no second host copy)."""
    if storage.numel() != ref.size:
        return False
    for c0 in range(0, ref.size, chunk):
        if not np.array_equal(storage[c0:c0 + chunk].cpu().numpy(), ref[c0:c0 + chunk]):
            return False
    return True


def u16(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


# ---------------------------------------------------------------------------
# config 2: decode-step batched append
# ---------------------------------------------------------------------------

class AppendWorkload:
    """Per-rank state of config 2: lengths, page table of the pages the run
    touches, per-step slot mappings, per-step input rows."""

    def __init__(self, n_steps: int, seed: int, dev: torch.device | None, make_rows: bool = True,
                 n_seq: int = N_SEQ_APPEND):
        from rsllm_b200 import synth

        self.n_steps, self.n_seq, self.seed = n_steps, n_seq, seed
        self.slots_np, self.n_pages, self.lens = synth.decode_slots(n_seq, n_steps, seed, LEN_RANGE)
        pos = self.lens[None, :] + np.arange(n_steps)[:, None]
        self.new_pages_per_step = (pos % 64 == 0).sum(axis=1)
        self.rows = None
        if dev is not None:
            self.slots = torch.from_numpy(self.slots_np).to(dev)
            if make_rows:
                n = N_LAYERS * n_seq
                self.rows = torch.empty((n_steps, N_LAYERS, n_seq, 576), dtype=torch.bfloat16, device=dev)
                for j in range(n_steps):
                    self.rows[j].copy_(synth.kv_rows(n, seed=seed * 1000 + j, device=dev).view(N_LAYERS, n_seq, 576))

    def bytes_per_step(self) -> int:
        return N_LAYERS * self.n_seq * APPEND_ROW_BYTES + self.n_seq * 4


def bench_append(args, dist: Dist, dev, peak, n_seq: int = N_SEQ_APPEND, e2e: bool = True) -> dict:
    import rsllm_b200 as rk

    W, K = args.warmup, args.steps
    wl = AppendWorkload(W + K, seed=3 + 7919 * dist.rank, dev=dev, n_seq=n_seq)
    pool = rk.PagedKvPool(wl.n_pages, N_LAYERS, device=dev)
    pool.storage.zero_()
    stream = torch.cuda.Stream(device=dev)

    def capture(inputs_ready: bool):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.stream(stream):
            with torch.cuda.graph(g, stream=stream):
                for j in range(W, W + K):
                    pool.append_layer(0, wl.rows[j], wl.slots[j], inputs_ready=inputs_ready)
        return g

    # the step's rows and slots exist before the previous step's append runs,
    # so the append may read them while that launch drains (inputs ready)
    with torch.cuda.stream(stream):
        for j in range(W):
            pool.append_layer(0, wl.rows[j], wl.slots[j], inputs_ready=True)
    pool.check("append warm-up", stream)
    graph = capture(True)

    def replay():
        with torch.cuda.stream(stream):
            graph.replay()

    # one untimed replay uploads the graph (it rewrites the same rows into the
    # same slots); the timed replay then measures only the K steps
    replay()
    stream.synchronize()
    flush_l2(dev)
    dist.barrier()
    ms_rank = events_time(replay, stream)
    dist.barrier()
    pool.check("append", stream)
    per_rank = dist.all(ms_rank)
    ms = max(per_rank)
    # five more K-step replays (L2 flushed before each), every rank's time
    # kept: the spread a single short window hides
    reps = []
    for _ in range(5):
        flush_l2(dev)
        dist.barrier()
        reps.append(dist.all(events_time(replay, stream)))
    del graph
    # the same steps with every read after the wait on the previous launch
    # (rkv_append_quant_bf16, for inputs a preceding kernel may still write)
    graph = capture(False)
    replay()
    stream.synchronize()
    flush_l2(dev)
    dist.barrier()
    wait_first = dist.max(events_time(replay, stream))
    pool.check("append wait-first", stream)
    del graph
    step_bytes = wl.bytes_per_step()
    res = {
        "ms_per_step": ms / K,
        "gbs_per_gpu": step_bytes * K / (ms * 1e-3) / GB,
        "tokens_per_s_per_gpu": n_seq * K / (ms * 1e-3),
        "step_bytes": step_bytes,
        "per_rank_ms_per_step": [t / K for t in per_rank],
        "repeats_max_over_ranks_ms_per_step": [max(r) / K for r in reps],
        "repeats_median_rank_ms_per_step": [float(np.median(r)) / K for r in reps],
        "wait_first_ms_per_step": wait_first / K,
        "wait_first_gbs_per_gpu": step_bytes * K / (wait_first * 1e-3) / GB,
        "pool": pool,
        "wl": wl,
    }
    # bit-exact check of the whole pool (W + K steps) against the oracle
    res["parity"] = dist.all_true(append_parity(pool, wl))
    # the append's own traffic as a plain copy (rkv_copy_floor_bf16: the same
    # grid, reads before the wait and launch arrangement, no codec), K steps
    # in one graph after an L2 flush like the append: the ceiling the append
    # is set against.  It overwrites the pool's rows, so it runs after the
    # parity check.
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(stream):
        for j in range(W):
            pool.copy_floor_layer(0, wl.rows[j], wl.slots[j])
        with torch.cuda.graph(g, stream=stream):
            for j in range(W, W + K):
                pool.copy_floor_layer(0, wl.rows[j], wl.slots[j])
    graph = g

    def replay_floor():
        with torch.cuda.stream(stream):
            graph.replay()

    replay_floor()
    stream.synchronize()
    floor = []
    for _ in range(3):
        flush_l2(dev)
        dist.barrier()
        floor.append(dist.max(events_time(replay_floor, stream)))
    del graph, g
    floor_ms = min(floor)
    res["copy_floor_ms_per_step"] = floor_ms / K
    res["copy_floor_gbs_per_gpu"] = step_bytes * K / (floor_ms * 1e-3) / GB
    res["append_speed_of_copy_floor"] = floor_ms / ms
    if e2e:
        # end to end through the public API: the host allocator reserves each
        # step's slots, pinned host rows and slots go to the device, append,
        # status word back, every step
        res["e2e"] = bench_append_e2e(wl, W, K, dist, dev)
    return res


def bench_append_f32(args, dist: Dist, dev, peak, n_seq: int = N_SEQ_APPEND) -> dict:
    """Config 2's decode step with f32 rows, rsLLM's own row type
    (rkv_append_quant_f32: the host log2f exponent through its threshold
    table, RoPE rounded to bf16): the headline's slots and values with f32-only
    low bits added, W eager steps then K steps in one CUDA graph after an L2
    flush, max over ranks; parity of the whole pool against the oracle's f32
    append."""
    import oracle
    import rsllm_b200 as rk

    W, K = args.warmup, args.steps
    wl = AppendWorkload(W + K, seed=5 + 7919 * dist.rank, dev=dev, n_seq=n_seq)
    g = torch.Generator(device=dev)
    g.manual_seed(17 + 7919 * dist.rank)
    rows = torch.empty(wl.rows.shape, dtype=torch.float32, device=dev)
    for j in range(W + K):
        r = wl.rows[j].float()
        rows[j] = r * (1.0 + torch.randn(r.shape, generator=g, device=dev) * 2.0 ** -10)
    wl.rows = None
    pool = rk.PagedKvPool(wl.n_pages, N_LAYERS, device=dev)
    pool.storage.zero_()
    stream = torch.cuda.Stream(device=dev)
    with torch.cuda.stream(stream):
        for j in range(W):
            pool.append_layer(0, rows[j], wl.slots[j])
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            for j in range(W, W + K):
                pool.append_layer(0, rows[j], wl.slots[j])

    def replay():
        with torch.cuda.stream(stream):
            graph.replay()

    replay()
    stream.synchronize()
    flush_l2(dev)
    dist.barrier()
    ms = dist.max(events_time(replay, stream))
    pool.check("append f32", stream)
    del graph
    ref = oracle.new_pool(wl.n_pages, N_LAYERS)
    ok = True
    for j in range(W + K):
        ok = ok and oracle.append_rows(ref, wl.n_pages, N_LAYERS, 0, rows[j].cpu().numpy(), wl.slots_np[j],
                                       n_threads=oracle.threads()) == 0
    ok = ok and same_bytes(pool.storage, ref)
    step_bytes = N_LAYERS * n_seq * (576 * 4 + 672) + n_seq * 4
    del pool, rows
    torch.cuda.empty_cache()
    return {"config": f"c2 shape with f32 rows: {n_seq} sequences x {N_LAYERS} layers per step, K = {K} steps in "
                      "one CUDA graph, L2 flushed",
            "ms_per_step": ms / K, "gbs_per_gpu": step_bytes * K / (ms * 1e-3) / GB,
            "frac_of_hbm_peak": step_bytes * K / (ms * 1e-3) / GB / peak, "step_bytes": step_bytes,
            "parity": dist.all_true(ok),
            "parity_sample": "the whole pool after all W + K steps vs the oracle's f32 append"}


def append_parity(pool, wl: AppendWorkload) -> bool:
    """The pool after every step of the run equals the oracle's pool after
    the same appends (fp8_kv_quantize_row_inplace + slot-mapped append)."""
    import oracle

    ref = oracle.new_pool(wl.n_pages, N_LAYERS)
    for j in range(wl.n_steps):
        st = oracle.append_rows(ref, wl.n_pages, N_LAYERS, 0, u16(wl.rows[j]), wl.slots_np[j],
                                n_threads=oracle.threads())
        if st != 0:
            return False
    return same_bytes(pool.storage, ref)


def bench_append_e2e(wl: AppendWorkload, W: int, K: int, dist: Dist, dev) -> dict:
    """Config 2 through the public API, as an engine's decode step runs it:
    ``rkv_seq_reserve`` (the host allocator: a slot per sequence, a new page
    from the free list when a sequence crosses a page boundary) writes the
    step's slots into a pinned buffer, the rows (pinned) and the slots go to
    the device, ``rkv_append_quant_bf16`` quantises them into the pool, the
    status word comes back.  The allocator's pool holds each sequence's
    current page (filled to its length mod 64, the sequences created in a
    seeded random order, so page ids are scattered) and the pages it grows
    into; the earlier full pages of a context play no part in a decode step."""
    from rsllm_b200.prefix_pool import PrefixKvPool

    n_seq = wl.n_seq
    steps = W + K
    n_pages = n_seq * (2 + (64 + steps) // 64)
    pool = PrefixKvPool(n_pages, N_LAYERS, device=dev)
    stream = torch.cuda.Stream(device=dev)
    order = np.random.default_rng(wl.seed).permutation(n_seq)
    seqs = np.empty(n_seq, np.int64)
    for i in order:
        seqs[i] = pool.create_sequence()
        r = int(wl.lens[i] % 64) or 64
        pool.reserve([int(seqs[i])], [r], stream=stream)
    ones = np.ones(n_seq, np.int64)
    n_host = min(K, 8)
    host_rows = [wl.rows[W + j].cpu().pin_memory() for j in range(n_host)]
    # one pinned tensor per step: copies out of slices of one pinned tensor
    # measured ~45% slower per step on this path
    host_slots = [torch.empty(n_seq, dtype=torch.int32).pin_memory() for _ in range(steps)]
    host_slots_np = [t.numpy() for t in host_slots]
    dev_rows = [torch.empty_like(wl.rows[0]) for _ in range(2)]
    dev_slots = [torch.empty(n_seq, dtype=torch.int32, device=dev) for _ in range(2)]
    status_host = torch.empty(steps, dtype=torch.int32).pin_memory()
    kv = pool.kv

    def run(j0, j1):
        with torch.cuda.stream(stream):
            for j in range(j0, j1):
                b = j & 1
                pool.reserve(seqs, ones, stream=stream, out=host_slots_np[j])
                dev_rows[b].copy_(host_rows[j % n_host], non_blocking=True)
                dev_slots[b].copy_(host_slots[j], non_blocking=True)
                kv.append_layer(0, dev_rows[b], dev_slots[b], inputs_ready=True)  # filled by the copies above
                status_host[j:j + 1].copy_(kv.status, non_blocking=True)

    run(0, W)  # warm-up steps
    torch.cuda.synchronize()
    kv.status.zero_()
    dist.barrier()
    ms_rank = events_time(lambda: run(W, steps), stream)
    per_rank = dist.all(ms_rank)
    ms = max(per_rank)
    assert int(status_host[W:].abs().sum()) == 0, "append reported device errors"
    new_pages = int(sum(int(np.count_nonzero(host_slots_np[j] % 64 == 0)) for j in range(W, steps)))
    pool.close()
    h2d = wl.rows[0].numel() * 2 + n_seq * 4
    return {"value": dist.world * wl.bytes_per_step() * K / (ms * 1e-3) / GB, "unit": "GB/s",
            "tokens_per_s": dist.world * n_seq * K / (ms * 1e-3),
            "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": 4, "ms_per_step": ms / K,
            "per_rank_ms_per_step": [t / K for t in per_rank],
            "pages_allocated_in_timed_steps": new_pages,
            "path": "rkv_seq_reserve -> pinned slots + rows H2D -> rkv_append_quant_bf16 -> status D2H, per step"}


def cpu_append_sample(wl: AppendWorkload, W: int, budget_s: float, threads: int) -> dict:
    """The oracle (C restatement of rsLLM's CPU path) on the same steps."""
    import oracle

    pool = oracle.new_pool(wl.n_pages, N_LAYERS)
    steps, t_total, done_bytes = 0, 0.0, 0
    while steps < wl.n_steps - W and (t_total < budget_s or steps == 0):
        rows = u16(wl.rows[W + steps])
        slots = wl.slots_np[W + steps]
        t0 = time.perf_counter()
        st = oracle.append_rows(pool, wl.n_pages, N_LAYERS, 0, rows, slots, n_threads=threads)
        t_total += time.perf_counter() - t0
        assert st == 0
        steps += 1
        done_bytes += wl.bytes_per_step()
    return {"value": done_bytes / t_total / GB, "unit": "GB/s", "cores": threads, "kind": "port",
            "sample": f"{steps} decode steps of config 2 ({steps * N_LAYERS * wl.n_seq} rows), "
                      f"{t_total:.1f} s on {threads} threads",
            "tokens_per_s": steps * wl.n_seq / t_total}


def cpu_phase_samples(threads: int, seed: int = 11) -> dict:
    """The oracle (C restatement of rsLLM's paths) on bounded samples of the
    config-3/4/5 work, on `threads` host threads: a rate per phase in the
    phase's own unit, which extrapolates linearly to the full configuration
    (every unit -- row, query, page -- costs the same).
      gather: 4 sequences x 32,768 rows of one layer, pages in seeded random
        order (the c3 shape per sequence);
      topk: 32 queries over 131,072 N(0,1) scores, k = 2048, the reference's
        repeated strict-`>` scan (indexer.rs:218-236);
      sparse_gather: 16 queries x 2048 selected rows of the gather sample;
      page moves: 4096 pages copied (compaction, 2 x 43,008 B per page)."""
    import oracle

    def timed(fn, min_s: float = 0.5, max_reps: int = 200):
        """Seconds per call of fn, repeated until min_s have passed."""
        reps, t0 = 0, time.perf_counter()
        while True:
            fn()
            reps += 1
            dt = time.perf_counter() - t0
            if dt >= min_s or reps >= max_reps:
                return dt / reps, reps

    rng = np.random.default_rng(seed)
    out = {}
    n_seq, ctx = 4, 32768
    ppseq = ctx // 64
    n_pages = n_seq * ppseq + 4096
    pool = oracle.new_pool(n_pages, 1)
    perm = rng.permutation(n_seq * ppseq).astype(np.int32)
    pt = perm.reshape(n_seq, ppseq)
    rows = rng.standard_normal((n_seq * ctx, 576)).astype(np.float32)
    bf = (rows.view(np.uint32) >> 16).astype(np.uint16)
    slots = (pt[:, :, None] * 64 + np.arange(64)[None, None, :]).reshape(-1).astype(np.int32)
    assert oracle.append_rows(pool, n_pages, 1, 0, bf, slots, n_threads=threads) == 0
    cu = (np.arange(n_seq + 1) * ctx).astype(np.int32)
    assert oracle.gather_rows(pool, n_pages, 1, 0, pt, cu, n_threads=threads)[1] == 0
    dt, reps = timed(lambda: oracle.gather_rows(pool, n_pages, 1, 0, pt, cu, n_threads=threads))
    out["gather"] = {"value": n_seq * ctx * GATHER_ROW_BYTES / dt / GB, "unit": "GB/s", "cores": threads,
                     "kind": "port",
                     "sample": f"{n_seq} sequences x {ctx} rows of one layer, {reps} x {dt * 1e3:.1f} ms"}

    n_q, n_keys, k = 32, 131072, 2048
    scores = rng.standard_normal((n_q, n_keys)).astype(np.float32)
    nv = np.full(n_q, n_keys, np.int32)
    t0 = time.perf_counter()
    oracle.topk_batch(scores, nv, k, scan=True, n_threads=threads)
    dt = time.perf_counter() - t0
    out["topk"] = {"value": n_q * n_keys * 4 / dt / GB, "unit": "GB/s", "queries_per_s": n_q / dt,
                   "cores": threads, "kind": "port",
                   "sample": f"{n_q} queries x {n_keys} scores, k = {k}, repeated best scan, {dt:.2f} s"}

    n_sq = 16
    idx = np.stack([rng.choice(ctx, k, replace=False) for _ in range(n_sq)]).astype(np.int32)
    sq = (np.arange(n_sq) % n_seq).astype(np.int32)
    sl = np.full(n_seq, ctx, np.int32)
    assert oracle.sparse_gather_rows(pool, n_pages, 1, 0, pt, sq, sl, idx, n_threads=threads)[1] == 0
    dt, reps = timed(lambda: oracle.sparse_gather_rows(pool, n_pages, 1, 0, pt, sq, sl, idx, n_threads=threads))
    out["sparse_gather"] = {"value": n_sq * k * (GATHER_ROW_BYTES + 8) / dt / GB, "unit": "GB/s",
                            "cores": threads, "kind": "port",
                            "sample": f"{n_sq} queries x {k} selected rows, {reps} x {dt * 1e3:.1f} ms"}

    n_move = 4096
    src = rng.permutation(n_seq * ppseq)[:n_move].astype(np.int32)
    dst = (n_seq * ppseq + np.arange(n_move)).astype(np.int32)
    dt, reps = timed(lambda: oracle.copy_pages(pool, n_pages, 1, src, dst))
    out["page_moves"] = {"value": 2 * n_move * 43008 / dt / GB, "unit": "GB/s", "cores": 1, "kind": "port",
                         "sample": f"{n_move} page moves, {reps} x {dt * 1e3:.1f} ms"}
    return out


# ---------------------------------------------------------------------------
# config 3: paged gather + dequant; config 4: top-k + sparse gather
# ---------------------------------------------------------------------------

FILL_CHUNK = 1 << 20


def fill_pool(pool, n_layers_phys: int, slots_all: torch.Tensor, seed: int, dev):
    """Fills every slot of every backed layer through the append kernel, from
    a seeded block of rows reused across chunks (``fill_rows_of`` gives the
    rows any position received)."""
    from rsllm_b200 import synth

    src = synth.kv_rows(FILL_CHUNK, seed=seed, device=dev)
    n = slots_all.numel()
    for layer in range(n_layers_phys):
        for c0 in range(0, n, FILL_CHUNK):
            c1 = min(n, c0 + FILL_CHUNK)
            rot = (layer * 7919 + c0) % FILL_CHUNK
            rows = src[: c1 - c0] if rot == 0 else torch.roll(src, rot, 0)[: c1 - c0]
            pool.append_layer(layer, rows.contiguous(), slots_all[c0:c1])
    pool.check("fill")
    del src


def fill_rows_of(seed: int, dev, layer: int, start: int, count: int) -> np.ndarray:
    """bf16 bits of the rows ``fill_pool`` appended at positions
    [start, start + count) of ``slots_all`` for ``layer`` (one chunk)."""
    from rsllm_b200 import synth

    c0 = start // FILL_CHUNK * FILL_CHUNK
    assert start + count <= c0 + FILL_CHUNK
    rot = (layer * 7919 + c0) % FILL_CHUNK
    src = synth.kv_rows(FILL_CHUNK, seed=seed, device=dev)
    i = (torch.arange(start - c0, start - c0 + count, device=dev) - rot) % FILL_CHUNK
    return u16(src[i])


def oracle_sequence_pool(rows: np.ndarray):
    """An oracle pool holding one sequence's rows in pages 0, 1, ... (its page
    table is the identity)."""
    import oracle

    n = rows.shape[0]
    n_pages = (n + 63) // 64
    ref = oracle.new_pool(n_pages, 1)
    assert oracle.append_rows(ref, n_pages, 1, 0, rows, np.arange(n, dtype=np.int32),
                              n_threads=oracle.threads()) == 0
    return ref, n_pages, np.arange(n_pages, dtype=np.int32).reshape(1, -1)


def bench_gather(args, dist: Dist, dev, peak, n_seq: int | None = None, mla: bool = True):
    import oracle
    import rsllm_b200 as rk
    from rsllm_b200 import synth

    ctx = 32768
    n_seq = n_seq or (8 if args.small else 64)
    pages_per = ctx // 64
    n_pages = n_seq * pages_per
    free, _ = torch.cuda.mem_get_info(dev)
    out_bytes = n_seq * ctx * 576 * 2
    per_layer = n_pages * rk.PAGE_BYTES
    n_layers = 1 if args.small else N_LAYERS
    l_phys = int(min(n_layers, (free - out_bytes - 8 * 2**30) // per_layer))
    if l_phys < 1:
        return {"skipped": "not enough device memory"}, None
    perm = synth.permutation(n_pages, seed=4 + 7919 * dist.rank).to(dev)
    pt = perm.view(n_seq, pages_per).contiguous()
    tok = torch.arange(ctx, device=dev, dtype=torch.int32)
    slots_all = (pt[:, tok // 64] * 64 + (tok % 64)).reshape(-1).contiguous()
    fill_seed = 40 + dist.rank
    pool = rk.PagedKvPool(n_pages, l_phys, device=dev)
    fill_pool(pool, l_phys, slots_all, seed=fill_seed, dev=dev)
    del slots_all
    cu = torch.arange(0, (n_seq + 1) * ctx, ctx, dtype=torch.int32, device=dev)
    out = torch.empty((n_seq * ctx, 576), dtype=torch.bfloat16, device=dev)
    stream = torch.cuda.Stream(device=dev)

    def step():
        for layer in range(n_layers):
            pool.rows(layer % l_phys, pt, cu, ctx, out=out, stream=stream)

    for _ in range(args.phase_warmup):
        step()
    pool.check("gather", stream)
    dist.barrier()
    per_rank = dist.all(events_time(lambda: [step() for _ in range(args.phase_steps)], stream))
    ms = max(per_rank)
    pool.check("gather", stream)
    # per-launch duration of the kernel alone
    one = events_time(lambda: pool.rows(0, pt, cu, ctx, out=out, stream=stream), stream)
    # parity: the first and last sequence of the first and last backed layer,
    # gathered by the timed launch shape, against the oracle's append + gather
    # of the rows the fill put there
    ok = True
    for layer in sorted({0, l_phys - 1}):
        pool.rows(layer, pt, cu, ctx, out=out, stream=stream)
        pool.check("gather parity", stream)
        for s in sorted({0, n_seq - 1}):
            ref, rp, rpt = oracle_sequence_pool(fill_rows_of(fill_seed, dev, layer, s * ctx, ctx))
            want, st = oracle.gather_rows(ref, rp, 1, 0, rpt, np.array([0, ctx], np.int32),
                                          n_threads=oracle.threads())
            ok = ok and st == 0 and np.array_equal(u16(out[s * ctx:(s + 1) * ctx]), want)
    rows = n_seq * ctx
    step_bytes = n_layers * (rows * GATHER_ROW_BYTES + n_pages * 4)
    res = {"config": f"c3: {n_seq} seqs x {ctx} ctx x {n_layers} layers, random page order",
           "layers_backed": l_phys, "ms_per_step": ms / args.phase_steps,
           "per_rank_ms_per_step": [t / args.phase_steps for t in per_rank],
           "gbs_per_gpu": step_bytes * args.phase_steps / (ms * 1e-3) / GB,
           "frac_of_hbm_peak": None, "kernel_ms_per_layer": one,
           "launches_per_step": n_layers, "step_bytes": step_bytes,
           "parity": dist.all_true(ok),
           "parity_sample": "sequences first + last of layers first + last backed, every lane vs the oracle"}
    res["frac_of_hbm_peak"] = res["gbs_per_gpu"] / peak
    del out
    torch.cuda.empty_cache()
    res_mla = None
    if mla:
        seq_lens = torch.full((n_seq,), ctx, dtype=torch.int32, device=dev)
        res_mla = bench_mla(args, dist, pool, pt, seq_lens, torch.arange(n_seq, dtype=torch.int32, device=dev),
                            None, n_layers, l_phys, stream, peak,
                            f"c3 shape: {n_seq} decode queries (one per sequence) x {ctx} rows x {n_layers} layers",
                            n_splits=args.mla_splits)
    del pool
    torch.cuda.empty_cache()
    return res, res_mla


def mla_flops_bytes(n_q: int, n_keys: int, with_index: bool) -> tuple[float, float]:
    """Algorithmic FLOPs and HBM bytes of one MLA decode launch over n_keys
    (query, key) pairs in total: 64 heads x
    (576 + 512) MACs per (query, key); each key row read once in its stored
    form (672 B, plus its 4 B page-table entry, plus its 4 B index when an
    index list selects it), q in bf16, the f32 output."""
    flops = 2.0 * n_keys * 64 * (576 + 512)
    per_key = 672 + (8 if with_index else 4.0 / 64)
    return flops, n_keys * per_key + n_q * (64 * 576 * 2 + 64 * 512 * 4)


def bench_mla(args, dist: Dist, pool, pt, seq_lens, seq_of_query, idx, n_layers: int, l_phys: int, stream, peak,
              config: str, n_splits: int = 1) -> dict:
    """MLA decode attention over the FP8 pages (rkv_mla_decode_fp8), one launch
    per layer; idx None = every row of each query's sequence."""
    dev = pt.device
    n_q = seq_of_query.numel()
    g = torch.Generator(device=dev)
    g.manual_seed(900 + 7919 * dist.rank)
    q = torch.randn((n_q, 64, 576), generator=g, device=dev, dtype=torch.float32).to(torch.bfloat16)
    out = torch.empty((n_q, 64, 512), dtype=torch.float32, device=dev)
    import rsllm_b200 as rk

    nbytes = rk._abi.load().rkv_mla_decode_workspace_bytes(n_q, n_splits)
    ws = torch.empty(max(1, nbytes // 4), dtype=torch.float32, device=dev)
    sinks = torch.zeros(64, dtype=torch.float32, device=dev)

    def one(layer):
        pool.mla_decode(layer % l_phys, q, pt, seq_lens, seq_of_query, None if idx is None else idx[layer], sinks,
                        None, n_splits, out=out, workspace=ws, stream=stream)

    def step():
        for layer in range(n_layers):
            one(layer)

    for _ in range(args.phase_warmup):
        step()
    pool.check("mla", stream)
    dist.barrier()
    per_rank = dist.all(events_time(lambda: [step() for _ in range(args.phase_steps)], stream))
    ms = max(per_rank)
    pool.check("mla", stream)
    kernel_ms = events_time(lambda: one(0), stream)  # leaves layer 0's output in out
    torch.cuda.synchronize(dev)
    sample = sorted({0, n_q - 1})
    ok = all(mla_parity(pool, pt, seq_lens, seq_of_query, None if idx is None else idx[0], q, out, qi)
             for qi in sample)
    if idx is None:
        n_keys = int(seq_lens[seq_of_query.long()].sum().item())
    else:
        n_keys = int(idx.shape[1] * idx.shape[2])
    flops, nbytes_alg = mla_flops_bytes(n_q, n_keys, idx is not None)
    peaks_all = json.loads((ROOT / "MEASURED_PEAKS.json").read_text()) if (ROOT / "MEASURED_PEAKS.json").exists() \
        else {"bf16_tflops_sustained": 1400.0}
    tc_peak = float(peaks_all.get("bf16_tflops_sustained", 1400.0))
    t_layer = ms / args.phase_steps / n_layers * 1e-3
    t_ideal = max(nbytes_alg / (peak * GB), flops / (tc_peak * 1e12))
    return {"config": config, "layers_backed": l_phys, "n_splits": n_splits,
            "ms_per_step": ms / args.phase_steps, "per_rank_ms_per_step": [t / args.phase_steps for t in per_rank],
            "kernel_ms_per_layer": kernel_ms,
            "gbs_per_gpu": nbytes_alg / t_layer / GB, "tflops_per_gpu": flops / t_layer / 1e12,
            "frac_of_hbm_peak": nbytes_alg / t_layer / GB / peak,
            "frac_of_tensor_peak_sustained": flops / t_layer / 1e12 / tc_peak,
            "roofline_frac": t_ideal / t_layer,
            "roofline_bound": "hbm" if nbytes_alg / (peak * GB) >= flops / (tc_peak * 1e12) else "tensor",
            "algorithmic_bytes_per_launch": nbytes_alg, "flops_per_launch": flops,
            "parity": dist.all_true(ok),
            "parity_sample": f"queries {sample} of layer 0 vs the oracle on their sequence's pages: every lane "
                             "within 2^-8 of the largest |latent| averaged, mean error 16x below"}


def mla_parity(pool, pt, seq_lens, seq_of_query, idx0, q, out, qi: int) -> bool:
    """Query qi of layer 0 against the oracle's attention.rs:493-663, run on a
    copy of just its sequence's pages (page i of the sequence as page i): the
    kernel's output must be within 2^-8 of the largest |latent| among the rows
    it averages in every lane, and 16x closer on average (the bound the MLA
    tests use: bf16-rounded softmax weights, f32 elsewhere)."""
    import oracle
    from rsllm_b200._abi import PAGE_BYTES

    s = int(seq_of_query[qi])
    n_keys = int(seq_lens[s])
    n_pg = (n_keys + 63) // 64
    if n_pg == 0:
        return bool(torch.all(out[qi] == 0))
    pages = pool.storage.view(pool.n_layers, pool.n_pages, PAGE_BYTES)[0]
    mini = np.ascontiguousarray(pages.index_select(0, pt[s, :n_pg].long()).cpu().numpy().reshape(-1))
    mpt = np.arange(n_pg, dtype=np.int32)[None, :]
    lens = np.array([n_keys], np.int32)
    qb = q[qi:qi + 1].view(torch.int16).cpu().numpy().view(np.uint16)
    ix = None if idx0 is None else np.ascontiguousarray(idx0[qi:qi + 1].cpu().numpy(), np.int32)
    ref, st = oracle.mla_decode(mini, n_pg, 1, 0, mpt, lens, np.zeros(1, np.int32), qb, ix,
                                np.zeros(64, np.float32), 1.0 / 24.0, oracle.threads())
    if ix is None:
        rows, st2 = oracle.gather_rows(mini, n_pg, 1, 0, mpt, np.array([0, n_keys], np.int32), oracle.threads())
    else:
        rows, st2 = oracle.sparse_gather_rows(mini, n_pg, 1, 0, mpt, np.zeros(1, np.int32), lens, ix,
                                              oracle.threads())
    latent = (rows.reshape(-1, rows.shape[-1])[:, :512].astype(np.uint32) << 16).view(np.float32)
    scale = float(np.abs(latent).max()) if latent.size else 1.0
    scale = scale if scale > 0 else 1.0
    err = np.abs(out[qi].cpu().numpy().astype(np.float64) - ref[0]) / scale
    return bool(st == 0 and st2 == 0 and np.all(np.isfinite(out[qi].cpu().numpy())) and
                err.max() <= 2.0 ** -8 and err.mean() <= 2.0 ** -12)


def bench_sparse(args, dist: Dist, dev, peak, n_seq: int | None = None, mla: bool = True) -> dict:
    import oracle
    import rsllm_b200 as rk
    from rsllm_b200 import synth

    ctx, n_qpos, k = 131072, 64, 2048
    n_seq = n_seq or (4 if args.small else 32)
    pages_per = ctx // 64
    n_pages = n_seq * pages_per
    n_q = n_seq * n_qpos
    n_score_mats = 1 if args.small else 4
    n_layers = 1 if args.small else N_LAYERS
    out_bytes = n_q * k * 576 * 2
    score_bytes = n_score_mats * n_q * ctx * 4
    idx_bytes = n_layers * n_q * k * 4
    free, _ = torch.cuda.mem_get_info(dev)
    per_layer = n_pages * rk.PAGE_BYTES
    l_phys = int(min(n_layers, (free - out_bytes - score_bytes - idx_bytes - 10 * 2**30) // per_layer))
    if l_phys < 1:
        return {"skipped": "not enough device memory"}
    perm = synth.permutation(n_pages, seed=6 + 7919 * dist.rank).to(dev)
    pt = perm.view(n_seq, pages_per).contiguous()
    tok = torch.arange(ctx, device=dev, dtype=torch.int32)
    slots_all = (pt[:, tok // 64] * 64 + (tok % 64)).reshape(-1).contiguous()
    fill_seed = 60 + dist.rank
    pool = rk.PagedKvPool(n_pages, l_phys, device=dev)
    fill_pool(pool, l_phys, slots_all, seed=fill_seed, dev=dev)
    del slots_all
    torch.cuda.empty_cache()
    scores = [synth.scores(n_q, ctx, seed=500 + 31 * i + 7919 * dist.rank, device=dev) for i in range(n_score_mats)]
    # query i of sequence s sits at position ctx - n_qpos + i: causal visibility
    n_visible = (ctx - n_qpos + 1 + torch.arange(n_qpos, device=dev, dtype=torch.int32)).repeat(n_seq).contiguous()
    seq_of_query = torch.arange(n_seq, device=dev, dtype=torch.int32).repeat_interleave(n_qpos).contiguous()
    seq_lens = torch.full((n_seq,), ctx, dtype=torch.int32, device=dev)
    idx = torch.empty((n_layers, n_q, k), dtype=torch.int32, device=dev)
    out = torch.empty((n_q, k, 576), dtype=torch.bfloat16, device=dev)
    stream = torch.cuda.Stream(device=dev)

    def topk_step():
        for layer in range(n_layers):
            rk.select_top_k(scores[layer % n_score_mats], n_visible, k, out=idx[layer], stream=stream)

    def sparse_step():
        for layer in range(n_layers):
            pool.sparse_rows(layer % l_phys, pt, seq_of_query, seq_lens, idx[layer], out=out, stream=stream)

    for _ in range(args.phase_warmup):
        topk_step()
        sparse_step()
    pool.check("sparse", stream)
    dist.barrier()
    rank_topk = dist.all(events_time(lambda: [topk_step() for _ in range(args.phase_steps)], stream))
    dist.barrier()
    rank_sparse = dist.all(events_time(lambda: [sparse_step() for _ in range(args.phase_steps)], stream))
    ms_topk, ms_sparse = max(rank_topk), max(rank_sparse)
    pool.check("sparse", stream)
    one_topk = events_time(lambda: rk.select_top_k(scores[0], n_visible, k, out=idx[0], stream=stream), stream)
    one_sparse = events_time(lambda: pool.sparse_rows(0, pt, seq_of_query, seq_lens, idx[0], out=out,
                                                      stream=stream), stream)
    pool.check("sparse", stream)
    # parity on layer 0 (idx[0] and out now hold its selection and rows):
    # sampled queries of the first and last sequence, every index against the
    # oracle's selection and every gathered lane against the oracle's pool
    sample = sorted({0, 1, n_qpos // 2, n_qpos - 1, n_q - n_qpos, n_q - 1})
    nv_np = n_visible.cpu().numpy()
    sc0 = scores[0][sample].cpu().numpy()
    want_idx = oracle.topk_batch(sc0, nv_np[sample], k, n_threads=oracle.threads())
    got_idx = idx[0][sample].cpu().numpy()
    ok_topk = bool(np.array_equal(got_idx, want_idx))
    ok_sparse = ok_topk
    sq_np = seq_of_query.cpu().numpy()
    for s in sorted({int(sq_np[q]) for q in sample}):
        qs = [q for q in sample if int(sq_np[q]) == s]
        ref, rp, rpt = oracle_sequence_pool(fill_rows_of(fill_seed, dev, 0, s * ctx, ctx))
        want, st = oracle.sparse_gather_rows(ref, rp, 1, 0, rpt, np.zeros(len(qs), np.int32),
                                             np.array([ctx], np.int32), idx[0][qs].cpu().numpy(),
                                             n_threads=oracle.threads())
        ok_sparse = ok_sparse and st == 0 and np.array_equal(u16(out[qs]), want)
    sel = n_q * k
    sparse_bytes = n_layers * sel * (GATHER_ROW_BYTES + 4 + 4)
    vis = int(n_visible.sum().item())
    topk_bytes = n_layers * (vis * 4 + sel * 4)
    P = args.phase_steps
    res = {
        "topk": {"config": f"c4: {n_q} queries ({n_seq} seqs x last 64 positions, causal) over 131072 keys, "
                           f"k=2048, {n_layers} layers cycling {n_score_mats} seeded N(0,1) score matrices",
                 "ms_per_step": ms_topk / P, "per_rank_ms_per_step": [t / P for t in rank_topk],
                 "gbs_per_gpu": topk_bytes * P / (ms_topk * 1e-3) / GB,
                 "frac_of_hbm_peak": topk_bytes * P / (ms_topk * 1e-3) / GB / peak,
                 "queries_per_s_per_gpu": n_layers * n_q * P / (ms_topk * 1e-3),
                 "kernel_ms_per_layer": one_topk, "step_bytes": topk_bytes,
                 "parity": dist.all_true(ok_topk),
                 "parity_sample": f"queries {sample} of layer 0: every index in order vs the oracle"},
        "sparse_gather": {"config": f"c4: {n_q} queries x 2048 selected rows x {n_layers} layers, random page order",
                          "layers_backed": l_phys, "ms_per_step": ms_sparse / P,
                          "per_rank_ms_per_step": [t / P for t in rank_sparse],
                          "gbs_per_gpu": sparse_bytes * P / (ms_sparse * 1e-3) / GB,
                          "frac_of_hbm_peak": sparse_bytes * P / (ms_sparse * 1e-3) / GB / peak,
                          "kernel_ms_per_layer": one_sparse, "step_bytes": sparse_bytes,
                          "parity": dist.all_true(ok_sparse),
                          "parity_sample": f"queries {sample} of layer 0: every lane of their 2048 rows vs the "
                                           "oracle"},
    }
    del out, scores
    torch.cuda.empty_cache()
    if mla:
        res["mla_decode_sparse"] = bench_mla(
            args, dist, pool, pt, seq_lens, seq_of_query, idx, n_layers, l_phys, stream, peak,
            f"c4 shape: {n_q} queries x 2048 top-k rows (the indices above) x {n_layers} layers")
    del pool, idx
    torch.cuda.empty_cache()
    return res


def bench_topk_only(args, dist: Dist, dev, peak) -> dict:
    """Config 4's top-k alone (no pool): 2048 queries (32 sequences x the last
    64 positions, causal) over 131072 seeded N(0,1) scores, k = 2048, two
    score matrices alternating -- about 1 GB on the device, a size for
    profiling the two top-k kernels."""
    import rsllm_b200 as rk
    from rsllm_b200 import synth

    n_seq, ctx, n_qpos, k = 32, 131072, 64, 2048
    n_q = n_seq * n_qpos
    scores = [synth.scores(n_q, ctx, seed=500 + 31 * i + 7919 * dist.rank, device=dev) for i in range(2)]
    n_visible = (ctx - n_qpos + 1 + torch.arange(n_qpos, device=dev, dtype=torch.int32)).repeat(n_seq).contiguous()
    out = torch.empty((n_q, k), dtype=torch.int32, device=dev)
    stream = torch.cuda.Stream(device=dev)
    for i in range(args.phase_warmup):
        rk.select_top_k(scores[i % 2], n_visible, k, out=out, stream=stream)
    P = max(1, args.phase_steps)
    ms = dist.max(events_time(lambda: [rk.select_top_k(scores[i % 2], n_visible, k, out=out, stream=stream)
                                       for i in range(P)], stream)) / P
    nbytes = int(n_visible.sum().item()) * 4 + n_q * k * 4
    return {"config": f"c4 top-k: {n_q} queries x {ctx} keys (causal), k = {k}", "ms_per_call": ms,
            "gbs_per_gpu": nbytes / (ms * 1e-3) / GB, "frac_of_hbm_peak": nbytes / (ms * 1e-3) / GB / peak}


def compress_bytes(n_tok: int, n_emit: int, ring_rows_written: int, ring_src_read: int) -> int:
    """Algorithmic HBM bytes of one rkv_compress_append call (ratio 4, two
    lanes of 576): every input (kv, score) row read once (9216 B), the ring
    rows written for the next call (9216 B each), the ring half-rows the
    emissions read (kv + score of one lane: 4608 B each) and the emitted
    stored rows (672 B)."""
    return n_tok * 9216 + ring_rows_written * 9216 + ring_src_read * 4608 + n_emit * 672


def bench_compress(args, dist: Dist, dev, peak) -> dict:
    """Compressor emission (rkv_compress_append, ratio 4, coff 2) as a decode
    step -- one token of each of 256 sequences per layer, 61 layers, a quarter
    of them emitting, the whole step captured in one CUDA graph -- and as a
    prefill -- 8 sequences x 4096 tokens per layer call, 61 layers."""
    import oracle
    import rsllm_b200 as rk

    res = {}
    g = torch.Generator(device=dev)
    g.manual_seed(500 + 7919 * dist.rank)
    norm = (torch.rand(576, generator=g, device=dev) + 0.5).contiguous()
    ape = torch.randn((4, 1152), generator=g, device=dev).contiguous()
    stream = torch.cuda.Stream(device=dev)
    n_layers = 1 if args.small else N_LAYERS

    # -- decode step ---------------------------------------------------------------
    n_seq, n_var, p0 = 256, 4, 8192
    pool = rk.PagedKvPool(n_seq, n_layers, device=dev)
    banks = rk.CompressorBank(4, n_seq * n_layers, device=dev, max_positions=p0 + 4096)
    kv = torch.randn((n_var, n_layers, n_seq, 1152), generator=g, device=dev)
    sc = torch.randn((n_var, n_layers, n_seq, 1152), generator=g, device=dev) * 3
    seq = torch.arange(n_seq, dtype=torch.int32, device=dev)
    sid = [(seq + layer * n_seq).contiguous() for layer in range(n_layers)]
    n_pos_steps = args.phase_warmup + 3 + args.phase_steps + 2
    pos = [(seq + p0 + j).contiguous() for j in range(n_pos_steps)]
    slot = [(seq * 64 + ((seq + p0 + j + 1) // 4) % 64).to(torch.int32).contiguous() for j in range(n_pos_steps)]
    state = {"j": 0}

    def dstep(j, flags=True):
        # a decode step: one token per state, metadata tensors made before the
        # step (RKV_COMPRESS_INPUTS_READY | RKV_COMPRESS_ONE_TOKEN_PER_STATE)
        for layer in range(n_layers):
            banks.append(pool, layer, kv[j % n_var, layer], sc[j % n_var, layer], pos[j], sid[layer], slot[j], norm,
                         ape, stream=stream, inputs_ready=flags, one_token_per_state=flags)

    # the timed steps (positions advancing) are one CUDA graph; an untimed
    # replay uploads it (it recomputes the same rows into the same slots)
    with torch.cuda.stream(stream):
        for j in range(args.phase_warmup + 3):
            dstep(j)
    pool.check("compress decode", stream)
    torch.cuda.synchronize(dev)

    def timed_graph(flags):
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            for j in range(args.phase_warmup + 3, args.phase_warmup + 3 + args.phase_steps):
                dstep(j, flags)

        def replay():
            with torch.cuda.stream(stream):
                graph.replay()

        replay()
        stream.synchronize()
        flush_l2(dev)
        dist.barrier()
        t = dist.max(events_time(replay, stream)) / args.phase_steps
        pool.check("compress decode", stream)
        del graph
        return t

    ms_plain = timed_graph(False)  # two launches per layer, every read after the wait
    ms = timed_graph(True)
    one = events_time(lambda: banks.append(pool, 0, kv[0, 0], sc[0, 0], pos[-1], sid[0], slot[-1], norm, ape,
                                           stream=stream), stream)
    n_emit = n_seq // 4
    per_layer = compress_bytes(n_seq, n_emit, n_seq, n_emit * 7)
    t_layer = ms * 1e-3 / n_layers
    res["compress_decode"] = {
        "config": f"ratio 4 (two lanes of 576), {n_seq} sequences x 1 token x {n_layers} layers per step, "
                  f"positions {p0}+i (a quarter emit), whole step in one CUDA graph",
        "ms_per_step": ms, "tokens_per_s_per_gpu": n_seq * n_layers / (ms * 1e-3),
        "emissions_per_s_per_gpu": n_emit * n_layers / (ms * 1e-3),
        "algorithmic_bytes_per_layer": per_layer, "gbs_per_gpu": per_layer / t_layer / GB,
        "frac_of_hbm_peak": per_layer / t_layer / GB / peak, "ms_per_layer": ms / n_layers,
        "ms_per_layer_plain": ms_plain / n_layers, "ms_per_layer_ungraphed": one,
        "launches_per_step": n_layers,
        "flags": "RKV_COMPRESS_INPUTS_READY | RKV_COMPRESS_ONE_TOKEN_PER_STATE",
        "ms_per_step_plain": ms_plain, "launches_per_step_plain": 2 * n_layers}
    del kv, sc, banks, pool
    torch.cuda.empty_cache()

    # -- prefill --------------------------------------------------------------------
    n_seq, per = (2, 4096) if args.small else (8, 4096)
    n_tok = n_seq * per
    pool = rk.PagedKvPool(n_seq * per // 4 // 64, n_layers, device=dev)
    banks = rk.CompressorBank(4, n_seq * n_layers, device=dev, max_positions=per)
    kvp = torch.randn((n_tok, 1152), generator=g, device=dev)
    scp = torch.randn((n_tok, 1152), generator=g, device=dev) * 3
    posp = torch.arange(per, dtype=torch.int32, device=dev).repeat(n_seq).contiguous()
    seqp = torch.arange(n_seq, dtype=torch.int32, device=dev).repeat_interleave(per)
    slotp = (seqp * (per // 4) + (posp + 1) // 4 - 1).to(torch.int32).contiguous()
    sidp = [(seqp + layer * n_seq).to(torch.int32).contiguous() for layer in range(n_layers)]

    def pstep():
        for layer in range(n_layers):
            banks.append(pool, layer, kvp, scp, posp, sidp[layer], slotp, norm, ape, stream=stream)

    for _ in range(args.phase_warmup):
        pstep()
    pool.check("compress prefill", stream)
    dist.barrier()
    msp = dist.max(events_time(lambda: [pstep() for _ in range(args.phase_steps)], stream)) / args.phase_steps
    pool.check("compress prefill", stream)
    onep = events_time(lambda: banks.append(pool, 0, kvp, scp, posp, sidp[0], slotp, norm, ape, stream=stream),
                       stream)
    n_emit = n_tok // 4
    per_layer = compress_bytes(n_tok, n_emit, n_seq * 8, 0)
    t_layer = msp * 1e-3 / n_layers
    # CPU: the oracle (reference state machine, threads over sequences) on one layer's first 512 tokens per seq
    cpu_per = 512
    sel = (posp < cpu_per).cpu().numpy()
    ref_pool = oracle.new_pool(pool.n_pages, 1)
    kv_c, sc_c = kvp.cpu().numpy()[sel], scp.cpu().numpy()[sel]
    args_c = (posp.cpu().numpy()[sel], seqp.cpu().numpy().astype(np.int32)[sel], slotp.cpu().numpy()[sel])
    t0 = time.perf_counter()
    oracle.compress_append(ref_pool, pool.n_pages, 1, 0, 4, oracle.compress_states(n_seq, 4), kv_c, sc_c, *args_c,
                           ape.cpu().numpy(), norm.cpu().numpy())
    cpu_s = time.perf_counter() - t0
    res["compress_prefill"] = {
        "config": f"ratio 4 (two lanes of 576), {n_seq} sequences x {per} tokens per layer call x {n_layers} layers",
        "ms_per_step": msp, "tokens_per_s_per_gpu": n_tok * n_layers / (msp * 1e-3),
        "algorithmic_bytes_per_layer": per_layer, "gbs_per_gpu": per_layer / t_layer / GB,
        "frac_of_hbm_peak": per_layer / t_layer / GB / peak, "kernel_ms_per_layer": onep,
        "cpu_baseline": {"tokens_per_s": n_seq * cpu_per / cpu_s, "cores": min(n_seq, oracle.threads()),
                         "kind": "port", "sample": f"{n_seq} x {cpu_per} tokens of one layer, threads over sequences"}}
    del kvp, scp, banks, pool
    torch.cuda.empty_cache()
    return res


FP32_OPS_PER_S = 35.79e12  # FMUL/FADD lane operations per second, measured on this pool's B200 (1965 MHz)


def bench_indexer(args, dist: Dist, dev, peak) -> dict:
    """Indexer scoring + top-k (rkv_indexer_topk_f32) as a decode step: one
    query per sequence for 32 sequences (config 4's count) at context 131072,
    i.e. 32768 compressed indexer rows each (ratio 4), k = 512 (rsLLM's
    DSV4_N_INDEXER_TOP_K), one launch pair per layer over the same rows (537 MB,
    read from HBM every layer)."""
    import oracle
    import rsllm_b200 as rk

    n_seq, n_rows, k = (8, 32768, 512) if args.small else (32, 32768, 512)
    n_layers = 1 if args.small else N_LAYERS
    g = torch.Generator(device=dev)
    g.manual_seed(700 + 7919 * dist.rank)
    rows = torch.randn((n_seq * n_rows, 128), generator=g, device=dev)
    row_start = (torch.arange(n_seq, device=dev, dtype=torch.int64) * n_rows).contiguous()
    seq_rows = torch.full((n_seq,), n_rows, dtype=torch.int32, device=dev)
    q = torch.randn((n_seq, 64, 128), generator=g, device=dev)
    w = (torch.randn((n_seq, 64), generator=g, device=dev) / 8192 ** 0.5).contiguous()
    sq = torch.arange(n_seq, dtype=torch.int32, device=dev)
    nv = torch.full((n_seq,), n_rows, dtype=torch.int32, device=dev)
    scores = torch.empty((n_seq, n_rows), dtype=torch.float32, device=dev)
    out = torch.empty((n_seq, k), dtype=torch.int32, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    stream = torch.cuda.Stream(device=dev)

    def one():
        rk.indexer_select_top_k(rows, row_start, seq_rows, q, w, sq, nv, n_rows, k, scores=scores, out=out,
                                status=status, stream=stream)

    def score_only():
        rk.indexer_scores(rows, row_start, seq_rows, q, w, sq, nv, n_rows, out=scores, status=status, stream=stream)

    for _ in range(args.phase_warmup):
        for _ in range(n_layers):
            one()
    stream.synchronize()
    dist.barrier()
    ms = dist.max(events_time(lambda: [one() for _ in range(args.phase_steps * n_layers)], stream)) / args.phase_steps
    score_ms = events_time(score_only, stream)
    assert int(status.item()) == 0
    ops = 2.0 * n_seq * n_rows * 64 * 128      # one multiply and one add per lane per head
    nbytes = n_seq * n_rows * 512 + n_seq * (64 * 128 * 4 + 64 * 4) + n_seq * n_rows * 4 + n_seq * k * 4
    t_layer = ms * 1e-3 / n_layers
    # CPU: the oracle's scoring (threads over queries) on 2048 rows of every sequence, then its selection
    sample_rows = 2048
    rows_c = rows.view(n_seq, n_rows, 128)[:, :sample_rows].reshape(-1, 128).cpu().numpy()
    t0 = time.perf_counter()
    sc_c, _ = oracle.indexer_scores(rows_c, np.arange(n_seq) * sample_rows, np.full(n_seq, sample_rows), q.cpu().numpy(),
                                    w.cpu().numpy(), np.arange(n_seq), np.full(n_seq, sample_rows), sample_rows)
    oracle.topk_batch(sc_c, np.full(n_seq, sample_rows, np.int32), k)
    cpu_s = time.perf_counter() - t0
    return {"config": f"{n_seq} decode queries x {n_rows} indexer rows (64 heads x 128, f32) x {n_layers} layers, "
                      f"k = {k}",
            "ms_per_step": ms, "ms_per_layer": ms / n_layers, "score_kernel_ms_per_layer": score_ms,
            "rows_scored_per_s_per_gpu": n_seq * n_rows / t_layer,
            "fp32_ops_per_s": ops / t_layer, "frac_of_fp32_issue_peak": ops / t_layer / FP32_OPS_PER_S,
            "fp32_peak_source": "measured FMUL/FADD-rate micro-benchmark, 35.79 T lane-ops/s",
            "gbs_per_gpu": nbytes / t_layer / GB, "frac_of_hbm_peak": nbytes / t_layer / GB / peak,
            "roofline_bound": "fp32 (bit-exact lane-by-lane f32 dots: no tensor cores, no FMA)",
            "cpu_baseline": {"rows_scored_per_s": n_seq * sample_rows / cpu_s, "cores": min(n_seq, oracle.threads()),
                             "kind": "port", "sample": f"{n_seq} queries x {sample_rows} rows, scoring + selection"}}


def bench_kvc(args, dist: Dist, dev) -> dict:
    """KVC file save and load (prefix persistence) of a config-5-sized prefix
    (8229 tokens) over 61 layers: host-synchronous (device pack / unpack,
    pinned copies, file IO), timed by wall clock; the loaded sequence's rows
    are checked against the saved one."""
    import tempfile

    import rsllm_b200 as rk
    from rsllm_b200 import synth
    from rsllm_b200.prefix_pool import PrefixKvPool

    n_tok, n_layers = (2048, 4) if args.small else (8229, N_LAYERS)
    n_pages = 2 * ((n_tok + 63) // 64) + 2
    pool = PrefixKvPool(n_pages, n_layers, device=dev)
    seq = pool.create_sequence()
    slots = torch.from_numpy(pool.reserve([seq], [n_tok])).to(dev)
    rows = synth.kv_rows(n_tok, seed=77 + dist.rank, device=dev)
    for layer in range(n_layers):
        pool.kv.append_layer(layer, rows, slots)
    pool.kv.check("kvc fill")
    tokens = np.arange(n_tok, dtype=np.int32) + 1000 * dist.rank
    page_bytes = n_layers * ((n_tok + 63) // 64) * rk.PAGE_BYTES
    with tempfile.TemporaryDirectory() as d:
        torch.cuda.synchronize(dev)
        t0 = time.perf_counter()
        path = pool.save_kvc(seq, tokens, d)
        t1 = time.perf_counter()
        s2, _ = pool.load_kvc(path, insert_prefix=False)
        torch.cuda.synchronize(dev)
        t2 = time.perf_counter()
        file_bytes = os.path.getsize(path)
    pt1 = torch.from_numpy(pool.page_table(seq).reshape(1, -1)).to(dev)
    pt2 = torch.from_numpy(pool.page_table(s2).reshape(1, -1)).to(dev)
    cu = torch.tensor([0, n_tok], dtype=torch.int32, device=dev)
    same = all(torch.equal(pool.kv.rows(layer, pt1, cu, n_tok), pool.kv.rows(layer, pt2, cu, n_tok))
               for layer in (0, n_layers - 1))
    return {"config": f"{n_tok} tokens x {n_layers} layers, one file ({file_bytes / 1e6:.1f} MB)",
            "timing": "wall clock around the host-synchronous calls (includes file IO)",
            "save_s": t1 - t0, "load_s": t2 - t1, "save_gbs": page_bytes / (t1 - t0) / GB,
            "load_gbs": page_bytes / (t2 - t1) / GB, "loaded_rows_equal": bool(same)}


# ---------------------------------------------------------------------------
# config 5: prefix cache -- copy-on-write branches, LRU eviction, compaction
# ---------------------------------------------------------------------------

def bench_prefix(args, dist: Dist, dev, peak, tail: int = 37, n_branch: int | None = None) -> dict:
    """Per GPU: a pool of 2^20 pages (1 layer) filled to 90% by released
    resident sequences (lengths U[1024, 32768], seeded), a shared prefix of
    8192 + tail tokens in the radix store, 512 branches that match it,
    copy-on-write its partial last page and append 2048 tokens each; then LRU
    eviction of 30% of the used pages and compaction (page moves + device
    page-table remap).  Host planning is timed with a wall clock; the device
    work of each phase with CUDA events on the pool's stream -- for the
    copy-on-write copies and the compaction moves by replaying the same page
    moves (their sources are unchanged free or shared pages, and the remap is
    idempotent), so no host planning time lands between the events.
    Parity: every branch's rows are gathered before the compaction and again
    through the remapped device tables after it (equal bit for bit), and the
    first and last branch's rows equal the oracle's append + gather of the
    prefix rows followed by the branch's own."""
    import oracle
    import rsllm_b200 as rk
    from rsllm_b200 import synth
    from rsllm_b200.prefix_pool import PrefixKvPool

    n_pages = 1 << 14 if args.small else 1 << 20
    n_branch = n_branch or (16 if args.small else 512)
    new_tok = 2048
    prefix_len = 8192 + tail
    stream = torch.cuda.Stream(device=dev)
    t0 = time.perf_counter()
    pool = PrefixKvPool(n_pages, 1, device=dev.index)
    pool.kv.storage.random_(0, 256)  # resident pages hold arbitrary bytes
    rng = np.random.default_rng(6 + 7919 * dist.rank)
    residents = []
    target = int(0.9 * n_pages)
    live = 0
    while live < target:
        s = pool.create_sequence()
        n = min(int(rng.integers(1024, 32769)), (target - live) * 64)
        pool.reserve([s], [n], stream=stream)
        live += (n + 63) // 64
        residents.append(s)
    for s in residents:
        pool.release(s)
    owner = pool.create_sequence()
    slots = pool.reserve([owner], [prefix_len], stream=stream)
    with torch.cuda.stream(stream):
        prefix_rows = synth.kv_rows(prefix_len, seed=70 + dist.rank, device=dev)
        pool.kv.append_layer(0, prefix_rows, torch.from_numpy(slots).to(dev))
    prefix_tokens = np.arange(prefix_len, dtype=np.int32)
    pool.insert_prefix(prefix_tokens, owner)
    pool.free(owner)
    branch_rows = synth.kv_rows(n_branch * new_tok, seed=80 + dist.rank, device=dev)
    stream.synchronize()
    setup_s = time.perf_counter() - t0

    def ev_pair():
        return torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)

    # (A) branches: radix match and batched reserve with copy-on-write (host
    # plan; the copies are enqueued), the copies timed by a replay, then 2048
    # rows appended per branch
    dist.barrier()
    h0 = time.perf_counter()
    branches = []
    for _ in range(n_branch):
        m, b = pool.match_prefix(prefix_tokens)
        assert m == prefix_len
        branches.append(b)
    shared_page = int(pool.page_table(branches[0])[-1])
    slots = pool.reserve(branches, [new_tok] * n_branch, stream=stream)
    h1 = time.perf_counter()
    d_slots = torch.from_numpy(slots).to(dev)
    stream.synchronize()
    cow_ms = None
    if tail:
        src = torch.full((n_branch,), shared_page, dtype=torch.int32, device=dev)
        dst = torch.tensor([int(pool.page_table(x)[prefix_len // 64]) for x in branches], dtype=torch.int32,
                           device=dev)
        a, b = ev_pair()
        a.record(stream)
        pool.kv.copy_pages(src, dst, stream=stream)
        b.record(stream)
        stream.synchronize()
        cow_ms = a.elapsed_time(b)
    a, b = ev_pair()
    a.record(stream)
    with torch.cuda.stream(stream):
        pool.kv.append_layer(0, branch_rows, d_slots)
    b.record(stream)
    stream.synchronize()
    append_ms = a.elapsed_time(b)
    pool.kv.check("prefix append", stream)

    # (B) LRU eviction of 30% of the used pages, then compaction with the
    # branches' device page table remapped in place
    tabs = [pool.page_table(x) for x in branches]
    stride = max(len(t) for t in tabs)
    pt = np.full((n_branch, stride), -1, np.int32)
    for i, t in enumerate(tabs):
        pt[i, :len(t)] = t
    d_pt = torch.from_numpy(pt).to(dev)
    L = prefix_len + new_tok
    cu = torch.arange(0, (n_branch + 1) * L, L, dtype=torch.int32, device=dev)
    pre = pool.kv.rows(0, d_pt, cu, L, stream=stream, total=n_branch * L)
    pool.kv.check("prefix gather", stream)
    ok_oracle = True
    for i in sorted({0, n_branch - 1}):
        rows = np.concatenate([u16(prefix_rows), u16(branch_rows[i * new_tok:(i + 1) * new_tok])])
        ref, rp, rpt = oracle_sequence_pool(rows)
        want, st = oracle.gather_rows(ref, rp, 1, 0, rpt, np.array([0, L], np.int32), n_threads=oracle.threads())
        ok_oracle = ok_oracle and st == 0 and np.array_equal(u16(pre[i * L:(i + 1) * L]), want)
    used = pool.stats()["live_pages"]
    stream.synchronize()
    dist.barrier()
    h2 = time.perf_counter()
    freed = pool.evict(int(0.3 * used))
    h3 = time.perf_counter()
    moved = pool.compact(device_tables=d_pt, stream=stream)
    h4 = time.perf_counter()
    stream.synchronize()
    assert pool.device_status() == 0
    remap = pool.last_remap()
    movers = np.nonzero(remap != np.arange(n_pages, dtype=np.int32))[0].astype(np.int32)
    d_src = torch.from_numpy(movers).to(dev)
    d_dst = torch.from_numpy(remap[movers]).to(dev)
    d_remap = torch.from_numpy(remap).to(dev)
    stream.synchronize()
    a, b = ev_pair()
    c = torch.cuda.Event(enable_timing=True)
    a.record(stream)
    pool.kv.copy_pages(d_src, d_dst, stream=stream)
    c.record(stream)
    rk.remap_pages(d_pt, d_remap, stream=stream)
    b.record(stream)
    stream.synchronize()
    compact_copy_ms, compact_ms = a.elapsed_time(c), a.elapsed_time(b)
    st = pool.stats()
    ok_tables = all(np.array_equal(pool.page_table(x), d_pt[i, :len(tabs[i])].cpu().numpy())
                    for i, x in enumerate(branches))
    post = pool.kv.rows(0, d_pt, cu, L, stream=stream, total=n_branch * L)
    pool.kv.check("prefix gather after compaction", stream)
    ok_same = bool(torch.equal(pre, post))
    del pre, post
    moved_bytes = 2 * moved * rk.PAGE_BYTES
    res = {
        "config": f"c5: pool 2^{int(np.log2(n_pages))} pages x 1 layer at 90% (released residents), prefix "
                  f"{prefix_len} tokens, {n_branch} branches x {new_tok} tokens, evict 30% of used, compact",
        "setup_s": setup_s,
        "host_match_reserve_ms": (h1 - h0) * 1e3, "cow_copies": n_branch if tail else 0,
        "device_cow_ms": cow_ms, "device_append_ms": append_ms,
        "append_gbs": n_branch * new_tok * APPEND_ROW_BYTES / (append_ms * 1e-3) / GB,
        "pages_used_before_evict": used, "pages_freed": freed, "host_evict_ms": (h3 - h2) * 1e3,
        "pages_moved": moved, "host_compact_ms": (h4 - h3) * 1e3, "device_compact_ms": compact_ms,
        "device_compact_copy_ms": compact_copy_ms,
        "compact_gbs": moved_bytes / (compact_copy_ms * 1e-3) / GB if moved else None,
        "compact_frac_of_hbm_peak": moved_bytes / (compact_copy_ms * 1e-3) / GB / peak if moved else None,
        "high_water_after": st["high_water"], "live_after": st["live_pages"],
        "device_tables_match_host": ok_tables,
        "rows_equal_after_compaction": ok_same,
        "branch_rows_match_oracle": ok_oracle,
        "parity": dist.all_true(ok_tables and ok_same and ok_oracle),
        "parity_sample": f"all {n_branch} branches x {L} rows equal before and after compaction; branches first + "
                         "last vs the oracle; device tables vs the host allocator",
    }
    pool.close()
    del pool, branch_rows, d_pt
    torch.cuda.empty_cache()
    return res


# ---------------------------------------------------------------------------
# reference arm: the CPU restatement of rsLLM's path on the host cores
# ---------------------------------------------------------------------------

METRIC = "KV append GB/s (config 2 decode append: FP8 quantize-on-append into a paged pool)"


def run_reference(args, dist: Dist) -> None:
    if dist.rank != 0:
        return
    import oracle

    threads = oracle.threads()
    W, K = args.warmup, args.steps
    wl = AppendWorkload(W + K, seed=3, dev=None)
    rows_cache = {}

    def rows(j):
        from rsllm_b200 import synth

        if j not in rows_cache:
            n = N_LAYERS * N_SEQ_APPEND
            rows_cache.clear()
            rows_cache[j] = synth.kv_rows(n, seed=3 * 1000 + j).view(torch.int16).numpy().view(np.uint16).reshape(
                N_LAYERS, N_SEQ_APPEND, 576)
        return rows_cache[j]

    pool = oracle.new_pool(wl.n_pages, N_LAYERS)
    for j in range(W):
        oracle.append_rows(pool, wl.n_pages, N_LAYERS, 0, rows(j), wl.slots_np[j], n_threads=threads)
    t = 0.0
    for j in range(W, W + K):
        r = rows(j)
        t0 = time.perf_counter()
        st = oracle.append_rows(pool, wl.n_pages, N_LAYERS, 0, r, wl.slots_np[j], n_threads=threads)
        t += time.perf_counter() - t0
        assert st == 0
    value = wl.bytes_per_step() * K / t / GB
    line = {
        "metric": METRIC,
        "value": value, "unit": "GB/s", "impl": "reference", "n_gpus": args.gpus, "steps": K, "warmup": W,
        "ms_per_step": t / K * 1e3, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "u8", "data": "synthetic (seeded N(0,1) bf16 rows, 1% x20 outliers; seeded page tables)",
        "config": {"workload": "c2-decode-append", "sequences": N_SEQ_APPEND, "layers": N_LAYERS,
                   "page_tokens": 64, "row": "512 latent fp8 + 64 rope bf16"},
        "tokens_per_s": N_SEQ_APPEND * K / t,
        "cpu_baseline": {"value": value, "unit": "GB/s", "cores": threads, "kind": "port",
                         "sample": f"{K} full decode steps of config 2 ({K * N_LAYERS * N_SEQ_APPEND} rows)"},
        "e2e": {"value": value, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "rsLLM is Rust (no cargo/rustc here); this arm times the C restatement of its CPU path "
                "(oracle/rkv_oracle.c: binary-search snap per lane, as dsv4_quant.rs) on all host threads",
    }
    print(json.dumps(line), flush=True)


def _r(x, nd: int = 3):
    """A number rounded to nd significant digits (None passes through)."""
    if x is None or isinstance(x, bool):
        return x
    return float(f"{x:.{nd}g}")


def summary(app: dict, phases: dict, split: dict | None) -> dict:
    """Compact per-phase figures (GB/s per GPU, fraction of the measured HBM
    peak, kernel ms per layer, parity), printed last in the line."""
    out = {"append_c2": {"gbs": _r(app["gbs_per_gpu"]), "frac": _r(app["frac"]), "us_step": _r(app["ms_per_step"] * 1e3),
                         "parity": app["parity"]}}
    if app.get("copy_floor_ms_per_step") is not None:
        out["append_c2"]["floor_us_step"] = _r(app["copy_floor_ms_per_step"] * 1e3)
        out["append_c2"]["of_floor"] = _r(app["append_speed_of_copy_floor"])
    keys = {"gather": "gather_c3", "topk": "topk_c4", "sparse_gather": "sparse_c4", "mla_decode_dense": "mla_c3",
            "mla_decode_sparse": "mla_c4", "compress_decode": "cmp_dec", "compress_prefill": "cmp_pre",
            "indexer_score_topk": "idx_c4"}
    for name, short in keys.items():
        p = phases.get(name)
        if not isinstance(p, dict) or "skipped" in p:
            continue
        d = {"gbs": _r(p.get("gbs_per_gpu")), "frac": _r(p.get("roofline_frac", p.get("frac_of_hbm_peak")))}
        ms = p.get("kernel_ms_per_layer", p.get("ms_per_layer", p.get("ms_per_layer_ungraphed")))
        if ms is not None:
            d["ms_l"] = _r(ms)
        if "parity" in p:
            d["parity"] = p["parity"]
        out[short] = d
    p = phases.get("append_f32")
    if isinstance(p, dict):
        out["append_f32_c2"] = {"gbs": _r(p.get("gbs_per_gpu")), "frac": _r(p.get("frac_of_hbm_peak")),
                                "us_step": _r(p["ms_per_step"] * 1e3), "parity": p.get("parity")}
    for name, short in (("prefix_cow_evict_compact", "prefix_c5"), ("prefix_cow_evict_compact_aligned", "prefix_c5a")):
        p = phases.get(name)
        if isinstance(p, dict):
            out[short] = {"compact_gbs": _r(p.get("compact_gbs")), "frac": _r(p.get("compact_frac_of_hbm_peak")),
                          "append_gbs": _r(p.get("append_gbs")), "parity": p.get("parity")}
    if split:
        out["split"] = {k: {"agg_gbs": _r(v.get("aggregate_gbs")), "parity": v.get("parity")}
                        for k, v in split.items() if isinstance(v, dict)}
    return out


def bench_split(args, dist: Dist, dev, peak) -> dict:
    """The configurations split over the ranks, as the multi-GPU plan states
    them (strong scaling): config 2's 256 sequences, config 3's 64 and
    config 4's 32 sequences and config 5's 512 branches, each divided evenly;
    aggregate GB/s = all ranks' algorithmic bytes / the slowest rank's time."""
    G = dist.world
    out = {}
    a = bench_append(args, dist, dev, peak, n_seq=max(1, N_SEQ_APPEND // G), e2e=False)
    out["append_c2"] = {"sequences_per_gpu": a["wl"].n_seq, "ms_per_step": a["ms_per_step"],
                        "per_rank_ms_per_step": a["per_rank_ms_per_step"],
                        "aggregate_gbs": G * a["step_bytes"] / (a["ms_per_step"] * 1e-3) / GB,
                        "parity": a["parity"]}
    del a
    torch.cuda.empty_cache()
    wanted = [] if args.phases == "none" else args.phases.split(",")
    if "gather" in wanted:
        g, _ = bench_gather(args, dist, dev, peak, n_seq=max(1, 64 // G), mla=False)
        if "skipped" not in g:
            out["gather_c3"] = {"sequences_per_gpu": max(1, 64 // G), "ms_per_step": g["ms_per_step"],
                                "per_rank_ms_per_step": g["per_rank_ms_per_step"],
                                "aggregate_gbs": G * g["step_bytes"] / (g["ms_per_step"] * 1e-3) / GB,
                                "parity": g["parity"]}
    if "sparse" in wanted:
        sp = bench_sparse(args, dist, dev, peak, n_seq=max(1, 32 // G), mla=False)
        if "skipped" not in sp:
            for name, short in (("topk", "topk_c4"), ("sparse_gather", "sparse_c4")):
                p = sp[name]
                out[short] = {"sequences_per_gpu": max(1, 32 // G), "ms_per_step": p["ms_per_step"],
                              "per_rank_ms_per_step": p["per_rank_ms_per_step"],
                              "aggregate_gbs": G * p["step_bytes"] / (p["ms_per_step"] * 1e-3) / GB,
                              "parity": p["parity"]}
    if "prefix" in wanted:
        p = bench_prefix(args, dist, dev, peak, n_branch=max(1, 512 // G))
        out["prefix_c5"] = {"branches_per_gpu": max(1, 512 // G), "pages_moved": p["pages_moved"],
                            "device_compact_ms": p["device_compact_ms"],
                            "aggregate_gbs": dist.world * p["compact_gbs"] if p["compact_gbs"] else None,
                            "parity": p["parity"]}
    return out


# ---------------------------------------------------------------------------

def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--phases", default="gather,sparse,prefix,kvc,compress,indexer,f32",
                    help="extra configs to measure (comma list of gather,sparse,prefix,kvc,compress,indexer,f32 "
                         "or 'none')")
    ap.add_argument("--phase-steps", type=int, default=3)
    ap.add_argument("--phase-warmup", type=int, default=1)
    ap.add_argument("--cpu-budget", type=float, default=10.0, help="seconds of CPU baseline sampling")
    ap.add_argument("--only", choices=["all", "append", "gather", "sparse", "prefix", "kvc", "compress", "indexer",
                                       "split", "topk", "f32"],
                    default="all",
                    help="run one workload alone (profiling)")
    ap.add_argument("--mla-splits", type=int, default=9,
                    help="page-range splits per query for the dense MLA decode phase")
    ap.add_argument("--small", action="store_true",
                    help="profiling sizes for the phases: 8 seqs / 1 layer (gather), 4 seqs / 1 layer (sparse)")
    ap.add_argument("--no-split", action="store_true", help="skip the strong-split phases at N > 1")
    args = ap.parse_args()
    if args.warmup < 3 and args.impl == "ours":
        ap.error("--warmup must be >= 3")

    dist = Dist()
    if args.impl == "reference":
        run_reference(args, dist)
        dist.close()
        return
    import oracle  # noqa: F401  (cpu_baseline leg and parity checks)
    import rsllm_b200 as rk  # noqa: F401

    dev = torch.device("cuda", dist.local if dist.world > 1 else torch.cuda.current_device())
    torch.cuda.set_device(dev)
    peak, peak_kind = peaks()
    clocks = ClockSampler(dev)
    t_start = time.time()

    if args.only != "all":
        if args.only == "append":
            res = bench_append(args, dist, dev, peak)
            res = {k: v for k, v in res.items() if k not in ("pool", "wl")}
        elif args.only == "gather":
            g, m = bench_gather(args, dist, dev, peak)
            res = {"gather": g, "mla_decode_dense": m}
        elif args.only == "prefix":
            res = {"prefix_cow_evict_compact": bench_prefix(args, dist, dev, peak),
                   "prefix_cow_evict_compact_aligned": bench_prefix(args, dist, dev, peak, tail=0)}
        elif args.only == "kvc":
            res = bench_kvc(args, dist, dev)
        elif args.only == "compress":
            res = bench_compress(args, dist, dev, peak)
        elif args.only == "indexer":
            res = bench_indexer(args, dist, dev, peak)
        elif args.only == "split":
            res = bench_split(args, dist, dev, peak)
        elif args.only == "topk":
            res = bench_topk_only(args, dist, dev, peak)
        elif args.only == "f32":
            res = bench_append_f32(args, dist, dev, peak)
        else:
            res = bench_sparse(args, dist, dev, peak)
        clocks.stop()
        dist.close()
        if dist.rank == 0:
            print(json.dumps({"only": args.only, "small": args.small, **res}), flush=True)
        return

    app = bench_append(args, dist, dev, peak)
    app["frac"] = app["gbs_per_gpu"] / peak
    phases = {}
    wanted = [] if args.phases == "none" else args.phases.split(",")
    if "gather" in wanted:
        phases["gather"], phases["mla_decode_dense"] = bench_gather(args, dist, dev, peak)
    if "sparse" in wanted:
        phases.update(bench_sparse(args, dist, dev, peak))
    if "prefix" in wanted:
        phases["prefix_cow_evict_compact"] = bench_prefix(args, dist, dev, peak)
        # the literal config: a page-aligned 8192-token prefix, so copy-on-write has nothing to copy
        phases["prefix_cow_evict_compact_aligned"] = bench_prefix(args, dist, dev, peak, tail=0)
    if "kvc" in wanted:
        phases["kvc_save_load"] = bench_kvc(args, dist, dev)
    if "compress" in wanted:
        phases.update(bench_compress(args, dist, dev, peak))
    if "indexer" in wanted:
        phases["indexer_score_topk"] = bench_indexer(args, dist, dev, peak)
    if "f32" in wanted:
        phases["append_f32"] = bench_append_f32(args, dist, dev, peak)
    split = bench_split(args, dist, dev, peak) if dist.world > 1 and not args.no_split else None
    clk = clocks.stop()

    K, W = args.steps, args.warmup
    line = None
    if dist.rank == 0:
        cpu = cpu_append_sample(app["wl"], W, args.cpu_budget, threads=__import__("oracle").threads())
        # the reference calls its quantiser single-threaded: the same port on one core, a shorter
        # sample; it and the per-phase samples are taken at N = 1 only
        cpu1 = cpu_append_sample(app["wl"], W, min(args.cpu_budget, 5.0), threads=1) if dist.world == 1 else None
        if dist.world == 1 and any(k in phases for k in ("gather", "topk", "sparse_gather",
                                                         "prefix_cow_evict_compact")):
            cpu_ph = cpu_phase_samples(__import__("oracle").threads())
            for name, key in (("gather", "gather"), ("topk", "topk"), ("sparse_gather", "sparse_gather"),
                              ("prefix_cow_evict_compact", "page_moves"),
                              ("prefix_cow_evict_compact_aligned", "page_moves")):
                if name in phases and isinstance(phases[name], dict):
                    phases[name]["cpu_baseline"] = cpu_ph[key]
        value = app["gbs_per_gpu"] * dist.world
        traffic = NCU_TRAFFIC_PER_ROW["append"]
        rows_per_launch = N_LAYERS * N_SEQ_APPEND
        e2e = app["e2e"]
        line = {
            "metric": METRIC,
            "value": value, "unit": "GB/s", "n_gpus": dist.world, "steps": K, "warmup": W,
            "ms_per_step": app["ms_per_step"], "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "u8", "data": "synthetic (seeded N(0,1) bf16 rows, 1% x20 outliers; seeded page tables)",
            "config": {"workload": "c2-decode-append", "sequences_per_gpu": N_SEQ_APPEND, "layers": N_LAYERS,
                       "seq_len": "U[1024,32768]", "page_tokens": 64, "row": "512 latent fp8 + 64 rope bf16",
                       "parallelism": f"request-sharded x{dist.world}, no collective",
                       "l2": "inputs larger than L2 (fresh rows every step, 1.9 GB total) + L2 flush before timing",
                       "launch": "K steps captured in one CUDA graph (uploaded by an untimed replay); a sleep "
                                 "kernel queued before the start event covers the host's graph launch; appends "
                                 "with RKV_APPEND_INPUTS_READY (each step's rows exist before the previous step's "
                                 "append, so its reads overlap that launch's drain; wait_first_* beside it)"},
            "tokens_per_s": app["tokens_per_s_per_gpu"] * dist.world,
            "rows_per_s": app["tokens_per_s_per_gpu"] * dist.world * N_LAYERS,
            "frac_of_hbm_peak_per_gpu": app["frac"],
            "per_rank_ms_per_step": app["per_rank_ms_per_step"],
            "repeats_max_over_ranks_ms_per_step": app["repeats_max_over_ranks_ms_per_step"],
            "repeats_median_rank_ms_per_step": app["repeats_median_rank_ms_per_step"],
            "wait_first_ms_per_step": app["wait_first_ms_per_step"],
            "wait_first_gbs_per_gpu": app["wait_first_gbs_per_gpu"],
            "copy_floor": {"kernel": "copy_floor_kernel (rkv_copy_floor_bf16: the append's bytes, same launch, "
                                     "no codec)",
                           "ms_per_step": app.get("copy_floor_ms_per_step"),
                           "gbs_per_gpu": app.get("copy_floor_gbs_per_gpu"),
                           "frac_of_hbm_peak": None if app.get("copy_floor_gbs_per_gpu") is None
                           else app["copy_floor_gbs_per_gpu"] / peak,
                           "append_speed_of_copy_floor": app.get("append_speed_of_copy_floor")},
            "parity": app["parity"],
            "roofline": {"bound": "hbm", "achieved": app["gbs_per_gpu"], "peak": peak, "unit": "GB/s",
                         "frac": app["frac"], "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)"
                         if peak_kind == "measured" else "fallback 6650 GB/s",
                         "kernel": "append_quant_early_kernel", "algorithmic_bytes_per_launch": app["step_bytes"],
                         "traffic": None if traffic is None else traffic * rows_per_launch},
            "cpu_baseline": cpu,
            "cpu_baseline_single_thread": cpu1,
            "e2e": {k: v for k, v in e2e.items() if k in ("value", "unit", "h2d_bytes_per_step",
                                                           "d2h_bytes_per_step")},
            "e2e_detail": e2e,
            "gpu_launches": K,
            "phases": phases,
            "split": split,
            "clocks": clk,
            "wall_s": time.time() - t_start,
        }
        line["summary"] = summary(app, phases, split)
    del app
    dist.close()
    if line is not None:
        print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
