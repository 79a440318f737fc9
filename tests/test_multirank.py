"""The multi-GPU path on the CPU: two gloo ranks (one process each, as
torchrun launches them) run the per-rank setup of the benchmark -- each rank
owns its own pool and its own seeded sequences, no collective touches the
data -- and the max-over-ranks timing reduction; the reference arm prints
from rank 0 only."""
import json
import os
import socket
import subprocess
import sys
import textwrap
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent.parent

CHILD = textwrap.dedent("""
    import json, sys
    sys.path.insert(0, {root!r})
    import numpy as np
    import bench
    d = bench.Dist(backend="gloo")
    wl = bench.AppendWorkload(12, seed=3 + 7919 * d.rank, dev=None)
    slots = wl.slots_np
    # every slot inside this rank's pool, no slot written twice, a new page
    # whenever a sequence crosses a 64-token boundary
    ok = bool((slots >= 0).all() and (slots < wl.n_pages * 64).all() and
              len(np.unique(slots)) == slots.size)
    t = d.max(1.0 + d.rank)  # per-rank time -> job time is the slowest rank
    every = d.all(10.0 + d.rank)  # every rank's time, in rank order
    both = d.all_true(True)
    one_fails = d.all_true(d.rank == 0)
    unchecked = d.all_true(None if d.rank else True)
    # the strong split of config 2 over the ranks: disjoint per-rank workloads
    half = bench.AppendWorkload(3, seed=3 + 7919 * d.rank, dev=None, n_seq=bench.N_SEQ_APPEND // d.world)
    print(json.dumps({{"rank": d.rank, "ok": ok, "max": t, "first": slots[0, :4].tolist(),
                       "pages": wl.n_pages, "every": every, "both": both, "one_fails": one_fails,
                       "unchecked": unchecked, "half_seqs": half.n_seq,
                       "half_bytes": half.bytes_per_step()}}), flush=True)
    d.close()
""")


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def launch(code: str, world: int = 2, extra_args=()) -> list[str]:
    port = free_port()
    procs = []
    for r in range(world):
        env = dict(os.environ, RANK=str(r), LOCAL_RANK=str(r), WORLD_SIZE=str(world), MASTER_ADDR="127.0.0.1",
                   MASTER_PORT=str(port), CUDA_VISIBLE_DEVICES="")
        procs.append(subprocess.Popen([sys.executable, "-c", code, *extra_args], env=env, stdout=subprocess.PIPE,
                                      stderr=subprocess.PIPE, text=True, cwd=str(ROOT)))
    outs = []
    for p in procs:
        out, err = p.communicate(timeout=300)
        assert p.returncode == 0, err[-2000:]
        outs.append(out)
    return outs


def test_two_gloo_ranks_own_their_work():
    outs = launch(CHILD.format(root=str(ROOT)))
    res = [json.loads(o.strip().splitlines()[-1]) for o in outs]
    assert [r["rank"] for r in res] == [0, 1]
    assert all(r["ok"] for r in res)
    assert all(r["max"] == 2.0 for r in res)  # max over ranks reaches every rank
    assert res[0]["first"] != res[1]["first"]  # each rank its own seeded sequences
    assert all(r["every"] == [10.0, 11.0] for r in res)
    assert all(r["both"] is True and r["one_fails"] is False and r["unchecked"] is None for r in res)
    assert all(r["half_seqs"] == 128 for r in res)
    assert res[0]["half_bytes"] * 2 == bench_step_bytes(256)


def bench_step_bytes(n_seq: int) -> int:
    return 61 * n_seq * (1152 + 672) + n_seq * 4


def test_reference_arm_prints_from_rank_zero_only():
    code = "import sys, runpy; sys.argv=['bench.py','--impl','reference','--gpus','2','--steps','1','--warmup','0']; " \
           "runpy.run_path('bench.py', run_name='__main__')"
    outs = launch(code)
    lines = [[ln for ln in o.splitlines() if ln.startswith("{")] for o in outs]
    assert len(lines[0]) == 1 and len(lines[1]) == 0
    line = json.loads(lines[0][0])
    assert line["impl"] == "reference" and line["value"] > 0 and line["e2e"]["h2d_bytes_per_step"] == 0
    assert line["cpu_baseline"]["kind"] == "port"
    # the GPU arm prints the same metric, unit and direction (the driver
    # divides the two arms' values only when they agree)
    sys.path.insert(0, str(ROOT))
    import bench

    assert line["metric"] == bench.METRIC and line["unit"] == "GB/s" and line["higher_is_better"] is True
    src = (ROOT / "bench.py").read_text()
    assert src.count('"metric": METRIC') == 2


def test_summary_fits_the_kept_tail():
    """The compact summary printed last in the line stays well inside the
    ~1.5 KB of stdout tail a driver keeps, with every phase present."""
    sys.path.insert(0, str(ROOT))
    import bench

    ph = {"gbs_per_gpu": 6123.456, "frac_of_hbm_peak": 0.9345, "kernel_ms_per_layer": 0.61234, "parity": True}
    phases = {k: dict(ph) for k in ("gather", "topk", "sparse_gather", "mla_decode_dense", "mla_decode_sparse",
                                    "compress_decode", "compress_prefill", "indexer_score_topk")}
    phases["mla_decode_dense"]["roofline_frac"] = 0.321
    for k in ("prefix_cow_evict_compact", "prefix_cow_evict_compact_aligned"):
        phases[k] = {"compact_gbs": 6600.1, "compact_frac_of_hbm_peak": 1.01, "append_gbs": 4400.2, "parity": True}
    split = {k: {"aggregate_gbs": 12345.678, "parity": True} for k in ("append_c2", "gather_c3", "topk_c4",
                                                                        "sparse_c4", "prefix_c5")}
    phases["append_f32"] = {"gbs_per_gpu": 5123.456, "frac_of_hbm_peak": 0.7834, "ms_per_step": 0.0090812,
                            "parity": True}
    app = {"gbs_per_gpu": 3500.123, "frac": 0.5432, "ms_per_step": 0.0081408, "parity": True,
           "copy_floor_ms_per_step": 0.0055497, "append_speed_of_copy_floor": 0.8971}
    s = json.dumps(bench.summary(app, phases, split))
    assert len(s) < 1400, len(s)
    assert json.loads(s)["mla_c3"]["frac"] == 0.321
    assert json.loads(s)["append_f32_c2"]["parity"] is True
