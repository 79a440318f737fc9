"""The CPU oracle against rsLLM's own known-answer tests for the KV-cache path
(transcribed in tests/golden/kat_reference.json, one reference file:line per
case).  These pin the oracle before anything is compared against it."""
import json
import math
import struct
from pathlib import Path

import numpy as np
import pytest

KAT = json.loads((Path(__file__).parent / "golden" / "kat_reference.json").read_text())


def f32(bits_hex: str) -> float:
    return struct.unpack("<f", struct.pack("<I", int(bits_hex, 16)))[0]


def bits(x: float) -> int:
    return struct.unpack("<I", struct.pack("<f", x))[0]


def test_e4m3fn_value(orc):
    L = orc.lib()
    for code, val in KAT["e4m3fn_value"]["cases"]:
        assert L.rkvo_e4m3fn_value(code) == val, code


def test_e4m3fn_dequant(orc):
    L = orc.lib()
    for x, want in KAT["e4m3fn_dequant"]["cases"]:
        got = L.rkvo_e4m3fn_dequant(x)
        assert got == want, (x, got, want)


@pytest.mark.parametrize("case", KAT["quantize_row"]["cases"], ids=lambda c: c["name"])
def test_quantize_row(orc, case):
    head_dim, n_rot = case["head_dim"], case["n_rot"]
    n = case.get("len", head_dim)
    x = np.full(n, case["fill"], np.float32)
    if "tail_formula" in case:
        for i in range(n_rot, head_dim):
            x[i] = np.float32(i) * np.float32(0.123)
    for lane, v in case["set"]:
        x[lane] = np.nan if v == "nan" else v
    before = x.copy()
    rc = orc.quantize_row_inplace(x, head_dim, n_rot)
    exp = case["expect"]
    want = {"ok": orc.OK, "shape_mismatch": orc.SHAPE_MISMATCH, "non_finite_input": orc.NON_FINITE_INPUT}[exp["status"]]
    assert rc == want
    if rc != orc.OK:
        return
    n_nope = head_dim - n_rot
    if "prefix_all" in exp:
        assert np.all(np.abs(x[:n_nope] - exp["prefix_all"]) < exp["prefix_tol"])
    if "tail_all" in exp:
        assert np.all(x[n_nope:] == exp["tail_all"])
    for lane, v, tol in exp.get("lanes", []):
        assert abs(x[lane] - v) < tol, (lane, x[lane], v)
    if exp.get("tail_unchanged"):
        assert np.array_equal(x[n_nope:], before[n_nope:])
    for lane in exp.get("nan_lanes", []):
        assert math.isnan(x[lane])


def test_byte_codec(orc):
    L = orc.lib()
    bc = KAT["byte_codec"]
    for src, code, _ in bc["encode"]:
        assert L.rkvo_f32_to_fp8_e4m3(f32(src)) == int(code, 16), (src, code)
    for code, val in bc["decode"]:
        assert bits(L.rkvo_fp8_e4m3_to_f32(int(code, 16))) == int(val, 16), code
    for code in bc["decode_nan"]:
        assert math.isnan(L.rkvo_fp8_e4m3_to_f32(int(code, 16)))
    # fp8_e4m3.rs:227-245: every code decodes and re-encodes to itself, NaN to 0x7f.
    for b in range(256):
        v = L.rkvo_fp8_e4m3_to_f32(b)
        want = int(bc["round_trip_all_codes"]["nan_reencode"], 16) if math.isnan(v) else b
        assert L.rkvo_f32_to_fp8_e4m3(v) == want, b


@pytest.mark.parametrize("case", KAT["select_top_k"]["cases"], ids=lambda c: c["name"])
@pytest.mark.parametrize("scan", [True, False], ids=["scan", "sorted"])
def test_select_top_k(orc, case, scan):
    sel = orc.select_top_k(np.array(case["scores"], np.float32), case["k"], scan=scan)
    if "expect_sorted" in case:
        assert sorted(sel.tolist()) == case["expect_sorted"]
    if "expect_len" in case:
        assert len(sel) == case["expect_len"]


def test_swa_order_restated_as_slots(orc):
    """swa.rs:203-214: a capacity-3 ring fed rows 0..4 reads back 2,3,4.  In
    the paged form a ring is a slot mapping; writing token t to slot t % 3 and
    reading slots in chronological order gives the same rows."""
    case = KAT["swa_ring"]["shift_case"]
    cap = case["cap"]
    pool = orc.new_pool(1, 1)
    rows = np.zeros((len(case["appended"]), 576), np.uint16)
    for t, seed in enumerate(case["appended"]):
        rows[t, :] = np.float32(seed).view(np.uint32) >> 16  # bf16 of the seed value
    n = len(case["appended"])
    slots = np.array([t % cap for t in range(n)], np.int32)
    for t in range(n):  # one append per token, like RawSwaRing::append
        assert orc.append_rows(pool, 1, 1, 0, rows[t:t + 1], slots[t:t + 1]) == 0
    oldest = n - cap
    order = [(oldest + i) % cap for i in range(cap)]
    pt = np.array([[0]], np.int32)
    out, st = orc.gather_rows(pool, 1, 1, 0, pt, np.array([0, cap], np.int32))
    assert st == 0
    by_slot = {s: out[s] for s in range(cap)}
    got = [np.frombuffer(np.array(by_slot[s][0], np.uint16).tobytes() + b"", np.uint16)[0] for s in order]
    want = [np.float32(v).view(np.uint32) >> 16 for v in case["rows"]]
    assert [int(g) for g in got] == [int(w) for w in want]
