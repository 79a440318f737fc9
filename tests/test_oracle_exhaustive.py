"""Exhaustive and randomized checks of the oracle's own consistency, each
against an independent statement of the same rule:

* the reference's binary-search snap (dsv4_quant.rs:128-163) equals
  round-to-nearest-even to E4M3FN with saturation (ml_dtypes' float8_e4m3fn
  cast) for every f32 in [-448, 448];
* the scale exponent ceil(log2f(max(amax,1e-4)/448)) with glibc log2f equals
  the exact integer exponent rule for every bf16 block amax -- the rule the
  CUDA encoder uses;
* the stored form (codes + power-of-two scale) decodes to the reference's own
  f32 round trip, rounded to bf16;
* the sort-based top-k equals the reference's repeated best-scan.
"""
import ml_dtypes
import numpy as np
import pytest
import torch


def test_snap_equals_rne_saturating_all_f32(orc):
    hi = 0x43E00000  # 448.0
    chunk = 1 << 26
    for first in range(0, hi + 1, chunk):
        n = min(chunk, hi + 1 - first)
        bits = np.arange(first, first + n, dtype=np.uint32)
        want = bits.view(np.float32).astype(ml_dtypes.float8_e4m3fn).view(np.uint8)
        got = orc.e4m3fn_code_range(first, n)
        bad = np.nonzero(got != want)[0]
        assert bad.size == 0, f"snap != RNE at f32 bits 0x{first + int(bad[0]):08x}"
        # negative side: code = 0x80 | magnitude code, except -0.0 -> 0x00
        got_neg = orc.e4m3fn_code_range(0x80000000 + first, n)
        want_neg = want | np.uint8(0x80)
        if first == 0:
            want_neg[0] = 0
        bad = np.nonzero(got_neg != want_neg)[0]
        assert bad.size == 0, f"negative snap mismatch at 0x{0x80000000 + first + int(bad[0]):08x}"


def integer_exponent(amax: np.ndarray) -> np.ndarray:
    """ceil(log2(y)) of y = RN(max(amax, 1e-4) / 448) from the bits of y."""
    a = np.maximum(amax.astype(np.float32), np.float32(1e-4))
    y = (a / np.float32(448.0)).astype(np.float32)
    b = y.view(np.uint32)
    e = ((b >> 23) & 0xFF).astype(np.int64) - 127
    return e + ((b & 0x7FFFFF) != 0)


def test_scale_exponent_rule_every_bf16_amax(orc):
    L = orc.lib()
    hb = np.arange(0, 0x7F80, dtype=np.uint32)  # every finite non-negative bf16
    amax = (hb << 16).view(np.float32)
    want = integer_exponent(amax)
    got = np.array([L.rkvo_scale_exponent(float(a)) for a in amax], np.int64)
    bad = np.nonzero(got != want)[0]
    assert bad.size == 0, f"exponent rule differs at bf16 0x{int(hb[bad[0]]):04x}"


def edge_rows() -> np.ndarray:
    """bf16 rows that hit the codec's corners."""
    r = np.zeros((12, 576), np.uint16)
    r[1, :512] = 0x8000                                   # all -0.0
    r[2, :512] = 0x0001                                   # tiny subnormals
    r[3, :512] = 0x8001                                   # tiny negative subnormals
    r[4, :512] = 0x7F7F                                   # bf16 max -> rounds past f32 max -> inf
    r[5, :512] = 0xFF7F                                   # -max -> -inf
    r[6, :512] = np.arange(512, dtype=np.uint16) * 63     # spread of magnitudes (all finite)
    r[7, :512] = 0x3F80                                   # 1.0
    r[7, 0] = 0x447A                                      # 1000 in block 0
    r[8, :512] = (np.arange(512) % 2 * 0x8000 + 0x3A83).astype(np.uint16)  # +-0.001
    r[9, :512] = 0x38D1                                   # 1e-4 (amax floor)
    r[10, :512] = 0x0000
    r[10, 5] = 0x8001                                     # -tiny in a zero block -> code 0x80
    r[11, :512] = 0x7F00                                  # 1.7e38: e = 120
    r[:, 512:] = 0x7FC0                                   # NaN rope lanes pass through
    return r


def reference_roundtrip_bf16(orc, rows: np.ndarray) -> np.ndarray:
    """The reference's own path: f32 row -> fp8_kv_quantize_row_inplace(576, 64)
    -> bf16 (rope lanes untouched)."""
    out = np.zeros_like(rows)
    L = orc.lib()
    for i in range(rows.shape[0]):
        x = (rows[i].astype(np.uint32) << 16).view(np.float32).copy()
        assert orc.quantize_row_inplace(x, 576, 64) == orc.OK
        out[i] = np.array([L.rkvo_f32_to_bf16(float(v)) for v in x], np.uint16)
        out[i, 512:] = rows[i, 512:]
    return out


def test_stored_form_matches_reference_roundtrip(orc):
    from rsllm_b200 import synth

    e = 64  # edge rows follow 64 synthetic rows
    rows = np.concatenate([synth.kv_rows(e, seed=11).view(torch.int16).numpy().view(np.uint16), edge_rows()])
    codes, scales, rope, st = orc.quantize_rows_bf16(rows)
    assert np.all(st == 0)
    assert np.all(np.log2(scales) == np.round(np.log2(scales)))  # powers of two
    dec = orc.dequant_rows_bf16(codes, scales, rope)
    ref = reference_roundtrip_bf16(orc, rows)
    assert np.array_equal(dec, ref)
    # -0.0 input maps to code 0x00, a tiny negative to 0x80 (dsv4_quant.rs:129 sign rule)
    assert np.all(codes[e + 1] == 0) and codes[e + 10, 5] == 0x80 and codes[e + 10, 4] == 0
    # bf16 max rounds up past f32 max: the reference's product is +-inf
    assert dec[e + 4, 0] == 0x7F80 and dec[e + 5, 0] == 0xFF80


def test_non_finite_latent_rejects_row(orc):
    rows = np.zeros((3, 576), np.uint16)
    rows[0, 7] = 0x7FC0   # NaN in latent
    rows[1, 300] = 0xFF80  # -inf in latent
    rows[2, 520] = 0x7F80  # inf in rope: allowed
    _, _, _, st = orc.quantize_rows_bf16(rows)
    assert st.tolist() == [orc.NON_FINITE_INPUT, orc.NON_FINITE_INPUT, orc.OK]


@pytest.mark.parametrize("kind", ["normal", "ties", "specials", "small"])
def test_topk_sorted_equals_scan(orc, kind):
    rng = np.random.default_rng(7)
    for trial in range(20):
        n = int(rng.integers(1, 3000)) if kind != "small" else int(rng.integers(1, 8))
        if kind == "normal":
            s = rng.standard_normal(n).astype(np.float32)
        elif kind == "ties":
            s = rng.integers(-3, 4, n).astype(np.float32)
            s[rng.random(n) < 0.2] = -0.0
        else:
            s = rng.standard_normal(n).astype(np.float32)
            m = rng.random(n)
            s[m < 0.3] = -np.inf
            s[(m >= 0.3) & (m < 0.5)] = np.nan
            s[(m >= 0.5) & (m < 0.55)] = np.inf
            if trial % 3 == 0:
                s[:] = -np.inf
        k = int(rng.integers(0, n + 5))
        a = orc.select_top_k(s, k, scan=True)
        b = orc.select_top_k(s, k, scan=False)
        assert np.array_equal(a, b), (kind, trial, n, k)
