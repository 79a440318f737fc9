"""The f32-row append rule, on the CPU.

* The product library's scale-exponent threshold table (built from the host's
  log2f) decides ceil(log2f(y)) correctly for every f32 y = amax / 448 that an
  amax in [1e-4, f32 max] produces -- checked against the oracle's direct
  evaluation of dsv4_quant.rs:346-355 for all 2^23 mantissas of each binade.
* The oracle's stored form of an f32 row (codes, power-of-two scales, bf16
  RoPE) decodes to the reference's own f32 round trip
  (fp8_kv_quantize_row_inplace, dsv4_quant.rs:316-362) rounded to bf16, on rows
  whose block maxima sit at the threshold of every binade.
"""
import numpy as np
import pytest

from rsllm_b200 import _abi

EB_LO = int((np.float32(1e-4) / np.float32(448.0)).view(np.uint32) >> 23)
EB_HI = int((np.finfo(np.float32).max / np.float32(448.0)).astype(np.float32).view(np.uint32) >> 23)


def product_table() -> np.ndarray:
    t = np.zeros(256, np.uint32)
    _abi.load().rkv_scale_threshold_table(t.ctypes.data)
    return t


def test_threshold_table_every_y(orc):
    t = product_table()
    assert (EB_LO, EB_HI) == (104, 246)
    bad, first = orc.threshold_mismatches(t, EB_LO, EB_HI)
    assert bad == 0, f"{bad} mismatches, first at y bits 0x{first:08x}"
    # The table is not the integer rule (exponent + 1 for any non-zero
    # mantissa): log2f rounds down to E just above 2^E in most binades.
    assert np.count_nonzero(t[EB_LO:EB_HI + 1] > 1) > 100


def threshold_amaxes(t: np.ndarray) -> np.ndarray:
    """Block maxima around 448 * 2^E and around the threshold of every binade."""
    out = []
    for eb in range(EB_LO, EB_HI + 1):
        for m in {0, 1, int(t[eb]) - 1, int(t[eb]), int(t[eb]) + 1, 0x7FFFFF}:
            if not 0 <= m <= 0x7FFFFF:
                continue
            y = np.array([(eb << 23) | m], np.uint32).view(np.float32)[0]
            with np.errstate(over="ignore"):
                a = int(np.array([y * np.float32(448.0)], np.float32).view(np.uint32)[0])
            v = np.array([a + k for k in range(-2, 3)], np.uint32).view(np.float32)
            out.extend(v[np.isfinite(v) & (v > 0)].tolist())
    return np.unique(np.array(out, np.float32))


def f32_rows_at_thresholds(t: np.ndarray, seed: int = 0) -> np.ndarray:
    """f32 rows whose latent blocks have the maxima of threshold_amaxes(),
    with random lanes below the maximum, random RoPE lanes."""
    rng = np.random.default_rng(seed)
    amax = threshold_amaxes(t)
    n_blocks = amax.size
    n_rows = (n_blocks + 7) // 8
    amax = np.concatenate([amax, np.full(n_rows * 8 - n_blocks, np.float32(1.0))])
    lat = (rng.uniform(-1, 1, (n_rows * 8, 64)) * amax[:, None].astype(np.float64)).astype(np.float32)
    lat = np.clip(lat, -amax[:, None], amax[:, None])
    lat[np.arange(n_rows * 8), rng.integers(0, 64, n_rows * 8)] = amax * np.where(rng.random(n_rows * 8) < 0.5, -1, 1)
    rows = np.zeros((n_rows, 576), np.float32)
    rows[:, :512] = lat.reshape(n_rows, 512)
    rows[:, 512:] = rng.standard_normal((n_rows, 64)).astype(np.float32) * 3
    return rows


def f32_to_bf16(x: np.ndarray) -> np.ndarray:
    b = x.astype(np.float32).view(np.uint32)
    nan = (b & 0x7FFFFFFF) > 0x7F800000
    r = ((b + 0x7FFF + ((b >> 16) & 1)) >> 16).astype(np.uint16)
    return np.where(nan, ((b >> 16) | 0x40).astype(np.uint16), r)


def reference_roundtrip_f32(orc, rows: np.ndarray) -> np.ndarray:
    """rsLLM's own path on f32 rows: fp8_kv_quantize_row_inplace(576, 64),
    then every lane rounded to bf16 (RoPE lanes are untouched in f32)."""
    out = np.empty(rows.shape, np.uint16)
    for i in range(rows.shape[0]):
        x = rows[i].copy()
        assert orc.quantize_row_inplace(x, 576, 64) == orc.OK
        out[i] = f32_to_bf16(x)
    return out


def test_f32_stored_form_matches_reference_roundtrip(orc):
    rows = f32_rows_at_thresholds(product_table())
    rng = np.random.default_rng(3)
    extra = rng.standard_normal((32, 576)).astype(np.float32)
    extra[0, :512] = -0.0
    extra[1, :512] = np.float32(1e-45)          # subnormal lanes, floored amax
    extra[2, :512] = -np.float32(1e-45)
    extra[3, :512] = np.finfo(np.float32).max   # e = 120; the product overflows to inf
    extra[4, :512] = np.float32(1e-4)
    extra[5, 512:] = np.nan                     # NaN RoPE lanes: stored as a quiet NaN
    rows = np.concatenate([rows, extra])
    codes, scales, rope, st = orc.quantize_rows_f32(rows)
    assert np.all(st == 0)
    assert np.all(np.log2(scales) == np.round(np.log2(scales)))
    dec = orc.dequant_rows_bf16(codes, scales, rope)
    assert np.array_equal(dec, reference_roundtrip_f32(orc, rows))
    n = rows.shape[0] - 32
    assert np.all(codes[n + 0] == 0) and np.all(codes[n + 2] == 0x80)
    assert dec[n + 3, 0] == 0x7F80


def test_f32_non_finite_rejects_row(orc):
    rows = np.zeros((3, 576), np.float32)
    rows[0, 7] = np.nan
    rows[1, 300] = -np.inf
    rows[2, 520] = np.inf
    _, _, rope, st = orc.quantize_rows_f32(rows)
    assert st.tolist() == [orc.NON_FINITE_INPUT, orc.NON_FINITE_INPUT, orc.OK]
    assert rope[2, 8] == 0x7F80


@pytest.mark.parametrize("eb", [EB_LO, 120, 127, 200, EB_HI])
def test_exponent_at_threshold(orc, eb):
    """The scale the oracle picks for amax = 448 * y flips exactly at the
    table's mantissa (where that amax reproduces y exactly)."""
    t = product_table()
    m = int(t[eb])
    assert 1 <= m <= 0x7FFFFF
    L = orc.lib()
    for mm, bump in ((m - 1, 0), (m, 1)):
        y = np.array([(eb << 23) | mm], np.uint32).view(np.float32)[0]
        a = np.float32(y * np.float32(448.0))
        if np.float32(a / np.float32(448.0)) != y or a < np.float32(1e-4):
            continue
        assert L.rkvo_scale_exponent(float(a)) == eb - 127 + bump
