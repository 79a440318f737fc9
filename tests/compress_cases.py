"""A compressor row whose RMSNorm mean needs rsLLM's in-order f64 sum.

The emission kernels sum the 576 squares as a tree (warp butterflies, then the
18 warp partials) and use that mean unless it lies within 2^11 units of the
last place of a rounding midpoint of the f32 mean, where one thread redoes the
sum in rsLLM's order (compressor.rs:292-296).  Random rows reach that band
about once in 2^16, so `midpoint_row` builds one: lane 0 is 1023.875 (square
~2^20), the next lanes add exact powers of four times 2^-32 so that the
in-order sum is exactly T, and every other lane is 2^-17, whose square (2^-34)
is below half an ulp of the running sum and vanishes in order, while the tree
adds those squares to each other first and keeps most of them.  T / 576 sits a
little below an f32 midpoint, the tree's mean a little above it: the two
round to different f32 means, so a kernel that skipped the in-order sum would
emit a different row.
"""
import numpy as np

N = 576
SMALL = np.float32(2.0 ** -17)


def kernel_tree_sum(sq: np.ndarray) -> np.float64:
    """The emission kernels' f64 tree over 576 squares (thread j holds lane
    j): per warp an xor butterfly (strides 16 .. 1), then the same butterfly
    over the 18 warp partials padded with zeros."""
    idx = np.arange(32)
    v = np.asarray(sq, np.float64).reshape(N // 32, 32).copy()
    for o in (16, 8, 4, 2, 1):
        v = v + v[:, idx ^ o]
    p = np.zeros(32)
    p[: N // 32] = v[:, 0]
    for o in (16, 8, 4, 2, 1):
        p = p + p[idx ^ o]
    return p[0]


def in_order_sum(sq: np.ndarray) -> np.float64:
    """rsLLM's sum, lane by lane (a cumulative sum is evaluated in order)."""
    return np.cumsum(np.asarray(sq, np.float64))[-1]


def mid_distance(q: np.float64) -> int:
    """Distance of the 29 bits that rounding q to f32 drops from 2^28."""
    low = int(np.array(q, np.float64).view(np.uint64)) & ((1 << 29) - 1)
    return abs(low - (1 << 28))


def midpoint_row(offset: int = 56) -> np.ndarray:
    """576 f32 lanes (see the module docstring); `offset` (units of 2^-32)
    sets how far T / 576 lies below the f32 midpoint 1820 + 2^-14."""
    big = np.float32(1023.875)
    # T = 576 * (1820 + 2^-14) - offset * 2^-32 = big^2 + rest * 2^-32
    rest = 5 * 2 ** 24 - offset
    lanes = [big]
    i = 0
    while rest:
        d = rest % 4
        lanes += [np.float32(2.0 ** (i - 16))] * d  # square 4^i * 2^-32
        rest //= 4
        i += 1
    lanes = lanes[:1] + sorted(lanes[1:], reverse=True)
    row = np.full(N, SMALL, np.float32)
    row[: len(lanes)] = lanes
    return row


def means(row: np.ndarray):
    """(in-order mean, tree mean) in f64, as rsLLM and the kernels form them."""
    sq = row.astype(np.float64) ** 2
    return in_order_sum(sq) / np.float64(N), kernel_tree_sum(sq) * np.float64(1.0 / N)


SENSITIVE_LANE = 500  # block 7, whose other lanes are all 2^-17


def normalized(row: np.ndarray, mean: np.float32) -> np.ndarray:
    """RMSNorm with unit weights and a given f32 mean (the latent lanes are all
    that matter here: no RoPE)."""
    rms = np.float32(1.0) / np.sqrt(np.float32(mean) + np.float32(1e-6), dtype=np.float32)
    return (row * rms).astype(np.float32)


def sensitive_row(quantize) -> np.ndarray:
    """midpoint_row with lane SENSITIVE_LANE set to an x a little above 2^-17
    (its square still vanishes in order) for which the FP8 code of the lane
    differs between the in-order mean and the tree's mean, so that the emitted
    bytes show which mean a kernel used.  `quantize` is the oracle's f32 row
    quantiser (rows -> (codes, scales, rope, status))."""
    base = midpoint_row()
    x = np.float32(1.04 * 2.0 ** -17)
    for _ in range(1 << 14):
        row = base.copy()
        row[SENSITIVE_LANE] = x
        qs, qt = means(row)
        ma, mb = np.float32(qs), np.float32(qt)
        if ma != mb and mid_distance(qt) <= 1 << 11:
            if (quantize(normalized(row, ma))[0] != quantize(normalized(row, mb))[0]).any():
                return row
        x = np.nextafter(x, np.float32(1.0))
    raise AssertionError("no sensitive lane value found")
