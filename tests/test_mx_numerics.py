"""Precision of the decode kernel's MXFP4 expert arithmetic, restated on the
CPU (no GPU needed).

The persistent decode kernel (strasgpt_b200/csrc/decode_mega.cu,
xm_store / mx_chunk_dot) multiplies MXFP4 expert rows on the tensor cores:
the e2m1 codes become f16 exactly, and the fp32 activation is held as two
f16 parts with a power-of-two scale per 32-column block,

    x * 2^s = hi + mid,  hi = f16(x * 2^s),  mid = f16(x * 2^s - hi),

s chosen so that the block's largest magnitude lies in [2^14, 2^15). A
block's products e2m1 x f16 are exact in fp32; the kernel sums them in
fp32 and scales the block sum by 2^(e - 127) * 2^-s. These tests pin the
error of that scheme against float64: the split keeps about 22 bits of
every element (down to a floor of 2^-38 of the block maximum), and a full
row dot stays within 1e-6 of the sum of |w x|, far inside the 1e-2 logits
tolerance of the parity tests.
"""
import numpy as np

E2M1 = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0,
                 -0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0], dtype=np.float64)


def split_block(x):
    """Two f16 parts and the exponent s of one 32-column block (fp32 in)."""
    x = np.asarray(x, dtype=np.float32)
    m = float(np.max(np.abs(x)))
    sh = 0
    if m > 0:
        ex = int(np.frexp(np.float32(m))[1]) - 1  # floor(log2 m)
        sh = min(max(14 - ex, -126), 126)
    xs = (x * np.float32(2.0 ** sh)).astype(np.float32)
    hi = xs.astype(np.float16)
    mid = (xs - hi.astype(np.float32)).astype(np.float16)
    return hi, mid, sh


def mx_dot(codes, scales, x):
    """Row dot as the kernel forms it: per block an fp32 sum of exact
    products (both parts), times 2^(e - 127) * 2^-s, added in fp32."""
    acc = np.float32(0.0)
    for b in range(len(scales)):
        w = E2M1[codes[b * 32:(b + 1) * 32]].astype(np.float32)
        hi, mid, sh = split_block(x[b * 32:(b + 1) * 32])
        t = np.float32(0.0)
        for part in (hi, mid):
            t = np.float32(t + np.sum(w * part.astype(np.float32), dtype=np.float32))
        f = np.float32(2.0 ** (int(scales[b]) - 127)) * np.float32(2.0 ** -sh)
        acc = np.float32(acc + t * f)
    return float(acc)


def test_split_keeps_22_bits_down_to_the_block_floor():
    rng = np.random.default_rng(7)
    for _ in range(200):
        mag = np.exp(rng.normal(0.0, 4.0, 32))  # wide dynamic range
        x = (mag * rng.choice([-1.0, 1.0], 32)).astype(np.float32)
        hi, mid, sh = split_block(x)
        back = (hi.astype(np.float64) + mid.astype(np.float64)) * 2.0 ** -sh
        m = np.max(np.abs(x.astype(np.float64)))
        bound = np.maximum(2.0 ** -22 * np.abs(x.astype(np.float64)), 2.0 ** -38 * m)
        assert np.all(np.abs(back - x) <= bound)
        assert np.all(np.isfinite(hi.astype(np.float32)))


def test_split_of_zero_and_tiny_blocks():
    hi, mid, sh = split_block(np.zeros(32, np.float32))
    assert sh == 0 and not hi.any() and not mid.any()
    x = np.full(32, 1e-30, np.float32)
    hi, mid, sh = split_block(x)
    back = (hi.astype(np.float64) + mid.astype(np.float64)) * 2.0 ** -sh
    assert np.allclose(back, x.astype(np.float64), rtol=2.0 ** -20, atol=0)


def test_row_dot_matches_float64():
    rng = np.random.default_rng(11)
    K = 2880  # the C4 row length
    nb = K // 32
    worst = 0.0
    for _ in range(20):
        codes = rng.integers(0, 16, K)
        scales = rng.integers(119, 135, nb)
        x = (rng.standard_normal(K) * np.exp(rng.normal(0, 2, K))).astype(np.float32)
        w = E2M1[codes] * np.repeat(2.0 ** (scales.astype(np.float64) - 127), 32)
        ref = float(np.dot(w, x.astype(np.float64)))
        got = mx_dot(codes, scales, x)
        scale = float(np.sum(np.abs(w * x.astype(np.float64))))
        worst = max(worst, abs(got - ref) / scale)
    assert worst < 1e-6, worst
