"""The arithmetic the int8 tensor-core product relies on (gemm_tc.cu),
restated in numpy and checked exhaustively on the CPU: a row segment's
exponent bounds every element and keeps the fixed-point values below 2^30;
the balanced base-256 digits the kernel takes from one 32-bit word per value
((X + 0x808080) XOR 0x808080, bytes 0..3 = d3, d2, d1, d0) recombine to X; and
the int32 sum of int8 x int8 digit products over a CTA's k cannot overflow."""

import numpy as np


def row_exponent(amax_bits):
    """RowExponent: e with every |y| < 2^e (at least -96); 0x7fff for Inf/NaN."""
    e = np.maximum((amax_bits >> 23).astype(np.int64) - 126, -96)
    return np.where(amax_bits >= 0x7F800000, 0x7FFF, e)


def digit_words(x):
    u = (x.astype(np.int64) & 0xFFFFFFFF).astype(np.uint64)
    return ((u + 0x808080) & 0xFFFFFFFF) ^ 0x808080


def signed_byte(w, b):
    v = ((w >> np.uint64(8 * b)) & np.uint64(0xFF)).astype(np.int64)
    return np.where(v >= 128, v - 256, v)


def test_digits_recombine():
    rng = np.random.default_rng(0)
    x = np.concatenate([rng.integers(-(2 ** 30) + 1, 2 ** 30, 500_000),
                        np.array([0, 1, -1, 127, 128, -128, -129, 255, 256, -256, 2 ** 30 - 1, -(2 ** 30) + 1,
                                  0x7F7F7F, -0x808080, 0x808080])])
    w = digit_words(x)
    d3, d2, d1, d0 = (signed_byte(w, b) for b in range(4))
    assert np.array_equal((d0 << 24) + (d1 << 16) + (d2 << 8) + d3, x)
    assert d0.min() >= -64 and d0.max() <= 64
    for d in (d1, d2, d3):
        assert d.min() >= -128 and d.max() <= 127


def test_exponent_bounds_fixed_point():
    rng = np.random.default_rng(1)
    y = np.concatenate([
        (rng.standard_normal(100_000) * 10.0 ** rng.integers(-30, 30, 100_000)).astype(np.float32),
        np.array([1.0, 2.0, 0.5, 1.9999999, 3.4e38, 1e-40, 1e-45, 0.0], np.float32)])
    bits = np.abs(y).view(np.uint32)
    e = row_exponent(bits)
    assert (e != 0x7FFF).all()
    a = np.abs(y.astype(np.float64))
    assert (a < 2.0 ** e).all()
    scaled = np.rint(a * 2.0 ** (30 - e))
    assert (scaled <= 2 ** 30).all()
    # 2^(30 - e) and 2^(e - 30) are normal floats for every exponent a row takes.
    assert (30 - e).min() >= -126 and (30 - e).max() <= 127
    assert (e - 30).min() >= -126
    bad = np.array([np.inf, -np.inf, np.nan], np.float32)
    assert (row_exponent(np.abs(bad).view(np.uint32)) == 0x7FFF).all()


def test_int32_digit_sums_cannot_overflow():
    # |w| <= 128, |digit| <= 128, at most 1023 x 128 k per CTA (kMaxBlocksPerCta x 128)
    assert 128 * 128 * 1023 * 128 < 2 ** 31
    # the int64 recombination of four such sums
    assert (2 ** 31) * (2 ** 24 + 2 ** 16 + 2 ** 8 + 1) < 2 ** 63
