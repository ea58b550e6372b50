"""The tcgen05 int8 product (accel_b200_matmul_q8 on its tensor-core path)
against the CPU checker and against the CUDA-core path: partial feature
tiles, partial row tiles, K that is not a multiple of the 64-deep block,
split K across a thread-block cluster (with a ragged last split), single
scales and the fused epilogue."""

import numpy as np
import pytest
import torch

from accelep_b200 import kernels as K
from accelep_b200 import synthetic as syn
from accelep_b200._lib import B200Error

pytestmark = pytest.mark.gpu


def T(a):
    return torch.as_tensor(np.ascontiguousarray(a)).to("cuda")


def H(t):
    torch.cuda.synchronize()
    return t.detach().cpu().numpy()


def check_close(got, want, k, scale_mag):
    tol = 1e-4 + 1e-4 * np.abs(want)
    tol = np.maximum(tol, 2 * k * np.finfo(np.float32).eps * scale_mag)
    err = np.abs(got - want)
    assert (err <= tol).all(), f"{(err > tol).sum()} of {err.size} outside tolerance, max err {err.max()}"


@pytest.fixture(autouse=True)
def tensor_cores():
    """Every product in this file on the tensor-core kernel where eligible
    (the default path sends m <= 16 to the GEMV)."""
    K.set_q8_path(2)
    yield
    K.set_q8_path(0)


@pytest.mark.parametrize("m,k,n", [(1, 64, 128), (32, 576, 960), (7, 100, 336), (33, 576, 576), (64, 1536, 576),
                                   (100, 192, 3072), (130, 576, 1536), (300, 640, 272), (32, 1536, 49152),
                                   (5, 4104, 256), (128, 8192, 512), (16, 16384, 16384), (12, 4096, 1024)])
def test_tc_matches_checker(lib, cuda, orc, m, k, n):
    x, w, s = syn.int8_gemm(m, k, n, m + k + n)
    res = np.random.default_rng(m).standard_normal((m, n), dtype=np.float32)
    ep = K.make_epilogue(act="gelu", residual=T(res))
    got = H(K.matmul_q8(T(x), T(w), T(s), epilogue=ep))
    mag = np.abs(x).astype(np.float64) @ (np.abs(w.astype(np.float64)) * s.astype(np.float64))
    cols = slice(None) if n <= 4096 else slice(n - 300, n)
    want = orc.execute_matmul_q(x, np.ascontiguousarray(w[:, cols]), s[cols], act="gelu",
                                residual=np.ascontiguousarray(res[:, cols]))
    check_close(got[:, cols], want, k, mag[:, cols])


def test_tc_equals_cuda_core_path(lib, cuda):
    x, w, s = syn.int8_gemm(32, 576, 960, 3)
    xt, wt, st = T(x), T(w), T(s)
    tc = H(K.matmul_q8(xt, wt, st))
    K.set_q8_path(1)
    simt = H(K.matmul_q8(xt, wt, st))
    mag = np.abs(x).astype(np.float64) @ (np.abs(w.astype(np.float64)) * s.astype(np.float64))
    check_close(tc, simt, 576, mag)


def test_tc_scalar_scale_and_repeat(lib, cuda, orc):
    """axis -1 (one scale) and repeated calls on one workspace: the split-K
    arrival counters return to zero after every call."""
    x, w, _ = syn.int8_gemm(16, 1536, 576, 8)
    scalar = np.array([0.004], np.float32)
    ws = torch.zeros(K.load().accel_b200_matmul_q8_workspace(16, 1536, 576), dtype=torch.uint8, device="cuda")
    want = orc.matmul_quantized(x, w, scalar, None, [1536, 576], -1, 0, 16, 1536, 576)
    first = None
    for _ in range(3):
        got = H(K.matmul_q8(T(x), T(w), T(scalar), axis=-1, workspace=ws))
        first = got if first is None else first
        assert np.array_equal(got, first)  # deterministic split order
    mag = np.abs(x).astype(np.float64) @ np.abs(w.astype(np.float64)) * 0.004
    check_close(first, want, 1536, mag)
    assert not H(ws[:256]).any()


@pytest.mark.parametrize("m,inter,n", [(1, 1536, 576), (32, 1536, 576), (40, 256, 384), (100, 320, 128),
                                       (7, 100, 336)])
def test_silu_product_matches_checker(lib, cuda, orc, m, inter, n):
    """SiluMul rows feeding the product (accel_b200_matmul_q8_silu): the
    in-kernel SiluMul (m <= 64, up to two k blocks per CTA), the digit pass of the
    planes path (m > 64), and the CUDA-core path (inter not a multiple of 4
    or 8 goes there too), each against SiluMul + MatMul of the checker."""
    rng = np.random.default_rng(m * inter + n)
    gu = rng.standard_normal((m, 2 * inter), dtype=np.float32) * 2
    _, w, s = syn.int8_gemm(1, inter, n, m + n)
    res = rng.standard_normal((m, n), dtype=np.float32)
    act = orc.silu_mul(np.ascontiguousarray(gu[:, :inter]), np.ascontiguousarray(gu[:, inter:]))
    want = orc.execute_matmul_q(act, w, s, residual=res)
    mag = np.abs(act).astype(np.float64) @ (np.abs(w.astype(np.float64)) * s.astype(np.float64))
    for path in (2, 1):
        K.set_q8_path(path)
        ep = K.make_epilogue(residual=T(res))
        got = H(K.matmul_q8_silu(T(gu), T(w), T(s), epilogue=ep))
        check_close(got, want, inter, mag)


def test_fp32_tile_product_every_row_count(lib, cuda, orc):
    """m = 1 .. 64 with the in-kernel operand (R = 16, 32 and 64, ragged row tiles)."""
    x, w, s = syn.int8_gemm(64, 576, 256, 11)
    xt, wt, st = T(x), T(w), T(s)
    want = orc.execute_matmul_q(x, w, s)
    mag = np.abs(x).astype(np.float64) @ (np.abs(w.astype(np.float64)) * s.astype(np.float64))
    for m in (1, 2, 15, 16, 17, 31, 32, 33, 63, 64):
        got = H(K.matmul_q8(xt[:m].contiguous(), wt, st))
        check_close(got, want[:m], 576, mag[:m])


@pytest.mark.parametrize("m,k,n,ldx", [(32, 576, 960, 576), (33, 576, 576, 600), (32, 576, 49152, 576),
                                       (100, 576, 384, 576), (1, 1536, 256, 1536), (7, 100, 336, 100)])
def test_rmsnorm_product(lib, cuda, orc, m, k, n, ldx):
    """RmsNorm rows feeding the product (accel_b200_matmul_q8_rmsnorm): the
    in-kernel norm (decode sizes), the norm variant of the digit pass (planes mode)
    (long K walks, m > 64) and the CUDA-core path (k % 8 != 0). The
    normalized values are those of accel_b200_rmsnorm, so the result equals
    RmsNorm then the product bit for bit, and the checker's RmsNorm + MatMul
    within tolerance."""
    rng = np.random.default_rng(m + k + n)
    xs = rng.standard_normal((m, ldx), dtype=np.float32) * 3
    gamma = (rng.standard_normal(k, dtype=np.float32) * 0.5 + 1).astype(np.float32)
    _, w, s = syn.int8_gemm(1, k, n, m * n)
    x = np.ascontiguousarray(xs[:, :k])
    normed = orc.rmsnorm(x, gamma, m, k, 1e-5)
    want = orc.execute_matmul_q(normed, w, s, act="relu")
    mag = np.abs(normed).astype(np.float64) @ (np.abs(w.astype(np.float64)) * s.astype(np.float64))
    xt, gt, wt, st = T(xs), T(gamma), T(w), T(s)
    got = H(K.matmul_q8_rmsnorm(xt, gt, 1e-5, wt, st, epilogue=K.make_epilogue(act="relu")))
    check_close(got, want, k, mag)
    dev_normed = K.rmsnorm(xt[:, :k].contiguous(), gt, m, k, 1e-5)
    two_step = H(K.matmul_q8(dev_normed, wt, st, epilogue=K.make_epilogue(act="relu")))
    assert np.array_equal(got, two_step)


@pytest.mark.parametrize("m,k,n,path", [(32, 576, 576, 2), (32, 1536, 576, 2), (200, 576, 576, 2), (4, 576, 576, 3),
                                        (1, 1536, 1000, 3)])
def test_row_sums_of_squares(lib, cuda, m, k, n, path):
    """accel_b200_epilogue.row_sq on the tensor-core (split and unsplit K) and
    GEMV paths: per row and 128-column block, the sum of squares of the final
    outputs (after the residual), against numpy's sum in float64."""
    K.set_q8_path(path)
    x, w, s = syn.int8_gemm(m, k, n, m + k + n)
    res = T(np.random.default_rng(m).standard_normal((m, n), dtype=np.float32))
    blocks = (n + 127) // 128
    sq = torch.full((m, blocks + 1), -1.0, dtype=torch.float64, device="cuda")
    out = H(K.matmul_q8(T(x), T(w), T(s), epilogue=K.make_epilogue(residual=res, row_sq=sq)))
    got = H(sq)
    o = out.astype(np.float64)
    want = np.stack([(o[:, b * 128:(b + 1) * 128] ** 2).sum(axis=1) for b in range(blocks)], axis=1)
    np.testing.assert_allclose(got[:, :blocks], want, rtol=1e-12)
    assert (got[:, blocks] == -1.0).all()  # nothing written past the blocks


def test_rmsnorm_from_sums_of_squares(lib, cuda, orc):
    """The RmsNorm-fed product with the row sums of squares supplied (as the
    engine's decode chains them: the residual product writes them, the next
    product reads them) against the row-reading form."""
    m, h, n = 32, 576, 960
    rng = np.random.default_rng(3)
    xs, w1, s1 = syn.int8_gemm(m, h, h, 5)
    resid = T(rng.standard_normal((m, h), dtype=np.float32))
    sq = torch.zeros(m, 5, dtype=torch.float64, device="cuda")
    hid = K.matmul_q8(T(xs), T(w1), T(s1), epilogue=K.make_epilogue(residual=resid, row_sq=sq))
    gamma = T(rng.uniform(0.5, 1.5, h).astype(np.float32))
    _, w2, s2 = syn.int8_gemm(1, h, n, 6)
    by_rows = H(K.matmul_q8_rmsnorm(hid, gamma, 1e-5, T(w2), T(s2)))
    by_sums = H(K.matmul_q8_rmsnorm_stats(hid, sq, gamma, 1e-5, T(w2), T(s2)))
    np.testing.assert_allclose(by_sums, by_rows, rtol=1e-6, atol=1e-6)
    want = orc.execute_matmul_q(orc.rmsnorm(H(hid), H(gamma), m, h, 1e-5), w2, s2)
    np.testing.assert_allclose(by_sums, want, rtol=1e-4, atol=1e-4)


# The integer tensor-core path puts each activation row segment in 30-bit fixed
# point against its largest magnitude and sums the int8 digit planes exactly.
# Shapes: in-kernel operand with and without split K, planes mode (long K walks
# and m > 64).
FIXED_POINT_SHAPES = [(32, 576, 256), (7, 256, 128), (16, 4096, 256), (100, 576, 384), (40, 1536, 128)]


@pytest.mark.parametrize("m,k,n", FIXED_POINT_SHAPES)
def test_power_of_two_scaling_is_exact(lib, cuda, m, k, n):
    """Scaling the activations by 2^-60 or 2^40 scales every output by the
    same power of two, bit for bit: the row exponents absorb the scale and the
    digits do not change."""
    x, w, s = syn.int8_gemm(m, k, n, m * 7 + k)
    wt, st = T(w), T(s)
    base = H(K.matmul_q8(T(x), wt, st))
    for p in (-60, 40):
        f = np.float32(2.0 ** p)
        got = H(K.matmul_q8(T(x * f), wt, st))
        assert np.array_equal(got, base * f), p


@pytest.mark.parametrize("m,k,n", FIXED_POINT_SHAPES)
def test_integer_activations_are_exact(lib, cuda, m, k, n):
    """Integer-valued activations are represented exactly, so every output is
    the exact integer dot product rounded once and times the column scale
    (all partial sums stay below 2^24, so split-K adds are exact too)."""
    rng = np.random.default_rng(k + n)
    x = rng.integers(-16, 17, (m, k)).astype(np.float32)
    w = rng.integers(-127, 128, (k, n)).astype(np.int8)
    s = rng.uniform(1e-3, 1e-2, n).astype(np.float32)
    got = H(K.matmul_q8(T(x), T(w), T(s)))
    exact = x.astype(np.int64) @ w.astype(np.int64)
    assert np.abs(exact).max() < 2 ** 24
    want = exact.astype(np.float32) * s[None, :]
    assert np.array_equal(got, want)


@pytest.mark.parametrize("m,k,n", FIXED_POINT_SHAPES)
def test_rows_of_different_magnitude(lib, cuda, orc, m, k, n):
    """Rows whose magnitudes differ by 2^60 are each scaled by their own
    exponent (every row keeps its precision), and a row with one element 2^20
    times its others stays within the fixed point's bound: per element an
    absolute error of at most 2^(e - 31)."""
    x, w, s = syn.int8_gemm(m, k, n, m + 3 * k)
    x = x.copy()
    x[::2] *= np.float32(2.0 ** -60)
    x[1, 3] = np.float32(2.0 ** 20)
    got = H(K.matmul_q8(T(x), T(w), T(s)))
    want = orc.execute_matmul_q(x, w, s)
    ws = np.abs(w.astype(np.float64)) * s.astype(np.float64)
    mag = np.abs(x).astype(np.float64) @ ws
    # fp32 accumulation of the checker plus the fixed point's bound on each row
    e = np.floor(np.log2(np.abs(x).max(axis=1).astype(np.float64))) + 1
    fixed = (2.0 ** (e - 31))[:, None] * ws.sum(axis=0)[None, :]
    tol = 2 * k * np.finfo(np.float32).eps * mag + fixed + 1e-30
    err = np.abs(got.astype(np.float64) - want)
    assert (err <= tol).all(), f"{(err > tol).sum()} outside, max ratio {(err / tol).max()}"


def test_non_finite_rows_give_nan(lib, cuda):
    """A row holding Inf or NaN yields NaN outputs; the other rows are the
    same as without it."""
    for m, k, n in [(32, 576, 256), (100, 576, 384)]:
        x, w, s = syn.int8_gemm(m, k, n, 5)
        wt, st = T(w), T(s)
        base = H(K.matmul_q8(T(x), wt, st))
        bad = x.copy()
        bad[3, 10] = np.inf
        bad[5, 0] = np.nan
        got = H(K.matmul_q8(T(bad), wt, st))
        assert np.isnan(got[3]).all() and np.isnan(got[5]).all()
        keep = [r for r in range(m) if r not in (3, 5)]
        assert np.array_equal(got[keep], base[keep])


@pytest.mark.parametrize("m,k,inter,stats", [(32, 576, 1536, True), (32, 576, 1536, False), (7, 576, 256, False),
                                             (200, 576, 384, False), (40, 1536, 128, True)])
def test_rmsnorm_silu_pairs(lib, cuda, orc, m, k, inter, stats):
    """The gate|up product with SiluMul in its epilogue
    (accel_b200_matmul_q8_rmsnorm_silu_pairs, columns in 64-column pairs)
    equals the plain RmsNorm-fed product of the unpaired columns followed by
    SiluMul bit for bit; that product is within tolerance of the checker's
    RmsNorm and MatMul."""
    rng = np.random.default_rng(m + k + inter)
    x = rng.standard_normal((m, k), dtype=np.float32) * 2
    gamma = rng.uniform(0.5, 1.5, k).astype(np.float32)
    _, w, s = syn.int8_gemm(1, k, 2 * inter, m + inter)
    xt, gt, wt, st = T(x), T(gamma), T(w), T(s)
    sq = None
    if stats:
        blocks = (k + 127) // 128
        x64 = x.astype(np.float64)
        sq = T(np.stack([(x64[:, b * 128:(b + 1) * 128] ** 2).sum(axis=1) for b in range(blocks)], axis=1))
    got = H(K.matmul_q8_rmsnorm_silu_pairs(xt, gt, 1e-5, K.pair_gate_up(wt, inter), K.pair_gate_up(st, inter),
                                           row_sq=sq))
    assert got.shape == (m, inter)
    gu = (K.matmul_q8_rmsnorm_stats(xt, sq, gt, 1e-5, wt, st) if stats else K.matmul_q8_rmsnorm(xt, gt, 1e-5, wt, st))
    gate, up = gu[:, :inter].contiguous(), gu[:, inter:].contiguous()
    assert np.array_equal(got, H(K.silu_mul(gate, up)))
    # The product part against the checker (fp32 accumulation bound), as the
    # other product tests compare it.
    normed = orc.rmsnorm(x, gamma, m, k, 1e-5)
    mag = np.abs(normed).astype(np.float64) @ (np.abs(w.astype(np.float64)) * s.astype(np.float64))
    check_close(H(gu), orc.execute_matmul_q(normed, w, s), k, mag)


def test_rmsnorm_silu_pairs_rejects(lib, cuda):
    x = torch.zeros(4, 576, device="cuda")
    g = torch.ones(576, device="cuda")
    w = torch.zeros(576, 200, dtype=torch.int8, device="cuda")
    s = torch.ones(200, device="cuda")
    with pytest.raises(B200Error):  # n not a multiple of 128
        K.matmul_q8_rmsnorm_silu_pairs(x, g, 1e-5, w, s)
