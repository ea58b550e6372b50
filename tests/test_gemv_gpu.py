"""The int8 GEMV (accel_b200_matmul_q8 for m <= 8): every row-tile width,
ragged k and n, split K across warps and cluster ranks, single scales and the
fused epilogue, against the CPU checker and against the tensor-core path;
and the C5 sweep's m = 1 shape at K = N = 4096 (m = 16 runs on the tensor
cores)."""

import numpy as np
import pytest
import torch

from accelep_b200 import kernels as K
from accelep_b200 import synthetic as syn

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
def gemv_path():
    K.set_q8_path(3)
    yield
    K.set_q8_path(0)


@pytest.mark.parametrize("m,k,n", [(1, 64, 128), (1, 576, 960), (2, 100, 336), (3, 1536, 576), (4, 4100, 260),
                                   (5, 576, 3072), (8, 333, 1000), (7, 1024, 128), (8, 576, 49152),
                                   (1, 16384, 64), (6, 3000, 4), (1, 17, 4)])
def test_gemv_matches_checker(lib, cuda, orc, m, k, n):
    x, w, s = syn.int8_gemm(m, k, n, m + 3 * k + n)
    res = np.random.default_rng(m + n).standard_normal((m, n), dtype=np.float32)
    ep = K.make_epilogue(act="gelu", residual=T(res))
    got = H(K.matmul_q8(T(x), T(w), T(s), epilogue=ep))
    cols = slice(None) if n <= 4096 else slice(n - 300, n)
    want = orc.execute_matmul_q(x, np.ascontiguousarray(w[:, cols]), s[cols], act="gelu",
                                residual=np.ascontiguousarray(res[:, cols]))
    mag = np.abs(x).astype(np.float64) @ (np.abs(w[:, cols].astype(np.float64)) * s[cols].astype(np.float64))
    check_close(got[:, cols], want, k, mag)


def test_gemv_scalar_scale_repeat_and_tc(lib, cuda, orc):
    x, w, _ = syn.int8_gemm(7, 1536, 576, 8)
    scalar = np.array([0.004], np.float32)
    want = orc.matmul_quantized(x, w, scalar, None, [1536, 576], -1, 0, 7, 1536, 576)
    first = None
    for _ in range(3):
        got = H(K.matmul_q8(T(x), T(w), T(scalar), axis=-1))
        first = got if first is None else first
        assert np.array_equal(got, first)  # fixed reduction order
    mag = np.abs(x).astype(np.float64) @ np.abs(w.astype(np.float64)) * 0.004
    check_close(first, want, 1536, mag)
    K.set_q8_path(2)
    tc = H(K.matmul_q8(T(x), T(w), T(scalar), axis=-1))
    check_close(first, tc, 1536, mag)


@pytest.mark.parametrize("m", [1, 8])
def test_gemv_c5_shape(lib, cuda, orc, m):
    """C5 sweep shape K = N = 4096 (the larger sizes only differ in length)."""
    x, w, s = syn.int8_gemm(m, 4096, 4096, 55 + m)
    got = H(K.matmul_q8(T(x), T(w), T(s)))
    cols = slice(0, 512)
    want = orc.execute_matmul_q(x, np.ascontiguousarray(w[:, cols]), s[cols])
    mag = np.abs(x).astype(np.float64) @ (np.abs(w[:, cols].astype(np.float64)) * s[cols].astype(np.float64))
    check_close(got[:, cols], want, 4096, mag)


def test_gemv_by_shape_default(lib, cuda, orc):
    """With the default path the GEMV serves m <= 16 and agrees with the
    CUDA-core kernel."""
    K.set_q8_path(0)
    x, w, s = syn.int8_gemm(6, 800, 640, 21)
    by_shape = H(K.matmul_q8(T(x), T(w), T(s)))
    K.set_q8_path(1)
    simt = H(K.matmul_q8(T(x), T(w), T(s)))
    mag = np.abs(x).astype(np.float64) @ (np.abs(w.astype(np.float64)) * s.astype(np.float64))
    check_close(by_shape, simt, 800, mag)
