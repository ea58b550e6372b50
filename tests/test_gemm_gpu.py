"""Parity of the int8 and fp32 products (accel_b200_matmul_q8 / _f32) with
the CPU checker: the reference's quantized panel (src/sim_device.cc:541-602)
and runtime epilogue (src/runtime.cc:326-344) on C1 (full size), the stored
reference cases (per-column, per-row with zero point, scalar scale) and the
C5 sweep shapes (column slices at full size). Tolerance rtol = atol = 1e-4
on top of the fp32 reassociation bound."""

import numpy as np
import pytest
import torch

from accelep_b200 import kernels as K
from accelep_b200 import synthetic as syn
from tests.conftest import GOLDEN

pytestmark = pytest.mark.gpu


def T(a, dtype=None):
    t = torch.as_tensor(np.ascontiguousarray(a))
    return t.to(device="cuda", dtype=dtype) if dtype is not None else t.to("cuda")


def H(t):
    torch.cuda.synchronize()
    return t.detach().cpu().numpy()


def close(got, want, k_terms=None, scale=None):
    """rtol = atol = 1e-4, widened by the bound on fp32 reassociation
    (k_terms * eps * sum |a_i w_i|) when that is larger."""
    tol = 1e-4 + 1e-4 * np.abs(want)
    if k_terms is not None:
        tol = np.maximum(tol, 2 * k_terms * np.finfo(np.float32).eps * scale)
    bad = np.abs(got - want) > tol
    assert not bad.any(), f"{bad.sum()} of {bad.size} outside tolerance; max err {np.max(np.abs(got - want))}"


def abs_dot(x, w, s):
    return np.abs(x).astype(np.float64) @ (np.abs(w.astype(np.float64)) * s.astype(np.float64))


def test_c1_relu_full(lib, cuda, orc):
    x, w, s = syn.int8_gemm(64, 576, 1536, 1)
    want = orc.execute_matmul_q(x, w, s, act="relu")
    got = H(K.matmul_q8(T(x), T(w), T(s), epilogue=K.make_epilogue(act="relu")))
    close(got, want, 576, abs_dot(x, w, s))


def test_stored_planes(lib, cuda):
    small = np.load(GOLDEN / "ref_small.npz")
    for tag in ("q1", "q2", "q3"):
        a, q = small[tag + "_a"], small[tag + "_q"]
        m, k = a.shape
        got = H(K.matmul_q8(T(a), T(q), T(small[tag + "_col"]), axis=1))
        close(got, small[tag + "_c_col"], k, abs_dot(a, q, small[tag + "_col"]))
        got = H(K.matmul_q8(T(a), T(q), T(small[tag + "_row"]), zero=T(small[tag + "_zero"]), axis=0))
        close(got, small[tag + "_c_row"], k, np.abs(a).astype(np.float64) @ (np.abs(q.astype(np.float64)) + 5) * 1.0)
        got = H(K.matmul_q8(T(a), T(q), T(np.array([0.5], np.float32)), axis=-1))
        close(got, small[tag + "_c_scalar"], k, abs_dot(a, q, np.full(q.shape[1], 0.5, np.float32)))


def test_dequantize_kat(lib, cuda):
    import json

    kat = json.loads((GOLDEN / "kats.json").read_text())["dequantize"]
    got = H(K.matmul_q8(T(np.array(kat["x"], np.float32)), T(np.array(kat["w"], np.int8)),
                        T(np.array(kat["scale"], np.float32)), zero=T(np.array(kat["zero"], np.int8)), axis=0))
    assert got.tolist() == kat["want"]


@pytest.mark.parametrize("m", [1, 2, 3, 5, 8, 13, 16, 32, 64, 130])
def test_epilogue_and_split_shapes(lib, cuda, orc, m):
    """Odd sizes that exercise the unaligned columns, the K split and the
    residual / Gelu epilogue (the runtime applies the activation, then adds
    the residual)."""
    rng = np.random.default_rng(m)
    k, n = 1000 + m, 333
    x, w, s = syn.int8_gemm(m, k, n, m)
    res = rng.standard_normal((m, n), dtype=np.float32)
    want = orc.execute_matmul_q(x, w, s, act="gelu", residual=res)
    got = H(K.matmul_q8(T(x), T(w), T(s), epilogue=K.make_epilogue(act="gelu", residual=T(res))))
    close(got, want, k, abs_dot(x, w, s))


def test_residual_in_place(lib, cuda, orc):
    x, w, s = syn.int8_gemm(32, 576, 576, 9)
    h = np.random.default_rng(9).standard_normal((32, 576), dtype=np.float32)
    want = orc.execute_matmul_q(x, w, s, residual=h)
    ht = T(h)
    K.matmul_q8(T(x), T(w), T(s), epilogue=K.make_epilogue(residual=ht), out=ht)
    close(H(ht), want, 576, abs_dot(x, w, s))


@pytest.mark.parametrize("m,kn", [(1, 4096), (16, 4096), (128, 4096), (1, 16384), (16, 8192), (2048, 4096)])
def test_c5_column_slice(lib, cuda, orc, m, kn):
    """The full C5 operands on the GPU; the checker recomputes a slice of
    columns (columns are independent) and a few rows at large M."""
    x, w, s = syn.int8_gemm(m, kn, kn, 5)
    got = H(K.matmul_q8(T(x), T(w), T(s)))
    cols = slice(kn // 2 - 48, kn // 2 + 80)
    rows = slice(None) if m <= 128 else slice(m - 7, m)
    want = orc.execute_matmul_q(x[rows], np.ascontiguousarray(w[:, cols]), s[cols])
    close(got[rows, cols], want, kn, abs_dot(x[rows], w[:, cols], s[cols]))
    # The full product against float64, as a size-independent check.
    full = (x.astype(np.float64)[rows] @ (w.astype(np.float64) * s.astype(np.float64)))
    close(got[rows], full.astype(np.float32), kn, abs_dot(x[rows], w, s))


def test_f32_product(lib, cuda, orc):
    rng = np.random.default_rng(11)
    for m, k, n in [(1, 576, 49152), (4, 576, 960), (32, 1536, 576), (7, 33, 70)]:
        a = rng.standard_normal((m, k), dtype=np.float32)
        b = rng.standard_normal((k, n), dtype=np.float32) * np.float32(0.02)
        got = H(K.matmul_f32(T(a), T(b)))
        close(got, orc.matmul(a, b), k, np.abs(a).astype(np.float64) @ np.abs(b).astype(np.float64))


def test_empty_k(lib, cuda):
    got = H(K.matmul_q8(T(np.zeros((3, 0), np.float32)), T(np.zeros((0, 4), np.int8)), T(np.ones(4, np.float32)),
                        epilogue=K.make_epilogue(alpha=2.0)))
    assert got.tolist() == [[0.0] * 4] * 3


def c2_chain_gpu(x, blocks, rows):
    """C2 on the device: per block h = Gelu(x @ W1) (fused Gelu epilogue),
    s = h @ W2 + x (fused residual), x' = RmsNorm(s) (eps 1e-5)."""
    h = T(x[:rows])
    for w1, s1, w2, s2, gamma in blocks:
        t = K.matmul_q8(h, T(w1), T(s1), epilogue=K.make_epilogue(act="gelu"))
        s = K.matmul_q8(t, T(w2), T(s2), epilogue=K.make_epilogue(residual=h))
        h = K.rmsnorm(s, T(gamma), rows, s.shape[1], 1e-5)
    return H(h)


def test_c2_mlp_chain(lib, cuda, orc):
    """Config C2, the whole 4-block chain at batch 256 (hidden 1024 -> 4096 ->
    1024; the rows run on the tensor cores), against the CPU checker's
    block-by-block chain (src/ep.cc:1602-1626 order) on all 256 rows and
    against the stored 16-row golden of the reference chain."""
    x, blocks = syn.mlp_stack()
    got = c2_chain_gpu(x, blocks, 256)
    want = x.copy()
    for w1, s1, w2, s2, gamma in blocks:
        want, _ = orc.mlp_block(want, w1, s1, w2, s2, gamma, 1e-5)
    np.testing.assert_allclose(got, want, rtol=1e-4, atol=1e-4)
    np.testing.assert_allclose(got[:16], np.load(GOLDEN / "ref_small.npz")["c2_rows16"], rtol=1e-4, atol=1e-4)
