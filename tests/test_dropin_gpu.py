"""AccelEP's own callers of accel::Device running on the B200 device.

tests/dropin/Makefile compiles the reference's runtime (src/runtime.cc), Llama
model (src/llama_model.cc) and one-matmul API (src/sim_api.cc) from a copy of
the AccelEP sources with reference_on_b200.patch applied (the MatMulQ8
virtual, the runtime.cc:326 switch, the factories, the Llama's host reads of
device memory), together with this repository's B200Device built against the
host's accel/device.h. Here those unchanged callers run on the GPU and are
compared with the same calls on SimDevice (oracle/_ref): results within
rtol = atol = 1e-4 (token ids exactly) and the reference's counters equal.
"""

import ctypes

import numpy as np
import pytest

from accelep_b200 import synthetic as syn
from tests.conftest import GOLDEN, ROOT

pytestmark = pytest.mark.gpu

TOL = 1e-4
DROPIN = ROOT / "tests" / "_build" / "dropin" / "libaccel_dropin.so"
STAT_KEYS = ("matmul_ops", "gemm_ops", "kernel_matmuls", "relu", "gelu", "add", "transposes", "bytes_to_device",
             "bytes_to_host")

_f32p = ctypes.POINTER(ctypes.c_float)
_i8p = ctypes.POINTER(ctypes.c_int8)
_i64p = ctypes.POINTER(ctypes.c_int64)
_i64 = ctypes.c_int64


def _p(a, t):
    return None if a is None else a.ctypes.data_as(t)


class DropIn:
    """libaccel_dropin.so: the reference's accel_llama_* / accel_sim_* and
    runtime entry points, all on B200Device."""

    llama_api = True

    def __init__(self, path):
        from oracle.oracle import _bind_llama_api

        self.lib = ctypes.CDLL(str(path))
        _bind_llama_api(self.lib)
        self.lib.dropin_last_error.restype = ctypes.c_char_p
        self.lib.dropin_device_name.restype = ctypes.c_char_p
        self.lib.dropin_execute_matmul_q.restype = ctypes.c_int
        self.lib.dropin_execute_matmul_q.argtypes = [_f32p, _i64, _i64, _i8p, _f32p, _i8p, _i64, _i64, ctypes.c_int,
                                                     _f32p, _f32p, _i64p]
        self.lib.dropin_mlp_block.restype = ctypes.c_int
        self.lib.dropin_mlp_block.argtypes = [_f32p, _i64, _i64, _i64, _i8p, _f32p, _i8p, _f32p, _f32p, ctypes.c_float,
                                              _f32p, _f32p, _i64p]

    def _ok(self, rc):
        if rc != 0:
            raise RuntimeError(self.lib.dropin_last_error().decode())

    def execute_matmul_q(self, x, q, scale, zero=None, axis=1, act="none", residual=None):
        x = np.ascontiguousarray(x, np.float32)
        q = np.ascontiguousarray(q, np.int8)
        m, k = x.shape
        n = q.shape[1]
        out = np.zeros((m, n), np.float32)
        stats = np.zeros(9, np.int64)
        z = None if zero is None else np.ascontiguousarray(zero, np.int8)
        r = None if residual is None else np.ascontiguousarray(residual, np.float32)
        self._ok(self.lib.dropin_execute_matmul_q(_p(x, _f32p), m, k, _p(q, _i8p),
                                                  _p(np.ascontiguousarray(scale, np.float32), _f32p), _p(z, _i8p),
                                                  axis, n, {"none": 0, "relu": 1, "gelu": 2}[act], _p(r, _f32p),
                                                  _p(out, _f32p), _p(stats, _i64p)))
        return out, dict(zip(STAT_KEYS, (int(v) for v in stats)))

    def mlp_block(self, x, w1, s1, w2, s2, gamma, eps):
        x = np.ascontiguousarray(x, np.float32)
        m, hidden = x.shape
        inter = w1.shape[1]
        pre, out = np.zeros((m, hidden), np.float32), np.zeros((m, hidden), np.float32)
        stats = np.zeros(9, np.int64)
        f = lambda a: np.ascontiguousarray(a, np.float32)  # noqa: E731
        self._ok(self.lib.dropin_mlp_block(_p(x, _f32p), m, hidden, inter, _p(np.ascontiguousarray(w1), _i8p),
                                           _p(f(s1), _f32p), _p(np.ascontiguousarray(w2), _i8p), _p(f(s2), _f32p),
                                           _p(f(gamma), _f32p), ctypes.c_float(eps), _p(pre, _f32p), _p(out, _f32p),
                                           _p(stats, _i64p)))
        return out, pre, dict(zip(STAT_KEYS, (int(v) for v in stats)))


@pytest.fixture(scope="module")
def dropin(cuda, lib):
    if not DROPIN.is_file():
        pytest.skip("tests/_build/dropin/libaccel_dropin.so is not built (make -C tests/dropin needs the AccelEP "
                    "sources)")
    return DropIn(DROPIN)


def check_close(got, want, k, mag):
    """The products' tolerance in this suite: rtol = atol = 1e-4, widened to
    2 k fp32 ulps of the sum of |terms| where long sums cancel (the reference
    accumulates in fp32 in its own order)."""
    tol = np.maximum(1e-4 + 1e-4 * np.abs(want), 2 * k * np.finfo(np.float32).eps * mag)
    err = np.abs(got - want)
    assert (err <= tol).all(), f"{(err > tol).sum()} of {err.size} outside tolerance, max err {err.max()}"


def _ref_stats(ref, call):
    ref.lib.ref_reset_stats()
    out = call()
    return out, ref.stats()


def test_device_is_the_b200(dropin):
    assert dropin.lib.dropin_device_name().decode() == "b200"


@pytest.mark.parametrize("case", ["c1", "rows_zero", "scalar_residual", "odd"])
def test_execute_matmul_quant_operand(dropin, ref, case):
    """accel::ExecuteMatMul's quant branch (src/runtime.cc:272-350) with the
    device's MatMulQ8: C1 (X [64, 576] @ int8 W [576, 1536], per-column
    scales, Relu), per-row scales with zero points, one scale with a residual,
    and odd sizes; outputs and all nine counters against SimDevice."""
    rng = np.random.default_rng({"c1": 1, "rows_zero": 2, "scalar_residual": 3, "odd": 4}[case])
    if case == "c1":
        x, w, s = syn.int8_gemm(64, 576, 1536, 1)
        args = dict(act="relu")
    elif case == "rows_zero":
        x, w, _ = syn.int8_gemm(16, 160, 300, 5)
        s = rng.uniform(0.1, 1.0, 160).astype(np.float32)
        args = dict(zero=rng.integers(-5, 6, 160).astype(np.int8), axis=0, act="gelu")
    elif case == "scalar_residual":
        x, w, _ = syn.int8_gemm(33, 576, 576, 6)
        s = np.array([0.004], np.float32)
        args = dict(axis=-1, residual=rng.standard_normal((33, 576), dtype=np.float32))
    else:
        x, w, s = syn.int8_gemm(5, 77, 261, 7)
        args = dict(act="relu")
    got, stats = dropin.execute_matmul_q(x, w, s, **args)
    want, want_stats = _ref_stats(ref, lambda: ref.execute_matmul_q(x, w, s, **args))
    wq = w.astype(np.float64)
    if args.get("axis", 1) == 0:
        deq = np.abs(wq - args["zero"].astype(np.float64)[:, None]) * s.astype(np.float64)[:, None]
    else:
        deq = np.abs(wq) * s.astype(np.float64)
    check_close(got, want, x.shape[1], np.abs(x).astype(np.float64) @ deq)
    assert stats == want_stats


def test_execute_matmul_c1_golden(dropin, ref):
    """C1 on the B200 through the reference's runtime against the stored
    reference output (tests/golden/ref_small.npz: digest and first row)."""
    small = np.load(GOLDEN / "ref_small.npz")
    x, w, s = syn.int8_gemm(64, 576, 1536, 1)
    got, _ = dropin.execute_matmul_q(x, w, s, act="relu")
    np.testing.assert_allclose(got[0], small["c1_row0"], rtol=TOL, atol=TOL)


def test_mlp_chain_c2(dropin, ref):
    """The plugin's prenorm int8 MLP block order (src/ep.cc:1602-1626) through
    the reference's runtime on the B200: C2's 4 blocks on 16 rows against the
    stored reference rows, and one small block's counters against SimDevice."""
    small = np.load(GOLDEN / "ref_small.npz")
    x, blocks = syn.mlp_stack()
    h = x[:16]
    for w1, s1, w2, s2, gamma in blocks:
        h, _, stats = dropin.mlp_block(h, w1, s1, w2, s2, gamma, 1e-5)
    np.testing.assert_allclose(h, small["c2_rows16"], rtol=TOL, atol=TOL)
    xs, bs = syn.mlp_stack(m=4, hidden=64, inter=256, blocks=1, seed=9)
    got, pre, stats = dropin.mlp_block(xs, *bs[0], 1e-5)
    (want, want_pre), want_stats = _ref_stats(ref, lambda: ref.mlp_block(xs, *bs[0], 1e-5))
    np.testing.assert_allclose(got, want, rtol=TOL, atol=TOL)
    np.testing.assert_allclose(pre, want_pre, rtol=TOL, atol=TOL)
    assert stats == want_stats


def test_reference_llama_on_b200_c3(dropin):
    """The reference's own LlamaModel (src/llama_model.cc: Forward's 17 device
    calls per layer, Generate's loop) on B200Device, C3 (fp32 SmolLM2-135M
    shape, context 128): the prefill logits within 1e-4 of the stored reference
    row (the reference's LogitMaxAbs), the 64 greedy ids equal, and the
    reference's counters: 211 kernel matmuls per forward, 16 bytes of prompt
    in; out, the 64 ids plus the patch's one 4-byte id read per generated
    token (SimDevice reads its host heap directly)."""
    from oracle.oracle import LlamaHandle

    g = np.load(GOLDEN / "c3_smollm.npz")
    cfg = dict(syn.SMOLLM2_135M, context=128)
    model = LlamaHandle(dropin, cfg)
    model.load(syn.llama_weights(cfg, 3))
    lib = dropin.lib
    lib.accel_sim_reset_stats()
    model.forward_ids(g["prompt"], True)
    assert lib.accel_sim_matmuls() == 211 and lib.accel_sim_bytes_to_device() == 16
    assert model.logit_max_abs(g["prefill_logits"]) <= TOL
    lib.accel_sim_reset_stats()
    ids = model.generate(g["prompt"], 64)
    assert np.array_equal(ids, g["ids"]), (ids, g["ids"])
    assert lib.accel_sim_matmuls() == 211 * 65
    assert lib.accel_sim_bytes_to_device() == 16
    assert lib.accel_sim_bytes_to_host() == 64 * 4 + 64 * 4
    model.close()


def test_reference_sim_api_on_b200(dropin, orc):
    """The reference's accel_sim_* (src/sim_api.cc) on B200Device: Device::MatMul
    keeps PackedMatMul's bits."""
    lib = dropin.lib
    lib.accel_sim_create.restype = ctypes.c_void_p
    lib.accel_sim_destroy.argtypes = [ctypes.c_void_p]
    lib.accel_sim_upload.restype = ctypes.c_void_p
    lib.accel_sim_upload.argtypes = [ctypes.c_void_p, _f32p, _i64]
    lib.accel_sim_release.argtypes = [ctypes.c_void_p, ctypes.c_void_p]
    lib.accel_sim_matmul.restype = ctypes.c_int
    lib.accel_sim_matmul.argtypes = [ctypes.c_void_p, _f32p, _i64, _i64, ctypes.c_void_p, _i64, _f32p]
    rng = np.random.default_rng(12)
    a = rng.standard_normal((13, 19), dtype=np.float32)
    b = rng.standard_normal((19, 17), dtype=np.float32)
    sim = lib.accel_sim_create()
    assert sim
    buf = lib.accel_sim_upload(sim, _p(b, _f32p), b.size)
    c = np.zeros((13, 17), np.float32)
    lib.accel_sim_reset_stats()
    assert lib.accel_sim_matmul(sim, _p(a, _f32p), 13, 19, buf, 17, _p(c, _f32p)) == 0
    assert np.array_equal(c, orc.matmul(a, b))
    assert lib.accel_sim_matmuls() == 1
    assert lib.accel_sim_bytes_to_device() == a.nbytes and lib.accel_sim_bytes_to_host() == c.nbytes
    lib.accel_sim_release(sim, buf)
    lib.accel_sim_destroy(sim)

