"""The drop-in seam: every accel::Device call of the B200 device
(include/accel/device.h:69-125 of the reference, plus the added MatMulQ8),
driven through its virtual interface by tests/device_shim.cc and compared
with the CPU checker's routine of the same name: bit for bit where the kernel
keeps the reference's arithmetic (MatMul, Transpose, non-Gelu epilogue,
Embedding, Rope, AppendCache, ResidualAdd, SampleToken), within tolerance
otherwise. Also the Device's error behaviour (exception types of
src/sim_device.cc:44-161: range checks, unknown frees, the embedding id
check) and that every allocation is freed."""

import ctypes
import subprocess
from pathlib import Path

import numpy as np
import pytest

from accelep_b200 import synthetic as syn
from tests.conftest import GOLDEN, ROOT

pytestmark = pytest.mark.gpu

BUILD = ROOT / "tests" / "_build"
SHIM = BUILD / "libdevice_shim.so"
LIB_DIR = ROOT / "accelep_b200" / "lib"
INVALID, OVERFLOW, LOGIC, BAD_ALLOC, RUNTIME = 1, 2, 3, 4, 5


def _shim():
    src = ROOT / "tests" / "device_shim.cc"
    lib = LIB_DIR / "libaccelep_b200.so"
    BUILD.mkdir(exist_ok=True)
    if not SHIM.is_file() or SHIM.stat().st_mtime < max(src.stat().st_mtime, lib.stat().st_mtime):
        subprocess.run(["g++", "-std=c++17", "-O2", "-shared", "-fPIC", f"-I{ROOT / 'include'}", str(src),
                        f"-L{LIB_DIR}", "-laccelep_b200", f"-Wl,-rpath,{LIB_DIR}", "-o", str(SHIM)], check=True)
    s = ctypes.CDLL(str(SHIM))
    vp, i32, i64, f32 = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64, ctypes.c_float
    pi64 = ctypes.POINTER(ctypes.c_int64)
    s.shim_create.restype = vp
    s.shim_destroy.argtypes = [vp]
    s.shim_error.restype = ctypes.c_char_p
    s.shim_name.argtypes, s.shim_name.restype = [vp], ctypes.c_char_p
    s.shim_live.restype = i64
    s.shim_alloc.argtypes = [vp, i64, ctypes.POINTER(ctypes.c_int)]
    s.shim_forged.argtypes = [vp, i64, ctypes.POINTER(ctypes.c_int)]
    s.shim_id.argtypes, s.shim_id.restype = [vp, ctypes.c_int], ctypes.c_uint64
    s.shim_free.argtypes = [vp, ctypes.c_int]
    s.shim_h2d.argtypes = [vp, ctypes.c_int, vp, i64]
    s.shim_d2h.argtypes = [vp, vp, ctypes.c_int, i64]
    s.shim_matmul.argtypes = [vp, ctypes.c_int, ctypes.c_int, ctypes.c_int, i64, i64, i64]
    s.shim_transpose.argtypes = [vp, ctypes.c_int, ctypes.c_int, i64, i64]
    s.shim_gemm_epilogue.argtypes = [vp, ctypes.c_int, i64, i64, f32, ctypes.c_int, pi64, ctypes.c_int, f32,
                                     ctypes.c_int]
    s.shim_embedding.argtypes = [vp, ctypes.c_int, i64, ctypes.c_int, ctypes.c_int, i64, i64, i64]
    s.shim_rmsnorm.argtypes = [vp, ctypes.c_int, ctypes.c_int, ctypes.c_int, i64, i64, f32, i64]
    s.shim_rope.argtypes = [vp, ctypes.c_int, ctypes.c_int, ctypes.c_int, i64, i64, i64, i64]
    s.shim_append_cache.argtypes = [vp, ctypes.c_int, ctypes.c_int, i64, i64, i64, i64]
    s.shim_attention.argtypes = [vp] + [ctypes.c_int] * 5 + [i64] * 5
    s.shim_silu_mul.argtypes = [vp, ctypes.c_int, ctypes.c_int, i64]
    s.shim_residual_add.argtypes = [vp, ctypes.c_int, ctypes.c_int, i64]
    s.shim_sample_token.argtypes = [vp, ctypes.c_int, ctypes.c_int, i64, i64, f32, ctypes.POINTER(ctypes.c_uint32),
                                    ctypes.c_int]
    s.shim_matmul_q8.argtypes = [vp, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, pi64, ctypes.c_int, i64,
                                 i64, ctypes.c_int, i64, i64, i64]
    return s


class Dev:
    def __init__(self, shim):
        self.s = shim
        self.h = shim.shim_create()
        assert self.h, shim.shim_error().decode()
        self.handles = []

    def ok(self, rc):
        assert rc == 0, self.s.shim_error().decode()

    def put(self, array):
        a = np.ascontiguousarray(array)
        h = ctypes.c_int()
        self.ok(self.s.shim_alloc(self.h, max(a.nbytes, 1), ctypes.byref(h)))
        if a.nbytes:
            self.ok(self.s.shim_h2d(self.h, h.value, a.ctypes.data, a.nbytes))
        self.handles.append(h.value)
        return h.value

    def get(self, h, like):
        out = np.empty_like(like)
        self.ok(self.s.shim_d2h(self.h, out.ctypes.data, h, out.nbytes))
        return out

    def close(self):
        for h in self.handles:
            self.ok(self.s.shim_free(self.h, h))
        self.s.shim_destroy(self.h)


@pytest.fixture
def dev(cuda):
    shim = _shim()
    live0 = shim.shim_live()
    d = Dev(shim)
    yield d
    d.close()
    assert shim.shim_live() == live0  # every allocation of the test was freed


def _kats():
    import json

    return json.loads((GOLDEN / "kats.json").read_text())


def test_name_and_matmul_bits(dev, orc):
    assert dev.s.shim_name(dev.h) == b"b200"
    rng = np.random.default_rng(1)
    a = rng.standard_normal((13, 19), dtype=np.float32)
    b = rng.standard_normal((19, 17), dtype=np.float32)
    c = np.zeros((13, 17), np.float32)
    ha, hb, hc = dev.put(a), dev.put(b), dev.put(c)
    dev.ok(dev.s.shim_matmul(dev.h, ha, hb, hc, 13, 19, 17))
    assert np.array_equal(dev.get(hc, c), orc.matmul(a, b))  # PackedMatMul's rounding, bit for bit
    t = np.zeros((17, 13), np.float32)
    ht = dev.put(t)
    dev.ok(dev.s.shim_transpose(dev.h, hc, ht, 13, 17))
    assert np.array_equal(dev.get(ht, t), orc.transpose(orc.matmul(a, b)))


@pytest.mark.parametrize("act,bias_shape", [("none", [17]), ("relu", [13, 1]), ("gelu", [1, 17]), ("relu", [1])])
def test_gemm_epilogue(dev, orc, act, bias_shape):
    rng = np.random.default_rng(len(bias_shape) + len(act))
    c = rng.standard_normal((13, 17), dtype=np.float32)
    bias = rng.standard_normal(int(np.prod(bias_shape)), dtype=np.float32)
    hc, hb = dev.put(c), dev.put(bias)
    shape = (ctypes.c_int64 * len(bias_shape))(*bias_shape)
    code = {"none": 0, "relu": 1, "gelu": 2}[act]
    dev.ok(dev.s.shim_gemm_epilogue(dev.h, hc, 13, 17, 0.5, hb, shape, len(bias_shape), 2.0, code))
    want = orc.gemm_epilogue(c, 0.5, bias, bias_shape, 2.0, act)
    got = dev.get(hc, c)
    if act == "gelu":
        np.testing.assert_allclose(got, want, rtol=1e-6, atol=1e-6)
    else:
        assert np.array_equal(got, want)


def test_row_calls_against_kats(dev, orc):
    k = _kats()
    # Embedding (test_sim_kernels.cc's table and ids; an id past the vocabulary throws)
    e = k["embed"]
    table = np.array(e["table"], np.float32)
    ids = np.array(e["ids"], np.int32)
    out = np.zeros((len(ids), table.shape[1]), np.float32)
    hi, ht, ho = dev.put(ids), dev.put(table), dev.put(out)
    dev.ok(dev.s.shim_embedding(dev.h, hi, 0, ht, ho, len(ids), table.shape[1], table.shape[0]))
    assert dev.get(ho, out).reshape(-1).tolist() == e["want"]
    bad = dev.put(np.array([e["bad_id"]], np.int32))
    assert dev.s.shim_embedding(dev.h, bad, 0, ht, ho, 1, table.shape[1], table.shape[0]) == INVALID
    # RmsNorm (the reference's test bound: 1e-6)
    r = k["rmsnorm"]
    x = np.array(r["x"], np.float32).reshape(2, 4)
    w = np.array(r["weight"], np.float32)
    y = np.zeros_like(x)
    hx, hw, hy = dev.put(x), dev.put(w), dev.put(y)
    dev.ok(dev.s.shim_rmsnorm(dev.h, hx, hw, hy, 2, 4, r["eps"], 0))
    np.testing.assert_allclose(dev.get(hy, y), orc.rmsnorm(x, w, 2, 4, r["eps"]), rtol=0, atol=r["tol"])


def test_llama_row_calls(dev, orc):
    """Embedding, RmsNorm, Rope, AppendCache, Attention, SiluMul and
    ResidualAdd on SmolLM2-shaped rows (3 new rows at position 11)."""
    rng = np.random.default_rng(5)
    vocab, hidden, heads, kvh, hd, ctx = 300, 576, 9, 3, 64, 16
    seq, pos = 3, 11
    table = rng.standard_normal((vocab, hidden), dtype=np.float32)
    ids = np.array([5, 299, 0, 17], np.int32)
    emb = np.zeros((seq, hidden), np.float32)
    hi, ht, he = dev.put(ids), dev.put(table), dev.put(emb)
    dev.ok(dev.s.shim_embedding(dev.h, hi, 1, ht, he, seq, hidden, vocab))
    assert np.array_equal(dev.get(he, emb), orc.embed(ids, 1, table, seq))

    w = rng.uniform(0.5, 1.5, hidden).astype(np.float32)
    normed = np.zeros((1, hidden), np.float32)
    hw, hn = dev.put(w), dev.put(normed)
    dev.ok(dev.s.shim_rmsnorm(dev.h, he, hw, hn, 1, hidden, 1e-5, seq - 1))  # the final-norm row offset
    np.testing.assert_allclose(dev.get(hn, normed), orc.rmsnorm(table[ids[1:4]], w, 1, hidden, 1e-5, seq - 1),
                               rtol=1e-6, atol=1e-6)

    ang = np.outer(np.arange(ctx), 1.0 / 1e5 ** (np.arange(0, hd, 2) / hd))
    cos_t = np.cos(np.concatenate([ang, ang], 1)).astype(np.float32)
    sin_t = np.sin(np.concatenate([ang, ang], 1)).astype(np.float32)
    q = rng.standard_normal((seq, heads, hd), dtype=np.float32)
    hq, hcos, hsin = dev.put(q), dev.put(cos_t), dev.put(sin_t)
    dev.ok(dev.s.shim_rope(dev.h, hq, hcos, hsin, seq, heads, hd, pos))
    q_roped = orc.rope(q, cos_t, sin_t, seq, heads, hd, pos)
    assert np.array_equal(dev.get(hq, q), q_roped)

    kc = rng.standard_normal((ctx, kvh, hd), dtype=np.float32)
    vc = rng.standard_normal((ctx, kvh, hd), dtype=np.float32)
    knew = rng.standard_normal((seq, kvh, hd), dtype=np.float32)
    vnew = rng.standard_normal((seq, kvh, hd), dtype=np.float32)
    hk, hv, hkn, hvn = dev.put(kc), dev.put(vc), dev.put(knew), dev.put(vnew)
    dev.ok(dev.s.shim_append_cache(dev.h, hkn, hk, seq, pos, kvh, hd))
    dev.ok(dev.s.shim_append_cache(dev.h, hvn, hv, seq, pos, kvh, hd))
    k_all = orc.append_cache(knew, kc, seq, pos, kvh, hd)
    v_all = orc.append_cache(vnew, vc, seq, pos, kvh, hd)
    assert np.array_equal(dev.get(hk, kc), k_all)
    assert np.array_equal(dev.get(hv, vc), v_all)

    scores = np.zeros(ctx, np.float32)
    out = np.zeros((seq, heads, hd), np.float32)
    hs, ho = dev.put(scores), dev.put(out)
    dev.ok(dev.s.shim_attention(dev.h, hq, hk, hv, hs, ho, seq, pos, heads, kvh, hd))
    want = orc.attend(q_roped, k_all[:pos + seq], v_all[:pos + seq], seq, pos, heads, kvh, hd)
    np.testing.assert_allclose(dev.get(ho, out), want, rtol=1e-4, atol=1e-4)

    gate = rng.standard_normal(1536, dtype=np.float32) * 3
    up = rng.standard_normal(1536, dtype=np.float32)
    hg, hu = dev.put(gate), dev.put(up)
    dev.ok(dev.s.shim_silu_mul(dev.h, hg, hu, 1536))
    np.testing.assert_allclose(dev.get(hg, gate), orc.silu_mul(gate, up), rtol=1e-6, atol=1e-7)
    dest = rng.standard_normal(hidden, dtype=np.float32)
    extra = rng.standard_normal(hidden, dtype=np.float32)
    hd_, hx = dev.put(dest), dev.put(extra)
    dev.ok(dev.s.shim_residual_add(dev.h, hd_, hx, hidden))
    assert np.array_equal(dev.get(hd_, dest), orc.add(dest, extra))


def test_sample_token(dev, orc):
    k = _kats()
    for case in k["sample"]:
        logits = np.array(case["logits"], np.float32)
        chosen = np.full(2, -1, np.int32)
        hl, hc = dev.put(logits), dev.put(chosen)
        rng = ctypes.c_uint32(case["rng"])
        dev.ok(dev.s.shim_sample_token(dev.h, hl, hc, 1, logits.size, case["temperature"], ctypes.byref(rng),
                                       case["top_k"]))
        got = dev.get(hc, chosen)
        want, want_rng = orc.sample(logits, logits.size, case["temperature"], case["rng"], case["top_k"])
        assert int(got[1]) == case["want"] == want and got[0] == -1
        assert rng.value == want_rng


@pytest.mark.parametrize("m,k,n,axis", [(64, 576, 1536, 1), (1, 4096, 512, 1), (32, 576, 960, 1), (7, 64, 48, -1)])
def test_matmul_q8(dev, orc, m, k, n, axis):
    """Device::MatMulQ8 (the entry runtime.cc:326 calls) against the
    reference's MatMulQuantized: GEMV, tensor-core and CUDA-core shapes."""
    x, w, s = syn.int8_gemm(m, k, n, m + k)
    if axis < 0:
        s = s[:1].copy()
    c = np.zeros((m, n), np.float32)
    hx, hq, hs, hc = dev.put(x), dev.put(w), dev.put(s), dev.put(c)
    shape = (ctypes.c_int64 * 2)(k, n)
    dev.ok(dev.s.shim_matmul_q8(dev.h, hx, hq, hs, -1, shape, 2, axis, 0, hc, m, k, n))
    want = orc.matmul_quantized(x, w, s, None, [k, n], axis, 0, m, k, n)
    mag = np.abs(x).astype(np.float64) @ (np.abs(w.astype(np.float64)) * (s if axis > 0 else s[0]))
    tol = np.maximum(1e-4 + 1e-4 * np.abs(want), 2 * k * np.finfo(np.float32).eps * mag)
    assert (np.abs(dev.get(hc, c) - want) <= tol).all()


def test_errors_keep_reference_types(dev):
    s, h = dev.s, dev.h
    a = dev.put(np.zeros((2, 3), np.float32))
    b = dev.put(np.zeros((3, 4), np.float32))
    c = dev.put(np.zeros((2, 4), np.float32))
    assert s.shim_matmul(h, a, b, c, 2, 3, 5) == INVALID  # C too small
    assert b"out of range" in s.shim_error()
    assert s.shim_matmul(h, a, b, c, -1, 3, 4) == INVALID
    forged = ctypes.c_int()
    s.shim_forged(h, 64, ctypes.byref(forged))
    assert s.shim_free(h, forged.value) == LOGIC  # a buffer this device never allocated
    huge = ctypes.c_int()
    assert s.shim_alloc(h, 1 << 50, ctypes.byref(huge)) == BAD_ALLOC
    # Embedding ids outside the vocabulary: the device reports it, like SimEmbed's throw.
    ids = dev.put(np.array([0, 7], np.int32))
    table = dev.put(np.zeros((4, 8), np.float32))
    out = dev.put(np.zeros((2, 8), np.float32))
    assert s.shim_embedding(h, ids, 0, table, out, 2, 8, 4) == INVALID
    # The device still works afterwards.
    assert s.shim_matmul(h, a, b, c, 2, 3, 4) == 0
