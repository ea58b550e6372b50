"""Parity of every named kernel, through the C ABI, with the CPU checker
(oracle/restate.c, pinned bit for bit to the reference) on the same seeded
inputs. Index, copy and integer results must be identical; entry points the
header marks bit-exact must give the reference's bits; the rest must agree
within rtol = atol = 1e-4."""

import json
import struct

import numpy as np
import pytest
import torch

from accelep_b200 import kernels as K
from accelep_b200 import synthetic as syn
from tests.conftest import GOLDEN

pytestmark = pytest.mark.gpu

RTOL = ATOL = 1e-4


def T(a, dtype=torch.float32):
    return torch.as_tensor(np.ascontiguousarray(a)).to(device="cuda", dtype=dtype)


def H(t):
    torch.cuda.synchronize()
    return t.detach().cpu().numpy()


def same_bits(a, b):
    a = np.ascontiguousarray(a, dtype=np.float32)
    b = np.ascontiguousarray(b, dtype=np.float32)
    return a.shape == b.shape and np.array_equal(a.view(np.uint32), b.view(np.uint32))


def close(got, want, rtol=RTOL, atol=ATOL):
    np.testing.assert_allclose(got, want, rtol=rtol, atol=atol)


@pytest.fixture(scope="module")
def kats():
    return json.loads((GOLDEN / "kats.json").read_text())


@pytest.fixture(scope="module")
def small():
    return np.load(GOLDEN / "ref_small.npz")


def test_embed(lib, cuda, orc, kats):
    k = kats["embed"]
    table = T(np.array(k["table"], np.float32))
    out = K.embed(T(np.array(k["ids"], np.int32), torch.int32), table, 2)
    assert H(out).reshape(-1).tolist() == k["want"]
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    K.embed(T(np.array([k["bad_id"]], np.int32), torch.int32), table, 1, status=status)
    assert int(H(status)[0]) & 1
    rng = np.random.default_rng(1)
    tab = rng.standard_normal((1000, 576), dtype=np.float32)
    ids = rng.integers(0, 1000, 37).astype(np.int32)
    got = H(K.embed(T(ids, torch.int32), T(tab), 30, id_offset=7))
    assert np.array_equal(got, orc.embed(ids, 7, tab, 30))


def test_rmsnorm(lib, cuda, orc, small, kats):
    y = H(K.rmsnorm(T(small["rms_x"]), T(small["rms_w"]), 7, 576, 1e-5))
    close(y, small["rms_y"], rtol=1e-6, atol=1e-6)
    y_off = H(K.rmsnorm(T(small["rms_x"]), T(small["rms_w"]), 2, 576, 1e-5, row_offset=5))
    close(y_off, small["rms_y_off"], rtol=1e-6, atol=1e-6)
    # The double sum differs from the reference's only in association.
    assert np.mean(y.view(np.uint32) == small["rms_y"].view(np.uint32)) > 0.99
    k = kats["rmsnorm"]
    x = np.array(k["x"], np.float32).reshape(2, 4)
    got = H(K.rmsnorm(T(x), T(np.array(k["weight"], np.float32)), 1, 4, k["eps"], row_offset=1))
    close(got, orc.rmsnorm(x, k["weight"], 1, 4, k["eps"], 1), rtol=0, atol=k["tol"])


def test_rope_bit_exact(lib, cuda, small, kats):
    st = T(small["rope_in"])
    K.rope(st, T(small["rope_cos"]), T(small["rope_sin"]), 3, 9, 64, 11)
    assert same_bits(H(st), small["rope_out"])
    r = kats["rope"]
    st = T(np.array(r["in"], np.float32))
    K.rope(st, T(np.array(r["cos"], np.float32)), T(np.array(r["sin"], np.float32)), 1, 1, 4, r["position"])
    assert H(st).tolist() == r["want"]


def test_append_cache(lib, cuda, kats):
    c = kats["cache"]
    cache = T(np.full(8, c["fill"], np.float32))
    K.append_cache(T(np.array(c["src"], np.float32)), cache, c["seq"], c["position"], c["n_heads"], c["head_dim"])
    assert H(cache).tolist() == c["want"]


@pytest.mark.parametrize("tag", ["at1", "at2", "at3", "at4"])
def test_attention_golden(lib, cuda, small, tag):
    seq, pos, heads, kvh, hd = (int(v) for v in small[tag + "_dims"])
    got = H(K.attention(T(small[tag + "_q"]), T(small[tag + "_k"]), T(small[tag + "_v"]), seq, pos, heads, kvh, hd))
    close(got, small[tag + "_out"])


def test_attention_kat_and_shapes(lib, cuda, orc, kats):
    a = kats["attention"]
    got = H(K.attention(T(np.full(1, a["q"], np.float32)), T(np.full(1, a["k"], np.float32)),
                        T(np.full(1, a["v"], np.float32)), 1, 0, 1, 1, 1))
    assert float(got.reshape(-1)[0]) == a["want"]
    rng = np.random.default_rng(3)
    for seq, pos, heads, kvh, hd in [(3, 1200, 9, 3, 64), (1, 0, 2, 2, 8), (6, 17, 8, 1, 128), (2, 5, 4, 2, 5)]:
        q = rng.standard_normal((seq, heads, hd), dtype=np.float32)
        k = rng.standard_normal((pos + seq, kvh, hd), dtype=np.float32)
        v = rng.standard_normal((pos + seq, kvh, hd), dtype=np.float32)
        got = H(K.attention(T(q), T(k), T(v), seq, pos, heads, kvh, hd))
        close(got, orc.attend(q, k, v, seq, pos, heads, kvh, hd))


def test_attention_decode_split(lib, cuda, orc):
    """Split-KV decode over ragged lengths, including a length that is a
    chunk multiple, one row, and the full context."""
    rng = np.random.default_rng(4)
    batch, heads, kvh, hd, max_len = 5, 9, 3, 64, 1100
    lens = np.array([1, 256, 700, 1100, 513], np.int32)
    kc = rng.standard_normal((batch, max_len, kvh, hd), dtype=np.float32)
    vc = rng.standard_normal((batch, max_len, kvh, hd), dtype=np.float32)
    q = rng.standard_normal((batch, heads * hd), dtype=np.float32)
    got = H(K.attention_decode(T(q), T(kc), T(vc), T(lens, torch.int32), heads, kvh, hd, max_len))
    # The engine's head-major layout, one row per bulk copy vs one per chunk.
    hm = H(K.attention_decode(T(q), T(kc.transpose(0, 2, 1, 3)), T(vc.transpose(0, 2, 1, 3)), T(lens, torch.int32),
                              heads, kvh, hd, max_len, head_major=True))
    ws = K.attention_decode_workspace(batch, heads, kvh, max_len)
    for _ in range(2):  # a reused workspace: the arrival counters return to zero
        again = H(K.attention_decode(T(q), T(kc), T(vc), T(lens, torch.int32), heads, kvh, hd, max_len, workspace=ws))
        assert np.array_equal(again, got)
    assert not H(ws[:batch * kvh * 4]).any()
    for b in range(batch):
        n = int(lens[b])
        want = orc.attend(q[b].reshape(1, heads, hd), kc[b, :n], vc[b, :n], 1, n - 1, heads, kvh, hd)
        close(got[b], want.reshape(-1))
        close(hm[b], want.reshape(-1))


def test_silu_add(lib, cuda, small, kats):
    g = T(small["silu_gate"])
    K.silu_mul(g, T(small["silu_up"]))
    close(H(g), small["silu_out"], rtol=1e-6, atol=1e-6)
    d = T(np.array(kats["add"]["dest"], np.float32))
    K.residual_add(d, T(np.array(kats["add"]["extra"], np.float32)))
    assert H(d).tolist() == kats["add"]["want"]
    rng = np.random.default_rng(5)
    a = rng.standard_normal(100003, dtype=np.float32)
    b = rng.standard_normal(100003, dtype=np.float32)
    d = T(a)
    K.residual_add(d, T(b))
    assert same_bits(H(d), a + b)


def test_sample_kats(lib, cuda, kats):
    for case in kats["sample"]:
        lg = T(np.array(case["logits"], np.float32))
        state = T(np.array([case["rng"]], np.uint32).view(np.int32), torch.int32)
        got = H(K.sample(lg, len(case["logits"]), case["temperature"], state, case["top_k"]))
        assert int(got[0]) == case["want"], case
        if case["want_rng"] is not None:
            assert int(H(state).view(np.uint32)[0]) == case["want_rng"]


def test_sample_golden(lib, cuda, small):
    logits = T(small["smp_logits"])
    mismatched = 0
    for seed, temp_milli, k, want, want_state in small["smp_rows"]:
        state = T(np.array([seed], np.uint32).view(np.int32), torch.int32)
        got = int(H(K.sample(logits, logits.numel(), temp_milli / 1000.0, state, int(k)))[0])
        if temp_milli == 0 or (0 < k < 4096):
            # Greedy and top-k walk their table in the reference's exact order.
            assert got == int(want), (seed, temp_milli, k)
        else:
            mismatched += got != int(want)
        assert int(H(state).view(np.uint32)[0]) == int(want_state)
    # The full-vocabulary walk sums 4096 doubles in another order; a flip needs
    # the draw within a few ulps of a boundary.
    assert mismatched == 0


def test_argmax_ties_nan(lib, cuda, orc):
    rng = np.random.default_rng(6)
    rows = rng.standard_normal((8, 49152), dtype=np.float32)
    rows[1, 100] = rows[1, 40000] = 9.0  # tie: the earlier id wins
    rows[2, :] = -np.inf
    rows[3, 5] = np.nan  # NaN never wins
    rows[3, 7] = 50.0
    rows[4, 0] = np.nan  # NaN at id 0 pins the answer to 0
    rows[5, 49151] = 1e30
    got = H(K.argmax_rows(T(rows)))
    for r in range(8):
        assert int(got[r]) == orc.sample(rows[r], 49152, 0.0, 1, 0)[0], r


def test_matmul_exact_bits(lib, cuda, small, kats):
    for m, k, n in [(128, 160, 96), (13, 19, 17), (3, 70, 33)]:
        t = f"mm_{m}_{k}_{n}"
        assert same_bits(H(K.matmul_exact(T(small[t + "_a"]), T(small[t + "_b"]))), small[t + "_c"]), t
    sp = kats["split_product"]
    a = np.array([struct.unpack("<f", struct.pack("<I", u))[0] for u in sp["a_bits"]], np.float32).reshape(1, 2)
    b = np.array([struct.unpack("<f", struct.pack("<I", u))[0] for u in sp["b_bits"]], np.float32).reshape(2, 1)
    out = H(K.matmul_exact(T(a), T(b)))
    assert struct.unpack("<I", struct.pack("<f", float(out[0, 0])))[0] == sp["want_bits"]
    z = H(K.matmul_exact(T(np.zeros((1, 0), np.float32)), T(np.zeros((0, 1), np.float32))))
    assert z.tolist() == [[0.0]]


def test_transpose_epilogue(lib, cuda, orc, small):
    rng = np.random.default_rng(7)
    x = rng.standard_normal((77, 131), dtype=np.float32)
    assert np.array_equal(H(K.transpose(T(x))), x.T)
    shapes = [((10,), 1.5, 0.5, "none"), ((6, 1), 1.0, 1.0, "relu"), ((1, 10), -0.75, 2.0, "gelu"),
              ((6, 10), 1.0, 1.0, "gelu"), ((), 1.0, 0.0, "relu"), ((1,), 2.0, 1.0, "none")]
    for i, (shape, alpha, beta, act) in enumerate(shapes):
        got = H(K.gemm_epilogue(T(small["ep_c"]), alpha, T(small[f"ep{i}_bias"]), list(shape), beta, act))
        close(got, small[f"ep{i}_out"], rtol=1e-6, atol=1e-6)
        if act != "gelu":
            assert same_bits(got, small[f"ep{i}_out"]), i
    inf = T(np.array([[np.inf, -np.inf, 0.0]], np.float32) * np.array([[0.0, 1.0, 1.0]], np.float32))
    got = H(K.gemm_epilogue(inf, 1.0, None, [], 0.0, "relu"))
    assert np.isnan(got[0, 0]) and got.view(np.uint32)[0, 1] == 0
    neg = H(K.gemm_epilogue(T(np.zeros((1, 1), np.float32)), -1.0, None, [], 0.0, "relu"))
    assert neg.view(np.uint32)[0, 0] == 0x80000000
