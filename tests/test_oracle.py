"""Pins the CPU checker (oracle/restate.c) before any GPU result is compared
with it: against the known answers of the reference's own tests, against the
reference's outputs stored in tests/golden, and, where oracle/_ref is built,
against the reference itself on fresh inputs. All bit-exact."""

import json
import struct

import numpy as np
import pytest

from accelep_b200 import synthetic as syn
from tests.conftest import GOLDEN


def bits(x):
    return struct.unpack("<I", struct.pack("<f", float(x)))[0]


def fbits(u):
    return struct.unpack("<f", struct.pack("<I", u))[0]


@pytest.fixture(scope="module")
def kats():
    return json.loads((GOLDEN / "kats.json").read_text())


@pytest.fixture(scope="module")
def small():
    return np.load(GOLDEN / "ref_small.npz")


def same_bits(a, b):
    a = np.ascontiguousarray(a, dtype=np.float32)
    b = np.ascontiguousarray(b, dtype=np.float32)
    return a.shape == b.shape and np.array_equal(a.view(np.uint32), b.view(np.uint32))


# ------------------------------------------------ known answers (reference tests)

def test_embed_kat(orc, kats):
    k = kats["embed"]
    out = orc.embed(k["ids"], 0, np.array(k["table"], np.float32), 2)
    assert out.reshape(-1).tolist() == k["want"]
    with pytest.raises(ValueError):
        orc.embed([k["bad_id"]], 0, np.array(k["table"], np.float32), 1)


def test_rmsnorm_kat(orc, kats):
    k = kats["rmsnorm"]
    x = np.array(k["x"], np.float32).reshape(2, 4)
    w = np.array(k["weight"], np.float32)
    for off in (0, 1):
        y = orc.rmsnorm(x, w, 1, 4, k["eps"], off)[0]
        row = x[off].astype(np.float64)
        inv = 1.0 / np.sqrt(np.sum(row * row) / 4 + np.float64(np.float32(k["eps"])))
        assert np.max(np.abs(y - row * inv * w.astype(np.float64))) <= k["tol"]


def test_rope_cache_attention_silu_add_kats(orc, kats):
    r = kats["rope"]
    assert orc.rope(np.array(r["in"], np.float32), r["cos"], r["sin"], 1, 1, 4, r["position"]).tolist() == r["want"]
    keep = orc.rope(np.array([8, -1, 0.5, 4], np.float32), [1] * 4, [0] * 4, 1, 1, 4, 0)
    assert keep.tolist() == [8, -1, 0.5, 4]
    c = kats["cache"]
    got = orc.append_cache(np.array(c["src"], np.float32), np.full(8, c["fill"], np.float32), c["seq"], c["position"],
                           c["n_heads"], c["head_dim"])
    assert got.tolist() == c["want"]
    a = kats["attention"]
    out = orc.attend(np.full(1, a["q"], np.float32), np.full(1, a["k"], np.float32), np.full(1, a["v"], np.float32),
                     1, 0, 1, 1, 1)
    assert float(out.reshape(-1)[0]) == a["want"]
    assert float(orc.silu_mul([kats["silu"]["gate"]], [kats["silu"]["up"]])[0]) == 0.0
    assert orc.add(kats["add"]["dest"], kats["add"]["extra"]).tolist() == kats["add"]["want"]


def test_sample_kats(orc, kats):
    for case in kats["sample"]:
        got, state = orc.sample(case["logits"], len(case["logits"]), case["temperature"], case["rng"], case["top_k"])
        assert got == case["want"], case
        if case["want_rng"] is not None:
            assert state == case["want_rng"]


def test_split_product_bits(orc, kats):
    k = kats["split_product"]
    a = np.array([fbits(u) for u in k["a_bits"]], np.float32).reshape(1, 2)
    b = np.array([fbits(u) for u in k["b_bits"]], np.float32).reshape(2, 1)
    assert bits(orc.matmul(a, b)[0, 0]) == k["want_bits"]


def test_dequantize_kat(orc, kats):
    k = kats["dequantize"]
    got = orc.execute_matmul_q(np.array(k["x"], np.float32), np.array(k["w"], np.int8), np.array(k["scale"], np.float32),
                               np.array(k["zero"], np.int8), axis=k["axis"])
    assert float(got[0, 0]) == k["want00"]
    assert got.tolist() == k["want"]


def test_nonfinite_epilogue(orc):
    e1 = orc.gemm_epilogue(orc.matmul([[np.inf]], [[0.0]]), 1.0, None, [], 0.0, "relu")
    e2 = orc.gemm_epilogue(orc.matmul([[-np.inf]], [[1.0]]), 1.0, None, [], 0.0, "relu")
    e3 = orc.gemm_epilogue(orc.matmul([[0.0]], [[1.0]]), -1.0, None, [], 0.0, "relu")
    assert np.isnan(e1[0, 0]) and bits(e2[0, 0]) == 0 and bits(e3[0, 0]) == 0x80000000


# ------------------------------------------------ reference outputs (golden)

def test_matmul_golden(orc, small):
    for m, k, n in [(128, 160, 96), (13, 19, 17), (3, 70, 33)]:
        t = f"mm_{m}_{k}_{n}"
        assert same_bits(orc.matmul(small[t + "_a"], small[t + "_b"]), small[t + "_c"]), t
    from tests.golden.make_golden import gemv_inputs

    a, b = gemv_inputs()
    assert same_bits(orc.matmul(a, b), small["mm_gemv_c"])


def test_quantized_golden(orc, small):
    for tag in ("q1", "q2", "q3"):
        a, q = small[tag + "_a"], small[tag + "_q"]
        m, k = a.shape
        n = q.shape[1]
        got = orc.matmul_quantized(a, q, small[tag + "_col"], None, [k, n], 1, 0, m, k, n)
        assert same_bits(got, small[tag + "_c_col"]), tag
        got = orc.matmul_quantized(a, q, small[tag + "_row"], small[tag + "_zero"], [k, n], 0, 0, m, k, n)
        assert same_bits(got, small[tag + "_c_row"]), tag
        got = orc.matmul_quantized(a, q, np.array([0.5], np.float32), None, [k, n], -1, 0, m, k, n)
        assert same_bits(got, small[tag + "_c_scalar"]), tag


def test_epilogue_golden(orc, small):
    shapes = [((10,), 1.5, 0.5, "none"), ((6, 1), 1.0, 1.0, "relu"), ((1, 10), -0.75, 2.0, "gelu"),
              ((6, 10), 1.0, 1.0, "gelu"), ((), 1.0, 0.0, "relu"), ((1,), 2.0, 1.0, "none")]
    for i, (shape, alpha, beta, act) in enumerate(shapes):
        got = orc.gemm_epilogue(small["ep_c"], alpha, small[f"ep{i}_bias"], list(shape), beta, act)
        assert same_bits(got, small[f"ep{i}_out"]), i


def test_rows_golden(orc, small):
    assert same_bits(orc.rmsnorm(small["rms_x"], small["rms_w"], 7, 576, 1e-5, 0), small["rms_y"])
    assert same_bits(orc.rmsnorm(small["rms_x"], small["rms_w"], 2, 576, 1e-5, 5), small["rms_y_off"])
    assert same_bits(orc.rope(small["rope_in"], small["rope_cos"], small["rope_sin"], 3, 9, 64, 11), small["rope_out"])
    assert same_bits(orc.silu_mul(small["silu_gate"], small["silu_up"]), small["silu_out"])


def test_attention_golden(orc, small):
    for tag in ("at1", "at2", "at3", "at4"):
        seq, pos, heads, kvh, hd = (int(v) for v in small[tag + "_dims"])
        got = orc.attend(small[tag + "_q"], small[tag + "_k"], small[tag + "_v"], seq, pos, heads, kvh, hd)
        assert same_bits(got, small[tag + "_out"]), tag


def test_sample_golden(orc, small):
    logits = small["smp_logits"]
    for seed, temp_milli, k, want, want_state in small["smp_rows"]:
        got, state = orc.sample(logits, logits.size, temp_milli / 1000.0, int(seed), int(k))
        assert (got, state) == (int(want), int(want_state)), (seed, temp_milli, k)


def test_c1_c2_golden(orc, small):
    import hashlib

    x, w, s = syn.int8_gemm(64, 576, 1536, 1)
    c1 = orc.execute_matmul_q(x, w, s, act="relu")
    assert hashlib.sha256(c1.tobytes()).digest() == bytes(small["c1_sha"])
    assert same_bits(c1[0], small["c1_row0"])
    x, blocks = syn.mlp_stack()
    h = x[:16]
    for w1, s1, w2, s2, gamma in blocks:
        h, _ = orc.mlp_block(h, w1, s1, w2, s2, gamma, 1e-5)
    assert same_bits(h, small["c2_rows16"])


def test_tiny_llama_golden(orc, small):
    from oracle.oracle import LlamaHandle

    cfg = syn.TINY_LLAMA
    model = LlamaHandle(orc, cfg)
    model.load(syn.llama_weights(cfg, 5))
    p = small["tiny_prompt"]
    assert np.array_equal(model.generate(p, 40), small["tiny_greedy"])
    assert np.array_equal(model.generate(p, 40, temperature=0.8, seed=3, top_k=10), small["tiny_sampled"])
    assert np.array_equal(model.generate(p, 40, temperature=1.1, seed=9, top_k=0), small["tiny_full"])


def test_c3_prefix_golden(orc):
    """First 8 greedy ids and the prefill logit row of C3 (fp32 SmolLM2-135M
    shape) match the reference's."""
    from oracle.oracle import LlamaHandle

    g = np.load(GOLDEN / "c3_smollm.npz")
    cfg = dict(syn.SMOLLM2_135M, context=128)
    model = LlamaHandle(orc, cfg)
    model.load(syn.llama_weights(cfg, 3))
    assert np.array_equal(g["prompt"], syn.prompts(cfg, 1, 4, 11)[0])
    model.forward_ids(g["prompt"], True)
    assert same_bits(model.logits(), g["prefill_logits"])
    ids = model.generate(g["prompt"], 8)
    assert np.array_equal(ids, g["ids"][:8])


# ------------------------------------------------ the reference itself

def test_restatement_matches_reference_fresh(orc, ref):
    rng = np.random.default_rng(99)
    for m, k, n in [(5, 33, 70), (1, 257, 129)]:
        a = rng.standard_normal((m, k), dtype=np.float32)
        b = rng.standard_normal((k, n), dtype=np.float32)
        assert same_bits(orc.matmul(a, b), ref.matmul(a, b))
    x, w, s = syn.int8_gemm(9, 100, 77, 5)
    assert same_bits(orc.execute_matmul_q(x, w, s, act="gelu"), ref.execute_matmul_q(x, w, s, act="gelu"))
    res = rng.standard_normal((9, 77), dtype=np.float32)
    assert same_bits(orc.execute_matmul_q(x, w, s, act="relu", residual=res),
                     ref.execute_matmul_q(x, w, s, act="relu", residual=res))
    q = rng.standard_normal((2, 6, 64), dtype=np.float32)
    kk = rng.standard_normal((40, 3, 64), dtype=np.float32)
    v = rng.standard_normal((40, 3, 64), dtype=np.float32)
    assert same_bits(orc.attend(q, kk, v, 2, 38, 6, 3, 64), ref.attend(q, kk, v, 2, 38, 6, 3, 64))
    logits = rng.standard_normal(999, dtype=np.float32)
    for seed in (1, 7, 123456):
        for t, k in ((0.0, 0), (0.9, 5), (1.0, 0), (1.2, 64), (1.2, 999)):
            assert orc.sample(logits, 999, t, seed, k) == ref.sample(logits, 999, t, seed, k)


def test_restatement_llama_matches_reference(orc, ref):
    from oracle.oracle import LlamaHandle

    cfg = dict(syn.TINY_LLAMA, layers=3, context=48)
    weights = syn.llama_weights(cfg, 12)
    mo, mr = LlamaHandle(orc, cfg), LlamaHandle(ref, cfg)
    mo.load(weights)
    mr.load(weights)
    p = syn.prompts(cfg, 1, 7, 3)[0]
    mo.forward_ids(p, True)
    mr.forward_ids(p, True)
    assert mr.logit_max_abs(mo.logits()) == 0.0
    mo.forward_ids(p[:2], False)
    mr.forward_ids(p[:2], False)
    assert mr.logit_max_abs(mo.logits()) == 0.0
    assert np.array_equal(mo.generate(p, 30, eos_id=int(p[0])), mr.generate(p, 30, eos_id=int(p[0])))
    assert np.array_equal(mo.generate(p, 60), mr.generate(p, 60))  # runs into the full context
