"""Generates the golden fixtures in this folder from the AccelEP reference.

Run here, where the reference sources exist (`python tests/golden/make_golden.py
[--c4]`). The reference is compiled from its own sources by oracle/Makefile
into oracle/_ref/libaccel_ref.so; every array written below is that library's
output on seeded inputs. The known-answer values copied into kats.json are the
literals of the reference's own tests (tests/test_sim_kernels.cc and
tests/test_runtime.cc), checked here against the reference before writing.

Outputs:
  kats.json         hand-written known answers from the reference's tests
  ref_small.npz     seeded small cases run through the reference
  c3_smollm.npz     C3: fp32 SmolLM2-135M shape, 4-token prompt, 64 greedy ids,
                    top-2 logit gaps and the prefill logit row
  c4_ids.npz        C4 (--c4): int8 SmolLM2-135M shape, 32 x 512-token
                    prompts decoded greedily to 2048 context; ids and gaps
                    (the reference fp32 model loaded with the dequantized
                    int8 weights; long, so the restatement runs it, after
                    the restatement was pinned bit for bit against the
                    reference on the first sequence's opening steps)
  c4_logits.npz     C4 (--c4-logits): logit rows of two greedy sequences (fed
                    the golden ids) and two sampled ones (temperature 1, full
                    vocabulary) after the prefill and after 513 and 1536
                    decode forwards, with the sampled ids; the sampled loop is
                    pinned against the reference's Generate on 8 ids
"""

import argparse
import hashlib
import json
import multiprocessing as mp
import struct
import sys
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

from accelep_b200 import synthetic as syn  # noqa: E402
from oracle.oracle import LlamaHandle, Reference, Restated  # noqa: E402

HERE = Path(__file__).resolve().parent


def bits(x):
    return struct.unpack("<I", struct.pack("<f", x))[0]


def fbits(u):
    return struct.unpack("<f", struct.pack("<I", u))[0]


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def make_kats(ref):
    """Literal known answers of tests/test_sim_kernels.cc:47-231 and
    tests/test_runtime.cc:413-459, each confirmed on the reference."""
    kats = {}
    table = np.arange(1, 9, dtype=np.float32).reshape(4, 2)
    got = ref.embed([2, 0], 0, table, 2)
    assert got.reshape(-1).tolist() == [5.0, 6.0, 1.0, 2.0]
    kats["embed"] = {"table": table.tolist(), "ids": [2, 0], "want": [5.0, 6.0, 1.0, 2.0], "bad_id": 9}
    try:
        ref.embed([9], 0, table, 1)
        raise AssertionError("reference accepted an out-of-vocabulary id")
    except ValueError:
        pass
    kats["rmsnorm"] = {"weight": [1.0, 2.0, 0.5, 1.5], "x": [1.0, -1.0, 2.0, 0.0, 4.0, -2.0, 0.5, 3.0], "eps": 1e-5,
                       "tol": 1e-6}
    turned = ref.rope(np.array([1, 2, 3, 4], np.float32), [1, 1, 1, 1, 0, 0, 0, 0], [0, 0, 0, 0, 1, 1, 1, 1], 1, 1, 4, 1)
    assert turned.tolist() == [-3.0, -4.0, 1.0, 2.0]
    kats["rope"] = {"in": [1.0, 2.0, 3.0, 4.0], "cos": [1, 1, 1, 1, 0, 0, 0, 0], "sin": [0, 0, 0, 0, 1, 1, 1, 1],
                    "position": 1, "want": [-3.0, -4.0, 1.0, 2.0]}
    cache = ref.append_cache(np.array([9, 8, 7, 6], np.float32), np.full(8, -5, np.float32), 2, 1, 1, 2)
    assert cache.tolist() == [-5, -5, 9, 8, 7, 6, -5, -5]
    kats["cache"] = {"src": [9, 8, 7, 6], "fill": -5.0, "seq": 2, "position": 1, "n_heads": 1, "head_dim": 2,
                     "want": [-5, -5, 9, 8, 7, 6, -5, -5]}
    att = ref.attend(np.ones(1, np.float32), np.ones(1, np.float32), np.full(1, 3, np.float32), 1, 0, 1, 1, 1)
    assert float(att.reshape(-1)[0]) == 3.0
    kats["attention"] = {"q": 1.0, "k": 1.0, "v": 3.0, "want": 3.0}
    assert float(ref.silu_mul([0.0], [2.0])[0]) == 0.0
    kats["silu"] = {"gate": 0.0, "up": 2.0, "want": 0.0}
    assert ref.add([1, 2], [3, 4]).tolist() == [4.0, 6.0]
    kats["add"] = {"dest": [1, 2], "extra": [3, 4], "want": [4, 6]}
    samples = [
        # logits, temperature, rng, top_k, want id, want rng after (None = not checked)
        ([1.0, 3.0, 3.0], 0.0, 1, 2, 1, None),
        ([1.0, 3.0, 3.0], -1.0, 1, 0, 1, None),
        ([1.0, 3.0, 0.0], 1.0, 1856, 2, 0, None),
        ([1.0, 3.0, 0.0], 1.0, 1856, 0, 1, None),
        ([1.0, 3.0, 0.0], 1.0, 0, 0, 0, 0),
        ([0.0] * 65, 1.0, 1000, 65, 4, None),
        ([0.0] * 65, 1.0, 1000, 64, 3, None),
    ]
    for logits, t, r, k, want, want_rng in samples:
        got, state = ref.sample(logits, len(logits), t, r, k)
        assert got == want, (logits[:3], t, r, k, got, want)
        if want_rng is not None:
            assert state == want_rng
    kats["sample"] = [{"logits": lg, "temperature": t, "rng": r, "top_k": k, "want": w, "want_rng": wr}
                      for lg, t, r, k, w, wr in samples]
    a = np.array([fbits(0xBE2694CD), fbits(0x3E41AF7D)], np.float32).reshape(1, 2)
    b = np.array([fbits(0x3F800000), fbits(0x3F5C2CB8)], np.float32).reshape(2, 1)
    out = ref.matmul(a, b)
    assert bits(float(out[0, 0])) == 0xB5200000
    kats["split_product"] = {"a_bits": [0xBE2694CD, 0x3E41AF7D], "b_bits": [0x3F800000, 0x3F5C2CB8],
                             "want_bits": 0xB5200000}
    x = np.array([[1, 2], [0, -1]], np.float32)
    w = np.array([[-128, 127], [1, -2]], np.int8)
    scale = np.array([0.5, 2.0], np.float32)
    zp = np.array([1, -3], np.int8)
    got = ref.execute_matmul_q(x, w, scale, zp, axis=0)
    assert float(got[0, 0]) == -48.5
    kats["dequantize"] = {"x": x.tolist(), "w": w.tolist(), "scale": scale.tolist(), "zero": zp.tolist(), "axis": 0,
                          "want00": -48.5, "want": got.tolist()}
    e1 = ref.gemm_epilogue(ref.matmul([[np.inf]], [[0.0]]), 1.0, None, [], 0.0, "relu")
    e2 = ref.gemm_epilogue(ref.matmul([[-np.inf]], [[1.0]]), 1.0, None, [], 0.0, "relu")
    e3 = ref.gemm_epilogue(ref.matmul([[0.0]], [[1.0]]), -1.0, None, [], 0.0, "relu")
    assert np.isnan(e1[0, 0]) and bits(float(e2[0, 0])) == 0 and bits(float(e3[0, 0])) == 0x80000000
    kats["nonfinite_epilogue"] = {"relu_of_inf_times_zero": "nan", "relu_of_neg_inf_bits": 0,
                                  "relu_of_alpha_neg1_zero_bits": 0x80000000}
    return kats


def gemv_inputs():
    """Inputs of the stored GEMV-shaped case: [1, 576] x [576, 1536], seed 77."""
    g = np.random.default_rng(77)
    return g.standard_normal((1, 576), dtype=np.float32), g.standard_normal((576, 1536), dtype=np.float32)


def make_small(ref):
    """Seeded small cases. Arrays are stored whole; bigger outputs as sha256."""
    out = {}
    rng = np.random.default_rng(1234)
    for m, k, n in [(128, 160, 96), (13, 19, 17), (3, 70, 33)]:
        a = rng.standard_normal((m, k), dtype=np.float32)
        b = rng.standard_normal((k, n), dtype=np.float32)
        c = ref.matmul(a, b)
        out[f"mm_{m}_{k}_{n}_a"], out[f"mm_{m}_{k}_{n}_b"], out[f"mm_{m}_{k}_{n}_c"] = a, b, c
    # A GEMV-shaped case whose inputs are regenerated from their own seed.
    a, b = gemv_inputs()
    out["mm_gemv_c"] = ref.matmul(a, b)
    # Quantized panel: per-column scale, per-row scale + zero, scalar scale; odd sizes.
    for tag, (m, k, n) in {"q1": (8, 160, 300), "q2": (5, 77, 261), "q3": (16, 64, 512)}.items():
        a = rng.standard_normal((m, k), dtype=np.float32)
        q = rng.integers(-128, 128, size=(k, n), dtype=np.int64).astype(np.int8)
        col = rng.uniform(1e-3, 1e-2, size=n).astype(np.float32)
        row = rng.uniform(0.1, 1.0, size=k).astype(np.float32)
        zero = rng.integers(-5, 6, size=k, dtype=np.int64).astype(np.int8)
        out[f"{tag}_a"], out[f"{tag}_q"], out[f"{tag}_col"], out[f"{tag}_row"], out[f"{tag}_zero"] = a, q, col, row, zero
        out[f"{tag}_c_col"] = ref.matmul_quantized(a, q, col, None, [k, n], 1, 0, m, k, n)
        out[f"{tag}_c_row"] = ref.matmul_quantized(a, q, row, zero, [k, n], 0, 0, m, k, n)
        out[f"{tag}_c_scalar"] = ref.matmul_quantized(a, q, np.array([0.5], np.float32), None, [k, n], -1, 0, m, k, n)
    # Epilogue: alpha, bias broadcast shapes, relu / gelu.
    c = rng.standard_normal((6, 10), dtype=np.float32) * np.float32(3)
    out["ep_c"] = c
    for i, (shape, alpha, beta, act) in enumerate([((10,), 1.5, 0.5, "none"), ((6, 1), 1.0, 1.0, "relu"),
                                                  ((1, 10), -0.75, 2.0, "gelu"), ((6, 10), 1.0, 1.0, "gelu"),
                                                  ((), 1.0, 0.0, "relu"), ((1,), 2.0, 1.0, "none")]):
        bias = rng.standard_normal(int(np.prod(shape)) if shape else 1, dtype=np.float32)
        out[f"ep{i}_bias"] = bias
        out[f"ep{i}_out"] = ref.gemm_epilogue(c, alpha, bias, list(shape), beta, act)
    # Row kernels.
    x = rng.standard_normal((7, 576), dtype=np.float32)
    w = rng.uniform(0.5, 1.5, size=576).astype(np.float32)
    out["rms_x"], out["rms_w"] = x, w
    out["rms_y"] = ref.rmsnorm(x, w, 7, 576, 1e-5, 0)
    out["rms_y_off"] = ref.rmsnorm(x, w, 2, 576, 1e-5, 5)
    states = rng.standard_normal((3, 9, 64), dtype=np.float32)
    ang = rng.uniform(-3, 3, size=(20, 64))
    cos_t, sin_t = np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)
    out["rope_in"], out["rope_cos"], out["rope_sin"] = states, cos_t, sin_t
    out["rope_out"] = ref.rope(states, cos_t, sin_t, 3, 9, 64, 11)
    g = rng.standard_normal(1000, dtype=np.float32) * np.float32(4)
    u = rng.standard_normal(1000, dtype=np.float32)
    out["silu_gate"], out["silu_up"], out["silu_out"] = g, u, ref.silu_mul(g, u)
    # Attention: decode (seq 1) and prefill (seq 5) shapes, GQA 9/3 x 64 and 4/2 x 8.
    for tag, (seq, pos, heads, kvh, hd) in {"at1": (1, 37, 9, 3, 64), "at2": (5, 0, 9, 3, 64),
                                             "at3": (4, 9, 4, 2, 8), "at4": (1, 300, 9, 3, 64)}.items():
        q = rng.standard_normal((seq, heads, hd), dtype=np.float32)
        kk = rng.standard_normal((pos + seq, kvh, hd), dtype=np.float32)
        vv = rng.standard_normal((pos + seq, kvh, hd), dtype=np.float32)
        out[f"{tag}_q"], out[f"{tag}_k"], out[f"{tag}_v"] = q, kk, vv
        out[f"{tag}_out"] = ref.attend(q, kk, vv, seq, pos, heads, kvh, hd)
        out[f"{tag}_dims"] = np.array([seq, pos, heads, kvh, hd], np.int64)
    # Sampling over many seeds and modes.
    logits = rng.standard_normal(4096, dtype=np.float32)
    logits[17] = logits[99] = np.float32(10.0)
    out["smp_logits"] = logits
    rows = []
    for seed in range(1, 41):
        for temp, k in [(0.0, 0), (1.0, 0), (0.7, 10), (1.3, 64), (1.0, 65), (2.0, 4096)]:
            got, state = ref.sample(logits, 4096, temp, seed, k)
            rows.append([seed, int(temp * 1000), k, got, state])
    out["smp_rows"] = np.array(rows, np.int64)
    # C1 at full size: output digest plus one full row.
    x, w, s = syn.int8_gemm(64, 576, 1536, 1)
    c1 = ref.execute_matmul_q(x, w, s, act="relu")
    out["c1_sha"] = np.frombuffer(bytes.fromhex(sha(c1)), np.uint8)
    out["c1_row0"] = c1[0]
    # C2 on 16 of the 256 rows (rows are independent): digest and values.
    x, blocks = syn.mlp_stack()
    h = x[:16]
    for w1, s1, w2, s2, gamma in blocks:
        h, _ = ref.mlp_block(h, w1, s1, w2, s2, gamma, 1e-5)
    out["c2_rows16"] = h
    # Tiny Llama through the reference's own C API.
    cfg = syn.TINY_LLAMA
    weights = syn.llama_weights(cfg, 5)
    model = LlamaHandle(ref, cfg)
    model.load(weights)
    p = syn.prompts(cfg, 1, 5, 7)[0]
    out["tiny_prompt"] = p
    out["tiny_greedy"] = model.generate(p, 40)
    out["tiny_sampled"] = model.generate(p, 40, temperature=0.8, seed=3, top_k=10)
    out["tiny_full"] = model.generate(p, 40, temperature=1.1, seed=9, top_k=0)
    model.close()
    return out


def make_c3(ref, orc):
    cfg = syn.SMOLLM2_135M
    weights = syn.llama_weights(cfg, 3)
    prompt = syn.prompts(cfg, 1, 4, 11)[0]
    ctx = dict(cfg, context=128)
    mo = LlamaHandle(orc, ctx)
    mo.load(weights)
    ids, gaps = mo.generate(prompt, 64, want_gaps=True)
    mo.forward_ids(prompt, True)
    logits = mo.logits()
    mr = LlamaHandle(ref, ctx)
    mr.load(weights)
    ref_ids = mr.generate(prompt, 64)
    assert np.array_equal(ref_ids, ids), "restatement and reference disagree on C3 ids"
    mr.forward_ids(prompt, True)
    assert mr.logit_max_abs(logits) == 0.0, "restatement and reference disagree on C3 logits"
    return {"prompt": prompt, "ids": ids, "gaps": gaps, "prefill_logits": logits}


def _c4_worker(args):
    index, prompt, steps = args
    cfg = syn.SMOLLM2_135M
    _, dense = syn.llama_int8(cfg, 4)
    model = LlamaHandle(Restated(), cfg)
    model.load(dense)
    t = time.time()
    ids, gaps = model.generate(prompt, steps, want_gaps=True)
    print(f"c4 seq {index}: {len(ids)} ids in {time.time() - t:.0f}s", flush=True)
    return index, ids, gaps


def make_c4(ref, orc, workers):
    cfg = syn.SMOLLM2_135M
    prompts = syn.prompts(cfg, 32, 512, 41)
    steps = cfg["context"] - 512
    # Pin: the reference itself on the first sequence, first 8 ids.
    _, dense = syn.llama_int8(cfg, 4)
    mr = LlamaHandle(ref, cfg)
    mr.load(dense)
    ref_head = mr.generate(prompts[0], 8)
    mr.close()
    del dense
    ctx = mp.get_context("spawn")
    with ctx.Pool(workers) as pool:
        results = pool.map(_c4_worker, [(i, prompts[i], steps) for i in range(32)])
    results.sort(key=lambda r: r[0])
    ids = np.stack([r[1] for r in results])
    gaps = np.stack([r[2] for r in results])
    assert np.array_equal(ids[0, :8], ref_head), "restatement and reference disagree on C4 ids"
    return {"prompts_sha": np.frombuffer(bytes.fromhex(sha(prompts)), np.uint8), "ids": ids, "gaps": gaps}


# Decode forwards after the prefill at which C4 logit rows are kept: 0 (the
# prefill's last row, position 511), 513 (position 1024) and 1536 (position
# 2047, the last row of the 2048-row context).
C4_LOGIT_STEPS = (0, 513, 1536)
C4_GREEDY_SEQS = (0, 17)
C4_SAMPLED_SEQS = (3, 29)
C4_TEMPERATURE = 1.0


def c4_seed(b):
    """Seed of sampled sequence b in the C4 logit fixtures."""
    return 1000 + b


def _c4_logit_worker(args):
    """One C4 sequence through the restatement, one forward at a time, keeping
    the logit rows at C4_LOGIT_STEPS. Greedy sequences are fed the stored
    golden ids (and each argmax is checked against them); sampled sequences
    draw with src/sim_sample.cc's full-vocabulary walk (top_k 0) from
    c4_seed(b), the seed rule of src/llama_model.cc:111."""
    index, prompt, golden_ids, sampled = args
    cfg = syn.SMOLLM2_135M
    _, dense = syn.llama_int8(cfg, 4)
    orc = Restated()
    model = LlamaHandle(orc, cfg)
    model.load(dense)
    t = time.time()
    steps = cfg["context"] - len(prompt)
    rows, ids = [], []
    rng = c4_seed(index)
    model.forward_ids(prompt, True)
    for n in range(steps + 1):
        logits = model.logits()
        if n in C4_LOGIT_STEPS:
            rows.append(logits)
        if n == steps:
            break
        if sampled:
            nxt, rng = orc.sample(logits, cfg["vocab"], C4_TEMPERATURE, rng, 0)
        else:
            nxt = int(golden_ids[n])
            assert int(np.argmax(logits)) == nxt, (index, n)
        ids.append(nxt)
        model.forward_ids(np.array([nxt], np.int32), False)
    model.close()
    head = None
    if sampled:
        # Pin the loop above against the reference's own Generate.
        mr = LlamaHandle(Reference(), cfg)
        mr.load(dense)
        head = mr.generate(prompt, 8, temperature=C4_TEMPERATURE, seed=c4_seed(index))
        mr.close()
        assert np.array_equal(head, np.array(ids[:8], np.int32)), (index, head, ids[:8])
    print(f"c4 logits seq {index} ({'sampled' if sampled else 'greedy'}): {time.time() - t:.0f}s", flush=True)
    return index, sampled, np.array(ids, np.int32), np.stack(rows)


def make_c4_logits(workers):
    """C4 logit rows of two greedy and two sampled sequences at the decode
    depths C4_LOGIT_STEPS, plus the sampled sequences' ids."""
    cfg = syn.SMOLLM2_135M
    prompts = syn.prompts(cfg, 32, 512, 41)
    golden = np.load(HERE / "c4_ids.npz")["ids"]
    jobs = [(b, prompts[b], golden[b], False) for b in C4_GREEDY_SEQS]
    jobs += [(b, prompts[b], None, True) for b in C4_SAMPLED_SEQS]
    ctx = mp.get_context("spawn")
    with ctx.Pool(min(workers, len(jobs))) as pool:
        results = pool.map(_c4_logit_worker, jobs)
    out = {"steps": np.array(C4_LOGIT_STEPS, np.int32), "temperature": np.float32(C4_TEMPERATURE)}
    greedy = [r for r in results if not r[1]]
    sampled = [r for r in results if r[1]]
    out["greedy_seqs"] = np.array([r[0] for r in greedy], np.int32)
    out["greedy_logits"] = np.stack([r[3] for r in greedy])  # [seq, step, vocab]
    out["sampled_seqs"] = np.array([r[0] for r in sampled], np.int32)
    out["sampled_seeds"] = np.array([c4_seed(r[0]) for r in sampled], np.uint32)
    out["sampled_ids"] = np.stack([r[2] for r in sampled])
    out["sampled_logits"] = np.stack([r[3] for r in sampled])
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--c4", action="store_true")
    ap.add_argument("--c4-logits", action="store_true")
    ap.add_argument("--workers", type=int, default=8)
    args = ap.parse_args()
    if args.c4_logits:
        np.savez_compressed(HERE / "c4_logits.npz", **make_c4_logits(args.workers))
        return
    ref, orc = Reference(), Restated()
    if args.c4:
        np.savez_compressed(HERE / "c4_ids.npz", **make_c4(ref, orc, args.workers))
        return
    (HERE / "kats.json").write_text(json.dumps(make_kats(ref), indent=1) + "\n")
    np.savez_compressed(HERE / "ref_small.npz", **make_small(ref))
    np.savez_compressed(HERE / "c3_smollm.npz", **make_c3(ref, orc))


if __name__ == "__main__":
    main()
