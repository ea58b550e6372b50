"""Parity of the Llama engine (accel_llama_* on the B200) with the reference:
token ids bit-exact, logits and KV-cache rows within rtol = atol = 1e-4, the
reference's counters (211 kernel matmuls per SmolLM2-135M forward, prompt
bytes in, id bytes out)."""

import numpy as np
import pytest

from accelep_b200 import synthetic as syn
from accelep_b200.llama import Llama
from tests.conftest import GOLDEN

pytestmark = pytest.mark.gpu

TOL = 1e-4


@pytest.fixture(scope="module")
def small():
    return np.load(GOLDEN / "ref_small.npz")


@pytest.fixture(scope="module")
def tiny(lib, cuda):
    cfg = syn.TINY_LLAMA
    model = Llama(cfg)
    model.load_fp32(syn.llama_weights(cfg, 5))
    yield model
    model.close()


def test_tiny_generate_matches_reference(tiny, small):
    p = small["tiny_prompt"]
    assert np.array_equal(tiny.generate(p, 40), small["tiny_greedy"])
    assert np.array_equal(tiny.generate(p, 40, temperature=0.8, seed=3, top_k=10), small["tiny_sampled"])
    assert np.array_equal(tiny.generate(p, 40, temperature=1.1, seed=9, top_k=0), small["tiny_full"])


def test_tiny_logits_and_cache(lib, cuda, orc):
    from oracle.oracle import LlamaHandle

    cfg = syn.TINY_LLAMA
    ref = LlamaHandle(orc, cfg)
    ref.load(syn.llama_weights(cfg, 5))
    tiny = Llama(cfg)  # a fresh model: its cache rows start at zero
    tiny.load_fp32(syn.llama_weights(cfg, 5))
    p = syn.prompts(cfg, 1, 9, 21)[0]
    for ids, reset in ((p, True), (p[:1], False), (p[:4], False)):
        tiny.forward_ids(ids, reset)
        ref.forward_ids(ids, reset)
        want = ref.logits()
        assert tiny.logit_max_abs(want) <= TOL
        np.testing.assert_allclose(tiny.logits(), want, rtol=TOL, atol=TOL)
    filled = 14
    hd = cfg["hidden"] // cfg["heads"]
    for layer in range(cfg["layers"]):
        for which in (0, 1):
            got = tiny.cache_rows(0, layer, which, cfg["context"])
            want = ref.cache(layer, which).reshape(cfg["context"], cfg["kv_heads"], hd)
            np.testing.assert_allclose(got[:filled], want[:filled], rtol=TOL, atol=TOL)
            # Rows past the fill were never written: indexing is exact.
            assert not got[filled:].any()
    tiny.close()


def test_tiny_eos_and_full_context(tiny, orc):
    from oracle.oracle import LlamaHandle

    cfg = syn.TINY_LLAMA
    ref = LlamaHandle(orc, cfg)
    ref.load(syn.llama_weights(cfg, 5))
    p = syn.prompts(cfg, 1, 60, 2)[0]
    assert np.array_equal(tiny.generate(p, 50), ref.generate(p, 50))  # stops at a full context
    want = ref.generate(p[:5], 30)
    eos = int(want[3])
    assert np.array_equal(tiny.generate(p[:5], 30, eos_id=eos), ref.generate(p[:5], 30, eos_id=eos))


def test_tiny_batch_equals_single(tiny, orc):
    from oracle.oracle import LlamaHandle

    cfg = syn.TINY_LLAMA
    ref = LlamaHandle(orc, cfg)
    ref.load(syn.llama_weights(cfg, 5))
    rng = np.random.default_rng(8)
    prompts = [rng.integers(0, cfg["vocab"], n).astype(np.int32) for n in (3, 17, 1, 40, 9, 60)]
    got = tiny.generate_batch(prompts, 30)
    for p, g in zip(prompts, got):
        assert np.array_equal(g, ref.generate(p, 30))
    got = tiny.generate_batch(prompts, 30, temperature=0.9, seeds=[5, 6, 7, 8, 9, 10], top_k=20)
    for i, (p, g) in enumerate(zip(prompts, got)):
        assert np.array_equal(g, ref.generate(p, 30, temperature=0.9, seed=5 + i, top_k=20))


def test_tiny_int8(lib, cuda, orc):
    from oracle.oracle import LlamaHandle

    cfg = syn.TINY_LLAMA
    planes, dense = syn.llama_int8(cfg, 7)
    model = Llama(cfg)
    model.load_int8(planes, dense)
    ref = LlamaHandle(orc, cfg)
    ref.load(dense)
    p = syn.prompts(cfg, 1, 6, 4)[0]
    model.forward_ids(p, True)
    ref.forward_ids(p, True)
    np.testing.assert_allclose(model.logits(), ref.logits(), rtol=TOL, atol=TOL)
    assert np.array_equal(model.generate(p, 40), ref.generate(p, 40))
    model.close()


def test_errors(tiny):
    with pytest.raises(RuntimeError, match="vocabulary"):
        tiny.generate(np.array([1, 99999], np.int32), 4)
    with pytest.raises(RuntimeError, match="context"):
        tiny.generate(np.zeros(65, np.int32), 4)
    bad = Llama(dict(syn.TINY_LLAMA))
    with pytest.raises(RuntimeError, match="incomplete"):
        bad.generate(np.array([1], np.int32), 2)
    with pytest.raises(RuntimeError, match="invalid weight"):
        bad.weight(syn.W_Q, 0, np.zeros((3, 3), np.float32))
    bad.close()


@pytest.fixture(scope="module")
def c3(lib, cuda):
    cfg = dict(syn.SMOLLM2_135M, context=128)
    model = Llama(cfg)
    model.load_fp32(syn.llama_weights(cfg, 3))
    yield model
    model.close()


def test_c3_ids_logits_counters(c3):
    g = np.load(GOLDEN / "c3_smollm.npz")
    c3.reset_stats()
    c3.forward_ids(g["prompt"], True)
    assert c3.matmuls() == 211 and c3.bytes_to_device() == 16 and c3.bytes_to_host() == 0
    err = c3.logit_max_abs(g["prefill_logits"])
    assert err <= TOL, err
    c3.reset_stats()
    ids = c3.generate(g["prompt"], 64)
    assert np.array_equal(ids, g["ids"]), (ids, g["ids"])
    assert c3.matmuls() == 211 * 65
    assert c3.bytes_to_device() == 16 and c3.bytes_to_host() == 64 * 4


@pytest.fixture(scope="module")
def c4_model(lib, cuda):
    cfg = syn.SMOLLM2_135M
    planes, dense = syn.llama_int8(cfg, 4)
    model = Llama(cfg)
    model.load_int8(planes, dense)
    yield model
    model.close()


def test_c4_batched_ids(c4_model):
    """C4: 32 x 512-token prompts decoded greedily to 2048 context on the int8
    model, every id against the reference's (tests/golden/c4_ids.npz)."""
    path = GOLDEN / "c4_ids.npz"
    if not path.is_file():
        pytest.skip("c4_ids.npz has not been generated")
    g = np.load(path)
    cfg = syn.SMOLLM2_135M
    prompts = syn.prompts(cfg, 32, 512, 41)
    out = c4_model.generate_batch(list(prompts), cfg["context"] - 512)
    got = np.stack(out)
    want = g["ids"]
    assert got.shape == want.shape
    diverged = [b for b in range(32) if not np.array_equal(got[b], want[b])]
    detail = []
    for b in diverged:
        step = int(np.argmax(got[b] != want[b]))
        detail.append((b, step, float(g["gaps"][b, step])))
    assert not diverged, f"sequences diverged (seq, step, reference top-2 gap): {detail}"


def _c4_golden():
    path = GOLDEN / "c4_logits.npz"
    if not path.is_file():
        pytest.skip("c4_logits.npz has not been generated")
    return np.load(path)


def test_c4_logits_greedy(c4_model):
    """C4 logit rows through generate_batch's captured decode loop (32
    sequences, int8 weights), against the reference's rows
    (tests/golden/c4_logits.npz) at rtol = atol = 1e-4: after the 512-token
    prefill, and after 513 and 1536 decode forwards (positions 1024 and 2047,
    the last row of the context)."""
    g = _c4_golden()
    cfg = syn.SMOLLM2_135M
    prompts = list(syn.prompts(cfg, 32, 512, 41))
    want_ids = np.load(GOLDEN / "c4_ids.npz")["ids"]
    for j, n in enumerate(g["steps"]):
        ids = c4_model.generate_batch(prompts, int(n))
        rows = c4_model.logits(32)
        for i, b in enumerate(g["greedy_seqs"]):
            assert np.array_equal(ids[b], want_ids[b, :n])
            want = g["greedy_logits"][i, j]
            np.testing.assert_allclose(rows[b], want, rtol=TOL, atol=TOL, err_msg=f"seq {b} after {n} forwards")
            if b == 0:  # the reference's own check, on the device (src/llama_model.cc:572-587)
                assert c4_model.logit_max_abs(want) <= TOL


def test_c4_logits_sampled(c4_model):
    """The same rows on full-vocabulary sampled sequences (temperature 1,
    top_k 0, one seed per sequence): the drawn ids equal the reference's and
    the contexts are made of diverse ids, not a greedy repeat loop."""
    g = _c4_golden()
    cfg = syn.SMOLLM2_135M
    prompts = list(syn.prompts(cfg, 32, 512, 41))
    seeds = 1000 + np.arange(32, dtype=np.uint32)
    assert np.array_equal(seeds[g["sampled_seqs"]], g["sampled_seeds"])
    for i in range(len(g["sampled_seqs"])):
        assert len(np.unique(g["sampled_ids"][i])) > 1000  # the context is not a repeat loop
    for j, n in enumerate(g["steps"]):
        ids = c4_model.generate_batch(prompts, int(n), temperature=float(g["temperature"]), seeds=seeds, top_k=0)
        rows = c4_model.logits(32)
        for i, b in enumerate(g["sampled_seqs"]):
            assert np.array_equal(ids[b], g["sampled_ids"][i, :n]), f"seq {b}: drawn ids differ"
            np.testing.assert_allclose(rows[b], g["sampled_logits"][i, j], rtol=TOL, atol=TOL,
                                       err_msg=f"seq {b} after {n} forwards")
