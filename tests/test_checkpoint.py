"""Hugging Face checkpoints into the engine (accelep_b200/checkpoint.py):
safetensors decoding of F32 / F16 / BF16 (bf16 as its 16 bits in the top half
of a float32, as serve/weights.py:36-46 decodes it), config.json checks
(serve/llama.py:187-196), the tensor-name to weight-kind map
(serve/llama.py:237-251) with a tied or separate LM head, the int8 upload,
and on the GPU a checkpoint-loaded model generating the ids of the same
weights loaded from arrays."""

import json

import numpy as np
import pytest

from accelep_b200 import checkpoint as ck
from accelep_b200 import synthetic as syn


def bf16_bits(x):
    """Round-to-nearest-even bf16 patterns of float32 values."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def test_safetensors_dtypes(tmp_path):
    rng = np.random.default_rng(0)
    a = rng.standard_normal((3, 5)).astype(np.float32)
    h = rng.standard_normal(7).astype(np.float16)
    b = bf16_bits(rng.standard_normal((2, 4)))
    path = tmp_path / "t.safetensors"
    ck.write_safetensors(path, {"a": (a, "F32"), "h": (h, "F16"), "b": (b, "BF16")})
    f = ck.SafetensorsFile(path)
    assert sorted(f.names()) == ["a", "b", "h"] and "a" in f and "zz" not in f
    assert np.array_equal(f.get("a"), a)
    assert np.array_equal(f.get("h"), h.astype(np.float32))
    got = f.get("b")
    assert got.dtype == np.float32 and got.shape == (2, 4)
    assert np.array_equal(got.view(np.uint32), b.astype(np.uint32) << 16)


def test_unsupported_dtype(tmp_path):
    path = tmp_path / "t.safetensors"
    ck.write_safetensors(path, {"i": (np.arange(4, dtype=np.int32), "I32")})
    with pytest.raises(ValueError):
        ck.SafetensorsFile(path).get("i")


def hf_config(cfg, **extra):
    out = {"architectures": ["LlamaForCausalLM"], "hidden_act": "silu", "vocab_size": cfg["vocab"],
           "hidden_size": cfg["hidden"], "num_hidden_layers": cfg["layers"], "num_attention_heads": cfg["heads"],
           "num_key_value_heads": cfg["kv_heads"], "intermediate_size": cfg["intermediate"],
           "rms_norm_eps": cfg["eps"], "rope_theta": cfg["rope_theta"], "max_position_embeddings": 8192}
    out.update(extra)
    return out


def write_checkpoint(d, cfg, weights, tied, dtype="F32"):
    (d / "config.json").write_text(json.dumps(hf_config(cfg)))
    tensors = {}
    for kind, layer, name in ck.tensor_names(cfg["layers"], tied):
        value = weights[(kind, layer)] if not (tied and kind == syn.W_LM_HEAD) else weights[(syn.W_EMBED, -1)]
        tensors[name] = (bf16_bits(value), "BF16") if dtype == "BF16" else (value, "F32")
    ck.write_safetensors(d / "model.safetensors", tensors)


def test_config_checks(tmp_path):
    cfg = syn.TINY_LLAMA
    (tmp_path / "config.json").write_text(json.dumps(hf_config(cfg)))
    got = ck.config_from_dir(tmp_path, 64)
    assert got == dict(cfg, context=64)
    for bad in ({"architectures": ["GPT2LMHeadModel"]}, {"hidden_act": "gelu"}, {"rope_scaling": {"factor": 2}}):
        (tmp_path / "config.json").write_text(json.dumps(hf_config(cfg, **bad)))
        with pytest.raises(ValueError):
            ck.config_from_dir(tmp_path, 64)


class Recorder:
    def __init__(self, cfg):
        self.cfg = cfg
        self.calls = []

    def weight(self, kind, layer, values):
        self.calls.append(("f32", kind, layer, values))

    def weight_q8(self, kind, layer, q, scale):
        self.calls.append(("q8", kind, layer, (q, scale)))


@pytest.mark.parametrize("tied,int8", [(True, False), (False, False), (False, True)])
def test_load_maps_every_weight(tmp_path, tied, int8):
    cfg = syn.TINY_LLAMA
    weights = syn.llama_weights(cfg, 3)
    write_checkpoint(tmp_path, cfg, weights, tied)
    rec = Recorder(cfg)
    ck.load_into(rec, tmp_path, int8=int8)
    assert len(rec.calls) == 3 + 9 * cfg["layers"]
    seen = {(kind, layer) for _, kind, layer, _ in rec.calls}
    assert seen == set(weights) | {(syn.W_LM_HEAD, -1)}
    for how, kind, layer, values in rec.calls:
        want = weights[(syn.W_EMBED, -1)] if (tied and kind == syn.W_LM_HEAD) else weights[(kind, layer)]
        quantized = int8 and (kind in syn.LINEAR_KINDS or kind == syn.W_LM_HEAD)
        assert how == ("q8" if quantized else "f32")
        if quantized:
            q, s = syn.quantize_rows(want)
            assert np.array_equal(values[0], q) and np.array_equal(values[1], s)
        else:
            assert np.array_equal(values, want)


def test_missing_tensor(tmp_path):
    cfg = syn.TINY_LLAMA
    (tmp_path / "config.json").write_text(json.dumps(hf_config(cfg)))
    ck.write_safetensors(tmp_path / "model.safetensors", {"model.norm.weight": (np.ones(cfg["hidden"],
                                                                                         np.float32), "F32")})
    with pytest.raises(KeyError):
        ck.load_into(Recorder(cfg), tmp_path)


@pytest.mark.gpu
def test_checkpoint_model_generates_same_ids(tmp_path, lib, cuda):
    """A tiny model written as a BF16 checkpoint and loaded through
    checkpoint.load_into generates the ids of the same (bf16-rounded) weights
    loaded from arrays."""
    from accelep_b200.llama import Llama

    cfg = syn.TINY_LLAMA
    weights = syn.llama_weights(cfg, 5)
    write_checkpoint(tmp_path, cfg, weights, tied=False, dtype="BF16")
    rounded = {key: (bf16_bits(v).astype(np.uint32) << 16).view(np.float32).reshape(v.shape)
               for key, v in weights.items()}
    prompt = syn.prompts(cfg, 1, 5, 7)[0]
    with Llama(ck.config_from_dir(tmp_path, cfg["context"])) as model:
        ck.load_into(model, tmp_path)
        got = model.generate(prompt, 12)
    with Llama(cfg) as model:
        model.load_fp32(rounded)
        want = model.generate(prompt, 12)
    assert np.array_equal(got, want)
