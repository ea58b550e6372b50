"""Hugging Face Llama checkpoints (config.json + model.safetensors) into the
B200 engine.

The reference server reads a safetensors file header-first and uploads one
tensor at a time (serve/weights.py:13-55, serve/llama.py:187-258): F32, F16 and
BF16 tensors become float32 (bf16 by moving its 16 bits into the top half of a
float32), the names `model.embed_tokens`, `model.norm`, `lm_head` (or the tied
embedding) and `model.layers.{i}.{input_layernorm, post_attention_layernorm,
self_attn.{q,k,v,o}_proj, mlp.{gate,up,down}_proj}` map to the weight kinds,
and config.json must describe a LlamaForCausalLM with a silu MLP and no RoPE
scaling. This module does the same for `accelep_b200.llama.Llama`, and can
upload the linear weights and the LM head as int8 instead (per output row,
scale = max|w| / 127, the C4 quantization).
"""

import json
import struct
from pathlib import Path

import numpy as np

from . import synthetic as syn

_DTYPES = {"F32": np.float32, "F16": np.float16, "BF16": np.uint16}


class SafetensorsFile:
    """Reads the header once; `get(name)` reads and decodes one tensor."""

    def __init__(self, path):
        self.path = str(path)
        with open(self.path, "rb") as f:
            (length,) = struct.unpack("<Q", f.read(8))
            self.header = json.loads(f.read(length))
        self.data_start = 8 + length

    def names(self):
        return [n for n in self.header if n != "__metadata__"]

    def __contains__(self, name):
        return name in self.header and name != "__metadata__"

    def get(self, name):
        info = self.header[name]
        dtype = info["dtype"]
        if dtype not in _DTYPES:
            raise ValueError(f"unsupported dtype {dtype} for {name}")
        begin, end = info["data_offsets"]
        with open(self.path, "rb") as f:
            f.seek(self.data_start + begin)
            raw = f.read(end - begin)
        values = np.frombuffer(raw, dtype=_DTYPES[dtype])
        if dtype == "BF16":
            values = (values.astype(np.uint32) << 16).view(np.float32)
        return np.ascontiguousarray(values.astype(np.float32, copy=False).reshape(info["shape"]))


def write_safetensors(path, tensors):
    """Writes {name: (array, dtype)} as a safetensors file, dtype "F32",
    "F16" or "BF16" (a BF16 array holds the 16-bit patterns as uint16). For
    tests and tools that make small checkpoints."""
    header, blobs, offset = {}, [], 0
    for name, (array, dtype) in tensors.items():
        data = np.ascontiguousarray(array).tobytes()
        header[name] = {"dtype": dtype, "shape": list(np.shape(array)), "data_offsets": [offset, offset + len(data)]}
        blobs.append(data)
        offset += len(data)
    raw = json.dumps(header).encode()
    raw += b" " * (-len(raw) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(raw)))
        f.write(raw)
        for b in blobs:
            f.write(b)


def config_from_dir(model_dir, context):
    """The engine configuration of a checkpoint directory's config.json, with
    the reference server's checks."""
    with open(Path(model_dir) / "config.json", encoding="utf-8") as f:
        hf = json.load(f)
    if hf.get("architectures") != ["LlamaForCausalLM"]:
        raise ValueError(f"expected LlamaForCausalLM, got {hf.get('architectures')}")
    if hf.get("hidden_act", "silu") != "silu":
        raise ValueError("only a silu MLP is implemented")
    if hf.get("rope_scaling"):
        raise ValueError("RoPE scaling is not implemented")
    return {"vocab": int(hf["vocab_size"]), "hidden": int(hf["hidden_size"]), "layers": int(hf["num_hidden_layers"]),
            "heads": int(hf["num_attention_heads"]), "kv_heads": int(hf["num_key_value_heads"]),
            "intermediate": int(hf["intermediate_size"]), "context": int(context),
            "eps": float(hf["rms_norm_eps"]), "rope_theta": float(hf["rope_theta"])}


def tensor_names(layers, tied):
    """(kind, layer, name) for every weight the engine needs."""
    out = [(syn.W_EMBED, -1, "model.embed_tokens.weight"), (syn.W_FINAL_NORM, -1, "model.norm.weight"),
           (syn.W_LM_HEAD, -1, "model.embed_tokens.weight" if tied else "lm_head.weight")]
    per_layer = [(syn.W_ATTN_NORM, "input_layernorm"), (syn.W_POST_NORM, "post_attention_layernorm"),
                 (syn.W_Q, "self_attn.q_proj"), (syn.W_K, "self_attn.k_proj"), (syn.W_V, "self_attn.v_proj"),
                 (syn.W_O, "self_attn.o_proj"), (syn.W_GATE, "mlp.gate_proj"), (syn.W_UP, "mlp.up_proj"),
                 (syn.W_DOWN, "mlp.down_proj")]
    for i in range(layers):
        out += [(kind, i, f"model.layers.{i}.{part}.weight") for kind, part in per_layer]
    return out


def load_into(model, model_dir, int8=False):
    """Uploads a checkpoint directory's weights into `model` (a Llama, or any
    object with weight(kind, layer, values) and weight_q8(kind, layer, q,
    scale)), one tensor at a time. int8: the linear weights and the LM head
    go up as per-output-row int8 planes."""
    reader = SafetensorsFile(Path(model_dir) / "model.safetensors")
    tied = "lm_head.weight" not in reader
    quantized = set(syn.LINEAR_KINDS) | {syn.W_LM_HEAD}
    for kind, layer, name in tensor_names(model.cfg["layers"], tied):
        if name not in reader:
            raise KeyError(f"checkpoint has no {name}")
        values = reader.get(name)
        if int8 and kind in quantized:
            q, s = syn.quantize_rows(values)
            model.weight_q8(kind, layer, q, s)
        else:
            model.weight(kind, layer, values)
        del values
