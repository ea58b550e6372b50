"""ctypes binding of the Llama C API on the B200 backend.

Mirrors the reference binding (serve/llama.py:96-439): the same create /
weight / generate / forward_ids / logit_max_abs / reset calls and counters,
plus the backend's additions: int8 weights, batched generation, the logit
row and cache rows as test hooks, and the model's CUDA stream. Weights come
from numpy arrays in Hugging Face layout (the reference reads them from
safetensors; no checkpoint is used here).
"""

import ctypes

import numpy as np

from . import synthetic
from ._lib import P_f32, P_i8, P_i32, P_u32, LlamaConfig, load


def _ptr(a, ptype):
    return a.ctypes.data_as(ptype)


class Llama:
    """One model in HBM of the CUDA device current at construction."""

    def __init__(self, cfg):
        self.cfg = dict(cfg)
        self._lib = load()
        native = LlamaConfig(cfg["vocab"], cfg["hidden"], cfg["layers"], cfg["heads"], cfg["kv_heads"],
                             cfg["intermediate"], cfg["context"], float(cfg["eps"]), float(cfg["rope_theta"]))
        self._model = self._lib.accel_llama_create(ctypes.byref(native))
        if not self._model:
            raise RuntimeError(self.error() or "create failed")

    def error(self):
        raw = self._lib.accel_llama_last_error()
        return raw.decode() if raw else ""

    def _check(self, status, what):
        if status != 0:
            raise RuntimeError(self.error() or f"{what} failed")

    def close(self):
        if self._model:
            self._lib.accel_llama_destroy(self._model)
            self._model = None

    def __enter__(self):
        return self

    def __exit__(self, *_):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # ------------------------------------------------------------- weights

    def weight(self, kind, layer, values):
        array = np.ascontiguousarray(values, dtype=np.float32)
        rows, cols = (array.shape[0], 1) if array.ndim == 1 else array.shape
        self._check(self._lib.accel_llama_weight(self._model, kind, layer, _ptr(array, P_f32), rows, cols), "weight")

    def weight_q8(self, kind, layer, q, scale):
        q = np.ascontiguousarray(q, dtype=np.int8)
        scale = np.ascontiguousarray(scale, dtype=np.float32)
        rows, cols = q.shape
        self._check(self._lib.accel_llama_weight_q8(self._model, kind, layer, _ptr(q, P_i8), _ptr(scale, P_f32), rows,
                                                    cols), "weight_q8")

    def load_fp32(self, weights):
        """weights: {(kind, layer): array} as synthetic.llama_weights returns."""
        for (kind, layer), values in weights.items():
            self.weight(kind, layer, values)

    def load_int8(self, planes, dense):
        """Int8 linear weights and LM head; fp32 embedding and norms."""
        for (kind, layer), values in dense.items():
            if (kind, layer) not in planes:
                self.weight(kind, layer, values)
        for (kind, layer), (q, s) in planes.items():
            self.weight_q8(kind, layer, q, s)

    # ----------------------------------------------------------- generation

    def generate(self, prompt, max_new, eos_id=-1, temperature=0.0, seed=0, top_k=0):
        prompt = np.ascontiguousarray(prompt, dtype=np.int32)
        out = np.zeros(max(1, max_new), dtype=np.int32)
        count = np.zeros(1, dtype=np.int32)
        self._check(self._lib.accel_llama_generate(self._model, _ptr(prompt, P_i32), prompt.size, max_new, eos_id,
                                                   temperature, seed, top_k, _ptr(out, P_i32), _ptr(count, P_i32)),
                    "generate")
        return out[:int(count[0])].copy()

    def generate_batch(self, prompts, max_new, eos_id=-1, temperature=0.0, seed=0, seeds=None, top_k=0):
        """prompts: list of id arrays (or a 2-D array). Returns a list of id arrays."""
        arrays = [np.ascontiguousarray(p, dtype=np.int32) for p in prompts]
        flat = np.ascontiguousarray(np.concatenate(arrays), dtype=np.int32)
        counts = np.array([a.size for a in arrays], dtype=np.int32)
        batch = len(arrays)
        out = np.zeros((batch, max(1, max_new)), dtype=np.int32)
        out_counts = np.zeros(batch, dtype=np.int32)
        seed_arr = None if seeds is None else np.ascontiguousarray(seeds, dtype=np.uint32)
        self._check(self._lib.accel_llama_generate_batch(
            self._model, _ptr(flat, P_i32), _ptr(counts, P_i32), batch, max_new, eos_id, temperature, seed,
            None if seed_arr is None else _ptr(seed_arr, P_u32), top_k, _ptr(out, P_i32), _ptr(out_counts, P_i32)),
            "generate_batch")
        return [out[b, :int(out_counts[b])].copy() for b in range(batch)]

    def forward_ids(self, ids, reset):
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        self._check(self._lib.accel_llama_forward_ids(self._model, _ptr(ids, P_i32), ids.size, 1 if reset else 0),
                    "forward")

    def logit_max_abs(self, reference):
        row = np.ascontiguousarray(reference, dtype=np.float32)
        out = np.zeros(1, dtype=np.float32)
        self._check(self._lib.accel_llama_logit_max_abs(self._model, _ptr(row, P_f32), row.size, _ptr(out, P_f32)),
                    "logit max abs")
        return float(out[0])

    def logits(self, rows=None):
        """The last forward's logit row, or with `rows` its first `rows` rows
        (one per sequence of a batched generate) as [rows, vocab]."""
        shape = (self.cfg["vocab"],) if rows is None else (rows, self.cfg["vocab"])
        out = np.zeros(shape, dtype=np.float32)
        self._check(self._lib.accel_llama_logits(self._model, _ptr(out, P_f32), out.size), "logits")
        return out

    def cache_rows(self, slot, layer, which, rows):
        head_dim = self.cfg["hidden"] // self.cfg["heads"]
        out = np.zeros((rows, self.cfg["kv_heads"], head_dim), dtype=np.float32)
        self._check(self._lib.accel_llama_cache_rows(self._model, slot, layer, which, rows, _ptr(out, P_f32)), "cache")
        return out

    def reset(self):
        self._lib.accel_llama_reset(self._model)

    def stream(self):
        """The model's cudaStream_t as an int (for torch.cuda.ExternalStream)."""
        return int(self._lib.accel_llama_stream(self._model) or 0)

    # ------------------------------------------------------------- counters

    def reset_stats(self):
        self._lib.accel_sim_reset_stats()

    def matmuls(self):
        return int(self._lib.accel_sim_matmuls())

    def bytes_to_device(self):
        return int(self._lib.accel_sim_bytes_to_device())

    def bytes_to_host(self):
        return int(self._lib.accel_sim_bytes_to_host())


def smollm_int8(seed=4, cfg=None):
    """A C4 model: SmolLM2-135M shape, int8 linear weights from `seed`."""
    cfg = dict(cfg or synthetic.SMOLLM2_135M)
    planes, dense = synthetic.llama_int8(cfg, seed)
    model = Llama(cfg)
    model.load_int8(planes, dense)
    return model, dense
