"""ctypes access to the parity checkers. TEST INFRASTRUCTURE ONLY.

`Restated` wraps oracle/_build/liboracle.so, the C restatement of AccelEP's
SimDevice arithmetic (oracle/restate.c). `Reference` wraps
oracle/_ref/libaccel_ref.so, the AccelEP reference compiled from its own
sources (oracle/Makefile). Only tests, the smoke check and bench.py's CPU legs
import this module; the product package never does.
"""

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ORACLE_LIB = HERE / "_build" / "liboracle.so"
REF_LIB = HERE / "_ref" / "libaccel_ref.so"
REF_C4_LIB = HERE / "_ref" / "libaccel_ref_c4.so"
# The AccelEP checkout the reference library is built from: ACCEL_REF_ROOT,
# else a directory named `reference` beside this repository's root.
REF_SOURCES = Path(os.environ.get("ACCEL_REF_ROOT", str(HERE.parent.parent / "reference")))

_f32p = ctypes.POINTER(ctypes.c_float)
_i32p = ctypes.POINTER(ctypes.c_int32)
_i64p = ctypes.POINTER(ctypes.c_int64)
_i8p = ctypes.POINTER(ctypes.c_int8)
_u32p = ctypes.POINTER(ctypes.c_uint32)
_i64 = ctypes.c_int64

ACT = {"none": 0, "relu": 1, "gelu": 2}


def build(quiet=True):
    """Builds the restatement, and the reference where its sources exist."""
    cmd = ["make", "-C", str(HERE), f"REF={REF_SOURCES}", "all"]
    out = subprocess.run(cmd, capture_output=quiet, text=True)
    if out.returncode != 0:
        raise RuntimeError(f"oracle build failed:\n{out.stdout}\n{out.stderr}")


def _p(array, ptype):
    if array is None:
        return None
    return array.ctypes.data_as(ptype)


def f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


class _Common:
    """Kernels whose C signature is the same in both libraries."""

    prefix = ""

    def _fn(self, name):
        return getattr(self.lib, self.prefix + name)

    def rmsnorm(self, x, w, rows, dim, eps, row_offset=0):
        x, w = f32(x), f32(w)
        y = np.zeros((rows, dim), dtype=np.float32)
        self._fn("rmsnorm")(_p(x, _f32p), _p(w, _f32p), _p(y, _f32p), rows, dim, ctypes.c_float(eps), row_offset)
        return y

    def rope(self, states, cos_t, sin_t, seq, n_heads, head_dim, position):
        out = f32(states).copy()
        self._fn("rope")(_p(out, _f32p), _p(f32(cos_t), _f32p), _p(f32(sin_t), _f32p), seq, n_heads, head_dim, position)
        return out

    def append_cache(self, src, cache, seq, position, n_heads, head_dim):
        out = f32(cache).copy()
        self._fn("append_cache")(_p(f32(src), _f32p), _p(out, _f32p), seq, position, n_heads, head_dim)
        return out

    def silu_mul(self, gate, up):
        g = f32(gate).copy()
        self._fn("silu_mul")(_p(g, _f32p), _p(f32(up), _f32p), g.size)
        return g

    def sample(self, logits, vocab, temperature, rng, top_k):
        lg = f32(logits)
        chosen = np.full(1, -1, dtype=np.int32)
        state = np.array([rng], dtype=np.uint32)
        self._fn("sample")(_p(lg, _f32p), _p(chosen, _i32p), 0, vocab, ctypes.c_float(temperature), _p(state, _u32p),
                           top_k)
        return int(chosen[0]), int(state[0])

    def matmul(self, a, b):
        a, b = f32(a), f32(b)
        m, k = a.shape
        n = b.shape[1]
        c = np.ones((m, n), dtype=np.float32)
        self._fn("matmul")(_p(a, _f32p), _p(b, _f32p), _p(c, _f32p), m, k, n)
        return c

    def transpose(self, src):
        s = f32(src)
        rows, cols = s.shape
        d = np.zeros((cols, rows), dtype=np.float32)
        self._fn("transpose")(_p(s, _f32p), _p(d, _f32p), rows, cols)
        return d

    def gemm_epilogue(self, c, alpha, bias, bias_shape, beta, act):
        out = f32(c).copy()
        m, n = out.shape
        shape = np.array(bias_shape if bias is not None else [0], dtype=np.int64)
        b = f32(bias) if bias is not None else None
        rc = self._fn("gemm_epilogue")(_p(out, _f32p), m, n, ctypes.c_float(alpha), _p(b, _f32p), _p(shape, _i64p),
                                       len(bias_shape) if bias is not None else 0, ctypes.c_float(beta), ACT[act])
        if rc != 0:
            raise ValueError("epilogue rejected")
        return out

    def matmul_quantized(self, a, q, scale, zero, shape, axis, offset, m, k, n):
        a = f32(a)
        q = np.ascontiguousarray(q, dtype=np.int8)
        scale = f32(scale)
        zero = None if zero is None else np.ascontiguousarray(zero, dtype=np.int8)
        shp = np.array(shape, dtype=np.int64)
        c = np.ones((m, n), dtype=np.float32)
        rc = self._fn("matmul_quantized" if self.prefix == "ref_" else "matmul_q")(
            _p(a, _f32p), _p(q, _i8p), _p(scale, _f32p), _p(zero, _i8p), _p(shp, _i64p), len(shape), axis, offset,
            _p(c, _f32p), m, k, n)
        if rc != 0:
            raise ValueError("quantized matmul rejected")
        return c

    def execute_matmul_q(self, x, q, scale, zero=None, axis=1, act="none", residual=None):
        x = f32(x)
        m, k = x.shape
        q = np.ascontiguousarray(q, dtype=np.int8)
        n = q.shape[1]
        out = np.zeros((m, n), dtype=np.float32)
        z = None if zero is None else np.ascontiguousarray(zero, dtype=np.int8)
        r = None if residual is None else f32(residual)
        rc = self._fn("execute_matmul_q")(_p(x, _f32p), m, k, _p(q, _i8p), _p(f32(scale), _f32p), _p(z, _i8p), axis, n,
                                          ACT[act], _p(r, _f32p), _p(out, _f32p))
        if rc != 0:
            raise ValueError("execute rejected")
        return out


def _declare(lib, prefix, names):
    for name, restype, argtypes in names:
        fn = getattr(lib, prefix + name)
        fn.restype = restype
        fn.argtypes = argtypes


_KERNEL_SIGS = [
    ("rmsnorm", None, [_f32p, _f32p, _f32p, _i64, _i64, ctypes.c_float, _i64]),
    ("rope", None, [_f32p, _f32p, _f32p, _i64, _i64, _i64, _i64]),
    ("append_cache", None, [_f32p, _f32p, _i64, _i64, _i64, _i64]),
    ("silu_mul", None, [_f32p, _f32p, _i64]),
    ("sample", None, [_f32p, _i32p, _i64, _i64, ctypes.c_float, _u32p, ctypes.c_int]),
    ("matmul", None, [_f32p, _f32p, _f32p, _i64, _i64, _i64]),
    ("transpose", None, [_f32p, _f32p, _i64, _i64]),
    ("gemm_epilogue", ctypes.c_int,
     [_f32p, _i64, _i64, ctypes.c_float, _f32p, _i64p, ctypes.c_int, ctypes.c_float, ctypes.c_int]),
    ("execute_matmul_q", ctypes.c_int, [_f32p, _i64, _i64, _i8p, _f32p, _i8p, _i64, _i64, ctypes.c_int, _f32p, _f32p]),
]


class Restated(_Common):
    """The C restatement (oracle/restate.c)."""

    prefix = "orc_"

    def __init__(self, path=ORACLE_LIB):
        if not Path(path).is_file():
            build()
        self.lib = ctypes.CDLL(str(path))
        sigs = list(_KERNEL_SIGS) + [
            ("embed", ctypes.c_int, [_i32p, _i64, _f32p, _f32p, _i64, _i64, _i64]),
            ("attend", None, [_f32p, _f32p, _f32p, _f32p, _f32p, _i64, _i64, _i64, _i64, _i64]),
            ("add", None, [_f32p, _f32p, _i64]),
            ("matmul_q", ctypes.c_int,
             [_f32p, _i8p, _f32p, _i8p, _i64p, ctypes.c_int, _i64, _i64, _f32p, _i64, _i64, _i64]),
            ("mlp_block", ctypes.c_int,
             [_f32p, _i64, _i64, _i64, _i8p, _f32p, _i8p, _f32p, _f32p, ctypes.c_float, _f32p, _f32p, _f32p]),
            ("llama_create", ctypes.c_void_p, [_i32p, ctypes.c_float, ctypes.c_float]),
            ("llama_destroy", None, [ctypes.c_void_p]),
            ("llama_weight", ctypes.c_int, [ctypes.c_void_p, ctypes.c_int32, ctypes.c_int32, _f32p, _i64, _i64]),
            ("llama_forward_ids", ctypes.c_int, [ctypes.c_void_p, _i32p, ctypes.c_int32, ctypes.c_int32]),
            ("llama_generate", ctypes.c_int,
             [ctypes.c_void_p, _i32p, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_float, ctypes.c_uint32,
              ctypes.c_int32, _i32p, _i32p, _f32p]),
            ("llama_logits", _f32p, [ctypes.c_void_p]),
            ("llama_filled", ctypes.c_int32, [ctypes.c_void_p]),
            ("llama_cache", _f32p, [ctypes.c_void_p, ctypes.c_int32, ctypes.c_int32]),
        ]
        _declare(self.lib, self.prefix, sigs)

    def embed(self, ids, id_offset, table, seq):
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        table = f32(table)
        vocab, hidden = table.shape
        out = np.zeros((seq, hidden), dtype=np.float32)
        rc = self.lib.orc_embed(_p(ids, _i32p), id_offset, _p(table, _f32p), _p(out, _f32p), seq, hidden, vocab)
        if rc != 0:
            raise ValueError("token id is outside the vocabulary")
        return out

    def attend(self, q, k, v, seq, position, heads, kv_heads, head_dim):
        q, k, v = f32(q), f32(k), f32(v)
        scores = np.zeros(position + seq, dtype=np.float32)
        out = np.zeros((seq, heads, head_dim), dtype=np.float32)
        self.lib.orc_attend(_p(q, _f32p), _p(k, _f32p), _p(v, _f32p), _p(scores, _f32p), _p(out, _f32p), seq, position,
                            heads, kv_heads, head_dim)
        return out

    def add(self, dest, extra):
        d = f32(dest).copy()
        self.lib.orc_add(_p(d, _f32p), _p(f32(extra), _f32p), d.size)
        return d

    def mlp_block(self, x, w1, s1, w2, s2, gamma, eps):
        x = f32(x)
        m, hidden = x.shape
        inter = w1.shape[1]
        h = np.zeros((m, inter), dtype=np.float32)
        s = np.zeros((m, hidden), dtype=np.float32)
        out = np.zeros((m, hidden), dtype=np.float32)
        rc = self.lib.orc_mlp_block(_p(x, _f32p), m, hidden, inter, _p(np.ascontiguousarray(w1), _i8p),
                                    _p(f32(s1), _f32p), _p(np.ascontiguousarray(w2), _i8p), _p(f32(s2), _f32p),
                                    _p(f32(gamma), _f32p), ctypes.c_float(eps), _p(h, _f32p), _p(s, _f32p),
                                    _p(out, _f32p))
        if rc != 0:
            raise ValueError("mlp block rejected")
        return out, s


class Reference(_Common):
    """The AccelEP reference compiled from source (oracle/_ref)."""

    prefix = "ref_"
    llama_api = True  # LlamaHandle drives the reference's own accel_llama_* API

    def __init__(self, path=REF_LIB):
        if not Path(path).is_file():
            if REF_SOURCES.is_dir():
                build()
            if not Path(path).is_file():
                raise FileNotFoundError(f"{path} is not built")
        self.lib = ctypes.CDLL(str(path))
        sigs = [(n, ctypes.c_int, a) if n not in ("gemm_epilogue", "execute_matmul_q") else (n, r, a)
                for n, r, a in _KERNEL_SIGS]
        sigs += [
            ("embed", ctypes.c_int, [_i32p, _i64, _f32p, _f32p, _i64, _i64, _i64]),
            ("attention", ctypes.c_int, [_f32p, _f32p, _f32p, _f32p, _f32p, _i64, _i64, _i64, _i64, _i64]),
            ("residual_add", ctypes.c_int, [_f32p, _f32p, _i64]),
            ("reference_matmul", None, [_f32p, _f32p, _f32p, _i64, _i64, _i64]),
            ("matmul_quantized", ctypes.c_int,
             [_f32p, _i8p, _f32p, _i8p, _i64p, ctypes.c_int, _i64, _i64, _f32p, _i64, _i64, _i64]),
            ("mlp_block", ctypes.c_int,
             [_f32p, _i64, _i64, _i64, _i8p, _f32p, _i8p, _f32p, _f32p, ctypes.c_float, _f32p, _f32p]),
            ("last_error", ctypes.c_char_p, []),
            ("reset_stats", None, []),
            ("stats", None, [_i64p]),
        ]
        _declare(self.lib, self.prefix, sigs)
        _bind_llama_api(self.lib)

    def error(self):
        return self.lib.ref_last_error().decode()

    def embed(self, ids, id_offset, table, seq):
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        table = f32(table)
        vocab, hidden = table.shape
        out = np.zeros((seq, hidden), dtype=np.float32)
        if self.lib.ref_embed(_p(ids, _i32p), id_offset, _p(table, _f32p), _p(out, _f32p), seq, hidden, vocab) != 0:
            raise ValueError(self.error())
        return out

    def attend(self, q, k, v, seq, position, heads, kv_heads, head_dim):
        q, k, v = f32(q), f32(k), f32(v)
        scores = np.zeros(position + seq, dtype=np.float32)
        out = np.zeros((seq, heads, head_dim), dtype=np.float32)
        if self.lib.ref_attention(_p(q, _f32p), _p(k, _f32p), _p(v, _f32p), _p(scores, _f32p), _p(out, _f32p), seq,
                                  position, heads, kv_heads, head_dim) != 0:
            raise ValueError(self.error())
        return out

    def add(self, dest, extra):
        d = f32(dest).copy()
        self.lib.ref_residual_add(_p(d, _f32p), _p(f32(extra), _f32p), d.size)
        return d

    def mlp_block(self, x, w1, s1, w2, s2, gamma, eps):
        x = f32(x)
        m, hidden = x.shape
        inter = w1.shape[1]
        s = np.zeros((m, hidden), dtype=np.float32)
        out = np.zeros((m, hidden), dtype=np.float32)
        rc = self.lib.ref_mlp_block(_p(x, _f32p), m, hidden, inter, _p(np.ascontiguousarray(w1), _i8p),
                                    _p(f32(s1), _f32p), _p(np.ascontiguousarray(w2), _i8p), _p(f32(s2), _f32p),
                                    _p(f32(gamma), _f32p), ctypes.c_float(eps), _p(s, _f32p), _p(out, _f32p))
        if rc != 0:
            raise ValueError(self.error())
        return out, s

    def stats(self):
        out = np.zeros(9, dtype=np.int64)
        self.lib.ref_stats(_p(out, _i64p))
        keys = ("matmul_ops", "gemm_ops", "kernel_matmuls", "relu", "gelu", "add", "transposes", "bytes_to_device",
                "bytes_to_host")
        return dict(zip(keys, (int(v) for v in out)))


class ReferenceLlamaTiming:
    """The reference's Llama alone (oracle/_ref/libaccel_ref_c4.so: its
    src/llama_model.cc unmodified, plus ref_llama_fill_context, which places a
    model at a given context length without running the forwards that would
    fill it). bench.py times the reference's decode deep into the context
    with it; nothing checks values through it."""

    llama_api = True

    def __init__(self, path=REF_C4_LIB):
        if not Path(path).is_file():
            if REF_SOURCES.is_dir():
                build()
            if not Path(path).is_file():
                raise FileNotFoundError(f"{path} is not built")
        self.lib = ctypes.CDLL(str(path))
        _bind_llama_api(self.lib)
        self.lib.ref_llama_fill_context.restype = ctypes.c_int
        self.lib.ref_llama_fill_context.argtypes = [ctypes.c_void_p, ctypes.c_int32, ctypes.c_uint32]


class LlamaConfig(ctypes.Structure):
    """AccelLlamaConfig (include/accel/sim_api.h:44-54)."""

    _fields_ = [("vocab", ctypes.c_int32), ("hidden", ctypes.c_int32), ("layers", ctypes.c_int32),
                ("heads", ctypes.c_int32), ("kv_heads", ctypes.c_int32), ("intermediate", ctypes.c_int32),
                ("context", ctypes.c_int32), ("eps", ctypes.c_float), ("rope_theta", ctypes.c_float)]


def _bind_llama_api(lib):
    lib.accel_llama_create.restype = ctypes.c_void_p
    lib.accel_llama_create.argtypes = [ctypes.POINTER(LlamaConfig)]
    lib.accel_llama_destroy.argtypes = [ctypes.c_void_p]
    lib.accel_llama_weight.restype = ctypes.c_int
    lib.accel_llama_weight.argtypes = [ctypes.c_void_p, ctypes.c_int32, ctypes.c_int32, _f32p, _i64, _i64]
    lib.accel_llama_generate.restype = ctypes.c_int
    lib.accel_llama_generate.argtypes = [ctypes.c_void_p, _i32p, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
                                         ctypes.c_float, ctypes.c_uint32, ctypes.c_int32, _i32p, _i32p]
    lib.accel_llama_forward_ids.restype = ctypes.c_int
    lib.accel_llama_forward_ids.argtypes = [ctypes.c_void_p, _i32p, ctypes.c_int32, ctypes.c_int32]
    lib.accel_llama_logit_max_abs.restype = ctypes.c_int
    lib.accel_llama_logit_max_abs.argtypes = [ctypes.c_void_p, _f32p, ctypes.c_int32, _f32p]
    lib.accel_llama_last_error.restype = ctypes.c_char_p
    lib.accel_sim_reset_stats.restype = None
    lib.accel_sim_matmuls.restype = ctypes.c_int64
    lib.accel_sim_bytes_to_device.restype = ctypes.c_int64
    lib.accel_sim_bytes_to_host.restype = ctypes.c_int64


class LlamaHandle:
    """One model on either checker: `api` is 'orc' (restatement) or 'ref'
    (the reference's own accel_llama_* C API in oracle/_ref)."""

    def __init__(self, owner, cfg):
        self.owner = owner
        self.cfg = cfg
        self.lib = owner.lib
        self.ref = getattr(owner, "llama_api", False)
        if self.ref:
            c = LlamaConfig(cfg["vocab"], cfg["hidden"], cfg["layers"], cfg["heads"], cfg["kv_heads"],
                            cfg["intermediate"], cfg["context"], cfg["eps"], cfg["rope_theta"])
            self.h = self.lib.accel_llama_create(ctypes.byref(c))
        else:
            arr = np.array([cfg["vocab"], cfg["hidden"], cfg["layers"], cfg["heads"], cfg["kv_heads"],
                            cfg["intermediate"], cfg["context"]], dtype=np.int32)
            self.h = self.lib.orc_llama_create(_p(arr, _i32p), ctypes.c_float(cfg["eps"]),
                                               ctypes.c_float(cfg["rope_theta"]))
        if not self.h:
            raise RuntimeError("llama create failed")

    def close(self):
        if self.h:
            (self.lib.accel_llama_destroy if self.ref else self.lib.orc_llama_destroy)(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def weight(self, kind, layer, values):
        a = f32(values)
        rows, cols = (a.shape[0], 1) if a.ndim == 1 else a.shape
        fn = self.lib.accel_llama_weight if self.ref else self.lib.orc_llama_weight
        if fn(self.h, kind, layer, _p(a, _f32p), rows, cols) != 0:
            raise RuntimeError("weight rejected")

    def load(self, weights):
        for (kind, layer), values in weights.items():
            self.weight(kind, layer, values)

    def forward_ids(self, ids, reset):
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        fn = self.lib.accel_llama_forward_ids if self.ref else self.lib.orc_llama_forward_ids
        if fn(self.h, _p(ids, _i32p), ids.size, 1 if reset else 0) != 0:
            raise RuntimeError("forward rejected")

    def fill_context(self, rows, seed=1):
        """ReferenceLlamaTiming only: the model's cache holds `rows` rows."""
        if self.lib.ref_llama_fill_context(self.h, rows, seed) != 0:
            raise RuntimeError(self.lib.accel_llama_last_error().decode())

    def logits(self):
        if self.ref:
            raise RuntimeError("the reference API keeps logits on its device; use logit_max_abs")
        ptr = self.lib.orc_llama_logits(self.h)
        return np.ctypeslib.as_array(ptr, shape=(self.cfg["vocab"],)).copy()

    def logit_max_abs(self, reference_row):
        out = np.zeros(1, dtype=np.float32)
        row = f32(reference_row)
        if self.lib.accel_llama_logit_max_abs(self.h, _p(row, _f32p), row.size, _p(out, _f32p)) != 0:
            raise RuntimeError(self.lib.accel_llama_last_error().decode())
        return float(out[0])

    def cache(self, layer, which):
        if self.ref:
            raise RuntimeError("the reference API does not expose its cache")
        ptr = self.lib.orc_llama_cache(self.h, layer, which)
        n = self.cfg["context"] * self.cfg["kv_heads"] * (self.cfg["hidden"] // self.cfg["heads"])
        return np.ctypeslib.as_array(ptr, shape=(n,)).copy()

    def generate(self, prompt, max_new, eos_id=-1, temperature=0.0, seed=0, top_k=0, want_gaps=False):
        prompt = np.ascontiguousarray(prompt, dtype=np.int32)
        out = np.zeros(max(1, max_new), dtype=np.int32)
        count = np.zeros(1, dtype=np.int32)
        gaps = np.zeros(max(1, max_new), dtype=np.float32) if want_gaps else None
        if self.ref:
            rc = self.lib.accel_llama_generate(self.h, _p(prompt, _i32p), prompt.size, max_new, eos_id,
                                               ctypes.c_float(temperature), seed, top_k, _p(out, _i32p),
                                               _p(count, _i32p))
        else:
            rc = self.lib.orc_llama_generate(self.h, _p(prompt, _i32p), prompt.size, max_new, eos_id,
                                             ctypes.c_float(temperature), seed, top_k, _p(out, _i32p),
                                             _p(count, _i32p), _p(gaps, _f32p))
        if rc != 0:
            raise RuntimeError("generate rejected")
        n = int(count[0])
        return (out[:n].copy(), gaps[:n].copy()) if want_gaps else out[:n].copy()
