"""Seeded synthetic inputs for the five workloads this backend is measured on.

No checkpoint or dataset is involved: every tensor is drawn from
numpy.random.default_rng(seed) in a fixed order, so the same seed gives the
same bytes on any machine with the same numpy. The shapes and distributions
follow the AccelEP workloads:

  C1  X [64, 576] ~ N(0, 1) times int8 W [576, 1536] in [-127, 127] with
      per-output-column scales U[1e-3, 1e-2], zero point 0, then Relu.
  C2  four MLP blocks, batch 256, hidden 1024 -> 4096 -> 1024, int8 weights
      with per-column scales, exact Gelu, residual add, RMSNorm (gamma
      U[0.9, 1.1], eps 1e-5).
  C3  a SmolLM2-135M-shaped Llama with N(0, 0.02) fp32 weights, unit norms,
      tied embedding / LM head; 4 prompt ids, 64 greedy steps.
  C4  the same model with every linear weight quantized per output row to
      int8 (scale = max|w| / 127); 32 prompts of 512 ids, decoded to 2048.
  C5  X [M, K] ~ N(0, 1) times int8 W [K, N] with per-column scales.
"""

import numpy as np

# Weight kinds of the Llama C API (accel_llama_weight).
W_EMBED, W_FINAL_NORM, W_LM_HEAD = 1, 2, 3
W_ATTN_NORM, W_POST_NORM = 4, 5
W_Q, W_K, W_V, W_O, W_GATE, W_UP, W_DOWN = 6, 7, 8, 9, 10, 11, 12
LINEAR_KINDS = (W_Q, W_K, W_V, W_O, W_GATE, W_UP, W_DOWN)

SMOLLM2_135M = dict(vocab=49152, hidden=576, layers=30, heads=9, kv_heads=3, intermediate=1536, context=2048,
                    eps=1e-5, rope_theta=100000.0)

# A small model of the same family, for checks the CPU checker finishes in seconds.
TINY_LLAMA = dict(vocab=512, hidden=64, layers=2, heads=4, kv_heads=2, intermediate=128, context=64, eps=1e-5,
                  rope_theta=10000.0)


def linear_shape(cfg, kind):
    """Hugging Face [out, in] shape of a linear weight."""
    hidden, inter = cfg["hidden"], cfg["intermediate"]
    head_dim = hidden // cfg["heads"]
    q_out, kv_out = cfg["heads"] * head_dim, cfg["kv_heads"] * head_dim
    return {W_Q: (q_out, hidden), W_K: (kv_out, hidden), W_V: (kv_out, hidden), W_O: (hidden, q_out),
            W_GATE: (inter, hidden), W_UP: (inter, hidden), W_DOWN: (hidden, inter)}[kind]


def llama_weights(cfg, seed, std=0.02):
    """fp32 weights keyed by (kind, layer) in Hugging Face layout.

    Draw order: embedding [vocab, hidden], then per layer q, k, v, o, gate, up,
    down. Norm weights are ones. The LM head is the embedding (tied) and layer
    -1 marks the model-level tensors.
    """
    rng = np.random.default_rng(seed)
    std = np.float32(std)
    out = {}
    embed = rng.standard_normal((cfg["vocab"], cfg["hidden"]), dtype=np.float32) * std
    out[(W_EMBED, -1)] = embed
    out[(W_FINAL_NORM, -1)] = np.ones(cfg["hidden"], dtype=np.float32)
    out[(W_LM_HEAD, -1)] = embed
    for layer in range(cfg["layers"]):
        out[(W_ATTN_NORM, layer)] = np.ones(cfg["hidden"], dtype=np.float32)
        out[(W_POST_NORM, layer)] = np.ones(cfg["hidden"], dtype=np.float32)
        for kind in LINEAR_KINDS:
            out[(kind, layer)] = rng.standard_normal(linear_shape(cfg, kind), dtype=np.float32) * std
    return out


def quantize_rows(w):
    """Symmetric per-output-row int8: scale = max|w_row| / 127 (fp32),
    q = clip(rint(w / scale), -127, 127)."""
    w = np.ascontiguousarray(w, dtype=np.float32)
    scale = (np.max(np.abs(w), axis=1) / np.float32(127.0)).astype(np.float32)
    scale = np.where(scale > 0, scale, np.float32(1.0)).astype(np.float32)
    q = np.clip(np.rint(w / scale[:, None]), -127, 127).astype(np.int8)
    return q, scale


def dequantize_rows(q, scale):
    """float(q) * scale in fp32, the value the reference's DequantAt gives for
    a zero point of 0."""
    return (q.astype(np.float32) * scale.astype(np.float32)[:, None]).astype(np.float32)


def llama_int8(cfg, seed):
    """C4 weights: (int8 planes, fp32 weights).

    The int8 planes map (kind, layer) -> (q [out, in] int8, scale [out] fp32)
    for every linear weight and the LM head. The fp32 dict holds the
    embedding table and norms unchanged and every quantized weight as its
    dequantized fp32 value, which is what the fp32 reference model is loaded
    with to act as the int8 oracle.
    """
    base = llama_weights(cfg, seed)
    planes = {}
    dense = {}
    for key, value in base.items():
        kind = key[0]
        if kind in LINEAR_KINDS or kind == W_LM_HEAD:
            q, s = quantize_rows(value)
            planes[key] = (q, s)
            dense[key] = dequantize_rows(q, s)
        else:
            dense[key] = value
    return planes, dense


def prompts(cfg, count, length, seed):
    """`count` prompts of `length` uniform ids in [0, vocab)."""
    rng = np.random.default_rng(seed)
    return rng.integers(0, cfg["vocab"], size=(count, length), dtype=np.int64).astype(np.int32)


def int8_gemm(m, k, n, seed):
    """C1 / C5 operands: X [m, k] ~ N(0, 1), W [k, n] int8 in [-127, 127],
    per-column scale [n] ~ U[1e-3, 1e-2]."""
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((m, k), dtype=np.float32)
    w = rng.integers(-127, 128, size=(k, n), dtype=np.int64).astype(np.int8)
    scale = rng.uniform(1e-3, 1e-2, size=n).astype(np.float32)
    return x, w, scale


def mlp_stack(m=256, hidden=1024, inter=4096, blocks=4, seed=2):
    """C2 operands: X [m, hidden], then per block (W1 [hidden, inter], s1,
    W2 [inter, hidden], s2, gamma [hidden])."""
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((m, hidden), dtype=np.float32)
    out = []
    for _ in range(blocks):
        w1 = rng.integers(-127, 128, size=(hidden, inter), dtype=np.int64).astype(np.int8)
        s1 = rng.uniform(1e-3, 1e-2, size=inter).astype(np.float32)
        w2 = rng.integers(-127, 128, size=(inter, hidden), dtype=np.int64).astype(np.int8)
        s2 = rng.uniform(1e-3, 1e-2, size=hidden).astype(np.float32)
        gamma = rng.uniform(0.9, 1.1, size=hidden).astype(np.float32)
        out.append((w1, s1, w2, s2, gamma))
    return x, out
