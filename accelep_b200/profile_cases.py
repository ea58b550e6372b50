"""Times single kernels of the backend on fixed cases, for profiling.

    python -m accelep_b200.profile_cases gemm [--path auto|tc|gemv|simt] [--shapes decode|prefill|c5|all]
    python -m accelep_b200.profile_cases attention [--batch 32] [--len 1280] [--kind fused|split|prefill]
    python -m accelep_b200.profile_cases step [--reps 3]
    python -m accelep_b200.profile_cases mlp [--reps 20]
    python -m accelep_b200.profile_cases list

Each case is launched `reps` times from one captured CUDA graph (no host
overhead between launches), after warm-up, and timed with CUDA events on the
capturing stream. Several input copies are rotated so that each launch reads
its operands from HBM rather than L2. The same commands run under ncu for the
summaries in profiles/.
"""

import argparse
import ctypes
import json

import numpy as np
import torch

from . import kernels as K
from . import synthetic as syn

GEMM_SHAPES = {
    "decode": [("qkv", 32, 576, 960), ("o", 32, 576, 576), ("gate_up", 32, 576, 3072), ("down", 32, 1536, 576),
               ("lm_head", 32, 576, 49152)],
    "prefill": [("p_qkv", 16384, 576, 960), ("p_gate_up", 16384, 576, 3072), ("p_down", 16384, 1536, 576)],
    "c5": [("c5_m1_k4096", 1, 4096, 4096), ("c5_m16_k4096", 16, 4096, 4096), ("c5_m1_k16384", 1, 16384, 16384),
           ("c5_m16_k16384", 16, 16384, 16384), ("c5_m128_k8192", 128, 8192, 8192),
           ("c5_m2048_k8192", 2048, 8192, 8192)],
}


def _time_graph(launch, reps, stream):
    """Captures `reps` calls of launch(i) into one graph; returns us per call."""
    for i in range(3):
        launch(i)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for i in range(reps):
            launch(i)
    graph.replay()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    graph.replay()
    end.record(stream)
    end.synchronize()
    return start.elapsed_time(end) * 1000.0 / reps


def gemm_case(name, m, k, n, reps, copies=None):
    """int8 product C = A @ dequant(W) at one shape; returns a result row."""
    weight_bytes = k * n
    copies = copies or max(1, min(8, int(np.ceil(300e6 / max(weight_bytes, 1)))))
    x, w, s = syn.int8_gemm(m, k, n, 1)
    xs = torch.from_numpy(x).cuda()
    ws_ = [torch.from_numpy(w).cuda() for _ in range(copies)]
    st = torch.from_numpy(s).cuda()
    out = torch.zeros(m, n, device="cuda")
    need = K.load().accel_b200_matmul_q8_workspace(m, k, n)
    work = torch.zeros(max(need, 1), dtype=torch.uint8, device="cuda")
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        us = _time_graph(lambda i: K.matmul_q8(xs, ws_[i % copies], st, out=out, workspace=work), reps, stream)
    nbytes = k * n + 4 * n + 4 * m * k + 4 * m * n
    return {"case": name, "m": m, "k": k, "n": n, "us": round(us, 3), "gbs": round(nbytes / us / 1e3, 1),
            "tflops": round(2 * m * k * n / us / 1e6, 2), "weight_copies": copies}


def decode_products(batch=32, layers=30, hidden=576, inter=1536, q_out=576, kv_out=192, vocab=49152, seed=5):
    """The int8 products of one decode step of the C4 model at its shapes:
    per layer the fused q|k|v projection fed by RmsNorm rows, the output
    projection (+ residual), the fused gate|up projection fed by RmsNorm rows
    and the down projection fed by SiluMul rows (+ residual), then the LM head
    fed by RmsNorm rows; synthetic weights of the same shapes. (The engine
    stores gate|up in column pairs and applies SiluMul in the gate|up
    epilogue, so its down product reads the activations directly; the
    product count and weight bytes are the same.)
    Returns (launch(i), algorithmic bytes per step, launches per step): the
    algorithmic bytes of a product are its int8 weights, scales, fp32 A rows
    read, C rows written and residual rows read."""
    g = torch.Generator(device="cuda").manual_seed(seed)

    def plane(k, n):
        w = torch.randint(-127, 128, (k, n), dtype=torch.int8, device="cuda", generator=g)
        s = torch.rand(n, device="cuda", generator=g) * 1e-3 + 1e-4
        return w, s

    layers_w = [(plane(hidden, q_out + 2 * kv_out), plane(q_out, hidden), plane(hidden, 2 * inter),
                 plane(inter, hidden)) for _ in range(layers)]
    head = plane(hidden, vocab)
    x = torch.randn(batch, hidden, device="cuda")
    attn = torch.randn(batch, q_out, device="cuda")
    qkv = torch.empty(batch, q_out + 2 * kv_out, device="cuda")
    gu = torch.randn(batch, 2 * inter, device="cuda")
    hid = torch.randn(batch, hidden, device="cuda")
    logits = torch.empty(batch, vocab, device="cuda")
    lib = K.load()
    need = max(lib.accel_b200_matmul_q8_rmsnorm_workspace(batch, hidden, vocab),
               lib.accel_b200_matmul_q8_silu_workspace(batch, inter, hidden))
    gamma = torch.rand(hidden, device="cuda", generator=g) + 0.5
    work = torch.zeros(need, dtype=torch.uint8, device="cuda")
    res = K.make_epilogue(residual=hid)
    out_h = torch.empty(batch, hidden, device="cuda")

    def launch(_):
        for (wqkv, wo, wgu, wd) in layers_w:
            K.matmul_q8_rmsnorm(x, gamma, 1e-5, wqkv[0], wqkv[1], out=qkv, workspace=work)
            K.matmul_q8(attn, wo[0], wo[1], epilogue=res, out=out_h, workspace=work)
            K.matmul_q8_rmsnorm(x, gamma, 1e-5, wgu[0], wgu[1], out=gu, workspace=work)
            K.matmul_q8_silu(gu, wd[0], wd[1], epilogue=res, out=out_h, workspace=work)
        K.matmul_q8_rmsnorm(x, gamma, 1e-5, head[0], head[1], out=logits, workspace=work)

    def nbytes(m, k, n, residual=False):
        return k * n + 4 * n + 4 * m * k + 4 * m * n + (4 * m * n if residual else 0)

    down = inter * hidden + 4 * hidden + 4 * batch * 2 * inter + 8 * batch * hidden  # reads gate|up rows
    per_layer = (nbytes(batch, hidden, q_out + 2 * kv_out) + nbytes(batch, q_out, hidden, True) +
                 nbytes(batch, hidden, 2 * inter) + down)
    total = layers * per_layer + nbytes(batch, hidden, vocab)
    launch._keep = (layers_w, head, x, attn, qkv, gu, hid, logits, work, res, out_h, gamma)
    return launch, total, 4 * layers + 1


def mlp_case(reps):
    """C2: the 4-block int8 MLP chain at batch 256 (17.2 GFLOP of products):
    per block Gelu(x @ W1), (h @ W2) + x, RmsNorm; one CUDA graph."""
    x, blocks = syn.mlp_stack()
    dev = [tuple(torch.from_numpy(np.ascontiguousarray(a)).cuda() for a in b) for b in blocks]
    h0 = torch.from_numpy(x).cuda()
    m, hidden = h0.shape
    inter = blocks[0][0].shape[1]
    t = torch.empty(m, inter, device="cuda")
    s = torch.empty(m, hidden, device="cuda")
    hs = [torch.empty(m, hidden, device="cuda") for _ in dev]
    lib = K.load()
    work = torch.zeros(max(lib.accel_b200_matmul_q8_workspace(m, hidden, inter),
                           lib.accel_b200_matmul_q8_workspace(m, inter, hidden)), dtype=torch.uint8, device="cuda")
    gelu = K.make_epilogue(act="gelu")
    res = [K.make_epilogue(residual=h0 if i == 0 else hs[i - 1]) for i in range(len(dev))]

    def launch(_):
        h = h0
        for i, (w1, s1, w2, s2, gamma) in enumerate(dev):
            K.matmul_q8(h, w1, s1, epilogue=gelu, out=t, workspace=work)
            K.matmul_q8(t, w2, s2, epilogue=res[i], out=s, workspace=work)
            check_rc = lib.accel_b200_rmsnorm(K._p(s), K._p(gamma), K._p(hs[i]), m, hidden, ctypes.c_float(1e-5), 0,
                                              K._s())
            assert check_rc == 0
            h = hs[i]

    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        us = _time_graph(launch, reps, stream)
    flops = 4 * 2 * (2.0 * m * hidden * inter)
    return {"case": "c2_mlp_4blocks_b256", "us": round(us, 2), "tflops": round(flops / us / 1e6, 1)}


def step_case(reps):
    stream = torch.cuda.Stream()
    launch, nbytes, count = decode_products()
    with torch.cuda.stream(stream):
        us = _time_graph(launch, reps, stream)
    return {"case": "decode_step_products", "launches": count, "us_per_step": round(us, 2),
            "us_per_launch": round(us / count, 3), "bytes_per_step": nbytes, "gbs": round(nbytes / us / 1e3, 1)}


def attention_case(batch, length, reps, kind="fused", context=2048, heads=9, kv_heads=3, head_dim=64):
    """Decode attention of `batch` sequences at context length `length` over
    head-major caches: the fused step (Rope, AppendCache, attention) or the
    split-KV kernel alone. Bytes counted: the key and value rows read."""
    copies = 4
    kc = [torch.randn(batch, kv_heads, context, head_dim, device="cuda") for _ in range(copies)]
    vc = [torch.randn(batch, kv_heads, context, head_dim, device="cuda") for _ in range(copies)]
    stream = torch.cuda.Stream()
    if kind == "prefill":
        # `batch` prompts of `length` rows each, attending causally.
        rows = batch * length
        q = torch.randn(rows, heads * head_dim, device="cuda")
        first = torch.arange(batch, dtype=torch.int32, device="cuda") * length
        count = torch.full((batch,), length, dtype=torch.int32, device="cuda")
        pos0 = torch.zeros(batch, dtype=torch.int32, device="cuda")
        out = torch.zeros(rows, heads * head_dim, device="cuda")
        with torch.cuda.stream(stream):
            us = _time_graph(lambda i: K.attention_prefill(q, kc[i % copies], vc[i % copies], first, count, pos0, heads,
                                                           kv_heads, out=out, max_rows=length), reps, stream)
        flops = 4.0 * batch * heads * head_dim * length * (length + 1) / 2
        return {"case": f"attention_prefill_b{batch}_len{length}", "us": round(us, 3),
                "tflops": round(flops / us / 1e6, 2)}
    if kind == "fused":
        qkv = torch.randn(batch, (heads + 2 * kv_heads) * head_dim, device="cuda")
        pos = torch.full((batch,), length - 1, dtype=torch.int32, device="cuda")
        ang = torch.arange(context, dtype=torch.float64, device="cuda")[:, None] * torch.ones(head_dim, device="cuda",
                                                                                              dtype=torch.float64)
        cos_t, sin_t = torch.cos(ang * 1e-3).float(), torch.sin(ang * 1e-3).float()
        out = torch.zeros(batch, heads * head_dim, device="cuda")
        with torch.cuda.stream(stream):
            us = _time_graph(lambda i: K.decode_attention(qkv, pos, heads, kv_heads, cos_t, sin_t, kc[i % copies],
                                                          vc[i % copies], out=out), reps, stream)
    else:
        q = torch.randn(batch, heads * head_dim, device="cuda")
        lens = torch.full((batch,), length, dtype=torch.int32, device="cuda")
        work = K.attention_decode_workspace(batch, heads, kv_heads, context)
        with torch.cuda.stream(stream):
            us = _time_graph(lambda i: K.attention_decode(q, kc[i % copies], vc[i % copies], lens, heads, kv_heads,
                                                          head_dim, context, head_major=True, workspace=work),
                             reps, stream)
    nbytes = batch * length * 2 * kv_heads * head_dim * 4
    return {"case": f"attention_{kind}_b{batch}_len{length}", "us": round(us, 3), "gbs": round(nbytes / us / 1e3, 1)}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("what", choices=["gemm", "attention", "step", "mlp", "list"])
    ap.add_argument("--path", default="auto", choices=["auto", "tc", "gemv", "simt"])
    ap.add_argument("--shapes", default="decode", choices=["decode", "prefill", "c5", "all"])
    ap.add_argument("--batch", type=int, default=32)
    ap.add_argument("--len", type=int, default=1280)
    ap.add_argument("--reps", type=int, default=50)
    ap.add_argument("--kind", default="fused", choices=["fused", "split", "prefill"])
    ap.add_argument("--only", default="", help="run one named gemm case")
    args = ap.parse_args()
    if args.what == "list":
        print(json.dumps(GEMM_SHAPES))
        return
    torch.cuda.set_device(0)
    if args.what == "gemm":
        K.set_q8_path({"auto": 0, "simt": 1, "tc": 2, "gemv": 3}[args.path])
        groups = list(GEMM_SHAPES) if args.shapes == "all" else [args.shapes]
        for group in groups:
            for name, m, k, n in GEMM_SHAPES[group]:
                if args.only and name != args.only:
                    continue
                reps = args.reps if m * k * n < 1e10 else max(3, args.reps // 10)
                print(json.dumps(dict(gemm_case(name, m, k, n, reps), path=args.path)), flush=True)
        K.set_q8_path(0)
    elif args.what == "mlp":
        print(json.dumps(mlp_case(args.reps)), flush=True)
    elif args.what == "step":
        print(json.dumps(step_case(args.reps)), flush=True)
    else:
        print(json.dumps(attention_case(args.batch, args.len, args.reps, args.kind)), flush=True)


if __name__ == "__main__":
    main()
