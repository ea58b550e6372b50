"""Decode throughput of the int8 SmolLM2-135M-shaped Llama on B200.

Workload (C4): 32 independent sequences per GPU, prompts of 512 uniform
random ids, decoded greedily to a 2048 context (1536 new ids each), through
the Llama C API (accel_llama_generate_batch). One step = one whole job:
prefill of the 32 prompts plus the 1536-token decode loop. Weights are
random-init (std 0.02, seeded) quantized per output row to int8; inputs are
synthetic. N GPUs run N independent replicas, each with its own 32
sequences (weak scaling, no data-path collective).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

Prints one JSON line. `--impl reference` times the AccelEP reference's own
CPU path (oracle/_ref, compiled from its sources) on the host cores, on a
sample of the same C4 job extrapolated to the whole job.
"""

import argparse
import ctypes
import json
import multiprocessing as mp
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

from accelep_b200 import synthetic as syn  # noqa: E402

METRIC = "decode tok/s (SmolLM2-shape, int8 W)"
UNIT = "tok/s"
SEQS = 32
PROMPT = 512
CONTEXT = 2048
NEW = CONTEXT - PROMPT
WEIGHT_SEED = 4
PROMPT_SEED = 41
PEAKS = ROOT / "MEASURED_PEAKS.json"
FALLBACK_HBM = 6650.0
# DRAM bytes (read + write) per launch from ncu captures of the same kernels
# (profiles/q8_product_decode_qkv_m32.md: per product kind, weighted by the
# step's launches, 158.0 MB over 121 products; profiles/decode_attention_b32_len1280.md).
PRODUCT_TRAFFIC = 1_305_636
ATTENTION_TRAFFIC = 63_667_968
GEMV_TRAFFIC = 274_861_568  # profiles/q8_gemv_c5_m1_k16384.md


def config(n, seqs=SEQS):
    return {"workload": f"C4: SmolLM2-135M shape, int8 per-row weights, {seqs} seqs/GPU x 512-token prompts, greedy "
                        "decode to 2048 context (1536 new ids per seq); one step = prefill + whole decode",
            "model": "SmolLM2-135M-shaped Llama (30 layers, hidden 576, 9/3 heads, inter 1536, vocab 49152)",
            "global_batch": seqs * n, "seq_len": CONTEXT, "prompt_len": PROMPT, "new_tokens_per_seq": NEW,
            "parallelism": f"replicas x{n} (independent sequences, no collective)",
            "l2": "inputs larger than L2: KV cache 3.0 GB and 135 MB of int8 weights per step"}


def hbm_peak():
    try:
        peaks = json.loads(PEAKS.read_text())
        return float(peaks["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM, "fallback"


class ClockSampler:
    """nvidia-smi clocks and throttle reasons, sampled during the timed region."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 7:
                continue
            try:
                sm.append(float(parts[0]))
                mx.append(float(parts[1]))
            except ValueError:
                continue
            for name, flag in zip(names, parts[3:7]):
                if flag.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(sm)}


# --------------------------------------------------------------- CPU baseline
#
# The reference (oracle/_ref/libaccel_ref_c4.so: AccelEP's own src/llama_model.cc
# on SimDevice, single-threaded) takes minutes per C4 sequence, so both CPU legs
# time a sample of C4's real work and extrapolate to the whole job:
#   - the 512-token prefill as 16 chunks of 32 prompt rows, each a reference
#     forward at its own position over the rows before it (the chunks sum to
#     0.96 of one 512-row forward on the same core: the estimate favours the
#     reference slightly);
#   - the 1536 decode steps as 16 bins of 96 positions over [512, 2048); in
#     each bin WINDOW consecutive reference decode forwards are timed at the
#     bin's middle, the model placed at that context length first
#     (ref_llama_fill_context), so attention runs over the real number of rows.
# Whole-job time of one sequence = sum of chunk times + sum over bins of 96 x
# the bin's mean step time. P concurrent processes (P = min(host cores, 32),
# one sequence each, as the reference would serve 32 sequences on P cores)
# finish 32 sequences in ceil(32 / P) such times.

PREFILL_CHUNK = 32
DECODE_BINS = 16
BIN_WIDTH = NEW // DECODE_BINS
WINDOW = 4
_REF = {}


def _ref_init():
    """Pool initializer: one reference model per process, loaded once."""
    sys.path.insert(0, str(ROOT))
    from oracle.oracle import LlamaHandle, ReferenceLlamaTiming

    cfg = syn.SMOLLM2_135M
    _, dense = syn.llama_int8(cfg, WEIGHT_SEED)
    model = LlamaHandle(ReferenceLlamaTiming(), cfg)
    model.load(dense)
    _REF["model"] = model
    _REF["prompts"] = syn.prompts(cfg, SEQS, PROMPT, PROMPT_SEED)


def _ref_task(task):
    """("prefill", chunk, seq) or ("decode", bin, seq) -> (kind, index, seconds
    per chunk or per decode step)."""
    kind, index, seq = task
    model, prompt = _REF["model"], _REF["prompts"][seq % SEQS]
    if kind == "prefill":
        first = index * PREFILL_CHUNK
        model.fill_context(first, seq + 1)
        t0 = time.perf_counter()
        model.forward_ids(prompt[first:first + PREFILL_CHUNK], False)
        return kind, index, time.perf_counter() - t0
    pos = PROMPT + index * BIN_WIDTH + (BIN_WIDTH - WINDOW) // 2
    model.fill_context(pos, seq + 1)
    t0 = time.perf_counter()
    for i in range(WINDOW):
        model.forward_ids(prompt[i:i + 1], False)
    return kind, index, (time.perf_counter() - t0) / WINDOW


def _job_seconds(results):
    """One sequence's whole C4 job from the sampled chunk and step times
    (several samples of one chunk or bin are averaged)."""
    chunks, bins = {}, {}
    for kind, index, sec in results:
        (chunks if kind == "prefill" else bins).setdefault(index, []).append(sec)
    prefill = sum(statistics.mean(chunks[i]) for i in range(PROMPT // PREFILL_CHUNK))
    decode = sum(BIN_WIDTH * statistics.mean(bins[i]) for i in range(DECODE_BINS))
    return prefill, decode


def c4_tasks():
    return ([("prefill", i, i) for i in range(PROMPT // PREFILL_CHUNK)] +
            [("decode", i, i) for i in range(DECODE_BINS)])


class ReferencePool:
    """`procs` single-threaded reference processes, each holding the C4 model
    (the reference fp32 Llama with the dequantized int8 weights, which is the
    reference's int8 arithmetic)."""

    def __init__(self, procs):
        self.procs = procs
        self.pool = mp.get_context("spawn").Pool(procs, initializer=_ref_init)

    def step(self):
        """One sample of C4 (all 16 chunks and 16 bins, spread over the
        processes, which run concurrently). Returns (tok/s, job seconds per
        sequence, prefill seconds, decode seconds)."""
        results = self.pool.map(_ref_task, c4_tasks(), chunksize=1)
        prefill, decode = _job_seconds(results)
        job = prefill + decode
        rounds = -(-SEQS // self.procs)
        return SEQS * NEW / (rounds * job), job, prefill, decode

    def close(self):
        self.pool.close()
        self.pool.join()


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    cores = os.cpu_count() or 1
    procs = max(1, min(SEQS, cores))
    pool = ReferencePool(procs)
    for _ in range(args.warmup):
        pool.step()
    vals, jobs = [], []
    t_all = time.perf_counter()
    for _ in range(args.steps):
        v, job, prefill, decode = pool.step()
        vals.append(v)
        jobs.append((job, prefill, decode))
    elapsed = time.perf_counter() - t_all
    pool.close()
    value = statistics.median(vals)
    job, prefill, decode = jobs[vals.index(value)] if value in vals else jobs[0]
    sample = (f"C4 extrapolated from a sample of its real work, run on {procs} concurrent single-threaded reference "
              f"processes (oracle/_ref/libaccel_ref_c4.so: AccelEP's src/llama_model.cc on SimDevice, the C4 model "
              f"with dequantized int8 weights): the 512-token prefill as 16 timed 32-row chunks and the 1536 decode "
              f"steps as 16 bins of 96 positions over contexts 512..2047 with {WINDOW} timed steps at each bin's "
              f"middle; one sequence's job = {job:.0f} s (prefill {prefill:.0f} s, decode {decode:.0f} s); 32 "
              f"sequences on {procs} processes = {-(-SEQS // procs)} x that; median of {args.steps} samples")
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000.0 * elapsed / max(1, args.steps),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32 (int8 weights dequantized)",
            "data": "synthetic", "config": config(args.gpus),
            "cpu_baseline": {"value": value, "unit": UNIT, "cores": procs, "kind": "reference", "sample": sample,
                             "extrapolated": True, "job_seconds_per_seq": job},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def cpu_baseline_one_core():
    """bench.py's cpu_baseline leg (rank 0, N = 1): the same C4 sample on one
    reference process, 4 of the 16 chunks and 4 of the 16 bins, with the step
    time linear in the context (least squares over the 4 bins) and the chunks'
    mean for the other chunks. About 15 s of CPU work after the model loads."""
    pool = ReferencePool(1)
    tasks = [("prefill", i, i) for i in (0, 5, 10, 15)] + [("decode", i, i) for i in (1, 5, 10, 14)]
    results = pool.pool.map(_ref_task, tasks, chunksize=1)
    pool.close()
    chunk = statistics.mean(sec for kind, _, sec in results if kind == "prefill")
    pts = [(PROMPT + i * BIN_WIDTH + BIN_WIDTH // 2, sec) for kind, i, sec in results if kind == "decode"]
    slope, icpt = np.polyfit([p for p, _ in pts], [t for _, t in pts], 1)
    decode = sum(icpt + slope * p for p in range(PROMPT, CONTEXT))
    job = (PROMPT // PREFILL_CHUNK) * chunk + decode
    return {"value": NEW / job, "unit": UNIT, "cores": 1, "kind": "reference", "extrapolated": True,
            "job_seconds_per_seq": job,
            "sample": f"one single-threaded reference process (oracle/_ref/libaccel_ref_c4.so, AccelEP's "
                      f"src/llama_model.cc) on C4: 4 of the 16 32-row prefill chunks and {WINDOW} decode steps at each "
                      f"of contexts {', '.join(str(p) for p, _ in pts)}, extrapolated (chunk mean x 16; step time "
                      f"linear in the context, summed over 512..2047) to one sequence's whole job of {job:.0f} s"}


# ------------------------------------------------------------------ B200 arm

def attention_roofline(torch, stream, batch=SEQS, length=1280, reps=50):
    """Times the engine's decode attention launch (Rope, AppendCache and
    attention fused, accel_b200_decode_attention) alone at the workload's mean
    context (1280 rows) with CUDA events on the launching stream; returns
    (algorithmic GB/s, seconds per launch, bytes per launch). Algorithmic
    bytes: the key and value rows read, the new rows written, the q|k|v rows
    read and the output written."""
    from accelep_b200 import kernels as K

    cfg = syn.SMOLLM2_135M
    heads, kvh, hd = cfg["heads"], cfg["kv_heads"], cfg["hidden"] // cfg["heads"]
    kvd = kvh * hd
    with torch.cuda.stream(stream):
        # The engine's head-major cache layout; several copies rotated so each
        # launch reads from HBM, not L2 (4 x 0.8 GB > 126 MB).
        copies = 4
        kc = [torch.randn(batch, kvh, CONTEXT, hd, device="cuda") for _ in range(copies)]
        vc = [torch.randn(batch, kvh, CONTEXT, hd, device="cuda") for _ in range(copies)]
        qkv = torch.randn(batch, (heads + 2 * kvh) * hd, device="cuda")
        pos = torch.full((batch,), length - 1, dtype=torch.int32, device="cuda")
        ang = torch.arange(CONTEXT, dtype=torch.float64, device="cuda")[:, None] * torch.ones(
            hd, dtype=torch.float64, device="cuda") * 1e-3
        cos_t, sin_t = torch.cos(ang).float(), torch.sin(ang).float()
        out = torch.zeros(batch, heads * hd, device="cuda")

        def launch(i):
            K.decode_attention(qkv, pos, heads, kvh, cos_t, sin_t, kc[i % copies], vc[i % copies], out=out)

        for i in range(3):
            launch(i)
        torch.cuda.synchronize()
        # `reps` launches in one CUDA graph (as the engine replays them), so
        # host launch overhead stays out of the per-launch time.
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            for i in range(reps):
                launch(i)
        graph.replay()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        start.record(stream)
        graph.replay()
        end.record(stream)
        end.synchronize()
        del graph
    sec = start.elapsed_time(end) / 1000.0 / reps
    nbytes = batch * (length - 1) * 2 * kvd * 4 + batch * 2 * kvd * 4 + batch * (heads + 2 * kvh) * hd * 4 + \
        batch * heads * hd * 4
    del kc, vc
    return nbytes / sec / 1e9, sec, nbytes


def step_roofline(torch, model, prompts, stream, job_sec, new, peak):
    seqs = len(prompts)
    """The whole decode step against HBM: the job's time minus its prefill
    (a generate of 0 new ids, timed the same way), per decode step, against
    the bytes one step must move at the job's mean context: the int8 weights
    and scales once, every sequence's key and value rows up to its position
    read, the new rows written."""
    model.generate_batch(prompts, 0)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for _ in range(3):
        model.generate_batch(prompts, 0)
    end.record(stream)
    end.synchronize()
    prefill = start.elapsed_time(end) / 1e3 / 3
    step = (job_sec - prefill) / new
    kv_row = 30 * 2 * 3 * 64 * 4  # bytes of one position's keys and values over the 30 layers
    mean_ctx = len(prompts[0]) + (new + 1) / 2.0
    nbytes = 134_479_872 + 818_688 + seqs * mean_ctx * kv_row + seqs * kv_row
    return {"what": "one C4 decode step (job time minus prefill, / new ids) against the bytes it must move at the "
                    "mean context (weights and scales once, KV rows read, new rows written)",
            "prefill_ms": prefill * 1e3, "decode_step_us": step * 1e6, "bytes_per_step": nbytes,
            "achieved": nbytes / step / 1e9, "peak": peak, "unit": "GB/s", "frac": nbytes / step / 1e9 / peak,
            "roofline_tok_s": seqs * peak * 1e9 / nbytes}


def products_roofline(torch, stream, reps=3):
    """Times the decode step's 121 int8 products (C4 shapes, synthetic weights)
    replayed from one CUDA graph, with CUDA events on the launching stream;
    returns (algorithmic GB/s, seconds per launch, bytes per launch) averaged
    over the step's launches."""
    from accelep_b200 import profile_cases as PC

    with torch.cuda.stream(stream):
        launch, nbytes, count = PC.decode_products()
        for i in range(2):
            launch(i)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            launch(0)
        graph.replay()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        start.record(stream)
        for _ in range(reps):
            graph.replay()
        end.record(stream)
        end.synchronize()
        del graph, launch
    sec = start.elapsed_time(end) / 1000.0 / reps / count
    per_launch = nbytes / count
    return per_launch / sec / 1e9, sec, per_launch


def gemv_roofline(torch, reps=20):
    """The C5 dequant GEMV at M=1, K=N=16384 (BASELINE's second metric:
    dequant-GEMV GB/s against HBM), timed as profile_cases times it."""
    from accelep_b200 import profile_cases as PC

    row = PC.gemm_case("c5_m1_k16384", 1, 16384, 16384, reps)
    torch.cuda.empty_cache()
    return row


def tensor_peaks(torch, reps=10):
    """Measured dense tensor peaks of this GPU for the C5 fractions at M >= 128
    (MEASURED_PEAKS.json has bf16 only): cuBLAS int8 (torch._int_mm, int32
    accumulate) and TF32 (fp32 matmul with TF32 allowed) on 8192^3, timed with
    CUDA events. Library GEMMs used only as denominators."""
    n = 8192
    a8 = torch.randint(-127, 128, (n, n), dtype=torch.int8, device="cuda")
    b8 = torch.randint(-127, 128, (n, n), dtype=torch.int8, device="cuda")
    a32 = torch.randn(n, n, device="cuda")
    b32 = torch.randn(n, n, device="cuda")
    out = {}
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = True
    try:
        for name, fn in (("int8_tops", lambda: torch._int_mm(a8, b8)), ("tf32_tflops", lambda: a32 @ b32)):
            for _ in range(3):
                fn()
            start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            torch.cuda.synchronize()
            start.record()
            for _ in range(reps):
                fn()
            end.record()
            end.synchronize()
            out[name] = 2.0 * n ** 3 * reps / (start.elapsed_time(end) / 1e3) / 1e12
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    del a8, b8, a32, b32
    torch.cuda.empty_cache()
    return out


def metric_set(torch, peak_hbm, reps=10):
    """The rest of BASELINE's metric set on one GPU: the C5 sweep grid
    (M in {1, 16, 128, 2048} x K = N in {4096, 8192, 16384}, accel_b200_matmul_q8
    graph-replayed over rotated weight copies larger than L2), C1, the C2 MLP
    chain and C3 (fp32 SmolLM2-135M shape, 4-token prompt, 64 greedy ids)."""
    from accelep_b200 import profile_cases as PC
    from accelep_b200.llama import Llama

    peaks = tensor_peaks(torch)
    grid = []
    for m in (1, 16, 128, 2048):
        for kn in (4096, 8192, 16384):
            row = PC.gemm_case(f"c5_m{m}_k{kn}", m, kn, kn, reps if m < 2048 else 4)
            torch.cuda.empty_cache()
            tops = 8.0 * m * kn * kn / row["us"] / 1e6  # int8 MMA ops: four digit planes per product
            row["frac_hbm"] = round(row["gbs"] / peak_hbm, 3)
            row["frac_int8_tensor"] = round(tops / peaks["int8_tops"], 3)
            grid.append(row)
    c1 = PC.gemm_case("c1_m64_k576_n1536", 64, 576, 1536, 50)
    c1["frac_hbm"] = round(c1["gbs"] / peak_hbm, 3)
    c2 = PC.mlp_case(5)
    cfg = dict(syn.SMOLLM2_135M, context=128)
    model = Llama(cfg)
    model.load_fp32(syn.llama_weights(cfg, 3))
    prompt = syn.prompts(cfg, 1, 4, 11)[0]
    stream = torch.cuda.ExternalStream(model.stream())
    model.generate(prompt, 64)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    ids = model.generate(prompt, 64)
    end.record(stream)
    end.synchronize()
    model.close()
    sec = start.elapsed_time(end) / 1e3
    c3_tps = len(ids) / sec
    weight_bytes = 134_479_872 * 4
    c3 = {"case": "C3 fp32 SmolLM2-135M shape, 4-token prompt + 64 greedy ids (batch 1)", "tok_s": round(c3_tps, 1),
          "roofline_tok_s": round(peak_hbm * 1e9 / weight_bytes, 1),
          "frac_hbm": round(c3_tps * weight_bytes / (peak_hbm * 1e9), 3)}
    return {"tensor_peaks_measured": {k: round(v, 1) for k, v in peaks.items()}, "c5_grid": grid, "c1": c1,
            "c2": c2, "c3": c3}


def c5_sharded(torch, dist, world, rank, reps=10):
    """C5 sweep points with W N-sharded across the ranks
    (accelep_b200/sharded.py), timed with CUDA events, max over ranks. At N > 1
    two ways to assemble Y: "nccl" (local product, NCCL all-gather, transpose
    copy) and "fused" (the product kernel stores its block into every rank's
    Y over NVLink, then a barrier over peer memory). Weights are seeded
    synthetic int8 with per-column scales (each rank draws its own block)."""
    from accelep_b200 import sharded

    out = []
    modes = ("nccl", "fused") if world > 1 else ("local",)
    for m, kn in ((1, 16384), (2048, 8192)):
        k = n = kn
        gen = torch.Generator(device="cuda").manual_seed(1000 + rank)
        nr = n // world
        copies = 2 if m == 1 else 1
        weights = []
        for _ in range(copies):
            w = torch.randint(-127, 128, (k, nr), dtype=torch.int8, device="cuda", generator=gen)
            sc = torch.rand(nr, device="cuda", generator=gen) * 9e-3 + 1e-3
            weights.append((w, sc))
        x = torch.randn(m, k, device="cuda", generator=torch.Generator(device="cuda").manual_seed(7))
        for mode in modes:
            layers = [sharded.ShardedQ8Linear(w, sc, mode="nccl" if mode == "local" else mode) for w, sc in weights]
            stream = torch.cuda.Stream()
            with torch.cuda.stream(stream):
                for i in range(4):
                    layers[i % copies](x)
                torch.cuda.synchronize()
                # `reps` calls in one CUDA graph (host launch cost out of the
                # per-call time; an even count keeps the fused mode's buffer
                # alternation aligned across replays).
                graph = torch.cuda.CUDAGraph()
                with torch.cuda.graph(graph, stream=stream):
                    for i in range(reps):
                        y = layers[i % copies](x)
                graph.replay()
                torch.cuda.synchronize()
                if world > 1:
                    dist.barrier()
                start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                start.record(stream)
                graph.replay()
                end.record(stream)
                end.synchronize()
                del graph
            sec = start.elapsed_time(end) / 1000.0 / reps
            t = torch.tensor([sec], dtype=torch.float64, device="cuda")
            if world > 1:
                dist.all_reduce(t, op=dist.ReduceOp.MAX)
            sec = float(t[0])
            assert y.shape == (m, n)
            bad = any(int(l.status.item()) != 0 for l in layers if l.status is not None)
            out.append({"mode": mode, "m": m, "k": k, "n": n, "us_per_call": sec * 1e6,
                        "weight_gbs_all_ranks": k * n / sec / 1e9,
                        "tflops_all_ranks": 2.0 * m * k * n / sec / 1e12, "barrier_timeout": bad})
            del layers, y
        del weights, x
        torch.cuda.empty_cache()
    return out


def run_b200(args):
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        dist.init_process_group("nccl", timeout=__import__("datetime").timedelta(seconds=600))
    torch.cuda.set_device(local)

    from accelep_b200 import load
    from accelep_b200.llama import Llama

    lib = load()
    cfg = syn.SMOLLM2_135M
    planes, dense = syn.llama_int8(cfg, WEIGHT_SEED)
    model = Llama(cfg)
    model.load_int8(planes, dense)
    del planes, dense
    prompt_len = args.prompt_len or PROMPT
    new = args.new_tokens or NEW
    seqs = args.seqs
    if not 1 <= seqs <= SEQS:
        raise SystemExit(f"--seqs must be in 1..{SEQS}")
    prompts = [p[:prompt_len] for p in syn.prompts(cfg, SEQS, max(PROMPT, prompt_len), PROMPT_SEED)][:seqs]
    stream = torch.cuda.ExternalStream(model.stream())

    def step():
        return model.generate_batch(prompts, new)

    # C5 first, on a cool GPU, with its own clock record.
    c5_clocks = ClockSampler(local)
    c5_clocks.start()
    sharded_rows = c5_sharded(torch, dist, world, rank)
    c5_clk = c5_clocks.stop()

    for _ in range(max(3, args.warmup)):
        out = step()
    assert all(len(o) == new for o in out)

    def barrier():
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
            torch.cuda.synchronize()

    clocks = ClockSampler(local)
    barrier()
    clocks.start()
    launches0 = lib.accel_b200_launch_count()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        out = step()
    end.record(stream)
    end.synchronize()
    wall = time.perf_counter() - t0
    barrier()
    launches = lib.accel_b200_launch_count() - launches0
    clk = clocks.stop()
    dev_sec = start.elapsed_time(end) / 1000.0
    tensor = torch.tensor([dev_sec, wall], dtype=torch.float64, device="cuda")
    if world > 1:
        dist.all_reduce(tensor, op=dist.ReduceOp.MAX)
    dev_sec, wall = float(tensor[0]), float(tensor[1])
    tokens = seqs * new * world * args.steps
    value = tokens / dev_sec

    if rank == 0:
        peak, peak_kind = hbm_peak()
        step_line = step_roofline(torch, model, prompts, stream, dev_sec / args.steps, new, peak)
        achieved, sec, nbytes = attention_roofline(torch, stream)
        p_achieved, p_sec, p_bytes = products_roofline(torch, stream)
        gemv = gemv_roofline(torch)
        extras = None if args.no_extras or world > 1 else metric_set(torch, peak)
        cpu = None
        if world == 1 and not args.no_cpu_baseline:
            cpu = cpu_baseline_one_core()
        cfg_line = config(world, seqs)
        if prompt_len != PROMPT or new != NEW:
            cfg_line["workload"] = f"profiling variant: prompt {prompt_len}, {new} new ids (not the C4 bench number)"
        if seqs != SEQS:
            cfg_line["workload"] += (f" [{seqs} seqs per GPU: one rank's share of a fixed {SEQS}-sequence batch split "
                                     f"over {SEQS // seqs} GPUs, not the C4 bench number]")
        line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
                "warmup": max(3, args.warmup), "ms_per_step": 1000.0 * dev_sec / args.steps,
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8 weights, f32 compute",
                "data": "synthetic (seeded random-init weights and prompts)", "config": cfg_line,
                "e2e": {"value": tokens / wall, "unit": UNIT, "h2d_bytes_per_step": seqs * prompt_len * 4,
                        "d2h_bytes_per_step": seqs * new * 4},
                "gpu_launches": int(launches),
                "roofline": {"kernel": "Q8GemmTcKernel: the decode step's 121 int8 products (largest share of the "
                                       "step), graph-replayed, per-launch average", "bound": "hbm",
                             "achieved": p_achieved, "peak": peak, "peak_kind": peak_kind, "unit": "GB/s",
                             "frac": p_achieved / peak, "traffic": PRODUCT_TRAFFIC,
                             "bytes_per_launch": p_bytes, "us_per_launch": p_sec * 1e6},
                "roofline_attention": {"kernel": "decode_attention (fused Rope+AppendCache+attention, B=32, 1280 "
                                                 "context rows)", "bound": "hbm",
                                       "achieved": achieved, "peak": peak, "peak_kind": peak_kind, "unit": "GB/s",
                                       "frac": achieved / peak, "traffic": ATTENTION_TRAFFIC,
                                       "bytes_per_launch": nbytes, "us_per_launch": sec * 1e6},
                "dequant_gemv": {"config": "C5 sweep point M=1, K=N=16384: fp32 X, int8 W [K,N], per-column fp32 "
                                           "scales; accel_b200_matmul_q8 (GEMV path), graph-replayed, 2 weight "
                                           "copies rotated (512 MB > L2)",
                                 "us_per_launch": gemv["us"], "achieved": gemv["gbs"], "peak": peak,
                                 "peak_kind": peak_kind, "unit": "GB/s", "frac": gemv["gbs"] / peak,
                                 "bytes_per_launch": 16384 * 16384 + 4 * 16384 * 3, "traffic": GEMV_TRAFFIC},
                "c5_sharded": {"what": "int8 GEMM sweep points with W N-sharded over the ranks; one call = local "
                                       "product + assembly of Y on every rank (nccl: all_gather_into_tensor + "
                                       "transpose; fused: peer stores from the product epilogue + peer-memory "
                                       "barrier); max over ranks", "ranks": world, "points": sharded_rows,
                               "clocks": c5_clk},
                "step_roofline": step_line, "metric_set": extras, "cpu_baseline": cpu, "clocks": clk}
        print(json.dumps(line), flush=True)
    model.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extras", action="store_true", help="skip the C1/C2/C3/C5-grid metric set")
    # Shorter jobs for profiling runs only; a bench number uses the defaults.
    ap.add_argument("--prompt-len", type=int, default=0)
    ap.add_argument("--new-tokens", type=int, default=0)
    # Sequences per rank (32: the C4 bench). A smaller count measures one
    # rank's share of a fixed 32-sequence batch split over 32 / seqs GPUs.
    ap.add_argument("--seqs", type=int, default=SEQS)
    args = ap.parse_args()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_b200(args)


if __name__ == "__main__":
    main()
