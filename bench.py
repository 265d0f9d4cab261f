#!/usr/bin/env python
"""Benchmark: batch-1 Q8_0 greedy decode of a Llama-3-8B-shaped model.

The workload is BASELINE.json's headline metric, "Q8 decode tok/s (8B shape,
bs1)": dim 4096, 32 layers, 32 heads / 8 KV heads, hidden 14336, vocab
128256, Q8_0 weights (group 32, the reference's only block size), random
N(0, 0.02) from a fixed seed, a 4096-token key/value context (synthetic
values) and one decode step per "step": embed -> 32 layers -> RMSNorm ->
classifier -> argmax, replayed as one CUDA graph.

value:  whole-job decode tokens/s with everything resident in HBM, timed on
        the device with CUDA events over K steps (max over ranks).
e2e:    the same through the public C ABI (rk_model_step): each step copies
        its token from pinned host memory and reads the logits back.
roofline: the Q8_0 matvec kernels inside the step, each launch timed with
        CUDA events: algorithmic bytes (weights + scales) / time, against the
        measured HBM copy bandwidth.
cpu_baseline: the CPU oracle (a C restatement of the reference's Go CPU
        path) on a bounded sample of the same step, on this host's cores.

--impl reference runs only that CPU implementation (no GPU).
With --gpus N (under torchrun) the default --mode rows shards every layer's
weight rows over the N GPUs (whole kv heads per GPU) and reassembles each
product's output inside the kernels (tagged words stored over NVLink; NCCL
all-gathers where that is not possible): one sequence decoded by all N GPUs
(strong scaling; value = its tokens/s). --mode replicas runs N independent
copies instead (weak scaling); --mode pipeline splits the layers into N
stages (rk_plan_stages) that pass the activation on (roofline not measured).

Other measurements (one JSON line each, not the headline):
  --kernel matvec        one decode matvec of --shape (L2 flushed)
  --kernel matvec_many   one batched Q8_0 product of --shape with --prefill vectors
  --kernel tensor        rakkan_tensor_v1 matmul / matmul_t, config 2's sweep
  --kernel prefill       ForwardMany over --prefill tokens of --model (config 3's 512-token prefill)
  --kernel decode_batch  one decode step of --batch sequences with --ctx-token caches (config 4's batch 32)
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "rakkan-mesh_b200"))
sys.path.insert(0, os.path.join(ROOT, "oracle"))

METRIC = "Q8 decode tok/s (8B shape, bs1)"
SEED = 20261201
CTX = 4096


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=50)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", default="ours", choices=["ours", "reference"])
    p.add_argument("--model", default="llama3-8b")
    p.add_argument("--dtype", default="q8_0")
    p.add_argument("--ctx", type=int, default=CTX)
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-workloads", action="store_true",
                   help="skip the other configurations' workloads (measured after the headline at N=1)")
    p.add_argument("--mode", default="rows", choices=["rows", "replicas", "pipeline"],
                   help="N>1: shard every layer's rows over the N GPUs (NCCL all-gather; one sequence), "
                        "or run N independent replicas")
    p.add_argument("--layers", type=int, default=0,
                   help="profiling aid: build the model with this many layers instead of the config's")
    p.add_argument("--tensor-shape", default=None,
                   help="--kernel tensor: one MxKxN shape instead of config 2's sweep")
    p.add_argument("--tensor-dtype", default="both", choices=["both", "i8", "f32"])
    p.add_argument("--tensor-op", default="both", choices=["both", "matmul", "matmul_t"])
    p.add_argument("--batch", type=int, default=32, help="--kernel decode_batch: sequences decoded together")
    p.add_argument("--kernel", default=None, choices=["matvec", "matvec_many", "tensor", "prefill", "decode_batch"],
                   help="time one kernel alone instead of the decode step, or a prefill (profiling aids)")
    p.add_argument("--prefill", type=int, default=512, help="--kernel prefill: prompt tokens")
    p.add_argument("--shape", default="28672x4096", help="rows x cols for --kernel matvec")
    p.add_argument("--prologue", default="fused", choices=["fused", "given"],
                   help="--kernel matvec: quantize the input inside the kernel (as the decode step does) "
                        "or read a quantized copy")
    return p.parse_args()


def run_kernel(args):
    """One matvec of --shape in --dtype (q8_0, q4_0, f32, bf16), L2 flushed
    before each launch."""
    import rkcuda as rk
    rows, cols = map(int, args.shape.split("x"))
    fmt = {"q8_0": rk.FMT_Q8_0, "q4_0": rk.FMT_Q4_0, "f32": rk.FMT_F32, "bf16": rk.FMT_BF16}[args.dtype]
    dev = rk.Device(int(os.environ.get("LOCAL_RANK", "0")))
    m = rk.Matrix.generate(dev, rows, cols, fmt, SEED, 1, 0.02)
    quantized = fmt in (rk.FMT_Q8_0, rk.FMT_Q4_0)
    fused = args.prologue == "fused" and quantized
    m.bench(max(1, args.warmup), flush=True, fused=fused)
    ms = m.bench(args.steps, flush=True, fused=fused)
    n = rows * cols
    nbytes = {rk.FMT_Q8_0: n + n // 32 * 4, rk.FMT_Q4_0: n // 2 + n // 32 * 4, rk.FMT_F32: 4 * n,
              rk.FMT_BF16: 2 * n}[fmt]
    peak, kind = measured_peak()
    kname = f"k_matvec_q<{args.dtype}>" if quantized else f"k_matvec_f<{args.dtype}>"
    print(json.dumps({"kernel": kname, "shape": args.shape, "prologue": args.prologue if quantized else "none",
                      "ms": ms,
                      "achieved_gbs": nbytes / (ms * 1e-3) / 1e9, "peak_gbs": peak, "peak_source": kind,
                      "frac": nbytes / (ms * 1e-3) / 1e9 / peak}), flush=True)
    m.free()
    dev.close()


def run_decode_batch(args):
    """Config 4's batch-32 decode: --batch sequences, each with a --ctx-token
    cache (seeded values, as the headline's), one decode step of all of them
    per call through the public stage API (activations in from host memory
    and back, timed on the host). The stage's layers only: no embedding
    lookup or classifier."""
    import numpy as np
    import rkcuda as rk
    import synth
    dev = rk.Device(int(os.environ.get("LOCAL_RANK", "0")))
    n = args.batch
    c = synth.config(args.model, args.dtype, seq_len=args.ctx + 64)
    dm = synth.DeviceModel(dev, c, SEED, ctx=args.ctx + 64, nseq=n)
    dm.stage.fill_cache(args.ctx, SEED)
    xs = np.random.default_rng(SEED).standard_normal((n, c.dim)).astype(np.float32)
    pos = [args.ctx] * n
    for _ in range(max(3, args.warmup)):
        dm.stage.forward_batch(xs, pos)
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        dm.stage.forward_batch(xs, pos)
        times.append(time.perf_counter() - t0)
    ms = 1000.0 * statistics.median(times)
    print(json.dumps({"kernel": "decode_batch", "model": args.model, "dtype": args.dtype, "batch": n,
                      "context": args.ctx, "ms_per_step": ms, "tok_s": n * 1000.0 / ms, "steps": args.steps,
                      "scope": "the stage's layers (no embedding or classifier), host buffers in and out"}),
          flush=True)
    dm.free()
    dev.close()


def run_kernel_many(args):
    """One batched Q8_0 (or, with --dtype q4_0, Q4_0) product of --shape
    with --prefill input vectors (at most 64, a ForwardMany submission), L2
    flushed before each launch. The weights are read once per launch; every
    (row, vector, block) costs the epilogue four f32 operations."""
    import rkcuda as rk
    rows, cols = map(int, args.shape.split("x"))
    n = args.prefill
    q4 = args.dtype == "q4_0"
    dev = rk.Device(int(os.environ.get("LOCAL_RANK", "0")))
    m = rk.Matrix.generate(dev, rows, cols, rk.FMT_Q4_0 if q4 else rk.FMT_Q8_0, SEED, 1, 0.02)
    m.bench_many(n, max(1, args.warmup))
    ms = m.bench_many(n, args.steps)
    nbytes = rows * cols // (2 if q4 else 1) + rows * cols // 32 * 4
    peak, kind = measured_peak()
    print(json.dumps({"kernel": "k_mv_many", "fmt": "q4_0" if q4 else "q8_0", "shape": args.shape, "vectors": n,
                      "ms": ms,
                      "achieved_gbs": nbytes / (ms * 1e-3) / 1e9, "peak_gbs": peak, "peak_source": kind,
                      "frac": nbytes / (ms * 1e-3) / 1e9 / peak,
                      "int8_tops": 2.0 * rows * cols * n / (ms * 1e-3) / 1e12,
                      "epilogue_gflops": 4.0 * rows * (cols // 32) * n / (ms * 1e-3) / 1e9}), flush=True)
    m.free()
    dev.close()


def run_tensor(args):
    """rakkan_tensor_v1 matmul_t of config 2 (M in {1, 16, 128, 512}, N = K =
    4096), int8 and f32, device-resident inputs, L2 flushed before each."""
    import rkcuda as rk
    dev = rk.Device(int(os.environ.get("LOCAL_RANK", "0")))
    peaks = {}
    try:
        peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
    except (OSError, ValueError):
        pass
    shapes = [(m, 4096, 4096) for m in (1, 16, 128, 512)]
    if args.tensor_shape:
        shapes = [tuple(int(v) for v in args.tensor_shape.split("x"))]
    for dtype, name in ((rk.TENSOR_I8, "i8"), (rk.TENSOR_F32, "f32")):
        if args.tensor_dtype not in ("both", name):
            continue
        for transposed in (True, False):
            if args.tensor_op not in ("both", "matmul_t" if transposed else "matmul"):
                continue
            for m, k, n in shapes:
                rk.bench_tensor(dev, dtype, transposed, m, k, n, max(1, args.warmup))
                ms = rk.bench_tensor(dev, dtype, transposed, m, k, n, args.steps)
                es = 1 if dtype == rk.TENSOR_I8 else 4
                nbytes = es * (m * k + k * n) + 4 * m * n
                print(json.dumps({"kernel": f"tensor_{name}", "op": "matmul_t" if transposed else "matmul",
                                  "m": m, "k": k, "n": n, "ms": ms, "tops": 2 * m * n * k / (ms * 1e-3) / 1e12,
                                  "gbs": nbytes / (ms * 1e-3) / 1e9, "hbm_peak_gbs": peaks.get("hbm_gbs")}),
                      flush=True)
    dev.close()


def run_prefill(args):
    """Stage.ForwardMany over a seeded prompt of --prefill activations from
    position 0, through the public stage API (activations in from host
    memory and back), timed on the host around the synchronous call. An
    all-Q8_0 stage runs each projection once per 64 tokens on the tensor
    cores; the attention goes token by token."""
    import numpy as np
    import rkcuda as rk
    import synth
    dev = rk.Device(int(os.environ.get("LOCAL_RANK", "0")))
    n = args.prefill
    c = synth.config(args.model, args.dtype, seq_len=n + 64)
    dm = synth.DeviceModel(dev, c, SEED, ctx=n + 64)
    xs = np.random.default_rng(SEED).standard_normal((n, c.dim)).astype(np.float32)
    for _ in range(max(1, args.warmup)):
        dm.stage.forward(xs, 0)
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        dm.stage.forward(xs, 0)
        times.append(time.perf_counter() - t0)
    ms = 1000.0 * statistics.median(times)
    print(json.dumps({"kernel": "prefill", "model": args.model, "dtype": args.dtype, "tokens": n,
                      "batched": dm.stage.batched(), "ms": ms, "tok_s": n * 1000.0 / ms,
                      "steps": args.steps}), flush=True)
    dm.free()
    dev.close()


def secondary_workloads(dev):
    """The other configurations' workloads, measured through the public API
    after the headline (one GPU, synthetic seeded weights and inputs, each
    timed after a warm-up): config 1's 8-token prompt + 128 greedy tokens;
    config 2's tensor matmul_t sweep (device time, L2 flushed); config 3's
    512-token prefill + 256 greedy tokens; config 4's Q4_0 batch-1 decode at
    a 4096-token context (graph replays, device time) and batch-32 decode in
    Q8_0 and Q4_0 (one step of 32 sequences per call, host time); config
    5's 2048-token prefill + 512 greedy tokens. Generation goes through
    rk_model_generate (the prompt in ForwardMany submissions of 64 tokens,
    then one step graph per token, each token read back); prefill figures
    are its time for the prompt and one token. A workload that fails
    reports its error instead of a number."""
    import numpy as np
    import rkcuda as rk
    import synth
    out = {}

    def timed(fn, reps=1):
        fn()  # warm-up
        t0 = time.perf_counter()
        for _ in range(reps):
            fn()
        return (time.perf_counter() - t0) * 1000.0 / reps

    def generation(key, name, dtype, n_prompt, n_new):
        c = synth.config(name, dtype, seq_len=n_prompt + n_new + 8)
        dm = synth.DeviceModel(dev, c, SEED, ctx=n_prompt + n_new + 8)
        try:
            p = np.random.default_rng(SEED).integers(0, c.vocab, n_prompt).astype(np.int32)
            pre = timed(lambda: dm.model.generate(p, 1))
            total = timed(lambda: dm.model.generate(p, n_new))
            out[key] = {"prompt": n_prompt, "new_tokens": n_new, "batched_prompt": dm.stage.batched(),
                        "total_ms": total, "prefill_ms": pre, "prefill_tok_s": n_prompt * 1000.0 / pre,
                        "decode_tok_s": (n_new - 1) * 1000.0 / max(total - pre, 1e-9),
                        "workload_tok_s": (n_prompt + n_new) * 1000.0 / total}
        finally:
            dm.free()

    def decode_bs1(key, name, dtype, ctx=4096, iters=20):
        c = synth.config(name, dtype, seq_len=ctx + 64)
        dm = synth.DeviceModel(dev, c, SEED, ctx=ctx + 64)
        try:
            dm.stage.fill_cache(ctx, SEED)
            dm.model.bench(ctx, 3)
            ms = dm.model.bench(ctx, iters)
            out[key] = {"context": ctx, "ms_per_step": ms, "tok_s": 1000.0 / ms, "timing": "device, graph replays"}
        finally:
            dm.free()

    def decode_batch(key, name, dtype, n=32, ctx=4096, steps=5):
        c = synth.config(name, dtype, seq_len=ctx + 64)
        dm = synth.DeviceModel(dev, c, SEED, ctx=ctx + 64, nseq=n)
        try:
            dm.stage.fill_cache(ctx, SEED)
            xs = np.random.default_rng(SEED).standard_normal((n, c.dim)).astype(np.float32)
            ms = timed(lambda: dm.stage.forward_batch(xs, [ctx] * n), steps)
            out[key] = {"batch": n, "context": ctx, "ms_per_step": ms, "tok_s": n * 1000.0 / ms,
                        "scope": "the stage's layers, host buffers in and out"}
        finally:
            dm.free()

    def tensor_sweep(key):
        rows = []
        for dtype, name in ((rk.TENSOR_I8, "i8"), (rk.TENSOR_F32, "f32")):
            for m in (1, 16, 128, 512):
                rk.bench_tensor(dev, dtype, True, m, 4096, 4096, 2)
                ms = rk.bench_tensor(dev, dtype, True, m, 4096, 4096, 10)
                rows.append({"dtype": name, "op": "matmul_t", "m": m, "n": 4096, "k": 4096, "ms": ms,
                             "tops": 2 * m * 4096 * 4096 / (ms * 1e-3) / 1e12})
        out[key] = rows

    jobs = [
        ("config1_stories15m_q8_0", lambda k: generation(k, "stories15M", "q8_0", 8, 128)),
        ("config2_tensor_matmul_t", tensor_sweep),
        ("config3_qwen2.5-0.5b_q8_0", lambda k: generation(k, "qwen2.5-0.5b", "q8_0", 512, 256)),
        ("config4_llama3-8b_q4_0_bs1", lambda k: decode_bs1(k, "llama3-8b", "q4_0")),
        ("config4_llama3-8b_q8_0_bs32", lambda k: decode_batch(k, "llama3-8b", "q8_0")),
        ("config4_llama3-8b_q4_0_bs32", lambda k: decode_batch(k, "llama3-8b", "q4_0")),
        ("config5_qwen3-32b_q8_0", lambda k: generation(k, "qwen3-32b", "q8_0", 2048, 512)),
    ]
    for key, job in jobs:
        try:
            job(key)
        except Exception as e:  # noqa: BLE001 (reported, not fatal to the headline)
            out[key] = {"error": f"{type(e).__name__}: {e}"}
    return out


def workload(args):
    return {"workload": f"{args.model}-shaped {args.dtype} greedy decode, batch 1, {args.ctx}-token KV context",
            "shape": "dim 4096, 32 layers, 32/8 heads, hidden 14336, vocab 128256" if args.model == "llama3-8b"
            else args.model,
            "weights": "random N(0,0.02), seeded, quantized by the reference's quantize8 (group 32)",
            "batch": 1, "context": args.ctx,
            "l2": "inputs larger than L2 (8.4 GB of weights + 1.07 GB of KV cache read per step)",
            **({"layers": f"{args.layers} (profiling run, not the headline)"} if args.layers > 0 else {})}


class Clocks:
    """nvidia-smi samples during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        self.p = None

    def __enter__(self):
        try:
            self.p = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}",
                                       "--format=csv,noheader,nounits", "-lms", "200"], stdout=self.f,
                                      stderr=subprocess.DEVNULL)
        except OSError:
            self.p = None
        time.sleep(0.3)
        return self

    def __exit__(self, *a):
        if self.p:
            self.p.terminate()
            self.p.wait()

    def summary(self):
        self.f.seek(0)
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.f:
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = max(mx, float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        os.unlink(self.f.name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx or None,
                "reasons": sorted(reasons), "samples": len(sm)}


def measured_peak():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, "fallback"


def traffic_ratio(chained=False):
    """DRAM bytes per algorithmic byte of a Q8_0 matvec launch, from the
    committed ncu summary (one launch of the 28672x4096 W1/W3 shape, or of
    one layer's chain when the step runs chains)."""
    name = "matvec_chain_q8_llama3-8b_layer.txt" if chained else "matvec_q8_28672x4096.txt"
    path = os.path.join(ROOT, "profiles", name)
    try:
        for line in open(path):
            if line.startswith("dram_bytes_per_algorithmic_byte:"):
                return float(line.split(":")[1])
    except (OSError, ValueError):
        pass
    return None


def cpu_sample(args, steps=1, sample_layers=2, threads=None):
    """Times the CPU oracle on a bounded sample of one decode step: the
    forward through `sample_layers` of the 32 layers at position ctx (over a
    synthetic ctx-token cache), plus the classifier; returns the extrapolated
    whole-step rate and the description."""
    import rk_oracle as ro
    import synth
    threads = threads or ro.THREADS
    full = synth.config(args.model, args.dtype)
    c = synth.config(args.model, args.dtype, layers=sample_layers, seq_len=args.ctx + 1)
    om = ro.OracleModel(c, SEED, ctx=args.ctx + 1, threads=threads)
    try:
        om.fill_cache(args.ctx, SEED)
        x = om.embed_token(1)
        t_layers, t_head = [], []
        for _ in range(max(1, steps)):
            t0 = time.perf_counter()
            y = om.forward(x, args.ctx)
            t1 = time.perf_counter()
            om.logits(y)
            t2 = time.perf_counter()
            t_layers.append(t1 - t0)
            t_head.append(t2 - t1)
        per_token = statistics.median(t_layers) * full.layers / sample_layers + statistics.median(t_head)
    finally:
        om.free()
    sample = (f"{sample_layers} of {full.layers} layers at position {args.ctx} plus the classifier, scaled to "
              f"the whole step; {max(1, steps)} step(s), median")
    return 1.0 / per_token, threads, sample


def run_reference(args, rank):
    """The reference arm: the CPU implementation of the path (the oracle, a C
    restatement of the reference's Go CPU path; the Go toolchain is absent
    on this box) on the same workload as the CUDA arm: the whole model
    (every layer and the classifier) at position ctx over a ctx-token cache,
    W untimed warm-up steps, then exactly K timed steps, each one whole
    decode step (forward, logits, argmax), on all the host threads it can
    use. Under torchrun only rank 0 runs it."""
    if rank != 0:
        return
    import rk_oracle as ro
    import synth
    c = synth.config(args.model, args.dtype, seq_len=args.ctx + 1)
    om = ro.OracleModel(c, SEED, ctx=args.ctx + 1)
    try:
        om.fill_cache(args.ctx, SEED)
        for _ in range(args.warmup):
            om.step(1, args.ctx)
        t0 = time.perf_counter()
        for _ in range(args.steps):
            om.step(1, args.ctx)
        ms = (time.perf_counter() - t0) * 1000.0 / max(1, args.steps)
    finally:
        om.free()
    value = 1000.0 / ms
    sample = (f"the whole decode step ({c.layers} layers at position {args.ctx}, classifier, argmax), "
              f"{args.steps} timed steps after {args.warmup} warm-ups")
    line = {"metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "int8xint8->int32, f32 combine", "data": "synthetic",
            "impl": "reference", "config": workload(args),
            "cpu_baseline": {"value": value, "unit": "tok/s", "cores": ro.THREADS, "kind": "port",
                             "sample": sample},
            "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def main():
    args = parse()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        return run_reference(args, rank)
    if args.kernel == "tensor":
        return run_tensor(args)
    if args.kernel == "prefill":
        return run_prefill(args)
    if args.kernel == "matvec_many":
        return run_kernel_many(args)
    if args.kernel == "decode_batch":
        return run_decode_batch(args)
    if args.kernel:
        return run_kernel(args)

    import torch
    dist = None
    if world > 1:
        # The ranks' collectives here are two small all-gathers per token
        # (the rest travel as NVLink stores inside the kernels); NCCL's
        # NVLink SHARP path would add multicast buffer registration for
        # nothing, so it stays off unless the caller sets it.
        os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=__import__("datetime").timedelta(seconds=600))
    import rkcuda as rk
    if world > 1 and args.mode == "pipeline":
        return run_pipeline(args, world, rank, local, dist, torch)
    import synth

    dev = rk.Device(local)
    over = {"layers": args.layers} if args.layers > 0 else {}
    c = synth.config(args.model, args.dtype, seq_len=args.ctx + 64, **over)
    sharded = world > 1 and args.mode == "rows"
    group = None
    if sharded:
        # Row shards of every layer over the N GPUs; the group id travels
        # over the torch process group.
        gid = [rk.group_id() if rank == 0 else None]
        dist.broadcast_object_list(gid, src=0)
        group = rk.Group(dev, world, rank, gid[0])
    dm = synth.DeviceModel(dev, c, SEED, ctx=args.ctx + 64, group=group)
    dm.stage.fill_cache(args.ctx, SEED)
    pos, tok = args.ctx, 1

    def barrier():
        if dist:
            dist.barrier()
        torch.cuda.synchronize(local)

    def max_over_ranks(v):
        if not dist:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=f"cuda:{local}")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # Warm-up, then K device-timed steps (graph replays at position ctx).
    # Starting the clock sampler takes a while and not the same on every
    # rank, so inside its context one more untimed replay (whose gathers
    # align the ranks) and a barrier come directly before the timed ones.
    dm.model.bench(pos, max(3, args.warmup))
    barrier()
    with Clocks(local) as clk:
        barrier()
        dm.model.bench(pos, 1)
        barrier()
        ms = dm.model.bench(pos, args.steps)
        barrier()
    clocks = clk.summary()
    ms = max_over_ranks(ms)

    # End to end through the public API: token in from pinned host memory,
    # logits and the next token back, every step.
    for _ in range(max(3, args.warmup)):
        dm.model.step(tok, pos)
    barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        dm.model.step(tok, pos)
    barrier()
    e2e_ms = max_over_ranks((time.perf_counter() - t0) * 1000.0 / args.steps)

    # Roofline of the dominant kernel: every Q8_0 matvec launch of a step
    # timed with CUDA events on its stream.
    prof = dm.model.profile(pos, 3)
    achieved = prof.matvec_bytes / (prof.matvec_ms * 1e-3) / 1e9
    peak, peak_kind = measured_peak()
    launches = dm.model.kernel_count()

    baseline = None
    # Rank 0 at N=1 only: a sharded peer would wait on its gathers meanwhile.
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        v, cores, sample = cpu_sample(args)
        baseline = {"value": v, "unit": "tok/s", "cores": cores, "kind": "port", "sample": sample}

    # DRAM bytes of the average matvec launch of a step: the captured
    # launch's traffic per algorithmic byte times the step's average
    # algorithmic bytes per launch (traffic scales with the rows read).
    ratio = traffic_ratio(dm.stage.chained())
    traffic = ratio * prof.matvec_bytes / prof.matvec_launches if ratio and prof.matvec_launches else None
    # Sequences decoded at once: one sharded over all GPUs, or one per replica.
    seqs = 1 if sharded else world
    parity = None
    if world > 1:
        barrier()
        _, lg = dm.model.step(tok, pos)
        parity = parity_vs_1gpu(args, dev, c, lg, rank, local, dist, torch)
    if rank == 0:
        cfg = workload(args)
        par = {"mode": f"rows{world}" if sharded else (f"replicas{world}" if world > 1 else "none")}
        if sharded:
            par["gathers"] = "fused (tagged words stored over NVLink)" if dm.stage.fused_gathers() else "NCCL all-gather"
        line = {
            "metric": METRIC, "value": seqs * 1000.0 / ms, "unit": "tok/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "strong" if sharded else "weak",
            "vs_baseline": None, "dtype": "int8xint8->int32, f32 combine", "data": "synthetic",
            "config": cfg,
            "e2e": {"value": seqs * 1000.0 / e2e_ms, "unit": "tok/s", "h2d_bytes_per_step": 8,
                    "d2h_bytes_per_step": 4 * c.vocab + 4},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "peak_source": peak_kind,
                         "traffic": traffic,
                         "kernel": "k_matvec_chain<Q8_0>" if dm.stage.chained() else "k_matvec_q<Q8_0>",
                         "bytes_per_step": prof.matvec_bytes, "matvec_ms_per_step": prof.matvec_ms,
                         "matvec_launches_per_step": prof.matvec_launches,
                         "eager_step_ms": prof.step_ms},
            # Where a step's time goes, from the eagerly launched steps of
            # the roofline pass (each launch timed with CUDA events): the
            # products (with their gathers when sharded) and the rest
            # (attention, glue, the gaps between launches); graph_step is
            # the timed graph replay's time.
            "breakdown_ms": {"graph_step": ms, "eager_step": prof.step_ms, "products": prof.matvec_ms,
                             "attention_and_rest": prof.step_ms - prof.matvec_ms,
                             "product_launches": prof.matvec_launches, "launches": prof.launches},
            "cpu_baseline": baseline,
            "gpu_launches": launches * args.steps,
            "clocks": clocks,
            "parallel": par,
        }
        if parity is not None:
            line["parity_vs_1gpu"] = parity
        if world == 1 and args.layers == 0 and not args.no_workloads:
            # The other configurations, once the headline model is freed.
            dm.free()
            dm = None
            line["workloads"] = secondary_workloads(dev)
        print(json.dumps(line), flush=True)
    if dm is not None:
        dm.free()
    if group:
        barrier()
        group.free()
    dev.close()
    if dist:
        dist.destroy_process_group()
    if parity is False:
        sys.exit(3)


def parity_vs_1gpu(args, dev, c, logits, rank, local, dist, torch):
    """After the timed region: the logits of one step at the bench position
    on every rank (None on a rank that has none) against the same step of an
    unsharded model built on rank 0's GPU (the one-GPU model is the one the
    parity tests check against the oracle). Every rank returns the verdict:
    True if all ranks' logits equal it bit for bit."""
    import numpy as np
    import synth
    got = [None] * dist.get_world_size()
    dist.all_gather_object(got, None if logits is None else np.asarray(logits, np.float32))
    ok = [True]
    if rank == 0:
        ref = synth.DeviceModel(dev, c, SEED, ctx=args.ctx + 64)
        try:
            ref.stage.fill_cache(args.ctx, SEED)
            _, want = ref.model.step(1, args.ctx)
        finally:
            ref.free()
        want = np.asarray(want, np.float32).view(np.uint32)
        have = [g for g in got if g is not None]
        ok[0] = bool(have) and all(np.array_equal(g.view(np.uint32), want) for g in have)
        if not ok[0]:
            print(json.dumps({"parity_vs_1gpu": False,
                              "ranks_differing": [i for i, g in enumerate(got) if g is not None
                                                  and not np.array_equal(g.view(np.uint32), want)]}),
                  file=sys.stderr, flush=True)
    dist.broadcast_object_list(ok, src=0)
    return bool(ok[0])


def run_pipeline(args, world, rank, local, dist, torch):
    """--mode pipeline: the layers split over the N GPUs by rk_plan_stages
    (planStages with equal speeds), the activation passed rank to rank;
    one sequence, so the stages run one after another (config 5's layer
    pipeline; no batch-1 speed-up is expected, as in the reference)."""
    import numpy as np
    import rkcuda as rk
    import synth
    dev = rk.Device(local)
    over = {"layers": args.layers} if args.layers > 0 else {}
    c = synth.config(args.model, args.dtype, seq_len=args.ctx + 64, **over)
    gid = [rk.group_id() if rank == 0 else None]
    dist.broadcast_object_list(gid, src=0)
    group = rk.Group(dev, world, rank, gid[0])
    per = sum(synth.matrix_bytes(synth.mat_fmt(c, k), int(np.prod(synth.mat_shape(c, k)))) for k in synth.MATS)
    spans = rk.plan_stages([per] * c.layers, [per] * c.layers, [1.0] * world, [per * c.layers] * world, world)
    node, first, end = spans[rank]
    pr = synth.PipelineRank(dev, c, SEED, group, first, end, ctx=args.ctx + 64)
    pr.stage.fill_cache(args.ctx, SEED, first_layer=first)
    pos, tok = args.ctx, 1

    def barrier():
        dist.barrier()
        torch.cuda.synchronize(local)

    def max_over_ranks(v):
        t = torch.tensor([v], dtype=torch.float64, device=f"cuda:{local}")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    pr.pipeline.bench(pos, max(3, args.warmup))
    barrier()
    with Clocks(local) as clk:
        barrier()
        pr.pipeline.bench(pos, 1)
        barrier()
        ms = pr.pipeline.bench(pos, args.steps)
        barrier()
    clocks = clk.summary()
    ms = max_over_ranks(ms)
    for _ in range(max(3, args.warmup)):
        pr.pipeline.step(tok, pos)
    barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        pr.pipeline.step(tok, pos)
    barrier()
    e2e_ms = max_over_ranks((time.perf_counter() - t0) * 1000.0 / args.steps)
    _, lg = pr.pipeline.step(tok, pos)
    parity = parity_vs_1gpu(args, dev, c, lg, rank, local, dist, torch)
    if rank == 0:
        cfg = workload(args)
        par = {"mode": f"pipeline{world}", "stages": [[a, b] for _, a, b in spans]}
        line = {
            "metric": METRIC, "value": 1000.0 / ms, "unit": "tok/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "int8xint8->int32, f32 combine", "data": "synthetic", "config": cfg,
            "e2e": {"value": 1000.0 / e2e_ms, "unit": "tok/s", "h2d_bytes_per_step": 8, "d2h_bytes_per_step": 4},
            "roofline": None, "cpu_baseline": None, "clocks": clocks, "parallel": par,
            "parity_vs_1gpu": parity,
        }
        print(json.dumps(line), flush=True)
    pr.free()
    barrier()
    group.free()
    dev.close()
    dist.destroy_process_group()
    if not parity:
        sys.exit(3)


if __name__ == "__main__":
    main()
