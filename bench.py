"""Benchmark: ModernBERT-base tokens/s on B200 through liblaya_cuda.

Workload: ModernBERT-base shape (22 layers, hidden
768, 12 heads, GeGLU 1152, window 128, RoPE 160000/10000), random-init fp16
weights N(0, 0.02), LayerNorm weights 1, prompts with lengths uniform in
[32, 512] (seeded), token ids uniform in [5, 50368) with CLS/SEP, an 8-way CLS
classifier + softmax. One step = one forward of the batch (ids -> class
probabilities) through the fused varlen encoder (lc_encoder_forward).

Multi-GPU (torchrun, N ranks): ONE global batch of 256·N prompts is drawn and
sharded over the ranks by longest-processing-time on each prompt's FLOPs
(laya_js_b200.dp.lpt_shards); every rank holds a full weight replica and runs
its shard. In the end-to-end leg each step's probabilities are gathered to
rank 0 on the host (a gloo group, 32 bytes per prompt). NCCL carries only the
start/stop barriers and the max-over-ranks time: no collective on the data
path. Inputs and all inputs of a step exceed L2 (activations ~0.5 GB).

Keys beyond the driver's contract (extras run on rank 0 of a 1-GPU run):
  e2e        the same metric through lc_encoder_forward_host (host ids in,
             host probabilities out, copies and the host gather inside the
             timed region);
  shards     tokens per rank and the cost imbalance of the LPT split;
  roofline   the tcgen05 GEMMs (dominant kernel class) vs the measured
             sustained bf16 tensor peak, with their DRAM traffic per launch;
  cpu_baseline  the C++ oracle (f32 storage, f64 accumulation) timed on one
             thread and on all host threads over a fixed sample of the batch;
  quantized  configs[3]: 4-bit and 8-bit affine g64 weights (batch 512,
             lengths U[64, 1024]) tokens/s, plus the configs[0]-shape graph
             latency with those weights (fused-dequant GEMMs);
  large_bf16 configs[4]: ModernBERT-large / mmBERT shape in bf16 on a fixed
             subset (the first 1024) of the 65,536-prompt length draw;
  contract   ModernBert.encode through Backend<T> ops (what laya's
             load()/predict() run), host buffers in and out: configs[0] p50
             and a padded configs[2] batch;
  p50_latency_ms / p50_latency_graph_ms  configs[0] (batch 1, seq 128,
             3-way head) end to end, eager and as a captured CUDA graph;
  predict    the DecisionModel forward (predict()'s model call) on one
             128-token prompt: p50 eager and through Backend.compile;
  microbench configs[1]: the row and elementwise contract ops over [M, N]
             (f16 / f32), GB/s against the measured copy bandwidth.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

BATCH, LO, HI, CLASSES = 256, 32, 512, 8
WORKLOAD = "configs[2]: ModernBERT-base fp16, 256 prompts per GPU (one global batch of 256·N, LPT-sharded), L~U[32,512], 8-way CLS head + softmax"
METRIC = "modernbert_base_fp16_tokens_per_s"
# DRAM bytes per GEMM launch of this workload (average over the four
# projections), scaled from the small-case capture in profiles/gemm_traffic_bench.md
GEMM_TRAFFIC_BYTES = 306.6e6


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", default="ours", choices=["ours", "reference"])
    p.add_argument("--no-extras", action="store_true", help="skip the extra legs (latency, quantized, large, contract, CPU)")
    return p.parse_args()


def config_of(world: int, tokens_per_gpu: int, tokens_total: int) -> dict:
    """The workload description both arms report (the reference arm times a
    stated fixed sample of it per step, see its cpu_baseline.sample)."""
    return {"workload": WORKLOAD, "global_batch": BATCH * world, "seq_len": f"U[{LO},{HI}]", "tokens_per_gpu_step": tokens_per_gpu,
            "tokens_per_step": tokens_total, "parallelism": f"dp{world}", "l2": "inputs larger than L2 (activations ~0.5 GB per step)"}


def linear_flops_per_token(cfg: dict) -> float:
    H, I, n = cfg["hidden_size"], cfg["intermediate_size"], cfg["num_hidden_layers"]
    return 2.0 * (H * 3 * H + H * H + H * 2 * I + I * H) * n


def attention_flops(cfg: dict, lens) -> float:
    """QKᵀ and P·V FLOPs of one forward over prompts of the given lengths:
    4·H per visible (query, key) pair; global layers (every third, from the
    first) see the whole prompt, sliding layers the keys within window/2."""
    H, n = cfg["hidden_size"], cfg["num_hidden_layers"]
    half = cfg.get("local_attention", 128) // 2
    n_global = (n + 2) // 3
    total = 0.0
    for L in np.asarray(lens, np.int64):
        i = np.arange(L)
        pairs_local = float((np.minimum(i + half, L - 1) - np.maximum(i - half, 0) + 1).sum())
        total += n_global * float(L) * float(L) + (n - n_global) * pairs_local
    return 4.0 * H * total


PEAK_SRC = {"measured": ("measured sustained bf16 (MEASURED_PEAKS.json)", "measured copy bandwidth (MEASURED_PEAKS.json)"),
            "fallback": ("fallback: the pool's earlier sustained bf16 measurement (MEASURED_PEAKS.json absent or incomplete)",
                         "fallback: the pool's earlier copy-bandwidth measurement (MEASURED_PEAKS.json absent or incomplete)")}


def measured_peaks() -> dict:
    """Roofline denominators: MEASURED_PEAKS.json (written per pod: sustained
    bf16 GEMM TFLOP/s, copy GB/s), else the pool's earlier measurement
    (1.4 PFLOP/s sustained, 6.65 TB/s), labelled "fallback"."""
    f = ROOT / "MEASURED_PEAKS.json"
    d = json.loads(f.read_text()) if f.exists() else {}
    if "bf16_tflops_sustained" in d and "hbm_gbs" in d:
        return {"bf16": float(d["bf16_tflops_sustained"]), "hbm": float(d["hbm_gbs"]), "src": "measured"}
    return {"bf16": 1400.0, "hbm": 6650.0, "src": "fallback"}


def shard(lens: np.ndarray, ids: np.ndarray, cu: np.ndarray, rank: int, world: int):
    """This rank's prompts of the global batch (LPT on prompt FLOPs), re-packed."""
    from laya_js_b200.dp import lpt_shards, prompt_cost
    shards = lpt_shards([prompt_cost(int(L)) for L in lens], world)
    mine = np.asarray(shards[rank], np.int64)
    parts = [ids[cu[i]:cu[i + 1]] for i in mine]
    my_ids = np.concatenate(parts).astype(np.int32)
    my_cu = np.concatenate([[0], np.cumsum([len(p) for p in parts])]).astype(np.int32)
    costs = [sum(prompt_cost(int(lens[i])) for i in s) for s in shards]
    info = {"tokens_per_rank": [int(lens[s].sum()) for s in shards], "prompts_per_rank": [len(s) for s in shards],
            "cost_imbalance": max(costs) / (sum(costs) / world), "split": "LPT on per-prompt FLOPs (linear + attention)"}
    return mine, my_ids, my_cu, info


class Clocks:
    """nvidia-smi sampling during the timed region: the sampler is started and
    its first sample read before the region begins (that sample is dropped),
    then it samples every 50 ms until the region ends."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu: int):
        self.gpu = gpu
        self.p = None

    def __enter__(self):
        try:
            self.p = subprocess.Popen(["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                       "-lms", "50"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.p.stdout.readline()  # the sampler is running: this sample precedes the timed region
        except OSError:
            self.p = None
        return self

    def __exit__(self, *a):
        self.lines = []
        if self.p is not None:
            self.p.terminate()
            try:
                out, _ = self.p.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.p.kill()
                out, _ = self.p.communicate()
            self.lines = [l for l in out.splitlines() if l.strip()]

    def summary(self) -> dict:
        sm, pw, mx, reasons = [], [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for l in getattr(self, "lines", []):
            f = [x.strip() for x in l.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            try:
                pw.append(float(f[3]))
            except ValueError:
                pass
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm),
                "power_w": statistics.median(pw) if pw else None}


# ---------------------------------------------------------------- CPU baseline / reference arm

def cpu_sample(lens: np.ndarray, every: int = 32) -> np.ndarray:
    """The fixed sample of the batch the CPU times: every 32nd prompt (8 of
    256: the same length distribution, ~2.2 k tokens)."""
    return np.arange(0, len(lens), every)


def cpu_model() -> str:
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def cpu_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def cpu_forward_rate(threads: int, steps: int, warmup: int) -> dict:
    """tokens/s of the C++ oracle (oracle/cpu_encoder.cpp: the encoder + head in
    f32 storage with f64 accumulation) over the fixed sample, `threads` threads."""
    from laya_js_b200 import workloads as WL
    from oracle import cpu
    W = WL.base_weights()
    lens, ids, cu = WL.cfg2_prompts()
    hw, hb = WL.head(WL.BASE, CLASSES)
    sel = cpu_sample(lens)
    seqs = [ids[cu[i]:cu[i + 1]] for i in sel]
    enc = cpu.Encoder(WL.BASE, W)
    times = []
    for i in range(warmup + steps):
        dt = enc.timed_forward(seqs, hw, hb, threads)
        if i >= warmup:
            times.append(dt)
    tokens = int(sum(len(s) for s in seqs))
    v = tokens / statistics.median(times)
    return {"value": v, "unit": "tokens/s", "cores": threads, "tokens_per_step": tokens, "ms_per_step": statistics.median(times) * 1e3}


def cpu_baseline() -> dict:
    """Rank 0 at N=1: the C++ oracle on one thread and on all host threads."""
    allt = cpu_threads()
    one = cpu_forward_rate(1, 1, 0)
    many = cpu_forward_rate(allt, 2, 1)
    return {"value": many["value"], "unit": "tokens/s", "cores": allt, "kind": "port",
            "single_thread": {"value": one["value"], "unit": "tokens/s", "cores": 1},
            "nproc": os.cpu_count(), "cpu_model": cpu_model(),
            "sample": f"every 32nd prompt of the configs[2] batch (8 prompts, {many['tokens_per_step']} tokens) per step, "
                      "C++ oracle (f32 storage, f64 accumulation, std::thread workers), same weights and head"}


def _batch_tokens(world: int) -> tuple[int, int]:
    """(tokens of rank 0's shard, tokens of the global batch) of an N-rank run."""
    from laya_js_b200 import workloads as WL
    lens, ids, cu = WL.cfg2_prompts(BATCH * world)
    _, my_ids, _, _ = shard(lens, ids, cu, 0, world)
    return int(len(my_ids)), int(lens.sum())


def run_reference(args, rank: int, world: int) -> None:
    """--impl reference: the reference's CPU path on this box's host cores. The
    reference's own CPU backend (npm @johnhenry/math-plus-tensor-cpu) is not
    vendored and no JS runtime exists, so the C++ port of its semantics
    (oracle/cpu_encoder.cpp) stands in, with every host thread; each step is the
    fixed sample of the configs[2] batch. Rank 0 alone runs and prints."""
    if rank != 0:
        return
    threads = cpu_threads()
    r = cpu_forward_rate(threads, args.steps, args.warmup)
    v = r["value"]
    line = {"impl": "reference", "metric": METRIC, "value": v, "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": r["ms_per_step"], "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded random-init N(0,0.02) weights, uniform token ids)",
            "config": config_of(world, *_batch_tokens(world)),
            "cpu_baseline": {"value": v, "unit": "tokens/s", "cores": threads, "kind": "port", "nproc": os.cpu_count(),
                             "cpu_model": cpu_model(),
                             "sample": f"every 32nd prompt of the configs[2] batch ({r['tokens_per_step']} tokens) per step"},
            "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "note": "the reference CPU backend (npm math-plus-tensor-cpu) is not vendored and no JS runtime exists; "
                    "the C++ port of its semantics (f32 storage, f64 accumulation) stands in"}
    print(json.dumps(line))


# ---------------------------------------------------------------- GPU arm

def b_stream(b) -> int:
    import ctypes as C
    from laya_js_b200 import _lib
    s = C.c_uint64()
    _lib.call("lc_get_stream", C.byref(s))
    return s.value


class Events:
    """CUDA events on the library stream (wrapped as a torch ExternalStream)."""

    def __init__(self, b):
        import torch
        self.torch = torch
        self.stream = torch.cuda.ExternalStream(b_stream(b))

    def time(self, fn, reps: int) -> float:
        """Device ms from before the first to after the last of `reps` calls."""
        t = self.torch
        t.cuda.synchronize()
        e0, e1 = t.cuda.Event(enable_timing=True), t.cuda.Event(enable_timing=True)
        with t.cuda.stream(self.stream):
            e0.record(self.stream)
            for _ in range(reps):
                fn()
            e1.record(self.stream)
        t.cuda.synchronize()
        return e0.elapsed_time(e1)

    def p50(self, fn, reps: int = 50, warm: int = 5) -> float:
        for _ in range(warm):
            fn()
        return statistics.median(self.time(fn, 1) for _ in range(reps))


def latency_cfg0(b, ev, fused, thw, thb, graph: bool = False) -> float:
    """batch 1, seq 128 (CLS ... SEP), the 3-way head; p50 over 50
    end-to-end calls (host ids in, host probabilities out), eager or as a
    captured CUDA graph; CUDA events on the library stream around each call."""
    from laya_js_b200 import workloads as WL
    _, ids, cu = WL.cfg0_prompt()
    out = np.empty((1, thw.shape[0]), np.float32)
    g = fused.graph(cu, thw, thb) if graph else None
    call = (lambda: g.run(ids, out=out)) if graph else (lambda: fused.forward_host(ids, cu, thw, thb, out=out))
    ms = ev.p50(call)
    if g is not None:
        g.free()
    return ms


def quantized_leg(b, ev, bits: int, steps: int) -> dict:
    """all Linear weights `bits`-bit affine g64 (fp16 scales/biases), 512 prompts, L~U[64,1024]."""
    from laya_js_b200 import encoder as E, workloads as WL
    from laya_js_b200.host import HostTensor
    from laya_js_b200.modernbert import loadModernBert, parseModernBertConfig
    W = WL.base_weights()
    enc = loadModernBert(b, parseModernBertConfig(WL.BASE), WL.host_getter(W, quant_bits=bits, group=64), "f16")
    fused = E.FusedEncoder(enc)
    lens, ids, cu = WL.cfg3_prompts()
    tids = b.fromHost(HostTensor("i32", ids.shape, ids))
    hw, hb = WL.head(WL.BASE, CLASSES)
    thw, thb = b.fromHost(HostTensor("f16", hw.shape, hw)), b.fromHost(HostTensor("f32", hb.shape, hb))

    def step():
        _, p = fused.forward(tids, cu, thw, thb, want_hidden=False)
        b.dispose(p)
    for _ in range(3):
        step()
    ms = ev.time(step, steps)
    T = int(cu[-1])
    hw3, hb3 = WL.head(WL.BASE, 3)
    t3w, t3b = b.fromHost(HostTensor("f16", hw3.shape, hw3)), b.fromHost(HostTensor("f32", hb3.shape, hb3))
    lat = latency_cfg0(b, ev, fused, t3w, t3b, graph=True)
    for t in (tids, thw, thb, t3w, t3b):
        b.dispose(t)
    fused.free()
    enc.dispose()
    return {"value": T * steps / (ms / 1e3), "unit": "tokens/s", "steps": steps, "ms_per_step": ms / steps, "tokens_per_step": T,
            "config": f"configs[3]: {bits}-bit affine g64 (fp16 scales and biases), batch 512, L~U[64,1024], 8-way head",
            "p50_latency_graph_ms": lat, "latency_config": f"configs[0] (one 128-token prompt, 3-way head) with these {bits}-bit weights"}


def large_leg(b, ev, steps: int, n_prompts: int = 1024) -> dict:
    """ModernBERT-large / mmBERT shape (28 layers, hidden 1024, 16
    heads, GeGLU 2624, vocab 256000) in bf16, 16-way CLS head; the first
    `n_prompts` of the 65,536-prompt log-uniform [16, 4096] length draw."""
    from laya_js_b200 import encoder as E, workloads as WL
    from laya_js_b200.host import HostTensor
    from laya_js_b200.modernbert import loadModernBert, parseModernBertConfig
    W = WL.large_weights_bf16()
    enc = loadModernBert(b, parseModernBertConfig(WL.LARGE), WL.host_getter(W), "bf16")
    del W
    fused = E.FusedEncoder(enc)
    lens = WL.cfg4_lengths()[:n_prompts]
    ids, cu = WL.cfg4_tokens(lens)
    tids = b.fromHost(HostTensor("i32", ids.shape, ids))
    hw, hb = WL.head(WL.LARGE, 16)
    thw, thb = b.fromHost(HostTensor("f16", hw.shape, hw)), b.fromHost(HostTensor("f32", hb.shape, hb))

    def step():
        _, p = fused.forward(tids, cu, thw, thb, want_hidden=False)
        b.dispose(p)
    step()
    ms = ev.time(step, steps)
    # one more step with CUDA events around every kernel class (not timed above)
    E.set_profiling(fused, True)
    E.profile_read(fused)
    step()
    b.flush()
    prof = E.profile_read(fused)
    E.set_profiling(fused, False)
    T = int(cu[-1])
    flops = linear_flops_per_token(WL.LARGE) * T
    aflops = attention_flops(WL.LARGE, lens)
    for t in (tids, thw, thb):
        b.dispose(t)
    fused.free()
    enc.dispose()
    return {"value": T * steps / (ms / 1e3), "unit": "tokens/s", "steps": steps, "ms_per_step": ms / steps, "tokens_per_step": T,
            "linear_tflops": flops / (ms / steps / 1e3) / 1e12,
            "linear_tflops_note": "linear-layer FLOPs over the whole step's time (attention included)",
            "kernel_ms_per_step": {k: v["ms"] for k, v in prof.items()},
            "gemm_tflops": flops / (prof["gemm"]["ms"] / 1e3) / 1e12 if prof["gemm"]["ms"] > 0 else None,
            "attention_tflops": aflops / (prof["attention"]["ms"] / 1e3) / 1e12 if prof["attention"]["ms"] > 0 else None,
            "attention_tflop_per_step": aflops / 1e12,
            "config": f"configs[4]: ModernBERT-large/mmBERT shape bf16, 28 layers, the first {n_prompts} prompts of the 65,536 "
                      "log-uniform [16,4096] draw, 16-way head"}


def contract_leg(b, ev, enc, thw3, thb3, thw8, thb8) -> dict:
    """ModernBert.encode through the Backend<T> ops (modernbert.py, the path of
    laya's load()/predict()): host ids + mask in (masks built on the host and
    uploaded, as packages/modernbert/src/index.ts:369-384 does), the CLS head as
    slice → linear → softmax, probabilities read back to the host."""
    from laya_js_b200 import workloads as WL

    def run(seqs, tw, tb):
        B, L = len(seqs), max(len(s) for s in seqs)
        pad = np.zeros((B, L), np.int32)
        valid = np.zeros((B, L), np.uint8)
        for i, s in enumerate(seqs):
            pad[i, :len(s)] = s
            valid[i, :len(s)] = 1

        def f():
            hid = enc.forward(pad, valid, B, L)
            H = hid.shape[-1]
            cls = b.reshape(b.slice(hid, [0, 0, 0], [B, 1, H]), [B, H])
            return b.read(b.softmax(b.linear(cls, tw, tb), -1))
        return lambda: b.scope(f)

    _, ids0, cu0 = WL.cfg0_prompt()
    lat = ev.p50(run([ids0], thw3, thb3), reps=30)
    lens, ids, cu = WL.cfg2_prompts()
    seqs = [ids[cu[i]:cu[i + 1]] for i in range(len(lens))]
    call = run(seqs, thw8, thb8)
    # the first calls of a process can take several times longer (a one-off
    # of 0.6 s was seen on the second call): median of 5 after 2 warm calls
    for _ in range(2):
        call()
    ms = statistics.median(ev.time(call, 1) for _ in range(5))
    T = int(lens.sum())
    return {"p50_latency_ms_cfg0": lat,
            "cfg2_padded": {"value": T / (ms / 1e3), "unit": "tokens/s (valid tokens)", "ms_per_step": ms,
                            "padded_tokens": int(len(lens) * lens.max()), "valid_tokens": T},
            "what": "ModernBert.forward over Backend<T> ops (tcgen05 linear, sdpa on the padded batch with host masks, "
                    "row kernels) + CLS head, host buffers in and out, CUDA events on the library stream"}


def microbench_leg(b, ev, hbm_peak: float, peak_src: str = "measured copy bandwidth (MEASURED_PEAKS.json)") -> dict:
    """the tensor-backend op microbench — add, mul, GELU, row
    broadcast add, row sum / max, softmax and LayerNorm over [M, N] in f16 and
    f32, M in {1024, 16384, 262144}, N in {768, 1152, 2304}, values N(0, 1)
    from one seeded buffer (the second operand of add / mul is its negation,
    in its own memory). GB/s = algorithmic bytes (inputs read once, output
    written once) / CUDA-event time per launch; only M = 262144 exceeds L2 at
    every N."""
    from laya_js_b200.host import HostTensor
    Ms, Ns = (1024, 16384, 262144), (768, 1152, 2304)
    rng = np.random.default_rng(20261201 + 30)
    nmax = Ms[-1] * Ns[-1]
    flat32 = b.fromHost(HostTensor("f32", (nmax,), rng.standard_normal(nmax, dtype=np.float32)))
    flat16 = b.cast(flat32, "f16")
    out: dict = {}
    fracs = []
    for dt, flat, e in (("f16", flat16, 2), ("f32", flat32, 4)):
        for N in Ns:
            g = b.fromHost(HostTensor(dt, (N,), np.ones(N, np.float16 if dt == "f16" else np.float32)))
            for M in Ms:
                x = b.reshape(b.slice(flat, [0], [M * N]), [M, N])
                y = b.neg(x)  # a second operand in its own memory (N(0, 1) as well)
                cases = (("add", lambda: b.add(x, y), 3 * M * N * e), ("mul", lambda: b.mul(x, y), 3 * M * N * e),
                         ("gelu", lambda: b.gelu(x), 2 * M * N * e), ("add_row", lambda: b.add(x, g), 2 * M * N * e + N * e),
                         ("sum", lambda: b.sum(x, -1), M * N * e + M * e), ("max", lambda: b.max(x, -1), M * N * e + M * e),
                         ("softmax", lambda: b.softmax(x, -1), 2 * M * N * e),
                         ("layerNorm", lambda: b.layerNorm(x, g, None, 1e-5), 2 * M * N * e + N * e))
                for name, fn, nbytes in cases:
                    run = lambda: b.dispose(fn())
                    run()
                    reps = 5
                    gbs = nbytes / (ev.time(run, reps) / reps * 1e-3) / 1e9
                    out.setdefault(f"{name}/{dt}", {}).setdefault(str(N), []).append(round(gbs, 1))
                    if M == Ms[-1]:
                        fracs.append(gbs / hbm_peak)
                b.dispose(x)
                b.dispose(y)
            b.dispose(g)
    b.dispose(flat16)
    b.dispose(flat32)
    return {"config": "configs[1]: add/mul/GELU/row-broadcast add/row sum/row max/softmax/LayerNorm, [M, N], "
                      "M in (1024, 16384, 262144), N in (768, 1152, 2304), f16 and f32, N(0, 1) seeded",
            "unit": "GB/s", "layout": "results[op/dtype][N] = GB/s at M = 1024, 16384, 262144",
            "peak_gbs": hbm_peak, "peak_src": peak_src,
            "frac_of_peak_at_M262144": {"median": round(statistics.median(fracs), 3), "min": round(min(fracs), 3),
                                        "max": round(max(fracs), 3)},
            "results": out}


def predict_leg(b, ev) -> dict:
    """The predict() path: the Laya DecisionModel (ModernBERT-base fp16 encoder +
    the two-layer head, scorer and action head, packages/laya/src/model.ts:124-285)
    through the contract ops on one 128-token prompt with four markers, host
    batch in and host logits/act out; p50 eager (forwardTensors) and through
    DecisionModel.compiled() (Backend.compile = one CUDA graph per signature)."""
    from laya_js_b200 import workloads as WL
    from laya_js_b200.decision import loadDecisionModel
    from laya_js_b200.host import HostTensor
    W = {**{k: v.astype(np.float32) for k, v in WL.base_weights().items()}, **WL.decision_head_weights(WL.BASE)}
    get = lambda n: HostTensor("f32", W[n].shape, W[n]) if n in W else None
    model = loadDecisionModel(b, dict(WL.BASE), {"head_layers": 2, "act_costs": {"escalate": 0.5}}, get, "f16")
    batch = WL.decision_batch(WL.BASE, [128])
    run = model.compiled()
    eager = ev.p50(lambda: model.readOutputs(model.forwardTensors(batch)), reps=30)
    graph = ev.p50(lambda: model.readOutputs(run(batch)), reps=30)
    del run
    model.dispose()
    return {"p50_predict_ms": eager, "p50_predict_compiled_ms": graph,
            "config": "DecisionModel (ModernBERT-base fp16 + laya head), 1 prompt of 128 tokens, 4 markers; "
                      "host batch in (ids, masks built on the host), logits + act read back"}


def main() -> None:
    args = parse()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank, world)
        return

    import torch
    dist = gloo = None
    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=torch.device(f"cuda:{local}"))
        gloo = dist.new_group(backend="gloo", timeout=datetime.timedelta(seconds=300))

    from laya_js_b200 import createCudaBackend, encoder as E, workloads as WL
    from laya_js_b200.host import HostTensor
    from laya_js_b200.modernbert import loadModernBert, parseModernBertConfig

    b = createCudaBackend(local)
    ev = Events(b)
    stream = ev.stream
    cfg_json = WL.BASE
    W = WL.base_weights()
    enc = loadModernBert(b, parseModernBertConfig(cfg_json), WL.host_getter(W), "f16")
    fused = E.FusedEncoder(enc)
    hw, hb = WL.head(cfg_json, CLASSES)
    thw = b.fromHost(HostTensor("f16", hw.shape, hw))
    thb = b.fromHost(HostTensor("f32", hb.shape, hb))
    lens_all, ids_all, cu_all = WL.cfg2_prompts(BATCH * world)
    mine, ids, cu, shard_info = shard(lens_all, ids_all, cu_all, rank, world)
    T = int(cu[-1])
    tok_total = int(lens_all.sum())
    tids = b.fromHost(HostTensor("i32", ids.shape, ids))

    def step():
        _, p = fused.forward(tids, cu, thw, thb, want_hidden=False)
        b.dispose(p)

    def barrier():
        if dist is not None:
            dist.barrier()

    def max_over_ranks(x: float) -> float:
        if dist is None:
            return x
        t = torch.tensor([x], device=f"cuda:{local}", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    for _ in range(args.warmup):
        step()
    b.flush()

    def timed(profile: bool):
        """K steps on device-resident inputs, CUDA events on the library stream."""
        E.set_profiling(fused, profile)
        E.profile_read(fused)
        l0 = b.stats()["launches"]
        barrier()
        torch.cuda.synchronize()
        with Clocks(local) as clk:
            with torch.cuda.stream(stream):
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(stream)
                for _ in range(args.steps):
                    step()
                e1.record(stream)
            torch.cuda.synchronize()
            b.flush()
        barrier()
        out = (max_over_ranks(e0.elapsed_time(e1)), b.stats()["launches"] - l0, E.profile_read(fused), clk.summary())
        E.set_profiling(fused, False)
        return out

    # ---- timed region (headline): no per-kernel events on the stream
    ms, launches, _, clocks = timed(False)
    # ---- second timed region: per-kernel-class CUDA events (roofline, breakdown)
    ms_prof, _, prof, _ = timed(True)
    value = tok_total * args.steps / (ms / 1e3)

    # ---- e2e: host ids -> host probabilities through the C ABI (copies inside
    # the timed region), then this step's probabilities gathered to rank 0 on the host
    probs = np.empty((len(mine), CLASSES), np.float32)
    gathered = np.zeros((len(lens_all), CLASSES), np.float32) if rank == 0 else None

    def e2e_step():
        fused.forward_host(ids, cu, thw, thb, out=probs)
        if gloo is not None:
            parts = [None] * world if rank == 0 else None
            dist.gather_object((mine, probs), parts, dst=0, group=gloo)
            if rank == 0:
                for idx, p in parts:
                    gathered[idx] = p
        else:
            gathered[mine] = probs

    for _ in range(2):
        e2e_step()
    barrier()
    e2e_ms = max_over_ranks(ev.time(e2e_step, args.steps))
    barrier()
    e2e_value = tok_total * args.steps / (e2e_ms / 1e3)
    if rank == 0:
        assert np.all(np.abs(gathered.sum(1) - 1) < 1e-3), "gathered probabilities incomplete"

    peaks = measured_peaks()
    gemm_flops = linear_flops_per_token(cfg_json) * T * args.steps
    g = prof["gemm"]
    achieved = gemm_flops / (g["ms"] / 1e3) / 1e12 if g["ms"] > 0 else None
    line = {
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "f16", "data": "synthetic (seeded random-init N(0,0.02) weights, uniform token ids)",
        "config": config_of(world, T, tok_total),
        "e2e": {"value": e2e_value, "unit": "tokens/s", "h2d_bytes_per_step": T * 4 + (len(mine) + 1) * 4,
                "d2h_bytes_per_step": len(mine) * CLASSES * 4,
                "what": "lc_encoder_forward_host per rank (H2D ids + cu_seqlens, D2H probabilities) and the host gather to rank 0"},
        "shards": shard_info,
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": peaks["bf16"], "unit": "TFLOP/s",
                     "frac": (achieved / peaks["bf16"]) if achieved else None, "traffic": GEMM_TRAFFIC_BYTES,
                     "traffic_src": "profiles/gemm_traffic_bench.md: ncu dram__bytes_read.sum + dram__bytes_write.sum per GEMM launch",
                     "flop_per_launch": gemm_flops / max(g["launches"], 1),
                     "kernel": "k_gemm_pair (tcgen05 CTA-pair GEMMs: Wqkv+RoPE+folded LN, Wo+residual, Wi+GeGLU+folded LN, mlp.Wo+residual)",
                     "peak_src": PEAK_SRC[peaks["src"]][0],
                     "gemm_ms_per_step": g["ms"] / args.steps, "gemm_launches_per_step": g["launches"] / args.steps,
                     "timing": "CUDA events around every GEMM launch on the library stream, second timed region of K steps"},
        "kernel_ms_per_step": {k: v["ms"] / args.steps for k, v in prof.items()},
        "profiled_ms_per_step": ms_prof / args.steps,
        "gpu_launches": launches,
        "clocks": clocks,
    }
    extras = rank == 0 and world == 1 and not args.no_extras
    if extras:
        hw3, hb3 = WL.head(cfg_json, 3)
        thw3, thb3 = b.fromHost(HostTensor("f16", hw3.shape, hw3)), b.fromHost(HostTensor("f32", hb3.shape, hb3))
        for key, fn in (("p50_latency_ms", lambda: latency_cfg0(b, ev, fused, thw3, thb3)),
                        ("p50_latency_graph_ms", lambda: latency_cfg0(b, ev, fused, thw3, thb3, graph=True))):
            try:
                line[key] = fn()
            except Exception as ex:  # noqa: BLE001
                line[key] = f"failed: {ex}"
        line["latency_config"] = "configs[0]: one 128-token prompt, 3-way CLS head, host ids in, host probabilities out"
        try:
            hb3_16 = b.fromHost(HostTensor("f16", hb3.shape, hb3.astype(np.float16)))
            hb8_16 = b.fromHost(HostTensor("f16", hb.shape, hb.astype(np.float16)))
            line["contract"] = contract_leg(b, ev, enc, thw3, hb3_16, thw, hb8_16)
        except Exception as ex:  # noqa: BLE001
            line["contract"] = f"failed: {ex}"
    fused.free()
    enc.dispose()
    b.dispose(tids)
    if extras:
        try:
            line["predict"] = predict_leg(b, ev)
        except Exception as ex:  # noqa: BLE001
            line["predict"] = f"failed: {ex}"
        q = {}
        for bits in (4, 8):
            try:
                q[f"int{bits}"] = quantized_leg(b, ev, bits, min(args.steps, 10))
            except Exception as ex:  # noqa: BLE001
                q[f"int{bits}"] = f"failed: {ex}"
        line["quantized"] = q
        try:
            line["large_bf16"] = large_leg(b, ev, min(args.steps, 3))
        except Exception as ex:  # noqa: BLE001
            line["large_bf16"] = f"failed: {ex}"
        try:
            line["microbench"] = microbench_leg(b, ev, peaks["hbm"], PEAK_SRC[peaks["src"]][1])
        except Exception as ex:  # noqa: BLE001
            line["microbench"] = f"failed: {ex}"
        try:
            line["cpu_baseline"] = cpu_baseline()
        except Exception as ex:  # noqa: BLE001
            line["cpu_baseline"] = f"failed: {ex}"
    if rank == 0:
        print(json.dumps(line))
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
