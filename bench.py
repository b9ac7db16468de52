"""Benchmark: ModernBERT-base tokens/s on B200 through liblaya_cuda.

Workload: ModernBERT-base shape (22 layers, hidden
768, 12 heads, GeGLU 1152, window 128, RoPE 160000/10000), random-init fp16
weights N(0, 0.02), 256 prompts per GPU with lengths uniform in [32, 512]
(seeded), token ids uniform in [5, 50368) with CLS/SEP, an 8-way CLS
classifier + softmax. One step = one forward of that batch (ids -> class
probabilities) through the fused varlen encoder (lc_encoder_forward).

Multi-GPU (torchrun): one process per GPU, full weight replica on each,
every rank runs its own 256-prompt batch (weak scaling); no collective on the
data path — NCCL is used only for the barrier and the max-over-ranks time.

Keys beyond the driver's contract:
  e2e        the same metric through lc_encoder_forward_host (host ids in,
             host probabilities out, copies inside the timed region);
  roofline   the tcgen05 GEMMs (dominant kernel class) vs the measured
             sustained bf16 tensor peak, with their DRAM traffic per launch
             from the committed ncu capture;
  cpu_baseline  the numpy oracle (float64) on a bounded sample, all cores;
  int4       configs[3]-style 4-bit affine g64 weights (batch 512, lengths
             U[64, 1024]) tokens/s on the same GPU, and the p50 graph latency
             of one 128-token prompt with those weights (fused-dequant GEMMs);
  p50_latency_ms  configs[0] (batch 1, seq 128) end-to-end latency;
  p50_latency_graph_ms  the same through a captured CUDA graph
             (lc_encoder_graph_run).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

BATCH, LO, HI, CLASSES = 256, 32, 512, 8
SEED = 20261201
# DRAM bytes per GEMM launch of this workload (average over the four projections),
# from the committed one-pass ncu capture in profiles/gemm_traffic_bench.md
GEMM_TRAFFIC_BYTES = 306.6e6


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", default="ours", choices=["ours", "reference"])
    p.add_argument("--no-extras", action="store_true", help="skip the int4 / latency / CPU-baseline legs")
    return p.parse_args()


def linear_flops_per_token(cfg: dict) -> float:
    H, I, n = cfg["hidden_size"], cfg["intermediate_size"], cfg["num_hidden_layers"]
    return 2.0 * (H * 3 * H + H * H + H * 2 * I + I * H) * n


def measured_peaks() -> dict:
    f = ROOT / "MEASURED_PEAKS.json"
    if f.exists():
        d = json.loads(f.read_text())
        return {"bf16": d.get("bf16_tflops_sustained", 1417.5), "hbm": d.get("hbm_gbs", 6449.7), "src": "measured"}
    return {"bf16": 1400.0, "hbm": 6650.0, "src": "fallback"}


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


def cpu_baseline(cfg_json: dict, W: dict, ids: np.ndarray, cu: np.ndarray, budget_s: float = 12.0) -> dict:
    """The oracle (numpy float64 restatement of the reference CPU backend) on a
    bounded sample of the same batch: whole sequences until `budget_s` elapse."""
    from oracle import models as M
    ocfg = M.parse_config(cfg_json)
    Wf = {k: v.astype(np.float32) for k, v in W.items()}
    t0 = time.perf_counter()
    tokens = n = 0
    for s in range(len(cu) - 1):
        seq = ids[cu[s]:cu[s + 1]]
        M.encoder_varlen(ocfg, Wf, [seq])
        tokens += len(seq)
        n += 1
        if time.perf_counter() - t0 > budget_s:
            break
    dt = time.perf_counter() - t0
    return {"value": tokens / dt, "unit": "tokens/s", "cores": os.cpu_count(), "kind": "port",
            "sample": f"{n} of {len(cu) - 1} sequences ({tokens} tokens) of the same batch, numpy float64 oracle, {dt:.1f} s"}


def run_reference(args, rank: int, world: int) -> None:
    """--impl reference: the reference's CPU path (here: the oracle port, since
    backend-cpu is an un-vendored npm package and no JS runtime exists) on this
    box's host cores, same config/metric; rank 0 only."""
    if rank != 0:
        return
    from laya_js_b200 import workloads as WL
    cfg_json = WL.BASE
    W = WL.random_weights(cfg_json, seed=SEED)
    lens = WL.lengths(BATCH, LO, HI, seed=SEED + 1)
    ids, cu = WL.token_batch(cfg_json, lens, seed=SEED + 2)
    steps = []
    for i in range(args.warmup + args.steps):
        r = cpu_baseline(cfg_json, W, ids, cu, budget_s=4.0 if i < args.warmup else 8.0)
        if i >= args.warmup:
            steps.append(r)
    v = statistics.median(s["value"] for s in steps)
    line = {"impl": "reference", "metric": "modernbert_base_fp16_tokens_per_s", "value": v, "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "f64", "data": "synthetic (seeded random-init weights and token ids)",
            "config": {"workload": "configs[2]: ModernBERT-base, batch 256 varlen L~U[32,512], 8-way CLS head", "global_batch": BATCH,
                       "seq_len": f"U[{LO},{HI}]"},
            "cpu_baseline": {**steps[-1], "value": v},
            "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "note": "reference CPU backend (npm math-plus-tensor-cpu) is not vendored and no JS runtime exists; the numpy port of its semantics stands in"}
    print(json.dumps(line))


def main() -> None:
    args = parse()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank, world)
        return

    import torch
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=torch.device(f"cuda:{local}"))
    else:
        torch.cuda.set_device(local)

    from laya_js_b200 import createCudaBackend, encoder as E, workloads as WL
    from laya_js_b200.host import HostTensor
    from laya_js_b200.modernbert import loadModernBert, parseModernBertConfig

    b = createCudaBackend(local)
    stream = torch.cuda.ExternalStream(b_stream(b))
    cfg_json = WL.BASE
    cfg = parseModernBertConfig(cfg_json)
    W = WL.random_weights(cfg_json, seed=SEED)
    enc = loadModernBert(b, cfg, WL.host_getter(W), "f16")
    fused = E.FusedEncoder(enc)
    hw, hb = WL.classifier(cfg_json, CLASSES, seed=SEED + 3)
    thw = b.fromHost(HostTensor("f16", hw.shape, hw))
    thb = b.fromHost(HostTensor("f32", hb.shape, hb))
    lens = WL.lengths(BATCH, LO, HI, seed=SEED + 1 + 1000 * rank)
    ids, cu = WL.token_batch(cfg_json, lens, seed=SEED + 2 + 1000 * rank)
    T = int(cu[-1])
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
    tok_total = T * world  # every rank's batch has its own lengths; sum them exactly
    if dist is not None:
        t = torch.tensor([T], device=f"cuda:{local}", dtype=torch.float64)
        dist.all_reduce(t)
        tok_total = int(t.item())
    value = tok_total * args.steps / (ms / 1e3)

    # ---- e2e: host ids -> host probabilities through the C ABI (copies inside the timed region)
    probs = np.empty((BATCH, CLASSES), np.float32)
    for _ in range(2):
        fused.forward_host(ids, cu, thw, thb, out=probs)
    barrier()
    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        f0.record(stream)
        for _ in range(args.steps):
            fused.forward_host(ids, cu, thw, thb, out=probs)
        f1.record(stream)
    torch.cuda.synchronize()
    barrier()
    e2e_ms = max_over_ranks(f0.elapsed_time(f1))
    e2e_value = tok_total * args.steps / (e2e_ms / 1e3)

    peaks = measured_peaks()
    gemm_flops = linear_flops_per_token(cfg_json) * T * args.steps
    g = prof["gemm"]
    achieved = gemm_flops / (g["ms"] / 1e3) / 1e12 if g["ms"] > 0 else None
    line = {
        "metric": "modernbert_base_fp16_tokens_per_s", "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "f16", "data": "synthetic (seeded random-init N(0,0.02) weights, uniform token ids)",
        "config": {"workload": "configs[2]: ModernBERT-base fp16, 256 prompts/GPU varlen L~U[32,512], 8-way CLS head + softmax",
                   "global_batch": BATCH * world, "seq_len": f"U[{LO},{HI}]", "tokens_per_gpu_step": T, "parallelism": f"dp{world}",
                   "l2": "inputs larger than L2 (activations ~0.5 GB per step)"},
        "e2e": {"value": e2e_value, "unit": "tokens/s", "h2d_bytes_per_step": T * 4 + (BATCH + 1) * 4,
                "d2h_bytes_per_step": BATCH * CLASSES * 4},
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": peaks["bf16"], "unit": "TFLOP/s",
                     "frac": (achieved / peaks["bf16"]) if achieved else None, "traffic": GEMM_TRAFFIC_BYTES,
                     "traffic_src": "profiles/gemm_traffic_bench.md: ncu dram__bytes_read.sum + dram__bytes_write.sum per GEMM launch, "
                                    "one-pass capture of this workload",
                     "flop_per_launch": gemm_flops / max(g["launches"], 1),
                     "kernel": "k_gemm_pair (tcgen05 CTA-pair GEMMs: Wqkv+RoPE+folded LN, Wo+residual, Wi+GeGLU+folded LN, mlp.Wo+residual)",
                     "peak_src": f"{peaks['src']} sustained bf16 (MEASURED_PEAKS.json)",
                     "gemm_ms_per_step": g["ms"] / args.steps, "gemm_launches_per_step": g["launches"] / args.steps,
                     "timing": "CUDA events around every GEMM launch on the library stream, second timed region of K steps"},
        "kernel_ms_per_step": {k: v["ms"] / args.steps for k, v in prof.items()},
        "profiled_ms_per_step": ms_prof / args.steps,
        "gpu_launches": launches,
        "clocks": clocks,
    }
    if rank == 0 and not args.no_extras:
        try:
            line["p50_latency_ms"] = latency_cfg0(b, fused, thw, thb, cfg_json)
            line["p50_latency_graph_ms"] = latency_cfg0(b, fused, thw, thb, cfg_json, graph=True)
        except Exception as ex:  # noqa: BLE001
            line["p50_latency_ms"] = f"failed: {ex}"
        try:
            line["cpu_baseline"] = cpu_baseline(cfg_json, W, ids, cu)
        except Exception as ex:  # noqa: BLE001
            line["cpu_baseline"] = f"failed: {ex}"
    fused.free()
    enc.dispose()
    if rank == 0 and not args.no_extras:
        try:
            line["int4"] = int4_leg(b, min(args.steps, 10))
        except Exception as ex:  # noqa: BLE001
            line["int4"] = f"failed: {ex}"
    if rank == 0:
        print(json.dumps(line))
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


def b_stream(b) -> int:
    import ctypes as C
    from laya_js_b200 import _lib
    s = C.c_uint64()
    _lib.call("lc_get_stream", C.byref(s))
    return s.value


def latency_cfg0(b, fused, thw, thb, cfg_json, graph: bool = False) -> float:
    """batch 1, seq 128 (CLS ... SEP), p50 over 50 end-to-end calls
    (host ids in, host probabilities out), eager or as a captured CUDA graph."""
    from laya_js_b200 import workloads as WL
    ids, cu = WL.token_batch(cfg_json, np.array([128]), seed=SEED + 5)
    out = np.empty((1, thw.shape[0]), np.float32)
    g = fused.graph(cu, thw, thb) if graph else None
    call = (lambda: g.run(ids, out=out)) if graph else (lambda: fused.forward_host(ids, cu, thw, thb, out=out))
    for _ in range(5):
        call()
    ts = []
    for _ in range(50):
        t0 = time.perf_counter()
        call()
        ts.append((time.perf_counter() - t0) * 1e3)
    if g is not None:
        g.free()
    return statistics.median(ts)


def int4_leg(b, steps: int) -> dict:
    """all Linear weights 4-bit affine g64 (fp16 scales/biases), 512 prompts, L~U[64,1024]."""
    import torch
    from laya_js_b200 import encoder as E, workloads as WL
    from laya_js_b200.host import HostTensor
    from laya_js_b200.modernbert import loadModernBert, parseModernBertConfig
    cfg_json = WL.BASE
    W = WL.random_weights(cfg_json, seed=SEED)
    enc = loadModernBert(b, parseModernBertConfig(cfg_json), WL.host_getter(W, quant_bits=4, group=64), "f16")
    fused = E.FusedEncoder(enc)
    lens = WL.lengths(512, 64, 1024, seed=SEED + 7)
    ids, cu = WL.token_batch(cfg_json, lens, seed=SEED + 8)
    tids = b.fromHost(HostTensor("i32", ids.shape, ids))
    for _ in range(3):
        h, _ = fused.forward(tids, cu, want_hidden=True)
        b.dispose(h)
    stream = torch.cuda.ExternalStream(b_stream(b))
    torch.cuda.synchronize()
    b.flush()
    with torch.cuda.stream(stream):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(steps):
            h, _ = fused.forward(tids, cu, want_hidden=True)
            b.dispose(h)
        e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    T = int(cu[-1])
    b.dispose(tids)
    # one 128-token prompt with these weights (the packed-weight GEMMs), as a CUDA graph
    hw, hb = WL.classifier(cfg_json, CLASSES, seed=SEED + 3)
    thw = b.fromHost(HostTensor("f16", hw.shape, hw))
    thb = b.fromHost(HostTensor("f32", hb.shape, hb))
    lat = latency_cfg0(b, fused, thw, thb, cfg_json, graph=True)
    b.dispose(thw)
    b.dispose(thb)
    fused.free()
    enc.dispose()
    return {"value": T * steps / (ms / 1e3), "unit": "tokens/s", "steps": steps, "tokens_per_step": T,
            "config": "configs[3]: 4-bit affine g64, batch 512, L~U[64,1024], hidden states out",
            "p50_latency_graph_ms": lat, "latency_config": "configs[0] shape (one 128-token prompt) with these 4-bit weights"}


if __name__ == "__main__":
    main()
