"""Small, self-contained cases of the hot kernels for profiling (ncu) and
quick timing. Each case fits in a few GB and ends in seconds.

    python -m laya_js_b200.profile_cases encoder   # 2-layer ModernBERT-base, 64 prompts L~U[32,512]
    python -m laya_js_b200.profile_cases gemm      # one 32768x2304x768 linear (f16)
    python -m laya_js_b200.profile_cases attention # varlen attention, 256 prompts, global + sliding
    python -m laya_js_b200.profile_cases hbm       # the HBM-bound contract ops on ~100-400 MB tensors
    python -m laya_js_b200.profile_cases prompt    # configs[0]: one 128-token prompt, 22 layers, CUDA-graph replays
    python -m laya_js_b200.profile_cases prompt_q4 # the same with 4-bit affine g64 weights (fused-dequant GEMMs)
    python -m laya_js_b200.profile_cases sdpa      # the contract's sdpa on the padded configs[2] batch (full / sliding masks)
    python -m laya_js_b200.profile_cases predict   # DecisionModel forward, one 128-token prompt, eager and compiled

Every case prints one line with its shape and the device time per launch
(CUDA events on the library stream, after warm-up).
"""
from __future__ import annotations

import ctypes as C
import sys
import time

import numpy as np

from . import _lib, workloads as WL
from .backend import createCudaBackend
from .encoder import FusedEncoder, attention_varlen
from .host import HostTensor
from .modernbert import loadModernBert, parseModernBertConfig


def _sync_time(b, fn, reps: int) -> float:
    b.flush()
    t0 = time.perf_counter()
    for _ in range(reps):
        fn()
    b.flush()
    return (time.perf_counter() - t0) / reps * 1e3


def case_encoder(b) -> str:
    cfg_json = {**WL.BASE, "num_hidden_layers": 2}
    W = WL.random_weights(cfg_json, seed=1)
    enc = loadModernBert(b, parseModernBertConfig(cfg_json), WL.host_getter(W), "f16")
    fused = FusedEncoder(enc)
    lens = WL.lengths(64, 32, 512, seed=2)
    ids, cu = WL.token_batch(cfg_json, lens, seed=3)
    tids = b.fromHost(HostTensor("i32", ids.shape, ids))

    def run():
        h, _ = fused.forward(tids, cu, want_hidden=True)
        b.dispose(h)
    run()
    ms = _sync_time(b, run, 3)
    fused.free()
    enc.dispose()
    return f"encoder 2 layers, T={int(cu[-1])} tokens: {ms:.3f} ms/forward"


def case_gemm(b) -> str:
    rng = np.random.default_rng(0)
    M, N, K = 32768, 2304, 768
    x = b.fromHost(HostTensor("f16", (M, K), rng.standard_normal((M, K), dtype=np.float32).astype(np.float16)))
    w = b.fromHost(HostTensor("f16", (N, K), (rng.standard_normal((N, K), dtype=np.float32) * 0.02).astype(np.float16)))
    run = lambda: b.dispose(b.linear(x, w))
    run()
    ms = _sync_time(b, run, 5)
    return f"gemm {M}x{N}x{K} f16: {ms * 1e3:.1f} us/launch, {2 * M * N * K / ms / 1e9:.0f} TFLOP/s (host-timed)"


def case_attention(b) -> str:
    rng = np.random.default_rng(0)
    lens = WL.lengths(256, 32, 512, seed=1)
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    T = int(cu[-1])
    qkv = b.fromHost(HostTensor("f16", (T, 2304), rng.standard_normal((T, 2304), dtype=np.float32).astype(np.float16)))
    out = []
    for hw in (-1, 64):
        run = lambda: b.dispose(attention_varlen(b, qkv, cu, hw, 0.125))
        run()
        out.append(f"{'global' if hw < 0 else 'sliding'} {_sync_time(b, run, 3):.3f} ms")
    return f"attention T={T}, 12 heads: " + ", ".join(out)


def _prompt(b, bits: int) -> str:
    import statistics
    cfg_json = WL.BASE
    W = WL.random_weights(cfg_json, seed=1)
    enc = loadModernBert(b, parseModernBertConfig(cfg_json), WL.host_getter(W, quant_bits=bits, group=64), "f16")
    fused = FusedEncoder(enc)
    hw, hb = WL.classifier(cfg_json, 3, seed=7)
    thw = b.fromHost(HostTensor("f16", hw.shape, hw))
    thb = b.fromHost(HostTensor("f32", hb.shape, hb))
    ids, cu = WL.token_batch(cfg_json, np.array([128]), seed=5)
    out = np.empty((1, 3), np.float32)
    g = fused.graph(cu, thw, thb)
    for _ in range(3):
        g.run(ids, out=out)
    ts = []
    for _ in range(20):
        t0 = time.perf_counter()
        g.run(ids, out=out)
        ts.append((time.perf_counter() - t0) * 1e3)
    g.free()
    fused.free()
    enc.dispose()
    return f"prompt L=128, 22 layers, {'f16' if bits == 0 else f'{bits}-bit'} weights, graph replay: p50 {statistics.median(ts):.3f} ms host to host"


def case_prompt(b) -> str:
    return _prompt(b, 0)


def case_prompt_q4(b) -> str:
    return _prompt(b, 4)


def case_hbm(b) -> str:
    """The HBM-bound contract ops on tensors larger than L2, each launch timed
    with its algorithmic bytes (read + write once) -> GB/s."""
    rng = np.random.default_rng(0)
    R, H = 65536, 768
    x = b.fromHost(HostTensor("f16", (R, H), rng.standard_normal((R, H), dtype=np.float32).astype(np.float16)))
    y = b.fromHost(HostTensor("f16", (R, H), rng.standard_normal((R, H), dtype=np.float32).astype(np.float16)))
    g = b.fromHost(HostTensor("f16", (H,), np.ones(H, np.float16)))
    z = b.fromHost(HostTensor("f16", (R, 2 * H), rng.standard_normal((R, 2 * H), dtype=np.float32).astype(np.float16)))
    V = 50368
    table = b.fromHost(HostTensor("f16", (V, H), (rng.standard_normal((V, H), dtype=np.float32) * 0.02).astype(np.float16)))
    ids = b.fromHost(HostTensor("i32", (R,), rng.integers(0, V, R, dtype=np.int32)))
    B, L = 128, 512
    mask = b.fromHost(HostTensor("i32", (B, L), np.ones((B, L), np.int32)))
    xb = b.reshape(x, [B, L, H])
    R2, N2 = 16384, 2304  # a configs[1] shape in f32
    xf = b.fromHost(HostTensor("f32", (R2, N2), rng.standard_normal((R2, N2), dtype=np.float32)))
    gf = b.fromHost(HostTensor("f32", (N2,), np.ones(N2, np.float32)))
    e = 2
    cases = [
        ("add [65536,768] f16", lambda: b.add(x, y), 3 * R * H * e),
        ("gelu [65536,768] f16", lambda: b.gelu(x), 2 * R * H * e),
        ("layerNorm [65536,768] f16", lambda: b.layerNorm(x, g, None, 1e-5), 2 * R * H * e),
        ("softmax rows [65536,768] f16", lambda: b.softmax(x, -1), 2 * R * H * e),
        ("geglu [65536,1536]->[65536,768] f16", lambda: b.geglu(z), (2 * R * H + R * H) * e),
        ("sum rows [65536,768] f16", lambda: b.sum(x, -1), R * H * e),
        ("embedding 65536 ids of [50368,768] f16", lambda: b.embedding(table, ids), 2 * R * H * e),
        ("meanPool [128,512,768] f16", lambda: b.meanPool(xb, mask), R * H * e),
        ("max rows [65536,768] f16", lambda: b.max(x, -1), R * H * e),
        ("mul row broadcast [65536,768]*[768] f16", lambda: b.mul(x, g), 2 * R * H * e),
        ("softmax rows [16384,2304] f32", lambda: b.softmax(xf, -1), 2 * R2 * N2 * 4),
        ("layerNorm [16384,2304] f32", lambda: b.layerNorm(xf, gf, None, 1e-5), 2 * R2 * N2 * 4),
        ("sum rows [16384,2304] f32", lambda: b.sum(xf, -1), R2 * N2 * 4),
    ]
    out = []
    for name, fn, nbytes in cases:
        run = lambda: b.dispose(fn())
        run()
        ms = _event_time(b, run, 10)
        out.append(f"{name}: {ms * 1e3:.1f} us, {nbytes / ms / 1e6:.0f} GB/s")
    return "hbm kernels (algorithmic bytes / CUDA-event time):\n  " + "\n  ".join(out)


def case_sdpa(b) -> str:
    """The contract's sdpa as ModernBert.layer calls it on the padded configs[2]
    batch (256 x 512, 12 heads; q/k dense, v a strided view of the QKV
    projection) with the full and sliding masks of attentionMasks."""
    from .modernbert import attentionMasks
    lens, _, _ = WL.cfg2_prompts()
    B, L, nh = len(lens), int(lens.max()), 12
    valid = (np.arange(L)[None, :] < lens[:, None]).astype(np.uint8)
    full, sliding = attentionMasks(valid, B, L, 128)
    rng = np.random.default_rng(0)
    qkv = b.fromHost(HostTensor("f16", (B, L, 3 * nh * 64), rng.standard_normal((B, L, 3 * nh * 64), dtype=np.float32).astype(np.float16)))
    t = b.transpose(b.reshape(qkv, [B, L, 3, nh, 64]), [2, 0, 3, 1, 4])
    q, k, v = [b.reshape(x, [B, nh, L, 64]) for x in b.split(t, 3, 0)]
    q, k = b.cast(q, "f16"), b.cast(k, "f16")  # dense, like rope's outputs
    out = []
    for name, m in (("full", full), ("sliding", sliding)):
        tm = b.fromHost(m)
        run = lambda: b.dispose(b.sdpa(q, k, v, tm, 0.125))
        run()
        out.append(f"{name} {_event_time(b, run, 5) * 1e3:.0f} us")
    return f"sdpa [{B},{nh},{L},64] padded configs[2] batch: " + ", ".join(out)


def case_predict(b) -> str:
    """The DecisionModel (ModernBERT-base fp16 + laya head) on one 128-token
    prompt: eager forward and DecisionModel.compiled() replays (CUDA graph)."""
    from .decision import loadDecisionModel
    W = {**{k: v.astype(np.float32) for k, v in WL.base_weights().items()}, **WL.decision_head_weights(WL.BASE)}
    get = lambda n: HostTensor("f32", W[n].shape, W[n]) if n in W else None
    model = loadDecisionModel(b, dict(WL.BASE), {"head_layers": 2, "act_costs": {"escalate": 0.5}}, get, "f16")
    batch = WL.decision_batch(WL.BASE, [128])
    run = model.compiled()
    eager = _event_time(b, lambda: model.readOutputs(model.forwardTensors(batch)), 5)
    for _ in range(3):
        model.readOutputs(run(batch))
    graph = _event_time(b, lambda: model.readOutputs(run(batch)), 5)
    del run
    model.dispose()
    return f"predict (DecisionModel, 1 x 128 tokens): eager {eager:.3f} ms, compiled {graph:.3f} ms"


def _event_time(b, fn, reps: int) -> float:
    """Device ms per call: CUDA events on the library stream around `reps` calls."""
    import torch
    s = C.c_uint64()
    _lib.call("lc_get_stream", C.byref(s))
    stream = torch.cuda.ExternalStream(s.value)
    b.flush()
    with torch.cuda.stream(stream):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(reps):
            fn()
        e1.record(stream)
    torch.cuda.synchronize()
    b.flush()
    return e0.elapsed_time(e1) / reps


def main(argv) -> None:
    b = createCudaBackend(0)
    cases = {"encoder": case_encoder, "gemm": case_gemm, "attention": case_attention, "hbm": case_hbm, "prompt": case_prompt,
             "prompt_q4": case_prompt_q4, "sdpa": case_sdpa, "predict": case_predict}
    for name in argv[1:] or list(cases):
        print(cases[name](b), flush=True)


if __name__ == "__main__":
    main(sys.argv)
