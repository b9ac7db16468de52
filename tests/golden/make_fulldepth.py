"""Writes ``fulldepth.npz``: the CPU oracle's outputs for the benchmark
configurations at their full depth, so the GPU parity tests can check the
22- and 28-layer forwards that bench.py times without spending minutes of
float64 work on the GPU box.

Every input comes from ``laya_js_b200.workloads`` (the seeds bench.py uses):

- ``cfg2``: configs[2], ModernBERT-base fp16, 22 layers, LayerNorm weights 1,
  the 8-way head; 8 of the 256 prompts of the bench's batch (the longest, the
  shortest and six fixed positions).
- ``cfg0``: configs[0], one 128-token prompt, the 3-way head.
- ``cfg3_q4`` / ``cfg3_q8``: configs[3], every Linear weight 4-bit / 8-bit
  affine g64 (fp16 scales and biases) quantized from the configs[2] fp16
  weights; the oracle computes with the dequantised values (each rounded once
  to fp16); 6 of the 512 prompts (the longest, the shortest, four fixed).
- ``cfg4``: configs[4], ModernBERT-large / mmBERT shape (28 layers, hidden
  1024, vocab 256000) with bf16 weights, the 16-way head; a batch of the
  first 7 prompts of the 65,536-prompt length draw plus one of 4096 tokens.

Per case: ``<case>.idx`` (positions of the checked prompts in the GPU batch),
``.lens`` (lengths of the whole GPU batch), ``.rows`` [n, 3, H] (final-norm
hidden rows at positions 0, L//2, L-1 of each checked prompt), ``.logits`` and
``.probs`` [n, C] (the CLS head, float64).

Usage: ``python tests/golden/make_fulldepth.py`` (about 10 minutes on 8 cores).
"""
from __future__ import annotations

import sys
import time
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent))

from laya_js_b200 import workloads as WL  # noqa: E402
from oracle import models as M  # noqa: E402
from oracle import ops as O  # noqa: E402

LINEAR = (".attn.Wqkv.weight", ".attn.Wo.weight", ".mlp.Wi.weight", ".mlp.Wo.weight")


def subset(lens: np.ndarray, fixed) -> np.ndarray:
    return np.array(sorted({int(np.argmax(lens)), int(np.argmin(lens)), *[int(f) % len(lens) for f in fixed]}))


def oracle_weights(W: dict, bits: int = 0) -> dict:
    """The weights the device computes with, as f32 (dequantised values when quantized)."""
    out = {}
    for k, v in W.items():
        if bits and k.endswith(LINEAR):
            q, s, b = WL.quantize_affine(v, bits, 64)
            out[k] = O.dequantize(q, s, b, 64, np.float16).astype(np.float32)
        else:
            out[k] = v.astype(np.float32)
    return out


def run_case(store: dict, name: str, cfg: dict, Wf: dict, ids, cu, lens, idx, classes: int) -> None:
    t0 = time.time()
    ocfg = M.parse_config(cfg)
    hw, hb = WL.head(cfg, classes)
    seqs = [ids[cu[s]:cu[s + 1]] for s in idx]
    hid = M.encoder_varlen(ocfg, Wf, seqs)
    rows = np.stack([h[[0, len(h) // 2, len(h) - 1]] for h in hid]).astype(np.float32)
    cls = np.stack([h[0] for h in hid])
    logits = cls.astype(np.float64) @ hw.astype(np.float64).T + hb.astype(np.float64)
    z = logits - logits.max(1, keepdims=True)
    probs = np.exp(z) / np.exp(z).sum(1, keepdims=True)
    store.update({f"{name}.idx": np.asarray(idx, np.int64), f"{name}.lens": np.asarray(lens, np.int64), f"{name}.rows": rows,
                  f"{name}.logits": logits, f"{name}.probs": probs})
    print(f"{name}: {len(idx)} prompts, {sum(len(s) for s in seqs)} tokens, {time.time() - t0:.0f} s", flush=True)


def main() -> None:
    store: dict = {}
    W = WL.base_weights()
    Wf = oracle_weights(W)
    lens, ids, cu = WL.cfg2_prompts()
    run_case(store, "cfg2", WL.BASE, Wf, ids, cu, lens, subset(lens, [0, 37, 101, 150, 203, 255]), 8)
    lens, ids, cu = WL.cfg0_prompt()
    run_case(store, "cfg0", WL.BASE, Wf, ids, cu, lens, [0], 3)
    lens, ids, cu = WL.cfg3_prompts()
    idx = subset(lens, [0, 200, 400, 511])
    for bits in (4, 8):
        run_case(store, f"cfg3_q{bits}", WL.BASE, oracle_weights(W, bits), ids, cu, lens, idx, 8)
    del W, Wf
    lens = np.concatenate([WL.cfg4_lengths()[:7], [4096]])
    ids, cu = WL.cfg4_tokens(lens)
    run_case(store, "cfg4", WL.LARGE, WL.large_weights_bf16(), ids, cu, lens, np.arange(len(lens)), 16)
    np.savez_compressed(HERE / "fulldepth.npz", **store)
    print(f"wrote {HERE / 'fulldepth.npz'}")


if __name__ == "__main__":
    main()
