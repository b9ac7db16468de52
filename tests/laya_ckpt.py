"""Writes laya quantized checkpoints (format version 1,
packages/laya/docs/QUANTIZATION.md:91-117) for the ingestion tests: the four
Linear weights of every ModernBERT layer quantized — q8 symmetric (scale =
max|w| / 127 rounded to f16, q = round(w / scale) clamped to [-127, 127],
packages/laya/src/quant.ts range fit) or q4 affine (bias = min, scale = (max −
min) / 15, both f16, q = round((w − bias) / scale) clamped to [0, 15], packed
two per byte with the even column in the low nibble) — and every other tensor
as plain F16 / F32."""
from __future__ import annotations

import numpy as np

from laya_js_b200 import workloads as WL

LINEAR = (".attn.Wqkv.weight", ".attn.Wo.weight", ".mlp.Wi.weight", ".mlp.Wo.weight")


def quantize_q8(w: np.ndarray, g: int):
    N, K = w.shape
    wg = w.astype(np.float64).reshape(N, K // g, g)
    s = (np.abs(wg).max(axis=2) / 127).astype(np.float16)
    s64 = s.astype(np.float64)[..., None]
    with np.errstate(divide="ignore", invalid="ignore"):
        q = np.where(s64 > 0, np.floor(wg / np.where(s64 > 0, s64, 1) + 0.5), 0)
    return np.clip(q, -127, 127).astype(np.int8).reshape(N, K), s


def write(path: str, W: dict, scheme: str, g: int = 64) -> dict:
    """Writes the checkpoint; returns {name: dequantised f32 values} of the quantized matrices."""
    from safetensors.numpy import save_file
    out, deq = {}, {}
    for name, a in W.items():
        if name.endswith(LINEAR):
            if scheme == "q8":
                q, s = quantize_q8(a, g)
                out[name], out[name + ".scales"] = q, s
                deq[name] = (q.astype(np.float64) * np.repeat(s.astype(np.float64), g, axis=1)).astype(np.float16).astype(np.float32)
            else:
                q, s, b = WL.quantize_affine(a, 4, g)
                out[name] = (q[:, 0::2] | (q[:, 1::2] << 4)).astype(np.uint8)
                out[name + ".scales"], out[name + ".biases"] = s, b
                r = lambda x: np.repeat(x.astype(np.float64), g, axis=1)
                deq[name] = (q.astype(np.float64) * r(s) + r(b)).astype(np.float16).astype(np.float32)
        else:
            out[name] = a
    save_file(out, path, metadata={"laya_quant": scheme, "group_size": str(g), "version": "1", "laya_quant_source_dtype": "F16"})
    return deq
