"""Seeded synthetic workloads with the shapes of the benchmark configurations:
ModernBERT-base / -large-shape random-init weights, token batches with the
stated length distributions, and 4/8-bit affine group quantization of the
Linear weights (packages/laya/src/quant.ts:157-187 min/max fit, no refinement).

No public dataset or checkpoint is involved: every tensor comes from
numpy's default_rng with the seed given.
"""
from __future__ import annotations

import numpy as np

from .host import HostQuantized, HostTensor, pack_quantized

CLS_ID, SEP_ID = 50281, 50282  # ModernBERT tokenizer [CLS] / [SEP]

BASE = {"model_type": "modernbert", "vocab_size": 50368, "hidden_size": 768, "intermediate_size": 1152,
        "num_hidden_layers": 22, "num_attention_heads": 12, "local_attention": 128, "global_attn_every_n_layers": 3,
        "global_rope_theta": 160000.0, "local_rope_theta": 10000.0, "norm_eps": 1e-5}
LARGE = {**BASE, "vocab_size": 256000, "hidden_size": 1024, "intermediate_size": 2624, "num_hidden_layers": 28,
         "num_attention_heads": 16}


def weight_names(cfg: dict) -> list[tuple[str, tuple]]:
    H, I, V, n = cfg["hidden_size"], cfg["intermediate_size"], cfg["vocab_size"], cfg["num_hidden_layers"]
    out = [("encoder.embeddings.tok_embeddings.weight", (V, H)), ("encoder.embeddings.norm.weight", (H,))]
    for i in range(n):
        p = f"encoder.layers.{i}."
        if i:
            out.append((p + "attn_norm.weight", (H,)))
        out += [(p + "attn.Wqkv.weight", (3 * H, H)), (p + "attn.Wo.weight", (H, H)), (p + "mlp_norm.weight", (H,)),
                (p + "mlp.Wi.weight", (2 * I, H)), (p + "mlp.Wo.weight", (H, I))]
    out.append(("encoder.final_norm.weight", (H,)))
    return out


def random_weights(cfg: dict, seed: int = 20261201, dtype=np.float16, norm_std: float = 0.0) -> dict:
    """N(0, 0.02) matrices; LayerNorm weights 1 (ModernBERT init) + N(0, norm_std)."""
    rng = np.random.default_rng(seed)
    W = {}
    for name, shape in weight_names(cfg):
        if len(shape) == 1:
            W[name] = (1.0 + norm_std * rng.standard_normal(shape)).astype(np.float32)
        else:
            W[name] = (rng.standard_normal(shape, dtype=np.float32) * 0.02).astype(dtype)
    return W


def classifier(cfg: dict, classes: int, seed: int = 7, dtype=np.float16):
    rng = np.random.default_rng(seed)
    H = cfg["hidden_size"]
    return (rng.standard_normal((classes, H), dtype=np.float32) * 0.02).astype(dtype), np.zeros(classes, np.float32)


def lengths(n: int, lo: int, hi: int, seed: int, dist: str = "uniform") -> np.ndarray:
    rng = np.random.default_rng(seed)
    if dist == "loguniform":
        return np.exp(rng.uniform(np.log(lo), np.log(hi + 1), size=n)).astype(np.int64).clip(lo, hi)
    return rng.integers(lo, hi + 1, size=n)


def token_batch(cfg: dict, lens: np.ndarray, seed: int):
    """Packed ids [T] (uniform in [5, vocab), CLS first, SEP last) and cu_seqlens [n + 1]."""
    rng = np.random.default_rng(seed)
    V = cfg["vocab_size"]
    cu = np.zeros(len(lens) + 1, np.int32)
    cu[1:] = np.cumsum(lens)
    ids = rng.integers(5, V, size=int(cu[-1])).astype(np.int32)
    cls, sep = (CLS_ID, SEP_ID) if V > SEP_ID else (1, 2)
    ids[cu[:-1]] = cls
    ids[cu[1:] - 1] = sep
    return ids, cu


def quantize_affine(w: np.ndarray, bits: int, group: int):
    """Affine group quantization (quant.ts:157-160 + assign rule :135-146):
    b = f16(min), s = f16((max − b)/(2^bits − 1)), q = clamp(⌊(w − b)/s + ½⌋)."""
    N, K = w.shape
    G = -(-K // group)
    lv = (1 << bits) - 1
    w64 = w.astype(np.float64)
    pad = G * group - K
    wp = np.pad(w64, ((0, 0), (0, pad)), mode="edge").reshape(N, G, group)
    lo, hi = wp.min(axis=2), wp.max(axis=2)
    b = lo.astype(np.float16)
    s = ((hi - b.astype(np.float64)) / lv).astype(np.float16)
    s64, b64 = s.astype(np.float64)[..., None], b.astype(np.float64)[..., None]
    ok = s64 > 0
    with np.errstate(divide="ignore", invalid="ignore"):
        q = np.where(ok, np.floor((wp - b64) / np.where(ok, s64, 1.0) + 0.5), 0.0)
    q = np.clip(q, 0, lv).astype(np.int64).reshape(N, G * group)[:, :K]
    return q, s, b


def quantized_host(w: np.ndarray, bits: int, group: int) -> HostQuantized:
    q, s, b = quantize_affine(w, bits, group)
    N, K = w.shape
    return HostQuantized((N, K), bits, group, "affine", pack_quantized(q, bits), HostTensor("f16", s.shape, s),
                         HostTensor("f16", b.shape, b))


def host_getter(W: dict, quant_bits: int = 0, group: int = 64):
    """WeightGetter over a dict of numpy arrays; Linear weights become HostQuantized when quant_bits != 0."""
    linear = (".attn.Wqkv.weight", ".attn.Wo.weight", ".mlp.Wi.weight", ".mlp.Wo.weight")
    cache = {}

    def get(name):
        if name not in W:
            return None
        if name in cache:
            return cache[name]
        a = W[name]
        if quant_bits and name.endswith(linear):
            h = quantized_host(a, quant_bits, group)
        else:
            dt = "f16" if a.dtype == np.float16 else "f32"
            h = HostTensor(dt, a.shape, a)
        cache[name] = h
        return h
    return get
