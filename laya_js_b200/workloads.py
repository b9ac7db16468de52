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


# ---------------------------------------------------------------- the benchmark configurations
#
# One seed family for every configuration, shared by bench.py and the parity
# tests, so the tests check exactly the inputs the bench times.

SEED = 20261201


def cfg2_prompts(n_prompts: int = 256):
    """n prompts with lengths uniform in [32, 512] (256 per GPU; a
    multi-GPU run draws one global batch of 256·N and shards it)."""
    lens = lengths(n_prompts, 32, 512, seed=SEED + 1)
    ids, cu = token_batch(BASE, lens, seed=SEED + 2)
    return lens, ids, cu


def cfg0_prompt():
    """batch 1, one 128-token prompt (CLS ... SEP)."""
    lens = np.array([128])
    ids, cu = token_batch(BASE, lens, seed=SEED + 5)
    return lens, ids, cu


def cfg3_prompts(n_prompts: int = 512):
    """n prompts with lengths uniform in [64, 1024]."""
    lens = lengths(n_prompts, 64, 1024, seed=SEED + 7)
    ids, cu = token_batch(BASE, lens, seed=SEED + 8)
    return lens, ids, cu


def cfg4_lengths(n_prompts: int = 65536) -> np.ndarray:
    """prompt lengths log-uniform in [16, 4096]."""
    return lengths(n_prompts, 16, 4096, seed=SEED + 9, dist="loguniform")


def cfg4_tokens(lens: np.ndarray):
    return token_batch(LARGE, lens, seed=SEED + 10)


def base_weights() -> dict:
    """ModernBERT-base fp16 weights N(0, 0.02), LayerNorm weights 1 (the bench's)."""
    return random_weights(BASE, seed=SEED)


def large_weights_bf16() -> dict:
    """ModernBERT-large / mmBERT-shape weights N(0, 0.02) rounded to bf16 (held
    as f32 values that bf16 represents exactly), LayerNorm weights 1."""
    from .host import bf16_bits_to_f32, f32_to_bf16_bits
    W = random_weights(LARGE, seed=SEED + 11, dtype=np.float32)
    return {k: (bf16_bits_to_f32(f32_to_bf16_bits(v)) if v.ndim == 2 else v) for k, v in W.items()}


def head(cfg: dict, classes: int):
    """The CLS classifier of a configuration: 3-way, 8-way
    (configs[2], [3]) or 16-way; N(0, 0.02) fp16, zero bias."""
    seeds = {3: SEED + 4, 8: SEED + 3, 16: SEED + 12}
    return classifier(cfg, classes, seed=seeds[classes])


def decision_head_weights(cfg: dict, seed: int = SEED + 20, head_layers: int = 2, n_act: int = 2) -> dict:
    """Random-init Laya DecisionModel head weights (laya-mlx names, the layout
    of packages/laya/src/model.ts:368-405) for an encoder of `cfg`'s width:
    two pre-norm head layers (4·D ReLU FFN), the marker scorer, the action
    head and the question-type embedding; N(0, 0.02) matrices, zero biases,
    LayerNorm weights 1 (f32)."""
    rng = np.random.default_rng(seed)
    D = cfg["hidden_size"]
    n = lambda *sh: (rng.standard_normal(sh, dtype=np.float32) * 0.02)
    z = lambda *sh: np.zeros(sh, np.float32)
    one = lambda *sh: np.ones(sh, np.float32)
    W = {"type_emb.weight": n(3, D)}
    for j in range(head_layers):
        p = f"head.layers.{j}."
        W.update({p + "norm1.weight": one(D), p + "norm1.bias": z(D), p + "norm2.weight": one(D), p + "norm2.bias": z(D),
                  p + "self_attn.in_proj.weight": n(3 * D, D), p + "self_attn.in_proj.bias": z(3 * D),
                  p + "self_attn.out_proj.weight": n(D, D), p + "self_attn.out_proj.bias": z(D),
                  p + "linear1.weight": n(4 * D, D), p + "linear1.bias": z(4 * D),
                  p + "linear2.weight": n(D, 4 * D), p + "linear2.bias": z(D)})
    W.update({"scorer.layers.0.weight": one(D), "scorer.layers.0.bias": z(D), "scorer.layers.1.weight": n(D, D),
              "scorer.layers.1.bias": z(D), "scorer.layers.3.weight": n(1, D), "scorer.layers.3.bias": z(1),
              "act_head.layers.0.weight": n(256, D + 4), "act_head.layers.0.bias": z(256),
              "act_head.layers.2.weight": n(n_act, 256), "act_head.layers.2.bias": z(n_act)})
    return W


def decision_batch(cfg: dict, lens, markers: int = 4, seed: int = SEED + 21) -> dict:
    """A collated DecisionModel batch (packages/laya/src/model.ts:146-170
    fields): prompts padded to the longest, `markers` marker positions per
    prompt inside it (the last slot masked off for odd rows), a question type
    per prompt."""
    rng = np.random.default_rng(seed)
    lens = np.asarray(lens, np.int64)
    B, L = len(lens), int(lens.max())
    ids, cu = token_batch(cfg, lens, seed=seed + 1)
    pad = np.zeros((B, L), np.int32)
    valid = np.zeros((B, L), np.uint8)
    pos = np.zeros((B, markers), np.int32)
    mm = np.ones((B, markers), np.uint8)
    for b in range(B):
        n = int(lens[b])
        pad[b, :n] = ids[cu[b]:cu[b + 1]]
        valid[b, :n] = 1
        pos[b] = np.sort(rng.choice(np.arange(1, max(n - 1, markers + 1)), size=markers, replace=False))
        pos[b] = np.minimum(pos[b], n - 1)
        if b % 2:
            mm[b, -1] = 0
    return {"size": B, "length": L, "markerCount": markers, "inputIds": pad.reshape(-1), "attentionMask": valid.reshape(-1),
            "markerPos": pos.reshape(-1), "markerMask": mm.reshape(-1), "qtype": rng.integers(0, 3, size=B).astype(np.int32)}
