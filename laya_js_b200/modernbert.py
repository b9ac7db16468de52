"""ModernBERT / mmBERT encoder on any backend of the contract — the host-side
mirror of packages/modernbert/src/index.ts, so the reference's model code
runs unchanged (op for op) on the CUDA backend:

- ``parseModernBertConfig``   index.ts:58-110
- ``attentionMasks``          index.ts:240-259
- ``ModernBert``              index.ts:322-474 (embeddings :336-339, layer
                              :342-357, finalNorm :359-362, forward :394-401,
                              encode :407-429, embed :435-443)
- ``loadModernBert``          index.ts:498-529 / buildEncoderWeights :532-559

The fused varlen path for throughput (one C call per forward, no padding, no
host-built masks) is ``laya_js_b200.encoder.FusedEncoder``.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Callable, Optional

import numpy as np

from . import compose as Cm
from .host import HostQuantized, HostTensor, to_f32


def parseModernBertConfig(j: dict) -> dict:
    """index.ts:58-110 (defaults and validation)."""
    if j.get("model_type", "modernbert") != "modernbert":
        raise ValueError(f"Unsupported encoder: {j.get('model_type')!r}; expected modernbert")
    if j.get("hidden_activation", "gelu") != "gelu":
        raise ValueError(f"Unsupported encoder activation: {j.get('hidden_activation')!r}")
    H, nh, n = int(j["hidden_size"]), int(j["num_attention_heads"]), int(j["num_hidden_layers"])
    if nh <= 0 or H % nh or (H // nh) % 2:
        raise ValueError("ModernBERT requires an even, integral attention head dimension")
    every = int(j.get("global_attn_every_n_layers", 3))
    lt = j.get("layer_types")
    if lt is None:
        lt = ["full_attention" if i % every == 0 else "sliding_attention" for i in range(n)]
    if len(lt) != n or any(k not in ("full_attention", "sliding_attention") for k in lt):
        raise ValueError("Invalid ModernBERT layer_types")
    rp = j.get("rope_parameters") or {}
    for kind in set(lt):
        if (rp.get(kind) or {}).get("rope_type", "default") != "default":
            raise ValueError("Only default (unscaled) ModernBERT RoPE is supported")
    g = float(j.get("global_rope_theta", 160000))
    l = float(j.get("local_rope_theta", 10000))
    return {
        "modelType": "modernbert", "vocabSize": int(j["vocab_size"]), "hiddenSize": H,
        "intermediateSize": int(j["intermediate_size"]), "numHiddenLayers": n, "numAttentionHeads": nh,
        "headDim": H // nh, "normEps": float(j.get("norm_eps", 1e-5)), "normBias": bool(j.get("norm_bias", False)),
        "attentionBias": bool(j.get("attention_bias", False)), "mlpBias": bool(j.get("mlp_bias", False)),
        "localAttention": int(j.get("local_attention", 128)), "globalAttnEveryNLayers": every,
        "maxPositionEmbeddings": int(j.get("max_position_embeddings", 8192)), "layerTypes": list(lt),
        "ropeBase": {"full_attention": float((rp.get("full_attention") or {}).get("rope_theta", g)),
                     "sliding_attention": float((rp.get("sliding_attention") or {}).get("rope_theta", l))},
    }


def attentionMasks(attention_mask: np.ndarray, B: int, L: int, window: int):
    """index.ts:240-259: full [B,1,1,L] = valid[j]; sliding [B,1,L,L] =
    valid[j] ∧ (query i is padding ∨ |i − j| ≤ window // 2)."""
    m = np.asarray(attention_mask).reshape(B, L).astype(bool)
    half = window // 2
    full = m.astype(np.uint8).reshape(B, 1, 1, L)
    i = np.arange(L)
    near = np.abs(i[:, None] - i[None, :]) <= half
    # two in-place passes over the [B, L, L] result (no temporaries of that size)
    sliding = np.empty((B, L, L), bool)
    np.logical_or((~m)[:, :, None], near[None], out=sliding)
    np.logical_and(sliding, m[:, None, :], out=sliding)
    return HostTensor("bool", (B, 1, 1, L), full), HostTensor("bool", (B, 1, L, L), sliding.view(np.uint8).reshape(B, 1, L, L))


def is_host_quantized(h) -> bool:
    return isinstance(h, HostQuantized)


def uploadAs(b, h, dtype: str):
    """index.ts:175-188."""
    if is_host_quantized(h):
        return Cm.uploadQuantized(b, h, dtype)
    if h.dtype not in ("f32", "f16", "bf16"):
        return b.fromHost(h)
    src = h if (h.dtype == dtype or b.supports(h.dtype)) else HostTensor("f32", h.shape, to_f32(h))
    t = b.fromHost(src)
    if t.dtype == dtype:
        return t
    c = b.cast(t, dtype)
    b.dispose(t)
    return c


def disposeWeight(b, w) -> None:
    if w is None:
        return
    if Cm.is_quantized(w):
        Cm.disposeQuantized(b, w)
    else:
        b.dispose(w)


@dataclass
class LayerWeights:
    kind: str
    attnNorm: Optional[tuple]
    Wqkv: object
    WqkvBias: object
    Wo: object
    WoBias: object
    mlpNorm: tuple
    Wi: object
    WiBias: object
    WoMlp: object
    WoMlpBias: object


@dataclass
class ModernBertWeights:
    tokEmbeddings: object
    embNorm: tuple  # (weight, bias)
    layers: list
    finalNorm: tuple


class ModernBert:
    """index.ts:322-474."""

    def __init__(self, backend, config: dict, weights: ModernBertWeights, dtype: str):
        self.backend = backend
        self.config = config
        self.weights = weights
        self.dtype = dtype

    def embeddings(self, ids):
        b, w = self.backend, self.weights
        return b.scope(lambda: b.layerNorm(Cm.embeddingAny(b, w.tokEmbeddings, ids), w.embNorm[0], w.embNorm[1],
                                           self.config["normEps"]))

    def layer(self, i: int, x, mask):
        """index.ts:342-357."""
        b, c, w = self.backend, self.config, self.weights.layers[i]

        def f():
            B, L, H = x.shape
            nh, hd = c["numAttentionHeads"], c["headDim"]
            h = b.layerNorm(x, w.attnNorm[0], w.attnNorm[1], c["normEps"]) if w.attnNorm else x
            qkv = b.transpose(b.reshape(Cm.linearAny(b, h, w.Wqkv, w.WqkvBias), [B, L, 3, nh, hd]), [2, 0, 3, 1, 4])
            q, k, v = [b.reshape(t, [B, nh, L, hd]) for t in b.split(qkv, 3, 0)]
            base = c["ropeBase"][w.kind]
            att = b.sdpa(b.rope(q, base), b.rope(k, base), v, mask, hd ** -0.5)
            merged = b.reshape(b.transpose(att, [0, 2, 1, 3]), [B, L, H])
            x1 = b.add(x, Cm.linearAny(b, merged, w.Wo, w.WoBias))
            m = Cm.linearAny(b, b.layerNorm(x1, w.mlpNorm[0], w.mlpNorm[1], c["normEps"]), w.Wi, w.WiBias)
            return b.add(x1, Cm.linearAny(b, Cm.geglu(b, m), w.WoMlp, w.WoMlpBias))
        return b.scope(f)

    def finalNorm(self, x):
        b, w = self.backend, self.weights
        return b.scope(lambda: b.layerNorm(x, w.finalNorm[0], w.finalNorm[1], self.config["normEps"]))

    def uploadInputs(self, input_ids: np.ndarray, attention_mask: np.ndarray, B: int, L: int) -> dict:
        """index.ts:369-384."""
        b, c = self.backend, self.config
        if np.asarray(input_ids).size != B * L:
            raise ValueError(f"modernbert: inputIds has {np.asarray(input_ids).size} values, want {B * L}")
        full, sliding = attentionMasks(attention_mask, B, L, c["localAttention"])
        out = {"ids": b.fromHost(HostTensor("i32", (B, L), np.asarray(input_ids, np.int32).reshape(B, L))),
               "mask": b.fromHost(HostTensor("bool", (B, L), np.asarray(attention_mask, np.uint8).reshape(B, L))),
               "masks": {"full_attention": None, "sliding_attention": None}}
        if "full_attention" in c["layerTypes"]:
            out["masks"]["full_attention"] = b.fromHost(full)
        if "sliding_attention" in c["layerTypes"]:
            out["masks"]["sliding_attention"] = b.fromHost(sliding)
        return out

    def disposeInputs(self, inp: dict) -> None:
        b = self.backend
        for t in (inp["ids"], inp["mask"], inp["masks"]["full_attention"], inp["masks"]["sliding_attention"]):
            if t is not None:
                b.dispose(t)

    def forward(self, input_ids, attention_mask, B: int, L: int, onStage: Optional[Callable] = None):
        """index.ts:394-401."""
        inp = self.uploadInputs(input_ids, attention_mask, B, L)
        try:
            return self.encode(inp, onStage)
        finally:
            self.disposeInputs(inp)

    def encode(self, inp: dict, onStage: Optional[Callable] = None):
        """index.ts:407-429."""
        b, c = self.backend, self.config
        kept = []

        def emit(name, t, last):
            if onStage is not None and onStage(name, t) is True and not last:
                kept.append(t)

        def f():
            masks = inp["masks"]
            x = self.embeddings(inp["ids"])
            emit("embeddings", x, False)
            for i in range(c["numHiddenLayers"]):
                nxt = self.layer(i, x, masks[c["layerTypes"][i]])
                if not any(k is x for k in kept):
                    b.dispose(x)
                x = nxt
                emit(f"layers.{i}", x, False)
            y = self.finalNorm(x)
            if not any(k is x for k in kept):
                b.dispose(x)
            emit("final_norm", y, True)
            return [y, *kept]
        return b.scope(f)[0]

    def embed(self, input_ids, attention_mask, B: int, L: int):
        """index.ts:435-443."""
        b = self.backend
        inp = self.uploadInputs(input_ids, attention_mask, B, L)
        try:
            return b.scope(lambda: Cm.meanPool(b, self.encode(inp), inp["mask"]))
        finally:
            self.disposeInputs(inp)

    def dispose(self) -> None:
        b, w = self.backend, self.weights
        for t in (w.tokEmbeddings, *w.embNorm, *w.finalNorm):
            disposeWeight(b, t)
        for l in w.layers:
            for t in (*(l.attnNorm or ()), *l.mlpNorm, l.Wqkv, l.WqkvBias, l.Wo, l.WoBias, l.Wi, l.WiBias, l.WoMlp, l.WoMlpBias):
                disposeWeight(b, t)


def detectPrefix(get: Callable[[str], object]) -> str:
    for p in ("encoder.", "model.", ""):
        if get(f"{p}embeddings.tok_embeddings.weight") is not None:
            return p
    raise KeyError("modernbert: no embeddings.tok_embeddings.weight under prefixes encoder., model. or ''")


def loadModernBert(b, config: dict, get: Callable[[str], object], dtype: str = "f32", prefix: Optional[str] = None) -> ModernBert:
    """index.ts:498-559: validates names/shapes, uploads every weight (freeing
    what was uploaded when one fails)."""
    if not b.supports(dtype):
        raise ValueError(f"{b.name} backend does not support {dtype}")
    prefix = detectPrefix(get) if prefix is None else prefix
    H, I = config["hiddenSize"], config["intermediateSize"]
    made = []

    def need(name, shape, matrix=False):
        key = prefix + name
        h = get(key)
        if h is None:
            raise KeyError(f"modernbert: missing weight {key}")
        if tuple(h.shape) != tuple(shape):
            raise ValueError(f"modernbert: {key} has shape {list(h.shape)}, want {list(shape)}")
        if not matrix and is_host_quantized(h):
            raise ValueError(f"modernbert: {key} cannot be quantized (only Linear weights and the token embedding)")
        t = uploadAs(b, h, dtype)
        made.append(t)
        return t

    def maybe(on, name, shape):
        return need(name, shape) if on else None

    def norm(p):
        return (need(f"{p}.weight", [H]), maybe(config["normBias"], f"{p}.bias", [H]))

    try:
        tok = need("embeddings.tok_embeddings.weight", [config["vocabSize"], H], True)
        emb_norm = norm("embeddings.norm")
        layers = []
        for i in range(config["numHiddenLayers"]):
            p = f"layers.{i}"
            layers.append(LayerWeights(
                kind=config["layerTypes"][i],
                attnNorm=None if i == 0 else norm(f"{p}.attn_norm"),
                Wqkv=need(f"{p}.attn.Wqkv.weight", [3 * H, H], True),
                WqkvBias=maybe(config["attentionBias"], f"{p}.attn.Wqkv.bias", [3 * H]),
                Wo=need(f"{p}.attn.Wo.weight", [H, H], True),
                WoBias=maybe(config["attentionBias"], f"{p}.attn.Wo.bias", [H]),
                mlpNorm=norm(f"{p}.mlp_norm"),
                Wi=need(f"{p}.mlp.Wi.weight", [2 * I, H], True),
                WiBias=maybe(config["mlpBias"], f"{p}.mlp.Wi.bias", [2 * I]),
                WoMlp=need(f"{p}.mlp.Wo.weight", [H, I], True),
                WoMlpBias=maybe(config["mlpBias"], f"{p}.mlp.Wo.bias", [H]),
            ))
        fin = norm("final_norm")
    except BaseException:
        for t in made:
            disposeWeight(b, t)
        raise
    return ModernBert(b, config, ModernBertWeights(tok, emb_norm, layers, fin), dtype)
