"""numpy restatement of the ModernBERT encoder and the Laya DecisionModel
(test oracle only), composed from ``oracle.ops`` exactly as the reference
composes contract ops.

- ``attention_masks``: packages/modernbert/src/index.ts:240-259
- ``encoder_forward``: packages/modernbert/src/index.ts:336-429
  (embeddings :336-339, layer :342-357, finalNorm :359-362, encode :407-429)
- ``decision_forward``: packages/laya/src/model.ts:124-137 (headLayer) and
  :182-235 (forwardCore)
- ``encoder_varlen``: the same encoder on unpadded sequences, one at a time,
  which equals the padded forward on valid tokens because every mask keeps
  keys inside the sequence (index.ts:240-259).
"""
from __future__ import annotations

import numpy as np

from . import ops as O


def parse_config(j: dict) -> dict:
    """packages/modernbert/src/index.ts:58-110 parseModernBertConfig (defaults only)."""
    H, nh, n = j["hidden_size"], j["num_attention_heads"], j["num_hidden_layers"]
    every = j.get("global_attn_every_n_layers", 3)
    lt = j.get("layer_types") or ["full_attention" if i % every == 0 else "sliding_attention" for i in range(n)]
    return {
        "vocab": j["vocab_size"], "H": H, "I": j["intermediate_size"], "layers": n, "nh": nh,
        "hd": H // nh, "eps": j.get("norm_eps", 1e-5), "window": j.get("local_attention", 128),
        "layer_types": lt,
        "rope": {"full_attention": j.get("global_rope_theta", 160000.0),
                 "sliding_attention": j.get("local_rope_theta", 10000.0)},
    }


def attention_masks(valid: np.ndarray, window: int):
    """index.ts:240-259: full [B,1,1,L] = valid[j]; sliding [B,1,L,L] =
    valid[j] ∧ (query i is padding ∨ |i − j| ≤ window // 2)."""
    B, L = valid.shape
    v = valid.astype(bool)
    full = v[:, None, None, :]
    i = np.arange(L)[:, None]
    j = np.arange(L)[None, :]
    near = np.abs(i - j) <= window // 2
    pad_q = ~v[:, :, None]
    sliding = (v[:, None, :] & (pad_q | near[None]))[:, None]
    return full, sliding


def _w(W, name):
    return W[name]


def encoder_layer(cfg, W, i, x, mask, prefix="encoder."):
    """index.ts:342-357 ModernBert.layer."""
    B, L, H = x.shape
    nh, hd = cfg["nh"], cfg["hd"]
    p = f"{prefix}layers.{i}."
    h = O.layer_norm(x, W[p + "attn_norm.weight"], None, cfg["eps"]) if i > 0 else x
    qkv = O.linear(h, W[p + "attn.Wqkv.weight"]).reshape(B, L, 3, nh, hd).transpose(2, 0, 3, 1, 4)
    q, k, v = (np.ascontiguousarray(t) for t in qkv)
    base = cfg["rope"][cfg["layer_types"][i]]
    att = O.sdpa(O.rope(q, base), O.rope(k, base), v, mask, hd ** -0.5)
    merged = att.transpose(0, 2, 1, 3).reshape(B, L, H)
    x1 = O.add(x, O.linear(merged, W[p + "attn.Wo.weight"]))
    m = O.linear(O.layer_norm(x1, W[p + "mlp_norm.weight"], None, cfg["eps"]), W[p + "mlp.Wi.weight"])
    return O.add(x1, O.linear(O.geglu(m), W[p + "mlp.Wo.weight"]))


def encoder_forward(cfg, W, ids, valid, prefix="encoder.", stages=None):
    """index.ts:407-429 encode: → final-norm hidden states [B, L, H] (f32).
    ``stages`` (dict) receives every stage output when given."""
    full, sliding = attention_masks(valid, cfg["window"])
    masks = {"full_attention": full, "sliding_attention": sliding}
    x = O.layer_norm(O.embedding(W[prefix + "embeddings.tok_embeddings.weight"], ids),
                     W[prefix + "embeddings.norm.weight"], None, cfg["eps"])
    if stages is not None:
        stages["embeddings"] = x
    for i in range(cfg["layers"]):
        x = encoder_layer(cfg, W, i, x, masks[cfg["layer_types"][i]], prefix)
        if stages is not None:
            stages[f"layers.{i}"] = x
    y = O.layer_norm(x, W[prefix + "final_norm.weight"], None, cfg["eps"])
    if stages is not None:
        stages["final_norm"] = y
    return y


def encoder_varlen(cfg, W, ids_list, prefix="encoder."):
    """The encoder on each unpadded sequence separately: list of [L_i, H] f32."""
    out = []
    for ids in ids_list:
        L = len(ids)
        y = encoder_forward(cfg, W, np.asarray(ids, np.int32)[None], np.ones((1, L), bool), prefix)
        out.append(y[0])
    return out


def classifier_head(hidden_cls, Wc, bc=None):
    """softmax(linear(CLS row, Wc), −1) → (logits f32 [B, C], probs f32 [B, C]);
    the op pattern of packages/laya/src/model.ts:228 (`slice` of the CLS row)."""
    logits = O.linear(hidden_cls, Wc, bc)
    return logits, O.softmax(logits, -1)


HEAD_EPS = 1e-5


def head_layer(W, j, x, mask):
    """packages/laya/src/model.ts:124-137 headLayer (PyTorch pre-norm layer, ReLU FFN)."""
    B, L, D = x.shape
    nh = max(1, D // 64)
    hd = D // nh
    p = f"head.layers.{j}."
    h = O.layer_norm(x, W[p + "norm1.weight"], W[p + "norm1.bias"], HEAD_EPS)
    qkv = O.linear(h, W[p + "self_attn.in_proj.weight"], W[p + "self_attn.in_proj.bias"])
    qkv = qkv.reshape(B, L, 3, nh, hd).transpose(2, 0, 3, 1, 4)
    q, k, v = (np.ascontiguousarray(t) for t in qkv)
    att = O.sdpa(q, k, v, mask, hd ** -0.5).transpose(0, 2, 1, 3).reshape(B, L, D)
    x1 = O.add(x, O.linear(att, W[p + "self_attn.out_proj.weight"], W[p + "self_attn.out_proj.bias"]))
    f = O.linear(O.relu(O.linear(O.layer_norm(x1, W[p + "norm2.weight"], W[p + "norm2.bias"], HEAD_EPS),
                                  W[p + "linear1.weight"], W[p + "linear1.bias"])),
                 W[p + "linear2.weight"], W[p + "linear2.bias"])
    return O.add(x1, f)


def decision_forward(cfg, W, ids, valid, qtype, marker_pos, marker_mask, head_layers=2, stages=None):
    """packages/laya/src/model.ts:182-235 forwardCore → (logits [B, M], act [B, nAct])."""
    B, L = ids.shape
    M = marker_pos.shape[1]
    D = cfg["H"]
    enc_stages = {} if stages is not None else None
    enc = encoder_forward(cfg, W, ids, valid, "encoder.", enc_stages)
    if stages is not None:
        for k, v in enc_stages.items():
            stages[k if k == "embeddings" else "encoder." + k] = v
    h = O.add(enc, O.embedding(W["type_emb.weight"], qtype).reshape(B, 1, D))
    if stages is not None:
        stages["type_emb_added"] = h
    head_mask = valid.astype(bool)[:, None, None, :]
    for j in range(head_layers):
        h = head_layer(W, j, h, head_mask)
        if stages is not None:
            stages[f"head.layers.{j}"] = h
    pos = np.maximum(marker_pos, 0)
    markers = O.gather_rows(h, pos)
    s1 = O.linear(O.layer_norm(markers, W["scorer.layers.0.weight"], W["scorer.layers.0.bias"], HEAD_EPS),
                  W["scorer.layers.1.weight"], W["scorer.layers.1.bias"])
    scored = O.linear(O.gelu(s1), W["scorer.layers.3.weight"], W["scorer.layers.3.bias"])
    logits = O.where(marker_mask.astype(bool), scored.reshape(B, M).astype(np.float32), np.float32(-1e4))
    k = np.maximum(marker_mask.astype(np.int64).sum(axis=1), 2).astype(np.float32)
    p = O.softmax(logits, -1)
    plogp = O.mul(p, O.log(O.maximum(p, np.float32(1e-9))))
    entropy = O.div(O.scale(O.sum_(plogp, -1), -1), O.log(k))
    top = O.sort(p, -1)[:, M - 2:]
    top2, top1 = top[:, 0:1], top[:, 1:2]
    k_scaled = O.div(k.reshape(B, 1), np.float32(255))
    features = np.concatenate([top1, O.sub(top1, top2), entropy.reshape(B, 1), k_scaled], -1)
    cls = h[:, 0, :]
    pooled = np.concatenate([cls, features], -1).astype(np.float32)
    a1 = O.linear(pooled, W["act_head.layers.0.weight"], W["act_head.layers.0.bias"])
    act = O.linear(O.gelu(a1), W["act_head.layers.2.weight"], W["act_head.layers.2.bias"])
    return logits, act
