"""The fused varlen encoder (lc_encoder_*) and the varlen attention kernel
against the CPU oracle and against the contract path, on ModernBERT-base
shapes (H 768, 12 heads of 64, GeGLU 1152, window 128)."""
from __future__ import annotations

import numpy as np
import pytest

from gpu_util import backend
from laya_js_b200 import workloads as WL
from laya_js_b200.encoder import FusedEncoder, attention_varlen
from laya_js_b200.host import HostTensor, to_f32
from laya_js_b200.modernbert import loadModernBert, parseModernBertConfig
from oracle import models as M
from oracle import ops as O

pytestmark = pytest.mark.gpu

LENS = np.array([1, 17, 64, 65, 130, 200, 300])


def small_base(layers=3):
    return {**WL.BASE, "num_hidden_layers": layers}


@pytest.mark.parametrize("kernel", [0, 1])
@pytest.mark.parametrize("half_window", [-1, 64, 8])
def test_attention_varlen_matches_oracle(half_window, kernel):
    b = backend()
    rng = np.random.default_rng(5)
    H, nh = 256, 4
    lens = np.array([1, 3, 63, 64, 65, 127, 128, 129, 257, 300])
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    T = int(cu[-1])
    qkv = rng.standard_normal((T, 3 * H)).astype(np.float16)
    att = to_f32(b.read(attention_varlen(b, b.fromHost(HostTensor("f16", qkv.shape, qkv)), cu, half_window, 0.125, kernel)))
    for s, L in enumerate(lens):
        seg = qkv[cu[s]:cu[s + 1]].astype(np.float32).reshape(L, 3, nh, 64).transpose(1, 2, 0, 3)
        mask = None
        if half_window >= 0:
            i = np.arange(L)
            mask = (np.abs(i[:, None] - i[None, :]) <= half_window)[None, None]
        want = O.sdpa(seg[0][None], seg[1][None], seg[2][None], mask, 0.125)[0].transpose(1, 0, 2).reshape(L, H)
        err = np.abs(att[cu[s]:cu[s + 1]] - want).max()
        assert err < 6e-3, f"seq {s} (L={L}) max err {err}"


def _model(cfg_json, quant_bits=0, seed=3):
    b = backend()
    W = WL.random_weights(cfg_json, seed=seed, norm_std=0.05)
    cfg = parseModernBertConfig(cfg_json)
    enc = loadModernBert(b, cfg, WL.host_getter(W, quant_bits), "f16")
    return b, W, cfg, enc


def _oracle_weights(W, quant_bits):
    """The weights the device computes with, widened to f32 (dequantised values when quantized)."""
    out = {}
    for k, v in W.items():
        if quant_bits and k.endswith((".attn.Wqkv.weight", ".attn.Wo.weight", ".mlp.Wi.weight", ".mlp.Wo.weight")):
            q, s, bb = WL.quantize_affine(v, quant_bits, 64)
            out[k] = O.dequantize(q, s, bb, 64, np.float16).astype(np.float32)
        else:
            out[k] = v.astype(np.float32)
    return out


@pytest.mark.parametrize("quant_bits,tol", [(0, 2e-2), (4, 5e-2), (8, 2e-2)])
def test_fused_encoder_matches_oracle(quant_bits, tol):
    cfg_json = small_base(3)
    b, W, cfg, enc = _model(cfg_json, quant_bits)
    ids, cu = WL.token_batch(cfg_json, LENS, seed=11)
    hw, hb = WL.classifier(cfg_json, 8, seed=2)
    hw = (hw.astype(np.float32) * 3).astype(np.float16)  # logits of O(1): argmax meaningful, no underflow
    fused = FusedEncoder(enc)
    tid = b.fromHost(HostTensor("i32", ids.shape, ids))
    thw, thb = b.fromHost(HostTensor("f16", hw.shape, hw)), b.fromHost(HostTensor("f32", hb.shape, hb))
    hid, probs = fused.forward(tid, cu, thw, thb)
    hid = to_f32(b.read(hid))
    probs = to_f32(b.read(probs))
    Wo = _oracle_weights(W, quant_bits)
    ocfg = M.parse_config(cfg_json)
    ref = M.encoder_varlen(ocfg, Wo, [ids[cu[s]:cu[s + 1]] for s in range(len(LENS))])
    ref_h = np.concatenate(ref)
    err = np.abs(hid - ref_h).max()
    assert err < 10 * tol, f"hidden max err {err}"
    logits_ref, probs_ref = M.classifier_head(np.stack([r[0] for r in ref]), hw.astype(np.float32), hb)
    logits = np.log(probs)  # softmax is shift-invariant: compare log-probs
    lref = np.log(probs_ref)
    assert np.abs((logits - logits.mean(1, keepdims=True)) - (lref - lref.mean(1, keepdims=True))).max() < tol
    assert np.array_equal(probs.argmax(1), probs_ref.argmax(1))
    assert np.abs(probs - probs_ref).max() < (1e-3 if quant_bits == 0 else 5e-3)
    # the host entry point gives the same probabilities
    p2 = fused.forward_host(ids, cu, thw, thb)
    assert np.array_equal(p2, probs)
    fused.free()
    enc.dispose()


@pytest.mark.parametrize("inter", [576, 2624])
def test_fused_encoder_geglu_width_not_a_multiple_of_256(inter):
    """Wi's accumulator (2I columns of interleaved gate / up units) of 1152 and
    5248 (configs[4]'s intermediate size): 256-wide CTA-pair tiles whose last
    tile holds one 128-column unit pair and leaves its upper half empty. 1990
    tokens, so the projections take the ordinary tiles, not the few-row
    split-K clusters."""
    cfg_json = {**small_base(2), "intermediate_size": inter}
    b, W, cfg, enc = _model(cfg_json)
    lens = np.array([1, 17, 64, 65, 130, 200, 300, 513, 700])
    ids, cu = WL.token_batch(cfg_json, lens, seed=12)
    fused = FusedEncoder(enc)
    hid, _ = fused.forward(b.fromHost(HostTensor("i32", ids.shape, ids)), cu)
    hid = to_f32(b.read(hid))
    ref = np.concatenate(M.encoder_varlen(M.parse_config(cfg_json), _oracle_weights(W, 0),
                                          [ids[cu[s]:cu[s + 1]] for s in range(len(lens))]))
    err = float(np.abs(hid - ref).max())
    assert err < 0.2, f"I={inter}: hidden max err {err}"
    fused.free()
    enc.dispose()


def test_fused_matches_contract_path():
    """The fused varlen forward equals ModernBert.forward (padded, host masks) on valid tokens."""
    cfg_json = small_base(3)
    b, W, cfg, enc = _model(cfg_json)
    lens = np.array([5, 140, 77])
    ids, cu = WL.token_batch(cfg_json, lens, seed=4)
    B, L = len(lens), int(lens.max())
    pad_ids = np.zeros((B, L), np.int32)
    valid = np.zeros((B, L), np.uint8)
    for s in range(B):
        pad_ids[s, :lens[s]] = ids[cu[s]:cu[s + 1]]
        valid[s, :lens[s]] = 1
    padded = to_f32(b.read(enc.forward(pad_ids, valid, B, L)))
    fused = FusedEncoder(enc)
    hid, _ = fused.forward(b.fromHost(HostTensor("i32", ids.shape, ids)), cu)
    hid = to_f32(b.read(hid))
    for s in range(B):
        err = np.abs(hid[cu[s]:cu[s + 1]] - padded[s, :lens[s]]).max()
        assert err < 5e-2, f"seq {s}: {err}"
    fused.free()
    enc.dispose()


def test_fused_encoder_deterministic_and_leak_free():
    cfg_json = small_base(2)
    b, W, cfg, enc = _model(cfg_json)
    ids, cu = WL.token_batch(cfg_json, np.array([33, 500, 129]), seed=9)
    hw, hb = WL.classifier(cfg_json, 3)
    thw = b.fromHost(HostTensor("f16", hw.shape, hw))
    fused = FusedEncoder(enc)
    base = b.stats()["live_tensors"]
    outs = [fused.forward_host(ids, cu, thw) for _ in range(3)]
    assert all(np.array_equal(outs[0], o) for o in outs[1:])
    assert b.stats()["live_tensors"] == base
    fused.free()
    enc.dispose()


@pytest.mark.parametrize("quant_bits", [0, 4])
def test_encoder_graph_replays_forward_host(quant_bits):
    """A captured graph gives the eager forward_host's probabilities bit for bit,
    for new ids on every replay, with eager forwards of other shapes in between."""
    cfg_json = small_base(2)
    b, W, cfg, enc = _model(cfg_json, quant_bits)
    lens = np.array([33, 500, 1, 129, 64])
    ids, cu = WL.token_batch(cfg_json, lens, seed=9)
    hw, hb = WL.classifier(cfg_json, 5, seed=2)
    hw = (hw.astype(np.float32) * 3).astype(np.float16)
    thw, thb = b.fromHost(HostTensor("f16", hw.shape, hw)), b.fromHost(HostTensor("f32", hb.shape, hb))
    fused = FusedEncoder(enc)
    g = fused.graph(cu, thw, thb)
    other_ids, other_cu = WL.token_batch(cfg_json, np.array([700, 9]), seed=1)
    rng = np.random.default_rng(5)
    for it in range(3):
        cur = ids if it == 0 else rng.integers(0, cfg_json["vocab_size"], ids.shape, dtype=np.int32)
        want = fused.forward_host(cur, cu, thw, thb)
        got = g.run(cur)
        assert np.array_equal(got, want), f"replay {it}: max diff {np.abs(got - want).max()}"
        fused.forward_host(other_ids, other_cu, thw, thb)  # grows the eager workspace between replays
    with pytest.raises(ValueError):
        g.run(ids[:-1])
    g.free()
    # freeing the encoder frees the graphs captured on it
    g2 = fused.graph(cu, thw, thb)
    fused.free()
    g2.free()  # no-op after the encoder is gone
    enc.dispose()


@pytest.mark.parametrize("half_window", [-1, 64])
def test_attention_varlen_many_items_per_cta(half_window):
    """Enough (query tile, head) items that every persistent CTA of the
    tcgen05 kernel walks several of them: the Q double buffer, the K/V ring
    running across items and the O buffer of one item stored while the next
    item runs are all exercised, against the oracle for every sequence."""
    b = backend()
    rng = np.random.default_rng(11)
    H, nh = 768, 12
    lens = rng.integers(1, 700, size=96)
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    T = int(cu[-1])
    items = sum(-(-int(L) // 128) for L in lens) * nh
    assert items > 8 * 296  # several items per CTA at two CTAs per SM
    qkv = (rng.standard_normal((T, 3 * H)) * 0.5).astype(np.float16)
    att = to_f32(b.read(attention_varlen(b, b.fromHost(HostTensor("f16", qkv.shape, qkv)), cu, half_window, 0.125, 0)))
    worst = 0.0
    for s, L in enumerate(lens):
        L = int(L)
        seg = qkv[cu[s]:cu[s + 1]].astype(np.float32).reshape(L, 3, nh, 64).transpose(1, 2, 0, 3)
        mask = None
        if half_window >= 0:
            i = np.arange(L)
            mask = (np.abs(i[:, None] - i[None, :]) <= half_window)[None, None]
        want = O.sdpa(seg[0][None], seg[1][None], seg[2][None], mask, 0.125)[0].transpose(1, 0, 2).reshape(L, H)
        worst = max(worst, float(np.abs(att[cu[s]:cu[s + 1]] - want).max()))
    assert worst < 6e-3, f"max err {worst}"
