"""configs[4] shape (ModernBERT-large / mmBERT: hidden 1024, 16 heads of 64,
GeGLU 2624, vocab 256000) in bf16 through the fused encoder, against the
oracle: a batch with long sequences from the configs[4] length range and a
batch of short prompts (the split-K GEMMs), 3 layers (one global, two
sliding-window), 16-way CLS head; plus the varlen attention alone at 4096
tokens (the range's upper end) in bf16."""
from __future__ import annotations

import numpy as np
import pytest

from gpu_util import backend
from laya_js_b200 import workloads as WL
from laya_js_b200.encoder import FusedEncoder, attention_varlen
from laya_js_b200.host import HostTensor, bf16_bits_to_f32, f32_to_bf16_bits, to_f32
from laya_js_b200.modernbert import loadModernBert, parseModernBertConfig
from oracle import models as M
from oracle import ops as O

pytestmark = pytest.mark.gpu

LARGE3 = {**WL.LARGE, "num_hidden_layers": 3}


def _bf16(a: np.ndarray) -> np.ndarray:
    """Round to bf16 (nearest even), widened back to f32."""
    return bf16_bits_to_f32(f32_to_bf16_bits(np.asarray(a, np.float32)))


@pytest.mark.parametrize("half_window", [-1, 64])
def test_attention_4096_tokens_bf16(half_window):
    b = backend()
    rng = np.random.default_rng(3)
    H, nh = 1024, 16
    lens = np.array([4096, 77])
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    T = int(cu[-1])
    qkv = _bf16(rng.standard_normal((T, 3 * H)))
    att = to_f32(b.read(attention_varlen(b, b.fromHost(HostTensor("bf16", qkv.shape, f32_to_bf16_bits(qkv))), cu, half_window, 0.125)))
    for s, L in enumerate(lens):
        seg = qkv[cu[s]:cu[s + 1]].reshape(L, 3, nh, 64)
        mask = None
        if half_window >= 0:
            i = np.arange(L)
            mask = (np.abs(i[:, None] - i[None, :]) <= half_window)[None, None]
        for h in (0, 7, 15):  # one head at a time keeps the f64 scores at L² values
            q, k, v = (seg[:, j, h][None, None] for j in range(3))
            want = O.sdpa(q, k, v, mask, 0.125)[0, 0]
            got = att[cu[s]:cu[s + 1], h * 64:(h + 1) * 64]
            err = np.abs(got - want).max()
            assert err < 1.5e-2, f"seq {s} (L={L}) head {h}: max err {err}"


def test_large_bf16_fused_encoder_matches_oracle():
    b = backend()
    W = WL.random_weights(LARGE3, seed=9, norm_std=0.05)
    cfg = parseModernBertConfig(LARGE3)
    enc = loadModernBert(b, cfg, WL.host_getter(W), "bf16")
    fused = FusedEncoder(enc)
    Wo = {k: _bf16(v.astype(np.float32)) for k, v in W.items()}  # the weights the device holds
    ocfg = M.parse_config(LARGE3)
    hw, hb = WL.classifier(LARGE3, 16, seed=4)
    hw = (hw.astype(np.float32) * 3).astype(np.float16)  # logits of O(1)
    thw, thb = b.fromHost(HostTensor("f16", hw.shape, hw)), b.fromHost(HostTensor("f32", hb.shape, hb))
    for j, lens in enumerate(([1536, 700, 300, 40, 16], [16, 33, 128])):
        ids, cu = WL.token_batch(LARGE3, np.array(lens), seed=20 + j)
        hid, probs = fused.forward(b.fromHost(HostTensor("i32", ids.shape, ids)), cu, thw, thb)
        hid = to_f32(b.read(hid))
        probs = to_f32(b.read(probs))
        ref = M.encoder_varlen(ocfg, Wo, [ids[cu[s]:cu[s + 1]] for s in range(len(lens))])
        err = np.abs(hid - np.concatenate(ref))
        # measured: max 6.4e-2, mean 3.6e-3 (bf16 storage of every activation, 3 layers)
        assert err.max() < 0.15 and err.mean() < 1e-2, f"batch {j}: hidden max err {err.max()}, mean {err.mean()}"
        _, probs_ref = M.classifier_head(np.stack([r[0] for r in ref]), hw.astype(np.float32), hb)
        assert np.abs(probs - probs_ref).max() < 1e-2, f"batch {j}: probs differ by {np.abs(probs - probs_ref).max()}"
        top2 = np.sort(probs_ref, 1)[:, -2:]
        clear = top2[:, 1] - top2[:, 0] > 4e-2  # argmax compared where the oracle's choice is not a near tie
        assert np.array_equal(probs.argmax(1)[clear], probs_ref.argmax(1)[clear])
    fused.free()
    enc.dispose()
