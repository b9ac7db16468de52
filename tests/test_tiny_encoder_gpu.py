"""The tiny laya checkpoint's encoder through the CUDA backend, stage by stage
against the MLX activations (packages/modernbert/test/modernbert.test.ts:65-117:
every stage within 1e-5 + 1e-5·|want| in f32)."""
from __future__ import annotations

import numpy as np
import pytest

from golden_io import decode, tiny
from gpu_util import backend
from laya_js_b200.host import HostTensor, to_f32
from laya_js_b200.modernbert import detectPrefix, loadModernBert, parseModernBertConfig

pytestmark = pytest.mark.gpu


def _getter(W):
    return lambda n: HostTensor("f32", W[n].shape, W[n]) if n in W else None


@pytest.mark.parametrize("dtype,tol", [("f32", 1e-5), ("f16", 2e-2), ("bf16", 8e-2)])
def test_tiny_encoder_every_stage(dtype, tol):
    enc_cfg, _, W, act = tiny()
    cfg = parseModernBertConfig(enc_cfg)
    b = backend()
    get = _getter(W)
    assert detectPrefix(get) == "encoder."
    enc = loadModernBert(b, cfg, get, dtype)
    ids = decode(act["inputs"]["input_ids"])
    mask = decode(act["inputs"]["attention_mask"])
    B, L = ids.shape
    stages = {}
    out = enc.forward(ids, mask.astype(np.uint8), B, L, onStage=lambda n, t: (stages.__setitem__(n, t), True)[1])
    assert stages["final_norm"] is out
    assert len(stages) == 2 + cfg["numHiddenLayers"]
    worst = 0.0
    for name, t in stages.items():
        want = decode(act["stages"][name if name == "embeddings" else "encoder." + name])
        got = to_f32(b.read(t))
        err = np.abs(got - want) - (tol + tol * np.abs(want))
        worst = max(worst, float(np.abs(got - want).max()))
        assert err.max() <= 0, f"{name}: max abs err {np.abs(got - want).max()}"
        b.dispose(t)
    enc.dispose()
    print(f"tiny encoder {dtype} max abs err {worst:.2e}")


def test_tiny_embed_mean_pool():
    enc_cfg, _, W, act = tiny()
    cfg = parseModernBertConfig(enc_cfg)
    b = backend()
    enc = loadModernBert(b, cfg, _getter(W), "f32")
    ids = decode(act["inputs"]["input_ids"])
    mask = decode(act["inputs"]["attention_mask"])
    B, L = ids.shape
    pooled = to_f32(b.read(enc.embed(ids, mask.astype(np.uint8), B, L)))
    fin = decode(act["stages"]["encoder.final_norm"])
    m = mask.astype(np.float64)[:, :, None]
    want = (fin * m).sum(1) / m.sum(1)
    assert np.max(np.abs(pooled - want)) <= 1e-5
    enc.dispose()
