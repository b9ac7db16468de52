"""A laya quantized checkpoint (format version 1: q8 symmetric I8 / q4 affine
U8 matrices with F16 .scales / .biases, docs/QUANTIZATION.md:91-117) read by
laya_js_b200.checkpoint (packages/laya/src/quant.ts:375-403,
packages/laya/src/weights.ts:71-175) and loaded with loadModernBert: every
Linear weight stays packed on the device (fromHostQuantized, the file's bytes
as the native layout), its device dequantisation equals the file's values bit
for bit, and the fused and contract-path forwards match the oracle run on
those values."""
from __future__ import annotations

import numpy as np
import pytest

import laya_ckpt
from gpu_util import backend
from laya_js_b200 import checkpoint as CK
from laya_js_b200 import compose as Cm
from laya_js_b200 import workloads as WL
from laya_js_b200.encoder import FusedEncoder
from laya_js_b200.host import HostTensor, to_f32
from laya_js_b200.modernbert import loadModernBert, parseModernBertConfig
from oracle import models as M

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("scheme", ["q8", "q4"])
def test_quantized_checkpoint_onto_device(tmp_path, scheme):
    b = backend()
    cfg = {**WL.BASE, "num_hidden_layers": 2}
    W = WL.random_weights(cfg, seed=6, norm_std=0.05)
    path = str(tmp_path / f"enc.{scheme}.safetensors")
    deq = laya_ckpt.write(path, W, scheme)
    # a consuming getter (each tensor handed out once): the prefix is given, as laya does
    enc = loadModernBert(b, parseModernBertConfig(cfg), CK.read_weights(path, quantized="device"), "f16", prefix="encoder.")
    for i, L in enumerate(enc.weights.layers):
        for attr, suffix in (("Wqkv", "attn.Wqkv.weight"), ("Wo", "attn.Wo.weight"), ("Wi", "mlp.Wi.weight"), ("WoMlp", "mlp.Wo.weight")):
            m = getattr(L, attr)
            assert Cm.is_quantized(m) and m.native and m.bits == (8 if scheme == "q8" else 4)
            N = m.shape[0]
            ids = b.fromHost(HostTensor("i32", (N,), np.arange(N, dtype=np.int32)))
            got = to_f32(b.read(b.quantizedEmbedding(m.w, m.scales, m.biases, m, ids)))
            assert np.array_equal(got, deq[f"encoder.layers.{i}.{suffix}"]), f"layer {i} {attr}: dequantisation differs"
    Wo = {k: (deq[k] if k in deq else v.astype(np.float32)) for k, v in W.items()}
    lens = np.array([40, 200, 129])
    ids, cu = WL.token_batch(cfg, lens, seed=8)
    ref = M.encoder_varlen(M.parse_config(cfg), Wo, [ids[cu[s]:cu[s + 1]] for s in range(len(lens))])
    fused = FusedEncoder(enc)
    hid, _ = fused.forward(b.fromHost(HostTensor("i32", ids.shape, ids)), cu)
    err = np.abs(to_f32(b.read(hid)) - np.concatenate(ref)).max()
    assert err < 5e-2, f"fused: max err {err}"
    fused.free()
    B, Lm = len(lens), int(lens.max())
    pad = np.zeros((B, Lm), np.int32)
    valid = np.zeros((B, Lm), np.uint8)
    for s in range(B):
        pad[s, :lens[s]] = ids[cu[s]:cu[s + 1]]
        valid[s, :lens[s]] = 1
    padded = to_f32(b.read(enc.forward(pad, valid, B, Lm)))
    for s in range(B):
        e = np.abs(padded[s, :lens[s]] - ref[s]).max()
        assert e < 5e-2, f"contract path, prompt {s}: max err {e}"
    enc.dispose()
