"""The laya quantized-checkpoint reader (laya_js_b200.checkpoint) on the host:
metadata rules (packages/laya/src/quant.ts:65-80), grouping of a matrix with
its .scales / .biases (quant.ts:375-403), the HostQuantized it hands out
(packages/laya/src/weights.ts:71-82) and the host dequantisation rule
(quant.ts:199-241) against the oracle's."""
from __future__ import annotations

import numpy as np
import pytest

import laya_ckpt
from laya_js_b200 import checkpoint as CK
from laya_js_b200 import workloads as WL
from oracle import ops as O


def test_quant_metadata_rules():
    assert CK.quant_metadata({}) is None and CK.quant_metadata(None) is None
    m = CK.quant_metadata({"laya_quant": "q4", "version": "1", "group_size": "64"})
    assert m["bits"] == 4 and m["groupSize"] == 64
    assert CK.quant_metadata({"laya_quant": "q8", "version": "1", "group_size": "row"})["groupSize"] is None
    with pytest.raises(ValueError, match="version"):
        CK.quant_metadata({"laya_quant": "q8", "version": "2"})
    with pytest.raises(ValueError, match="scheme"):
        CK.quant_metadata({"laya_quant": "q3", "version": "1"})
    with pytest.raises(ValueError, match="group_size"):
        CK.quant_metadata({"laya_quant": "q8", "version": "1", "group_size": "0"})


def _raw(**kw):
    return {k: CK.RawTensor(dt, a.shape, a) for k, (dt, a) in kw.items()}


def test_group_quantized_validates_companions():
    s = np.ones((4, 2), np.float16)
    q, plain = CK.group_quantized(_raw(**{"w": ("I8", np.zeros((4, 128), np.int8)), "w.scales": ("F16", s),
                                          "x": ("F32", np.zeros(3, np.float32))}))
    assert set(q) == {"w"} and q["w"].bits == 8 and q["w"].groupSize == 64 and set(plain) == {"x"}
    with pytest.raises(ValueError, match="q4 needs .biases"):
        CK.group_quantized(_raw(**{"w": ("U8", np.zeros((4, 64), np.uint8)), "w.scales": ("F16", s)}))
    with pytest.raises(ValueError, match="not a quantized dtype"):
        CK.group_quantized(_raw(**{"w": ("F16", np.zeros((4, 128), np.float16)), "w.scales": ("F16", s)}))
    with pytest.raises(ValueError, match="does not match"):
        CK.group_quantized(_raw(**{"w": ("I8", np.zeros((3, 128), np.int8)), "w.scales": ("F16", s)}))


@pytest.mark.parametrize("scheme", ["q8", "q4"])
def test_read_weights_hands_out_packed_matrices(tmp_path, scheme):
    cfg = {**WL.BASE, "num_hidden_layers": 1, "vocab_size": 512}
    W = WL.random_weights(cfg, seed=4)
    path = str(tmp_path / f"m.{scheme}.safetensors")
    deq = laya_ckpt.write(path, W, scheme)
    get = CK.read_weights(path, quantized="device")
    name = "encoder.layers.0.attn.Wqkv.weight"
    h = get(name)
    assert h.bits == (8 if scheme == "q8" else 4) and h.mode == ("symmetric" if scheme == "q8" else "affine")
    assert h.shape == W[name].shape and h.scales.dtype == "f16"
    # the contract's unpacking of the handed-out bytes + the oracle's dequantisation = the file's values
    qv = O.unpack_quantized(h.data, *h.shape, h.bits, h.mode)
    d = O.dequantize(qv, h.scales.data, None if h.biases is None else h.biases.data, h.groupSize, np.float16)
    assert np.array_equal(d.astype(np.float32), deq[name])
    assert get(name) is None  # consumed
    plain = get("encoder.final_norm.weight")
    assert plain.dtype == "f32" and np.array_equal(plain.data, W["encoder.final_norm.weight"])
    # host dequantisation (the "dequantize" load mode) gives the same bits
    get2 = CK.read_weights(path, quantized="dequantize")
    assert np.array_equal(get2(name).data.astype(np.float32), deq[name])
