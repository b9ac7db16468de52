"""The tiny Laya DecisionModel through the CUDA backend, every stage against
the MLX activations (packages/laya/test/model.test.ts: all stages within
1e-5 in f32, including padded positions; masked logits exactly -1e4)."""
from __future__ import annotations

import numpy as np
import pytest

from golden_io import decode, tiny
from gpu_util import backend
from laya_js_b200.decision import loadDecisionModel
from laya_js_b200.host import HostTensor, to_f32

pytestmark = pytest.mark.gpu


def _batch(act):
    ins = {k: decode(v) for k, v in act["inputs"].items()}
    B, L = ins["input_ids"].shape
    M = ins["marker_pos"].shape[1]
    return {"size": B, "length": L, "markerCount": M, "inputIds": ins["input_ids"].reshape(-1),
            "attentionMask": ins["attention_mask"].astype(np.uint8).reshape(-1), "markerPos": ins["marker_pos"].reshape(-1),
            "markerMask": ins["marker_mask"].astype(np.uint8).reshape(-1), "qtype": ins["qtype"]}


@pytest.mark.parametrize("dtype,tol", [("f32", 1e-5), ("f16", 3e-2)])
def test_tiny_decision_model_every_stage(dtype, tol):
    enc_cfg, agent_cfg, W, act = tiny()
    b = backend()
    get = lambda n: HostTensor("f32", W[n].shape, W[n]) if n in W else None
    model = loadDecisionModel(b, enc_cfg, agent_cfg, get, dtype)
    stages = {}
    out = model.forward(_batch(act), onStage=lambda n, t: (stages.__setitem__(n, t), True)[1])
    got = {n: to_f32(b.read(t)) for n, t in stages.items()}
    for t in stages.values():
        b.dispose(t)
    got["logits"], got["act"] = out["logits"], out["act"]
    assert set(got) == set(act["stages"])
    for name, e in act["stages"].items():
        want = decode(e)
        err = np.abs(got[name] - want) - (tol + tol * np.abs(want))
        assert err.max() <= 0, f"{name} ({dtype}): max abs err {np.abs(got[name] - want).max()}"
    masked = decode(act["inputs"]["marker_mask"]) == 0
    assert np.all(out["logits"][masked] == np.float32(-1e4))
    model.dispose()


def test_decision_model_leak_free():
    enc_cfg, agent_cfg, W, act = tiny()
    b = backend()
    get = lambda n: HostTensor("f32", W[n].shape, W[n]) if n in W else None
    base = b.stats()["live_tensors"]
    model = loadDecisionModel(b, enc_cfg, agent_cfg, get, "f32")
    for _ in range(2):
        model.forward(_batch(act))
    model.dispose()
    assert b.stats()["live_tensors"] == base
