"""Backend.compile as CUDA-graph capture per input signature
(packages/tensor-backend/src/index.ts:244-245) and DecisionModel.compiled()
(packages/laya/src/model.ts:250-272) through it, after the reference's own
compile test (packages/backend-mlx/test/backend.test.ts:124-149): results
equal eager, tensor / list / dict outputs, one recording per shape, a
raising fn leaves the backend healthy; replays are bit-identical to eager on
new inputs of the same signature and allocate nothing that outlives a call."""
from __future__ import annotations

import numpy as np
import pytest

from golden_io import decode, tiny
from gpu_util import backend
from laya_js_b200 import workloads as WL
from laya_js_b200.decision import loadDecisionModel
from laya_js_b200.host import HostTensor, to_f32

pytestmark = pytest.mark.gpu


def _f32(b, shape, vals):
    return b.fromHost(HostTensor("f32", tuple(shape), np.asarray(vals, np.float32).reshape(shape)))


def test_compile_matches_eager_outputs_and_records_per_shape():
    b = backend()
    calls = {"n": 0}

    def fn(x, y):
        calls["n"] += 1
        return {"s": b.add(b.gelu(x), y), "p": b.mul(x, y)}
    cf = b.compile(fn)
    x, y = _f32(b, [3], [-1, 0, 2]), _f32(b, [3], [1, 2, 3])
    eager = fn(x, y)
    r = cf(x, y)  # first call of this signature: eager, then recorded
    assert np.array_equal(b.read(r["s"]).data, b.read(eager["s"]).data)
    assert list(b.read(r["p"]).data) == [-1, 0, 6]
    n = calls["n"]
    r2 = cf(x, y)  # replay: fn is not called again
    assert calls["n"] == n
    assert np.array_equal(b.read(r2["s"]).data, b.read(eager["s"]).data)
    x2, y2 = _f32(b, [3], [0.5, -3, 7]), _f32(b, [3], [2, 2, 2])
    r3 = cf(x2, y2)  # new values, same signature
    assert calls["n"] == n
    assert np.array_equal(b.read(r3["s"]).data, b.read(fn(x2, y2)["s"]).data)
    cf(_f32(b, [2], [1, 1]), _f32(b, [2], [1, 1]))
    assert calls["n"] == n + 3, "a new shape records again (eager call + capture)"
    arr = b.compile(lambda a: [b.exp(a), a])
    arr(x)
    out = arr(x)
    assert len(out) == 2 and list(b.read(out[1]).data) == [-1, 0, 2]


def test_compile_error_inside_fn_leaves_backend_healthy():
    b = backend()
    x, y = _f32(b, [3], [-1, 0, 2]), _f32(b, [3], [1, 2, 3])

    def bad(a):
        raise RuntimeError("inside trace")
    with pytest.raises(RuntimeError, match="inside trace"):
        b.compile(bad)(x)
    state = {"first": True}

    def fails_when_recorded(a):
        if state["first"]:
            state["first"] = False
            return b.exp(a)
        raise RuntimeError("during capture")
    with pytest.raises(RuntimeError, match="during capture"):
        b.compile(fails_when_recorded)(x)
    assert list(b.read(b.add(x, y)).data) == [0, 2, 5]


def _tiny_batch(act):
    ins = {k: decode(v) for k, v in act["inputs"].items()}
    B, L = ins["input_ids"].shape
    return {"size": B, "length": L, "markerCount": ins["marker_pos"].shape[1], "inputIds": ins["input_ids"].reshape(-1),
            "attentionMask": ins["attention_mask"].astype(np.uint8).reshape(-1), "markerPos": ins["marker_pos"].reshape(-1),
            "markerMask": ins["marker_mask"].astype(np.uint8).reshape(-1), "qtype": ins["qtype"]}


@pytest.mark.parametrize("dtype", ["f32", "f16"])
def test_decision_model_compiled_equals_eager(dtype):
    enc_cfg, agent_cfg, W, act = tiny()
    b = backend()
    get = lambda n: HostTensor("f32", W[n].shape, W[n]) if n in W else None
    model = loadDecisionModel(b, enc_cfg, agent_cfg, get, dtype)
    run = model.compiled()
    assert run is not None
    batch = _tiny_batch(act)
    rng = np.random.default_rng(1)
    other = dict(batch, inputIds=rng.integers(0, enc_cfg["vocab_size"], batch["inputIds"].shape).astype(np.int32))
    base = b.stats()["live_tensors"]
    for it, bt in enumerate([batch, batch, other, batch]):
        want = model.readOutputs(model.forwardTensors(bt))
        got = model.readOutputs(run(bt))
        assert np.array_equal(got["logits"], want["logits"]), f"call {it}: logits differ"
        assert np.array_equal(got["act"], want["act"]), f"call {it}: act differ"
        if it >= 2:
            assert b.stats()["live_tensors"] == live, "replays leak tensors"
        live = b.stats()["live_tensors"]
    # a second shape records a second graph
    short = dict(batch, length=20, inputIds=batch["inputIds"].reshape(3, 40)[:, :20].reshape(-1),
                 attentionMask=batch["attentionMask"].reshape(3, 40)[:, :20].reshape(-1),
                 markerPos=np.minimum(batch["markerPos"], 19))
    for _ in range(2):
        want = model.readOutputs(model.forwardTensors(short))
        got = model.readOutputs(run(short))
        assert np.array_equal(got["logits"], want["logits"]) and np.array_equal(got["act"], want["act"])
    # the tiny checkpoint's MLX activations hold through the graph too
    np.testing.assert_allclose(got["logits"].shape, (3, 3))
    out = model.readOutputs(run(batch))
    tol = 1e-5 if dtype == "f32" else 3e-2
    want_logits = decode(act["stages"]["logits"])
    assert np.max(np.abs(out["logits"] - want_logits) - (tol + tol * np.abs(want_logits))) <= 0
    del run
    model.dispose()
    assert b.stats()["live_tensors"] <= base


def test_decision_model_base_shape_compiled_equals_eager():
    """ModernBERT-base encoder (22 layers, fp16) + the Laya head at the
    predict latency shape (one 128-token prompt, four markers)."""
    b = backend()
    W = {**{k: v.astype(np.float32) for k, v in WL.base_weights().items()}, **WL.decision_head_weights(WL.BASE)}
    enc_cfg = dict(WL.BASE)
    get = lambda n: HostTensor("f32", W[n].shape, W[n]) if n in W else None
    model = loadDecisionModel(b, enc_cfg, {"head_layers": 2, "act_costs": {"escalate": 0.5}}, get, "f16")
    run = model.compiled()
    batch = WL.decision_batch(WL.BASE, [128])
    for _ in range(3):
        want = model.readOutputs(model.forwardTensors(batch))
        got = model.readOutputs(run(batch))
        assert np.array_equal(got["logits"], want["logits"]) and np.array_equal(got["act"], want["act"])
    del run
    model.dispose()


def test_recorded_rope_survives_a_longer_sequence():
    """A recording keeps the cos/sin table it was captured with: a later eager
    rope over more positions (a larger table for the same head dim and base)
    must not free it under the graph."""
    b = backend()
    base = 12345.0  # a base no other test uses: the table starts at this test's length
    rng = np.random.default_rng(4)
    x = rng.standard_normal((1, 2, 40, 64)).astype(np.float32)
    cf = b.compile(lambda t: b.rope(t, base))
    tx = _f32(b, x.shape, x)
    want = b.read(b.rope(tx, base)).data.copy()
    cf(tx)
    assert np.array_equal(b.read(cf(tx)).data, want)
    long = rng.standard_normal((1, 1, 3000, 64)).astype(np.float32)
    b.read(b.rope(_f32(b, long.shape, long), base))  # grows the table past 40 positions
    assert np.array_equal(b.read(cf(tx)).data, want)
