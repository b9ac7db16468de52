"""Pins the CPU oracle to the reference's golden vectors (no GPU)."""
from __future__ import annotations

import numpy as np
import pytest

from golden_io import decode, load_cases, tiny
from oracle import models as M
from oracle import ops as O
from oracle_dispatch import close, run_case

CASES = load_cases()


def test_case_count():
    # 49 core + 95 numerics + 26 quantized (packages/tensor-backend/test/fixtures.test.ts)
    assert len(CASES) == 170


@pytest.mark.parametrize("c", CASES, ids=[c["name"] for c in CASES])
def test_oracle_matches_fixture(c):
    xs = [decode(e) for e in c["inputs"]]
    out = run_case(c, xs)
    outs = out if isinstance(out, list) else [out]
    assert len(outs) == len(c["outputs"])
    for got, e in zip(outs, c["outputs"]):
        want = decode(e)
        assert list(np.shape(got)) == list(want.shape)
        ok, msg = close(got, want, c["atol"], c["rtol"])
        assert ok, f"{c['name']}: {msg}"
        if e["dtype"] not in ("f32", "f16", "bf16"):
            assert O.dtype_name(np.asarray(got)) == e["dtype"], c["name"]


def test_attention_masks_reproduce_fixture_masks():
    """packages/modernbert/test/modernbert.test.ts:52-63: the sdpa fixtures' masks
    are attentionMasks(valid, window 16)."""
    by = {c["name"]: c for c in CASES}
    full = decode(by["sdpa/full_attention"]["inputs"][3])
    sliding = decode(by["sdpa/sliding_attention"]["inputs"][3])
    valid = full[:, 0, 0, :]
    f, s = M.attention_masks(valid, 16)
    assert np.array_equal(f, full)
    assert np.array_equal(s, sliding)


def test_tiny_decision_model_every_stage():
    """packages/laya/test/model.test.ts / modernbert.test.ts:65-117: every stage of
    the tiny checkpoint within 1e-5 (+1e-5 relative) of the MLX activations."""
    enc_cfg, agent_cfg, W, act = tiny()
    cfg = M.parse_config(enc_cfg)
    assert cfg["layer_types"] == act["layer_types"]
    ins = {k: decode(v) for k, v in act["inputs"].items()}
    stages = {}
    logits, a = M.decision_forward(cfg, W, ins["input_ids"], ins["attention_mask"], ins["qtype"],
                                   ins["marker_pos"], ins["marker_mask"], agent_cfg["head_layers"], stages)
    stages["logits"], stages["act"] = logits, a
    for name, e in act["stages"].items():
        want = decode(e)
        got = stages[name]
        err = np.abs(got - want) - (1e-5 + 1e-5 * np.abs(want))
        assert err.max() <= 0, f"{name}: max excess {err.max()}"


def test_quantize_dequantize_roundtrip_error_bound():
    rng = np.random.default_rng(0)
    w = (rng.standard_normal((16, 128)) * 0.02).astype(np.float16)
    q, s, b = O.quantize_affine(w, 4, 64)
    assert q.min() >= 0 and q.max() <= 15
    d = O.dequantize(q, s, b, 64)
    step = s.astype(np.float64).repeat(64, axis=1)
    assert np.all(np.abs(d - w.astype(np.float64)) <= 0.5 * step + 1e-3)
    packed = O.pack_quantized(q, 4)
    assert np.array_equal(O.unpack_quantized(packed, 16, 128, 4, "affine"), q)
