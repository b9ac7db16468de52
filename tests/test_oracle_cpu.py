"""Pins the C++ CPU restatement (oracle/cpu_encoder.cpp: the timed CPU
baseline) to the reference's golden vectors and to the numpy oracle (no GPU):
the fixture cases of every op the encoder uses, the tiny checkpoint's encoder
output (MLX activations, 1e-5), and a ModernBERT-base forward bit for bit
against oracle/models.py."""
from __future__ import annotations

import numpy as np
import pytest

from golden_io import decode, load_cases, tiny
from oracle import cpu
from oracle import models as M
from oracle_dispatch import close

OPS = ("linear", "layerNorm", "rope", "sdpa", "geglu")
CASES = [c for c in load_cases() if c["op"] in OPS]


@pytest.fixture(scope="module", autouse=True)
def _built():
    cpu.build()


def test_cases_present():
    assert {c["op"] for c in CASES} == set(OPS)


@pytest.mark.parametrize("c", CASES, ids=[c["name"] for c in CASES])
def test_cpp_op_matches_fixture(c):
    xs = [decode(e) for e in c["inputs"]]
    a = c["args"]
    op = c["op"]
    if op == "linear":
        got = cpu.linear(xs[0], xs[1], xs[2], threads=2)
    elif op == "layerNorm":
        got = cpu.layer_norm(xs[0], xs[1], xs[2], a["eps"])
    elif op == "rope":
        got = cpu.rope(xs[0], a["base"])
    elif op == "sdpa":
        got = cpu.sdpa(xs[0], xs[1], xs[2], xs[3], a["scale"])
    else:
        got = cpu.geglu(xs[0])
    want = decode(c["outputs"][0])
    assert list(got.shape) == list(want.shape)
    ok, msg = close(got, want, c["atol"], c["rtol"])
    assert ok, f"{c['name']}: {msg}"


def test_cpp_encoder_matches_tiny_activations():
    """The tiny checkpoint's encoder (packages/laya/test/model.test.ts pins
    every stage at 1e-5): final-norm states on the valid tokens of each row."""
    enc_cfg, _, W, act = tiny()
    ins = {k: decode(v) for k, v in act["inputs"].items()}
    want = decode(act["stages"]["encoder.final_norm"])
    ids, valid = ins["input_ids"], ins["attention_mask"].astype(bool)
    seqs = [ids[b][valid[b]] for b in range(ids.shape[0])]
    enc = cpu.Encoder(enc_cfg, W)
    hid, _, cu = enc.forward(seqs, threads=2)
    for b in range(len(seqs)):
        w = want[b][valid[b]]
        err = np.abs(hid[cu[b]:cu[b + 1]] - w) - (1e-5 + 1e-5 * np.abs(w))
        assert err.max() <= 0, f"row {b}: max abs err {np.abs(hid[cu[b]:cu[b + 1]] - w).max()}"


def test_cpp_encoder_equals_numpy_oracle_base_shape():
    from laya_js_b200 import workloads as WL
    cfg = {**WL.BASE, "num_hidden_layers": 4}
    W = WL.random_weights(cfg, seed=3, norm_std=0.05)
    Wf = {k: v.astype(np.float32) for k, v in W.items()}
    lens = np.array([1, 70, 140])
    ids, cu = WL.token_batch(cfg, lens, seed=5)
    seqs = [ids[cu[s]:cu[s + 1]] for s in range(len(lens))]
    hw, hb = WL.classifier(cfg, 8, seed=2)
    enc = cpu.Encoder(cfg, W)
    hid, probs, _ = enc.forward(seqs, hw, hb, threads=4)
    ref = M.encoder_varlen(M.parse_config(cfg), Wf, seqs)
    assert np.abs(hid - np.concatenate(ref)).max() <= 1e-6
    _, pref = M.classifier_head(np.stack([r[0] for r in ref]), hw.astype(np.float32), hb)
    assert np.abs(probs - pref).max() <= 1e-6
    # one thread gives the same bits as four
    hid1, probs1, _ = enc.forward(seqs, hw, hb, threads=1)
    assert np.array_equal(hid1, hid) and np.array_equal(probs1, probs)
