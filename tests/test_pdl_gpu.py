"""Programmatic dependent launch of the contract's ops: every kernel launched
through the chain waits for its predecessor on the device before it touches
memory, and a GEMM reads an uploaded weight before that wait. Scheduling must
not change a single bit, so the contract ModernBERT forward (padded batch,
bool mask) and the DecisionModel forward, eager and through compiled(), run
in fresh processes with LAYA_CUDA_PDL=1 and =0 and must agree exactly."""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parent.parent

SCRIPT = r'''
import sys
import numpy as np
sys.path.insert(0, sys.argv[1])
from laya_js_b200 import createCudaBackend, workloads as WL
from laya_js_b200.decision import loadDecisionModel
from laya_js_b200.host import HostTensor, to_f32
from laya_js_b200.modernbert import loadModernBert, parseModernBertConfig
b = createCudaBackend(0)
cfg = {**WL.BASE, "num_hidden_layers": 3}
W = {k: v.astype(np.float32) for k, v in WL.random_weights(cfg, seed=11).items()}
get = lambda n: HostTensor("f32", W[n].shape, W[n]) if n in W else None
out = {}
enc = loadModernBert(b, parseModernBertConfig(cfg), get, "f16")
lens = np.array([97, 128, 5, 64])
B, L = len(lens), int(lens.max())
rng = np.random.default_rng(3)
ids = rng.integers(0, cfg["vocab_size"], size=(B, L)).astype(np.int32)
mask = (np.arange(L)[None, :] < lens[:, None]).astype(np.int32)
h = enc.forward(ids.reshape(-1), mask.reshape(-1), B, L)
out["encoder"] = to_f32(b.read(h))
H = {**W, **WL.decision_head_weights(cfg)}
get2 = lambda n: HostTensor("f32", H[n].shape, H[n]) if n in H else None
model = loadDecisionModel(b, dict(cfg), {"head_layers": 2, "act_costs": {"escalate": 0.5}}, get2, "f16")
batch = WL.decision_batch(cfg, [128, 40, 77])
eager = model.readOutputs(model.forwardTensors(batch))
run = model.compiled()
for _ in range(3):
    graph = model.readOutputs(run(batch))
for k, v in eager.items():
    if isinstance(v, np.ndarray):
        out["eager_" + k] = v
        out["graph_" + k] = graph[k]
np.savez(sys.argv[2], **out)
'''


def _run(pdl: str, tmp_path) -> dict:
    path = tmp_path / f"pdl{pdl}.npz"
    env = dict(os.environ, LAYA_CUDA_PDL=pdl)
    r = subprocess.run([sys.executable, "-c", SCRIPT, str(ROOT), str(path)], env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-3000:]
    z = np.load(path)
    return {k: z[k] for k in z.files}


def test_chained_launches_change_no_bit(tmp_path):
    on, off = _run("1", tmp_path), _run("0", tmp_path)
    assert set(on) == set(off) and "encoder" in on
    for k in on:
        assert on[k].shape == off[k].shape, k
        assert np.array_equal(on[k], off[k], equal_nan=True), f"{k}: LAYA_CUDA_PDL=1 and =0 differ by {np.abs(on[k] - off[k]).max()}"
    for k in on:
        if k.startswith("eager_"):
            assert np.array_equal(on[k], on["graph_" + k[6:]], equal_nan=True), f"compiled() differs from eager for {k[6:]}"
