"""Both tcgen05 GEMM kernels — single CTA and CTA pair (cta_group::2) — on the
shapes that select 256-wide tiles, each forced through LAYA_CUDA_GEMM_PAIR in a
fresh process (the choice is read once per process), against an f64 reference,
plus the fused encoder's epilogues (RoPE, GeGLU, residual + folded LayerNorm)
compared between the two kernels."""
from __future__ import annotations

import json
import os
import subprocess
import sys
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parent.parent

SCRIPT = r'''
import json, sys
import numpy as np
sys.path.insert(0, sys.argv[1])
from laya_js_b200 import createCudaBackend, encoder as E, workloads as WL
from laya_js_b200.host import HostTensor, to_f32
from laya_js_b200.modernbert import loadModernBert, parseModernBertConfig
b = createCudaBackend(0)
worst = 0.0
for (M, N, K) in [(1, 2304, 768), (300, 768, 768), (1000, 2304, 768), (4096, 768, 1152), (513, 5248, 1024), (77, 1024, 2624)]:
    rng = np.random.default_rng(M + N + K)
    x = rng.standard_normal((M, K)).astype(np.float16)
    w = (rng.standard_normal((N, K)) * 0.05).astype(np.float16)
    bias = rng.standard_normal(N).astype(np.float16)
    y = to_f32(b.read(b.linear(b.fromHost(HostTensor("f16", x.shape, x)), b.fromHost(HostTensor("f16", w.shape, w)),
                               b.fromHost(HostTensor("f16", bias.shape, bias))))).astype(np.float64)
    ref = x.astype(np.float64) @ w.astype(np.float64).T + bias.astype(np.float64)
    err = np.abs(y - ref) / (2 ** -8 * np.abs(ref) + 2e-3 * np.sqrt(K) * 0.05)
    worst = max(worst, float(err.max()))
cfg = dict(WL.BASE); cfg["num_hidden_layers"] = 2
W = WL.random_weights(cfg, seed=5, norm_std=0.05)
enc = loadModernBert(b, parseModernBertConfig(cfg), WL.host_getter(W), "f16")
fused = E.FusedEncoder(enc)
ids, cu = WL.token_batch(cfg, np.array([300, 17, 513, 129, 64]), seed=6)
h, _ = fused.forward(b.fromHost(HostTensor("i32", ids.shape, ids)), cu)
np.save(sys.argv[2], to_f32(b.read(h)))
print(json.dumps({"gemm_err_over_tol": worst}))
'''


def _run(mode: str, tmp_path) -> tuple[float, str]:
    out = tmp_path / f"hidden_{mode}.npy"
    env = dict(os.environ, LAYA_CUDA_GEMM_PAIR=mode)
    r = subprocess.run([sys.executable, "-c", SCRIPT, str(ROOT), str(out)], env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    return json.loads(r.stdout.strip().splitlines()[-1])["gemm_err_over_tol"], str(out)


def test_single_and_pair_kernels_agree(tmp_path):
    import numpy as np
    e1, h1 = _run("0", tmp_path)
    e2, h2 = _run("1", tmp_path)
    assert e1 <= 1.0, f"single-CTA GEMM: error {e1:.2f} x tolerance"
    assert e2 <= 1.0, f"CTA-pair GEMM: error {e2:.2f} x tolerance"
    a, b = np.load(h1), np.load(h2)
    assert a.shape == b.shape
    assert np.abs(a - b).max() < 2e-2, f"encoder hidden states differ by {np.abs(a - b).max()} between the kernels"
