"""The tcgen05 GEMM kernels — single CTA, CTA pair (cta_group::2) and the
small-M split-K clusters — each forced through LAYA_CUDA_GEMM_PAIR /
LAYA_CUDA_GEMM_SPLIT in a fresh process (the choice is read once per
process), against an f64 reference, plus the fused encoder's epilogues (RoPE,
GeGLU, residual + folded LayerNorm) compared between the kernels on a batch
of 1023 tokens and on single short prompts (the split-K shapes)."""
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
hs = [to_f32(b.read(h))]
for lens in ([128], [33, 95], [7]):
    ids, cu = WL.token_batch(cfg, np.array(lens), seed=7)
    h, _ = fused.forward(b.fromHost(HostTensor("i32", ids.shape, ids)), cu)
    hs.append(to_f32(b.read(h)))
np.savez(sys.argv[2], *hs)
print(json.dumps({"gemm_err_over_tol": worst}))
'''


def _run(pair: str, split: str, tmp_path) -> tuple[float, str]:
    out = tmp_path / f"hidden_{pair}{split}.npz"
    env = dict(os.environ, LAYA_CUDA_GEMM_PAIR=pair, LAYA_CUDA_GEMM_SPLIT=split)
    r = subprocess.run([sys.executable, "-c", SCRIPT, str(ROOT), str(out)], env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    return json.loads(r.stdout.strip().splitlines()[-1])["gemm_err_over_tol"], str(out)


def test_single_pair_and_split_kernels_agree(tmp_path):
    import numpy as np
    runs = {name: _run(pair, split, tmp_path) for name, pair, split in
            (("single-CTA", "0", "0"), ("CTA-pair", "1", "0"), ("split-K", "1", "1"))}
    for name, (err, _) in runs.items():
        assert err <= 1.0, f"{name} GEMM: error {err:.2f} x tolerance"
    ref = np.load(runs["single-CTA"][1])
    for name in ("CTA-pair", "split-K"):
        got = np.load(runs[name][1])
        for key in ref.files:
            a, b = ref[key], got[key]
            assert a.shape == b.shape
            d = float(np.abs(a - b).max())
            assert d < 2e-2, f"encoder hidden states ({key}) differ by {d} between single-CTA and {name}"
