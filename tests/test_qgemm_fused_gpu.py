"""The packed-weight GEMM (dequantisation inside the tcgen05 kernel, taken for
few rows) against dequantising into a dense matrix first: in a fresh process
each (LAYA_CUDA_QGEMM_FUSED is read once per process), the contract's
quantizedLinear on 4/8-bit, symmetric/affine weights with groups of 16..128,
ragged N, and the quantized fused encoder (folded LayerNorm weight applied in
the dequantisation, GeGLU row order) on short prompts. Both routes feed the MMA
the same 16-bit operand, so the outputs must be bit-identical; quantizedLinear
is also checked against an f64 product of the dequantised weight."""
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
from laya_js_b200.host import HostTensor, HostQuantized, pack_quantized, to_f32
from laya_js_b200.modernbert import loadModernBert, parseModernBertConfig
b = createCudaBackend(0)
out, worst = {}, 0.0
cases = [(16, 2304, 768, 4, 64, "affine"), (128, 768, 1152, 8, 64, "affine"), (100, 768, 768, 4, 32, "symmetric"),
         (77, 1000, 640, 8, 128, "affine"), (130, 2304, 768, 4, 64, "symmetric"), (40, 256, 64, 8, 16, "symmetric"),
         (9, 520, 832, 4, 64, "affine")]
for i, (M, N, K, bits, g, mode) in enumerate(cases):
    rng = np.random.default_rng(100 + i)
    w = (rng.standard_normal((N, K)) * 0.05).astype(np.float16)
    G = -(-K // g)
    if mode == "affine":
        q, s, bb = WL.quantize_affine(w, bits, g)
    else:
        lim = (1 << (bits - 1)) - 1
        s = (np.abs(w.astype(np.float64).reshape(N, G, g)).max(-1) / lim).astype(np.float16)
        s[s == 0] = 1
        q = np.clip(np.round(w.astype(np.float64) / np.repeat(s.astype(np.float64), g, 1)), -lim - 1, lim).astype(np.int64)
        bb = None
    hq = HostQuantized((N, K), bits, g, mode, pack_quantized(q, bits), HostTensor("f16", s.shape, s),
                       HostTensor("f16", bb.shape, bb) if bb is not None else None)
    tq = b.fromHostQuantized(hq, "f16")
    x = rng.standard_normal((M, K)).astype(np.float16)
    bias = (rng.standard_normal(N) * 0.1).astype(np.float16)
    y = to_f32(b.read(b.quantizedLinear(b.fromHost(HostTensor("f16", x.shape, x)), tq.w, tq.scales, tq.biases, tq,
                                        b.fromHost(HostTensor("f16", bias.shape, bias)))))
    wd = q.astype(np.float64) * np.repeat(s.astype(np.float64), g, 1)[:, :K]
    if bb is not None:
        wd = wd + np.repeat(bb.astype(np.float64), g, 1)[:, :K]
    wd = wd.astype(np.float16).astype(np.float64)  # the dequantised weight in the compute dtype
    ref = x.astype(np.float64) @ wd.T + bias.astype(np.float64)
    err = np.abs(y - ref) / (2 ** -8 * np.abs(ref) + 2e-3 * np.sqrt(K) * 0.05)
    worst = max(worst, float(err.max()))
    out[f"lin{i}"] = y
for bits in (4, 8):
    cfg = dict(WL.BASE); cfg["num_hidden_layers"] = 3
    W = WL.random_weights(cfg, seed=bits, norm_std=0.05)
    enc = loadModernBert(b, parseModernBertConfig(cfg), WL.host_getter(W, quant_bits=bits, group=64), "f16")
    fused = E.FusedEncoder(enc)
    for j, lens in enumerate(([128], [33, 95], [7], [300, 212])):
        ids, cu = WL.token_batch(cfg, np.array(lens), seed=7 + j)
        h, _ = fused.forward(b.fromHost(HostTensor("i32", ids.shape, ids)), cu)
        out[f"enc{bits}_{j}"] = to_f32(b.read(h))
    fused.free()
    enc.dispose()
np.savez(sys.argv[2], **out)
print(json.dumps({"err_over_tol": worst}))
'''


def _run(fused: str, tmp_path) -> tuple[float, str]:
    out = tmp_path / f"q_{fused}.npz"
    env = dict(os.environ, LAYA_CUDA_QGEMM_FUSED=fused)
    r = subprocess.run([sys.executable, "-c", SCRIPT, str(ROOT), str(out)], env=env, capture_output=True, text=True, timeout=900)
    assert r.returncode == 0, r.stderr[-2000:]
    return json.loads(r.stdout.strip().splitlines()[-1])["err_over_tol"], str(out)


def test_fused_dequant_gemm_bit_identical_to_dequant_first(tmp_path):
    import numpy as np
    e_fused, f_fused = _run("1", tmp_path)
    e_dense, f_dense = _run("0", tmp_path)
    assert e_fused <= 1.0, f"packed-weight GEMM: error {e_fused:.2f} x tolerance"
    assert e_dense <= 1.0, f"dequantise-first GEMM: error {e_dense:.2f} x tolerance"
    a, b = np.load(f_fused), np.load(f_dense)
    assert sorted(a.files) == sorted(b.files)
    for k in a.files:
        assert a[k].shape == b[k].shape, k
        d = np.abs(a[k] - b[k]).max()
        assert np.array_equal(a[k], b[k]), f"{k}: the two routes differ (max {d})"
