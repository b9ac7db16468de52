"""The row fast paths (softmax, layerNorm, sum / mean / max / min over the
last axis, meanPool) against float64 numpy, across the widths that select
them (a multiple of the 16-byte vector: one warp per row up to 32 lanes x 12
vectors for softmax / layerNorm and x 24 for the reductions, one 256-thread
block per row up to 256 x 8 vectors) and the widths that fall back to the
generic kernels, in f32 / f16 / bf16; NaN propagation of max / min; meanPool
with masked-out and fully masked rows."""
from __future__ import annotations

import numpy as np
import pytest

from gpu_util import backend
from laya_js_b200.host import HostTensor, f32_to_bf16_bits, to_f32

pytestmark = pytest.mark.gpu

WIDTHS = {"f32": [4, 256, 1024, 1028, 770, 1152, 1536, 1540, 2048, 2304, 3072, 3076, 8192, 8196],
          "f16": [8, 768, 1152, 2048, 2056, 770, 2304, 3072, 3080, 4096, 6144, 6152, 16384, 16392],
          "bf16": [8, 512, 2048, 2056, 770, 1152, 3072, 4096, 16384]}
EPS = {"f32": 1e-5, "f16": 2e-3, "bf16": 1.6e-2}


def _host(dt, a):
    if dt == "f32":
        return HostTensor("f32", a.shape, a.astype(np.float32))
    if dt == "f16":
        return HostTensor("f16", a.shape, a.astype(np.float16))
    return HostTensor("bf16", a.shape, f32_to_bf16_bits(a.astype(np.float32)))


@pytest.mark.parametrize("dt", ["f32", "f16", "bf16"])
def test_softmax_and_reductions_over_rows(dt):
    b = backend()
    rng = np.random.default_rng(7)
    for n in WIDTHS[dt]:
        a = (rng.standard_normal((37, n)) * 3).astype(np.float32)
        h = _host(dt, a)
        x = to_f32(h).astype(np.float64)  # the values the device sees
        t = b.fromHost(h)
        sm = to_f32(b.read(b.softmax(t, -1))).astype(np.float64)
        e = np.exp(x - x.max(-1, keepdims=True))
        ref = e / e.sum(-1, keepdims=True)
        assert np.abs(sm - ref).max() <= EPS[dt], f"softmax n={n}"
        for name, fn, want, tol in [("sum", b.sum, x.sum(-1), EPS[dt] * np.sqrt(n) * 8 + EPS[dt] * np.abs(x).sum(-1)),
                                    ("mean", b.mean, x.mean(-1), 1e-6 + 1e-6 * np.abs(x).mean(-1)),
                                    ("max", b.max, x.max(-1), 0.0), ("min", b.min, x.min(-1), 0.0)]:
            got = to_f32(b.read(fn(t, -1))).astype(np.float64)
            assert np.all(np.abs(got - want) <= tol + (EPS[dt] * np.abs(want) if name == "sum" else 0)), f"{name} n={n}"
        b.dispose(t)


@pytest.mark.parametrize("n", [768, 2304])
def test_max_min_propagate_nan(n):
    b = backend()
    a = (np.arange(2 * n, dtype=np.float32).reshape(2, n) % 1000)
    a[1, 500] = np.nan
    t = b.fromHost(HostTensor("f16", a.shape, a.astype(np.float16)))
    mx, mn = to_f32(b.read(b.max(t, -1))), to_f32(b.read(b.min(t, -1)))
    assert not np.isnan(mx[0]) and np.isnan(mx[1]) and np.isnan(mn[1])


@pytest.mark.parametrize("dt", ["f32", "f16", "bf16"])
def test_layer_norm_over_rows(dt):
    b = backend()
    rng = np.random.default_rng(9)
    for n in WIDTHS[dt]:
        a = (rng.standard_normal((23, n)) * 2 + 0.5).astype(np.float32)
        h = _host(dt, a)
        x = to_f32(h).astype(np.float64)
        w = (1 + 0.1 * rng.standard_normal(n)).astype(np.float32)
        bias = (0.1 * rng.standard_normal(n)).astype(np.float32)
        got = to_f32(b.read(b.layerNorm(b.fromHost(h), b.fromHost(HostTensor("f32", (n,), w)),
                                        b.fromHost(HostTensor("f32", (n,), bias)), 1e-5))).astype(np.float64)
        mu = x.mean(-1, keepdims=True)
        ref = (x - mu) / np.sqrt(((x - mu) ** 2).mean(-1, keepdims=True) + 1e-5) * w + bias
        tol = {"f32": 2e-5, "f16": 8e-3, "bf16": 6e-2}[dt]
        assert np.abs(got - ref).max() <= tol, f"layerNorm n={n}"


@pytest.mark.parametrize("dt", ["f32", "f16", "bf16"])
@pytest.mark.parametrize("L", [77, 600])
def test_mean_pool_masks(dt, L):
    """meanPool over one slice of 256 positions (the block writes the mean)
    and over three (slice sums added in order by a second kernel)."""
    b = backend()
    rng = np.random.default_rng(3)
    B, D = 5, 768
    a = rng.standard_normal((B, L, D)).astype(np.float32)
    h = _host(dt, a)
    x = to_f32(h).astype(np.float64)
    mask = (rng.random((B, L)) < 0.6).astype(np.int32)
    mask[2] = 0  # a fully masked row pools to zeros
    got = to_f32(b.read(b.meanPool(b.fromHost(h), b.fromHost(HostTensor("i32", mask.shape, mask))))).astype(np.float64)
    cnt = np.maximum(mask.sum(1, keepdims=True), 1)
    ref = (x * mask[:, :, None]).sum(1) / cnt
    assert got.shape == (B, D)
    assert np.abs(got - ref).max() < 1e-5
    assert np.all(got[2] == 0)


@pytest.mark.parametrize("dt", ["f32", "f16", "bf16"])
@pytest.mark.parametrize("D", [64, 48, 40, 6])
def test_rope_paths_against_f64(dt, D):
    """rope (index.ts:225-229) on every kernel: 8 pairs per thread with 16-byte
    loads (16-bit, half % 8 == 0), 4 pairs (half % 4 == 0), the generic one;
    dense rows, the strided q/k views ModernBert.layer makes (reshape ->
    transpose -> split of the QKV projection), and a batch of one (whose
    size-1 axis carries an arbitrary stride)."""
    from oracle import ops as O
    b = backend()
    rng = np.random.default_rng(D)
    B, H, L = 2, 3, 37
    x = rng.standard_normal((B, H, L, D)).astype(np.float32)
    hx = _host(dt, x)
    ref = O.rope(to_f32(hx), 10000.0)
    got = to_f32(b.read(b.rope(b.fromHost(hx), 10000.0)))
    tol = {"f32": 1e-5, "f16": 2e-3, "bf16": 1.6e-2}[dt] * (1 + np.abs(ref))
    assert np.all(np.abs(got - ref) <= tol)
    for Bv in (B, 1):
        qkv = rng.standard_normal((Bv, L, 3, H, D)).astype(np.float32)
        hq = _host(dt, qkv)
        t = b.transpose(b.fromHost(hq), [2, 0, 3, 1, 4])
        q, k, _ = [b.reshape(s, [Bv, H, L, D]) for s in b.split(t, 3, 0)]
        vals = to_f32(hq).transpose(2, 0, 3, 1, 4)
        for view, i in ((q, 0), (k, 1)):
            ref = O.rope(vals[i], 10000.0)
            got = to_f32(b.read(b.rope(view, 10000.0)))
            assert np.all(np.abs(got - ref) <= {"f32": 1e-5, "f16": 2e-3, "bf16": 1.6e-2}[dt] * (1 + np.abs(ref)))
