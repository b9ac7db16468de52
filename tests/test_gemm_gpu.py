"""The tcgen05 GEMM behind `linear` (f16 / bf16) against an f64 reference:
every tile path (BN 128 / 256, the split-K clusters for few rows), M and N
tails, K not a multiple of 64; and the warp-per-output kernel that takes few
rows of a small product (M <= 16, M*N*K <= 2^23: the (1, 2304, 768),
(4, 768, 768) and (3, 2, 256) cases with 16-byte loads, (1, 256, 772) and
(2, 40, 68) with 8-byte loads)."""
from __future__ import annotations

import numpy as np
import pytest

from gpu_util import backend
from laya_js_b200.host import HostTensor, bf16_bits_to_f32, f32_to_bf16_bits, to_f32

pytestmark = pytest.mark.gpu

SHAPES = [(1, 40, 64), (127, 128, 64), (128, 256, 768), (300, 768, 768), (1000, 2304, 768), (4096, 768, 1152),
          (513, 5248, 1024), (77, 1024, 2624), (2048, 3072, 1024), (130, 24, 128), (64, 200, 200),
          (5, 44, 64), (300, 129, 128), (1, 2304, 768), (4, 768, 768), (3, 2, 256),
          (16, 2304, 768), (12, 768, 1152), (1, 256, 772), (2, 40, 68)]


def _mk(dtype, a):
    if dtype == "f16":
        return HostTensor("f16", a.shape, a.astype(np.float16))
    return HostTensor("bf16", a.shape, f32_to_bf16_bits(a))


def _vals(h):
    return to_f32(h).astype(np.float64)


@pytest.mark.parametrize("dtype", ["f16", "bf16"])
@pytest.mark.parametrize("M,N,K", SHAPES)
def test_linear_matches_f64(dtype, M, N, K):
    b = backend()
    rng = np.random.default_rng(M * 7 + N + K)
    x = rng.standard_normal((M, K)).astype(np.float32)
    w = (rng.standard_normal((N, K)) * 0.05).astype(np.float32)
    bias = rng.standard_normal(N).astype(np.float32)
    hx, hw, hb = _mk(dtype, x), _mk(dtype, w), _mk(dtype, bias)
    y = b.read(b.linear(b.fromHost(hx), b.fromHost(hw), b.fromHost(hb)))
    assert y.dtype == dtype and y.shape == (M, N)
    ref = _vals(hx) @ _vals(hw).T + _vals(hb)
    tol = (2 ** -8 if dtype == "f16" else 2 ** -5) * np.abs(ref) + 2e-3 * np.sqrt(K) * 0.05
    err = np.abs(_vals(y) - ref)
    assert np.all(err <= tol), f"max err {err.max()} at {np.unravel_index(err.argmax(), err.shape)}"


def test_linear_batched_leading_dims_and_repeat():
    b = backend()
    rng = np.random.default_rng(11)
    x = rng.standard_normal((3, 50, 768)).astype(np.float16)
    w = (rng.standard_normal((2304, 768)) * 0.02).astype(np.float16)
    tx, tw = b.fromHost(HostTensor("f16", x.shape, x)), b.fromHost(HostTensor("f16", w.shape, w))
    ys = [b.read(b.linear(tx, tw)).data for _ in range(3)]
    assert ys[0].shape == (3, 50, 2304)
    assert np.array_equal(ys[0], ys[1]) and np.array_equal(ys[1], ys[2])  # deterministic
    ref = x.astype(np.float64) @ w.astype(np.float64).T
    assert np.max(np.abs(ys[0] - ref)) < 2e-2
