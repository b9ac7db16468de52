"""lc_quantized_linear_noalloc — the quantized linear for callers that cannot
allocate device memory (their device memory belongs to another framework's
allocator, or their hot path must not call cudaMalloc/cudaFree, which can
synchronise the device). It must give the same result as the allocating entry
point lc_quantized_linear, call after call, while the dequantised weight lives in
the library's fixed scratch array.

This file is collected last on purpose (tests/test_zz_*), so a run that stops
at the first failure has already run every other test; it also passes alone in a
fresh process.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

from gpu_util import backend
from laya_js_b200 import _lib
from laya_js_b200 import workloads as WL
from laya_js_b200._lib import LayaCudaError
from laya_js_b200.host import HostTensor, bf16_bits_to_f32, f32_to_bf16_bits, host, to_f32
from oracle import ops as O

pytestmark = pytest.mark.gpu


def _dev(t) -> int:
    d = C.c_uint64()
    _lib.call("lc_tensor_data", C.c_uint64(t.handle), C.byref(d))
    assert d.value, "expected a dense tensor"
    return d.value


def _stream() -> int:
    s = C.c_uint64()
    _lib.call("lc_get_stream", C.byref(s))
    return s.value


_CODE = {"f32": 0, "f16": 1, "bf16": 2}


def _host16(dtype, a):
    return host(dtype, a.shape, a)


def _case(b, rng, M, N, K, bits, dtype="f16", sb="f16"):
    """A packed affine g64 weight with scales/biases stored in `sb` and x, bias in `dtype`."""
    w = (rng.standard_normal((N, K), dtype=np.float32) * 0.02).astype(np.float16)
    q = b.fromHostQuantized(WL.quantized_host(w, bits, 64), sb)
    x = b.fromHost(_host16(dtype, rng.standard_normal((M, K), dtype=np.float32)))
    bias = b.fromHost(_host16(dtype, rng.standard_normal(N, dtype=np.float32) * 0.1))
    return q, x, bias


def _noalloc(b, y, x, q, bias, M, N, K, bits, dtype="f16", sb="f16"):
    _lib.call("lc_quantized_linear_noalloc", C.c_void_p(_dev(y)), C.c_void_p(_dev(x)), C.c_int64(M), C.c_int64(K), _CODE[dtype],
              C.c_void_p(_dev(q.w)), C.c_void_p(_dev(q.scales)), C.c_void_p(_dev(q.biases)), C.c_int64(N), bits, 64, 1, _CODE[sb],
              C.c_void_p(_dev(bias)), _CODE[dtype], C.c_uint64(_stream()))


def _oracle(b, x, q, bias, N, K, bits, dtype):
    """f64 product of the operands as stored on the device: the packed bytes
    unpacked, each weight dequantised and rounded once to x's dtype (the rule
    both entry points follow), then x · wᵀ + bias."""
    raw = b.read(q.w).data.reshape(-1).view(np.uint8)
    qv = O.unpack_quantized(raw, N, K, bits, "affine")
    s = to_f32(b.read(q.scales)).astype(np.float64)
    bb = to_f32(b.read(q.biases)).astype(np.float64)
    wd = O.dequantize(qv, s, bb, 64, np.float64)
    wd = wd.astype(np.float16) if dtype == "f16" else bf16_bits_to_f32(f32_to_bf16_bits(wd.astype(np.float32)))
    return to_f32(b.read(x)).astype(np.float64) @ wd.astype(np.float64).T + to_f32(b.read(bias)).astype(np.float64)


def test_noalloc_matches_quantized_linear_on_consecutive_calls():
    """Consecutive calls through the scratch path: each call must launch the
    dequantisation into the scratch array and the GEMM (two launches, nothing
    allocated), and agree with lc_quantized_linear and with an f64 product.
    The second call has a smaller weight, so the scratch still holds the first
    call's values beyond its N·K; the bf16 and f32-scale calls cover the other
    operand types."""
    b = backend()
    rng = np.random.default_rng(20261201)
    # enough rows that the in-GEMM dequantisation declines (its tiles would
    # cover more than a quarter of the SMs), so the scratch is used
    cases = [(2048, 2304, 768, 4, "f16", "f16"), (2048, 768, 1152, 8, "f16", "f16"),
             (1024, 1152, 768, 4, "bf16", "bf16"), (2048, 768, 768, 8, "f16", "f32")]
    for (M, N, K, bits, dtype, sb) in cases:
        q, x, bias = _case(b, rng, M, N, K, bits, dtype, sb)
        want = to_f32(b.read(b.quantizedLinear(x, q.w, q.scales, q.biases, q, bias)))
        y = b.fromHost(host(dtype, (M, N)))
        before = b.stats()
        _noalloc(b, y, x, q, bias, M, N, K, bits, dtype, sb)
        after = b.stats()
        assert after["launches"] - before["launches"] == 2, f"{M}x{N}x{K}: expected dequantise + GEMM launches"
        assert after["live_bytes"] == before["live_bytes"] and after["live_tensors"] == before["live_tensors"]
        got = to_f32(b.read(y))
        tol = 1e-3 * max(1.0, float(np.abs(want).max()))
        assert np.max(np.abs(got - want)) <= tol, f"{M}x{N}x{K} q{bits} {dtype}/{sb}: max diff {np.max(np.abs(got - want))}"
        ref = _oracle(b, x, q, bias, N, K, bits, dtype)
        rtol, atol = (2 ** -9, 1e-3) if dtype == "f16" else (2 ** -7, 4e-3)
        err = np.abs(got - ref)
        assert np.all(err <= rtol * np.abs(ref) + atol), f"{M}x{N}x{K} q{bits} {dtype}/{sb}: vs f64 max err {err.max()}"


def test_noalloc_large_weight_few_rows_needs_no_scratch_many_rows_rejected():
    b = backend()
    rng = np.random.default_rng(1)
    N, K = 4608, 1024  # 4608 * 1024 f16 values = 9 MiB > the 8 MiB scratch
    # few rows: the weight is dequantised inside the GEMM, no scratch involved
    M = 4
    q, x, bias = _case(b, rng, M, N, K, 4)
    y = b.fromHost(HostTensor("f16", (M, N), np.zeros((M, N), np.float16)))
    _noalloc(b, y, x, q, bias, M, N, K, 4)
    # (the allocating entry runs four rows as a GEMV: same values, another summation order)
    want = to_f32(b.read(b.quantizedLinear(x, q.w, q.scales, q.biases, q, bias)))
    assert np.abs(to_f32(b.read(y)) - want).max() < 1e-2
    # many rows: dequantise-first, and the dense weight does not fit the scratch
    M = 4096
    x = b.fromHost(HostTensor("f16", (M, K), rng.standard_normal((M, K), dtype=np.float32).astype(np.float16)))
    y = b.fromHost(HostTensor("f16", (M, N), np.zeros((M, N), np.float16)))
    with pytest.raises(LayaCudaError, match="scratch"):
        _noalloc(b, y, x, q, bias, M, N, K, 4)
