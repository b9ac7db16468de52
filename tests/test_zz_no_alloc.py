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
from laya_js_b200.host import HostTensor, to_f32

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


def _case(b, rng, M, N, K, bits):
    w = (rng.standard_normal((N, K), dtype=np.float32) * 0.02).astype(np.float16)
    q = b.fromHostQuantized(WL.quantized_host(w, bits, 64), "f16")
    x = b.fromHost(HostTensor("f16", (M, K), rng.standard_normal((M, K), dtype=np.float32).astype(np.float16)))
    bias = b.fromHost(HostTensor("f16", (N,), (rng.standard_normal(N, dtype=np.float32) * 0.1).astype(np.float16)))
    return q, x, bias


def _noalloc(b, y, x, q, bias, M, N, K, bits):
    _lib.call("lc_quantized_linear_noalloc", C.c_void_p(_dev(y)), C.c_void_p(_dev(x)), C.c_int64(M), C.c_int64(K), 1,
              C.c_void_p(_dev(q.w)), C.c_void_p(_dev(q.scales)), C.c_void_p(_dev(q.biases)), C.c_int64(N), bits, 64, 1, 1,
              C.c_void_p(_dev(bias)), 1, C.c_uint64(_stream()))


def test_noalloc_matches_quantized_linear_on_consecutive_calls():
    b = backend()
    rng = np.random.default_rng(20261201)
    # two calls in a row, the second with a smaller weight: the shared scratch
    # still holds the first call's values beyond the second's N·K
    for (M, N, K, bits) in [(300, 2304, 768, 4), (130, 768, 1152, 8)]:
        q, x, bias = _case(b, rng, M, N, K, bits)
        want = to_f32(b.read(b.quantizedLinear(x, q.w, q.scales, q.biases, q, bias)))
        y = b.fromHost(HostTensor("f16", (M, N), np.zeros((M, N), np.float16)))
        _noalloc(b, y, x, q, bias, M, N, K, bits)
        got = to_f32(b.read(y))
        tol = 1e-3 * max(1.0, float(np.abs(want).max()))
        assert np.max(np.abs(got - want)) <= tol, f"{M}x{N}x{K} q{bits}: max diff {np.max(np.abs(got - want))}"


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
