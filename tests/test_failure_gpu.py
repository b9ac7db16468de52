"""Failure handling without a GPU fault: a pipeline wait that runs out and an
allocation that fails both surface as errors on the host, and the backend
keeps working afterwards.

- Every mbarrier wait of the pipelined kernels is bounded; on timeout the
  kernel records an error word and returns (lc_sm100.cuh). The test shortens
  the limit to 1 ms and launches a kernel whose one wait nothing satisfies
  (lc_debug_stuck_wait), then checks that lc_flush reports the timeout, that
  the report clears, and that GEMMs still give correct results.
- Out of memory: a capped allocator (lc_debug_set_alloc_cap) makes a large
  upload fail with the out-of-memory error; a scope that fails midway frees
  what it made (packages/tensor-backend/src/index.ts:159-163), and
  allocation works again once the cap is lifted.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

from gpu_util import backend
from laya_js_b200 import _lib
from laya_js_b200._lib import LayaCudaError
from laya_js_b200.host import HostTensor

pytestmark = pytest.mark.gpu


def _linear_ok(b):
    rng = np.random.default_rng(0)
    x = rng.standard_normal((256, 768)).astype(np.float16)
    w = (rng.standard_normal((512, 768)) * 0.05).astype(np.float16)
    y = b.read(b.linear(b.fromHost(HostTensor("f16", x.shape, x)), b.fromHost(HostTensor("f16", w.shape, w)))).data
    ref = x.astype(np.float64) @ w.astype(np.float64).T
    assert np.abs(y - ref).max() < 2e-2


def test_bounded_wait_timeout_is_reported_and_device_stays_usable():
    b = backend()
    b.flush()
    _lib.call("lc_debug_set_wait_limit", C.c_uint64(1_000_000))  # 1 ms
    try:
        _lib.call("lc_debug_stuck_wait")
        with pytest.raises(LayaCudaError, match="timed out"):
            b.flush()
    finally:
        _lib.call("lc_debug_set_wait_limit", C.c_uint64(0))
    b.flush()  # the error word was cleared by the report
    _linear_ok(b)
    b.flush()


def test_capped_allocator_out_of_memory_then_recovers():
    b = backend()
    base = b.stats()
    _lib.call("lc_debug_set_alloc_cap", C.c_int64(base["live_bytes"] + (1 << 20)))
    try:
        big = np.zeros((64, 1 << 20), np.float16)  # 128 MB
        with pytest.raises(LayaCudaError, match="out of device memory"):
            b.fromHost(HostTensor("f16", big.shape, big))

        def scoped():
            small = b.fromHost(HostTensor("f32", (1024,), np.ones(1024, np.float32)))
            b.exp(small)
            b.fromHost(HostTensor("f16", big.shape, big))  # fails: the scope frees small and exp(small)
        with pytest.raises(LayaCudaError, match="out of device memory"):
            b.scope(scoped)
        assert b.stats()["live_tensors"] == base["live_tensors"]
        assert b.stats()["live_bytes"] == base["live_bytes"]
    finally:
        _lib.call("lc_debug_set_alloc_cap", C.c_int64(0))
    t = b.fromHost(HostTensor("f16", big.shape, big))
    b.dispose(t)
    _linear_ok(b)
