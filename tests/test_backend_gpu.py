"""Backend behaviour beyond the fixtures, after the reference's backend unit
tests (packages/backend-cpu/test/backend.test.ts:28-120,
packages/backend-mlx/test/backend.test.ts:20-281)."""
from __future__ import annotations

import numpy as np
import pytest

from gpu_util import backend
from laya_js_b200._lib import LayaCudaError
from laya_js_b200.host import HostTensor, host, to_f32

pytestmark = pytest.mark.gpu


def test_round_trips_every_dtype():
    b = backend()
    rng = np.random.default_rng(0)
    for dt, arr in [("f32", rng.standard_normal(7).astype(np.float32)), ("f16", rng.standard_normal(7).astype(np.float16)),
                    ("i32", np.arange(7, dtype=np.int32)), ("bool", np.array([0, 1, 1, 0, 1, 0, 1], np.uint8)),
                    ("u8", np.arange(7, dtype=np.uint8)), ("i64", np.arange(-3, 4, dtype=np.int64)),
                    ("u64", np.array([2**63 + 5, 1, 2, 3, 4, 5, 6], np.uint64)), ("f64", rng.standard_normal(7))]:
        t = b.fromHost(HostTensor(dt, (7,), arr))
        assert t.dtype == dt and t.shape == (7,)
        assert np.array_equal(b.read(t).data, arr)
        b.dispose(t)


def test_from_host_copies_at_call_time():
    b = backend()
    data = np.array([1, 2, 3], np.float32)
    t = b.fromHost(HostTensor("f32", (3,), data))
    data[:] = 9
    assert np.array_equal(b.read(t).data, [1, 2, 3])


def test_f16_stays_f16():
    b = backend()
    x = b.fromHost(host("f16", [2, 8], np.arange(16) / 8))
    y = b.add(b.gelu(x), x)
    assert y.dtype == "f16"


def test_nested_scopes_keep_returned_array_and_object():
    b = backend()
    x = b.fromHost(host("f32", [2], [1, 2]))
    box = {}

    def inner():
        box["tmp"] = b.exp(x)
        box["inner"] = b.add(box["tmp"], x)
        return {"y": box["inner"], "n": 3}

    def outer():
        kept = b.scope(inner)
        assert box["tmp"].disposed and not kept["y"].disposed
        return [b.mul(kept["y"], x)]

    out = b.scope(outer)
    assert box["inner"].disposed and not out[0].disposed and not x.disposed
    with pytest.raises(RuntimeError, match="boom"):
        b.scope(lambda: (b.exp(x), (_ for _ in ()).throw(RuntimeError("boom"))))
    b.dispose(x)
    b.dispose(x)
    with pytest.raises(LayaCudaError, match="after dispose"):
        b.exp(x)


def test_errors_become_exceptions():
    b = backend()
    x = b.fromHost(host("f32", [2, 3]))
    with pytest.raises(LayaCudaError, match="changes the size"):
        b.reshape(x, [4, 2])
    with pytest.raises(LayaCudaError, match="broadcast"):
        b.add(x, b.fromHost(host("f32", [4])))
    with pytest.raises(LayaCudaError, match="bool"):
        q = b.fromHost(host("f32", [1, 1, 2, 4]))
        b.sdpa(q, q, q, b.fromHost(host("f32", [1, 1, 2, 2])), 1.0)


def test_reshape_minus_one_and_views():
    b = backend()
    x = b.fromHost(host("f32", [2, 3, 4], np.arange(24)))
    assert b.reshape(x, [-1]).shape == (24,)
    t = b.transpose(x, [2, 0, 1])
    r = b.reshape(t, [4, 6])
    assert np.array_equal(b.read(r).data, np.arange(24).reshape(2, 3, 4).transpose(2, 0, 1).reshape(4, 6))
    parts = b.split(x, 2, 2)
    assert np.array_equal(b.read(b.reshape(parts[1], [6, 2])).data, np.arange(24).reshape(2, 3, 4)[:, :, 2:].reshape(6, 2))


def test_memory_flat_across_iterations():
    b = backend()
    x = b.fromHost(host("f32", [64, 64], np.ones(64 * 64)))
    base = b.stats()["live_tensors"]
    for _ in range(20):
        b.dispose(b.scope(lambda: b.softmax(b.add(b.gelu(x), x), -1)))
    assert b.stats()["live_tensors"] == base


def test_sdpa_bool_padding_mask_long_rows():
    """backend-webgpu/test/kernels.test.ts: sdpa L=100 with sliding + padding."""
    from oracle import models as M, ops as O
    b = backend()
    rng = np.random.default_rng(3)
    B, H, L, D = 2, 3, 100, 64
    q, k, v = (rng.standard_normal((B, H, L, D)).astype(np.float32) for _ in range(3))
    valid = np.ones((B, L), bool)
    valid[1, 70:] = False
    _, sliding = M.attention_masks(valid, 32)
    want = O.sdpa(q, k, v, sliding, 0.125)
    got = b.read(b.sdpa(*(b.fromHost(HostTensor("f32", a.shape, a)) for a in (q, k, v)),
                        b.fromHost(HostTensor("bool", sliding.shape, sliding.astype(np.uint8))), 0.125)).data
    assert np.max(np.abs(got - want)) < 1e-4


def test_sort_long_rows_and_nan_last():
    b = backend()
    rng = np.random.default_rng(4)
    x = rng.standard_normal((3, 3000)).astype(np.float32)
    x[0, 5] = np.nan
    got = b.read(b.sort(b.fromHost(HostTensor("f32", x.shape, x)), -1)).data
    assert np.array_equal(np.isnan(got), np.isnan(np.sort(x, -1)))
    ok = ~np.isnan(got)
    assert np.array_equal(got[ok], np.sort(x, -1)[ok])


def test_large_uploads_through_the_staging_buffers():
    """fromHost copies before it returns (index.ts:146-154) also for uploads
    that go through the pinned double buffer: ragged chunk counts, the caller
    overwriting its array right after the call, back-to-back uploads."""
    b = backend()
    rng = np.random.default_rng(5)
    for n in ((8 << 20) * 2 + 12345, (4 << 20), (8 << 20) * 5 - 7):
        a = rng.integers(0, 256, size=n, dtype=np.uint8)
        want = a.copy()
        t1 = b.fromHost(HostTensor("u8", (n,), a))
        a[:] = 0  # the caller reuses its buffer at once
        c = rng.integers(0, 256, size=n, dtype=np.uint8)
        t2 = b.fromHost(HostTensor("u8", (n,), c))
        assert np.array_equal(b.read(t1).data, want)
        assert np.array_equal(b.read(t2).data, c)
        b.dispose(t1)
        b.dispose(t2)
    x = rng.standard_normal((4096, 2048)).astype(np.float16)
    t = b.fromHost(HostTensor("f16", x.shape, x))
    assert np.array_equal(b.read(t).data, x)
    b.dispose(t)
