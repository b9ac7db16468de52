"""The contract's sdpa (index.ts:230-237) on its tensor-core path — f16/bf16,
head dim 64: the tcgen05 attention kernel (lc_attention_tc.cu, batched mode
with the bool mask read per key block) — against the oracle: no mask, the attentionMasks padding
[B,1,1,L] and sliding [B,1,L,L] masks (packages/modernbert/src/index.ts:240-259),
an arbitrary [B,H,Lq,Lk] mask, Lq != Lk, lengths off the 64-row tiles, and q/k/v
as the strided views ModernBert.layer makes (reshape -> transpose -> split of the
QKV projection) rather than dense tensors."""
from __future__ import annotations

import numpy as np
import pytest

from gpu_util import backend
from laya_js_b200.host import HostTensor, bf16_bits_to_f32, f32_to_bf16_bits, to_f32
from oracle import models as M
from oracle import ops as O

pytestmark = pytest.mark.gpu

TOL = {"f16": 4e-3, "bf16": 3e-2}


def _up(b, a, dt):
    a = np.asarray(a, np.float32)
    if dt == "f16":
        return b.fromHost(HostTensor("f16", a.shape, a.astype(np.float16))), a.astype(np.float16).astype(np.float32)
    r = bf16_bits_to_f32(f32_to_bf16_bits(a))
    return b.fromHost(HostTensor("bf16", a.shape, f32_to_bf16_bits(a))), r


@pytest.mark.parametrize("dt", ["f16", "bf16"])
@pytest.mark.parametrize("mask_kind", ["none", "padding", "sliding", "random"])
def test_sdpa_tensor_core_path(dt, mask_kind):
    b = backend()
    rng = np.random.default_rng(11)
    B, H, L = 3, 4, 130
    q, qr = _up(b, rng.standard_normal((B, H, L, 64)), dt)
    k, kr = _up(b, rng.standard_normal((B, H, L, 64)), dt)
    v, vr = _up(b, rng.standard_normal((B, H, L, 64)), dt)
    valid = np.ones((B, L), bool)
    valid[1, 77:] = False
    valid[2, 5:] = False
    mask = None
    if mask_kind == "padding":
        mask = M.attention_masks(valid, 128)[0]
    elif mask_kind == "sliding":
        mask = M.attention_masks(valid, 128)[1]
    elif mask_kind == "random":
        mask = rng.random((B, H, L, L)) < 0.7
        mask[..., 0] = True  # no fully masked row (undefined in the contract)
    tm = b.fromHost(HostTensor("bool", mask.shape, mask.astype(np.uint8))) if mask is not None else None
    got = to_f32(b.read(b.sdpa(q, k, v, tm, 0.125)))
    want = O.sdpa(qr, kr, vr, mask, 0.125)
    err = np.abs(got - want).max()
    assert err < TOL[dt], f"{dt} {mask_kind}: max err {err}"


@pytest.mark.parametrize("dt", ["f16", "bf16"])
def test_sdpa_strided_views_and_unequal_lengths(dt):
    b = backend()
    rng = np.random.default_rng(12)
    B, L, nh = 2, 300, 3
    # the QKV projection as ModernBert.layer views it: [B, L, 3, nh, 64] -> [3, B, nh, L, 64] -> split
    qkv, qkvr = _up(b, rng.standard_normal((B, L, 3 * nh * 64)), dt)
    t = b.transpose(b.reshape(qkv, [B, L, 3, nh, 64]), [2, 0, 3, 1, 4])
    q, k, v = [b.reshape(x, [B, nh, L, 64]) for x in b.split(t, 3, 0)]
    valid = np.ones((B, L), bool)
    valid[0, 200:] = False
    full, sliding = M.attention_masks(valid, 128)
    r = qkvr.reshape(B, L, 3, nh, 64).transpose(2, 0, 3, 1, 4)
    for mask in (full, sliding):
        got = to_f32(b.read(b.sdpa(q, k, v, b.fromHost(HostTensor("bool", mask.shape, mask.astype(np.uint8))), 0.125)))
        want = O.sdpa(r[0], r[1], r[2], mask, 0.125)
        assert np.abs(got - want).max() < TOL[dt]
    # fewer queries than keys (a slice of q's rows)
    qs = b.slice(q, [0, 0, 10, 0], [B, nh, 75, 64])
    got = to_f32(b.read(b.sdpa(qs, k, v, None, 0.125)))
    want = O.sdpa(r[0][:, :, 10:75], r[1], r[2], None, 0.125)
    assert np.abs(got - want).max() < TOL[dt]


def _dense(t) -> bool:
    import ctypes as C
    from laya_js_b200 import _lib
    d = C.c_uint64()
    _lib.call("lc_tensor_data", C.c_uint64(t.handle), C.byref(d))
    return d.value != 0


@pytest.mark.parametrize("dt", ["f16", "bf16"])
def test_sdpa_tcgen05_long_padded_batch(dt):
    """ModernBERT-base shape (12 heads) at 600 positions with padding: the
    sliding mask leaves most key blocks of a query tile empty (skipped by the
    kernel's per-tile key-block ranges); the result is the [B, nh, L, 64]
    view of [B, L, nh, 64] rows that the tcgen05 path writes."""
    b = backend()
    rng = np.random.default_rng(13)
    B, L, nh = 2, 600, 12
    qkv, qkvr = _up(b, rng.standard_normal((B, L, 3 * nh * 64)), dt)
    t = b.transpose(b.reshape(qkv, [B, L, 3, nh, 64]), [2, 0, 3, 1, 4])
    q, k, v = [b.reshape(x, [B, nh, L, 64]) for x in b.split(t, 3, 0)]
    valid = np.ones((B, L), bool)
    valid[1, 451:] = False
    r = qkvr.reshape(B, L, 3, nh, 64).transpose(2, 0, 3, 1, 4)
    for mask in M.attention_masks(valid, 128):
        out = b.sdpa(q, k, v, b.fromHost(HostTensor("bool", mask.shape, mask.astype(np.uint8))), 0.125)
        assert out.shape == (B, nh, L, 64) and not _dense(out), "expected the tcgen05 path's [B, L, nh, 64] rows"
        # the layer's transpose + reshape back to [B, L, H] is a view of those rows
        merged = b.reshape(b.transpose(out, [0, 2, 1, 3]), [B, L, nh * 64])
        assert _dense(merged)
        got = to_f32(b.read(out))
        want = O.sdpa(r[0], r[1], r[2], mask, 0.125)
        err = np.abs(got - want).max()
        assert err < TOL[dt], f"{dt}: max err {err}"


def test_sdpa_tcgen05_batch_of_one():
    """B = 1 (one prompt, the predict() case): the batch dimension's stride of
    a view is arbitrary and must not keep the call off the tcgen05 path."""
    b = backend()
    rng = np.random.default_rng(14)
    L, nh = 128, 12
    qkv, qkvr = _up(b, rng.standard_normal((1, L, 3 * nh * 64)), "f16")
    t = b.transpose(b.reshape(qkv, [1, L, 3, nh, 64]), [2, 0, 3, 1, 4])
    q, k, v = [b.reshape(x, [1, nh, L, 64]) for x in b.split(t, 3, 0)]
    r = qkvr.reshape(1, L, 3, nh, 64).transpose(2, 0, 3, 1, 4)
    mask = np.ones((1, 1, 1, L), bool)
    mask[0, 0, 0, 100:] = False
    out = b.sdpa(q, k, v, b.fromHost(HostTensor("bool", mask.shape, mask.astype(np.uint8))), 0.125)
    assert not _dense(out), "expected the tcgen05 path"
    err = np.abs(to_f32(b.read(out)) - O.sdpa(r[0], r[1], r[2], mask, 0.125)).max()
    assert err < TOL["f16"], f"max err {err}"


def _stats(b):
    import ctypes as C
    from laya_js_b200 import _lib
    lt, lb, ln = C.c_int64(), C.c_int64(), C.c_int64()
    _lib.call("lc_stats", C.byref(lt), C.byref(lb), C.byref(ln))
    return lt.value, lb.value, ln.value


def test_sdpa_packed_mask_reused_and_invalidated():
    """One mask tensor across calls (a forward's layers) is packed once; a
    write into it (lc_copy_into, what a compiled replay does to its inputs)
    is packed again; no tensor outlives the calls."""
    import ctypes as C
    from laya_js_b200 import _lib
    b = backend()
    rng = np.random.default_rng(21)
    B, H, L = 2, 3, 200
    q, qr = _up(b, rng.standard_normal((B, H, L, 64)), "f16")
    k, kr = _up(b, rng.standard_normal((B, H, L, 64)), "f16")
    v, vr = _up(b, rng.standard_normal((B, H, L, 64)), "f16")
    valid = np.ones((B, L), bool)
    valid[1, 150:] = False
    m1 = M.attention_masks(valid, 128)[1]
    valid[0, 60:] = False
    m2 = M.attention_masks(valid, 128)[1]

    def run(tm):
        n0 = _stats(b)[2]
        t = b.sdpa(q, k, v, tm, 0.125)
        n = _stats(b)[2] - n0
        y = to_f32(b.read(t))
        b.dispose(t)
        return y, n
    b.flush()
    bytes0 = _stats(b)[1]
    tm = b.fromHost(HostTensor("bool", m1.shape, m1.astype(np.uint8)))
    mask_bytes = _stats(b)[1] - bytes0
    ys = [run(tm) for _ in range(3)]
    assert [n for _, n in ys] == [2, 1, 1], f"mask packed once, then attention alone: {[n for _, n in ys]}"
    assert np.array_equal(ys[0][0], ys[1][0]) and np.array_equal(ys[0][0], ys[2][0])
    assert np.abs(ys[0][0] - O.sdpa(qr, kr, vr, m1, 0.125)).max() < TOL["f16"]
    src = b.fromHost(HostTensor("bool", m2.shape, m2.astype(np.uint8)))
    _lib.call("lc_copy_into", C.c_uint64(tm.handle), C.c_uint64(src.handle))
    b.dispose(src)
    y2, n = run(tm)
    assert n == 2, "a written mask is packed again"
    assert np.abs(y2 - O.sdpa(qr, kr, vr, m2, 0.125)).max() < TOL["f16"]
    b.flush()
    assert _stats(b)[1] == bytes0 + mask_bytes
    b.dispose(tm)
    b.flush()
    assert _stats(b)[1] == bytes0


def test_sdpa_packed_mask_inside_a_recording():
    """Backend.compile over two sdpa calls sharing a mask: the replay packs the
    replayed mask (not one cached before the recording) and matches eager."""
    b = backend()
    rng = np.random.default_rng(22)
    B, H, L = 2, 2, 160
    q, _ = _up(b, rng.standard_normal((B, H, L, 64)), "f16")
    k, _ = _up(b, rng.standard_normal((B, H, L, 64)), "f16")
    v, _ = _up(b, rng.standard_normal((B, H, L, 64)), "f16")

    def fn(q, k, v, m):
        return b.add(b.sdpa(q, k, v, m, 0.125), b.sdpa(v, k, q, m, 0.125))
    cf = b.compile(fn)
    masks = []
    for cut in (160, 90, 33, 120):
        valid = np.ones((B, L), bool)
        valid[1, cut:] = False
        masks.append(b.fromHost(HostTensor("bool", (B, 1, L, L), M.attention_masks(valid, 128)[1].astype(np.uint8))))
    for tm in masks:
        want = to_f32(b.read(fn(q, k, v, tm)))
        got = to_f32(b.read(cf(q, k, v, tm)))
        assert np.array_equal(got, want)
