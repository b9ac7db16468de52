"""Call-site helpers for the optional ops of the contract, mirroring
packages/tensor-backend/src/compose.ts: each uses the backend's native op when
it has one and the reference's default composition from required ops
otherwise. ``without_optional_ops`` mirrors conformance.ts:131-144
(``withoutOptionalOps``) so the compositions can be checked on a real backend.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Any, Optional

import numpy as np

from .host import HostQuantized, HostTensor, to_f32, unpack_quantized, validate_quantized

NUMERICS_OPS = ("equal", "notEqual", "less", "lessEqual", "greater", "greaterEqual", "logicalAnd", "logicalOr",
                "logicalNot", "sqrt", "rsqrt", "pow", "neg", "abs", "tanh", "sigmoid", "erf", "argmax", "argmin",
                "mean", "min", "cumsum")
QUANTIZED_OPS = ("fromHostQuantized", "quantizedLinear", "quantizedEmbedding")
_FLOATS = ("f32", "f16", "bf16", "f64")


def has_native(b, op: str) -> bool:
    """compose.ts:48-50 hasNative."""
    return callable(getattr(b, op, None))


def has_native_quantized(b) -> bool:
    """compose.ts:313-315."""
    return all(has_native(b, op) for op in QUANTIZED_OPS)


class without_optional_ops:
    """conformance.ts:131-144: a view of `b` that hides the given optional ops."""

    def __init__(self, b, ops=NUMERICS_OPS):
        object.__setattr__(self, "_b", b)
        object.__setattr__(self, "_hidden", set(ops))

    def __getattr__(self, name):
        if name in self._hidden:
            raise AttributeError(name)
        return getattr(self._b, name)


def _is_float(d):
    return d in _FLOATS


def _as_float(b, x):
    return x if _is_float(x.dtype) else b.cast(x, "f32")


def _bit(b, x):
    return b.cast(b.cast(x, "bool"), "f32")


def zerosLike(b, x, dtype=None):
    return b.scope(lambda: b.cast(b.scale(_bit(b, x), 0), dtype or x.dtype))


def onesLike(b, x, dtype=None):
    return b.scope(lambda: b.cast(b.cast(b.exp(b.scale(_bit(b, x), 0)), "bool"), dtype or x.dtype))


# ---------------------------------------------------------------- fused

def geglu(b, x):
    """compose.ts:87-93."""
    if has_native(b, "geglu"):
        return b.geglu(x)

    def f():
        value, gate = b.split(x, 2, len(x.shape) - 1)
        return b.mul(b.gelu(value), gate)
    return b.scope(f)


def meanPool(b, x, mask):
    """compose.ts:96-105."""
    if has_native(b, "meanPool"):
        return b.meanPool(x, mask)

    def f():
        B, L = x.shape[0], x.shape[1]
        m = b.cast(b.reshape(mask, [B, L, 1]), "f32")
        total = b.sum(b.mul(b.cast(x, "f32"), m), 1)
        n = b.sum(m, 1)
        return b.div(total, b.maximum(n, onesLike(b, n)))
    return b.scope(f)


# ---------------------------------------------------------------- logical / comparisons (compose.ts:109-185)

def logicalNot(b, x):
    if has_native(b, "logicalNot"):
        return b.logicalNot(x)
    return b.scope(lambda: (lambda v: b.cast(b.sub(onesLike(b, v), v), "bool"))(_bit(b, x)))


def logicalAnd(b, x, y):
    if has_native(b, "logicalAnd"):
        return b.logicalAnd(x, y)
    return b.scope(lambda: b.cast(b.mul(_bit(b, x), _bit(b, y)), "bool"))


def logicalOr(b, x, y):
    if has_native(b, "logicalOr"):
        return b.logicalOr(x, y)
    return b.scope(lambda: b.cast(b.maximum(_bit(b, x), _bit(b, y)), "bool"))


def _diff(b, x, y):
    def wide(t):
        if t.dtype == "bool":
            return b.cast(t, "i32")
        return t if (t.dtype == "i32" or _is_float(t.dtype)) else b.cast(t, "f32")
    return b.sub(wide(x), wide(y))


def greater(b, x, y):
    if has_native(b, "greater"):
        return b.greater(x, y)
    return b.scope(lambda: b.cast(b.relu(_diff(b, x, y)), "bool"))


def less(b, x, y):
    if has_native(b, "less"):
        return b.less(x, y)
    return greater(b, y, x)


def notEqual(b, x, y):
    if has_native(b, "notEqual"):
        return b.notEqual(x, y)
    return b.scope(lambda: b.cast(_diff(b, x, y), "bool"))


def equal(b, x, y):
    if has_native(b, "equal"):
        return b.equal(x, y)
    return b.scope(lambda: logicalNot(b, notEqual(b, x, y)))


def lessEqual(b, x, y):
    if has_native(b, "lessEqual"):
        return b.lessEqual(x, y)
    return b.scope(lambda: logicalNot(b, greater(b, x, y)))


def greaterEqual(b, x, y):
    if has_native(b, "greaterEqual"):
        return b.greaterEqual(x, y)
    return b.scope(lambda: logicalNot(b, less(b, x, y)))


# ---------------------------------------------------------------- unary math (compose.ts:189-273)

def neg(b, x):
    if has_native(b, "neg"):
        return b.neg(x)
    if _is_float(x.dtype):
        return b.scale(x, -1)
    if x.dtype == "bool":
        return b.scope(lambda: b.sub(zerosLike(b, x, "i32"), b.cast(x, "i32")))
    return b.scope(lambda: b.sub(zerosLike(b, x, x.dtype), x))


def abs(b, x):
    if has_native(b, "abs"):
        return b.abs(x)
    return b.scope(lambda: b.maximum(x, neg(b, x)))


def sqrt(b, x):
    if has_native(b, "sqrt"):
        return b.sqrt(x)
    return b.scope(lambda: b.exp(b.scale(b.log(_as_float(b, x)), 0.5)))


def rsqrt(b, x):
    if has_native(b, "rsqrt"):
        return b.rsqrt(x)
    return b.scope(lambda: b.exp(b.scale(b.log(_as_float(b, x)), -0.5)))


def pow(b, x, y):
    if has_native(b, "pow"):
        return b.pow(x, y)
    return b.scope(lambda: b.exp(b.mul(_as_float(b, y), b.log(_as_float(b, x)))))


def sigmoid(b, x):
    if has_native(b, "sigmoid"):
        return b.sigmoid(x)

    def f():
        fx = _as_float(b, x)
        one = onesLike(b, fx)
        return b.div(one, b.add(one, b.exp(neg(b, fx))))
    return b.scope(f)


def tanh(b, x):
    if has_native(b, "tanh"):
        return b.tanh(x)

    def f():
        fx = _as_float(b, x)
        return b.sub(b.scale(sigmoid(b, b.scale(fx, 2)), 2), onesLike(b, fx))
    return b.scope(f)


_ERF_SERIES_TERMS, _ERF_CF_DEPTH = 10, 28
_TWO_OVER_SQRT_PI = 1.1283791670955126


def erf(b, x):
    """compose.ts:228-253 (series below 1, continued fraction above)."""
    if has_native(b, "erf"):
        return b.erf(x)

    def f():
        fx = _as_float(b, x)
        one = onesLike(b, fx)
        c = lambda v: b.scale(one, v)
        x2 = b.mul(fx, fx)
        term, s = fx, fx
        for n in range(1, _ERF_SERIES_TERMS + 1):
            term = b.mul(term, b.scale(x2, -1 / n))
            s = b.add(s, b.scale(term, 1 / (2 * n + 1)))
        series = b.scale(s, _TWO_OVER_SQRT_PI)
        z = abs(b, fx)
        t = b.add(b.scale(x2, 2), one)
        fr = zerosLike(b, fx)
        for n in range(_ERF_CF_DEPTH, 0, -1):
            fr = b.div(c((2 * n - 1) * (2 * n)), b.sub(b.add(t, c(4 * n)), fr))
        erfc = b.div(b.mul(b.exp(neg(b, x2)), b.scale(z, _TWO_OVER_SQRT_PI)), b.sub(t, fr))
        tail = b.sub(one, erfc)
        signed = b.where(less(b, fx, zerosLike(b, fx)), neg(b, tail), tail)
        return b.where(less(b, z, one), series, signed)
    return b.scope(f)


# ---------------------------------------------------------------- reductions (compose.ts:257-302)

def _axis_len(x, axis):
    r = len(x.shape)
    a = axis + r if axis < 0 else axis
    if a < 0 or a >= r:
        raise IndexError(f"axis {axis} out of range for rank {r}")
    return x.shape[a]


def mean(b, x, axis, keepDims=False):
    if has_native(b, "mean"):
        return b.mean(x, axis, keepDims)
    n = _axis_len(x, axis)
    return b.scope(lambda: b.scale(b.sum(_as_float(b, x), axis, keepDims), 1 / n))


def min(b, x, axis, keepDims=False):
    if has_native(b, "min"):
        return b.min(x, axis, keepDims)
    if x.dtype == "bool":
        return b.scope(lambda: logicalNot(b, b.max(logicalNot(b, x), axis, keepDims)))
    return b.scope(lambda: neg(b, b.max(neg(b, x), axis, keepDims)))


def cumsum(b, x, axis):
    if has_native(b, "cumsum"):
        return b.cumsum(x, axis)
    raise RuntimeError(f"cumsum: the {b.name} backend has no native cumsum and there is no default composition")


def _arg_reduce(b, x, axis, keepDims, which):
    if not has_native(b, "cumsum"):
        raise RuntimeError(f"{which}: the {b.name} backend has neither a native {which} nor a native cumsum to compose it from")
    n = _axis_len(x, axis)

    def f():
        best = b.max(x, axis, True) if which == "argmax" else min(b, x, axis, True)
        ones = onesLike(b, x, "i32")
        iota = b.sub(cumsum(b, ones, axis), ones)
        cand = b.where(equal(b, x, best), iota, b.cast(b.scale(onesLike(b, x, "f32"), n), "i32"))
        return b.cast(min(b, cand, axis, keepDims), "i32")
    return b.scope(f)


def argmax(b, x, axis, keepDims=False):
    if has_native(b, "argmax"):
        return b.argmax(x, axis, keepDims)
    return _arg_reduce(b, x, axis, keepDims, "argmax")


def argmin(b, x, axis, keepDims=False):
    if has_native(b, "argmin"):
        return b.argmin(x, axis, keepDims)
    return _arg_reduce(b, x, axis, keepDims, "argmin")


# ---------------------------------------------------------------- quantized (compose.ts:305-438)

@dataclass
class QuantizedTensor:
    """index.ts:122-137."""
    shape: tuple
    bits: int
    groupSize: int
    mode: str
    dtype: str
    native: bool
    w: Any
    scales: Any
    biases: Optional[Any]


def is_quantized(x) -> bool:
    return isinstance(x, QuantizedTensor)


def _upload_float(b, h: HostTensor, dtype: str):
    src = h if (h.dtype == "f32" or b.supports(h.dtype)) else HostTensor("f32", h.shape, to_f32(h))
    t = b.fromHost(src)
    if t.dtype == dtype:
        return t
    c = b.cast(t, dtype)
    b.dispose(t)
    return c


def uploadQuantized(b, h: HostQuantized, dtype: str) -> QuantizedTensor:
    """compose.ts:342-365."""
    validate_quantized(h)
    if not _is_float(dtype):
        raise TypeError(f"uploadQuantized: dtype must be float, got {dtype}")
    if has_native_quantized(b):
        q = b.fromHostQuantized(h, dtype)
        if q is not None:
            return q
    N, K = h.shape
    q = unpack_quantized(h)
    made = []
    try:
        made.append(_upload_float(b, HostTensor("f32", (N, K), q.astype(np.float32).reshape(N, K)), dtype))
        made.append(_upload_float(b, h.scales, dtype))
        if h.mode == "affine":
            made.append(_upload_float(b, h.biases, dtype))
    except BaseException:
        for t in made:
            b.dispose(t)
        raise
    return QuantizedTensor((N, K), h.bits, h.groupSize, h.mode, dtype, False, made[0], made[1], made[2] if len(made) > 2 else None)


def disposeQuantized(b, q: QuantizedTensor) -> None:
    b.dispose(q.w)
    b.dispose(q.scales)
    if q.biases is not None:
        b.dispose(q.biases)


def _dequant_rows(b, w, scales, biases, group_size, dtype):
    """compose.ts:372-399 dequantRows."""
    def f():
        R, K = w.shape
        G, full = -(-K // group_size), K // group_size
        fl = lambda t: b.cast(t, "f32")

        def part(w0, w1, g0, g1):
            n = g1 - g0
            gs = (w1 - w0) // n
            wq = b.reshape(fl(b.slice(w, [0, w0], [R, w1])), [R, n, gs])
            s = b.reshape(fl(b.slice(scales, [0, g0], [R, g1])), [R, n, 1])
            v = b.mul(wq, s)
            if biases is not None:
                v = b.add(v, b.reshape(fl(b.slice(biases, [0, g0], [R, g1])), [R, n, 1]))
            return b.reshape(v, [R, w1 - w0])
        pieces = []
        if full:
            pieces.append(part(0, full * group_size, 0, full))
        if G > full:
            pieces.append(part(full * group_size, K, full, G))
        v = pieces[0] if len(pieces) == 1 else b.concat(pieces, 1)
        return v if v.dtype == dtype else b.cast(v, dtype)
    return b.scope(f)


def quantizedLinear(b, x, q: QuantizedTensor, bias=None):
    """compose.ts:407-417."""
    if x.shape[-1] != q.shape[1]:
        raise ValueError(f"quantizedLinear: x {list(x.shape)} vs w {list(q.shape)}")
    if q.native:
        if not has_native(b, "quantizedLinear"):
            raise RuntimeError(f"quantizedLinear: the {b.name} backend has no native quantizedLinear for its native-layout weight")
        return b.quantizedLinear(x, q.w, q.scales, q.biases, q, bias)
    return b.scope(lambda: b.linear(x, _dequant_rows(b, q.w, q.scales, q.biases, q.groupSize,
                                                     x.dtype if _is_float(x.dtype) else "f32"), bias))


def quantizedEmbedding(b, q: QuantizedTensor, ids):
    """compose.ts:420-429."""
    if q.native:
        if not has_native(b, "quantizedEmbedding"):
            raise RuntimeError(f"quantizedEmbedding: the {b.name} backend has no native quantizedEmbedding")
        return b.quantizedEmbedding(q.w, q.scales, q.biases, q, ids)

    def f():
        n = int(np.prod(ids.shape))
        flat = b.reshape(ids, [n])
        rows = _dequant_rows(b, b.embedding(q.w, flat), b.embedding(q.scales, flat),
                             b.embedding(q.biases, flat) if q.biases is not None else None, q.groupSize, q.dtype)
        return b.reshape(rows, [*ids.shape, q.shape[1]])
    return b.scope(f)


def linearAny(b, x, w, bias=None):
    """compose.ts:432-434."""
    return quantizedLinear(b, x, w, bias) if is_quantized(w) else b.linear(x, w, bias)


def embeddingAny(b, table, ids):
    """compose.ts:437-439."""
    return quantizedEmbedding(b, table, ids) if is_quantized(table) else b.embedding(table, ids)
