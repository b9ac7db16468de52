"""numpy restatement of the tensor-backend contract ops (test oracle only).

Every function takes and returns numpy arrays. Float math is done in float64
and the result is rounded once to the storage dtype (float32 unless the input
is float64), which is how the reference CPU backend is documented to work
("f32 reference backend ... over packed f64 panels",
packages/backend-cpu/README.md:37-39). Integer ops keep their own dtype and
wrap like fixed-width integers.

Each function cites the contract line it restates
(packages/tensor-backend/src/index.ts unless another file is named).
"""
from __future__ import annotations

import math

import numpy as np
from scipy.special import erf as _erf

# contract dtype name -> numpy dtype (bf16 has no numpy type; it is carried as f32 here)
NP = {
    "f32": np.float32, "f16": np.float16, "bf16": np.float32, "i32": np.int32,
    "bool": np.bool_, "u8": np.uint8, "i8": np.int8, "u16": np.uint16,
    "i16": np.int16, "u32": np.uint32, "u64": np.uint64, "i64": np.int64,
    "f64": np.float64,
}


def dtype_name(a: np.ndarray) -> str:
    for k, v in NP.items():
        if k in ("bf16",):
            continue
        if a.dtype == v:
            return k
    raise TypeError(a.dtype)


def _is_float(a: np.ndarray) -> bool:
    return a.dtype.kind == "f"


def _out_float(*xs: np.ndarray):
    return np.float64 if any(x.dtype == np.float64 for x in xs) else np.float32


def _f64(a: np.ndarray) -> np.ndarray:
    return a.astype(np.float64)


# ---------------------------------------------------------------- elementwise
# index.ts:180-198 — numpy broadcasting; float math rounded once to storage.

def _binary(a, b, f):
    if _is_float(a) or _is_float(b):
        return f(_f64(a), _f64(b)).astype(_out_float(a, b))
    if a.dtype == np.bool_ and b.dtype == np.bool_:
        a, b = a.astype(np.int32), b.astype(np.int32)
    with np.errstate(over="ignore"):
        return f(a, b).astype(np.result_type(a, b))


def add(a, b):
    """index.ts:180 add."""
    return _binary(a, b, np.add)


def sub(a, b):
    """index.ts:181 sub."""
    return _binary(a, b, np.subtract)


def mul(a, b):
    """index.ts:182 mul."""
    return _binary(a, b, np.multiply)


def div(a, b):
    """index.ts:183-188 div: true division (integer inputs give f32)."""
    return (_f64(a) / _f64(b)).astype(_out_float(a, b))


def maximum(a, b):
    """index.ts:189 maximum."""
    return _binary(a, b, np.maximum)


def where(cond, a, b):
    """index.ts:190-191 where: cond bool, a/b broadcast against cond."""
    out = np.where(cond.astype(bool), a, b)
    return out.astype(np.result_type(a, b))


def scale(x, s):
    """index.ts:192-193 scale by a scalar."""
    return (_f64(x) * s).astype(x.dtype if _is_float(x) else np.float32)


def _unary_float(x, f):
    return f(_f64(x)).astype(x.dtype if _is_float(x) else np.float32)


def exp(x):
    """index.ts:194 exp."""
    with np.errstate(over="ignore"):
        return _unary_float(x, np.exp)


def log(x):
    """index.ts:195 log."""
    with np.errstate(divide="ignore", invalid="ignore"):
        return _unary_float(x, np.log)


def relu(x):
    """index.ts:196 relu."""
    return np.maximum(x, np.zeros((), x.dtype))


def gelu_f64(v):
    return 0.5 * v * (1.0 + _erf(v / math.sqrt(2.0)))


def gelu(x):
    """index.ts:197-198 exact-erf GELU 0.5·x·(1 + erf(x/√2))."""
    return _unary_float(x, gelu_f64)


def cast(x, dtype: str):
    """index.ts:177 cast (float -> int truncates toward zero; -> bool is nonzero)."""
    t = NP[dtype]
    if dtype == "bool":
        return x != 0
    if np.issubdtype(t, np.integer) and _is_float(x):
        return np.trunc(x).astype(t)
    return x.astype(t)


# ---------------------------------------------------------------- shape ops
# index.ts:169-177 — numpy semantics.

def reshape(x, shape):
    return x.reshape(shape)


def transpose(x, perm):
    return np.ascontiguousarray(np.transpose(x, perm))


def slice_(x, begin, end):
    idx = tuple(slice(b, e) for b, e in zip(begin, end))
    return np.ascontiguousarray(x[idx])


def split(x, parts, axis):
    return [np.ascontiguousarray(p) for p in np.split(x, parts, axis=axis)]


def concat(xs, axis):
    return np.concatenate(xs, axis=axis)


# ---------------------------------------------------------------- reductions
# index.ts:201-206

def sum_(x, axis, keep_dims=False):
    if _is_float(x):
        return _f64(x).sum(axis=axis, keepdims=keep_dims).astype(x.dtype)
    if x.dtype == np.bool_:
        return x.astype(np.int32).sum(axis=axis, keepdims=keep_dims).astype(np.int32)
    return x.sum(axis=axis, keepdims=keep_dims, dtype=x.dtype)


def max_(x, axis, keep_dims=False):
    return x.max(axis=axis, keepdims=keep_dims)


def softmax(x, axis):
    """index.ts:203-204 numerically stable softmax, f32 (here f64) internally."""
    v = _f64(x)
    m = v.max(axis=axis, keepdims=True)
    e = np.exp(v - m)
    return (e / e.sum(axis=axis, keepdims=True)).astype(x.dtype if _is_float(x) else np.float32)


def sort(x, axis):
    """index.ts:205-206 ascending sort."""
    return np.sort(x, axis=axis, kind="stable")


# ---------------------------------------------------------------- linear algebra / NN

def matmul(a, b):
    """index.ts:209-210 batched matmul with broadcast leading dims."""
    return np.matmul(_f64(a), _f64(b)).astype(_out_float(a, b))


def linear(x, w, b=None):
    """index.ts:211-215 y = x·wᵀ (+ b), accumulated wide."""
    y = _f64(x) @ _f64(w).T
    if b is not None:
        y = y + _f64(b)
    return y.astype(np.float32)


def layer_norm(x, weight, bias, eps):
    """index.ts:216-217 LayerNorm over the last axis (biased variance), f32 stats."""
    v = _f64(x)
    mu = v.mean(axis=-1, keepdims=True)
    var = ((v - mu) ** 2).mean(axis=-1, keepdims=True)
    y = (v - mu) / np.sqrt(var + eps)
    if weight is not None:
        y = y * _f64(weight)
    if bias is not None:
        y = y + _f64(bias)
    return y.astype(np.float32)


def embedding(table, ids):
    """index.ts:218-219 row gather table[ids]."""
    return table[ids.astype(np.int64)]


def gather_rows(x, idx):
    """index.ts:220-224 x[arange(B)[:, None], idx]."""
    B = x.shape[0]
    return x[np.arange(B)[:, None], idx.astype(np.int64)]


def rope_tables(L: int, D: int, base: float):
    """cos/sin [L, D/2] with MLX's float32 angle rounding, as the reference
    restates it (packages/backend-webgpu/src/backend.ts:1179-1195: the
    inverse frequency and the product l·inv are rounded to f32; cos and sin
    themselves are exact)."""
    half = D // 2
    f32 = lambda v: float(np.float32(v))
    lb = f32(math.log2(base))
    cos = np.empty((L, half))
    sin = np.empty((L, half))
    for i in range(half):
        inv = f32(2.0 ** f32(-f32(i / half) * lb))
        for l in range(L):
            th = f32(l * inv)
            cos[l, i] = math.cos(th)
            sin[l, i] = math.sin(th)
    return cos, sin


def rope(x, base, positions=None):
    """index.ts:225-229 split-half (NeoX) rotation of x [..., L, D], positions 0..L-1."""
    L, D = x.shape[-2], x.shape[-1]
    half = D // 2
    n = L if positions is None else int(np.max(positions)) + 1
    cos, sin = rope_tables(max(n, 1), D, base)
    if positions is not None:
        cos, sin = cos[positions], sin[positions]
    else:
        cos, sin = cos[:L], sin[:L]
    v = _f64(x)
    a, b = v[..., :half], v[..., half:]
    out = np.concatenate([a * cos - b * sin, b * cos + a * sin], axis=-1)
    return out.astype(x.dtype if _is_float(x) else np.float32)


def sdpa(q, k, v, mask, scale_):
    """index.ts:230-237 softmax(q·kᵀ·scale masked by bool)·v, softmax wide."""
    s = np.matmul(_f64(q), np.swapaxes(_f64(k), -1, -2)) * scale_
    if mask is not None:
        s = np.where(np.broadcast_to(mask.astype(bool), s.shape), s, -np.inf)
    m = s.max(axis=-1, keepdims=True)
    e = np.exp(s - m)
    p = e / e.sum(axis=-1, keepdims=True)
    return np.matmul(p, _f64(v)).astype(np.float32)


def geglu(x):
    """compose.ts:87-93 gelu(x[..., :F]) · x[..., F:]."""
    F = x.shape[-1] // 2
    v = _f64(x)
    return (gelu_f64(v[..., :F]) * v[..., F:]).astype(np.float32)


def mean_pool(x, mask):
    """compose.ts:96-105 masked mean over axis 1 → f32 [B, D]."""
    m = mask.astype(np.float64)[:, :, None]
    total = (_f64(x) * m).sum(axis=1)
    n = m.sum(axis=1)
    return (total / np.maximum(n, 1.0)).astype(np.float32)


# ---------------------------------------------------------------- general numerics
# index.ts:265-316

def _cmp(a, b, f):
    if a.dtype == np.uint64 or b.dtype == np.uint64:
        return f(a, b)
    if _is_float(a) or _is_float(b):
        return f(_f64(a), _f64(b))
    return f(a.astype(np.int64), b.astype(np.int64))


def equal(a, b): return _cmp(a, b, np.equal)
def not_equal(a, b): return _cmp(a, b, np.not_equal)
def less(a, b): return _cmp(a, b, np.less)
def less_equal(a, b): return _cmp(a, b, np.less_equal)
def greater(a, b): return _cmp(a, b, np.greater)
def greater_equal(a, b): return _cmp(a, b, np.greater_equal)
def logical_and(a, b): return np.logical_and(a != 0, b != 0)
def logical_or(a, b): return np.logical_or(a != 0, b != 0)
def logical_not(x): return x == 0


def sqrt(x):
    with np.errstate(invalid="ignore"):
        return _unary_float(x, np.sqrt)


def rsqrt(x):
    with np.errstate(divide="ignore", invalid="ignore"):
        return _unary_float(x, lambda v: 1.0 / np.sqrt(v))


def pow_(a, b):
    with np.errstate(invalid="ignore", divide="ignore", over="ignore"):
        return np.power(_f64(a), _f64(b)).astype(_out_float(a, b))


def neg(x):
    if x.dtype == np.bool_:
        return -x.astype(np.int32)
    with np.errstate(over="ignore"):
        return np.negative(x)


def abs_(x):
    if x.dtype == np.bool_:
        return x.astype(np.int32)
    return np.abs(x)


def tanh(x): return _unary_float(x, np.tanh)


def sigmoid(x):
    with np.errstate(over="ignore"):
        return _unary_float(x, lambda v: 1.0 / (1.0 + np.exp(-v)))


def erf(x): return _unary_float(x, _erf)


def argmax(x, axis, keep_dims=False):
    r = np.argmax(x, axis=axis).astype(np.int32)
    return np.expand_dims(r, axis) if keep_dims else r


def argmin(x, axis, keep_dims=False):
    r = np.argmin(x, axis=axis).astype(np.int32)
    return np.expand_dims(r, axis) if keep_dims else r


def mean(x, axis, keep_dims=False):
    """index.ts:302-303 mean (integer input -> f32)."""
    out = _f64(x).mean(axis=axis, keepdims=keep_dims)
    return out.astype(np.float64 if x.dtype == np.float64 else np.float32)


def min_(x, axis, keep_dims=False):
    return x.min(axis=axis, keepdims=keep_dims)


def cumsum(x, axis):
    """index.ts:306-315 inclusive prefix sum; integers wrap in their own dtype, bool -> i32."""
    if x.dtype == np.bool_:
        return np.cumsum(x.astype(np.int32), axis=axis, dtype=np.int32)
    if _is_float(x):
        return np.cumsum(_f64(x), axis=axis).astype(x.dtype)
    with np.errstate(over="ignore"):
        return np.cumsum(x, axis=axis, dtype=x.dtype)


# ---------------------------------------------------------------- quantized
# index.ts:98-137, 250-263; host.ts:136-184; compose.ts:367-438

def pack_quantized(q: np.ndarray, bits: int) -> np.ndarray:
    """host.ts:174-184 packQuantized: 8-bit one byte per value; 4-bit two per
    byte, the even column in the low nibble."""
    q = np.asarray(q).astype(np.int64).reshape(-1)
    if bits == 8:
        return (q & 255).astype(np.uint8)
    lo, hi = q[0::2] & 15, q[1::2] & 15
    return (lo | (hi << 4)).astype(np.uint8)


def unpack_quantized(data: np.ndarray, N: int, K: int, bits: int, mode: str) -> np.ndarray:
    """host.ts:155-171 unpackQuantized → int values [N, K] (signed for symmetric)."""
    d = np.asarray(data, dtype=np.uint8)
    signed = mode == "symmetric"
    if bits == 8:
        q = d.astype(np.int8).astype(np.int64) if signed else d.astype(np.int64)
    else:
        lo = (d & 15).astype(np.int64)
        hi = (d >> 4).astype(np.int64)
        if signed:
            lo = np.where(lo >= 8, lo - 16, lo)
            hi = np.where(hi >= 8, hi - 16, hi)
        q = np.empty(d.size * 2, np.int64)
        q[0::2], q[1::2] = lo, hi
    return q.reshape(N, K)


def dequantize(q: np.ndarray, scales: np.ndarray, biases, group_size: int, out_dtype=np.float32):
    """compose.ts:367-399 dequantRows: value (r, j) = q·scale[r, ⌊j/g⌋] (+ bias),
    computed wide and rounded once (packages/laya/src/quant.ts:189-195)."""
    N, K = q.shape
    gidx = np.arange(K) // group_size
    v = q.astype(np.float64) * scales.astype(np.float64)[:, gidx]
    if biases is not None:
        v = v + biases.astype(np.float64)[:, gidx]
    return v.astype(out_dtype)


def quantized_linear(x, q, scales, biases, group_size, bias=None):
    """index.ts:256-259 y = x·dequant(w)ᵀ (+ bias)."""
    w = dequantize(q, scales, biases, group_size, np.float64)
    y = _f64(x) @ w.T
    if bias is not None:
        y = y + _f64(bias)
    return y.astype(np.float32)


def quantized_embedding(q, scales, biases, group_size, ids):
    """index.ts:260-262 row gather of dequant(w) by ids."""
    w = dequantize(q, scales, biases, group_size, np.float32)
    return w[ids.astype(np.int64)]


def quantize_affine(w: np.ndarray, bits: int, group_size: int):
    """Min/max range fit of packages/laya/src/quant.ts:157-160 (`fitAffine`
    without its refinement steps) and the assignment rule of quant.ts:135-146:
    b = f16(min), s = f16((max − b) / (2^bits − 1)),
    q = clamp(⌊(w − b)/s + ½⌋, 0, 2^bits − 1) (JS Math.round), q = 0 when s ≤ 0.
    Returns (q int [N, K], scales f16 [N, G], biases f16 [N, G])."""
    N, K = w.shape
    G = -(-K // group_size)
    lv = (1 << bits) - 1
    q = np.zeros((N, K), np.int64)
    s_out = np.zeros((N, G), np.float16)
    b_out = np.zeros((N, G), np.float16)
    w64 = w.astype(np.float64)
    for g in range(G):
        seg = w64[:, g * group_size:(g + 1) * group_size]
        lo, hi = seg.min(axis=1), seg.max(axis=1)
        b = lo.astype(np.float16)
        s = ((hi - b.astype(np.float64)) / lv).astype(np.float16)
        s64 = s.astype(np.float64)[:, None]
        ok = s64 > 0
        with np.errstate(divide="ignore", invalid="ignore"):
            qq = np.where(ok, np.floor((seg - b.astype(np.float64)[:, None]) / np.where(ok, s64, 1.0) + 0.5), 0.0)
        qq = np.clip(qq, 0, lv)
        q[:, g * group_size:(g + 1) * group_size] = qq.astype(np.int64)
        s_out[:, g], b_out[:, g] = s, b
    return q, s_out, b_out
