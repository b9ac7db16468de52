"""The tensor-backend conformance runner, mirroring
packages/tensor-backend/src/conformance.ts:238-320 (runConformance): every
case in f32, and in f16 / bf16 when supported (inputs rounded to that dtype,
tolerance floors 2e-2 / 5e-2), optional ops through their compose helper,
quantized cases packed exactly as a laya-js checkpoint stores them.

``run_conformance(backend, cases, dtype)`` returns the list of failure
messages (empty = pass) instead of registering node:test cases.
"""
from __future__ import annotations

import base64
from typing import Iterable

import numpy as np

from . import compose as Cm
from .host import HostQuantized, HostTensor, pack_quantized, to_f32

REDUCED_TOLERANCE = {"f16": 2e-2, "bf16": 5e-2}
_NP = {"i32": "<i4", "bool": "u1", "u8": "u1", "i8": "i1", "u16": "<u2", "i16": "<i2", "u32": "<u4", "u64": "<u8",
       "i64": "<i8", "f64": "<f8"}
UNARY_NUMERICS = {"logicalNot", "sqrt", "rsqrt", "neg", "abs", "tanh", "sigmoid", "erf"}
BINARY_NUMERICS = {"equal", "notEqual", "less", "lessEqual", "greater", "greaterEqual", "logicalAnd", "logicalOr", "pow"}
REDUCE_NUMERICS = {"argmax", "argmin", "mean", "min"}
QUANTIZED_CASE_OPS = {"quantizedLinear", "quantizedEmbedding"}
FOLLOWS_RUN = {"f32", "f16", "bf16"}


def decode_tensor(e: dict) -> HostTensor:
    """conformance.ts:54-83 decodeTensor (float fixtures are always f32)."""
    raw = base64.b64decode(e["b64"])
    dt = e["dtype"] if e["dtype"] in _NP else "f32"
    a = np.frombuffer(raw, dtype=_NP.get(dt, "<f4")).reshape(e["shape"]).copy()
    return HostTensor(dt, tuple(e["shape"]), a)


def _upload(b, h: HostTensor, float_dtype: str):
    """conformance.ts:114-120."""
    if h.dtype != "f32" or float_dtype == "f32":
        return b.fromHost(h)
    f = b.fromHost(h)
    c = b.cast(f, float_dtype)
    b.dispose(f)
    return c


def case_quantized(c: dict, first: int) -> HostQuantized:
    """conformance.ts:153-162 caseQuantized."""
    a = c["args"]
    q = decode_tensor(c["inputs"][first])
    scales = decode_tensor(c["inputs"][first + 1])
    bi = c["inputs"][first + 2]
    N, K = q.shape
    return HostQuantized((N, K), a["bits"], a["groupSize"], a["mode"], pack_quantized(q.data, a["bits"]), scales,
                         decode_tensor(bi) if bi else None)


def _run_quantized(b, c, dtype, owned):
    """conformance.ts:164-182."""
    q = None
    try:
        if c["op"] == "quantizedLinear":
            x = _upload(b, decode_tensor(c["inputs"][0]), dtype)
            owned.append(x)
            bias = _upload(b, decode_tensor(c["inputs"][4]), dtype) if c["inputs"][4] else None
            if bias is not None:
                owned.append(bias)
            q = Cm.uploadQuantized(b, case_quantized(c, 1), dtype)
            return Cm.quantizedLinear(b, x, q, bias)
        ids = b.fromHost(decode_tensor(c["inputs"][3]))
        owned.append(ids)
        q = Cm.uploadQuantized(b, case_quantized(c, 0), dtype)
        return Cm.quantizedEmbedding(b, q, ids)
    finally:
        if q is not None:
            owned.extend([q.w, q.scales] + ([q.biases] if q.biases is not None else []))


def call_op(b, c: dict, xs: list):
    """conformance.ts:187-221 callOp."""
    a = c["args"]
    op = c["op"]
    x = xs[0]
    if op in UNARY_NUMERICS:
        return getattr(Cm, op)(b, x)
    if op in BINARY_NUMERICS:
        return getattr(Cm, op)(b, x, xs[1])
    if op in REDUCE_NUMERICS:
        return getattr(Cm, op)(b, x, a["axis"], a.get("keepDims", False))
    if op == "cumsum":
        return Cm.cumsum(b, x, a["axis"])
    if op in ("add", "sub", "mul", "div", "maximum"):
        return getattr(b, op)(x, xs[1])
    if op == "where":
        return b.where(x, xs[1], xs[2])
    if op == "scale":
        return b.scale(x, a["s"])
    if op in ("exp", "log", "relu", "gelu"):
        return getattr(b, op)(x)
    if op in ("sum", "max"):
        return getattr(b, op)(x, a["axis"], a.get("keepDims", False))
    if op in ("softmax", "sort"):
        return getattr(b, op)(x, a["axis"])
    if op == "matmul":
        return b.matmul(x, xs[1])
    if op == "linear":
        return b.linear(x, xs[1], xs[2] if len(xs) > 2 else None)
    if op == "layerNorm":
        return b.layerNorm(x, xs[1], xs[2], a["eps"])
    if op == "embedding":
        return b.embedding(x, xs[1])
    if op == "gatherRows":
        return b.gatherRows(x, xs[1])
    if op == "rope":
        return b.rope(x, a["base"])
    if op == "sdpa":
        return b.sdpa(x, xs[1], xs[2], xs[3], a["scale"])
    if op == "reshape":
        return b.reshape(x, a["shape"])
    if op == "transpose":
        return b.transpose(x, a["perm"])
    if op == "slice":
        return b.slice(x, a["begin"], a["end"])
    if op == "split":
        return b.split(x, a["parts"], a["axis"])
    if op == "concat":
        return b.concat(xs, a["axis"])
    if op == "cast":
        return b.cast(x, a["dtype"])
    if op == "geglu":
        return Cm.geglu(b, x)
    if op == "meanPool":
        return Cm.meanPool(b, x, xs[1])
    raise KeyError(f"conformance: unknown op {op}")


def assert_close(actual: np.ndarray, expected: np.ndarray, atol: float, rtol: float, label: str) -> None:
    """conformance.ts:223-236 assertClose."""
    g = np.asarray(actual, np.float64).reshape(-1)
    w = np.asarray(expected, np.float64).reshape(-1)
    if g.size != w.size:
        raise AssertionError(f"{label}: length {g.size} != {w.size}")
    gn, wn = np.isnan(g), np.isnan(w)
    if not np.array_equal(gn, wn):
        raise AssertionError(f"{label}: NaN mismatch at {int(np.argmax(gn != wn))}")
    ok = ~wn
    with np.errstate(invalid="ignore"):
        err = np.abs(g[ok] - w[ok]) - (atol + rtol * np.abs(w[ok]))
    if err.size and np.max(err) > 0:
        i = int(np.argmax(err))
        raise AssertionError(f"{label}: [{i}] got {g[ok][i]} want {w[ok][i]} (atol {atol}, rtol {rtol})")


def _host_values(h: HostTensor, f64: bool) -> np.ndarray:
    if h.dtype == "bf16" or not f64:
        return to_f32(h) if h.dtype != "f64" else np.asarray(h.data, np.float64)
    return np.asarray(h.data, np.float64)


def run_case(b, c: dict, dtype: str) -> None:
    """conformance.ts:257-290 (one case in one run dtype)."""
    quantized = c["op"] in QUANTIZED_CASE_OPS
    xs = [] if quantized else [(_upload(b, decode_tensor(e), dtype) if e else None) for e in c["inputs"]]
    outs = []
    try:
        out = _run_quantized(b, c, dtype, xs) if quantized else call_op(b, c, xs)
        outs.extend(out if isinstance(out, list) else [out])
        if len(outs) != len(c["outputs"]):
            raise AssertionError(f"{c['name']}: {len(outs)} outputs, want {len(c['outputs'])}")
        tol = REDUCED_TOLERANCE.get(dtype, 0.0)
        for i, (o, e) in enumerate(zip(outs, c["outputs"])):
            want = decode_tensor(e)
            got = b.read(o)
            if list(got.shape) != list(want.shape):
                raise AssertionError(f"{c['name']}: shape {list(got.shape)} want {list(want.shape)}")
            if c["op"] in Cm.NUMERICS_OPS and want.dtype not in FOLLOWS_RUN:
                if got.dtype != want.dtype:
                    raise AssertionError(f"{c['name']}[{i}] {dtype}: dtype {got.dtype} want {want.dtype}")
            f64 = want.dtype == "f64" or got.dtype == "f64"
            assert_close(_host_values(got, f64), _host_values(want, f64), max(c["atol"], tol), max(c["rtol"], tol),
                         f"{c['name']}[{i}] {dtype}")
    finally:
        for t in [*xs, *outs]:
            if t is not None:
                b.dispose(t)


def applicable(b, c) -> bool:
    """conformance.ts:294-295."""
    return not (c.get("nativeOnly") and c["op"] in Cm.NUMERICS_OPS and not Cm.has_native(b, c["op"]))


def case_supported(b, c) -> bool:
    """conformance.ts:303-308."""
    fixed = [e["dtype"] for e in [*c["inputs"], *c["outputs"]] if e and e["dtype"] not in FOLLOWS_RUN]
    tgt = c["args"].get("dtype") if c["op"] == "cast" else None
    if tgt and tgt not in FOLLOWS_RUN:
        fixed.append(tgt)
    return all(b.supports(d) for d in fixed)


def run_conformance(b, cases: Iterable[dict], dtype: str) -> list[str]:
    """conformance.ts:309-316 runAll for one dtype: the failure messages."""
    if not b.supports(dtype):
        return []
    failures = []
    for c in cases:
        if dtype != "f32" and c.get("f32Only"):
            continue
        if not applicable(b, c) or not case_supported(b, c):
            continue
        try:
            run_case(b, c, dtype)
        except Exception as e:  # noqa: BLE001 - collected like the reference's runAll
            failures.append(f"{c['name']}: {e}")
    return failures
