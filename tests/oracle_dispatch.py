"""Maps a conformance case (conformance.ts:187-221 callOp) onto the oracle."""
from __future__ import annotations

import numpy as np

from oracle import ops as O


def run_case(c: dict, xs: list):
    a = c["args"]
    op = c["op"]
    x = xs[0]
    simple = {
        "add": O.add, "sub": O.sub, "mul": O.mul, "div": O.div, "maximum": O.maximum,
        "equal": O.equal, "notEqual": O.not_equal, "less": O.less, "lessEqual": O.less_equal,
        "greater": O.greater, "greaterEqual": O.greater_equal, "logicalAnd": O.logical_and,
        "logicalOr": O.logical_or, "pow": O.pow_, "matmul": O.matmul,
    }
    unary = {"exp": O.exp, "log": O.log, "relu": O.relu, "gelu": O.gelu, "logicalNot": O.logical_not,
             "sqrt": O.sqrt, "rsqrt": O.rsqrt, "neg": O.neg, "abs": O.abs_, "tanh": O.tanh,
             "sigmoid": O.sigmoid, "erf": O.erf, "geglu": O.geglu}
    red = {"sum": O.sum_, "max": O.max_, "argmax": O.argmax, "argmin": O.argmin, "mean": O.mean, "min": O.min_}
    if op in simple:
        return simple[op](x, xs[1])
    if op in unary:
        return unary[op](x)
    if op in red:
        return red[op](x, a["axis"], a.get("keepDims", False))
    if op == "where":
        return O.where(x, xs[1], xs[2])
    if op == "scale":
        return O.scale(x, a["s"])
    if op == "softmax":
        return O.softmax(x, a["axis"])
    if op == "sort":
        return O.sort(x, a["axis"])
    if op == "cumsum":
        return O.cumsum(x, a["axis"])
    if op == "linear":
        return O.linear(x, xs[1], xs[2])
    if op == "layerNorm":
        return O.layer_norm(x, xs[1], xs[2], a["eps"])
    if op == "embedding":
        return O.embedding(x, xs[1])
    if op == "gatherRows":
        return O.gather_rows(x, xs[1])
    if op == "rope":
        return O.rope(x, a["base"])
    if op == "sdpa":
        return O.sdpa(x, xs[1], xs[2], xs[3], a["scale"])
    if op == "reshape":
        return O.reshape(x, a["shape"])
    if op == "transpose":
        return O.transpose(x, a["perm"])
    if op == "slice":
        return O.slice_(x, a["begin"], a["end"])
    if op == "split":
        return O.split(x, a["parts"], a["axis"])
    if op == "concat":
        return O.concat(xs, a["axis"])
    if op == "cast":
        return O.cast(x, a["dtype"])
    if op == "meanPool":
        return O.mean_pool(x, xs[1])
    if op == "quantizedLinear":
        q, s, b = xs[1], xs[2], xs[3]
        packed = O.pack_quantized(q, a["bits"])
        qq = O.unpack_quantized(packed, q.shape[0], q.shape[1], a["bits"], a["mode"])
        return O.quantized_linear(x, qq, s, b, a["groupSize"], xs[4])
    if op == "quantizedEmbedding":
        q, s, b, ids = xs
        packed = O.pack_quantized(q, a["bits"])
        qq = O.unpack_quantized(packed, q.shape[0], q.shape[1], a["bits"], a["mode"])
        return O.quantized_embedding(qq, s, b, a["groupSize"], ids)
    raise KeyError(op)


def close(got: np.ndarray, want: np.ndarray, atol: float, rtol: float) -> tuple[bool, str]:
    """conformance.ts:223-236 assertClose (NaN positions must agree)."""
    g = np.asarray(got, dtype=np.float64).reshape(-1)
    w = np.asarray(want, dtype=np.float64).reshape(-1)
    if g.shape != w.shape:
        return False, f"length {g.size} != {w.size}"
    if not np.array_equal(np.isnan(g), np.isnan(w)):
        return False, "NaN mismatch"
    ok = ~np.isnan(w)
    with np.errstate(invalid="ignore"):
        err = np.abs(g[ok] - w[ok]) - (atol + rtol * np.abs(w[ok]))
    if err.size and np.nanmax(err) > 0:
        i = int(np.nanargmax(err))
        return False, f"[{i}] got {g[ok][i]} want {w[ok][i]} (atol {atol}, rtol {rtol})"
    return True, ""
