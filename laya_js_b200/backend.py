"""``createCudaBackend()`` — the B200 backend of the laya-js tensor-backend
contract, over liblaya_cuda's C ABI.

This is the host-side mirror of the reference interface ``Backend<T>``
(packages/tensor-backend/src/index.ts:139-317): same method names, argument
meaning and error behaviour, so the parity tests read like the reference's
own conformance and backend tests. Each method is one C call
(``lc_<op>``), the way the reference's native backend makes one mlx-c call
per op (packages/backend-mlx/src/index.ts:150-848).

Differences forced by the host language, not by design:
  * ``fromHost`` / ``read`` return values instead of Promises;
  * HostTensor data is a numpy array (index.ts:47-60 TypedArrays).
"""
from __future__ import annotations

import ctypes as C
import weakref
from typing import Any, Callable, Optional, Sequence

import numpy as np

from . import _lib
from ._lib import LayaCudaError
from .host import CODE, DTYPES, FLOATS, NP_STORAGE, HostQuantized, HostTensor, quant_groups, validate_quantized

_MODE = {"symmetric": 0, "affine": 1}


class CudaTensor:
    """An opaque device tensor handle (index.ts:75-78 Tensor: shape + dtype)."""

    __slots__ = ("handle", "shape", "dtype", "disposed", "_backend", "__weakref__")

    def __init__(self, backend: "CudaBackend", handle: int):
        self._backend = backend
        self.handle = handle
        dt = C.c_int()
        nd = C.c_int()
        sh = (C.c_int64 * 8)()
        _lib.call("lc_tensor_info", C.c_uint64(handle), C.byref(dt), C.byref(nd), sh)
        self.shape = tuple(int(sh[i]) for i in range(nd.value))
        self.dtype = DTYPES[dt.value]
        self.disposed = False

    def __repr__(self) -> str:
        return f"CudaTensor({self.dtype}, {list(self.shape)}{', disposed' if self.disposed else ''})"


def _i64(seq: Sequence[int]):
    arr = (C.c_int64 * max(1, len(seq)))(*[int(v) for v in seq])
    return arr


class CudaBackend:
    """``Backend<CudaTensor>`` on one CUDA device (index.ts:139-317)."""

    name = "cuda"

    def __init__(self, device: int = 0):
        _lib.load()
        _lib.call("lc_init", int(device))
        self.device = device
        self._scopes: list[list[CudaTensor]] = []
        self._destroyed = False

    # ------------------------------------------------------------ plumbing
    def _wrap(self, h: int) -> CudaTensor:
        t = CudaTensor(self, h)
        if self._scopes:
            self._scopes[-1].append(t)
        return t

    def _h(self, t: Optional[CudaTensor], what: str = "tensor") -> int:
        if t is None:
            return 0
        if not isinstance(t, CudaTensor):
            raise TypeError(f"{what}: expected a CudaTensor, got {type(t).__name__}")
        if t.disposed:
            raise LayaCudaError(f"{what}: tensor used after dispose")
        return t.handle

    def _op(self, fn: str, *args) -> CudaTensor:
        out = C.c_uint64()
        _lib.call(fn, C.byref(out), *args)
        return self._wrap(out.value)

    def _t(self, t, what="tensor"):
        return C.c_uint64(self._h(t, what))

    # ------------------------------------------------------------ contract: lifetime
    def supports(self, dtype: str) -> bool:
        """index.ts:142-143: every contract dtype is stored natively."""
        return dtype in CODE

    def fromHost(self, t: HostTensor) -> CudaTensor:
        """index.ts:146-154: copies at call time (the caller may reuse t.data on return)."""
        if t.dtype not in CODE:
            raise TypeError(f"fromHost: unknown dtype {t.dtype}")
        arr = np.ascontiguousarray(np.asarray(t.data).astype(NP_STORAGE[t.dtype], copy=False))
        shape = tuple(int(d) for d in t.shape)
        return self._op("lc_from_host", CODE[t.dtype], _i64(shape), len(shape), arr.ctypes.data_as(C.c_void_p),
                        C.c_size_t(arr.nbytes))

    def read(self, t: CudaTensor) -> HostTensor:
        """index.ts:155-156: materialises and copies to the host."""
        h = self._h(t, "read")
        out = np.empty(t.shape, NP_STORAGE[t.dtype])
        _lib.call("lc_read", C.c_uint64(h), out.ctypes.data_as(C.c_void_p), C.c_size_t(out.nbytes))
        return HostTensor(t.dtype, t.shape, out)

    def dispose(self, t: CudaTensor) -> None:
        """index.ts:157-158: idempotent."""
        if t is None or t.disposed:
            return
        t.disposed = True
        if not self._destroyed:
            _lib.call("lc_tensor_free", C.c_uint64(t.handle))

    def scope(self, fn: Callable[[], Any]) -> Any:
        """index.ts:159-163: tensors created in fn and not returned (directly, or
        in a returned list/tuple/dict one level deep) are disposed; returned ones
        move to the enclosing scope. A raising fn frees everything it made."""
        frame: list[CudaTensor] = []
        self._scopes.append(frame)
        try:
            r = fn()
        except BaseException:
            self._scopes.pop()
            for t in frame:
                self.dispose(t)
            raise
        self._scopes.pop()
        keep = set()
        if isinstance(r, CudaTensor):
            keep.add(id(r))
        elif isinstance(r, (list, tuple)):
            keep.update(id(x) for x in r if isinstance(x, CudaTensor))
        elif isinstance(r, dict):
            keep.update(id(x) for x in r.values() if isinstance(x, CudaTensor))
        for t in frame:
            if id(t) in keep:
                if self._scopes:
                    self._scopes[-1].append(t)
            else:
                self.dispose(t)
        return r

    def flush(self, *ts: CudaTensor) -> None:
        """index.ts:163-164."""
        _lib.call("lc_flush")

    def destroy(self) -> None:
        """index.ts:165-166."""
        if not self._destroyed:
            _lib.call("lc_destroy")
            self._destroyed = True

    def stats(self) -> dict:
        """Live tensors / bytes and kernel launches issued (tracing counters)."""
        a, b, c = C.c_int64(), C.c_int64(), C.c_int64()
        _lib.call("lc_stats", C.byref(a), C.byref(b), C.byref(c))
        return {"live_tensors": a.value, "live_bytes": b.value, "launches": c.value}

    # ------------------------------------------------------------ shape
    def reshape(self, x, shape):
        return self._op("lc_reshape", self._t(x, "reshape"), _i64(shape), len(shape))

    def transpose(self, x, perm):
        p = (C.c_int32 * max(1, len(perm)))(*perm)
        return self._op("lc_transpose", self._t(x, "transpose"), p, len(perm))

    def slice(self, x, begin, end):
        return self._op("lc_slice", self._t(x, "slice"), _i64(begin), _i64(end), len(begin))

    def split(self, x, parts: int, axis: int):
        outs = (C.c_uint64 * parts)()
        _lib.call("lc_split", outs, self._t(x, "split"), int(parts), int(axis))
        return [self._wrap(outs[i]) for i in range(parts)]

    def concat(self, xs, axis: int):
        hs = (C.c_uint64 * len(xs))(*[self._h(x, "concat") for x in xs])
        return self._op("lc_concat", hs, len(xs), int(axis))

    def cast(self, x, dtype: str):
        return self._op("lc_cast", self._t(x, "cast"), CODE[dtype])

    # ------------------------------------------------------------ elementwise
    def add(self, a, b): return self._op("lc_add", self._t(a), self._t(b))
    def sub(self, a, b): return self._op("lc_sub", self._t(a), self._t(b))
    def mul(self, a, b): return self._op("lc_mul", self._t(a), self._t(b))
    def div(self, a, b): return self._op("lc_div", self._t(a), self._t(b))
    def maximum(self, a, b): return self._op("lc_maximum", self._t(a), self._t(b))
    def where(self, c, a, b): return self._op("lc_where", self._t(c), self._t(a), self._t(b))
    def scale(self, x, s: float): return self._op("lc_scale", self._t(x), C.c_double(s))
    def exp(self, x): return self._op("lc_exp", self._t(x))
    def log(self, x): return self._op("lc_log", self._t(x))
    def relu(self, x): return self._op("lc_relu", self._t(x))
    def gelu(self, x): return self._op("lc_gelu", self._t(x))

    # ------------------------------------------------------------ reductions
    def sum(self, x, axis: int, keepDims: bool = False): return self._op("lc_sum", self._t(x), int(axis), int(bool(keepDims)))
    def max(self, x, axis: int, keepDims: bool = False): return self._op("lc_max", self._t(x), int(axis), int(bool(keepDims)))
    def softmax(self, x, axis: int): return self._op("lc_softmax", self._t(x), int(axis))
    def sort(self, x, axis: int): return self._op("lc_sort", self._t(x), int(axis))

    # ------------------------------------------------------------ linear algebra & NN
    def matmul(self, a, b): return self._op("lc_matmul", self._t(a), self._t(b))

    def linear(self, x, w, b=None):
        return self._op("lc_linear", self._t(x, "linear"), self._t(w, "linear"), self._t(b, "linear"))

    def layerNorm(self, x, weight, bias, eps: float):
        return self._op("lc_layer_norm", self._t(x), self._t(weight), self._t(bias), C.c_double(eps))

    def embedding(self, table, ids): return self._op("lc_embedding", self._t(table), self._t(ids))
    def gatherRows(self, x, idx): return self._op("lc_gather_rows", self._t(x), self._t(idx))
    def rope(self, x, base: float): return self._op("lc_rope", self._t(x), C.c_double(base))

    def sdpa(self, q, k, v, mask, scale: float):
        return self._op("lc_sdpa", self._t(q), self._t(k), self._t(v), self._t(mask), C.c_double(scale))

    # ------------------------------------------------------------ optional fused
    def geglu(self, x): return self._op("lc_geglu", self._t(x))
    def meanPool(self, x, mask): return self._op("lc_mean_pool", self._t(x), self._t(mask))

    # ------------------------------------------------------------ optional quantized trio
    def fromHostQuantized(self, h: HostQuantized, dtype: str):
        """index.ts:250-255: keeps the laya-js packed bytes as the native layout."""
        validate_quantized(h)
        if dtype not in ("f32", "f16", "bf16"):
            return None
        N, K = h.shape
        data = np.ascontiguousarray(np.asarray(h.data, np.uint8))
        s = np.ascontiguousarray(np.asarray(h.scales.data).astype(NP_STORAGE[h.scales.dtype], copy=False))
        b = None if h.biases is None else np.ascontiguousarray(np.asarray(h.biases.data).astype(NP_STORAGE[h.biases.dtype], copy=False))
        if b is not None and h.biases.dtype != h.scales.dtype:
            raise TypeError("fromHostQuantized: scales and biases must share a dtype")
        w, sc, bi = C.c_uint64(), C.c_uint64(), C.c_uint64()
        _lib.call("lc_from_host_quantized", C.byref(w), C.byref(sc), C.byref(bi), C.c_int64(N), C.c_int64(K), int(h.bits),
                  int(h.groupSize), _MODE[h.mode], data.ctypes.data_as(C.c_void_p), CODE[h.scales.dtype],
                  s.ctypes.data_as(C.c_void_p), None if b is None else b.ctypes.data_as(C.c_void_p), CODE[dtype])
        from .compose import QuantizedTensor
        return QuantizedTensor(shape=(N, K), bits=h.bits, groupSize=h.groupSize, mode=h.mode, dtype=dtype, native=True,
                               w=self._wrap(w.value), scales=self._wrap(sc.value),
                               biases=self._wrap(bi.value) if bi.value else None)

    def quantizedLinear(self, x, w, scales, biases, opts, bias=None):
        """index.ts:256-259."""
        return self._op("lc_quantized_linear", self._t(x), self._t(w), self._t(scales), self._t(biases), int(opts.bits),
                        int(opts.groupSize), _MODE[opts.mode], self._t(bias))

    def quantizedEmbedding(self, w, scales, biases, opts, ids):
        """index.ts:260-262."""
        return self._op("lc_quantized_embedding", self._t(w), self._t(scales), self._t(biases), int(opts.bits),
                        int(opts.groupSize), _MODE[opts.mode], self._t(ids))

    # ------------------------------------------------------------ optional: compile
    def compile(self, fn: Callable[..., Any]) -> Callable[..., Any]:
        """index.ts:244-245 compile: ``fn`` (a pure function of its tensor
        arguments; tensors it captures from outside are constants, as under
        MLX's compile, packages/backend-mlx/src/index.ts:773-781) is run
        eagerly on the first call of each input signature (dtypes and shapes)
        and recorded as a CUDA graph on that call's tensors; later calls with
        the same signature copy their arguments into the recorded inputs,
        replay the graph in one launch and return fresh copies of its outputs.
        Outputs may be a tensor, a list/tuple of tensors or a dict of tensors."""
        return _Compiled(self, fn)

    # ------------------------------------------------------------ optional general numerics
    def equal(self, a, b): return self._op("lc_equal", self._t(a), self._t(b))
    def notEqual(self, a, b): return self._op("lc_not_equal", self._t(a), self._t(b))
    def less(self, a, b): return self._op("lc_less", self._t(a), self._t(b))
    def lessEqual(self, a, b): return self._op("lc_less_equal", self._t(a), self._t(b))
    def greater(self, a, b): return self._op("lc_greater", self._t(a), self._t(b))
    def greaterEqual(self, a, b): return self._op("lc_greater_equal", self._t(a), self._t(b))
    def logicalAnd(self, a, b): return self._op("lc_logical_and", self._t(a), self._t(b))
    def logicalOr(self, a, b): return self._op("lc_logical_or", self._t(a), self._t(b))
    def logicalNot(self, x): return self._op("lc_logical_not", self._t(x))
    def sqrt(self, x): return self._op("lc_sqrt", self._t(x))
    def rsqrt(self, x): return self._op("lc_rsqrt", self._t(x))
    def pow(self, a, b): return self._op("lc_pow", self._t(a), self._t(b))
    def neg(self, x): return self._op("lc_neg", self._t(x))
    def abs(self, x): return self._op("lc_abs", self._t(x))
    def tanh(self, x): return self._op("lc_tanh", self._t(x))
    def sigmoid(self, x): return self._op("lc_sigmoid", self._t(x))
    def erf(self, x): return self._op("lc_erf", self._t(x))
    def argmax(self, x, axis, keepDims=False): return self._op("lc_argmax", self._t(x), int(axis), int(bool(keepDims)))
    def argmin(self, x, axis, keepDims=False): return self._op("lc_argmin", self._t(x), int(axis), int(bool(keepDims)))
    def mean(self, x, axis, keepDims=False): return self._op("lc_mean", self._t(x), int(axis), int(bool(keepDims)))
    def min(self, x, axis, keepDims=False): return self._op("lc_min", self._t(x), int(axis), int(bool(keepDims)))
    def cumsum(self, x, axis): return self._op("lc_cumsum", self._t(x), int(axis))


def _flatten(r):
    """(flat tensor list, rebuild(list) -> same structure) of a compiled fn's result."""
    if isinstance(r, CudaTensor):
        return [r], lambda xs: xs[0]
    if isinstance(r, (list, tuple)):
        if not all(isinstance(x, CudaTensor) for x in r):
            raise TypeError("compile: outputs must be tensors (a tensor, a list/tuple or a dict of tensors)")
        kind = type(r)
        return list(r), lambda xs: kind(xs)
    if isinstance(r, dict):
        keys = list(r)
        if not all(isinstance(r[k], CudaTensor) for k in keys):
            raise TypeError("compile: outputs must be tensors (a tensor, a list/tuple or a dict of tensors)")
        return [r[k] for k in keys], lambda xs: dict(zip(keys, xs))
    raise TypeError("compile: outputs must be tensors (a tensor, a list/tuple or a dict of tensors)")


class _Graph:
    """One recorded signature: input and output tensors owned by the graph."""

    def __init__(self, b: "CudaBackend", handle: int, ins: list, outs: list, rebuild):
        self.b, self.handle, self.ins, self.outs, self.rebuild = b, handle, ins, outs, rebuild
        self._fin = weakref.finalize(self, _Graph._release, b, handle, ins + outs)

    @staticmethod
    def _release(b, handle, ts):
        if b._destroyed:
            return
        try:
            _lib.call("lc_graph_destroy", C.c_uint64(handle))
        finally:
            for t in ts:
                b.dispose(t)

    def run(self, args):
        b = self.b
        for slot, a in zip(self.ins, args):
            _lib.call("lc_copy_into", C.c_uint64(slot.handle), C.c_uint64(b._h(a, "compiled call")))
        _lib.call("lc_graph_launch", C.c_uint64(self.handle))
        return self.rebuild([b.cast(o, o.dtype) for o in self.outs])


class _Compiled:
    """The function ``Backend.compile`` returns (CUDA graph per input signature)."""

    def __init__(self, b: "CudaBackend", fn: Callable[..., Any]):
        self.b, self.fn = b, fn
        self.graphs: dict[tuple, _Graph] = {}

    def __call__(self, *args):
        b = self.b
        sig = tuple((a.dtype, tuple(a.shape)) if isinstance(a, CudaTensor) else ("?", type(a).__name__) for a in args)
        if not all(isinstance(a, CudaTensor) for a in args):
            raise TypeError("compile: arguments must be tensors")
        g = self.graphs.get(sig)
        if g is not None:
            return g.run(args)
        result = self.fn(*args)  # the first call of a signature runs eagerly
        self.graphs[sig] = self._record(args, result)
        return result

    def _record(self, args, result) -> _Graph:
        b = self.b
        flat, rebuild = _flatten(result)
        zeros = lambda dt, sh: b.fromHost(HostTensor(dt, tuple(sh), np.zeros(tuple(sh), NP_STORAGE[dt])))
        saved, b._scopes = b._scopes, []  # the graph's tensors belong to no caller scope
        try:
            ins = [zeros(a.dtype, a.shape) for a in args]
            outs = [zeros(t.dtype, t.shape) for t in flat]
            _lib.call("lc_graph_capture_begin")
            try:
                def body():
                    views = [b.reshape(t, list(t.shape)) for t in ins]  # fn may dispose its arguments
                    got, _ = _flatten(self.fn(*views))
                    if [(t.dtype, tuple(t.shape)) for t in got] != [(t.dtype, tuple(t.shape)) for t in outs]:
                        raise ValueError("compile: fn returned different outputs for the same input signature")
                    for o, t in zip(outs, got):
                        _lib.call("lc_copy_into", C.c_uint64(o.handle), C.c_uint64(t.handle))
                    return None
                b.scope(body)
                h = C.c_uint64()
                _lib.call("lc_graph_capture_end", C.byref(h))
            except BaseException:
                _lib.call("lc_graph_capture_abort")
                for t in ins + outs:
                    b.dispose(t)
                raise
        finally:
            b._scopes = saved
        return _Graph(b, h.value, ins, outs, rebuild)


_BACKENDS: dict[int, CudaBackend] = {}


def createCudaBackend(device: int = 0) -> CudaBackend:
    """The backend factory (cf. createMlxBackend, packages/backend-mlx/src/index.ts:150).
    One library state per process and device."""
    b = _BACKENDS.get(device)
    if b is None or b._destroyed:
        b = CudaBackend(device)
        _BACKENDS[device] = b
    return b
