"""ctypes wrapper of the C++ CPU restatement (oracle/cpu_encoder.cpp) — TEST
INFRASTRUCTURE and the timed CPU baseline only.

``build()`` compiles ``liboracle_cpu.so`` next to the source (g++, std::thread,
AVX2/FMA code that any x86-64 server of the last decade runs); ``Encoder``
runs the ModernBERT encoder + CLS head over packed unpadded sequences with a
given thread count; ``linear`` / ``layer_norm`` / ``rope`` / ``sdpa`` /
``geglu`` expose single ops so the tests can pin this file to the reference's
golden vectors, as oracle/ops.py is pinned.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
SRC = HERE / "cpu_encoder.cpp"
LIB = HERE / "liboracle_cpu.so"
CXX = os.environ.get("CXX", "g++")
FLAGS = ["-O3", "-std=c++17", "-pthread", "-mavx2", "-mfma", "-fPIC", "-shared"]

_lib = None


def build(force: bool = False) -> Path:
    if force or not LIB.exists() or LIB.stat().st_mtime < SRC.stat().st_mtime:
        tmp = LIB.with_suffix(".so.tmp")
        r = subprocess.run([CXX, *FLAGS, str(SRC), "-o", str(tmp)], capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"building {SRC.name} failed:\n{r.stderr}")
        os.replace(tmp, LIB)
    return LIB


def lib():
    global _lib
    if _lib is None:
        if not LIB.exists():
            build()
        L = C.CDLL(str(LIB))
        P, I64, F = C.c_void_p, C.c_int64, C.POINTER(C.c_float)
        L.oc_encoder_create.restype = P
        L.oc_encoder_create.argtypes = [C.POINTER(C.c_int32), C.POINTER(C.c_double), C.POINTER(P), C.c_int]
        L.oc_encoder_free.argtypes = [P]
        L.oc_encoder_forward.restype = C.c_double
        L.oc_encoder_forward.argtypes = [P, C.POINTER(C.c_int32), C.POINTER(C.c_int32), C.c_int, P, P, C.c_int, P, P, C.c_int]
        L.oc_linear.argtypes = [P, I64, I64, P, I64, P, P, C.c_int]
        L.oc_layer_norm.argtypes = [P, I64, I64, P, P, C.c_double, P]
        L.oc_rope.argtypes = [P, I64, I64, I64, C.c_double, P]
        L.oc_sdpa.argtypes = [P, P, P, P, I64, I64, I64, I64, I64, C.c_double, P]
        L.oc_geglu.argtypes = [P, I64, I64, P]
        del F
        _lib = L
    return _lib


def _f32(a):
    return np.ascontiguousarray(a, np.float32)


def _p(a):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


class Encoder:
    """The ModernBERT encoder of a config json (workloads.BASE / LARGE shape) over a weight dict."""

    def __init__(self, cfg: dict, W: dict, prefix: str = "encoder."):
        n = cfg["num_hidden_layers"]
        names = [prefix + "embeddings.tok_embeddings.weight", prefix + "embeddings.norm.weight"]
        for i in range(n):
            p = f"{prefix}layers.{i}."
            names += [p + "attn_norm.weight" if i else None, p + "attn.Wqkv.weight", p + "attn.Wo.weight", p + "mlp_norm.weight",
                      p + "mlp.Wi.weight", p + "mlp.Wo.weight"]
        names.append(prefix + "final_norm.weight")
        self._keep = [None if k is None else _f32(W[k]) for k in names]
        ptrs = (C.c_void_p * len(names))(*[None if a is None else a.ctypes.data for a in self._keep])
        icfg = (C.c_int32 * 7)(cfg["vocab_size"], cfg["hidden_size"], cfg["intermediate_size"], n, cfg["num_attention_heads"],
                               cfg.get("local_attention", 128), cfg.get("global_attn_every_n_layers", 3))
        dcfg = (C.c_double * 3)(cfg.get("norm_eps", 1e-5), cfg.get("global_rope_theta", 160000.0), cfg.get("local_rope_theta", 10000.0))
        self.H = cfg["hidden_size"]
        self.h = lib().oc_encoder_create(icfg, dcfg, ptrs, len(names))
        self._keep = None  # weights are packed into the encoder
        if not self.h:
            raise ValueError("oc_encoder_create rejected the weights")

    def _run(self, seqs, hw, hb, threads, want_hidden):
        ids = np.ascontiguousarray(np.concatenate(seqs), np.int32)
        cu = np.concatenate([[0], np.cumsum([len(s) for s in seqs])]).astype(np.int32)
        hw32 = None if hw is None else _f32(hw)
        hb32 = None if hb is None else _f32(hb)
        ncls = 0 if hw is None else hw32.shape[0]
        probs = np.empty((len(seqs), max(ncls, 1)), np.float32)
        hidden = np.empty((int(cu[-1]), self.H), np.float32) if want_hidden else None
        dt = lib().oc_encoder_forward(self.h, ids.ctypes.data_as(C.POINTER(C.c_int32)), cu.ctypes.data_as(C.POINTER(C.c_int32)),
                                      len(seqs), _p(hw32), _p(hb32), ncls, _p(probs), _p(hidden), int(threads))
        return dt, probs, hidden, cu

    def forward(self, seqs, hw=None, hb=None, threads: int = 0, want_hidden: bool = True):
        """(hidden [T, H] packed, probs [nseq, C], cu_seqlens)."""
        _, probs, hidden, cu = self._run(seqs, hw, hb, threads or os.cpu_count(), want_hidden)
        return hidden, probs, cu

    def timed_forward(self, seqs, hw, hb, threads: int) -> float:
        """Seconds of one forward (ids -> probabilities), measured inside the library."""
        return self._run(seqs, hw, hb, threads, False)[0]

    def __del__(self):
        if getattr(self, "h", None) and _lib is not None:
            _lib.oc_encoder_free(self.h)
            self.h = None


def linear(x, w, b=None, threads: int = 1):
    x, w = _f32(x), _f32(w)
    K = x.shape[-1]
    M = x.size // K
    N = w.shape[0]
    b32 = None if b is None else _f32(b)
    y = np.empty(x.shape[:-1] + (N,), np.float32)
    lib().oc_linear(_p(x), M, K, _p(w), N, _p(b32), _p(y), threads)
    return y


def layer_norm(x, w, b, eps):
    x = _f32(x)
    H = x.shape[-1]
    y = np.empty_like(x)
    lib().oc_layer_norm(_p(x), x.size // H, H, _p(None if w is None else _f32(w)), _p(None if b is None else _f32(b)), float(eps), _p(y))
    return y


def rope(x, base):
    x = _f32(x)
    L, D = x.shape[-2], x.shape[-1]
    y = np.empty_like(x)
    lib().oc_rope(_p(x), x.size // (L * D), L, D, float(base), _p(y))
    return y


def sdpa(q, k, v, mask, scale):
    q, k, v = _f32(q), _f32(k), _f32(v)
    lead = np.broadcast_shapes(q.shape[:-2], k.shape[:-2], v.shape[:-2])
    Lq, Lk, D, Dv = q.shape[-2], k.shape[-2], q.shape[-1], v.shape[-1]
    q = np.ascontiguousarray(np.broadcast_to(q, lead + (Lq, D)))
    k = np.ascontiguousarray(np.broadcast_to(k, lead + (Lk, D)))
    v = np.ascontiguousarray(np.broadcast_to(v, lead + (Lk, Dv)))
    m = None
    if mask is not None:
        m = np.ascontiguousarray(np.broadcast_to(mask.astype(bool), lead + (Lq, Lk)), np.uint8)
    BH = int(np.prod(lead)) if lead else 1
    out = np.empty(lead + (Lq, Dv), np.float32)
    lib().oc_sdpa(_p(q), _p(k), _p(v), _p(m), BH, Lq, Lk, D, Dv, float(scale), _p(out))
    return out


def geglu(x):
    x = _f32(x)
    F = x.shape[-1] // 2
    y = np.empty(x.shape[:-1] + (F,), np.float32)
    lib().oc_geglu(_p(x), x.size // (2 * F), F, _p(y))
    return y
