"""The fused varlen ModernBERT encoder (include/laya_cuda_encoder.h) over
weights loaded through the contract path (``loadModernBert``).

``FusedEncoder.forward`` is ModernBert.encode (packages/modernbert/src/index.ts:407-429)
on packed sequences plus the CLS classifier head; ``forward_host`` is the
end-to-end call with host buffers (H2D of ids, D2H of probabilities).
"""
from __future__ import annotations

import ctypes as C
from typing import Optional

import numpy as np

from . import _lib
from . import compose as Cm
from .host import CODE


class lc_encoder_config(C.Structure):
    _fields_ = [("vocab_size", C.c_int32), ("hidden_size", C.c_int32), ("intermediate_size", C.c_int32),
                ("num_layers", C.c_int32), ("num_heads", C.c_int32), ("local_attention", C.c_int32),
                ("dtype", C.c_int32), ("quant_bits", C.c_int32), ("quant_group", C.c_int32), ("quant_mode", C.c_int32),
                ("norm_eps", C.c_double), ("rope_theta_global", C.c_double), ("rope_theta_local", C.c_double)]


class FusedEncoder:
    """Built from a ``ModernBert`` whose weights live on a CUDA backend."""

    def __init__(self, model):
        b, c, w = model.backend, model.config, model.weights
        if c["attentionBias"] or c["mlpBias"] or c["normBias"]:
            raise ValueError("FusedEncoder: biases are not supported on the fused path (use ModernBert.forward)")
        if Cm.is_quantized(w.tokEmbeddings):
            raise ValueError("FusedEncoder: the token embedding must be a dense table")
        mats = [w.layers[0].Wqkv, w.layers[0].Wo, w.layers[0].Wi, w.layers[0].WoMlp]
        quant = Cm.is_quantized(mats[0])
        handles: list[int] = [b._h(w.tokEmbeddings), b._h(w.embNorm[0])]
        qb = qg = qm = 0
        for i, L in enumerate(w.layers):
            handles.append(b._h(L.attnNorm[0]) if L.attnNorm else 0)
            for m in (L.Wqkv, L.Wo):
                handles.extend(self._mat(b, m, quant))
            handles.append(b._h(L.mlpNorm[0]))
            for m in (L.Wi, L.WoMlp):
                handles.extend(self._mat(b, m, quant))
            if quant:
                qb, qg, qm = m.bits, m.groupSize, 0 if m.mode == "symmetric" else 1
        handles.append(b._h(w.finalNorm[0]))
        cfg = lc_encoder_config(c["vocabSize"], c["hiddenSize"], c["intermediateSize"], c["numHiddenLayers"],
                                c["numAttentionHeads"], c["localAttention"], CODE[model.dtype], qb, qg, qm, c["normEps"],
                                c["ropeBase"]["full_attention"], c["ropeBase"]["sliding_attention"])
        kinds = (C.c_int32 * len(w.layers))(*[0 if L.kind == "full_attention" else 1 for L in w.layers])
        arr = (C.c_uint64 * len(handles))(*handles)
        h = C.c_uint64()
        _lib.call("lc_encoder_create", C.byref(h), C.byref(cfg), kinds, arr, len(handles))
        self.handle = h.value
        self.backend = b
        self.config = c
        self.dtype = model.dtype

    @staticmethod
    def _mat(b, m, quant):
        if quant != Cm.is_quantized(m):
            raise ValueError("FusedEncoder: every Linear weight must be quantized, or none")
        if not quant:
            return [b._h(m)]
        if not m.native:
            raise ValueError("FusedEncoder: quantized weights must be in the backend's native layout")
        return [b._h(m.w), b._h(m.scales), b._h(m.biases) if m.biases is not None else 0]

    def forward(self, ids, cu_seqlens: np.ndarray, head_w=None, head_b=None, want_hidden: bool = True):
        """ids: device i32 [T]; cu_seqlens: host int32 [nseq + 1]. Returns (hidden [T, H] | None, probs [nseq, C] | None)."""
        b = self.backend
        cu = np.ascontiguousarray(cu_seqlens, np.int32)
        hid, pr = C.c_uint64(), C.c_uint64()
        _lib.call("lc_encoder_forward", C.byref(hid) if want_hidden else None, C.byref(pr) if head_w is not None else None,
                  C.c_uint64(self.handle), C.c_uint64(b._h(ids)), cu.ctypes.data_as(C.POINTER(C.c_int32)),
                  len(cu) - 1, C.c_uint64(b._h(head_w)), C.c_uint64(b._h(head_b)))
        return (b._wrap(hid.value) if want_hidden else None, b._wrap(pr.value) if head_w is not None else None)

    def forward_host(self, ids: np.ndarray, cu_seqlens: np.ndarray, head_w, head_b=None, out: Optional[np.ndarray] = None) -> np.ndarray:
        """End to end: host ids [T] -> host probabilities [nseq, C] (f32)."""
        ids = np.ascontiguousarray(ids, np.int32)
        cu = np.ascontiguousarray(cu_seqlens, np.int32)
        nseq = len(cu) - 1
        if out is None:
            out = np.empty((nseq, head_w.shape[0]), np.float32)
        _lib.call("lc_encoder_forward_host", C.c_uint64(self.handle), ids.ctypes.data_as(C.POINTER(C.c_int32)),
                  cu.ctypes.data_as(C.POINTER(C.c_int32)), nseq, C.c_uint64(self.backend._h(head_w)),
                  C.c_uint64(self.backend._h(head_b)), out.ctypes.data_as(C.POINTER(C.c_float)))
        return out

    def graph(self, cu_seqlens: np.ndarray, head_w, head_b=None) -> "EncoderGraph":
        """Capture forward_host for this fixed batch shape as a CUDA graph."""
        return EncoderGraph(self, cu_seqlens, head_w, head_b)

    def free(self) -> None:
        if self.handle:
            _lib.call("lc_encoder_free", C.c_uint64(self.handle))
            self.handle = 0


class EncoderGraph:
    """lc_encoder_graph_*: forward_host replayed as one CUDA graph launch for a
    fixed cu_seqlens and head; ``run(ids)`` -> probabilities [nseq, C] (f32)."""

    def __init__(self, fused: FusedEncoder, cu_seqlens: np.ndarray, head_w, head_b=None):
        cu = np.ascontiguousarray(cu_seqlens, np.int32)
        self.nseq, self.tokens, self.classes = len(cu) - 1, int(cu[-1]), int(head_w.shape[0])
        self.fused = fused
        h = C.c_uint64()
        _lib.call("lc_encoder_graph_create", C.byref(h), C.c_uint64(fused.handle), cu.ctypes.data_as(C.POINTER(C.c_int32)),
                  self.nseq, C.c_uint64(fused.backend._h(head_w)), C.c_uint64(fused.backend._h(head_b)))
        self.handle = h.value

    def run(self, ids: np.ndarray, out: Optional[np.ndarray] = None) -> np.ndarray:
        ids = np.ascontiguousarray(ids, np.int32)
        if ids.shape != (self.tokens,):
            raise ValueError(f"encoder graph: expected {self.tokens} ids, got shape {ids.shape}")
        if out is None:
            out = np.empty((self.nseq, self.classes), np.float32)
        _lib.call("lc_encoder_graph_run", C.c_uint64(self.handle), ids.ctypes.data_as(C.POINTER(C.c_int32)),
                  out.ctypes.data_as(C.POINTER(C.c_float)))
        return out

    def free(self) -> None:
        if self.handle and self.fused.handle:
            _lib.call("lc_encoder_graph_free", C.c_uint64(self.handle))
        self.handle = 0


def attention_varlen(backend, qkv, cu_seqlens: np.ndarray, half_window: int, scale: float, kernel: int = 0):
    """lc_attention_varlen: qkv [T, 3H] (RoPE applied) -> att [T, H]; kernel 0 tcgen05, 1 mma.sync."""
    cu = np.ascontiguousarray(cu_seqlens, np.int32)
    out = C.c_uint64()
    _lib.call("lc_attention_varlen", C.byref(out), C.c_uint64(backend._h(qkv)), cu.ctypes.data_as(C.POINTER(C.c_int32)),
              len(cu) - 1, int(half_window), C.c_double(scale), int(kernel))
    return backend._wrap(out.value)


def set_profiling(fused: FusedEncoder, on: bool) -> None:
    _lib.call("lc_encoder_set_profiling", C.c_uint64(fused.handle), int(bool(on)))


def profile_read(fused: FusedEncoder) -> dict:
    """Summed device ms and launch counts per kernel class since the last read."""
    ms = (C.c_double * 8)()
    n = (C.c_int64 * 8)()
    _lib.call("lc_encoder_profile_read", C.c_uint64(fused.handle), ms, n)
    names = ("gemm_qkv", "attention", "layernorm", "other", "gemm_o", "gemm_i", "gemm_mlp_o")
    out = {k: {"ms": ms[i], "launches": n[i]} for i, k in enumerate(names)}
    out["gemm"] = {"ms": sum(out[k]["ms"] for k in names if k.startswith("gemm")),
                   "launches": sum(out[k]["launches"] for k in names if k.startswith("gemm"))}
    return out
