"""Laya quantized checkpoints (format version 1) straight onto the device —
the host-side mirror of the reference's reader:

- ``quant_metadata``     packages/laya/src/quant.ts:65-80 (``__metadata__``:
                         ``laya_quant`` q8 | q4, ``version`` "1", ``group_size``)
- ``group_quantized``    packages/laya/src/quant.ts:375-403 (a matrix ``W`` plus its
                         ``W.scales`` / ``W.biases`` companions; I8 = q8, U8 = q4)
- ``host_quantized``     packages/laya/src/weights.ts:71-82 (q8 → 8-bit symmetric,
                         q4 → 4-bit affine, f16 scales and biases, zero copies)
- ``read_weights``       packages/laya/src/weights.ts:95-175 (``readWeights`` with
                         ``quantized="device"``: quantized matrices are handed out
                         as ``HostQuantized``, so ``loadModernBert`` / ``loadDecisionModel``
                         keep them packed on the backend through ``fromHostQuantized``)

The file layout (docs/QUANTIZATION.md:91-117): a safetensors file whose
quantized matrices are ``I8 [rows, cols]`` (q8, q in [-127, 127], w = q·scale) or
``U8 [rows, cols/2]`` (q4: column 2k in the low nibble, 2k+1 in the high one,
w = q·scale + bias), with ``F16 [rows, cols/g]`` scales (and biases). The
packed bytes are exactly the backend's native layout, so nothing is repacked.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Callable, Optional

import numpy as np

from .host import HostQuantized, HostTensor

QUANT_FORMAT_VERSION = "1"

# safetensors dtype -> contract dtype (packages/laya/src/weights.ts DTYPES)
_DTYPES = {"F32": "f32", "F16": "f16", "BF16": "bf16", "I32": "i32", "I64": "i64", "U8": "u8", "I8": "i8", "BOOL": "bool",
           "F64": "f64", "I16": "i16", "U16": "u16", "U32": "u32", "U64": "u64"}


@dataclass
class QuantizedMatrix:
    """quant.ts QuantizedMatrix: packed values, f16 scales (+ biases) per group."""
    bits: int
    rows: int
    cols: int
    data: np.ndarray  # int8 [rows, cols] (q8) or uint8 [rows, cols / 2] (q4)
    scales: np.ndarray  # float16 [rows, G]
    biases: Optional[np.ndarray]
    groupSize: int


@dataclass
class RawTensor:
    dtype: str  # safetensors dtype name
    shape: tuple
    data: np.ndarray


def quant_metadata(metadata: Optional[dict]) -> Optional[dict]:
    """quant.ts:65-80: the checkpoint's scheme, or None for a float checkpoint;
    raises on an unknown scheme or another format version."""
    scheme = (metadata or {}).get("laya_quant")
    if scheme is None:
        return None
    if scheme not in ("q8", "q4"):
        raise ValueError(f"laya: unknown quantization scheme laya_quant={scheme!r} (expected \"q8\" or \"q4\")")
    version = metadata.get("version", "")
    if version != QUANT_FORMAT_VERSION:
        raise ValueError(f"laya: quantized checkpoint format version {version!r} is not supported "
                         f"(this reader reads version {QUANT_FORMAT_VERSION})")
    g = metadata.get("group_size")
    group = None if g is None or g == "row" else g
    if group is not None:
        try:
            group = int(group)
        except ValueError:
            group = -1
        if group <= 0:
            raise ValueError(f"laya: invalid group_size {g!r} in quantized checkpoint")
    return {"scheme": scheme, "bits": 8 if scheme == "q8" else 4, "groupSize": group, "version": version,
            "sourceDtype": metadata.get("laya_quant_source_dtype")}


def group_quantized(tensors: dict) -> tuple[dict, dict]:
    """quant.ts:375-403: (name -> QuantizedMatrix, name -> RawTensor of plain tensors)."""
    quantized: dict = {}
    companion: set = set()
    for name, t in tensors.items():
        scales = tensors.get(name + ".scales")
        if scales is None:
            continue
        where = f"laya: quantized tensor {name}"
        if scales.dtype != "F16" or len(scales.shape) != 2:
            raise ValueError(f"{where}: .scales must be F16 [rows, groups]")
        rows, G = scales.shape
        biases = None
        if t.dtype == "I8":
            bits, cols = 8, t.shape[1]
        elif t.dtype == "U8":
            bits, cols = 4, 2 * t.shape[1]
            b = tensors.get(name + ".biases")
            if b is None or b.dtype != "F16" or tuple(b.shape) != (rows, G):
                raise ValueError(f"{where}: q4 needs .biases F16 [{rows}, {G}]")
            biases = b.data
            companion.add(name + ".biases")
        else:
            raise ValueError(f"{where}: dtype {t.dtype} is not a quantized dtype (I8 or U8)")
        if len(t.shape) != 2 or t.shape[0] != rows or cols % G:
            raise ValueError(f"{where}: shape {list(t.shape)} does not match .scales {list(scales.shape)}")
        companion.add(name + ".scales")
        quantized[name] = QuantizedMatrix(bits, rows, cols, t.data, scales.data, biases, cols // G)
    plain = {n: t for n, t in tensors.items() if n not in quantized and n not in companion}
    return quantized, plain


def host_quantized(m: QuantizedMatrix) -> HostQuantized:
    """weights.ts:71-82."""
    G = m.cols // m.groupSize
    return HostQuantized((m.rows, m.cols), m.bits, m.groupSize, "symmetric" if m.bits == 8 else "affine",
                         np.ascontiguousarray(m.data).view(np.uint8).reshape(-1), HostTensor("f16", (m.rows, G), m.scales),
                         HostTensor("f16", (m.rows, G), m.biases) if m.biases is not None else None)


def sanitize_name(name: str) -> str:
    """weights.ts:16-22."""
    n = name.replace(".in_proj_weight", ".in_proj.weight").replace(".in_proj_bias", ".in_proj.bias")
    for prefix in ("scorer", "act_head"):
        if n.startswith(prefix + ".") and not n.startswith(prefix + ".layers."):
            n = prefix + ".layers." + n[len(prefix) + 1:]
    return n


def read_raw(path: str) -> tuple[dict, dict]:
    """(name -> RawTensor, __metadata__) of a safetensors file."""
    from safetensors import safe_open
    out = {}
    with safe_open(path, framework="numpy") as f:
        meta = f.metadata() or {}
        for name in f.keys():
            a = f.get_tensor(name)
            sl = f.get_slice(name)
            out[name] = RawTensor(sl.get_dtype(), tuple(a.shape), a)
    return out, meta


def read_weights(path: str, quantized: str = "device") -> Callable[[str], object]:
    """weights.ts readWeights / dequantizingWeights(keepQuantized): a consuming
    WeightGetter (each tensor is handed out once). Quantized matrices come out
    as HostQuantized when ``quantized == "device"``; a float checkpoint's
    tensors as HostTensor."""
    if quantized not in ("device", "dequantize"):
        raise ValueError('quantized must be "device" or "dequantize"')
    raw, meta = read_raw(path)
    q: dict = {}
    plain = raw
    if quant_metadata(meta) is not None:
        qm, plain = group_quantized(raw)
        for name, m in qm.items():
            key = sanitize_name(name)
            if key in q:
                raise ValueError(f"Duplicate checkpoint parameter after conversion: {key}")
            q[key] = m
    hosts = {}
    for name, t in plain.items():
        d = _DTYPES.get(t.dtype)
        if d is None:
            raise TypeError(f"laya: unsupported safetensors dtype {t.dtype} for {name}")
        key = sanitize_name(name)
        if key in hosts or key in q:
            raise ValueError(f"Duplicate checkpoint parameter after conversion: {key}")
        hosts[key] = HostTensor(d, tuple(t.shape), t.data)

    def get(name: str):
        if name in q:
            m = q.pop(name)
            if quantized == "device":
                return host_quantized(m)
            return HostTensor("f16", (m.rows, m.cols), dequantize_matrix(m))
        return hosts.pop(name, None)
    get.remaining = lambda: [*q.keys(), *hosts.keys()]  # type: ignore[attr-defined]
    return get


def dequantize_matrix(m: QuantizedMatrix) -> np.ndarray:
    """quant.ts:199-241 with dtype f16: q·s (q8) or q·s + b (q4) rounded once to f16."""
    G = m.cols // m.groupSize
    s = np.repeat(m.scales.astype(np.float64).reshape(m.rows, G), m.groupSize, axis=1)
    if m.bits == 8:
        return (m.data.astype(np.int8).astype(np.float64) * s).astype(np.float16)
    d = m.data.astype(np.uint8).reshape(m.rows, m.cols // 2)
    qv = np.empty((m.rows, m.cols), np.float64)
    qv[:, 0::2] = d & 15
    qv[:, 1::2] = d >> 4
    b = np.repeat(m.biases.astype(np.float64).reshape(m.rows, G), m.groupSize, axis=1)
    return (qv * s + b).astype(np.float16)
