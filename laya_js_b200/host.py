"""Host-side tensors and quantized-matrix helpers, mirroring
packages/tensor-backend/src/index.ts:39-137 (HostTensor, HostQuantized) and
packages/tensor-backend/src/host.ts (sizeOf, host, toF32, f32ToBf16Bits,
validateQuantized, unpackQuantized, packQuantized).

Host storage per dtype follows index.ts:47-60 with numpy arrays in place of
TypedArrays: f16 -> float16, bf16 -> uint16 raw bits, bool -> uint8 0/1.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional, Sequence

import numpy as np

DTYPES = ("f32", "f16", "bf16", "i32", "bool", "u8", "i8", "u16", "i16", "u32", "u64", "i64", "f64")
CODE = {d: i for i, d in enumerate(DTYPES)}
NP_STORAGE = {
    "f32": np.float32, "f16": np.float16, "bf16": np.uint16, "i32": np.int32, "bool": np.uint8, "u8": np.uint8,
    "i8": np.int8, "u16": np.uint16, "i16": np.int16, "u32": np.uint32, "u64": np.uint64, "i64": np.int64,
    "f64": np.float64,
}
FLOATS = ("f32", "f16", "bf16", "f64")


@dataclass(frozen=True)
class HostTensor:
    """index.ts:68-72."""
    dtype: str
    shape: tuple
    data: np.ndarray


@dataclass(frozen=True)
class HostQuantized:
    """index.ts:109-115: packed [out, in] matrix in the laya-js layout."""
    shape: tuple  # (N, K)
    bits: int
    groupSize: int
    mode: str  # "symmetric" | "affine"
    data: np.ndarray  # uint8, N*K*bits/8 bytes
    scales: HostTensor
    biases: Optional[HostTensor]


def size_of(shape: Sequence[int]) -> int:
    n = 1
    for d in shape:
        n *= int(d)
    return n


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """host.ts:71-76 round-to-nearest-even f32 -> bf16 bits (NaN -> 0x7fc0)."""
    u = np.asarray(x, np.float32).view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) & 0xFFFF
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    return np.where(nan, 0x7FC0, r).astype(np.uint16)


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, np.uint16).astype(np.uint32) << 16).view(np.float32)


def host(dtype: str, shape: Sequence[int], data=None) -> HostTensor:
    """host.ts:53-66."""
    shape = tuple(int(d) for d in shape)
    if data is None:
        arr = np.zeros(size_of(shape), NP_STORAGE[dtype])
    elif dtype == "bf16":
        arr = f32_to_bf16_bits(np.asarray(data, np.float32).reshape(-1))
    else:
        arr = np.asarray(data).astype(NP_STORAGE[dtype]).reshape(-1)
    if arr.size != size_of(shape):
        raise ValueError(f"host(): {arr.size} values for shape {list(shape)}")
    return HostTensor(dtype, shape, arr.reshape(shape))


def to_f32(t: HostTensor) -> np.ndarray:
    """host.ts:84-100 toF32."""
    if t.dtype == "bf16":
        return bf16_bits_to_f32(t.data)
    return np.asarray(t.data).astype(np.float32)


def quant_groups(in_features: int, group_size: int) -> int:
    return -(-in_features // group_size)


def validate_quantized(h: HostQuantized) -> None:
    """host.ts:136-153 validateQuantized (same messages)."""
    N, K = h.shape
    where = f"quantized [{N}, {K}] q{h.bits}/{h.mode}/g{h.groupSize}"
    if h.bits not in (4, 8):
        raise ValueError(f"{where}: bits must be 4 or 8")
    if h.mode not in ("symmetric", "affine"):
        raise ValueError(f'{where}: mode must be "symmetric" or "affine"')
    if not (N > 0 and K > 0):
        raise ValueError(f"{where}: bad shape")
    if not (isinstance(h.groupSize, int) and h.groupSize > 0):
        raise ValueError(f"{where}: bad group size")
    if (K * h.bits) % 32:
        raise ValueError(f"{where}: in · bits must be a multiple of 32")
    if h.data.size != N * K * h.bits // 8:
        raise ValueError(f"{where}: data has {h.data.size} bytes, want {N * K * h.bits // 8}")
    G = quant_groups(K, h.groupSize)

    def check(t, name):
        if t is None:
            raise ValueError(f"{where}: missing {name}")
        if t.dtype not in ("f32", "f16", "bf16"):
            raise TypeError(f"{where}: {name} must be float")
        if tuple(t.shape) != (N, G):
            raise ValueError(f"{where}: {name} has shape {list(t.shape)}, want [{N}, {G}]")

    check(h.scales, "scales")
    if h.mode == "affine":
        check(h.biases, "biases")
    elif h.biases is not None:
        raise ValueError(f"{where}: symmetric quantization takes no biases")


def unpack_quantized(h: HostQuantized) -> np.ndarray:
    """host.ts:155-171 → int32 values [N*K] (signed for symmetric)."""
    d = np.asarray(h.data, np.uint8).reshape(-1)
    signed = h.mode == "symmetric"
    if h.bits == 8:
        return (d.view(np.int8) if signed else d).astype(np.int32)
    lo = (d & 15).astype(np.int32)
    hi = (d >> 4).astype(np.int32)
    if signed:
        lo = np.where(lo >= 8, lo - 16, lo)
        hi = np.where(hi >= 8, hi - 16, hi)
    q = np.empty(d.size * 2, np.int32)
    q[0::2], q[1::2] = lo, hi
    return q


def pack_quantized(q, bits: int) -> np.ndarray:
    """host.ts:174-184 packQuantized."""
    q = np.asarray(q).astype(np.int64).reshape(-1)
    if bits == 8:
        return (q & 255).astype(np.uint8)
    if q.size % 2:
        raise ValueError("packQuantized: 4-bit needs an even value count")
    return ((q[0::2] & 15) | ((q[1::2] & 15) << 4)).astype(np.uint8)
