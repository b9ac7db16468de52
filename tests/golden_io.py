"""Loading of the reference's golden fixtures (tests/golden/*) as numpy.

The fixture format is the conformance-case format of
packages/tensor-backend/src/conformance.ts:29-52 (base64 little-endian
element bytes; float tensors are always stored as f32, :80-82).
"""
from __future__ import annotations

import base64
import json
from pathlib import Path

import numpy as np

GOLDEN = Path(__file__).resolve().parent / "golden"
CASE_FILES = ("ops.json", "ops-numerics.json", "ops-quantized.json")

_NP = {"i32": "<i4", "bool": "u1", "u8": "u1", "i8": "i1", "u16": "<u2", "i16": "<i2",
       "u32": "<u4", "u64": "<u8", "i64": "<i8", "f64": "<f8"}


def decode(e: dict | None) -> np.ndarray | None:
    """conformance.ts:54-83 decodeTensor."""
    if e is None:
        return None
    raw = base64.b64decode(e["b64"])
    dt = _NP.get(e["dtype"], "<f4")
    a = np.frombuffer(raw, dtype=dt).reshape(e["shape"]).copy()
    if e["dtype"] == "bool":
        a = a.astype(bool)
    return a


def load_cases(files=CASE_FILES) -> list[dict]:
    out = []
    for f in files:
        out.extend(json.loads((GOLDEN / f).read_text()))
    return out


def tiny():
    """(encoder config json, agent config json, weights dict of f32 arrays, activations json)."""
    from safetensors.numpy import load_file
    t = GOLDEN / "tiny"
    return (json.loads((t / "encoder_config.json").read_text()),
            json.loads((t / "rl_agent_config.json").read_text()),
            load_file(str(t / "model.safetensors")),
            json.loads((t / "activations.json").read_text()))
