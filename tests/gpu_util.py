"""Shared GPU-test helpers: one backend per process, on cuda:0."""
from __future__ import annotations

import numpy as np

_B = None


def backend():
    global _B
    if _B is None:
        from laya_js_b200 import createCudaBackend
        _B = createCudaBackend(0)
    return _B


def rel_err(got, want) -> float:
    g = np.asarray(got, np.float64)
    w = np.asarray(want, np.float64)
    return float(np.max(np.abs(g - w)) / max(1e-30, np.max(np.abs(w))))
