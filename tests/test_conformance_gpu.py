"""The reference's conformance suite (170 golden cases) on the CUDA backend,
through the C ABI: packages/tensor-backend/src/conformance.ts:238-320."""
from __future__ import annotations

import numpy as np
import pytest

from golden_io import load_cases
from gpu_util import backend
from laya_js_b200 import compose as Cm
from laya_js_b200.conformance import run_conformance
from laya_js_b200.host import host, to_f32

pytestmark = pytest.mark.gpu
CASES = load_cases()


@pytest.mark.parametrize("dtype", ["f32", "f16", "bf16"])
def test_all_cases(dtype):
    fails = run_conformance(backend(), CASES, dtype)
    assert not fails, f"{len(fails)} failing:\n" + "\n".join(fails)


@pytest.mark.parametrize("dtype", ["f32", "f16"])
def test_composed_numerics(dtype):
    """withoutOptionalOps: the compose.ts default compositions on this backend
    (cumsum stays native: it has no composition — packages/backend-cpu/test/conformance.test.ts:14-17)."""
    b = Cm.without_optional_ops(backend(), [o for o in Cm.NUMERICS_OPS if o != "cumsum"])
    fails = run_conformance(b, CASES, dtype)
    assert not fails, "\n".join(fails)


def test_composed_quantized():
    b = Cm.without_optional_ops(backend(), Cm.QUANTIZED_OPS)
    fails = run_conformance(b, [c for c in CASES if c["op"].startswith("quantized")], "f32")
    assert not fails, "\n".join(fails)


def test_scope_disposes_intermediates_and_keeps_results():
    """conformance.ts:311-318."""
    b = backend()
    x = b.fromHost(host("f32", [2], [1, 2]))
    y = b.scope(lambda: b.add(b.exp(x), x))
    got = to_f32(b.read(y))
    assert np.allclose(got, [np.e + 1, np.exp(2) + 2], atol=1e-5, rtol=1e-5)
    b.dispose(y)
    b.dispose(x)
    b.dispose(x)  # idempotent
