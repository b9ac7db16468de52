"""Host-side workload generators and the quantizer (no GPU)."""
from __future__ import annotations

import numpy as np

from laya_js_b200 import workloads as WL
from laya_js_b200.host import unpack_quantized, validate_quantized
from oracle import ops as O


def test_quantizer_matches_oracle_restatement():
    rng = np.random.default_rng(0)
    w = (rng.standard_normal((32, 200)) * 0.02).astype(np.float16)
    for bits in (4, 8):
        q, s, b = WL.quantize_affine(w, bits, 64)
        q2, s2, b2 = O.quantize_affine(w, bits, 64)
        assert np.array_equal(q, q2) and np.array_equal(s, s2) and np.array_equal(b, b2)


def test_quantized_host_layout():
    rng = np.random.default_rng(1)
    w = (rng.standard_normal((8, 128)) * 0.02).astype(np.float16)
    h = WL.quantized_host(w, 4, 64)
    validate_quantized(h)
    q, _, _ = WL.quantize_affine(w, 4, 64)
    assert np.array_equal(unpack_quantized(h).reshape(8, 128), q)


def test_token_batch_shape_and_markers():
    lens = WL.lengths(256, 32, 512, seed=1)
    assert lens.min() >= 32 and lens.max() <= 512
    ids, cu = WL.token_batch(WL.BASE, lens, seed=2)
    assert cu[-1] == lens.sum() and len(ids) == cu[-1]
    assert np.all(ids[cu[:-1]] == WL.CLS_ID) and np.all(ids[cu[1:] - 1] == WL.SEP_ID)
    assert ids.min() >= 5 and ids.max() < WL.BASE["vocab_size"]
    ll = WL.lengths(1000, 16, 4096, seed=3, dist="loguniform")
    assert ll.min() >= 16 and ll.max() <= 4096
