"""The FLOP counts bench.py divides by (no GPU): the linear layers' per-token
count against the projection shapes, and the attention count against a
brute-force count of visible (query, key) pairs over the layer kinds that
parseModernBertConfig gives (global every third layer from the first,
sliding layers seeing |i - j| <= window / 2); and the roofline denominators,
which come from MEASURED_PEAKS.json only when it holds both figures."""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

sys.path.insert(0, str(Path(__file__).resolve().parent.parent))
import bench  # noqa: E402
from laya_js_b200 import workloads as WL  # noqa: E402
from laya_js_b200.modernbert import parseModernBertConfig  # noqa: E402


def test_linear_flops_per_token():
    for cfg in (WL.BASE, WL.LARGE):
        H, I, n = cfg["hidden_size"], cfg["intermediate_size"], cfg["num_hidden_layers"]
        shapes = [(3 * H, H), (H, H), (2 * I, H), (H, I)]  # Wqkv, Wo, Wi, mlp.Wo as [out, in]
        assert bench.linear_flops_per_token(cfg) == sum(2 * o * k for o, k in shapes) * n
    assert round(bench.linear_flops_per_token(WL.BASE) / 1e6, 1) == 220.6


@pytest.mark.parametrize("layers", [1, 3, 7, 22])
def test_attention_flops_against_pair_count(layers):
    cfg = {**WL.BASE, "num_hidden_layers": layers}
    kinds = parseModernBertConfig(cfg)["layerTypes"]
    half = cfg["local_attention"] // 2
    lens = [1, 2, 63, 64, 65, 129, 300]
    pairs = 0
    for L in lens:
        i = np.arange(L)
        d = np.abs(i[:, None] - i[None, :])
        pairs += sum(L * L if k == "full_attention" else int((d <= half).sum()) for k in kinds)
    assert bench.attention_flops(cfg, lens) == 4.0 * cfg["hidden_size"] * pairs


def test_attention_flops_configs2_step():
    lens, _, _ = WL.cfg2_prompts()
    assert abs(bench.attention_flops(WL.BASE, lens) / 1e12 - 0.911) < 5e-4


def test_peaks_fall_back_only_when_the_measured_file_lacks_them(tmp_path, monkeypatch):
    import json
    monkeypatch.setattr(bench, "ROOT", tmp_path)
    assert bench.measured_peaks()["src"] == "fallback"  # no file
    (tmp_path / "MEASURED_PEAKS.json").write_text(json.dumps({"hbm_gbs": 6000.0}))
    assert bench.measured_peaks()["src"] == "fallback"  # sustained bf16 figure missing
    (tmp_path / "MEASURED_PEAKS.json").write_text(json.dumps({"hbm_gbs": 6000.0, "bf16_tflops_sustained": 1300.0}))
    p = bench.measured_peaks()
    assert p == {"bf16": 1300.0, "hbm": 6000.0, "src": "measured"}
    assert "MEASURED_PEAKS.json" in bench.PEAK_SRC[p["src"]][0]
