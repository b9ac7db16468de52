"""Regenerates the golden fixtures in this folder from a checkout of laya-js.

The files written here are the reference's own test data, unchanged in
content, so that the parity tests can run on a machine that has no copy of
the reference:

- ``ops.json``, ``ops-numerics.json``, ``ops-quantized.json``: the
  tensor-backend conformance cases (packages/tensor-backend/fixtures/*.json,
  loaded by ``loadOpCases`` in packages/tensor-backend/src/conformance.ts:98-112).
- ``tiny/``: the tiny Laya checkpoint and its per-stage activations
  (packages/laya-fixtures/data/tiny/{model.safetensors, activations.json,
  encoder/config.json, rl_agent_config.json}), the end-to-end pin used by
  packages/modernbert/test/modernbert.test.ts:65-117 and
  packages/laya/test/model.test.ts.

Usage: ``python tests/golden/make_golden.py <path-to-laya-js-checkout>``.
"""
from __future__ import annotations

import json
import shutil
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent


def main(ref: Path) -> None:
    fx = ref / "packages" / "tensor-backend" / "fixtures"
    for name in ("ops.json", "ops-numerics.json", "ops-quantized.json"):
        cases = json.loads((fx / name).read_text())
        (HERE / name).write_text(json.dumps(cases, separators=(",", ":")))
    tiny_src = ref / "packages" / "laya-fixtures" / "data" / "tiny"
    tiny = HERE / "tiny"
    tiny.mkdir(exist_ok=True)
    shutil.copyfile(tiny_src / "model.safetensors", tiny / "model.safetensors")
    shutil.copyfile(tiny_src / "rl_agent_config.json", tiny / "rl_agent_config.json")
    shutil.copyfile(tiny_src / "encoder" / "config.json", tiny / "encoder_config.json")
    act = json.loads((tiny_src / "activations.json").read_text())
    (tiny / "activations.json").write_text(json.dumps(act, separators=(",", ":")))


if __name__ == "__main__":
    main(Path(sys.argv[1] if len(sys.argv) > 1 else "../laya-js"))
