"""The createBackend("cuda") edit for laya
(laya_js_b200/ts/patches/laya-create-backend-cuda.patch against
packages/laya/src/io-node.ts:83-108, packages/laya/src/common.ts:7-8 and
packages/laya/package.json): it parses, it adds "cuda" to BackendName and to
the "auto" order between mlx and webgpu, and — when LAYA_JS_CHECKOUT points at
a laya-js checkout — it applies cleanly to that checkout's files."""
from __future__ import annotations

import os
import shutil
import subprocess
from pathlib import Path

import pytest

PATCH = Path(__file__).resolve().parents[1] / "laya_js_b200" / "ts" / "patches" / "laya-create-backend-cuda.patch"
FILES = ("packages/laya/src/common.ts", "packages/laya/src/io-node.ts", "packages/laya/package.json")


def test_patch_parses_and_adds_cuda():
    r = subprocess.run(["git", "apply", "--numstat", str(PATCH)], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    touched = {l.split("\t")[2] for l in r.stdout.splitlines()}
    assert touched == set(FILES)
    text = PATCH.read_text()
    assert '+export type BackendName = "mlx" | "cuda" | "webgpu" | "cpu";' in text
    assert '+  for (const [name, make] of [["mlx", mlx], ["cuda", cuda], ["webgpu", webgpu]] as const) {' in text
    assert 'import("@johnhenry/backend-cuda")' in text


@pytest.mark.skipif(not os.environ.get("LAYA_JS_CHECKOUT"), reason="LAYA_JS_CHECKOUT (a laya-js checkout) is not set")
def test_patch_applies_to_checkout(tmp_path):
    src = Path(os.environ["LAYA_JS_CHECKOUT"])
    for f in FILES:
        (tmp_path / f).parent.mkdir(parents=True, exist_ok=True)
        shutil.copy(src / f, tmp_path / f)
    r = subprocess.run(["git", "apply", "-v", str(PATCH)], cwd=tmp_path, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    io = (tmp_path / "packages/laya/src/io-node.ts").read_text()
    assert 'if (req === "cuda") return cuda();' in io
