"""C-ABI checks that need no GPU: the library loads and exports every
function include/*.h declares; the TypeScript binding (ffi.ts table, index.ts
call sites, Backend members) agrees with the header and with the Python
mirror; every environment setting is documented; the host helpers mirror
host.ts."""
from __future__ import annotations

import ctypes

import numpy as np

from laya_js_b200 import _lib
from laya_js_b200.host import HostQuantized, host, pack_quantized, to_f32, unpack_quantized, validate_quantized
from oracle import ops as O


def test_library_exports_every_declared_symbol():
    decls = _lib.header_declarations()
    assert len(decls) >= 60
    lib = ctypes.CDLL(str(_lib.lib_path()))
    missing = [n for n in decls if not hasattr(lib, n)]
    assert not missing, missing


def test_binding_signatures_resolve():
    lib = _lib.load()
    for name in _lib.header_declarations():
        assert getattr(lib, name).argtypes is not None or name in ("lc_destroy", "lc_last_error", "lc_flush")


def _ts_sources():
    from pathlib import Path
    d = Path(_lib.__file__).resolve().parent / "ts" / "backend-cuda" / "src"
    return (d / "ffi.ts").read_text(), (d / "index.ts").read_text()


def _ts_symbol_table() -> dict[str, list[str]]:
    """ffi.ts SYMBOLS: name -> argument codes (aliases OP1 / OP2 / RED expanded)."""
    import re
    src, _ = _ts_sources()
    alias = {k: re.findall(r'"(\w)"', v) for k, v in re.findall(r"const (\w+): A\[\] = (\[[^\]]*\]);", src)}
    start = src.index("export const SYMBOLS")
    return {name: alias[spec] if spec in alias else re.findall(r'"(\w)"', spec)
            for name, spec in re.findall(r"(lc_\w+):\s*(\[[^\]]*\]|\w+)", src[start:src.index("};", start)])}


def test_typescript_ffi_table_matches_header():
    """The TypeScript binding (ts/backend-cuda/src/ffi.ts SYMBOLS) declares each
    entry's argument codes by hand; they must follow include/laya_cuda.h:
    pointers 'p', 64-bit integers (tensor handles, int64 sizes) 'h', int 'i',
    double 'd', size_t 'z'."""
    table = _ts_symbol_table()
    assert len(table) >= 60
    codes = {"lc_tensor": "h", "uint64_t": "h", "int64_t": "h", "int": "i", "int32_t": "i", "double": "d", "size_t": "z"}
    decls = _lib.header_declarations()
    for name, got in table.items():
        assert name in decls, f"{name} is bound in ffi.ts but not declared in include/"
        want = ["p" if t.endswith("*") else codes.get(t, "?" + t) for t in decls[name][1]]
        assert got == want, f"{name}: ffi.ts {got}, header {want} ({decls[name][1]})"


def _top_level_args(text: str, i: int) -> list[str]:
    """Arguments of the call whose '(' is text[i], split at top-level commas."""
    depth, cur, out = 0, "", []
    for c in text[i:]:
        if c in "([{":
            depth += 1
            if depth == 1:
                continue
        elif c in ")]}":
            depth -= 1
            if depth == 0:
                out.append(cur.strip())
                break
        elif c == "," and depth == 1:
            out.append(cur.strip())
            cur = ""
            continue
        cur += c
    return [a for a in out if a]


def test_typescript_call_sites_pass_every_argument():
    """index.ts calls the binding as op("lc_x", ...) (the output pointer is
    prepended), N.call("lc_x", ...), or through un / bin / red (2, 3 and 4
    arguments): each call's argument count must equal the entry's arity."""
    import re
    table = _ts_symbol_table()
    _, src = _ts_sources()
    sites = []
    for kind, implicit in (("op", 1), ("N.call", 0)):
        for m in re.finditer(r"\b" + re.escape(kind) + r'\(\s*"(lc_\w+)"', src):
            args = _top_level_args(src, m.start() + len(kind))
            sites.append((m.group(1), len(args) - 1 + implicit))
    for helper, n in (("un", 2), ("bin", 3), ("red", 4)):
        sites += [(name, n) for name in re.findall(r"\b" + helper + r'\(\s*"(lc_\w+)"\s*\)', src)]
    assert len(sites) >= 60
    for name, n in sites:
        assert name in table, f"index.ts calls {name}, which ffi.ts does not bind"
        assert n == len(table[name]), f"index.ts passes {n} arguments to {name}, which takes {len(table[name])}"


def _ts_backend_members(src: str) -> set[str]:
    """Top-level keys of the `const b = { ... }` object in index.ts (properties
    `name: ...` and methods `name(...) {`, `async name(...)`, `name<R>(...)`)."""
    import re
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    src = re.sub(r"//[^\n]*", "", src)
    i = src.index("const b = {") + len("const b = ")
    keys, tok, depth, generic = set(), "", 0, 0
    for c in src[i:]:
        if tok is not None and depth == 1:  # reading a member's key
            if c == "<":
                generic += 1
                continue
            if generic:
                generic -= c == ">"
                continue
            if c in ":(":
                m = re.fullmatch(r"\s*(?:async\s+)?(\w+)\s*", tok)
                if m:
                    keys.add(m.group(1))
                tok = None  # skip to the next top-level comma
            else:
                tok += c
        if c in "([{":
            depth += 1
        elif c in ")]}":
            depth -= 1
            if depth == 0:
                break
        elif c == "," and depth == 1:
            tok = ""
    return keys


def test_typescript_and_python_backends_expose_the_same_methods():
    """The two host mirrors of Backend<T> (ts/backend-cuda/src/index.ts and
    laya_js_b200/backend.py) offer the same public members."""
    import inspect

    from laya_js_b200.backend import CudaBackend
    _, src = _ts_sources()
    ts = _ts_backend_members(src) - {"name"}
    py = {n for n, _ in inspect.getmembers(CudaBackend, predicate=inspect.isfunction) if not n.startswith("_")}
    assert len(ts) >= 55
    assert ts == py, f"only in TypeScript: {sorted(ts - py)}; only in Python: {sorted(py - ts)}"


def test_lc_supports_without_device():
    lib = _lib.load()
    out = ctypes.c_int()
    assert lib.lc_supports(0, ctypes.byref(out)) == 0 and out.value == 1
    assert lib.lc_supports(99, ctypes.byref(out)) == 0 and out.value == 0


def test_calls_before_init_fail_with_message():
    lib = _lib.load()
    out = ctypes.c_uint64()
    rc = lib.lc_exp(ctypes.byref(out), ctypes.c_uint64(0))
    assert rc != 0
    assert b"lc_init" in lib.lc_last_error() or b"null" in lib.lc_last_error()


def test_pack_unpack_match_oracle():
    rng = np.random.default_rng(1)
    for bits, mode in ((8, "symmetric"), (4, "affine"), (4, "symmetric"), (8, "affine")):
        lo, hi = ((-128, 127) if bits == 8 else (-8, 7)) if mode == "symmetric" else (0, (1 << bits) - 1)
        q = rng.integers(lo, hi + 1, size=(6, 64))
        packed = pack_quantized(q, bits)
        assert np.array_equal(packed, O.pack_quantized(q, bits))
        h = HostQuantized((6, 64), bits, 32, mode, packed, host("f32", (6, 2)), host("f32", (6, 2)) if mode == "affine" else None)
        validate_quantized(h)
        assert np.array_equal(unpack_quantized(h).reshape(6, 64), q)


def test_bf16_host_rounding():
    x = np.array([1.0, 1.00390625, -3.3, np.nan], np.float32)
    h = host("bf16", (4,), x)
    back = to_f32(h)
    assert back[0] == 1.0 and back[2] == np.float32(-3.296875) and np.isnan(back[3])


def test_every_environment_setting_is_documented():
    """Each LAYA_CUDA_* variable the library or the Python mirror reads is in
    INTEGRATION.md's table of settings."""
    import re
    from pathlib import Path
    pkg = Path(_lib.__file__).resolve().parent
    read = set()
    for f in list((pkg / "csrc").glob("*.cu")) + list((pkg / "csrc").glob("*.cuh")) + list(pkg.glob("*.py")):
        read |= set(re.findall(r"""(?:getenv|environ\.get)\(\s*["'](LAYA_CUDA_\w+)["']""", f.read_text()))
    assert {"LAYA_CUDA_LIB", "LAYA_CUDA_PDL"} <= read
    doc = (pkg.parent / "INTEGRATION.md").read_text()
    missing = sorted(v for v in read if f"`{v}`" not in doc)
    assert not missing, f"settings read by the code but not in INTEGRATION.md: {missing}"
