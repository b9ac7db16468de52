"""Loads liblaya_cuda.so through ctypes, the Python stand-in for the FFI
routes the reference's native backend uses (koffi / bun:ffi / Deno.dlopen,
packages/backend-mlx/src/ffi.ts:169-318).

Library resolution mirrors packages/backend-mlx/src/lib.ts:473-511: when
``$LAYA_CUDA_LIB`` is set it must name an existing file (set-but-missing is
an error, never a fallback); otherwise the in-tree build next to this file is
used. There is no CPU fallback: a missing library raises.

Signatures are read from include/laya_cuda*.h so the Python binding and the C
ABI cannot drift apart.
"""
from __future__ import annotations

import ctypes as C
import os
import re
from pathlib import Path

PKG = Path(__file__).resolve().parent
INCLUDE = PKG.parent / "include"
DEFAULT_LIB = PKG / "liblaya_cuda.so"

_TYPES = {
    "int": C.c_int, "int*": C.POINTER(C.c_int), "int64_t": C.c_int64, "int64_t*": C.POINTER(C.c_int64),
    "constint64_t*": C.POINTER(C.c_int64), "constint32_t*": C.POINTER(C.c_int32), "double": C.c_double,
    "constvoid*": C.c_void_p, "void*": C.c_void_p, "size_t": C.c_size_t, "constuint8_t*": C.c_void_p,
    "uint64_t": C.c_uint64, "uint64_t*": C.POINTER(C.c_uint64), "lc_tensor": C.c_uint64,
    "lc_tensor*": C.POINTER(C.c_uint64), "constlc_tensor*": C.POINTER(C.c_uint64), "void": None,
    "constchar*": C.c_char_p, "float*": C.POINTER(C.c_float), "constfloat*": C.POINTER(C.c_float),
    "int32_t*": C.POINTER(C.c_int32), "constlc_encoder_config*": C.c_void_p, "double*": C.POINTER(C.c_double),
}


def header_declarations() -> dict[str, tuple[str, list[str]]]:
    """name -> (return type, [param types]) for every function in include/*.h."""
    decls: dict[str, tuple[str, list[str]]] = {}
    for h in sorted(INCLUDE.glob("*.h")):
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        text = re.sub(r"//[^\n]*", "", text)
        for m in re.finditer(r"^\s*((?:const\s+)?\w+\s*\*?)\s*(\w+)\s*\(([^)]*)\)\s*;", text, flags=re.M):
            ret, name, params = m.group(1), m.group(2), m.group(3)
            if not name.startswith("lc_"):
                continue
            types = []
            if params.strip() not in ("", "void"):
                for p in params.split(","):
                    p = p.strip()
                    p = re.sub(r"\b\w+\s*$", "", p) if not p.endswith("*") else p  # drop the parameter name
                    types.append(p.replace(" ", ""))
            decls[name] = (ret.replace(" ", ""), types)
    return decls


class LayaCudaError(RuntimeError):
    """An error reported by liblaya_cuda (the message of lc_last_error())."""


def lib_path() -> Path:
    env = os.environ.get("LAYA_CUDA_LIB")
    if env:
        p = Path(env)
        if not p.is_file():
            raise FileNotFoundError(f"LAYA_CUDA_LIB={env} does not exist (set-but-missing is an error, not a fallback)")
        return p
    if not DEFAULT_LIB.is_file():
        raise FileNotFoundError(f"{DEFAULT_LIB} is not built: run `python -m laya_js_b200.build` (there is no CPU fallback)")
    return DEFAULT_LIB


_LIB = None


def load() -> C.CDLL:
    global _LIB
    if _LIB is not None:
        return _LIB
    lib = C.CDLL(str(lib_path()))
    for name, (ret, params) in header_declarations().items():
        fn = getattr(lib, name)
        fn.restype = _TYPES[ret]
        fn.argtypes = [_TYPES[p] for p in params]
    _LIB = lib
    return lib


def call(fn_name: str, *args) -> None:
    """Calls lc_<name>; a nonzero return raises LayaCudaError with lc_last_error()."""
    lib = load()
    rc = getattr(lib, fn_name)(*args)
    if rc != 0:
        msg = lib.lc_last_error().decode("utf-8", "replace")
        raise LayaCudaError(msg)
