"""Loader of ``libhca_b200.so`` with argument types read from ``include/hca_b200.h``.

The library is the only compute path: if it is missing or a call fails the
wrappers raise; there is no fallback.
"""

from __future__ import annotations

import ctypes
import os
import re
from functools import lru_cache
from pathlib import Path

PKG = Path(__file__).resolve().parent
REPO = PKG.parent.parent
HEADER = REPO / "include" / "hca_b200.h"
LIB_PATH = Path(os.environ.get("HCA_B200_LIB", PKG / "lib" / "libhca_b200.so"))

_CTYPES = {
    "int": ctypes.c_int,
    "int32_t": ctypes.c_int32,
    "int64_t": ctypes.c_int64,
    "float": ctypes.c_float,
    "void": None,
}


class HcaError(RuntimeError):
    """A libhca_b200 entry point returned a negative status."""

    def __init__(self, name: str, status: int, message: str):
        super().__init__(f"{name} failed: {message} (status {status})")
        self.status = status


def _ctype(decl: str):
    decl = decl.strip()
    if "*" in decl:
        base = decl.replace("const", "").replace("*", "").split()[0]
        return ctypes.c_char_p if base == "char" else ctypes.c_void_p
    base = decl.replace("const", "").split()[0]
    return _CTYPES[base]


def parse_header(path: Path = HEADER) -> dict[str, tuple[object, list[object]]]:
    """``{name: (restype, [argtypes])}`` of every function the header declares."""
    text = re.sub(r"/\*.*?\*/", "", path.read_text(), flags=re.S)
    text = re.sub(r"//[^\n]*", "", text)
    out = {}
    pat = re.compile(r"^\s*((?:const\s+)?[A-Za-z_][A-Za-z0-9_]*\s*\**)\s*(hca_[A-Za-z0-9_]+)\s*\(([^)]*)\)\s*;",
                     re.M)
    for m in pat.finditer(text):
        ret, name, args = m.group(1), m.group(2), m.group(3)
        argtypes = []
        for a in [x.strip() for x in args.split(",")]:
            if not a or a == "void":
                continue
            typ = re.sub(r"\s*[A-Za-z_][A-Za-z0-9_]*$", "", a) if not a.endswith("*") else a
            if "*" in a and not typ.endswith("*"):
                typ = a[: a.rfind("*") + 1]
            argtypes.append(_ctype(typ))
        out[name] = (_ctype(ret), argtypes)
    return out


@lru_cache(maxsize=1)
def lib() -> ctypes.CDLL:
    if not LIB_PATH.exists():
        raise RuntimeError(
            f"{LIB_PATH} is missing: build it with `python -m vllm_ernie_b200.build` "
            "(the HCA path has no fallback)")
    handle = ctypes.CDLL(str(LIB_PATH))
    for name, (res, args) in parse_header().items():
        fn = getattr(handle, name)
        fn.restype = res
        fn.argtypes = args
    return handle


def call(name: str, *args) -> int:
    """Call an ``int``-returning entry point and raise on a negative status."""
    status = getattr(lib(), name)(*args)
    if status != 0:
        msg = lib().hca_status_string(status).decode()
        if status == -3:  # HCA_E_CUDA: the CUDA error behind it
            msg += ": " + lib().hca_last_cuda_error().decode()
        raise HcaError(name, status, msg)
    return status
