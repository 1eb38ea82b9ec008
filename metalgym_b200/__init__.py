"""Python binding of the metalgym_b200 C ABI (include/metalgym_b200.h).

The product is the CUDA library libmetalgym_b200.so and the C++ drop-in
headers under include/metalgym/. This module only loads that library with
ctypes and declares the argument types of every exported function, for the
tests, the benchmark and Python callers. There is no fallback: if the library
is missing or fails to load, importing `lib()` raises.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

from ._abi import SIGNATURES

PKG = Path(__file__).resolve().parent
LIB_PATH = PKG / "libmetalgym_b200.so"

_lib = None


class MgError(RuntimeError):
    """A metalgym_b200 call returned an error code."""


def lib() -> ctypes.CDLL:
    """The loaded product library (loaded once, with every signature declared)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise ImportError(f"{LIB_PATH} is missing: run `python -m metalgym_b200.build` (or __graft_entry__.build())")
        handle = ctypes.CDLL(str(LIB_PATH), mode=os.RTLD_NOW | os.RTLD_GLOBAL)
        for name, (restype, argtypes) in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = restype
            fn.argtypes = argtypes
        _lib = handle
    return _lib


def check(rc: int, what: str = "") -> None:
    """Raises MgError with mg_last_error() if rc is not MG_OK."""
    if rc != 0:
        msg = lib().mg_last_error().decode(errors="replace")
        raise MgError(f"{what or 'metalgym_b200'} failed with code {rc}: {msg}")


def call(name: str, *args) -> None:
    """Calls C-ABI function `name` and raises on a non-zero status."""
    check(getattr(lib(), name)(*args), name)
