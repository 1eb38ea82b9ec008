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


class EnvOps(ctypes.Structure):
    """Layout of mg_env_ops (include/metalgym_b200.h)."""

    _fields_ = [("abi_version", ctypes.c_uint32), ("name", ctypes.c_char_p),
                ("state_bytes", ctypes.c_uint32), ("action_bytes", ctypes.c_uint32),
                ("obs_bytes", ctypes.c_uint32), ("obs_dim", ctypes.c_uint32),
                ("act_dim", ctypes.c_uint32), ("continuous", ctypes.c_uint32),
                ("step", ctypes.c_void_p), ("run_random", ctypes.c_void_p),
                ("collect_step", ctypes.c_void_p), ("collect_fused", ctypes.c_void_p)]


class CollectFusedArgs(ctypes.Structure):
    """Layout of mg_collect_fused_args (include/metalgym_b200.h)."""

    _fields_ = [("parallels", ctypes.c_int), ("horizon", ctypes.c_int), ("layers", ctypes.c_int),
                ("obs_dim", ctypes.c_int), ("w_in", ctypes.c_void_p), ("b_in", ctypes.c_void_p),
                ("ln_gamma", ctypes.c_void_p * 5), ("ln_beta", ctypes.c_void_p * 5),
                ("w_up", ctypes.c_void_p * 4), ("w_down", ctypes.c_void_p * 4), ("w_head", ctypes.c_void_p),
                ("log_std", ctypes.c_void_p), ("states", ctypes.c_void_p), ("done", ctypes.c_void_p),
                ("rng", ctypes.c_void_p), ("obs_slots", ctypes.c_void_p), ("action_slots", ctypes.c_void_p),
                ("logp_slots", ctypes.c_void_p), ("value_slots", ctypes.c_void_p),
                ("reward_slots", ctypes.c_void_p), ("done_slots", ctypes.c_void_p), ("adv_slots", ctypes.c_void_p),
                ("ret_slots", ctypes.c_void_p), ("boot_head", ctypes.c_void_p), ("gamma", ctypes.c_float),
                ("lambda_", ctypes.c_float)]


def _env_ops_info(name: str) -> dict:
    """Sizes and dims of a registered environment."""
    p = lib().mg_env_find(name.encode())
    if not p:
        raise MgError(f"no environment registered as {name!r}")
    o = EnvOps.from_address(p)
    return dict(state_bytes=o.state_bytes, action_bytes=o.action_bytes, obs_bytes=o.obs_bytes,
                obs_dim=o.obs_dim, act_dim=o.act_dim, continuous=o.continuous)


def _env_has_fused_collect(name: str) -> bool:
    """Whether the registered environment brought the persistent collect() kernel."""
    p = lib().mg_env_find(name.encode())
    if not p:
        raise MgError(f"no environment registered as {name!r}")
    return bool(EnvOps.from_address(p).collect_fused)
