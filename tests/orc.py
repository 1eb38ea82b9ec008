"""ctypes bindings of the CPU oracles used as checkers by the tests.

  load_oracle()   oracle/_build/libmg_oracle.so  (C++ restatement; built if missing)
  load_ref()      oracle/_ref/libmg_ref.so       (the reference's own sources; built
                                                  if the reference tree is present)
  load_hostenv()  tests/_build/libmg_hostenv.so  (the product's env structs compiled
                                                  for the host; built if missing)
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent.parent
ORACLE_LIB = ROOT / "oracle" / "_build" / "libmg_oracle.so"
REF_LIB = ROOT / "oracle" / "_ref" / "libmg_ref.so"
HOSTENV_LIB = ROOT / "tests" / "_build" / "libmg_hostenv.so"


def reference_tree() -> Path | None:
    """The reference's source tree: $METALGYM_REFERENCE, else the tree that
    `make -C oracle ref REF=<dir>` recorded in oracle/_ref/tree, else None
    (a GPU box has the built oracle/_ref library but not the tree)."""
    env = os.environ.get("METALGYM_REFERENCE")
    if env:
        return Path(env) if Path(env).is_dir() else None
    rec = ROOT / "oracle" / "_ref" / "tree"
    if rec.exists():
        t = Path(rec.read_text().strip())
        return t if t.is_dir() else None
    return None

I, U, F, D = C.c_int, C.c_uint32, C.c_float, C.c_double
U16 = C.c_uint16


class P(C.c_void_p):
    """Pointer argument that also accepts a numpy array: the array object is
    the call's argument, so it stays alive until the C function returns (a
    raw address of a temporary array could be freed before the call)."""

    @classmethod
    def from_param(cls, obj):
        if isinstance(obj, np.ndarray):
            if not obj.flags["C_CONTIGUOUS"]:
                raise ValueError("array argument must be C-contiguous")
            return obj.ctypes.data_as(C.c_void_p)
        return C.c_void_p.from_param(obj)


def _sig(lib, name, res, args):
    fn = getattr(lib, name)
    fn.restype = res
    fn.argtypes = args


def _make(target: str, extra: list[str] | None = None) -> None:
    subprocess.run(["make", "-s", "-C", str(ROOT / "oracle"), target, *(extra or [])], check=True)


def load_oracle():
    _make("port")
    lib = C.CDLL(str(ORACLE_LIB))
    _sig(lib, "orc_f2bf", U16, [F])
    _sig(lib, "orc_bf2f", F, [U16])
    _sig(lib, "orc_input_forward", None, [P, P, P, P, U, U, U])
    _sig(lib, "orc_input_backward", None, [P, P, P, P, U, U, U])
    _sig(lib, "orc_layernorm_forward", None, [P, P, P, P, P, P, U, U])
    _sig(lib, "orc_layernorm_backward", None, [P, P, P, P, P, P, U, U])
    _sig(lib, "orc_gemm_f32acc", None, [P, P, P, U, U, U, I, I])
    _sig(lib, "orc_sample_action", None, [P, P, P, P, P, U, U, U])
    _sig(lib, "orc_sample_gaussian", None, [P, P, P, P, P, U, U, U, P])
    _sig(lib, "orc_policy_loss", None, [P, P, P, P, P, P, P, U, U, U, F, F, F])
    _sig(lib, "orc_gaussian_loss", None, [P, P, P, P, P, P, P, U, U, U, F, F, F, P, P])
    _sig(lib, "orc_gae", None, [P, P, P, P, P, P, U, U, F, F])
    _sig(lib, "orc_normalize_advantage", None, [P, P, U])
    _sig(lib, "orc_grad_norm_sq", D, [P, U])
    _sig(lib, "orc_adam_step", None, [P, P, P, P, P, F, U, F, F, F, F])
    _sig(lib, "orc_model_create", P, [U, U, U, I, U, U, U, F, U, U])
    _sig(lib, "orc_model_destroy", None, [P])
    _sig(lib, "orc_model_opt_count", U, [P])
    _sig(lib, "orc_model_opt_float_count", U, [P])
    _sig(lib, "orc_model_param_count", U, [P])
    _sig(lib, "orc_model_param_info", None, [P, U, C.POINTER(U), C.POINTER(U), C.POINTER(I)])
    for n in ("orc_model_weights", "orc_model_master", "orc_model_momentum", "orc_model_variance", "orc_model_grad"):
        _sig(lib, n, P, [P])
    _sig(lib, "orc_model_step_counter", F, [P])
    _sig(lib, "orc_model_set_step_counter", None, [P, F])
    _sig(lib, "orc_model_set_hparams", None, [P, F, F, F, F, F, F])
    _sig(lib, "orc_model_forward", None, [P, P, U, P])
    _sig(lib, "orc_model_train_minibatch", None, [P, P, P, P, P, P, U, P, P])
    _sig(lib, "orc_model_gradient", None, [P, P, P, P, P, P, U, P, P])
    _sig(lib, "orc_model_collect", None, [P, P, I, P, P, P, P, P, P, P, P, P, P, P, P, P, I])
    _sig(lib, "orc_model_train", None, [P, P, P, P, P, P, U, P])
    return lib


REF_HOST_LIB = ROOT / "oracle" / "_ref" / "libmg_ref_host.so"


def load_ref_host():
    """The reference's own host code (oracle/ref_host.cpp), or None when it was
    not built and the reference tree is absent."""
    if not REF_HOST_LIB.exists():
        tree = reference_tree()
        if tree is None:
            return None
        _make("ref-host", [f"REF={tree}"])
    lib = C.CDLL(str(REF_HOST_LIB))
    _sig(lib, "ref_host_create", C.c_void_p, [I, I, I, I, I, F, I, U])
    _sig(lib, "ref_host_destroy", None, [C.c_void_p])
    _sig(lib, "ref_host_sizes", None, [C.c_void_p, P])
    _sig(lib, "ref_host_params", None, [C.c_void_p, P, P])
    _sig(lib, "ref_host_param_info", None, [C.c_void_p, U, P, P])
    _sig(lib, "ref_host_set_head", None, [C.c_void_p, P])
    _sig(lib, "ref_host_act", None, [C.c_void_p, U, I, P, P, P])
    _sig(lib, "ref_host_act_greedy", None, [C.c_void_p, P])
    _sig(lib, "ref_host_set_log_std", None, [C.c_void_p, F])
    _sig(lib, "ref_host_log_std", F, [C.c_void_p, I])
    _sig(lib, "ref_host_last_stats", None, [C.c_void_p, P, F, P])
    return lib


def load_ref():
    if not REF_LIB.exists():
        tree = reference_tree()
        if tree is None:
            return None
        _make("ref", [f"REF={tree}"])
    lib = C.CDLL(str(REF_LIB))
    _sig(lib, "ref_env_sizes", I, [I, P])
    _sig(lib, "ref_rollout", None, [I, P, P, P, P, P, P, U, I])
    _sig(lib, "ref_sample_action", None, [P, P, P, P, P, U, U, U])
    _sig(lib, "ref_sample_gaussian", None, [P, P, P, P, P, U, U, U, P])
    _sig(lib, "ref_policy_loss", None, [P, P, P, P, P, P, P, U, U, U, F, F, F])
    _sig(lib, "ref_gaussian_loss", None, [P, P, P, P, P, P, P, U, U, U, F, F, F, P, P])
    _sig(lib, "ref_gae", None, [P, P, P, P, P, P, U, U, U, U, F, F])
    _sig(lib, "ref_normalize_advantage", None, [P, P, U])
    _sig(lib, "ref_grad_norm_sq", None, [P, P, P, U, U])
    _sig(lib, "ref_adam_step", None, [P, P, P, P, P, P, P, U, U, F, F, F, F])
    _sig(lib, "ref_residual_add", None, [P, P, P, U])
    _sig(lib, "ref_reduce_partials", None, [P, P, U, U])
    _sig(lib, "ref_input_forward", None, [P, P, P, P, U, U, U])
    _sig(lib, "ref_input_backward", None, [P, P, P, P, U, U, U, U])
    _sig(lib, "ref_layernorm_forward", None, [P, P, P, P, P, P, U, U])
    _sig(lib, "ref_layernorm_backward", None, [P, P, P, P, P, P, P, U, U])
    return lib


def load_hostenv():
    src = ROOT / "tests" / "helpers" / "host_envs.cpp"
    hdrs = list((ROOT / "include" / "metalgym").rglob("*.h"))
    stale = not HOSTENV_LIB.exists() or any(p.stat().st_mtime > HOSTENV_LIB.stat().st_mtime for p in [src, *hdrs])
    if stale:
        HOSTENV_LIB.parent.mkdir(parents=True, exist_ok=True)
        subprocess.run(["g++", "-std=c++17", "-O2", "-fPIC", "-shared", "-fopenmp", "-ffp-contract=off",
                        "-I", str(ROOT / "include"), str(src), "-o", str(HOSTENV_LIB)], check=True)
    lib = C.CDLL(str(HOSTENV_LIB))
    _sig(lib, "hostenv_rollout", None, [I, P, P, P, P, P, P, U, I])
    for n in ("hostenv_sinf", "hostenv_cosf", "hostenv_expf", "hostenv_logf", "hostenv_tanhf"):
        _sig(lib, n, F, [F])
    return lib


HOST_SAMPLER_LIB = ROOT / "tests" / "_build" / "libmg_host_sampler.so"


def load_host_sampler():
    """metalgym::sample_actions_host (the drop-in act(), include/metalgym/ppo.h)
    built for the host (tests/helpers/host_sampler.cpp)."""
    src = ROOT / "tests" / "helpers" / "host_sampler.cpp"
    hdrs = list((ROOT / "include").rglob("*.h"))
    lib_ = HOST_SAMPLER_LIB
    stale = not lib_.exists() or any(p.stat().st_mtime > lib_.stat().st_mtime for p in [src, *hdrs])
    if stale:
        lib_.parent.mkdir(parents=True, exist_ok=True)
        subprocess.run(["g++", "-std=c++17", "-O2", "-fPIC", "-shared", "-ffp-contract=off", "-I",
                        str(ROOT / "include"), str(src), "-o", str(lib_)], check=True)
    lib = C.CDLL(str(lib_))
    _sig(lib, "host_act", None, [I, P, U, P, U, I, P, P, P])
    return lib


# ---------------------------------------------------------------- helpers

def ptr(a: np.ndarray) -> np.ndarray:
    """The array itself, checked contiguous: the bindings take arrays, not addresses."""
    assert a.flags["C_CONTIGUOUS"]
    return a


def bf16_round(x: np.ndarray) -> np.ndarray:
    """float32 -> nearest-even bf16, returned as uint16 bit patterns."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    nan = np.isnan(x)
    if nan.any():
        r[nan] = ((u[nan] >> 16) | 0x40).astype(np.uint16)
    return r


def bf16_to_f32(h: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(h, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


# Environment ids shared by the reference build, the host build and the product.
ENV_IDS = {"rollout_cartpole": 0, "rollout_cartpole_continuous": 1, "rollout_voxelnav": 2}
ENV_SIZES = {  # state, action, obs bytes, obs dim, act dim, continuous
    "rollout_cartpole": (20, 4, 16, 4, 2, False),
    "rollout_cartpole_continuous": (20, 4, 16, 4, 1, True),
    "rollout_voxelnav": (1056, 4, 160, 40, 6, False),
}


def seed_words(n: int, seed: int = 0, first: int = 0) -> np.ndarray:
    """Per-env xorshift seeds (gym.h:57-61 with the seed folded into the index)."""
    i = np.arange(first, first + n, dtype=np.uint64) + np.uint64(seed)
    w = ((i * np.uint64(2654435761) + np.uint64(1)) & np.uint64(0xFFFFFFFF)).astype(np.uint32)
    w[w == 0] = 1
    return w
