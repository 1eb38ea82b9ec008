"""The C ABI: every function declared in include/metalgym_b200.h is exported
by the built library and has a ctypes signature; no compute (CPU only)."""
import ctypes
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent


def declared_functions():
    text = (ROOT / "include" / "metalgym_b200.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    text = re.sub(r"typedef struct mg_env_ops \{.*?\} mg_env_ops;", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(mg_[a-z0-9_]+)\s*\(", text)))


def test_header_matches_ctypes_table():
    from metalgym_b200._abi import SIGNATURES

    assert declared_functions() == sorted(SIGNATURES)


def test_library_exports_every_declared_symbol():
    import metalgym_b200

    if not metalgym_b200.LIB_PATH.exists():
        pytest.fail("libmetalgym_b200.so not built: run __graft_entry__.build()")
    lib = ctypes.CDLL(str(metalgym_b200.LIB_PATH))
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, missing


def test_builtin_envs_registered_and_sized():
    """Loading the library registers the reference's three example envs with
    the reference's struct sizes (no GPU work)."""
    import metalgym_b200
    from metalgym_b200 import _env_ops_info

    lib = metalgym_b200.lib()
    names = {lib.mg_env_name(i).decode() for i in range(lib.mg_env_count())}
    assert {"rollout_cartpole", "rollout_cartpole_continuous", "rollout_voxelnav"} <= names
    from orc import ENV_SIZES

    for name, (sb, ab, ob, od, ad, cont) in ENV_SIZES.items():
        info = _env_ops_info(name)
        assert info == dict(state_bytes=sb, action_bytes=ab, obs_bytes=ob, obs_dim=od, act_dim=ad,
                            continuous=int(cont)), name


def test_errors_are_reported_without_a_gpu():
    import metalgym_b200

    lib = metalgym_b200.lib()
    rc = lib.mg_env_step(b"no_such_env", None, None, None, None, None, None, None, 4, None)
    assert rc == 5  # MG_ERR_NOT_FOUND
    assert b"no_such_env" in lib.mg_last_error()
    rc = lib.mg_gemm_bf16(None, 0, 64, None, 0, 64, 128, 128, 64, 0, None, 128, None, 0, 1, None)
    assert rc == 1  # MG_ERR_ARGUMENT (checked before any CUDA call)


def declared_parameter_counts():
    """Number of parameters of every function the header declares."""
    text = (ROOT / "include" / "metalgym_b200.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    text = re.sub(r"typedef struct mg_env_ops \{.*?\} mg_env_ops;", "", text, flags=re.S)
    counts = {}
    for m in re.finditer(r"\b(mg_[a-z0-9_]+)\s*\(([^)]*)\)\s*;", text):
        params = m.group(2).strip()
        counts[m.group(1)] = 0 if params in ("", "void") else params.count(",") + 1
    return counts


def test_ctypes_signatures_have_the_declared_arity():
    """A ctypes signature with the wrong number of parameters would shift every
    argument after the first difference."""
    from metalgym_b200._abi import SIGNATURES

    counts = declared_parameter_counts()
    wrong = {n: (len(SIGNATURES[n][1]), counts[n]) for n in counts if len(SIGNATURES[n][1]) != counts[n]}
    assert not wrong, wrong


# Entry points that only query, release or read state: null pointers are valid
# (release / no output) or there is nothing to validate.
_NO_ARGUMENT_CHECK = {
    "mg_last_error", "mg_version", "mg_env_count", "mg_env_name", "mg_env_find", "mg_device_status",
    "mg_gemm_rows_splits", "mg_input_backward_num_partials", "mg_layernorm_backward_num_partials",
    "mg_gaussian_loss_num_partials", "mg_reduce_partials_num_norm_partials", "mg_gym_destroy", "mg_ppo_destroy",
    "mg_comm_destroy", "mg_host_free",
    "mg_set_tile_trace",  # NULL turns the trace off
}


def _null_pointer_arguments(argtypes):
    """Null for every pointer, 128 for every count or width, 0.1 for every
    float and the CartPole kernel name for every string."""
    vals = []
    for a in argtypes:
        if a in (ctypes.c_int, ctypes.c_uint32, ctypes.c_int64, ctypes.c_uint64):
            vals.append(128)
        elif a is ctypes.c_float:
            vals.append(0.1)
        elif a is ctypes.c_char_p:
            vals.append(b"rollout_cartpole")
        else:
            vals.append(None)
    return vals


def test_null_pointers_are_argument_errors():
    """Every entry point that takes buffers rejects null ones with
    MG_ERR_ARGUMENT and a message before it reaches CUDA, so that a caller's
    missing buffer never becomes a kernel reading address 0."""
    import torch

    if torch.cuda.is_available():
        pytest.skip("runs where no GPU is visible: an entry point without the check would launch")
    import metalgym_b200
    from metalgym_b200._abi import SIGNATURES

    lib = metalgym_b200.lib()
    wrong = {}
    for name, (_, argtypes) in SIGNATURES.items():
        if name in _NO_ARGUMENT_CHECK or name.startswith("mg_env_register"):
            continue
        rc = getattr(lib, name)(*_null_pointer_arguments(argtypes))
        msg = lib.mg_last_error() or b""
        if rc != 1 or not msg:
            wrong[name] = (rc, msg.decode(errors="replace"))
    assert not wrong, wrong


def test_header_is_plain_c(tmp_path):
    """include/metalgym_b200.h is a C header (hosts bind it through C FFIs):
    it compiles as C99 with every warning an error."""
    import subprocess

    src = tmp_path / "use.c"
    src.write_text('#include "metalgym_b200.h"\nint main(void) {\n    mg_collect_fused_args a = {0};\n'
                   '    mg_env_ops o = {0};\n    (void)a; (void)o;\n    return mg_version() == MG_VERSION ? 0 : 1;\n}\n')
    r = subprocess.run(["gcc", "-std=c99", "-Wall", "-Wextra", "-Werror", "-pedantic", "-I", str(ROOT / "include"),
                        "-fsyntax-only", str(src)], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
