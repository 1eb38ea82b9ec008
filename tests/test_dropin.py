"""The drop-in C++ API (include/gym.h, include/model/ppo.h -> include/metalgym/).

CPU: the reference's own host programs (its examples and benchmarks) compile
and link UNCHANGED against these headers and the product library, and so do
this repository's examples. GPU: the examples run, and so does the
reference's benchmark program built from its unmodified source.
"""
import os
import subprocess
from pathlib import Path

import pytest
from orc import reference_tree

ROOT = Path(__file__).resolve().parent.parent
BUILD = ROOT / "tests" / "_build"
LIB_DIR = ROOT / "metalgym_b200"
REFERENCE_TREE = reference_tree()
REF_PROGRAMS = ["examples/CartPole/main.cpp", "examples/CartPoleContinuous/main.cpp", "examples/VoxelNav/main.cpp",
                "bench/metalrl_bench.cpp", "bench/metalrl_bench_voxelnav.cpp"]
OWN_EXAMPLES = ["cartpole", "raw_step", "checkpoint_resume"]


def compile_program(src: Path, out: Path) -> None:
    out.parent.mkdir(parents=True, exist_ok=True)
    cmd = ["g++", "-std=c++17", "-O2", "-Wall", "-Werror", "-Wno-unused-variable", "-I", str(ROOT / "include"),
           str(src), "-L", str(LIB_DIR), "-lmetalgym_b200", f"-Wl,-rpath,{LIB_DIR}", "-o", str(out)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr


def ref_binary(rel: str) -> Path:
    return BUILD / ("ref_" + rel.replace("/", "_").replace(".cpp", ""))


@pytest.mark.parametrize("rel", REF_PROGRAMS)
def test_reference_programs_compile_unchanged(rel):
    if REFERENCE_TREE is None:
        pytest.skip("reference source tree not present (set METALGYM_REFERENCE or build oracle/_ref)")
    compile_program(REFERENCE_TREE / rel, ref_binary(rel))


@pytest.mark.parametrize("name", OWN_EXAMPLES)
def test_own_examples_compile(name):
    compile_program(ROOT / "examples" / name / "main.cpp", BUILD / f"example_{name}")


def run(binary: Path, *args, timeout=600):
    env = dict(os.environ)
    env["LD_LIBRARY_PATH"] = f"{LIB_DIR}:{env.get('LD_LIBRARY_PATH', '')}"
    r = subprocess.run([str(binary), *args], capture_output=True, text=True, timeout=timeout, env=env)
    assert r.returncode == 0, r.stdout + r.stderr
    return r.stdout


@pytest.mark.gpu
def test_cartpole_example_runs_and_learns():
    b = BUILD / "example_cartpole"
    if not b.exists():
        compile_program(ROOT / "examples" / "cartpole" / "main.cpp", b)
    out = run(b, "15")
    lengths = [float(l.split("episode length")[1].split()[0]) for l in out.splitlines() if "episode length" in l]
    assert len(lengths) == 15 and lengths[-1] > 1.5 * lengths[0], out
    assert "greedy step reward 1.0" in out


@pytest.mark.gpu
def test_raw_step_example_runs():
    b = BUILD / "example_raw_step"
    if not b.exists():
        compile_program(ROOT / "examples" / "raw_step" / "main.cpp", b)
    out = run(b, "1024")
    lines = [l for l in out.splitlines() if "steps/s" in l]
    assert len(lines) == 2 and lines[0].startswith("CartPole") and lines[1].startswith("VoxelNav"), out


@pytest.mark.gpu
def test_checkpoint_resume_example_is_identical(tmp_path):
    b = BUILD / "example_checkpoint_resume"
    if not b.exists():
        compile_program(ROOT / "examples" / "checkpoint_resume" / "main.cpp", b)
    out = run(b, str(tmp_path / "ckpt.bin"))
    assert "resumed training identical" in out, out


@pytest.mark.gpu
def test_reference_benchmark_program_runs_on_the_b200():
    """The reference's own benchmark (bench/metalrl_bench.cpp), compiled from
    its unmodified source against the drop-in headers, runs end to end."""
    b = ref_binary("bench/metalrl_bench.cpp")
    if not b.exists():
        pytest.skip("reference benchmark binary not built (needs the reference tree at build time)")
    out = run(b, "4096", "2")
    assert "collect + train (4 epochs):" in out, out
