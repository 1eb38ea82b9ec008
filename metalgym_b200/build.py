"""Builds the product library libmetalgym_b200.so (in-tree) with nvcc for sm_100a.

Each CUDA source is compiled to an object under metalgym_b200/_build/ (only
when it or a header changed) and the objects are linked into
metalgym_b200/libmetalgym_b200.so. Environment translation units are compiled
with --fmad=false so that environment arithmetic rounds every multiply and add
separately, exactly as the reference environment code does when it is
compiled as host C++ (trajectories are compared bit for bit).
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
LIB = PKG / "libmetalgym_b200.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
          "-I", str(ROOT / "include"), "-I", str(CSRC)]

# source -> extra nvcc flags
SOURCES: dict[str, list[str]] = {
    "runtime.cu": [],
    "gemm.cu": [],
    "gemm_rows.cu": [],
    "policy.cu": [],
    "block_fwd.cu": [],
    "block_cluster.cu": [],
    "collect_fused.cu": [],
    "head_tail.cu": [],
    "minibatch_tiles.cu": [],
    "envs.cu": [],
    "envs_builtin.cu": ["--fmad=false"],
    "p2p.cu": [],
    "engine.cu": [],
    "capi_session.cu": [],
    "noalloc.cu": [],
}


def _nvcc() -> str:
    cand = os.environ.get("NVCC") or "/usr/local/cuda/bin/nvcc"
    return cand if Path(cand).exists() else "nvcc"


def _headers() -> list[Path]:
    hs = list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h"))
    hs += list((ROOT / "include").rglob("*.h")) + list((ROOT / "include").rglob("*.cuh"))
    return hs


def _stale(src: Path, obj: Path, newest_header: float) -> bool:
    if not obj.exists():
        return True
    t = obj.stat().st_mtime
    return src.stat().st_mtime > t or newest_header > t


def _compile(src: Path, obj: Path, extra: list[str], verbose: bool) -> None:
    cmd = [_nvcc(), *ARCH, *COMMON, *extra, "-c", str(src), "-o", str(obj)]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{r.stdout}\n{r.stderr}")


def build(verbose: bool = False, jobs: int = 8, force: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    newest = max((h.stat().st_mtime for h in _headers()), default=0.0)
    objs = []
    todo = []
    for name, extra in SOURCES.items():
        src = CSRC / name
        obj = BUILD / (src.stem + ".o")
        objs.append(obj)
        if force or _stale(src, obj, newest):
            todo.append((src, obj, extra))
    if todo:
        with cf.ThreadPoolExecutor(max_workers=jobs) as ex:
            for f in [ex.submit(_compile, s, o, e, verbose) for s, o, e in todo]:
                f.result()
    if todo or not LIB.exists() or any(o.stat().st_mtime > LIB.stat().st_mtime for o in objs):
        tmp = LIB.with_suffix(".so.tmp")
        cmd = [_nvcc(), *ARCH, "-shared", "-o", str(tmp), *map(str, objs), "-ldl"]
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
        os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    build(verbose="-v" in sys.argv, force="-f" in sys.argv)
    print(LIB)
