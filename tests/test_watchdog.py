"""The train() watchdog's wait loop (metalgym_b200/csrc/watchdog.h) on the
CPU, driven by fake streams, communicators and clocks: a finished stream
returns at once and aborts nothing; a peer's asynchronous error or the
deadline releases the graphs that captured the collectives (NCCL's abort
waits for them) and then aborts the communicator exactly once and waits,
bounded, for the stream to drain; a CUDA error returns without an abort. No GPU, no NCCL:
the failure is made on the host, as the real test on two GPUs does by
keeping one rank out of the all-reduce."""
import subprocess
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent

DONE, CUDA_ERROR, PEER_ERROR, TIMEOUT = 0, 1, 2, 3


def test_watch_wait_scenarios(tmp_path):
    exe = tmp_path / "watchdog_check"
    r = subprocess.run(["g++", "-std=c++17", "-O1", "-Wall", "-Werror", "-I", str(ROOT / "metalgym_b200" / "csrc"),
                        str(ROOT / "tests" / "helpers" / "watchdog_check.cpp"), "-o", str(exe)],
                       capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    out = subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout
    res = {}
    for line in out.splitlines():
        name, result, drained, aborts, polls, released_first = line.split()
        res[name] = (int(result), int(drained), int(aborts), int(polls))
        assert int(released_first) == (int(aborts) > 0), name
    assert res["finishes"] == (DONE, 1, 0, 51)
    result, drained, aborts, _ = res["peer_error"]
    assert (result, drained, aborts) == (PEER_ERROR, 1, 1)
    result, drained, aborts, polls = res["timeout"]
    assert (result, drained, aborts) == (TIMEOUT, 1, 1) and polls > 100  # 0.1 s at 1 ms per poll
    result, drained, aborts, _ = res["timeout_undrained"]
    assert (result, drained, aborts) == (TIMEOUT, 0, 1)
    assert res["cuda_error"] == (CUDA_ERROR, 0, 0, 8)
