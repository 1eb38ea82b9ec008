"""Data parallelism with world size 2, as torch.distributed.run launches it
(one process per rank; tests/dp_worker.py is the rank program).

CPU (gloo): the host logic of metalgym_b200.dist and the all-reduce update
semantics on the oracle. GPU (two B200s, NCCL or the library's all-reduce
over NVLink peer memory): the product's all-reduced gradient against the
per-rank gradients, bit for bit, and bit-identical weights across ranks after
train(); skipped with fewer than two GPUs.
"""
import json
import os
import socket
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def launch(mode, nproc=2, limit=600, extra=(), env=None):
    cmd = ["timeout", "-k", "30", str(limit), sys.executable, "-m", "torch.distributed.run", "--nnodes", "1",
           "--nproc-per-node", str(nproc), "--master-addr", "127.0.0.1", "--master-port", str(free_port()),
           str(ROOT / "tests" / "dp_worker.py"), "--mode", mode, *extra]
    p = subprocess.run(cmd, capture_output=True, text=True, cwd=ROOT, env={**os.environ, **(env or {})})
    lines = [l for l in p.stdout.splitlines() if l.startswith("{")]
    progress = "\n".join(l for l in p.stderr.splitlines() if l.startswith(("[rank", "Timeout (")) or "dp_worker.py" in l or "metalgym_b200" in l)
    assert p.returncode == 0 and lines, f"rc={p.returncode}\n{progress}\n{p.stdout[-3000:]}\n{p.stderr[-3000:]}"
    return json.loads(lines[-1])


def test_data_parallel_host_logic_gloo(oracle):
    res = launch("cpu")
    assert res["ok"], res
    assert res["ranks"][0]["equals_single_process"] and res["ranks"][0]["ranks_identical"]


@pytest.mark.gpu
@pytest.mark.parametrize("allreduce", ["nccl", "p2p", "nccl-overlap"])
def test_data_parallel_two_gpus(mg, allreduce):
    import torch

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    res = launch("gpu", extra=("--allreduce", allreduce))
    assert res["ok"], res
    for r in res["ranks"]:
        assert r["grad_mismatches"] == 0, r
        assert r["ranks_identical"] and r["stats_finite"], r


@pytest.mark.gpu
def test_rank_that_leaves_turns_into_an_error_two_gpus(mg):
    """A rank that stays out of the gradient all-reduce: the other rank's
    train() returns MG_ERR_COMM within its communication timeout. NVLink
    multicast (NVLS) is off in NCCL for this test: no rank leaves while its
    memory is bound to a multicast object."""
    import torch

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    res = launch("gpu-rank-leaves", limit=180, env={"NCCL_NVLS_ENABLE": "0"})
    assert res["ok"], res
    r0 = res["ranks"][0]
    assert r0["comm_error"] and r0["within_deadline"] and r0["second_comm_error"], r0
