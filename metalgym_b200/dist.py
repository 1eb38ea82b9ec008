"""Data parallelism over one process per GPU.

Every rank steps its own shard of environments and trains on its own rollout;
the only collective of the hot path is the NCCL all-reduce of each
minibatch's flat gradient inside the train graph (mg_ppo_set_comm). This
module holds the host-side setup around it, on top of an existing
torch.distributed process group of any backend (NCCL or gloo):

* env_shard: the first env id of a rank. Env seeds are (seed + env id), so
  the shards are disjoint RNG streams, as if one gym held all ranks' envs.
* broadcast_comm_id / nccl_comm: rank 0 makes the 128-byte NCCL id, the
  process group carries it to the other ranks, each rank joins the
  communicator on its device.
* p2p_allreduce: the alternative to NCCL, the library's own all-reduce over
  NVLink peer memory; the process group carries the CUDA IPC handles.
* max_over_ranks: the device time of a step is the slowest rank's.
* weights_digest: a hash of a rank's weight arena and fp32 master copy; the
  all-reduced gradient, clip and Adam are computed identically everywhere, so
  the digests of all ranks must agree after every train().
"""
from __future__ import annotations

import ctypes
import hashlib

from . import check, lib


def env_shard(rank: int, envs_per_rank: int) -> int:
    """First env id of `rank` when every rank holds envs_per_rank envs."""
    return rank * envs_per_rank


def broadcast_comm_id(dist, rank: int, make_id) -> bytes:
    """Rank 0 calls make_id() for a 128-byte id; every rank returns it."""
    obj = [make_id() if rank == 0 else None]
    dist.broadcast_object_list(obj, src=0)
    cid = obj[0]
    if not isinstance(cid, (bytes, bytearray)) or len(cid) != 128:
        raise RuntimeError("communicator id must be 128 bytes")
    return bytes(cid)


def nccl_unique_id() -> bytes:
    buf = (ctypes.c_char * 128)()
    check(lib().mg_comm_unique_id(buf), "mg_comm_unique_id")
    return bytes(buf)


def nccl_comm(dist, rank: int, world: int, device: int) -> ctypes.c_void_p:
    """The NCCL communicator of this rank for mg_ppo_set_comm."""
    cid = broadcast_comm_id(dist, rank, nccl_unique_id)
    buf = (ctypes.c_char * 128).from_buffer_copy(cid)
    comm = ctypes.c_void_p()
    check(lib().mg_comm_init(world, rank, buf, device, ctypes.byref(comm)), "mg_comm_init")
    return comm


def destroy_comm(comm) -> None:
    if comm:
        check(lib().mg_comm_destroy(comm), "mg_comm_destroy")


def p2p_allreduce(model, dist, rank: int, world: int) -> None:
    """Switches the model's per-minibatch gradient all-reduce to the kernels
    over NVLink peer memory: exchanges every rank's region handle over the
    process group, opens them all, then synchronises the ranks."""
    mine = model.p2p_handle()
    handles = [None] * world
    dist.all_gather_object(handles, mine)
    model.p2p_open(handles, rank, world)
    dist.barrier()


def max_over_ranks(x: float, dist, device: str = "cuda") -> float:
    """Maximum of x over the ranks of the default process group (identity
    without one). device: where the backend reduces (cuda for NCCL, cpu for
    gloo)."""
    if dist is None:
        return x
    import torch

    t = torch.tensor([float(x)], device=device, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def weights_digest(model) -> str:
    """sha256 of the model's bf16 weight arena and fp32 master weights."""
    h = hashlib.sha256()
    h.update(model.download("weights").tobytes())
    h.update(model.download("master").tobytes())
    return h.hexdigest()
