"""One rank of the data-parallel tests, launched by torch.distributed.run.

--mode cpu (gloo, no GPU): the host logic of metalgym_b200.dist (comm-id
  broadcast, max over ranks, env shards) and the data-parallel update
  semantics on the oracle: every rank takes the gradient of its own rows,
  the sum over ranks is scaled by 1/world, the clip and Adam run on every
  rank; the ranks' weights must stay bit-identical and equal a single
  process that averages the shards' gradients itself.
--mode gpu (one GPU per rank, NCCL or the library's own all-reduce over
  NVLink peer memory (--allreduce p2p) for the gradient, gloo for the host):
  a rank's all-reduced gradient must equal the average over ranks of the
  gradients that an identical model without the communicator computes on
  the same rollout, bit for bit; after train() the weight digests of all
  ranks agree.

Rank 0 prints one JSON line; the exit status is 0 when every check passed.
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "tests"))


def oracle_shard(orc, rows, rank, seed=3):
    """A synthetic minibatch of `rows` CartPole-shaped rows for one rank."""
    rng = np.random.default_rng(100 + rank)
    obs = rng.normal(0, 0.5, (rows, 4)).astype(np.float32)
    act = rng.integers(0, 2, rows).astype(np.int32)
    adv = rng.normal(0, 1, rows).astype(np.float32)
    ret = rng.normal(1, 0.5, rows).astype(np.float32)
    logp = (np.log(0.5) + rng.normal(0, 0.05, rows)).astype(np.float32)
    return obs, act, adv, ret, logp


def oracle_arrays(orc, om, n):
    import ctypes as C

    def view(fn, dt):
        p = getattr(orc, fn)(om)
        return np.ctypeslib.as_array(C.cast(p, C.POINTER(np.ctypeslib.as_ctypes_type(dt))), shape=(n,))

    return dict(weights=view("orc_model_weights", np.uint16), master=view("orc_model_master", np.float32),
                mom=view("orc_model_momentum", np.float32), var=view("orc_model_variance", np.float32),
                grad=view("orc_model_grad", np.float32))


def oracle_gradient(orc, om, shard, rows):
    stats = np.zeros((rows, 5), np.float32)
    nsq = np.zeros(1, np.float32)
    orc.orc_model_gradient(om, *shard, rows, stats, nsq)


def oracle_step(orc, om, a, grad, lr, max_norm):
    """Clip + Adam on the given (already averaged) gradient: model/ppo.h:873-903."""
    step = orc.orc_model_step_counter(om) + 1.0
    orc.orc_model_set_step_counter(om, step)
    nsq = float(np.dot(grad.astype(np.float64), grad.astype(np.float64)))
    orc.orc_adam_step(a["master"], grad, a["mom"], a["var"], a["weights"], nsq, len(grad), lr,
                      np.float32(0.9) ** np.float32(step), np.float32(0.999) ** np.float32(step), max_norm)


def digest(a):
    import hashlib

    return hashlib.sha256(a["weights"].tobytes() + a["master"].tobytes()).hexdigest()


def run_cpu(rank, world, dist):
    from orc import load_oracle

    from metalgym_b200.dist import broadcast_comm_id, env_shard, max_over_ranks

    out = {}
    cid = broadcast_comm_id(dist, rank, lambda: os.urandom(128))
    ids = [None] * world
    dist.all_gather_object(ids, cid)
    out["comm_id_shared"] = all(i == ids[0] for i in ids)
    out["max_over_ranks"] = max_over_ranks(rank + 1.5, dist, device="cpu") == world - 1 + 1.5
    shards = [set(range(env_shard(r, 64), env_shard(r, 64) + 64)) for r in range(world)]
    out["shards_disjoint"] = len(set().union(*shards)) == 64 * world

    import torch

    orc = load_oracle()
    rows, lr, max_norm = 256, 3e-4, 0.5
    om = orc.orc_model_create(rows, 4, 2, 0, 64, 2, 1, lr, 4, 3)
    n = orc.orc_model_opt_count(om)
    a = oracle_arrays(orc, om, n)
    for it in range(3):
        oracle_gradient(orc, om, oracle_shard(orc, rows, rank + world * it), rows)
        g = torch.from_numpy(a["grad"].copy())
        dist.all_reduce(g)
        avg = (g.numpy() * np.float32(1.0 / world)).astype(np.float32)
        oracle_step(orc, om, a, avg, lr, max_norm)
    mine = digest(a)
    digests = [None] * world
    dist.all_gather_object(digests, mine)
    out["ranks_identical"] = all(d == mine for d in digests)
    if rank == 0:
        # one process holding every shard: average the shards' gradients itself
        om1 = orc.orc_model_create(rows, 4, 2, 0, 64, 2, 1, lr, 4, 3)
        b = oracle_arrays(orc, om1, n)
        for it in range(3):
            acc = np.zeros(n, np.float32)
            for r in range(world):
                oracle_gradient(orc, om1, oracle_shard(orc, rows, r + world * it), rows)
                acc = (acc + b["grad"]).astype(np.float32)
            oracle_step(orc, om1, b, (acc * np.float32(1.0 / world)).astype(np.float32), lr, max_norm)
        out["equals_single_process"] = digest(b) == mine
        orc.orc_model_destroy(om1)
    orc.orc_model_destroy(om)
    return out


def run_gpu(rank, world, local, dist, allreduce):
    import torch

    from metalgym_b200.dist import destroy_comm, env_shard, nccl_comm, p2p_allreduce, weights_digest
    from metalgym_b200.session import Gym, PPOModel

    torch.cuda.set_device(local)
    R, T = 1024, 4
    out = {}
    gym = Gym("rollout_cartpole", R, seed=0, first_env_id=env_shard(rank, R), device=local)
    model = PPOModel(gym, 128, 4, 2, 3e-4, T, seed=7)
    comm = None
    if allreduce in ("nccl", "nccl-overlap"):
        comm = nccl_comm(dist, rank, world, local)
        model.set_comm(comm, rank, world)
        model.set_allreduce_overlap(allreduce == "nccl-overlap")
    else:
        p2p_allreduce(model, dist, rank, world)
    model.collect()
    # an identical model without the communicator, on the same rollout
    gym1 = Gym("rollout_cartpole", R, seed=0, first_env_id=env_shard(rank, R), device=local)
    solo = PPOModel(gym1, 128, 4, 2, 3e-4, T, seed=7)
    for buf in ("obs", "actions", "logp", "value", "reward", "done", "adv", "ret", "adv_stats", "weights", "master",
                "momentum", "variance"):
        solo.upload(buf, model.download(buf))
    solo.set_step_counter(model.step_counter())
    model.train_slot(1)
    solo.train_slot(1)
    g_dp = model.download("grad").view(np.float32)
    g_local = torch.from_numpy(solo.download("grad").view(np.float32).copy())
    dist.all_reduce(g_local)
    g_avg = (g_local.numpy() * np.float32(1.0 / world)).astype(np.float32)
    out["grad_mismatches"] = int((g_dp != g_avg).sum())
    out["grad_max_abs_diff"] = float(np.abs(g_dp - g_avg).max())
    # full train() through the captured graph (one all-reduce per minibatch)
    for _ in range(2):
        model.collect()
        model.train(2)
    mine = weights_digest(model)
    digests = [None] * world
    dist.all_gather_object(digests, mine)
    out["ranks_identical"] = all(d == mine for d in digests)
    st = model.last_stats()
    out["stats_finite"] = bool(all(np.isfinite(v) for v in st.values()))
    solo.close()
    gym1.close()
    model.close()  # releases the train graph that holds the NCCL calls
    gym.close()
    destroy_comm(comm)
    return out


def log(rank, msg):
    """Progress on stderr, so a failing run shows where each rank was."""
    import time

    print(f"[rank {rank} {time.strftime('%H:%M:%S')}] {msg}", file=sys.stderr, flush=True)


def run_gpu_rank_leaves(rank, world, local, dist):
    """Both ranks train one step together; then rank 1 leaves between steps
    (with nothing in flight) and stays out of the next all-reduce. Rank 0
    trains with a 5 s communication timeout: its train() must fail with
    MG_ERR_COMM (6) well within the deadline instead of blocking, and keep
    failing; then rank 1 aborts its own communicator. The failure is made on
    the host; no kernel is broken."""
    import time

    import torch

    import metalgym_b200
    from metalgym_b200 import MgError
    from metalgym_b200.dist import destroy_comm, env_shard, nccl_comm
    from metalgym_b200.session import Gym, PPOModel

    import faulthandler

    faulthandler.dump_traceback_later(90, exit=False)  # where a rank still waits after 90 s
    torch.cuda.set_device(local)
    R, T = 512, 4
    gym = Gym("rollout_cartpole", R, seed=0, first_env_id=env_shard(rank, R), device=local)
    model = PPOModel(gym, 128, 4, 2, 3e-4, T, seed=7)
    comm = nccl_comm(dist, rank, world, local)
    model.set_comm(comm, rank, world)
    model.set_comm_timeout(5.0)
    log(rank, "communicator ready; one step with both ranks")
    model.collect()
    model.train(1)
    model.collect()
    dist.barrier()
    log(rank, "rank 1 leaves")
    out = {}
    if rank == 0:
        t0 = time.time()
        try:
            model.train(1)
            out["comm_error"] = False
        except MgError as e:
            out["comm_error"] = "code 6" in str(e)
        log(rank, f"train() returned after {time.time() - t0:.1f} s: comm_error={out['comm_error']}")
        out["within_deadline"] = time.time() - t0 < 60.0
        try:
            model.train(1)
            out["second_comm_error"] = False
        except MgError as e:
            out["second_comm_error"] = "code 6" in str(e)
        log(rank, f"second train(): comm_error={out['second_comm_error']}")
    dist.barrier()  # rank 1 stayed out until rank 0 gave up
    log(rank, "past the barrier")
    if rank != 0:
        metalgym_b200.check(metalgym_b200.lib().mg_comm_abort(comm), "mg_comm_abort")
        out["aborted"] = True
    model.close()
    gym.close()
    destroy_comm(comm)  # nothing to do for an aborted communicator
    log(rank, "closed")
    faulthandler.cancel_dump_traceback_later()
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--mode", choices=["cpu", "gpu", "gpu-rank-leaves"], required=True)
    ap.add_argument("--allreduce", choices=["nccl", "nccl-overlap", "p2p"], default="nccl")
    args = ap.parse_args()
    import torch.distributed as dist

    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=120))
    try:
        if args.mode == "cpu":
            out = run_cpu(rank, world, dist)
        elif args.mode == "gpu":
            out = run_gpu(rank, world, local, dist, args.allreduce)
        else:
            os.environ["NCCL_NVLS_ENABLE"] = "0"  # no NVLink multicast objects when a rank leaves
            out = run_gpu_rank_leaves(rank, world, local, dist)
        results = [None] * world
        dist.all_gather_object(results, out)
    finally:
        dist.barrier()
        dist.destroy_process_group()
    ok = all(v is True or (k == "grad_mismatches" and v == 0) or k == "grad_max_abs_diff"
             for r in results for k, v in r.items())
    if rank == 0:
        print(json.dumps({"ok": ok, "world": world, "ranks": results}), flush=True)
    sys.exit(0 if ok else 1)


if __name__ == "__main__":
    main()
