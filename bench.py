"""Benchmark of the MetalGym hot path on B200: env steps/s for the raw env
step, collect() (policy + env + GAE) and the full PPO loop (collect + train),
on the reference README's CartPole configuration (4096 envs per GPU, T = 32,
residual MLP 128 -> 512 -> 128 x 2 blocks, 4 epochs, minibatch = one 4096-row
slot).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl mine|reference]

One step = one PPO iteration (collect() + train(4)) = envs x T env steps per
GPU. The headline `value` is the full-loop throughput, device-timed with CUDA
events on the engine's stream (inputs resident, L2 flushed by a 256 MiB write
between timed steps, outside the events), max over ranks; `e2e` is the same
loop through the C ABI as a host program drives it (wall clock, including the
per-call synchronisation, the schedule upload and the LossStats / done-slot
read-back). With N > 1 (torchrun, one process per GPU) every rank steps its
own 4096 envs (disjoint env ids / RNG streams) and the gradients are
all-reduced with NCCL once per minibatch (weak scaling).

`--impl reference` times the reference's CPU implementation of the same
loop on the host cores: its own environment and per-thread kernels compiled
from source (oracle/_ref) and the C++ restatement of its PPO arithmetic
(oracle/), on a bounded sample of each step.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import re
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

ENV = "rollout_cartpole"
ENVS_PER_GPU = 4096
HORIZON = 32
EMBED, SCALE, LAYERS, EPOCHS, LR = 128, 4, 2, 4, 3e-4
RAW_STEPS = 1000
L2_FLUSH_BYTES = 256 << 20
METRIC = "env steps/s: raw step, with policy, full PPO loop (CartPole, VoxelNav) @1-8 GPU"
REFERENCE_M4_FULL_LOOP = 296e3  # reference README, CartPole full loop, 2 blocks (Apple M4; context only)


def flops_per_row(obs_dim, act_dim, E, H, L):
    """Algorithmic forward / backward FLOPs per row (head counts act_dim + 1 columns)."""
    fwd = 2 * obs_dim * E + L * 4 * E * H + 2 * E * (act_dim + 1)
    bwd = 2 * fwd - 2 * obs_dim * E  # dX and dW for every GEMM; no dX for the input layer
    return fwd, bwd


def measured_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d["hbm_gbs"], d["bf16_tflops"], "measured"
    return 6650.0, 1590.0, "fallback"


class Clocks:
    """nvidia-smi samples (SM clock, throttle reasons) during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index):
        self.dev = device_index
        self.proc = None
        self.file = None

    def __enter__(self):
        try:
            self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.dev), f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=self.file, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        if not self.proc or not self.file:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        self.file.flush()
        rows = []
        for line in Path(self.file.name).read_text().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) >= 9 and f[1].replace(".", "").isdigit():
                rows.append(f)
        os.unlink(self.file.name)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in rows]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": float(rows[0][2]), "reasons": reasons,
                "samples": len(rows), "power_w_max": max(float(r[3]) for r in rows if r[3].replace(".", "").isdigit())}


# ------------------------------------------------------------------ our arm

def run_mine(args, rank, world, local_rank, dist):
    import torch

    import metalgym_b200
    from metalgym_b200.dist import env_shard, nccl_comm, p2p_allreduce
    from metalgym_b200.session import Gym, PPOModel

    torch.cuda.set_device(local_rank)
    lib = metalgym_b200.lib()
    gym = Gym(ENV, ENVS_PER_GPU, seed=0, first_env_id=env_shard(rank, ENVS_PER_GPU), device=local_rank)
    model = PPOModel(gym, EMBED, SCALE, LAYERS, LR, HORIZON, seed=0)
    if args.collect != "auto":
        model.collect_fused = args.collect == "fused"
    model.fused_minibatch = args.fused_minibatch
    comm = None

    def connect(m):
        """The gradient all-reduce of a model: NCCL, or the library's own over NVLink peer memory."""
        if world == 1:
            return
        if args.allreduce == "nccl":
            m.set_comm(comm, rank, world)
            if args.allreduce_overlap:
                m.set_allreduce_overlap(True)
        else:
            p2p_allreduce(m, dist, rank, world)

    if world > 1 and args.allreduce == "nccl":
        if args.allreduce_overlap:
            # the overlapped all-reduce runs beside the last backward layer's
            # kernel (128 CTAs, one per SM): leave it SMs of its own
            os.environ.setdefault("NCCL_MAX_NCHANNELS", "16")
        comm = nccl_comm(dist, rank, world, local_rank)
    connect(model)
    stream = torch.cuda.ExternalStream(gym.stream(), device=local_rank)
    flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=f"cuda:{local_rank}")

    def barrier():
        if dist is not None:
            dist.barrier()

    def iteration():
        model.collect()
        model.train(EPOCHS)

    for _ in range(args.warmup):
        iteration()
    barrier()
    torch.cuda.synchronize()
    # ---- device-timed full loop
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    # Under a profiler started with --profile-from-start off, only the first
    # timed iteration is inside the profiled range.
    profile_range = os.environ.get("MG_PROFILE_FIRST_TIMED_STEP") == "1"
    with Clocks(local_rank) as clk:
        for k in range(args.steps):
            with torch.cuda.stream(stream):
                flush.fill_(float(k))
                starts[k].record(stream)
            if profile_range and k == 0:
                torch.cuda.synchronize()
                torch.cuda.profiler.start()
            iteration()
            if profile_range and k == 0:
                torch.cuda.profiler.stop()
            with torch.cuda.stream(stream):
                ends[k].record(stream)
        torch.cuda.synchronize()
    barrier()
    ms = sum(s.elapsed_time(e) for s, e in zip(starts, ends)) / args.steps
    ms = max_over_ranks(ms, dist)
    steps_per_iter = ENVS_PER_GPU * HORIZON
    value = steps_per_iter * world / (ms / 1e3)
    collect_k, train_k = model.graph_kernels()

    # ---- e2e: the loop as a host program drives it through the C ABI
    done_host = np.zeros(HORIZON * ENVS_PER_GPU, np.uint8)
    barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        iteration()
        model.last_stats()  # 24 B
        metalgym_b200.check(lib.mg_ppo_download(model.handle, 5, -1, done_host.ctypes.data, done_host.nbytes))
    e2e_s = (time.perf_counter() - t0) / args.steps
    e2e_s = max_over_ranks(e2e_s, dist)
    e2e = {"value": steps_per_iter * world / e2e_s, "unit": "env steps/s",
           "h2d_bytes_per_step": EPOCHS * HORIZON * 32, "d2h_bytes_per_step": done_host.nbytes + 24 + 4 * 3,
           "api": "mg_ppo_collect + mg_ppo_train(4) + mg_ppo_last_stats + done-slot download"}

    legs = {}
    # ---- collect only
    cs = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ce = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    for k in range(args.steps):
        with torch.cuda.stream(stream):
            flush.fill_(float(k))
            cs[k].record(stream)
        model.collect()
        with torch.cuda.stream(stream):
            ce[k].record(stream)
    torch.cuda.synchronize()
    cms = max_over_ranks(sum(s.elapsed_time(e) for s, e in zip(cs, ce)) / args.steps, dist)
    # its roofline: the T + 1 policy forwards' algorithmic FLOPs per collect() over its device time
    # (latency bound at 4096 envs: the fraction says how far from the tensor roof, not the bound)
    c_fwd, _ = flops_per_row(4, 2, EMBED, EMBED * SCALE, LAYERS)
    c_flop = ENVS_PER_GPU * (HORIZON + 1) * c_fwd
    _, c_peak, c_kind = measured_peaks()
    legs["collect"] = {"value": steps_per_iter * world / (cms / 1e3), "ms_per_call": cms,
                       "path": "one persistent kernel (fused)" if model.collect_fused else "captured per-step graph",
                       "flop_per_call": c_flop, "achieved_tflops": c_flop / (cms / 1e3) / 1e12,
                       "tensor_frac": c_flop / (cms / 1e3) / 1e12 / c_peak, "peak_kind": c_kind}
    legs["full_loop"] = {"value": value, "ms_per_iteration": ms}

    # ---- raw env step (config 1): fused multi-step kernel and the gym.run loop
    raw = Gym(ENV, ENVS_PER_GPU, seed=0, first_env_id=env_shard(rank, ENVS_PER_GPU), device=local_rank)
    rstream = torch.cuda.ExternalStream(raw.stream(), device=local_rank)
    raw.run_random(RAW_STEPS)
    raw.synchronize()
    rs, re_ = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(rstream):
        rs.record(rstream)
    raw.run_random(RAW_STEPS)
    with torch.cuda.stream(rstream):
        re_.record(rstream)
    raw.synchronize()
    rms = max_over_ranks(rs.elapsed_time(re_), dist)
    legs["raw_env"] = {"value": RAW_STEPS * ENVS_PER_GPU * world / (rms / 1e3), "steps": RAW_STEPS,
                       "kernel": "one launch, 1000 fused steps (random policy drawn on the env's RNG)",
                       "scaling": "weak (4096 envs per GPU)"}
    if world > 1:
        # strong scaling: BASELINE configs[0]'s 4096 envs in all, split over the
        # ranks. Every rank reaches the max over ranks, whatever happened.
        n_strong = ENVS_PER_GPU // world
        strong_ms = float("inf")
        try:
            sg = Gym(ENV, n_strong, seed=0, first_env_id=env_shard(rank, n_strong), device=local_rank)
            sst = torch.cuda.ExternalStream(sg.stream(), device=local_rank)
            sg.run_random(RAW_STEPS)
            sg.synchronize()
            ss, se = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            with torch.cuda.stream(sst):
                ss.record(sst)
            sg.run_random(RAW_STEPS)
            with torch.cuda.stream(sst):
                se.record(sst)
            sg.synchronize()
            strong_ms = ss.elapsed_time(se)
            sg.close()
        except Exception as ex:  # reported in the leg; the headline run goes on
            print(f"rank {rank}: strong-scaling raw leg failed: {ex}", file=sys.stderr, flush=True)
        strong_ms = max_over_ranks(strong_ms, dist)
        legs["raw_env"]["strong_4096_envs_total"] = (
            {"value": RAW_STEPS * n_strong * world / (strong_ms / 1e3), "envs_per_gpu": n_strong}
            if strong_ms != float("inf") else {"value": None, "error": "failed on a rank (see stderr)"})
    # gym.run loop with host actions / rewards (the reference benchmark's loop)
    pinned = ctypes.c_void_p()
    metalgym_b200.check(lib.mg_host_alloc(ENVS_PER_GPU * 8, ctypes.byref(pinned)))
    acts = np.ctypeslib.as_array(ctypes.cast(pinned, ctypes.POINTER(ctypes.c_int32)), shape=(ENVS_PER_GPU,))
    rew = np.ctypeslib.as_array(ctypes.cast(pinned.value + ENVS_PER_GPU * 4, ctypes.POINTER(ctypes.c_float)),
                                shape=(ENVS_PER_GPU,))
    acts[:] = 0
    for _ in range(10):
        lib.mg_gym_run(raw.handle, acts.ctypes.data, rew.ctypes.data, ENVS_PER_GPU)
    t0 = time.perf_counter()
    for _ in range(RAW_STEPS):
        lib.mg_gym_run(raw.handle, acts.ctypes.data, rew.ctypes.data, ENVS_PER_GPU)
    run_s = max_over_ranks((time.perf_counter() - t0) / RAW_STEPS, dist)
    legs["raw_env"]["gym_run_e2e"] = ENVS_PER_GPU * world / run_s
    lib.mg_host_free(pinned)

    # ---- the full loop at the other two configurations (weak scaling per GPU)
    if not args.no_extra_legs:
        for name, cfg in EXTRA_LOOPS.items():
            if args.c4_action == "tanh" and cfg["env"] == "rollout_cartpole_continuous":
                cfg = dict(cfg, env="rollout_cartpole_continuous_tanh")
            legs[name] = extra_loop_leg(cfg, rank, world, local_rank, connect, flush, dist, collect=args.collect)

    # ---- dominant kernel, timed live: see profiles/ for the launch-share list
    roof = dominant_kernel_roofline(lib, torch, local_rank, stream)

    result = None
    if rank == 0:
        result = {
            "metric": METRIC, "value": value, "unit": "env steps/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": value / REFERENCE_M4_FULL_LOOP, "dtype": "bf16", "data": "synthetic (simulated CartPole)",
            "config": workload_config(world),
            "setup": {"collect": ("one persistent kernel (fused)" if model.collect_fused else
                                  "captured per-step graph"),
                      "minibatch": ("tile passes as one kernel" if model.fused_minibatch else
                                    "separate cluster kernels chained by PDL"),
                      "allreduce": ("none" if world == 1 else
                                    "NVLink peer memory (library kernels)" if args.allreduce == "p2p" else
                                    "NCCL, overlapped with the last backward layer" if args.allreduce_overlap else
                                    "NCCL"),
                      "timing": "CUDA events on the engine stream, max over ranks"},
            "raw_env_steps_per_s": legs["raw_env"]["value"],
            "collect_env_steps_per_s": legs["collect"]["value"],
            "legs": legs, "e2e": e2e, "roofline": roof,
            "gpu_launches": args.steps * (collect_k + EPOCHS * train_k),
            "gpu_launches_per_step": {"collect_graph": collect_k, "train_graph_per_epoch": train_k,
                                      "epochs": EPOCHS},
            "clocks": clk.summary(),
        }
    model.close()  # the train graph holds NCCL calls: release it before the communicator
    gym.close()
    raw.close()
    if comm is not None:
        lib.mg_comm_destroy(comm)
    return result


def workload_config(world):
    """The headline workload, identical in both arms' JSON lines."""
    fwd, bwd = flops_per_row(4, 2, EMBED, EMBED * SCALE, LAYERS)
    return {"workload": "CartPole full PPO loop (BASELINE configs[2]): collect() + train(4) per step",
            "envs_per_gpu": ENVS_PER_GPU, "horizon": HORIZON, "embed": EMBED, "hidden": EMBED * SCALE,
            "blocks": LAYERS, "epochs": EPOCHS, "minibatch": "one slot (4096 rows)", "parallelism": f"dp{world}",
            "l2": "GPU arm: flushed between timed steps (256 MiB write, outside the events)",
            "env_steps_per_step": ENVS_PER_GPU * HORIZON * world,
            "flop_per_env_step": (HORIZON + 1) / HORIZON * fwd + EPOCHS * (fwd + bwd)}


# (env, envs per GPU, embed, scale, blocks,
# minibatch rows, timed iterations, warm-up iterations)
EXTRA_LOOPS = {
    "c4_cartpole_continuous_full_loop": dict(env="rollout_cartpole_continuous", envs=16384, embed=128, scale=4,
                                             blocks=2, minibatch=8192, steps=3, warmup=2),
    "c5_voxelnav_full_loop": dict(env="rollout_voxelnav", envs=262144, embed=256, scale=4, blocks=4,
                                  minibatch=32768, steps=2, warmup=1),
}


def extra_loop_leg(cfg, rank, world, local_rank, connect, flush, dist, collect="auto"):
    """collect() + train(4) at another configuration, device-timed like the
    headline (CUDA events on the engine stream, L2 flushed between steps).
    collect: "fused" runs collect() as the persistent kernel where the
    configuration has one (embed 128 / hidden 512 with a small env state; not
    VoxelNav), "graph" as the per-step graph, "auto" as the library chooses."""
    import torch

    from metalgym_b200 import MgError
    from metalgym_b200.dist import env_shard
    from metalgym_b200.session import Gym, PPOModel

    n = cfg["envs"]
    gym = Gym(cfg["env"], n, seed=0, first_env_id=env_shard(rank, n), device=local_rank)
    model = PPOModel(gym, cfg["embed"], cfg["scale"], cfg["blocks"], LR, HORIZON, seed=0)
    model.minibatch_rows = cfg["minibatch"]
    if collect != "auto":
        try:
            model.collect_fused = collect == "fused"
        except MgError:
            pass  # no fused kernel for this configuration: the per-step graph
    connect(model)
    stream = torch.cuda.ExternalStream(gym.stream(), device=local_rank)
    for _ in range(cfg["warmup"]):
        model.collect()
        model.train(EPOCHS)
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(cfg["steps"])]
    cev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(cfg["steps"])]
    for k, (s0, s1) in enumerate(ev):
        with torch.cuda.stream(stream):
            flush.fill_(float(k))
            s0.record(stream)
            cev[k][0].record(stream)
        model.collect()
        with torch.cuda.stream(stream):
            cev[k][1].record(stream)
        model.train(EPOCHS)
        with torch.cuda.stream(stream):
            s1.record(stream)
    torch.cuda.synchronize()
    ms = max_over_ranks(sum(a.elapsed_time(b) for a, b in ev) / len(ev), dist)
    cms = max_over_ranks(sum(a.elapsed_time(b) for a, b in cev) / len(cev), dist)
    st = model.last_stats()
    fwd, bwd = flops_per_row(model.obs_dim, model.act_dim, cfg["embed"], cfg["embed"] * cfg["scale"], cfg["blocks"])
    steps_per_iter = n * HORIZON
    flop = steps_per_iter * ((HORIZON + 1) / HORIZON * fwd + EPOCHS * (fwd + bwd))
    out = {"value": steps_per_iter * world / (ms / 1e3), "unit": "env steps/s", "env": cfg["env"],
           "ms_per_iteration": ms,
           "collect_ms": cms, "collect": "fused kernel" if model.collect_fused else "per-step graph",
           "envs_per_gpu": n, "horizon": HORIZON, "embed": cfg["embed"],
           "hidden": cfg["embed"] * cfg["scale"], "blocks": cfg["blocks"], "epochs": EPOCHS,
           "minibatch_rows": cfg["minibatch"], "minibatches_per_iteration": EPOCHS * steps_per_iter // cfg["minibatch"],
           "steps": cfg["steps"], "warmup": cfg["warmup"],
           "achieved_tflops": flop / (ms / 1e3) / 1e12, "last_stats": {k: float(v) for k, v in st.items()}}
    model.close()
    gym.close()
    return out


def max_over_ranks(x, dist):
    from metalgym_b200.dist import max_over_ranks as mor

    return mor(x, dist, device="cuda")


def _time_launches(launch, torch, stream, iters=200):
    """Average device time of `launch` run back to back on `stream` (CUDA events)."""
    for _ in range(5):
        launch()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        s.record(stream)
    for _ in range(iters):
        launch()
    with torch.cuda.stream(stream):
        e.record(stream)
    torch.cuda.synchronize()
    return s.elapsed_time(e) * 1e3 / iters


def dominant_kernel_roofline(lib, torch, dev, stream):
    """The kernel with the largest share of the loop's GPU time in the ncu
    launch list of one CartPole minibatch (profiles/launches_c3_minibatch.md):
    the residual-block backward on 4-CTA clusters, k_block_cluster<backward>,
    two launches per minibatch. Timed here at the minibatch's shape (4096 rows,
    embed 128, hidden 512) alone and back to back on the engine's stream with
    CUDA events.

    Per launch it computes four 4096 x 128 x 512 products (dV, the branch
    gradient and the two weight gradients: 2.15 GFLOP). Its algorithmic bytes
    are its inputs and outputs once each: dS, V, the LayerNorm output, x-hat
    and sigma in, both weights in, dV and the new dS out, the two weight
    gradients (fp32) and dgamma / dbeta out (13.4 MB). The 32 row tiles' fp32
    weight-gradient partials it writes for the gradient sums (16.8 MB) are
    this implementation's own traffic, reported beside the roofline, not in
    it. At the measured peaks the bytes take 2.0 us and the FLOPs 1.3 us; the
    kernel takes far longer than either, so it is latency bound (the
    `regime`), and `frac` is the fraction of the HBM roof it reaches. The
    DRAM traffic per launch comes from the committed ncu capture of the same
    launch (profiles/block_cluster_backward_4096x128x512.md)."""
    R, E, H = ENVS_PER_GPU, EMBED, EMBED * SCALE
    d = f"cuda:{dev}"
    tiles = (R + 127) // 128
    dS1 = torch.randn(R, E, device=d).bfloat16()
    dS0 = torch.empty_like(dS1)
    v = torch.relu(torch.randn(R, H, device=d)).bfloat16()
    dv = torch.empty_like(v)
    ln_out = torch.randn(R, E, device=d).bfloat16()
    xn = torch.randn(R, E, device=d).bfloat16()
    g = torch.ones(E, device=d).bfloat16()
    bt = torch.zeros(E, device=d).bfloat16()
    sd = 0.5 + torch.rand(R, device=d)
    up = (torch.randn(E, H, device=d) / E ** 0.5).bfloat16()
    dn = (torch.randn(H, E, device=d) / H ** 0.5).bfloat16()
    upp = torch.empty(tiles, E, H, device=d)
    dnp = torch.empty(tiles, H, E, device=d)
    part = torch.empty(lib.mg_layernorm_backward_num_partials(R), 2 * E, device=d)
    h = torch.randn(R, E, device=d).bfloat16()
    y = torch.empty_like(h)
    sp = ctypes.c_void_p(stream.cuda_stream)

    def launch_bwd():
        return lib.mg_block_cluster_backward(dS1.data_ptr(), dn.data_ptr(), v.data_ptr(), up.data_ptr(),
                                             dv.data_ptr(), ln_out.data_ptr(), upp.data_ptr(), dnp.data_ptr(),
                                             xn.data_ptr(), g.data_ptr(), sd.data_ptr(), dS1.data_ptr(),
                                             dS0.data_ptr(), part.data_ptr(), None, 0, None, R, sp)

    us = _time_launches(launch_bwd, torch, stream)
    flops = 4 * 2.0 * R * E * H
    # inputs: dS, lnOut, x-hat (bf16 [R][E]), V ([R][H]), sigma, W_up and W_down;
    # outputs: dS (bf16 [R][E]), dV ([R][H]), dW_up and dW_down (fp32), dgamma and dbeta
    alg_bytes = (R * E * 2 * 3 + R * H * 2 + R * 4 + 2 * E * H * 2
                 + R * E * 2 + R * H * 2 + 2 * E * H * 4 + 2 * E * 4)
    partial_bytes = 2 * tiles * E * H * 4 + part.numel() * 4
    hbm, tflops, kind = measured_peaks()
    t_mem, t_flop = alg_bytes / (hbm * 1e9), flops / (tflops * 1e12)
    achieved = alg_bytes / (us * 1e-6) / 1e9
    bound = "hbm" if t_mem >= t_flop else "tensor"
    frac = achieved / hbm if bound == "hbm" else flops / (us * 1e-6) / 1e12 / tflops
    roof = {"kernel": "k_block_cluster<backward> (residual-block backward on 4-CTA clusters: dV, branch gradient, "
                      "LayerNorm backward + skip, weight-gradient tile partials; 4096 rows, 128 x 512)",
            "bound": bound, "achieved": achieved if bound == "hbm" else flops / (us * 1e-6) / 1e12,
            "peak": hbm if bound == "hbm" else tflops, "unit": "GB/s" if bound == "hbm" else "TFLOP/s",
            "frac": frac, "peak_kind": f"{kind} " + ("HBM copy" if bound == "hbm" else "bf16 GEMM (burst)"),
            "regime": ("latency-bound: neither roof is within 2x (roof times: bytes %.2f us, FLOPs %.2f us)"
                       % (t_mem * 1e6, t_flop * 1e6)) if us * 1e-6 > 2 * max(t_mem, t_flop) else "roof-bound",
            "us_per_launch": us, "algorithmic_bytes_per_launch": alg_bytes, "flop_per_launch": flops,
            "tensor_frac": flops / (us * 1e-6) / 1e12 / tflops,
            "partial_bytes_per_launch": partial_bytes,
            "partial_bytes_note": "fp32 weight-gradient tile partials and LayerNorm partials written for the "
                                  "gradient sums: implementation traffic, not algorithmic bytes",
            "traffic": profile_traffic("block_cluster_backward_4096x128x512.md")}

    # the forward of a residual block on 4-CTA clusters (up, ReLU, down, skip,
    # the next LayerNorm), two launches per minibatch and per collect step
    def launch_fwd():
        return lib.mg_block_cluster_forward(ln_out.data_ptr(), up.data_ptr(), dn.data_ptr(), h.data_ptr(),
                                            v.data_ptr(), g.data_ptr(), bt.data_ptr(), xn.data_ptr(), y.data_ptr(),
                                            sd.data_ptr(), R, sp)

    usf = _time_launches(launch_fwd, torch, stream)
    ff = 2 * 2.0 * R * E * H
    # lnOut and h in; h, x-hat and the next LayerNorm output out (bf16 [R][E]), V
    # out ([R][H]), sigma out, both weights in
    bf = R * E * 2 * 5 + R * H * 2 + 2 * E * H * 2 + R * 4
    roof["critical_path_kernel"] = {
        "kernel": "k_block_cluster<forward> (residual block on 4-CTA clusters + next LayerNorm, 4096 x 128 x 512)",
        "bound": "hbm" if bf / (hbm * 1e9) >= ff / (tflops * 1e12) else "tensor",
        "achieved": bf / (usf * 1e-6) / 1e9, "peak": hbm, "unit": "GB/s",
        "frac": bf / (usf * 1e-6) / 1e9 / hbm, "tensor_frac": ff / (usf * 1e-6) / 1e12 / tflops,
        "us_per_launch": usf, "flop_per_launch": ff, "algorithmic_bytes_per_launch": bf,
        "traffic": profile_traffic("block_cluster_forward_4096x128x512.md")}
    return roof


def profile_traffic(name):
    """DRAM bytes per launch from a committed ncu summary under profiles/."""
    p = ROOT / "profiles" / name
    if p.exists():
        m = re.search(r"traffic_bytes_per_launch:\s*([0-9.eE+]+)", p.read_text())
        if m:
            return float(m.group(1))
    return None


# ------------------------------------------------------------------ CPU baselines

def cpu_full_loop(seconds_budget=20.0, threads=None):
    """The reference's CPU path for the full loop: its environment compiled
    from source (oracle/_ref) and the C++ restatement of its PPO arithmetic,
    OpenMP over rows on all host cores. Bounded sample: one collect() (the
    whole T-step rollout of 4096 envs) and as many of the 128 minibatches as
    fit in the budget; the iteration time is extrapolated to 128 minibatches
    (wall_s: the sample's own wall time)."""
    sys.path.insert(0, str(ROOT / "tests"))
    from orc import load_hostenv, load_oracle, load_ref, ptr, seed_words  # noqa: F401

    threads = threads or os.cpu_count()
    os.environ.setdefault("OMP_NUM_THREADS", str(threads))
    orc = load_oracle()
    ref = load_ref()
    env_lib = ref if ref is not None else load_hostenv()
    env_fn = ctypes.cast(env_lib.ref_rollout if ref is not None else env_lib.hostenv_rollout, ctypes.c_void_p)
    R, T, O = ENVS_PER_GPU, HORIZON, 4
    m = orc.orc_model_create(R, O, 2, 0, EMBED, SCALE, LAYERS, LR, T, 0)
    states = np.zeros(R * 20, np.uint8)
    done = np.ones(R, np.uint8)
    rng = seed_words(R)
    obs = np.zeros((T + 1) * R * O, np.float32)
    act = np.zeros(T * R, np.int32)
    lp, val, rew, adv, ret = (np.zeros(T * R, np.float32) for _ in range(5))
    dns = np.zeros(T * R, np.uint8)
    started = ctypes.c_int(0)
    t0 = time.perf_counter()
    orc.orc_model_collect(m, env_fn, 0, ptr(states), ptr(done), ptr(rng), ptr(obs), ptr(act), ptr(lp), ptr(val),
                          ptr(rew), ptr(dns), ptr(adv), ptr(ret), ctypes.byref(started), None, threads)
    t_collect = time.perf_counter() - t0
    stats = np.zeros((R, 5), np.float32)
    nsq = np.zeros(1, np.float32)
    n_mb, t_mb = 0, 0.0
    while n_mb < 4 * T and (n_mb < 2 or t_collect + t_mb < seconds_budget):
        t = n_mb % T
        t1 = time.perf_counter()
        orc.orc_model_train_minibatch(m, ptr(obs[t * R * O:(t + 1) * R * O]), ptr(act[t * R:(t + 1) * R]),
                                      ptr(adv[t * R:(t + 1) * R]), ptr(ret[t * R:(t + 1) * R]),
                                      ptr(lp[t * R:(t + 1) * R]), R, ptr(stats), ptr(nsq))
        t_mb += time.perf_counter() - t1
        n_mb += 1
    orc.orc_model_destroy(m)
    per_iter = t_collect + (t_mb / n_mb) * EPOCHS * T
    return {"value": R * T / per_iter, "unit": "env steps/s", "cores": threads, "wall_s": t_collect + t_mb,
            "iteration_s_extrapolated": per_iter,
            "kind": "reference" if ref is not None else "port",
            "sample": f"1 collect (4096 envs x 32 steps, {t_collect:.2f} s) + {n_mb} of 128 minibatches "
                      f"({t_mb / n_mb:.3f} s each), iteration time extrapolated",
            "env_code": "reference sources (oracle/_ref)" if ref is not None else "host build of the env port",
            "policy_code": "oracle restatement of model/ppo.h + model/*.metal"}


def run_reference(args, rank, world):
    """--impl reference: the reference's CPU path on this box's host cores.

    A whole iteration of that path takes about 20 s on 16 cores, so each step
    here is a bounded sample of one iteration (one collect() and as many
    minibatches as fit in ~8 s; cpu_full_loop), and the line says so: `steps`
    and `warmup` are the samples actually run, `ms_per_step` is a sample's
    measured wall time, and `value` is the env-step rate of the whole
    iteration extrapolated from each sample (median over the samples)."""
    if rank != 0:
        return None
    n_warm, n_timed = 1, max(1, min(args.steps, 3))
    for _ in range(n_warm):
        cpu_full_loop(seconds_budget=3.0)
    runs = [cpu_full_loop(seconds_budget=8.0) for _ in range(n_timed)]
    v = statistics.median(r["value"] for r in runs)
    wall_ms = 1e3 * statistics.mean(r["wall_s"] for r in runs)
    base = runs[len(runs) // 2]
    return {"impl": "reference", "metric": METRIC, "value": v, "unit": "env steps/s", "n_gpus": world,
            "steps": n_timed, "warmup": n_warm, "ms_per_step": wall_ms,
            "ms_per_step_kind": "wall time of one bounded sample (a collect() plus some of the 128 minibatches)",
            "ms_per_iteration_extrapolated": ENVS_PER_GPU * HORIZON / v * 1e3,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": v / REFERENCE_M4_FULL_LOOP, "dtype": "bf16",
            "data": "synthetic (simulated CartPole)",
            "config": workload_config(world),
            "setup": {"arm": "the reference's CPU path on the host cores (OpenMP), rank 0 only",
                      "requested_steps": args.steps, "requested_warmup": args.warmup},
            "cpu_baseline": {"value": v, "unit": "env steps/s", "cores": base["cores"], "kind": base["kind"],
                             "sample": base["sample"]},
            "e2e": {"value": v, "unit": "env steps/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def cpu_raw_env(seconds_budget=10.0):
    """Config 1 on the host: the reference's own sampleAction (all-zero head)
    and rollout<CartPole> compiled from source, OpenMP over envs."""
    sys.path.insert(0, str(ROOT / "tests"))
    from orc import load_ref, ptr, seed_words

    ref = load_ref()
    if ref is None:
        return None
    threads = os.cpu_count()
    n = ENVS_PER_GPU
    states = np.zeros(n * 20, np.uint8)
    obs = np.zeros(n * 16, np.uint8)
    rew = np.zeros(n, np.float32)
    done = np.ones(n, np.uint8)
    rng = seed_words(n)
    head = np.zeros((n, 64), np.uint16)
    act = np.zeros(n, np.uint32)
    lp = np.zeros(n, np.float32)
    v = np.zeros(n, np.float32)
    steps = 0
    t0 = time.perf_counter()
    while steps < RAW_STEPS and time.perf_counter() - t0 < seconds_budget:
        ref.ref_sample_action(ptr(head), ptr(rng), ptr(act), ptr(lp), ptr(v), n, 2, 64)
        ref.ref_rollout(0, ptr(states), ptr(act), ptr(obs), ptr(rew), ptr(done), ptr(rng), n, threads)
        steps += 1
    dt = time.perf_counter() - t0
    return {"value": steps * n / dt, "unit": "env steps/s", "cores": threads, "kind": "reference",
            "sample": f"{steps} steps x {n} envs (sampler single-threaded, env OpenMP)"}


# ------------------------------------------------------------------ main

def profile_minibatch(which, fused_minibatch=False):
    """Builds the configuration's model, collects once, runs one minibatch and
    one forward as warm-up, then one minibatch and one forward inside the
    profiler range (fused_minibatch: the minibatch's tile passes as one
    kernel, mg_ppo_set_fused_minibatch)."""
    import torch

    from metalgym_b200.session import Gym, PPOModel

    env, n, embed, blocks, rows = {
        "c3": (ENV, ENVS_PER_GPU, EMBED, LAYERS, 0),
        "c4": ("rollout_cartpole_continuous", 16384, 128, 2, 8192),
        "c5": ("rollout_voxelnav", 262144, 256, 4, 32768)}[which]
    gym = Gym(env, n, seed=0)
    model = PPOModel(gym, embed, SCALE, blocks, LR, HORIZON, seed=0)
    model.minibatch_rows = rows
    model.fused_minibatch = fused_minibatch
    model.collect()

    def minibatch(k):
        if rows:
            model.train_rows([1, 2, 3, 4], k * rows)
        else:
            model.train_slot(k % HORIZON)

    minibatch(0)
    model.forward()
    torch.cuda.synchronize()
    torch.cuda.profiler.start()
    minibatch(1)
    model.forward()
    torch.cuda.synchronize()
    torch.cuda.profiler.stop()


def profile_collect():
    """The configs[1] model (4096 CartPole envs, T = 32): one collect() as
    warm-up, then one collect() inside the profiler range (the library's
    default path: the fused collect kernel)."""
    import torch

    from metalgym_b200.session import Gym, PPOModel

    gym = Gym(ENV, ENVS_PER_GPU, seed=0)
    model = PPOModel(gym, EMBED, SCALE, LAYERS, LR, HORIZON, seed=0)
    model.collect()
    torch.cuda.synchronize()
    torch.cuda.profiler.start()
    model.collect()
    torch.cuda.synchronize()
    torch.cuda.profiler.stop()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["mine", "reference"], default="mine")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extra-legs", action="store_true", help="skip the configs[3] / configs[4] loops")
    ap.add_argument("--allreduce", choices=["nccl", "p2p"], default="p2p",
                    help="N > 1: gradient all-reduce with the library's own kernel over NVLink peer memory "
                         "(default, at every N: measured faster than NCCL at 2 and 8 GPUs) or with NCCL")
    ap.add_argument("--allreduce-overlap", action="store_true",
                    help="N > 1 with NCCL: all-reduce all but the last backward layer's gradients on a side "
                         "stream while that layer's backward runs (default: one all-reduce after the backward)")
    ap.add_argument("--c4-action", choices=["clamp", "tanh"], default="clamp",
                    help="configs[3] leg: the reference code's clamped force (default) or the BASELINE text's "
                         "tanh-squashed one (rollout_cartpole_continuous_tanh)")
    ap.add_argument("--collect", choices=["auto", "graph", "fused"], default="auto",
                    help="collect(): the library's choice (default: the persistent kernel of collect_fused.cu "
                         "where it applies, up to 4096 envs), the captured per-step graph, or the kernel")
    ap.add_argument("--fused-minibatch", action="store_true",
                    help="a minibatch's block forwards, head and block backwards as one kernel "
                         "(mg_ppo_set_fused_minibatch; default: the separate kernels)")
    ap.add_argument("--profile-minibatch", choices=["c3", "c4", "c5"],
                    help="profiling driver: one training minibatch and one forward of that configuration, "
                         "bracketed by cudaProfilerStart / Stop (for ncu --profile-from-start off); no JSON line")
    ap.add_argument("--profile-collect", action="store_true",
                    help="profiling driver: one collect() of the configs[1] model inside the profiler range")
    args = ap.parse_args()
    if args.allreduce_overlap:
        args.allreduce = "nccl"  # the overlapped all-reduce is NCCL's
    if args.profile_minibatch:
        profile_minibatch(args.profile_minibatch, args.fused_minibatch)
        return
    if args.profile_collect:
        profile_collect()
        return
    args.warmup = max(3, args.warmup)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    dist = None
    if args.impl == "reference":
        out = run_reference(args, rank, world)
        if out is not None:
            print(json.dumps(out), flush=True)
        return
    if world > 1:
        import datetime

        import torch
        import torch.distributed as tdist

        torch.cuda.set_device(local_rank)
        tdist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                 device_id=torch.device(f"cuda:{local_rank}"))
        dist = tdist
    result = run_mine(args, rank, world, local_rank, dist)
    if rank == 0 and result is not None:
        if world == 1 and not args.no_cpu_baseline:
            result["cpu_baseline"] = cpu_full_loop()
            raw = cpu_raw_env()
            if raw is not None:
                result["legs"]["raw_env"]["cpu_baseline"] = raw
        print(json.dumps(result), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
