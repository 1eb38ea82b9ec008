"""Generates tests/golden/learning_curves.npz (and, with `c3`,
tests/golden/learning_curves_c3.npz): mean episode length per iteration of
the CartPole PPO loop on the CPU reference path, for five seeds.

The environment is the reference's own code (oracle/_ref, built from the
reference sources) when available, else the host build of the environment
port (bit-identical); the policy, sampler, GAE and PPO update are the C++
restatement in oracle/. Configuration: 1024 envs, T = 32, embed 64, hidden
256, 2 blocks, lr 3e-4, train(4) per iteration, one-slot minibatches,
15 iterations; seed s drives the env seeds (gym seed s) and the model
(initial weights and slot shuffle). Mean episode length of an iteration =
envs x T / (number of done flags in the rollout) (examples/CartPoleContinuous/
main.cpp:33-39).

`c3` is BASELINE configs[2]'s shape instead: 4096 envs, T = 32, embed 128,
hidden 512, 2 blocks, train(4), 20 iterations (the reference's own CartPole
driver trains 40 iterations of that shape, examples/CartPole/main.cpp:20-34).

    python tests/golden/make_learning_curves.py      (about a minute per seed)
    python tests/golden/make_learning_curves.py c3   (about 15 minutes per seed on 8 cores)
"""
import ctypes
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent))
from orc import load_hostenv, load_oracle, load_ref, ptr, seed_words  # noqa: E402

CONFIGS = {
    "small": (dict(envs=1024, horizon=32, embed=64, scale=4, layers=2, lr=3e-4, epochs=4, iterations=15,
                   seeds=(0, 1, 2, 3, 4)), "learning_curves.npz"),
    "c3": (dict(envs=4096, horizon=32, embed=128, scale=4, layers=2, lr=3e-4, epochs=4, iterations=20,
                seeds=(0, 1, 2, 3, 4)), "learning_curves_c3.npz"),
}
CFG = CONFIGS["small"][0]


def curve(orc, env_fn, seed, threads):
    R, T, O = CFG["envs"], CFG["horizon"], 4
    m = orc.orc_model_create(R, O, 2, 0, CFG["embed"], CFG["scale"], CFG["layers"], CFG["lr"], T, seed)
    states = np.zeros(R * 20, np.uint8)
    done = np.ones(R, np.uint8)
    rng = seed_words(R, seed=seed)
    obs = np.zeros((T + 1) * R * O, np.float32)
    act = np.zeros(T * R, np.int32)
    lp, val, rew, adv, ret = (np.zeros(T * R, np.float32) for _ in range(5))
    dns = np.zeros(T * R, np.uint8)
    started = ctypes.c_int(0)
    lengths, stats = [], []
    for _ in range(CFG["iterations"]):
        orc.orc_model_collect(m, env_fn, 0, ptr(states), ptr(done), ptr(rng), ptr(obs), ptr(act), ptr(lp),
                              ptr(val), ptr(rew), ptr(dns), ptr(adv), ptr(ret), ctypes.byref(started), None,
                              threads)
        lengths.append(R * T / max(1, int(dns.sum())))
        st = np.zeros(6, np.float32)
        orc.orc_model_train(m, ptr(obs), ptr(act), ptr(lp), ptr(adv), ptr(ret), CFG["epochs"], ptr(st))
        stats.append(st)
    orc.orc_model_destroy(m)
    return np.array(lengths), np.array(stats)


def main():
    global CFG
    which = sys.argv[1] if len(sys.argv) > 1 else "small"
    CFG, out_name = CONFIGS[which]
    threads = os.cpu_count()
    os.environ.setdefault("OMP_NUM_THREADS", str(threads))
    orc = load_oracle()
    ref = load_ref()
    env_lib = ref if ref is not None else load_hostenv()
    env_fn = ctypes.cast(env_lib.ref_rollout if ref is not None else env_lib.hostenv_rollout, ctypes.c_void_p)
    curves, stats = [], []
    for s in CFG["seeds"]:
        c, st = curve(orc, env_fn, s, threads)
        print(f"seed {s}: " + " ".join(f"{x:.1f}" for x in c), flush=True)
        curves.append(c)
        stats.append(st)
    np.savez(HERE / out_name, lengths=np.array(curves), stats=np.array(stats),
             config=np.array([repr(CFG)]), env_code=np.array(["reference" if ref is not None else "port"]))


if __name__ == "__main__":
    main()
