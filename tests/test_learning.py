"""Learning curves of the CartPole PPO loop against the CPU reference path.

tests/golden/learning_curves.npz and learning_curves_c3.npz hold the mean
episode length per iteration (envs x T / number of done flags of the
rollout) for five seeds of the reference's environment code with the C++
restatement of its PPO arithmetic (tests/golden/make_learning_curves.py):
1024 envs, T = 32, embed 64, hidden 256, 2 blocks, train(4), 15 iterations;
and BASELINE configs[2]'s shape, 4096 envs, T = 32, embed 128, hidden 512,
2 blocks, train(4), 20 iterations. The GPU runs the same five seeds
(same initial weights, env seeds and slot shuffles). Training trajectories
diverge once a sampled action differs, so the comparison is statistical.
The band:

* iteration 0 (the initial policy, before any update): the GPU mean over the
  seeds within 10% of the reference mean;
* every iteration: the GPU mean over the seeds inside the reference runs'
  envelope [0.6 x min, 1.5 x max];
* the last five iterations: the GPU mean within a factor 1.5 of the
  reference mean, and both above 1.5 x their iteration-0 value (learning).
"""
import ast
from pathlib import Path

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden"


@pytest.mark.parametrize("fixture", ["learning_curves.npz", "learning_curves_c3.npz"])
def test_learning_curves_within_reference_band(mg, fixture):
    from metalgym_b200.session import Gym, PPOModel

    if not (GOLDEN / fixture).exists():
        pytest.skip(f"{fixture} not generated (tests/golden/make_learning_curves.py)")
    g = np.load(GOLDEN / fixture)
    ref = g["lengths"]
    cfg = ast.literal_eval(str(g["config"][0]))
    gpu = []
    for s in cfg["seeds"]:
        gym = Gym("rollout_cartpole", cfg["envs"], seed=s)
        model = PPOModel(gym, cfg["embed"], cfg["scale"], cfg["layers"], cfg["lr"], cfg["horizon"], s)
        lengths = []
        for _ in range(cfg["iterations"]):
            model.collect()
            done = model.slots("done")
            lengths.append(done.size / max(1, int(done.sum())))
            model.train(cfg["epochs"])
        gpu.append(lengths)
        model.close()
        gym.close()
    gpu = np.array(gpu)
    print("reference mean", np.round(ref.mean(0), 1))
    print("gpu mean      ", np.round(gpu.mean(0), 1))
    assert abs(gpu[:, 0].mean() - ref[:, 0].mean()) <= 0.1 * ref[:, 0].mean()
    lo, hi = 0.6 * ref.min(0), 1.5 * ref.max(0)
    m = gpu.mean(0)
    assert np.all((m >= lo) & (m <= hi)), (m, lo, hi)
    last_ref, last_gpu = ref[:, -5:].mean(), gpu[:, -5:].mean()
    assert last_ref / 1.5 <= last_gpu <= last_ref * 1.5, (last_gpu, last_ref)
    assert last_gpu > 1.5 * gpu[:, 0].mean() and last_ref > 1.5 * ref[:, 0].mean()
