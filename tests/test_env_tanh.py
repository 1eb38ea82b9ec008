"""CartPoleContinuousTanh: the BASELINE text's tanh-squashed continuous
CartPole (registered as rollout_cartpole_continuous_tanh; the reference code,
and CartPoleContinuous, clamp the action instead).

It has no reference counterpart, so it is pinned through one that has: with
action a it must step exactly as the reference-pinned CartPoleContinuous
stepped with action tanh(a) (|tanh a| < 1, so the clamp changes nothing). CPU:
the project's own tanh (mathf.h) within one float ulp of the correctly rounded
value, and that equivalence on the host build. GPU: the device build steps
bit for bit as the host build, and a short PPO loop runs on it.
"""
import numpy as np
import pytest

from orc import ENV_IDS, ptr, seed_words

TANH_ID = 3  # tests/helpers/host_envs.cpp
CLAMP_ID = ENV_IDS["rollout_cartpole_continuous"]


def ulps(a, b):
    a, b = np.float32(a), np.float32(b)
    return abs(int(a.view(np.int32)) - int(b.view(np.int32)))


def test_own_tanh_accuracy(hostenv):
    rs = np.random.default_rng(5)
    xs = np.concatenate([rs.uniform(-12, 12, 6000), rs.uniform(-0.01, 0.01, 2000), rs.uniform(-60, 60, 500),
                         [1e-30, -1e-30, 1e-8, 0.3465, -0.3466, 9.0, -9.1, 20.0, 25.0, -300.0]]).astype(np.float32)
    for x in xs:
        assert ulps(hostenv.hostenv_tanhf(float(x)), np.tanh(np.float64(x))) <= 1, x
    assert np.float32(hostenv.hostenv_tanhf(0.0)).view(np.uint32) == 0
    assert np.float32(hostenv.hostenv_tanhf(-0.0)).view(np.uint32) == 0x80000000
    assert np.isnan(hostenv.hostenv_tanhf(float("nan")))
    assert hostenv.hostenv_tanhf(float("inf")) == 1.0 and hostenv.hostenv_tanhf(float("-inf")) == -1.0


def _host_rollout(hostenv, which, actions, n, steps):
    hs = np.zeros(n * 20, np.uint8)
    ho = np.zeros((n, 4), np.float32)
    hr = np.zeros(n, np.float32)
    hd = np.ones(n, np.uint8)
    hg = seed_words(n, seed=3)
    trace = []
    for t in range(steps):
        a = np.ascontiguousarray(actions[t])
        hostenv.hostenv_rollout(which, ptr(hs), ptr(a), ptr(ho), ptr(hr), ptr(hd), ptr(hg), n, 4)
        trace.append((ho.copy(), hr.copy(), hd.copy()))
    return trace, hs, hg


def test_tanh_variant_steps_as_the_clamp_env_on_tanh_actions(hostenv):
    n, steps = 2048, 200
    rs = np.random.default_rng(9)
    a = (rs.standard_normal((steps, n, 1)) * 2.0).astype(np.float32)
    squashed = np.vectorize(lambda x: np.float32(hostenv.hostenv_tanhf(float(x))), otypes=[np.float32])(a)
    tr_tanh, s1, g1 = _host_rollout(hostenv, TANH_ID, a, n, steps)
    tr_clamp, s2, g2 = _host_rollout(hostenv, CLAMP_ID, squashed, n, steps)
    for t, ((o1, r1, d1), (o2, r2, d2)) in enumerate(zip(tr_tanh, tr_clamp)):
        assert np.array_equal(o1.view(np.uint32), o2.view(np.uint32)), t
        assert np.array_equal(r1, r2) and np.array_equal(d1, d2), t
    assert np.array_equal(s1, s2) and np.array_equal(g1, g2)
    # and it differs from the clamp env on the raw actions (large |a| saturate differently)
    tr_raw, _, _ = _host_rollout(hostenv, CLAMP_ID, a, n, steps)
    assert not np.array_equal(tr_raw[-1][0], tr_tanh[-1][0])


@pytest.mark.gpu
def test_device_steps_as_host(mg, hostenv):
    import torch

    from test_kernels import dev, host, ok, sync_status

    name, n, steps = "rollout_cartpole_continuous_tanh", 4096, 200
    rs = np.random.default_rng(21)
    hs = np.zeros(n * 20, np.uint8)
    ho = np.zeros(n * 16, np.uint8)
    hr = np.zeros(n, np.float32)
    hd = np.ones(n, np.uint8)
    hg = seed_words(n, seed=4, first=0)
    st = torch.zeros(n * 20, dtype=torch.uint8, device="cuda")
    obs = torch.zeros(n * 16, dtype=torch.uint8, device="cuda")
    rew = torch.zeros(n, dtype=torch.float32, device="cuda")
    done = torch.zeros(n, dtype=torch.uint8, device="cuda")
    rng = torch.zeros(n, dtype=torch.int32, device="cuda")
    ok(mg, mg.mg_env_init(name.encode(), st.data_ptr(), done.data_ptr(), rng.data_ptr(), n, 4, 0, None))
    for t in range(steps):
        a = (rs.standard_normal((n, 1)) * 2.0).astype(np.float32)
        da = dev(a)
        ok(mg, mg.mg_env_step(name.encode(), st.data_ptr(), da.data_ptr(), obs.data_ptr(), rew.data_ptr(),
                              done.data_ptr(), None, rng.data_ptr(), n, None))
        hostenv.hostenv_rollout(TANH_ID, ptr(hs), ptr(a), ptr(ho), ptr(hr), ptr(hd), ptr(hg), n, 8)
        assert np.array_equal(host(obs, np.uint8), ho), f"obs step {t}"
        assert np.array_equal(host(rew, np.uint32), hr.view(np.uint32)) and np.array_equal(host(done, np.uint8), hd)
    sync_status(mg)
    assert np.array_equal(host(st, np.uint8), hs) and np.array_equal(host(rng, np.uint32), hg)


@pytest.mark.gpu
def test_ppo_loop_runs_on_the_tanh_variant(mg):
    from metalgym_b200.session import Gym, PPOModel

    gym = Gym("rollout_cartpole_continuous_tanh", 1024, seed=0)
    model = PPOModel(gym, 128, 4, 2, 3e-4, 8, 0)
    for _ in range(2):
        model.collect()
        model.train(2)
    st = model.last_stats()
    assert all(np.isfinite(v) for v in st.values()), st
    model.close()
    gym.close()
