"""collect() as one persistent kernel (mg_ppo_set_collect_fused,
metalgym_b200/csrc/collect_fused.cu) against the captured per-step graph.

Both run the same products with the same K split, the same row epilogues,
samplers and environment code, so up to 4096 parallels (where the per-step
graph uses the cluster block kernels) the rollouts must be bit-identical:
every slot (obs, actions, log-probs, values, rewards, dones, advantages,
returns), the bootstrap head rows, the per-slot advantage statistics and the
gym's env states / RNG words / done flags after collect(). Several collect()
calls in a row with a train() between them check the carried state and the
updated weights. A teacher-forced replay of the fused rollout against the
CPU oracle checks it against the reference independently of the graph path.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

SLOTS = ("obs", "actions", "logp", "value", "reward", "done", "adv", "ret")


def make(name, R, L, T, seed=0, fused=False, embed=128, scale=4):
    from metalgym_b200.session import Gym, PPOModel

    gym = Gym(name, R, seed=0)
    model = PPOModel(gym, embed, scale, L, 3e-4, T, seed)
    if embed == 128 and scale == 4 and name != "rollout_voxelnav":
        model.collect_fused = fused
    return gym, model


def assert_same_rollout(ref, fused, it):
    (g1, m1), (g2, m2) = ref, fused
    for name in SLOTS:
        a, b = m1.slots(name), m2.slots(name)
        assert np.array_equal(a.view(np.uint8), b.view(np.uint8)), f"collect {it}: slot {name}"
    for name in ("head", "adv_stats"):
        assert np.array_equal(m1.download(name), m2.download(name)), f"collect {it}: {name}"
    for name in ("states", "rng", "done"):
        assert np.array_equal(g1.download(name), g2.download(name)), f"collect {it}: gym {name}"


def test_unsupported_configurations_are_rejected(mg):
    """No fused kernel for VoxelNav (a 1 KB state, 40 observations, embed 256)
    or for widths other than embed 128 / hidden 512: MG_ERR_UNSUPPORTED, and
    the model keeps the per-step graph."""
    from metalgym_b200 import MgError

    for name, embed, scale in [("rollout_voxelnav", 256, 4), ("rollout_cartpole", 64, 4),
                               ("rollout_cartpole", 128, 2)]:
        _, model = make(name, 256, 1, 2, embed=embed, scale=scale)
        with pytest.raises(MgError, match="code 3"):  # MG_ERR_UNSUPPORTED
            model.collect_fused = True
        assert model.collect_fused is False
    _, model = make("rollout_cartpole", 256, 2, 2)
    model.collect_fused = True
    assert model.collect_fused is True
    model.collect_fused = False
    assert model.collect_fused is False
    model.collect_fused = None  # the library's choice: the kernel, at 256 parallels
    assert model.collect_fused is True


def test_automatic_choice(mg):
    """Without a choice, collect() runs the kernel where it applies up to 4096
    parallels (one wave of clusters) and the per-step graph above."""
    from metalgym_b200.session import Gym, PPOModel

    for R, want in [(4096, True), (4097, False)]:
        model = PPOModel(Gym("rollout_cartpole", R), 128, 4, 2, 3e-4, 2, 0)
        assert model.collect_fused is want, R
    model = PPOModel(Gym("rollout_cartpole", 512), 64, 4, 2, 3e-4, 2, 0)
    assert model.collect_fused is False


@pytest.mark.parametrize("name,R,L,T", [("rollout_cartpole", 4096, 2, 32), ("rollout_cartpole", 1000, 1, 8),
                                        ("rollout_cartpole_continuous", 2048, 2, 16),
                                        ("rollout_cartpole", 300, 4, 3)])
def test_fused_collect_is_bit_identical_to_the_step_graph(mg, name, R, L, T):
    ref = make(name, R, L, T, seed=3)
    fused = make(name, R, L, T, seed=3, fused=True)
    for it in range(3):
        ref[1].collect()
        fused[1].collect()
        assert_same_rollout(ref, fused, it)
        assert fused[1].graph_kernels()[0] == 2  # the fused kernel and the advantage statistics
        ref[1].train(1)
        fused[1].train(1)
        assert np.array_equal(ref[1].download("master"), fused[1].download("master")), f"train after collect {it}"


@pytest.mark.parametrize("name,R,T", [("rollout_cartpole", 1024, 8), ("rollout_cartpole_continuous", 512, 6)])
def test_fused_collect_teacher_forced(mg, oracle, hostenv, name, R, T):
    from test_engine import replay_collect

    _, model = make(name, R, 2, T, seed=1, fused=True)
    model.collect()
    replay_collect(oracle, hostenv, model, name, 1)


def test_fused_collect_can_be_switched_between_calls(mg):
    """Switching paths between collect() calls recaptures the collect graph and
    continues the same rollout."""
    ref = make("rollout_cartpole", 512, 2, 4, seed=5)
    mixed = make("rollout_cartpole", 512, 2, 4, seed=5)
    for it, on in enumerate([True, False, True]):
        mixed[1].collect_fused = on
        ref[1].collect()
        mixed[1].collect()
        assert_same_rollout(ref, mixed, it)


@pytest.mark.parametrize("name", ["rollout_test_walk", "rollout_test_glide"])
def test_fused_collect_of_a_user_environment(mg, tmp_path, name):
    """A user environment built against the public headers alone (the walk and
    glide environments of tests/test_env_register.py) runs its own
    instantiation of the fused kernel: bit-identical to the per-step graph."""
    import ctypes
    import subprocess

    from test_env_register import LIB_DIR, NVCC, ROOT, USER_ENV

    src = tmp_path / "walk.cu"
    src.write_text(USER_ENV)
    so = tmp_path / "libwalk.so"
    r = subprocess.run([NVCC, "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-std=c++17", "--fmad=false",
                        "-Xcompiler", "-fPIC", "-shared", "-I", str(ROOT / "include"), str(src), "-o", str(so),
                        "-L", str(LIB_DIR), "-lmetalgym_b200", f"-Xlinker=-rpath,{LIB_DIR}"],
                       capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    ctypes.CDLL(str(so))
    ref = make(name, 640, 2, 8, seed=2)
    fused = make(name, 640, 2, 8, seed=2, fused=True)
    for it in range(2):
        ref[1].collect()
        fused[1].collect()
        assert_same_rollout(ref, fused, it)


@pytest.mark.parametrize("name,L", [("rollout_cartpole", 2), ("rollout_cartpole_continuous", 3)])
def test_c_entry_point_on_session_buffers(mg, name, L):
    """mg_env_collect_fused on the buffers of a PPO session (weights located
    by mg_ppo_param_info, slots and env buffers by mg_ppo_buffer /
    mg_gym_buffer) continues the rollout exactly as the session's own
    collect() does."""
    import ctypes

    import metalgym_b200
    from metalgym_b200 import CollectFusedArgs

    R, T = 768, 6
    ref = make(name, R, L, T, seed=6)
    mine = make(name, R, L, T, seed=6)
    ref[1].collect()
    mine[1].collect()
    gym, model = mine
    # the session's next collect() starts from the last observation slot
    model.upload("obs", model.download("obs", T), 0)
    w, _ = model.buffer("weights")
    par = lambda i: w + 2 * model.param_info(i)[0]  # bf16 weights
    a = CollectFusedArgs(parallels=R, horizon=T, layers=L, obs_dim=model.obs_dim, gamma=0.99, lambda_=0.95)
    a.w_in, a.b_in = par(0), par(1)
    for n in range(L):
        a.ln_gamma[n], a.ln_beta[n], a.w_up[n], a.w_down[n] = (par(2 + 4 * n + k) for k in range(4))
    a.ln_gamma[L], a.ln_beta[L], a.w_head = par(2 + 4 * L), par(3 + 4 * L), par(4 + 4 * L)
    a.log_std = par(5 + 4 * L) if model.continuous else None
    a.states, a.done, a.rng = (gym.buffer(k)[0] for k in ("states", "done", "rng"))
    a.obs_slots, a.action_slots, a.logp_slots, a.value_slots = (model.buffer(k)[0]
                                                                 for k in ("obs", "actions", "logp", "value"))
    a.reward_slots, a.done_slots, a.adv_slots, a.ret_slots = (model.buffer(k)[0]
                                                              for k in ("reward", "done", "adv", "ret"))
    a.boot_head = model.buffer("head")[0]
    metalgym_b200.check(metalgym_b200.lib().mg_env_collect_fused(name.encode(), ctypes.byref(a), gym.stream()),
                        "mg_env_collect_fused")
    gym.synchronize()
    ref[1].collect()
    for k in SLOTS:
        assert np.array_equal(ref[1].slots(k).view(np.uint8), model.slots(k).view(np.uint8)), k
    assert np.array_equal(ref[1].download("head"), model.download("head"))
    for k in ("states", "rng", "done"):
        assert np.array_equal(ref[0].download(k), gym.download(k)), k
