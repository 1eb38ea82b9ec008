"""The PPO engine (collect / train through the mg_ppo_* C ABI) vs the oracle.

collect() is checked by a teacher-forced replay on the CPU: the oracle model
(same seed, hence bit-identical initial weights) runs the forward pass on
the GPU's observation slots, the host build of the environment steps with
the GPU's actions, and the reference's GAE runs on the GPU's rewards / dones
/ values. Env outputs, RNG words and GAE are bit-exact; values / log-probs
come from bf16 GEMMs with a different accumulation order and must agree
within rel 1e-2 (BF16 operands, fp32 accumulation); sampled actions may
differ only where the oracle's logits move a draw across a CDF boundary
(< 1% of rows).

trainSlot(t) is checked against the oracle's minibatch on identical state:
loss statistics rel 1e-2, per-parameter gradients relative L2 error < 3e-2,
Adam update direction agreeing on > 97% of the weights with a clear gradient.
"""
import ctypes

import numpy as np
import pytest

from orc import ENV_IDS, ENV_SIZES, bf16_to_f32, ptr, seed_words

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

HEAD = 64


def make(name, R, E, s, L, T, seed=0, lr=3e-4):
    from metalgym_b200.session import Gym, PPOModel

    gym = Gym(name, R, seed=0)
    model = PPOModel(gym, E, s, L, lr, T, seed)
    return gym, model


def oracle_model(oracle, model, seed):
    ad = model.act_dim
    return oracle.orc_model_create(model.rows, model.obs_dim, ad, int(model.continuous), model.embed,
                                   model.hidden // model.embed, model.layers, 3e-4, model.horizon, seed)


def arr(oracle, fn, m, n, dtype):
    p = getattr(oracle, fn)(m)
    return np.ctypeslib.as_array(ctypes.cast(p, ctypes.POINTER(np.ctypeslib.as_ctypes_type(dtype))), shape=(n,))


@pytest.mark.parametrize("name", ["rollout_cartpole", "rollout_cartpole_continuous", "rollout_voxelnav"])
def test_init_and_layout_match_reference_restatement(mg, oracle, name):
    gym, model = make(name, 256, 128, 4, 2, 4, seed=3)
    om = oracle_model(oracle, model, 3)
    assert oracle.orc_model_opt_count(om) == model.opt_count
    assert oracle.orc_model_opt_float_count(om) == model.opt_float_count
    for i in range(model.param_count):
        o, c, g = ctypes.c_uint32(), ctypes.c_uint32(), ctypes.c_int()
        oracle.orc_model_param_info(om, i, ctypes.byref(o), ctypes.byref(c), ctypes.byref(g))
        assert model.param_info(i) == (o.value, c.value, bool(g.value))
    n = model.opt_count
    assert np.array_equal(model.download("weights").view(np.uint16), arr(oracle, "orc_model_weights", om, n, np.uint16))
    assert np.array_equal(model.download("master").view(np.float32), arr(oracle, "orc_model_master", om, n, np.float32))
    oracle.orc_model_destroy(om)


def replay_collect(oracle, hostenv, model, name, seed):
    """Teacher-forced CPU replay of one collect() from a fresh gym."""
    which = ENV_IDS[name]
    sb, ab, ob, od, ad, cont = ENV_SIZES[name]
    R, T = model.rows, model.horizon
    obs = model.slots("obs")
    act = model.slots("actions")
    logp = model.slots("logp")
    val = model.slots("value")
    rew = model.slots("reward")
    done = model.slots("done")
    adv = model.slots("adv")
    ret = model.slots("ret")
    om = oracle_model(oracle, model, seed)
    hs = np.zeros(R * sb, np.uint8)
    hd = np.ones(R, np.uint8)
    hg = seed_words(R)
    ho = np.zeros((R, od), np.float32)
    hr = np.zeros(R, np.float32)
    zero = np.zeros((R, ad), np.float32) if cont else np.zeros(R, np.int32)
    hostenv.hostenv_rollout(which, ptr(hs), ptr(zero), ptr(ho), ptr(hr), ptr(hd), ptr(hg), R, 8)
    assert np.array_equal(obs[0].view(np.uint32), ho.view(np.uint32)), "first obs slot"
    head = np.zeros((R, HEAD), np.uint16)
    mismatched = 0
    logstd = None
    if cont:
        off, cnt, _ = model.param_info(model.param_count - 1)
        logstd = model.download("weights").view(np.uint16)[off:off + cnt].copy()
    for t in range(T):
        oracle.orc_model_forward(om, ptr(np.ascontiguousarray(obs[t])), R, ptr(head))
        hv = bf16_to_f32(head[:, ad])
        np.testing.assert_allclose(val[t], hv, rtol=1e-2, atol=1e-2 * max(1.0, np.abs(hv).max()))
        a_gpu = np.ascontiguousarray(act[t])
        lp = np.zeros(R, np.float32)
        v = np.zeros(R, np.float32)
        if cont:
            a_or = np.zeros((R, ad), np.float32)
            oracle.orc_sample_gaussian(ptr(head), ptr(hg), ptr(a_or), ptr(lp), ptr(v), R, ad, HEAD, ptr(logstd))
            np.testing.assert_allclose(a_or, a_gpu, rtol=1e-2, atol=2e-2)
        else:
            a_or = np.zeros(R, np.int32)
            oracle.orc_sample_action(ptr(head), ptr(hg), ptr(a_or), ptr(lp), ptr(v), R, ad, HEAD)
            mismatched += int((a_or != a_gpu).sum())
            same = a_or == a_gpu
            np.testing.assert_allclose(logp[t][same], lp[same], rtol=1e-2, atol=2e-2)
        # the env steps with the GPU's actions (teacher forcing): bit-exact
        hostenv.hostenv_rollout(which, ptr(hs), ptr(a_gpu), ptr(ho), ptr(hr), ptr(hd), ptr(hg), R, 8)
        assert np.array_equal(obs[t + 1].view(np.uint32), ho.view(np.uint32)), f"obs slot {t + 1}"
        assert np.array_equal(rew[t].view(np.uint32), hr.view(np.uint32)), f"reward slot {t}"
        assert np.array_equal(done[t], hd), f"done slot {t}"
    if not cont:
        assert mismatched <= max(2, 0.01 * R * T), f"{mismatched} sampled actions differ"
    # bootstrap value and the reference GAE on the GPU's buffers: bit-exact
    gpu_head = model.download("head").view(np.uint16).reshape(R, HEAD)
    oracle.orc_model_forward(om, ptr(np.ascontiguousarray(obs[T])), R, ptr(head))
    boot = bf16_to_f32(gpu_head[:, ad]).copy()
    np.testing.assert_allclose(boot, bf16_to_f32(head[:, ad]), rtol=1e-2, atol=1e-2)
    hadv = np.zeros(T * R, np.float32)
    hret = np.zeros(T * R, np.float32)
    hyper = model.hyper()
    oracle.orc_gae(ptr(rew), ptr(done), ptr(np.ascontiguousarray(val)), ptr(boot), ptr(hadv), ptr(hret), R, T,
                   hyper["gamma"], hyper["lambda"])
    assert np.array_equal(adv.reshape(-1).view(np.uint32), hadv.view(np.uint32))
    assert np.array_equal(ret.reshape(-1).view(np.uint32), hret.view(np.uint32))
    # the env's RNG words after T draws + resets
    assert np.array_equal(model.gym.download("rng").view(np.uint32), hg)
    oracle.orc_model_destroy(om)


@pytest.mark.parametrize("name,R,T", [("rollout_cartpole", 1024, 8), ("rollout_cartpole_continuous", 512, 6),
                                      ("rollout_voxelnav", 256, 4)])
def test_collect_teacher_forced(mg, oracle, hostenv, name, R, T):
    gym, model = make(name, R, 128, 4, 2, T, seed=1)
    model.collect()
    replay_collect(oracle, hostenv, model, name, 1)
    # per-slot advantage statistics (model/gae.metal:42-77)
    st = model.download("adv_stats").view(np.float32).reshape(T, 2)
    a = model.slots("adv").astype(np.float64)
    np.testing.assert_allclose(st[:, 0], a.mean(1), rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(st[:, 1], 1.0 / (a.std(1) + 1e-8), rtol=1e-4)


def test_second_collect_continues_from_last_obs(mg):
    gym, model = make("rollout_cartpole", 512, 128, 4, 1, 4)
    model.collect()
    last = model.slots("obs")[4].copy()
    model.collect()
    assert np.array_equal(model.slots("obs")[0], last)


def copy_optimiser_state(oracle, om, model):
    n = model.opt_count
    for fn, buf, dt in [("orc_model_weights", "weights", np.uint16), ("orc_model_master", "master", np.float32),
                        ("orc_model_momentum", "momentum", np.float32), ("orc_model_variance", "variance", np.float32)]:
        arr(oracle, fn, om, n, dt)[:] = model.download(buf).view(dt)


def compare_minibatch(oracle, om, model, stats, nsq, m0):
    """The GPU's last minibatch (statistics, gradient, Adam step) against the
    oracle's on the same rows and optimiser state."""
    n = model.opt_count
    ls = model.last_stats()
    ref = stats.mean(0)
    for k, key in enumerate(("policy", "value", "entropy", "approxKl", "clipFrac")):
        np.testing.assert_allclose(ls[key], ref[k], rtol=2e-2, atol=2e-3, err_msg=key)
    np.testing.assert_allclose(ls["gradNorm"], np.sqrt(nsq[0]), rtol=2e-2)
    g_gpu = model.download("grad").view(np.float32)
    g_orc = arr(oracle, "orc_model_grad", om, n, np.float32)
    for i in range(model.param_count):
        off, cnt, _ = model.param_info(i)
        a, b = g_gpu[off:off + cnt], g_orc[off:off + cnt]
        err = np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-12)
        assert err < 3e-2, f"param {i}: relative gradient error {err:.3g}"
    m1 = model.download("master").view(np.float32)
    o1 = arr(oracle, "orc_model_master", om, n, np.float32)
    clear = np.abs(g_orc) > 1e-3 * np.abs(g_orc).max()
    agree = (np.sign(m1 - m0) == np.sign(o1 - m0))[clear].mean()
    assert agree > 0.97, agree
    assert model.step_counter() == oracle.orc_model_step_counter(om)


@pytest.mark.parametrize("name", ["rollout_cartpole", "rollout_cartpole_continuous"])
def test_train_slot_matches_oracle(mg, oracle, name):
    R, T, E, s, L = 1024, 4, 128, 4, 2
    gym, model = make(name, R, E, s, L, T, seed=2)
    model.collect()
    om = oracle_model(oracle, model, 2)
    copy_optimiser_state(oracle, om, model)
    t = 2
    obs = np.ascontiguousarray(model.slots("obs")[t])
    act = np.ascontiguousarray(model.slots("actions")[t])
    adv = np.ascontiguousarray(model.slots("adv")[t])
    ret = np.ascontiguousarray(model.slots("ret")[t])
    logp = np.ascontiguousarray(model.slots("logp")[t])
    stats = np.zeros((R, 5), np.float32)
    nsq = np.zeros(1, np.float32)
    m0 = model.download("master").view(np.float32).copy()
    oracle.orc_model_set_step_counter(om, model.step_counter())
    oracle.orc_model_train_minibatch(om, ptr(obs), ptr(act), ptr(adv), ptr(ret), ptr(logp), R, ptr(stats), ptr(nsq))
    model.train_slot(t)
    compare_minibatch(oracle, om, model, stats, nsq, m0)
    oracle.orc_model_destroy(om)


def test_fused_head_loss_matches_standalone_loss(mg):
    """The categorical loss computed in the head GEMM's epilogue gives the
    same per-row statistics, bit for bit, as the standalone loss kernel on the
    same head rows."""
    R, T = 1024, 4
    gym, model = make("rollout_cartpole", R, 128, 4, 2, T, seed=6)
    model.collect()
    t = 3
    model.train_slot(t)
    head = torch.from_numpy(model.download("train_head").view(np.int16).copy()).cuda()
    st = model.download("adv_stats").view(np.float32)[2 * t:2 * t + 2].copy()
    cols = [torch.from_numpy(np.ascontiguousarray(model.slots(k)[t])).cuda()
            for k in ("actions", "adv", "ret", "logp")]
    d_st = torch.from_numpy(st).cuda()
    dz = torch.zeros(R * HEAD, dtype=torch.int16, device="cuda")
    stats = torch.zeros(R * 5, dtype=torch.float32, device="cuda")
    hyp = model.hyper()
    rc = mg.mg_policy_loss(head.data_ptr(), cols[0].data_ptr(), cols[1].data_ptr(), d_st.data_ptr(),
                           cols[2].data_ptr(), cols[3].data_ptr(), dz.data_ptr(), stats.data_ptr(), R, 2,
                           hyp["clip"], hyp["valueCoef"], hyp["entropyCoef"], None)
    assert rc == 0, mg.mg_last_error()
    torch.cuda.synchronize()
    assert np.array_equal(stats.cpu().numpy(), model.download("stats").view(np.float32))


@pytest.mark.parametrize("name", ["rollout_cartpole", "rollout_cartpole_continuous"])
def test_train_rows_matches_oracle(mg, oracle, name):
    """A row-mode minibatch (B rows gathered across slots through the keyed
    permutation, advantages normalised over those rows) against the oracle's
    minibatch on the same rows, gathered on the host."""
    from metalgym_b200.session import minibatch_rows

    R, T, E, s, L, B = 1024, 4, 128, 4, 2, 512
    gym, model = make(name, R, E, s, L, T, seed=4)
    model.collect()
    model.minibatch_rows = B
    om = oracle_model(oracle, model, 4)
    copy_optimiser_state(oracle, om, model)
    key, base = [0x9E3779B9, 0x7F4A7C15, 0x2545F491, 0x61C88647], 3 * B
    idx = minibatch_rows(key, base, B, T * R).astype(np.int64)
    t, i = idx // R, idx % R
    assert len(np.unique(t)) == T  # the minibatch mixes every slot
    obs = np.ascontiguousarray(model.slots("obs")[t, i])
    act = np.ascontiguousarray(model.slots("actions")[t, i])
    adv = np.ascontiguousarray(model.slots("adv")[t, i])
    ret = np.ascontiguousarray(model.slots("ret")[t, i])
    logp = np.ascontiguousarray(model.slots("logp")[t, i])
    stats = np.zeros((B, 5), np.float32)
    nsq = np.zeros(1, np.float32)
    m0 = model.download("master").view(np.float32).copy()
    oracle.orc_model_set_step_counter(om, model.step_counter())
    oracle.orc_model_train_minibatch(om, ptr(obs), ptr(act), ptr(adv), ptr(ret), ptr(logp), B, ptr(stats), ptr(nsq))
    model.train_rows(key, base)
    compare_minibatch(oracle, om, model, stats, nsq, m0)
    oracle.orc_model_destroy(om)


def test_row_mode_loop_runs_and_learns(mg):
    """train(4) with 2048-row minibatches (every rollout row once per epoch):
    step counter, finite statistics, improving episodes; then back to slot
    minibatches on the same model."""
    gym, model = make("rollout_cartpole", 4096, 128, 4, 2, 32)
    model.minibatch_rows = 2048
    lengths = []
    for it in range(10):
        model.collect()
        done = model.slots("done")
        lengths.append(done.size / max(1, int(done.sum())))
        model.train(4)
        st = model.last_stats()
        assert all(np.isfinite(v) for v in st.values()), st
    assert model.step_counter() == 10 * 4 * 64
    assert np.mean(lengths[-3:]) > 1.5 * np.mean(lengths[:2]), lengths
    model.minibatch_rows = 0
    model.collect()
    model.train(1)
    assert model.step_counter() == 10 * 4 * 64 + 32


def test_train_rows_matches_oracle_voxelnav_widths(mg, oracle):
    """A row-mode minibatch at the VoxelNav policy widths of the scale-out
    configuration (embed 256, hidden 1024, 4 blocks, 40 observations, 6
    actions) against the oracle, on a small rollout."""
    from metalgym_b200.session import minibatch_rows

    R, T, E, s, L, B = 512, 4, 256, 4, 4, 256
    gym, model = make("rollout_voxelnav", R, E, s, L, T, seed=5)
    model.collect()
    model.minibatch_rows = B
    om = oracle_model(oracle, model, 5)
    copy_optimiser_state(oracle, om, model)
    key, base = [11, 22, 33, 44], 2 * B
    idx = minibatch_rows(key, base, B, T * R).astype(np.int64)
    t, i = idx // R, idx % R
    cols = [np.ascontiguousarray(model.slots(k)[t, i]) for k in ("obs", "actions", "adv", "ret", "logp")]
    stats = np.zeros((B, 5), np.float32)
    nsq = np.zeros(1, np.float32)
    m0 = model.download("master").view(np.float32).copy()
    oracle.orc_model_set_step_counter(om, model.step_counter())
    oracle.orc_model_train_minibatch(om, *[ptr(c) for c in cols], B, ptr(stats), ptr(nsq))
    model.train_rows(key, base)
    compare_minibatch(oracle, om, model, stats, nsq, m0)
    oracle.orc_model_destroy(om)


def test_config4_continuous_full_size(mg):
    """CartPoleContinuous at its benchmark shape: 16384 envs, T = 32, embed
    128, 2 blocks, 8192-row minibatches (64 per epoch), 4 epochs."""
    gym, model = make("rollout_cartpole_continuous", 16384, 128, 4, 2, 32)
    model.minibatch_rows = 8192
    for it in range(3):
        model.collect()
        model.train(4)
        st = model.last_stats()
        assert all(np.isfinite(v) for v in st.values()), st
    assert model.step_counter() == 3 * 4 * 64
    assert np.isfinite(model.log_std_value(0))


def test_config5_voxelnav_full_size(mg):
    """VoxelNav at the scale-out shape of one GPU: 262144 envs, T = 32,
    embed 256, hidden 1024, 4 blocks, 32768-row minibatches (256 per epoch):
    one collect and one epoch."""
    gym, model = make("rollout_voxelnav", 262144, 256, 4, 4, 32)
    model.minibatch_rows = 32768
    model.collect()
    adv = model.slots("adv")
    assert np.isfinite(adv).all() and adv.std() > 0
    model.train(1)
    st = model.last_stats()
    assert all(np.isfinite(v) for v in st.values()), st
    assert model.step_counter() == 256


@pytest.mark.parametrize("name,rows", [("rollout_cartpole", 0), ("rollout_cartpole_continuous", 512)])
def test_checkpoint_resume_is_exact(mg, tmp_path, name, rows):
    """Training resumed from a checkpoint continues exactly: a fresh model
    (different seed) loaded from the checkpoint reaches the same weights,
    Adam state and rollout as the model that kept going."""
    gym, model = make(name, 1024, 128, 4, 2, 4, seed=1)
    model.minibatch_rows = rows
    for _ in range(2):
        model.collect()
        model.train(2)
    ck = tmp_path / "state.ckpt"
    model.save(ck)
    for _ in range(2):
        model.collect()
        model.train(2)
    gym2, model2 = make(name, 1024, 128, 4, 2, 4, seed=9)
    model2.load(ck)
    assert model2.minibatch_rows == rows
    for _ in range(2):
        model2.collect()
        model2.train(2)
    for buf in ("weights", "master", "momentum", "variance", "obs", "actions", "reward", "done"):
        assert np.array_equal(model.download(buf), model2.download(buf)), buf
    assert model.step_counter() == model2.step_counter()


def test_checkpoint_rejects_other_shapes(mg, tmp_path):
    from metalgym_b200 import MgError

    gym, model = make("rollout_cartpole", 512, 128, 4, 2, 4)
    model.save(tmp_path / "a.ckpt")
    gym2, model2 = make("rollout_cartpole", 512, 64, 4, 2, 4)
    with pytest.raises(MgError, match="different model"):
        model2.load(tmp_path / "a.ckpt")


def test_row_mode_rejects_non_dividing_rows(mg):
    gym, model = make("rollout_cartpole", 1000, 64, 2, 1, 4)
    from metalgym_b200 import MgError

    with pytest.raises(MgError, match="divide"):
        model.minibatch_rows = 3000
    model.minibatch_rows = 500
    assert model.minibatch_rows == 500


def test_full_loop_runs_and_learns(mg):
    """collect + train(4) at the CartPole config: finite statistics, every
    minibatch applied, and the policy improves (mean episode length)."""
    gym, model = make("rollout_cartpole", 4096, 128, 4, 2, 32)
    lengths = []
    for it in range(12):
        model.collect()
        done = model.slots("done")
        lengths.append(done.size / max(1, int(done.sum())))
        model.train(4)
        st = model.last_stats()
        assert all(np.isfinite(v) for v in st.values()), st
    assert model.step_counter() == 12 * 4 * 32
    assert np.mean(lengths[-3:]) > 1.5 * np.mean(lengths[:2]), lengths


def test_two_host_threads_train_independently(mg):
    """Two models driven from two host threads at once on one GPU (the
    one-rank-per-thread use) end exactly where the same models end when run
    one after the other: no shared state between sessions, and the one-time
    kernel set-up is safe under concurrent first calls."""
    import threading

    cases = [("rollout_cartpole", 4096, 0), ("rollout_cartpole_continuous", 1024, 512)]

    def run(name, rows, mb_rows, out, key):
        gym, model = make(name, rows, 128, 4, 2, 8, seed=3)
        model.minibatch_rows = mb_rows
        for _ in range(2):
            model.collect()
            model.train(2)
        out[key] = {b: model.download(b) for b in ("weights", "master", "obs", "done")}
        out[key]["stats"] = model.last_stats()
        model.close()
        gym.close()

    together, errors = {}, []

    def guarded(*a):
        try:
            run(*a)
        except Exception as e:  # reported below; a thread's exception would be lost
            errors.append(repr(e))

    threads = [threading.Thread(target=guarded, args=(n, r, m, together, i)) for i, (n, r, m) in enumerate(cases)]
    for t in threads:
        t.start()
    for t in threads:
        t.join(timeout=300)
    assert not errors, errors
    assert not any(t.is_alive() for t in threads)
    alone = {}
    for i, (n, r, m) in enumerate(cases):
        run(n, r, m, alone, i)
    for i in range(len(cases)):
        for b in ("weights", "master", "obs", "done"):
            assert np.array_equal(together[i][b], alone[i][b]), (cases[i][0], b)
        assert together[i]["stats"] == alone[i]["stats"]


def test_phase_times_are_device_times(mg):
    """mg_ppo_phase_ms: the device time of the last collect() and train()."""
    _, model = make("rollout_cartpole", 512, 128, 4, 2, 4)
    assert model.phase_ms() == (0.0, 0.0)
    model.collect()
    c0, t0 = model.phase_ms()
    assert 0.0 < c0 < 5000.0 and t0 == 0.0
    model.train(1)
    c1, t1 = model.phase_ms()
    assert c1 == c0 and 0.0 < t1 < 5000.0
