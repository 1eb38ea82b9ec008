"""Pins the CPU checkers against the reference (CPU only).

* oracle/ (the C++ restatement) vs the golden vectors made by the reference's
  own sources (tests/golden/make_golden.py): bit-exact where the restatement
  keeps the reference's operation order, within a stated tolerance where the
  reference reduces in an order it does not specify (atomics, threadgroups).
* the product's environment structs compiled for the host vs the reference
  environments: bit-exact trajectories, including resets and the RNG words.
* the project-owned transcendentals vs float64 math: error bounds.
"""
from pathlib import Path

import numpy as np
import pytest

from orc import ENV_IDS, ENV_SIZES, bf16_round, bf16_to_f32, ptr, seed_words

GOLD = Path(__file__).resolve().parent / "golden"
HEAD = 64


@pytest.fixture(scope="module")
def g():
    return dict(np.load(GOLD / "kernels.npz"))


def test_sample_action_bit_exact(oracle, g):
    rows, A = g["sa_head"].shape[0], 6
    rng = g["sa_rng"].copy()
    act = np.zeros(rows, np.int32)
    lp = np.zeros(rows, np.float32)
    v = np.zeros(rows, np.float32)
    oracle.orc_sample_action(ptr(g["sa_head"]), ptr(rng), ptr(act), ptr(lp), ptr(v), rows, A, HEAD)
    assert np.array_equal(act, g["sa_action"].astype(np.int32))
    assert np.array_equal(lp.view(np.uint32), g["sa_logp"].view(np.uint32))
    assert np.array_equal(v, g["sa_value"])
    assert np.array_equal(rng, g["sa_rng_out"])


def test_sample_gaussian_bit_exact(oracle, g):
    rows, A = g["sg_head"].shape[0], 3
    rng = g["sg_rng"].copy()
    act = np.zeros(rows * A, np.float32)
    lp = np.zeros(rows, np.float32)
    v = np.zeros(rows, np.float32)
    oracle.orc_sample_gaussian(ptr(g["sg_head"]), ptr(rng), ptr(act), ptr(lp), ptr(v), rows, A, HEAD,
                               ptr(g["sg_logstd"]))
    assert np.array_equal(act.view(np.uint32), g["sg_action"].view(np.uint32))
    assert np.array_equal(lp.view(np.uint32), g["sg_logp"].view(np.uint32))
    assert np.array_equal(rng, g["sg_rng_out"])


def test_policy_loss_bit_exact(oracle, g):
    rows, A = g["pl_head"].shape[0], 6
    dz = np.zeros((rows, HEAD), np.uint16)
    st = np.zeros((rows, 5), np.float32)
    act = g["pl_action"].astype(np.int32)
    oracle.orc_policy_loss(ptr(g["pl_head"]), ptr(act), ptr(g["pl_adv"]), ptr(g["pl_ret"]), ptr(g["pl_old"]),
                           ptr(dz), ptr(st), rows, A, HEAD, 0.2, 0.5, 0.01)
    assert np.array_equal(dz, g["pl_dz"])
    assert np.array_equal(st.view(np.uint32), g["pl_stats"].view(np.uint32))


def test_gaussian_loss_bit_exact(oracle, g):
    rows, A = g["gl_head"].shape[0], 3
    dz = np.zeros((rows, HEAD), np.uint16)
    st = np.zeros((rows, 5), np.float32)
    dls = np.zeros(A, np.float32)
    oracle.orc_gaussian_loss(ptr(g["gl_head"]), ptr(g["gl_action"]), ptr(g["pl_adv"]), ptr(g["pl_ret"]),
                             ptr(g["pl_old"]), ptr(dz), ptr(st), rows, A, HEAD, 0.2, 0.5, 0.01, ptr(g["gl_logstd"]),
                             ptr(dls))
    assert np.array_equal(dz, g["gl_dz"])
    assert np.array_equal(st.view(np.uint32), g["gl_stats"].view(np.uint32))
    assert np.array_equal(dls.view(np.uint32), g["gl_dlogstd"].view(np.uint32))


def test_gae_bit_exact_and_normalize(oracle, g):
    R, T = 256, 32
    boot = bf16_to_f32(g["gae_boot"].reshape(R, HEAD)[:, 2]).copy()
    adv = np.zeros(T * R, np.float32)
    ret = np.zeros(T * R, np.float32)
    oracle.orc_gae(ptr(g["gae_reward"]), ptr(g["gae_done"]), ptr(g["gae_value"]), ptr(boot), ptr(adv), ptr(ret), R,
                   T, 0.99, 0.95)
    assert np.array_equal(adv.view(np.uint32), g["gae_adv"].view(np.uint32))
    assert np.array_equal(ret.view(np.uint32), g["gae_ret"].view(np.uint32))
    nrm = np.zeros(R, np.float32)
    oracle.orc_normalize_advantage(ptr(adv), ptr(nrm), R)
    # the reference sums in float (order unspecified), the checker in double
    np.testing.assert_allclose(nrm, g["gae_norm"], rtol=1e-5, atol=1e-6)


def test_adam_bit_exact(oracle, g):
    count, fcount = 4096, 1024
    grad = np.concatenate([g["ad_gradF"], bf16_to_f32(g["ad_gradB"])]).astype(np.float32)
    nsq = oracle.orc_grad_norm_sq(ptr(grad), count)
    # the reference accumulates in float in thread order; the checker in double
    np.testing.assert_allclose(nsq, g["ad_normsq"][0], rtol=2e-5)
    p, m, v = g["ad_param"].copy(), g["ad_mom"].copy(), g["ad_var"].copy()
    w = np.zeros(count, np.uint16)
    oracle.orc_adam_step(ptr(p), ptr(grad), ptr(m), ptr(v), ptr(w), float(g["ad_normsq"][0]), count, 3e-4,
                         float(g["ad_b1p"]), float(g["ad_b2p"]), 0.5)
    assert np.array_equal(p.view(np.uint32), g["ad_param_out"].view(np.uint32))
    assert np.array_equal(m.view(np.uint32), g["ad_mom_out"].view(np.uint32))
    assert np.array_equal(v.view(np.uint32), g["ad_var_out"].view(np.uint32))
    assert np.array_equal(w, g["ad_weights"])


def test_input_projection(oracle, g):
    R, O, E = 256, 40, 128
    out = np.zeros((R, E), np.uint16)
    oracle.orc_input_forward(ptr(g["in_obs"]), ptr(g["in_w"]), ptr(g["in_b"]), ptr(out), R, O, E)
    assert np.array_equal(out, g["in_out"])
    dW = np.zeros((O, E), np.float32)
    dB = np.zeros(E, np.float32)
    oracle.orc_input_backward(ptr(g["in_obs"]), ptr(g["in_dz"]), ptr(dW), ptr(dB), R, O, E)
    # the reference adds 64-row chunk sums atomically: order differs
    np.testing.assert_allclose(dW, g["in_dw"], rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(dB, g["in_db"], rtol=1e-5, atol=1e-6)


def test_layernorm_bit_exact(oracle, g):
    R, E = 256, 128
    xn = np.zeros((R, E), np.uint16)
    y = np.zeros((R, E), np.uint16)
    sd = np.zeros(R, np.float32)
    oracle.orc_layernorm_forward(ptr(g["ln_x"]), ptr(xn), ptr(y), ptr(g["ln_gamma"]), ptr(g["ln_beta"]), ptr(sd), R, E)
    assert np.array_equal(xn, g["ln_xn"])
    assert np.array_equal(y, g["ln_y"])
    assert np.array_equal(sd, g["ln_sd"])
    dz = g["ln_dz"].copy()
    dg = np.zeros(E, np.float32)
    db = np.zeros(E, np.float32)
    oracle.orc_layernorm_backward(ptr(dz), ptr(g["ln_xn"]), ptr(g["ln_gamma"]), ptr(g["ln_sd"]), ptr(dg), ptr(db), R, E)
    assert np.array_equal(dz, g["ln_dx"])
    assert np.array_equal(dg.view(np.uint32), g["ln_dg"].view(np.uint32))
    assert np.array_equal(db.view(np.uint32), g["ln_db"].view(np.uint32))


@pytest.mark.parametrize("name", sorted(ENV_IDS))
def test_host_env_port_matches_reference_golden(hostenv, name):
    """The product's env structs (host build) reproduce the reference env
    trajectories bit for bit: obs, reward, done every step, final state and RNG."""
    gd = dict(np.load(GOLD / f"env_{name}.npz"))
    which = ENV_IDS[name]
    sb, ab, ob, od, ad, cont = ENV_SIZES[name]
    steps, n = gd["reward"].shape
    states = np.zeros(n * sb, np.uint8)
    obs = np.zeros(n * ob, np.uint8)
    rew = np.zeros(n, np.float32)
    done = np.ones(n, np.uint8)
    rng = seed_words(n)
    for t in range(steps):
        a = np.ascontiguousarray(gd["actions"][t])
        hostenv.hostenv_rollout(which, ptr(states), ptr(a), ptr(obs), ptr(rew), ptr(done), ptr(rng), n, 1)
        assert np.array_equal(obs, gd["obs"][t]), f"obs differs at step {t}"
        assert np.array_equal(rew.view(np.uint32), gd["reward"][t].view(np.uint32)), f"reward differs at step {t}"
        assert np.array_equal(done, gd["done"][t]), f"done differs at step {t}"
    assert np.array_equal(states, gd["final_states"])
    assert np.array_equal(rng, gd["final_rng"])
    assert gd["done"].sum() > 0  # the trajectories exercise resets


@pytest.mark.parametrize("name", sorted(ENV_IDS))
def test_host_env_port_matches_reference_live(hostenv, refimpl, name):
    """Same, against the reference build directly, at more envs and threads."""
    which = ENV_IDS[name]
    sb, ab, ob, od, ad, cont = ENV_SIZES[name]
    n, steps = (1024, 400) if which < 2 else (128, 200)
    rs = np.random.default_rng(5)
    st = [np.zeros(n * sb, np.uint8) for _ in range(2)]
    obs = [np.zeros(n * ob, np.uint8) for _ in range(2)]
    rew = [np.zeros(n, np.float32) for _ in range(2)]
    done = [np.ones(n, np.uint8) for _ in range(2)]
    rng = [seed_words(n, seed=3) for _ in range(2)]
    for t in range(steps):
        a = (rs.standard_normal((n, ad)) * 1.5).astype(np.float32) if cont else rs.integers(0, ad, n).astype(np.int32)
        refimpl.ref_rollout(which, ptr(st[0]), ptr(a), ptr(obs[0]), ptr(rew[0]), ptr(done[0]), ptr(rng[0]), n, 4)
        hostenv.hostenv_rollout(which, ptr(st[1]), ptr(a), ptr(obs[1]), ptr(rew[1]), ptr(done[1]), ptr(rng[1]), n, 4)
        assert np.array_equal(obs[0], obs[1]) and np.array_equal(done[0], done[1]), f"step {t}"
        assert np.array_equal(rew[0].view(np.uint32), rew[1].view(np.uint32)), f"step {t}"
    assert np.array_equal(st[0], st[1]) and np.array_equal(rng[0], rng[1])


def test_own_transcendentals_accuracy(hostenv):
    """mg_sinf / mg_cosf / mg_expf / mg_logf are within 1 float ulp of the
    correctly rounded result on a sweep of arguments (and NaN / inf behave)."""
    rs = np.random.default_rng(0)
    xs = np.concatenate([rs.uniform(-8, 8, 4000), rs.uniform(-200, 200, 1000), [0.0, 1e-30, -1e-30, np.pi / 4]])
    xs = xs.astype(np.float32)

    def ulps(a, b):
        a = np.float32(a)
        b = np.float32(b)
        return abs(int(a.view(np.int32)) - int(b.view(np.int32)))

    for x in xs:
        assert ulps(hostenv.hostenv_sinf(float(x)), np.sin(np.float64(x))) <= 1, x
        assert ulps(hostenv.hostenv_cosf(float(x)), np.cos(np.float64(x))) <= 1, x
    for x in np.concatenate([rs.uniform(-80, 80, 3000), [0.0, -100.0, 88.0]]).astype(np.float32):
        assert ulps(hostenv.hostenv_expf(float(x)), np.exp(np.float64(x))) <= 1, x
    for x in np.concatenate([np.exp(rs.uniform(-80, 80, 3000)), [1.0, 2.0, 1e-38]]).astype(np.float32):
        assert ulps(hostenv.hostenv_logf(float(x)), np.log(np.float64(x))) <= 1, x
    assert hostenv.hostenv_expf(0.0) == 1.0
    assert np.isnan(hostenv.hostenv_sinf(float("nan"))) and np.isnan(hostenv.hostenv_cosf(float("inf")))
    assert hostenv.hostenv_logf(0.0) == -np.inf and np.isnan(hostenv.hostenv_logf(-1.0))
