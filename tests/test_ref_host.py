"""The reference's own host code (gym.h, model/ppo.h, compiled unmodified for
the CPU through oracle/shim_host/ into oracle/_ref/libmg_ref_host.so) as the
checker of the host-side parts of the drop-in PPOModel:

CPU
* act(rng) (model/ppo.h:636-686): the drop-in sampler
  (metalgym::sample_actions_host, include/metalgym/ppo.h) draws the same
  actions, log-probabilities and values as the reference's act() on the same
  head rows with the same std::mt19937 seed, bit for bit, over several calls
  (categorical and Gaussian heads, ties and saturated logits included);
* actGreedy() (model/ppo.h:688-702) of the reference against numpy's first
  argmax / the means (the contract the device kernel implements);
* the seeded parameter init and layout (model/ppo.h:375-445): the oracle
  restatement's weights and fp32 master equal the reference constructor's,
  bit for bit, so the GPU tests that compare the product's init with the
  oracle are pinned to the reference;
* setLogStd / logStdValue (model/ppo.h:454-469) and lastStats()
  (model/ppo.h:925-943) on given statistics rows.
GPU
* mg_ppo_act_greedy on the head rows of forward() equals the reference's
  actGreedy() on the same rows; the product's initial weights and master
  equal the reference constructor's.
"""
import numpy as np
import pytest

from orc import bf16_round, load_host_sampler, load_oracle, load_ref_host

REF = load_ref_host()
pytestmark = pytest.mark.skipif(REF is None, reason="oracle/_ref/libmg_ref_host.so not built (needs the reference tree)")


def ref_model(kind, R=256, L=2, T=4, seed=0):
    return REF.ref_host_create(kind, R, 128, 4, L, 3e-4, T, seed)


def random_head(R, act_dim, rng, ties=True):
    h = np.zeros((R, 64), np.float32)
    h[:, :act_dim] = rng.normal(0, 2.0, (R, act_dim))
    h[:, act_dim] = rng.normal(0, 1.0, R)
    if ties:
        h[::7, 1 % act_dim] = h[::7, 0]        # equal logits
        h[::11, 0] = 60.0                      # saturated softmax
    return bf16_round(h).reshape(R, 64)


@pytest.mark.parametrize("kind,act_dim", [(0, 2), (1, 1)])
@pytest.mark.parametrize("seed,calls", [(0, 1), (12345, 3)])
def test_act_draws_like_the_reference(kind, act_dim, seed, calls):
    R = 256
    host = load_host_sampler()
    h = ref_model(kind, R)
    head = random_head(R, act_dim, np.random.default_rng(seed))
    REF.ref_host_set_head(h, head)
    ls = np.zeros(1, np.float32)
    if kind == 1:
        REF.ref_host_set_log_std(h, -0.5)
        ls[0] = REF.ref_host_log_std(h, 0)
    adt, na = (np.int32, R) if kind == 0 else (np.float32, R * act_dim)
    ra, rv, rl = np.zeros(na, adt), np.zeros(R, np.float32), np.zeros(R, np.float32)
    REF.ref_host_act(h, seed, calls, ra, rv, rl)
    ma, mv, ml = np.zeros(na, adt), np.zeros(R, np.float32), np.zeros(R, np.float32)
    host.host_act(kind, head, R, ls, seed, calls, ma, mv, ml)
    REF.ref_host_destroy(h)
    assert np.array_equal(ra.view(np.uint32), ma.view(np.uint32))
    assert np.array_equal(rv.view(np.uint32), mv.view(np.uint32))
    assert np.array_equal(rl.view(np.uint32), ml.view(np.uint32))
    if kind == 0:
        assert set(np.unique(ma)) <= {0, 1} and 0 < ma.mean() < 1


@pytest.mark.parametrize("kind,act_dim", [(0, 2), (1, 1)])
def test_reference_act_greedy_is_first_argmax_or_mean(kind, act_dim):
    R = 256
    h = ref_model(kind, R)
    head = random_head(R, act_dim, np.random.default_rng(3))
    REF.ref_host_set_head(h, head)
    out = np.zeros(R, np.int32) if kind == 0 else np.zeros(R * act_dim, np.float32)
    REF.ref_host_act_greedy(h, out)
    REF.ref_host_destroy(h)
    vals = (head.astype(np.uint32) << 16).view(np.float32)[:, :act_dim]
    want = vals.argmax(1).astype(np.int32) if kind == 0 else vals.reshape(-1)
    assert np.array_equal(out, want)


@pytest.mark.parametrize("kind,L,seed", [(0, 2, 0), (0, 1, 7), (1, 2, 3)])
def test_oracle_init_equals_the_reference_constructor(kind, L, seed):
    orc = load_oracle()
    R, T = 128, 4
    h = ref_model(kind, R, L, T, seed)
    sz = np.zeros(3, np.uint64)
    REF.ref_host_sizes(h, sz)
    n = int(sz[0])
    w, m = np.zeros(n, np.uint16), np.zeros(n, np.float32)
    REF.ref_host_params(h, w, m)
    REF.ref_host_destroy(h)
    act_dim = 2 if kind == 0 else 1
    om = orc.orc_model_create(R, 4, act_dim, kind, 128, 4, L, 3e-4, T, seed)
    assert orc.orc_model_opt_count(om) == n and orc.orc_model_opt_float_count(om) == int(sz[1])
    import ctypes

    ow = np.ctypeslib.as_array(ctypes.cast(orc.orc_model_weights(om), ctypes.POINTER(ctypes.c_uint16)), shape=(n,))
    omr = np.ctypeslib.as_array(ctypes.cast(orc.orc_model_master(om), ctypes.POINTER(ctypes.c_float)), shape=(n,))
    same_w, same_m = np.array_equal(ow, w), np.array_equal(omr.view(np.uint32), m.view(np.uint32))
    orc.orc_model_destroy(om)
    assert same_w and same_m


def test_log_std_and_last_stats_host_code():
    h = ref_model(1, 128)
    REF.ref_host_set_log_std(h, 0.3)
    bf = (bf16_round(np.array([0.3], np.float32)).astype(np.uint32) << 16).view(np.float32)[0]
    assert REF.ref_host_log_std(h, 0) == bf
    rows = np.random.default_rng(5).normal(0, 1, (128, 5)).astype(np.float32)
    out = np.zeros(6, np.float32)
    REF.ref_host_last_stats(h, rows, np.float32(2.25), out)
    REF.ref_host_destroy(h)
    acc = rows.sum(0, dtype=np.float64) / 128
    np.testing.assert_allclose(out[:5], acc, rtol=1e-5, atol=1e-6)
    assert out[5] == np.float32(1.5)


# ---------------------------------------------------------------- GPU

@pytest.mark.gpu
@pytest.mark.parametrize("name,kind,act_dim", [("rollout_cartpole", 0, 2), ("rollout_cartpole_continuous", 1, 1)])
def test_device_act_greedy_equals_the_reference(mg, name, kind, act_dim):
    import ctypes

    import metalgym_b200
    from metalgym_b200.session import Gym, PPOModel

    R = 512
    gym = Gym(name, R, seed=1)
    model = PPOModel(gym, 128, 4, 2, 3e-4, 4, 1)
    model.collect()
    model.forward()
    head = model.download("head").view(np.uint16).reshape(R, 64).copy()
    out = np.zeros(R, np.int32) if kind == 0 else np.zeros(R * act_dim, np.float32)
    metalgym_b200.check(metalgym_b200.lib().mg_ppo_act_greedy(model.handle, 8, out.ctypes.data_as(ctypes.c_void_p)),
                        "mg_ppo_act_greedy")  # 8: MG_PPO_HEAD
    h = ref_model(kind, R)
    REF.ref_host_set_head(h, head)
    want = np.zeros_like(out)
    REF.ref_host_act_greedy(h, want)
    REF.ref_host_destroy(h)
    assert np.array_equal(out.view(np.uint32), want.view(np.uint32))
    # the actions landed in the gym's device buffer too
    dev = gym.download("actions").view(out.dtype)
    assert np.array_equal(dev.view(np.uint32), out.view(np.uint32))


@pytest.mark.gpu
@pytest.mark.parametrize("name,kind,L,seed", [("rollout_cartpole", 0, 2, 0), ("rollout_cartpole_continuous", 1, 1, 4)])
def test_product_init_equals_the_reference_constructor(mg, name, kind, L, seed):
    from metalgym_b200.session import Gym, PPOModel

    R = 128
    model = PPOModel(Gym(name, R), 128, 4, L, 3e-4, 4, seed)
    h = ref_model(kind, R, L, 4, seed)
    sz = np.zeros(3, np.uint64)
    REF.ref_host_sizes(h, sz)
    n = int(sz[0])
    w, m = np.zeros(n, np.uint16), np.zeros(n, np.float32)
    REF.ref_host_params(h, w, m)
    REF.ref_host_destroy(h)
    assert np.array_equal(model.download("weights").view(np.uint16)[:n], w)
    assert np.array_equal(model.download("master").view(np.uint32)[:n], m.view(np.uint32))
