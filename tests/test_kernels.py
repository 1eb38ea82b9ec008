"""GPU kernels vs the CPU checkers, through the C ABI.

Bit-exact (integer state, RNG words, and float work whose operation order
the kernel keeps): environment steps, the random-policy raw step, the fused
sample + step of collect(), the samplers, PPO losses, GAE, input projection
and Adam without clipping. Within tolerance (reductions in a different
order): LayerNorm (bf16 outputs within one bf16 ulp, statistics rtol 1e-5),
weight-gradient partial sums (rtol 1e-5), clipped Adam (rtol 1e-6).
"""
import ctypes
from pathlib import Path

import numpy as np
import pytest

from orc import ENV_IDS, ENV_SIZES, bf16_round, bf16_to_f32, ptr, seed_words

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

HEAD = 64
GOLD = Path(__file__).resolve().parent / "golden"


_KEEP = []


@pytest.fixture(autouse=True)
def _keep_device_temporaries():
    """Device copies made by dev() live until the test ends, so no buffer a
    kernel still reads can be recycled into another argument of the call."""
    yield
    torch.cuda.synchronize()
    _KEEP.clear()


def dev(a):
    """numpy -> CUDA tensor with the same bytes (kept alive until the test ends)."""
    a = np.ascontiguousarray(a)
    t = torch.from_numpy(a.view(np.uint8).copy()).cuda()
    _KEEP.append(t)
    return t


def host(t, dtype, shape=None):
    a = t.cpu().numpy().view(dtype)
    return a.reshape(shape) if shape is not None else a


def ok(mg, rc):
    assert rc == 0, mg.mg_last_error().decode()


def sync_status(mg):
    torch.cuda.synchronize()
    st = ctypes.c_int(0)
    ok(mg, mg.mg_device_status(1, ctypes.byref(st)))
    assert st.value == 0, f"device status {st.value}"


def random_actions(rs, n, ad, cont):
    if cont:
        return (rs.standard_normal((n, ad)) * 1.5).astype(np.float32)
    return rs.integers(0, ad, n).astype(np.int32)


@pytest.mark.parametrize("name", sorted(ENV_IDS))
def test_env_step_matches_golden(mg, name):
    """Device rollout<Env> on the reference's golden action sequence."""
    gd = dict(np.load(GOLD / f"env_{name}.npz"))
    sb, ab, ob, od, ad, cont = ENV_SIZES[name]
    steps, n = gd["reward"].shape
    st = torch.zeros(n * sb, dtype=torch.uint8, device="cuda")
    obs = torch.zeros(n * ob, dtype=torch.uint8, device="cuda")
    rew = torch.zeros(n, dtype=torch.float32, device="cuda")
    done = torch.zeros(n, dtype=torch.uint8, device="cuda")
    rng = torch.zeros(n, dtype=torch.int32, device="cuda")
    ok(mg, mg.mg_env_init(name.encode(), st.data_ptr(), done.data_ptr(), rng.data_ptr(), n, 0, 0, None))
    acts = dev(gd["actions"])
    for t in range(steps):
        ok(mg, mg.mg_env_step(name.encode(), st.data_ptr(), acts.data_ptr() + t * n * ab, obs.data_ptr(),
                              rew.data_ptr(), done.data_ptr(), None, rng.data_ptr(), n, None))
        if t % 50 == 0 or t == steps - 1:
            assert np.array_equal(host(obs, np.uint8), gd["obs"][t]), f"obs step {t}"
            assert np.array_equal(host(rew, np.uint32), gd["reward"][t].view(np.uint32)), f"reward step {t}"
            assert np.array_equal(host(done, np.uint8), gd["done"][t]), f"done step {t}"
    sync_status(mg)
    assert np.array_equal(host(st, np.uint8), gd["final_states"])
    assert np.array_equal(host(rng, np.uint32), gd["final_rng"])


@pytest.mark.parametrize("name,n,steps", [("rollout_cartpole", 4096, 300), ("rollout_cartpole_continuous", 4096, 300),
                                          ("rollout_voxelnav", 1024, 120)])
def test_env_step_full_size_vs_host(mg, hostenv, name, n, steps):
    """Device vs host build of the same env, at benchmark size, every step."""
    which = ENV_IDS[name]
    sb, ab, ob, od, ad, cont = ENV_SIZES[name]
    rs = np.random.default_rng(17)
    hs = np.zeros(n * sb, np.uint8)
    ho = np.zeros(n * ob, np.uint8)
    hr = np.zeros(n, np.float32)
    hd = np.ones(n, np.uint8)
    hg = seed_words(n, seed=11, first=1000)
    st = torch.zeros(n * sb, dtype=torch.uint8, device="cuda")
    obs = torch.zeros(n * ob, dtype=torch.uint8, device="cuda")
    rew = torch.zeros(n, dtype=torch.float32, device="cuda")
    done = torch.zeros(n, dtype=torch.uint8, device="cuda")
    dcopy = torch.zeros(n, dtype=torch.uint8, device="cuda")
    rng = torch.zeros(n, dtype=torch.int32, device="cuda")
    ok(mg, mg.mg_env_init(name.encode(), st.data_ptr(), done.data_ptr(), rng.data_ptr(), n, 11, 1000, None))
    assert np.array_equal(host(rng, np.uint32), hg)
    for t in range(steps):
        a = random_actions(rs, n, ad, cont)
        da = dev(a)
        ok(mg, mg.mg_env_step(name.encode(), st.data_ptr(), da.data_ptr(), obs.data_ptr(), rew.data_ptr(),
                              done.data_ptr(), dcopy.data_ptr(), rng.data_ptr(), n, None))
        hostenv.hostenv_rollout(which, ptr(hs), ptr(a), ptr(ho), ptr(hr), ptr(hd), ptr(hg), n, 8)
        assert np.array_equal(host(obs, np.uint8), ho), f"obs step {t}"
        assert np.array_equal(host(rew, np.uint32), hr.view(np.uint32)), f"reward step {t}"
        assert np.array_equal(host(done, np.uint8), hd) and np.array_equal(host(dcopy, np.uint8), hd)
    sync_status(mg)
    assert np.array_equal(host(st, np.uint8), hs) and np.array_equal(host(rng, np.uint32), hg)


@pytest.mark.parametrize("name,mode", [("rollout_cartpole", 0), ("rollout_cartpole", 1),
                                       ("rollout_cartpole_continuous", 0), ("rollout_voxelnav", 0)])
def test_run_random_matches_reference_sampler_and_env(mg, oracle, hostenv, name, mode):
    """The fused multi-step raw kernel = per step: the sampler on an all-zero
    head (or action 0), then rollout<Env>; every step's outputs kept in the ring."""
    which = ENV_IDS[name]
    sb, ab, ob, od, ad, cont = ENV_SIZES[name]
    n, steps = (2048, 64) if which < 2 else (256, 48)
    st = torch.zeros(n * sb, dtype=torch.uint8, device="cuda")
    done = torch.zeros(n, dtype=torch.uint8, device="cuda")
    rng = torch.zeros(n, dtype=torch.int32, device="cuda")
    ok(mg, mg.mg_env_init(name.encode(), st.data_ptr(), done.data_ptr(), rng.data_ptr(), n, 5, 0, None))
    obs_r = torch.zeros(steps * n * ob, dtype=torch.uint8, device="cuda")
    rew_r = torch.zeros(steps * n, dtype=torch.float32, device="cuda")
    done_r = torch.zeros(steps * n, dtype=torch.uint8, device="cuda")
    ok(mg, mg.mg_env_run_random(name.encode(), st.data_ptr(), obs_r.data_ptr(), rew_r.data_ptr(), done_r.data_ptr(),
                                done.data_ptr(), rng.data_ptr(), n, steps, steps, mode, None))
    sync_status(mg)
    hs = np.zeros(n * sb, np.uint8)
    ho = np.zeros(n * ob, np.uint8)
    hr = np.zeros(n, np.float32)
    hd = np.ones(n, np.uint8)
    hg = seed_words(n, seed=5)
    zero_head = np.zeros((n, HEAD), np.uint16)
    zero_ls = np.zeros(ad, np.uint16)
    lp = np.zeros(n, np.float32)
    v = np.zeros(n, np.float32)
    gobs = host(obs_r, np.uint8, (steps, n * ob))
    grew = host(rew_r, np.uint32, (steps, n))
    gdone = host(done_r, np.uint8, (steps, n))
    for t in range(steps):
        if mode == 1:
            a = np.zeros((n, ad), np.float32) if cont else np.zeros(n, np.int32)
        elif cont:
            a = np.zeros((n, ad), np.float32)
            oracle.orc_sample_gaussian(ptr(zero_head), ptr(hg), ptr(a), ptr(lp), ptr(v), n, ad, HEAD, ptr(zero_ls))
        else:
            a = np.zeros(n, np.int32)
            oracle.orc_sample_action(ptr(zero_head), ptr(hg), ptr(a), ptr(lp), ptr(v), n, ad, HEAD)
        hostenv.hostenv_rollout(which, ptr(hs), ptr(a), ptr(ho), ptr(hr), ptr(hd), ptr(hg), n, 8)
        assert np.array_equal(gobs[t], ho), f"obs step {t}"
        assert np.array_equal(grew[t], hr.view(np.uint32)) and np.array_equal(gdone[t], hd), f"step {t}"
    assert np.array_equal(host(st, np.uint8), hs) and np.array_equal(host(rng, np.uint32), hg)


@pytest.mark.parametrize("name", sorted(ENV_IDS))
def test_collect_step_fused_matches_sampler_then_env(mg, oracle, hostenv, name):
    which = ENV_IDS[name]
    sb, ab, ob, od, ad, cont = ENV_SIZES[name]
    n = 2048 if which < 2 else 512
    rs = np.random.default_rng(3)
    st = torch.zeros(n * sb, dtype=torch.uint8, device="cuda")
    done = torch.zeros(n, dtype=torch.uint8, device="cuda")
    rng = torch.zeros(n, dtype=torch.int32, device="cuda")
    ok(mg, mg.mg_env_init(name.encode(), st.data_ptr(), done.data_ptr(), rng.data_ptr(), n, 0, 0, None))
    hs = np.zeros(n * sb, np.uint8)
    hd = np.ones(n, np.uint8)
    hg = seed_words(n)
    ho = np.zeros(n * ob, np.uint8)
    hr = np.zeros(n, np.float32)
    logstd = bf16_round((rs.standard_normal(max(ad, 1)) * 0.3).astype(np.float32))
    d_ls = dev(logstd)
    act = torch.zeros(n * ab, dtype=torch.uint8, device="cuda")
    lp = torch.zeros(n, dtype=torch.float32, device="cuda")
    val = torch.zeros(n, dtype=torch.float32, device="cuda")
    obs = torch.zeros(n * ob, dtype=torch.uint8, device="cuda")
    rew = torch.zeros(n, dtype=torch.float32, device="cuda")
    dslot = torch.zeros(n, dtype=torch.uint8, device="cuda")
    for t in range(40):
        h = np.zeros((n, HEAD), np.float32)
        h[:, :ad + 1] = rs.standard_normal((n, ad + 1)) * 1.5
        head = bf16_round(h)
        ok(mg, mg.mg_env_collect_step(name.encode(), dev(head).data_ptr(), d_ls.data_ptr(), st.data_ptr(),
                                      act.data_ptr(), lp.data_ptr(), val.data_ptr(), obs.data_ptr(), rew.data_ptr(),
                                      done.data_ptr(), dslot.data_ptr(), rng.data_ptr(), n, None))
        hlp = np.zeros(n, np.float32)
        hv = np.zeros(n, np.float32)
        if cont:
            ha = np.zeros((n, ad), np.float32)
            oracle.orc_sample_gaussian(ptr(head), ptr(hg), ptr(ha), ptr(hlp), ptr(hv), n, ad, HEAD, ptr(logstd))
        else:
            ha = np.zeros(n, np.int32)
            oracle.orc_sample_action(ptr(head), ptr(hg), ptr(ha), ptr(hlp), ptr(hv), n, ad, HEAD)
        hostenv.hostenv_rollout(which, ptr(hs), ptr(ha), ptr(ho), ptr(hr), ptr(hd), ptr(hg), n, 8)
        assert np.array_equal(host(act, np.uint8), ha.view(np.uint8).ravel()), f"action step {t}"
        assert np.array_equal(host(lp, np.uint32), hlp.view(np.uint32)), f"logp step {t}"
        assert np.array_equal(host(val, np.float32), hv)
        assert np.array_equal(host(obs, np.uint8), ho) and np.array_equal(host(rew, np.uint32), hr.view(np.uint32))
        assert np.array_equal(host(done, np.uint8), hd) and np.array_equal(host(dslot, np.uint8), hd)
    sync_status(mg)
    assert np.array_equal(host(st, np.uint8), hs) and np.array_equal(host(rng, np.uint32), hg)


def test_samplers_bit_exact(mg, oracle):
    g = dict(np.load(GOLD / "kernels.npz"))
    rows = g["sa_head"].shape[0]
    rng = dev(g["sa_rng"])
    a = torch.zeros(rows, dtype=torch.int32, device="cuda")
    lp = torch.zeros(rows, dtype=torch.float32, device="cuda")
    v = torch.zeros(rows, dtype=torch.float32, device="cuda")
    ok(mg, mg.mg_sample_categorical(dev(g["sa_head"]).data_ptr(), rng.data_ptr(), a.data_ptr(), lp.data_ptr(),
                                    v.data_ptr(), rows, 6, None))
    sync_status(mg)
    assert np.array_equal(host(a, np.int32), g["sa_action"].astype(np.int32))
    assert np.array_equal(host(lp, np.uint32), g["sa_logp"].view(np.uint32))
    assert np.array_equal(host(rng, np.uint32), g["sa_rng_out"])
    rng = dev(g["sg_rng"])
    ga = torch.zeros(rows * 3, dtype=torch.float32, device="cuda")
    ok(mg, mg.mg_sample_gaussian(dev(g["sg_head"]).data_ptr(), dev(g["sg_logstd"]).data_ptr(), rng.data_ptr(),
                                 ga.data_ptr(), lp.data_ptr(), v.data_ptr(), rows, 3, None))
    sync_status(mg)
    assert np.array_equal(host(ga, np.uint32), g["sg_action"].view(np.uint32))
    assert np.array_equal(host(lp, np.uint32), g["sg_logp"].view(np.uint32))
    assert np.array_equal(host(rng, np.uint32), g["sg_rng_out"])


def test_losses_bit_exact(mg, oracle):
    g = dict(np.load(GOLD / "kernels.npz"))
    rows = g["pl_head"].shape[0]
    dz = torch.zeros(rows * HEAD, dtype=torch.int16, device="cuda")
    stats = torch.zeros(rows * 5, dtype=torch.float32, device="cuda")
    ok(mg, mg.mg_policy_loss(dev(g["pl_head"]).data_ptr(), dev(g["pl_action"].astype(np.int32)).data_ptr(),
                             dev(g["pl_adv"]).data_ptr(), None, dev(g["pl_ret"]).data_ptr(), dev(g["pl_old"]).data_ptr(),
                             dz.data_ptr(), stats.data_ptr(), rows, 6, 0.2, 0.5, 0.01, None))
    sync_status(mg)
    assert np.array_equal(host(dz, np.uint16, (rows, HEAD)), g["pl_dz"])
    assert np.array_equal(host(stats, np.uint32, (rows, 5)), g["pl_stats"].view(np.uint32))
    # with on-device advantage statistics: identical to pre-normalised advantages
    mean, inv = np.float32(0.25), np.float32(1.75)
    advn = ((g["pl_adv"] - mean) * inv).astype(np.float32)
    dz2 = torch.zeros_like(dz)
    ok(mg, mg.mg_policy_loss(dev(g["pl_head"]).data_ptr(), dev(g["pl_action"].astype(np.int32)).data_ptr(),
                             dev(g["pl_adv"]).data_ptr(), dev(np.array([mean, inv], np.float32)).data_ptr(),
                             dev(g["pl_ret"]).data_ptr(), dev(g["pl_old"]).data_ptr(), dz2.data_ptr(), stats.data_ptr(),
                             rows, 6, 0.2, 0.5, 0.01, None))
    hdz = np.zeros((rows, HEAD), np.uint16)
    hst = np.zeros((rows, 5), np.float32)
    act32 = g["pl_action"].astype(np.int32)  # a named array: ptr() of a temporary would dangle
    oracle.orc_policy_loss(ptr(g["pl_head"]), ptr(act32), ptr(advn), ptr(g["pl_ret"]),
                           ptr(g["pl_old"]), ptr(hdz), ptr(hst), rows, 6, HEAD, 0.2, 0.5, 0.01)
    sync_status(mg)
    assert np.array_equal(host(dz2, np.uint16, (rows, HEAD)), hdz)
    # Gaussian loss; the log-std gradient comes as per-block partials
    nparts = mg.mg_gaussian_loss_num_partials(rows)
    part = torch.zeros(nparts * 3, dtype=torch.float32, device="cuda")
    ok(mg, mg.mg_gaussian_loss(dev(g["gl_head"]).data_ptr(), dev(g["gl_action"]).data_ptr(),
                               dev(g["pl_adv"]).data_ptr(), None, dev(g["pl_ret"]).data_ptr(),
                               dev(g["pl_old"]).data_ptr(), dz.data_ptr(), stats.data_ptr(),
                               dev(g["gl_logstd"]).data_ptr(), part.data_ptr(), rows, 3, 0.2, 0.5, 0.01, None))
    sync_status(mg)
    assert np.array_equal(host(dz, np.uint16, (rows, HEAD)), g["gl_dz"])
    assert np.array_equal(host(stats, np.uint32, (rows, 5)), g["gl_stats"].view(np.uint32))
    np.testing.assert_allclose(host(part, np.float32, (nparts, 3)).sum(0), g["gl_dlogstd"], rtol=1e-5, atol=1e-7)


def test_gae_and_advantage_stats(mg, oracle):
    g = dict(np.load(GOLD / "kernels.npz"))
    R, T = 256, 32
    adv = torch.zeros(T * R, dtype=torch.float32, device="cuda")
    ret = torch.zeros(T * R, dtype=torch.float32, device="cuda")
    ok(mg, mg.mg_gae(dev(g["gae_reward"]).data_ptr(), dev(g["gae_done"]).data_ptr(), dev(g["gae_value"]).data_ptr(),
                     dev(g["gae_boot"]).data_ptr(), adv.data_ptr(), ret.data_ptr(), R, T, 2, 0.99, 0.95, None))
    sync_status(mg)
    assert np.array_equal(host(adv, np.uint32), g["gae_adv"].view(np.uint32))
    assert np.array_equal(host(ret, np.uint32), g["gae_ret"].view(np.uint32))
    stats = torch.zeros(2 * T, dtype=torch.float32, device="cuda")
    ok(mg, mg.mg_advantage_stats(adv.data_ptr(), stats.data_ptr(), R, T, None))
    sync_status(mg)
    s = host(stats, np.float32, (T, 2))
    a = g["gae_adv"].reshape(T, R).astype(np.float64)
    np.testing.assert_allclose(s[:, 0], a.mean(1), rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(s[:, 1], 1.0 / (a.std(1) + 1e-8), rtol=1e-5)
    # slot 0's normalised advantages match the reference kernel's output
    normed = (g["gae_adv"][:R] - s[0, 0]) * s[0, 1]
    np.testing.assert_allclose(normed, g["gae_norm"], rtol=1e-5, atol=1e-5)


def test_input_projection(mg, oracle):
    g = dict(np.load(GOLD / "kernels.npz"))
    R, O, E = 256, 40, 128
    out = torch.zeros(R * E, dtype=torch.int16, device="cuda")
    ok(mg, mg.mg_input_forward(dev(g["in_obs"]).data_ptr(), dev(g["in_w"]).data_ptr(), dev(g["in_b"]).data_ptr(),
                               out.data_ptr(), R, O, E, None))
    sync_status(mg)
    assert np.array_equal(host(out, np.uint16, (R, E)), g["in_out"])
    P = mg.mg_input_backward_num_partials(R, O, E)
    part = torch.zeros(P * (O + 1) * E, dtype=torch.float32, device="cuda")
    ok(mg, mg.mg_input_backward_partials(dev(g["in_obs"]).data_ptr(), dev(g["in_dz"]).data_ptr(), part.data_ptr(), R,
                                         O, E, None))
    sync_status(mg)
    tot = host(part, np.float32, (P, O + 1, E)).sum(0)
    np.testing.assert_allclose(tot[:O], g["in_dw"], rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(tot[O], g["in_db"], rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("R,O,E", [(256, 40, 128), (1000, 4, 128), (4096, 4, 128), (300, 40, 256), (64, 8, 64)])
def test_input_projection_with_layernorm(mg, R, O, E):
    """The input projection with block 0's LayerNorm fused in: the projection
    bit-identical to mg_input_forward, the LayerNorm outputs bit-identical to
    mg_layernorm_forward on that projection."""
    rs = np.random.default_rng(R + O + E)
    obs = rs.standard_normal((R, O)).astype(np.float32)
    w = bf16_round((rs.standard_normal((O, E)) / np.sqrt(O)).astype(np.float32))
    b = bf16_round((rs.standard_normal(E) * 0.1).astype(np.float32))
    gam = bf16_round((1 + rs.standard_normal(E) * 0.1).astype(np.float32))
    bet = bf16_round((rs.standard_normal(E) * 0.1).astype(np.float32))
    h_ref = torch.zeros(R * E, dtype=torch.int16, device="cuda")
    xn_ref, y_ref = torch.zeros_like(h_ref), torch.zeros_like(h_ref)
    sd_ref = torch.zeros(R, dtype=torch.float32, device="cuda")
    d_obs, d_w, d_b, d_g, d_bt = dev(obs), dev(w), dev(b), dev(gam), dev(bet)
    ok(mg, mg.mg_input_forward(d_obs.data_ptr(), d_w.data_ptr(), d_b.data_ptr(), h_ref.data_ptr(), R, O, E, None))
    ok(mg, mg.mg_layernorm_forward(h_ref.data_ptr(), xn_ref.data_ptr(), y_ref.data_ptr(), d_g.data_ptr(),
                                   d_bt.data_ptr(), sd_ref.data_ptr(), R, E, None))
    h, xn, y = torch.zeros_like(h_ref), torch.zeros_like(h_ref), torch.zeros_like(h_ref)
    sd = torch.zeros_like(sd_ref)
    ok(mg, mg.mg_input_forward_layernorm(d_obs.data_ptr(), d_w.data_ptr(), d_b.data_ptr(), h.data_ptr(),
                                         d_g.data_ptr(), d_bt.data_ptr(), xn.data_ptr(), y.data_ptr(), sd.data_ptr(),
                                         R, O, E, None))
    sync_status(mg)
    assert torch.equal(h, h_ref) and torch.equal(xn, xn_ref) and torch.equal(y, y_ref) and torch.equal(sd, sd_ref)


def bf16_close(a_u16, b_u16, max_ulps=1, min_exact=0.99):
    d = np.abs(a_u16.astype(np.int32) - b_u16.astype(np.int32))
    assert d.max() <= max_ulps, d.max()
    assert (d == 0).mean() >= min_exact, (d == 0).mean()


@pytest.mark.parametrize("R,E", [(256, 128), (4096, 128), (1000, 256)])
def test_layernorm(mg, oracle, R, E):
    rs = np.random.default_rng(R + E)
    x = bf16_round((rs.standard_normal((R, E)) * 2 + 0.3).astype(np.float32))
    gam = bf16_round((1 + rs.standard_normal(E) * 0.1).astype(np.float32))
    bet = bf16_round((rs.standard_normal(E) * 0.1).astype(np.float32))
    xn = torch.zeros(R * E, dtype=torch.int16, device="cuda")
    y = torch.zeros_like(xn)
    sd = torch.zeros(R, dtype=torch.float32, device="cuda")
    ok(mg, mg.mg_layernorm_forward(dev(x).data_ptr(), xn.data_ptr(), y.data_ptr(), dev(gam).data_ptr(),
                                   dev(bet).data_ptr(), sd.data_ptr(), R, E, None))
    hxn = np.zeros((R, E), np.uint16)
    hy = np.zeros((R, E), np.uint16)
    hsd = np.zeros(R, np.float32)
    oracle.orc_layernorm_forward(ptr(x), ptr(hxn), ptr(hy), ptr(gam), ptr(bet), ptr(hsd), R, E)
    sync_status(mg)
    bf16_close(host(xn, np.uint16, (R, E)), hxn)
    bf16_close(host(y, np.uint16, (R, E)), hy)
    np.testing.assert_allclose(host(sd, np.float32), hsd, rtol=1e-5)
    # backward, standalone and with the residual add of the stream
    dz = bf16_round((rs.standard_normal((R, E)) * 0.01).astype(np.float32))
    resid = bf16_round((rs.standard_normal((R, E)) * 0.01).astype(np.float32))
    P = mg.mg_layernorm_backward_num_partials(R)
    part = torch.zeros(P * 2 * E, dtype=torch.float32, device="cuda")
    d_dz = dev(dz)
    d_res = dev(resid)
    ok(mg, mg.mg_layernorm_backward(d_dz.data_ptr(), dev(hxn).data_ptr(), dev(gam).data_ptr(), dev(hsd).data_ptr(),
                                    d_res.data_ptr(), part.data_ptr(), R, E, None))
    hdz = dz.copy()
    hdg = np.zeros(E, np.float32)
    hdb = np.zeros(E, np.float32)
    oracle.orc_layernorm_backward(ptr(hdz), ptr(hxn), ptr(gam), ptr(hsd), ptr(hdg), ptr(hdb), R, E)
    sync_status(mg)
    expect = bf16_round(bf16_to_f32(hdz) + bf16_to_f32(resid))
    bf16_close(host(d_res, np.uint16, (R, E)), expect)
    assert np.array_equal(host(d_dz, np.uint16, (R, E)), dz)  # dZ untouched with resid
    tot = host(part, np.float32, (P, 2, E)).sum(0)
    np.testing.assert_allclose(tot[0], hdg, rtol=1e-4, atol=1e-6)
    np.testing.assert_allclose(tot[1], hdb, rtol=1e-4, atol=1e-6)


@pytest.mark.parametrize("max_norm", [0.0, 0.5])
def test_reduce_partials_and_adam(mg, oracle, max_norm):
    rs = np.random.default_rng(9)
    count, nparts = 70000, 5
    parts = (rs.standard_normal((nparts, count)) * 0.05).astype(np.float32)
    grad = torch.zeros(count, dtype=torch.float32, device="cuda")
    nn = mg.mg_reduce_partials_num_norm_partials(count)
    normp = torch.zeros(nn, dtype=torch.float32, device="cuda")
    ok(mg, mg.mg_reduce_partials(dev(parts).data_ptr(), count, nparts, count, grad.data_ptr(), 1, normp.data_ptr(),
                                 None))
    sync_status(mg)
    hg = np.zeros(count, np.float32)
    for p in range(nparts):
        hg = (hg + parts[p]).astype(np.float32)
    hg = bf16_to_f32(bf16_round(hg))
    assert np.array_equal(host(grad, np.uint32), hg.view(np.uint32))
    nsq = float(host(normp, np.float32).astype(np.float64).sum())
    np.testing.assert_allclose(nsq, oracle.orc_grad_norm_sq(ptr(hg), count), rtol=1e-5)
    param = rs.standard_normal(count).astype(np.float32)
    m = (rs.standard_normal(count) * 1e-3).astype(np.float32)
    v = (rs.random(count) * 1e-3).astype(np.float32)
    dp, dm, dv = dev(param), dev(m), dev(v)
    w = torch.zeros(count, dtype=torch.int16, device="cuda")
    nsq_out = torch.zeros(1, dtype=torch.float32, device="cuda")
    b1p, b2p = float(np.float32(0.9) ** 5), float(np.float32(0.999) ** 5)
    ok(mg, mg.mg_adam_step(dp.data_ptr(), grad.data_ptr(), dm.data_ptr(), dv.data_ptr(), w.data_ptr(),
                           normp.data_ptr(), nn, count, 3e-4, b1p, b2p, max_norm, nsq_out.data_ptr(), None))
    sync_status(mg)
    gpu_nsq = float(host(nsq_out, np.float32)[0])
    hw = np.zeros(count, np.uint16)
    oracle.orc_adam_step(ptr(param), ptr(hg), ptr(m), ptr(v), ptr(hw), gpu_nsq, count, 3e-4, b1p, b2p, max_norm)
    # given the same squared norm the update is bit-exact
    assert np.array_equal(host(dp, np.uint32), param.view(np.uint32))
    assert np.array_equal(host(dm, np.uint32), m.view(np.uint32))
    assert np.array_equal(host(dv, np.uint32), v.view(np.uint32))
    assert np.array_equal(host(w, np.uint16), hw)
