"""Generates the golden vectors in tests/golden/*.npz from the reference itself.

The reference's own Metal sources (rollout.h, the three example environments
and the per-thread model kernels) are compiled unmodified as host C++ through
the shim in oracle/shim (oracle/Makefile target `ref`, output
oracle/_ref/libmg_ref.so). This script drives that build on small seeded
inputs and stores inputs and outputs, so the restatement in oracle/ and the
CUDA kernels can be checked against the reference's behaviour on machines
without the reference tree.

Run: python tests/golden/make_golden.py   (needs the reference tree)
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent))

from orc import ENV_IDS, ENV_SIZES, bf16_round, load_ref, ptr, seed_words  # noqa: E402

HEAD = 64


def env_trajectory(ref, name: str, n: int, steps: int, seed: int):
    """Reference rollout<Env> driven by a seeded action sequence; every step's outputs."""
    which = ENV_IDS[name]
    sb, ab, ob, od, ad, cont = ENV_SIZES[name]
    rs = np.random.default_rng(seed)
    states = np.zeros(n * sb, np.uint8)
    obs = np.zeros(n * ob, np.uint8)
    reward = np.zeros(n, np.float32)
    done = np.ones(n, np.uint8)
    rng = seed_words(n)
    if cont:
        actions = (rs.standard_normal((steps, n, ad)) * 1.5).astype(np.float32)
    else:
        actions = rs.integers(0, ad, (steps, n)).astype(np.int32)
    out_obs = np.zeros((steps, n * ob), np.uint8)
    out_rew = np.zeros((steps, n), np.float32)
    out_done = np.zeros((steps, n), np.uint8)
    for t in range(steps):
        a = np.ascontiguousarray(actions[t])
        ref.ref_rollout(which, ptr(states), ptr(a), ptr(obs), ptr(reward), ptr(done), ptr(rng), n, 1)
        out_obs[t] = obs
        out_rew[t] = reward
        out_done[t] = done
    return dict(actions=actions, obs=out_obs, reward=out_rew, done=out_done, final_states=states.copy(),
                final_rng=rng.copy())


def make_head(rs, rows, act_dim, scale=2.0):
    h = np.zeros((rows, HEAD), np.float32)
    h[:, :act_dim + 1] = rs.standard_normal((rows, act_dim + 1)) * scale
    return bf16_round(h)


def kernels(ref, seed: int):
    rs = np.random.default_rng(seed)
    g = {}
    # sampleAction (model/sample.metal)
    rows, A = 256, 6
    head = make_head(rs, rows, A)
    rng = seed_words(rows, seed=7)
    act = np.zeros(rows, np.uint32)
    lp = np.zeros(rows, np.float32)
    val = np.zeros(rows, np.float32)
    rng_out = rng.copy()
    ref.ref_sample_action(ptr(head), ptr(rng_out), ptr(act), ptr(lp), ptr(val), rows, A, HEAD)
    g.update(sa_head=head, sa_rng=rng, sa_action=act, sa_logp=lp.copy(), sa_value=val.copy(), sa_rng_out=rng_out)
    # sampleGaussian (model/gaussian.metal)
    A2 = 3
    head = make_head(rs, rows, A2, 1.0)
    logstd = bf16_round((rs.standard_normal(A2) * 0.5).astype(np.float32))
    rng_out = rng.copy()
    gact = np.zeros(rows * A2, np.float32)
    ref.ref_sample_gaussian(ptr(head), ptr(rng_out), ptr(gact), ptr(lp), ptr(val), rows, A2, HEAD, ptr(logstd))
    g.update(sg_head=head, sg_logstd=logstd, sg_rng=rng, sg_action=gact, sg_logp=lp.copy(), sg_value=val.copy(),
             sg_rng_out=rng_out)
    # policyLossBackward (model/policy.metal)
    head = make_head(rs, rows, A)
    action = rs.integers(0, A, rows).astype(np.uint32)
    adv = rs.standard_normal(rows).astype(np.float32)
    ret = rs.standard_normal(rows).astype(np.float32)
    old = (rs.standard_normal(rows) * 0.3 - 1.8).astype(np.float32)
    dz = np.zeros((rows, HEAD), np.uint16)
    stats = np.zeros((rows, 5), np.float32)
    ref.ref_policy_loss(ptr(head), ptr(action), ptr(adv), ptr(ret), ptr(old), ptr(dz), ptr(stats), rows, A, HEAD,
                        0.2, 0.5, 0.01)
    g.update(pl_head=head, pl_action=action, pl_adv=adv, pl_ret=ret, pl_old=old, pl_dz=dz, pl_stats=stats)
    # gaussianLossBackward (model/gaussian.metal)
    head = make_head(rs, rows, A2, 1.0)
    gaction = (rs.standard_normal(rows * A2)).astype(np.float32)
    dz = np.zeros((rows, HEAD), np.uint16)
    stats = np.zeros((rows, 5), np.float32)
    dls = np.zeros(A2, np.float32)
    ref.ref_gaussian_loss(ptr(head), ptr(gaction), ptr(adv), ptr(ret), ptr(old), ptr(dz), ptr(stats), rows, A2, HEAD,
                          0.2, 0.5, 0.01, ptr(logstd), ptr(dls))
    g.update(gl_head=head, gl_action=gaction, gl_dz=dz, gl_stats=stats, gl_dlogstd=dls, gl_logstd=logstd)
    # gaeBackward + normalizeAdvantage (model/gae.metal)
    R, T = 256, 32
    reward = rs.standard_normal(T * R).astype(np.float32)
    done = (rs.random(T * R) < 0.1).astype(np.uint8)
    value = rs.standard_normal(T * R).astype(np.float32)
    boot = make_head(rs, R, 2)
    advo = np.zeros(T * R, np.float32)
    reto = np.zeros(T * R, np.float32)
    ref.ref_gae(ptr(reward), ptr(done), ptr(value), ptr(boot), ptr(advo), ptr(reto), R, T, HEAD, 2, 0.99, 0.95)
    nrm = np.zeros(R, np.float32)
    ref.ref_normalize_advantage(ptr(advo), ptr(nrm), R)
    g.update(gae_reward=reward, gae_done=done, gae_value=value, gae_boot=boot, gae_adv=advo, gae_ret=reto,
             gae_norm=nrm)
    # adamStep + gradNormSq (model/optimizer.metal)
    count, fcount = 4096, 1024
    param = rs.standard_normal(count).astype(np.float32)
    gradF = (rs.standard_normal(fcount) * 0.1).astype(np.float32)
    gradB = bf16_round((rs.standard_normal(count - fcount) * 0.1).astype(np.float32))
    mom = (rs.standard_normal(count) * 0.01).astype(np.float32)
    var = (rs.random(count) * 0.01).astype(np.float32)
    weights = np.zeros(count, np.uint16)
    nsq = np.zeros(1, np.float32)
    ref.ref_grad_norm_sq(ptr(gradF), ptr(gradB), ptr(nsq), count, fcount)
    p2, m2, v2 = param.copy(), mom.copy(), var.copy()
    b1p, b2p = np.float32(0.9) ** 3, np.float32(0.999) ** 3
    ref.ref_adam_step(ptr(p2), ptr(gradF), ptr(gradB), ptr(m2), ptr(v2), ptr(weights), ptr(nsq), count, fcount,
                      3e-4, float(b1p), float(b2p), 0.5)
    g.update(ad_param=param, ad_gradF=gradF, ad_gradB=gradB, ad_mom=mom, ad_var=var, ad_normsq=nsq,
             ad_b1p=np.float32(b1p), ad_b2p=np.float32(b2p), ad_param_out=p2, ad_mom_out=m2, ad_var_out=v2,
             ad_weights=weights)
    # inputForward / inputBackward (model/input.metal)
    R, O, E = 256, 40, 128
    obs = rs.standard_normal((R, O)).astype(np.float32)
    w = bf16_round((rs.standard_normal((O, E)) / np.sqrt(O)).astype(np.float32))
    b = bf16_round((rs.standard_normal(E) * 0.1).astype(np.float32))
    out = np.zeros((R, E), np.uint16)
    ref.ref_input_forward(ptr(obs), ptr(w), ptr(b), ptr(out), R, O, E)
    dzi = bf16_round((rs.standard_normal((R, E)) * 0.01).astype(np.float32))
    dW = np.zeros((O, E), np.float32)
    dB = np.zeros(E, np.float32)
    ref.ref_input_backward(ptr(obs), ptr(dzi), ptr(dW), ptr(dB), R, O, E, 64)
    g.update(in_obs=obs, in_w=w, in_b=b, in_out=out, in_dz=dzi, in_dw=dW, in_db=dB)
    # layernormForward / layernormBackward (model/layernorm.metal)
    R, E = 256, 128
    x = bf16_round((rs.standard_normal((R, E)) * 2 + 0.5).astype(np.float32))
    gam = bf16_round((1 + rs.standard_normal(E) * 0.1).astype(np.float32))
    bet = bf16_round((rs.standard_normal(E) * 0.1).astype(np.float32))
    xn = np.zeros((R, E), np.uint16)
    y = np.zeros((R, E), np.uint16)
    sd = np.zeros(R, np.float32)
    ref.ref_layernorm_forward(ptr(x), ptr(xn), ptr(y), ptr(gam), ptr(bet), ptr(sd), R, E)
    dzl = bf16_round((rs.standard_normal((R, E)) * 0.01).astype(np.float32))
    dzl_out = dzl.copy()
    dxn = np.zeros((R, E), np.uint16)
    dg = np.zeros(E, np.float32)
    db = np.zeros(E, np.float32)
    ref.ref_layernorm_backward(ptr(dzl_out), ptr(xn), ptr(gam), ptr(sd), ptr(dxn), ptr(dg), ptr(db), R, E)
    g.update(ln_x=x, ln_gamma=gam, ln_beta=bet, ln_xn=xn, ln_y=y, ln_sd=sd, ln_dz=dzl, ln_dx=dzl_out, ln_dg=dg,
             ln_db=db)
    return g


def main():
    ref = load_ref()
    if ref is None:
        raise SystemExit("the reference build is unavailable (no reference source tree)")
    np.savez_compressed(HERE / "kernels.npz", **kernels(ref, 1234))
    for name, n, steps in [("rollout_cartpole", 32, 300), ("rollout_cartpole_continuous", 32, 300),
                           ("rollout_voxelnav", 8, 300)]:
        np.savez_compressed(HERE / f"env_{name}.npz", **env_trajectory(ref, name, n, steps, seed=99))
    print("wrote", sorted(p.name for p in HERE.glob("*.npz")))


if __name__ == "__main__":
    main()
