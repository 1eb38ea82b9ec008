"""The head of a training minibatch in one kernel (head GEMM, categorical PPO
loss, head dX, final-LayerNorm backward, dW_head partial per 128-row tile)
against the separate kernels it replaces: the head GEMM, the standalone loss
kernel, the dX GEMM, the LayerNorm backward kernel and the split-K weight
GEMM with one split per 128 rows. Every output is compared bit for bit.
"""
import ctypes

import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

E, HEAD, A = 128, 64, 2
CLIP, VCOEF, ECOEF = 0.2, 0.5, 0.01


def bits(t):
    return t.view(torch.int16) if t.dtype == torch.bfloat16 else t


@pytest.mark.parametrize("rows,normalise", [(4096, True), (1000, False), (300, True), (8192, True), (200, False)])
def test_head_tail_bit_exact(mg, rows, normalise):
    gen = torch.Generator(device="cuda").manual_seed(rows + 17)
    f_out = torch.randn(rows, E, device="cuda", generator=gen).bfloat16()
    w = torch.zeros(E, HEAD, device="cuda")
    w[:, :A + 1] = torch.randn(E, A + 1, device="cuda", generator=gen) / E ** 0.5
    w = w.bfloat16()
    action = torch.randint(0, A, (rows,), device="cuda", generator=gen, dtype=torch.int32)
    adv = torch.randn(rows, device="cuda", generator=gen)
    ret = torch.randn(rows, device="cuda", generator=gen)
    logp = -0.69 + 0.05 * torch.randn(rows, device="cuda", generator=gen)
    adv_stats = torch.tensor([0.1, 1.3], device="cuda") if normalise else None
    st_ptr = adv_stats.data_ptr() if normalise else None
    g = (1 + 0.1 * torch.randn(E, device="cuda", generator=gen)).bfloat16()
    xn = torch.randn(rows, E, device="cuda", generator=gen).bfloat16()
    sd = 0.5 + torch.rand(rows, device="cuda", generator=gen)
    tiles = (rows + 127) // 128
    nparts = mg.mg_layernorm_backward_num_partials(rows)
    # the separate kernels
    head_ref = torch.empty(rows, HEAD, device="cuda", dtype=torch.bfloat16)
    assert mg.mg_gemm_bf16(f_out.data_ptr(), 0, E, w.data_ptr(), 1, HEAD, rows, HEAD, E, 0, head_ref.data_ptr(),
                           HEAD, None, HEAD, 1, None) == 0, mg.mg_last_error()
    dz_ref = torch.zeros(rows, HEAD, device="cuda", dtype=torch.bfloat16)
    stats_ref = torch.zeros(rows, 5, device="cuda")
    assert mg.mg_policy_loss(head_ref.data_ptr(), action.data_ptr(), adv.data_ptr(), st_ptr, ret.data_ptr(),
                             logp.data_ptr(), dz_ref.data_ptr(), stats_ref.data_ptr(), rows, A, CLIP, VCOEF, ECOEF,
                             None) == 0, mg.mg_last_error()
    ds_ref = torch.empty(rows, E, device="cuda", dtype=torch.bfloat16)
    assert mg.mg_gemm_bf16(dz_ref.data_ptr(), 0, HEAD, w.data_ptr(), 0, HEAD, rows, E, HEAD, 0, ds_ref.data_ptr(), E,
                           None, E, 1, None) == 0, mg.mg_last_error()
    lnp_ref = torch.empty(nparts, 2 * E, device="cuda")
    assert mg.mg_layernorm_backward(ds_ref.data_ptr(), xn.data_ptr(), g.data_ptr(), sd.data_ptr(), None,
                                    lnp_ref.data_ptr(), rows, E, None) == 0, mg.mg_last_error()
    hp_ref = torch.empty(tiles, E, HEAD, device="cuda")
    assert mg.mg_gemm_bf16(f_out.data_ptr(), 1, E, dz_ref.data_ptr(), 1, HEAD, E, HEAD, rows, 4, hp_ref.data_ptr(),
                           HEAD, None, 0, tiles, None) == 0, mg.mg_last_error()
    # one kernel
    head = torch.full_like(head_ref, float("nan"))
    dz = torch.full_like(dz_ref, float("nan"))
    stats = torch.full_like(stats_ref, float("nan"))
    ds = torch.full_like(ds_ref, float("nan"))
    lnp = torch.full_like(lnp_ref, float("nan"))
    hp = torch.full_like(hp_ref, float("nan"))
    rc = mg.mg_head_tail(f_out.data_ptr(), w.data_ptr(), head.data_ptr(), action.data_ptr(), adv.data_ptr(), st_ptr,
                         ret.data_ptr(), logp.data_ptr(), dz.data_ptr(), stats.data_ptr(), rows, A, CLIP, VCOEF,
                         ECOEF, hp.data_ptr(), g.data_ptr(), xn.data_ptr(), sd.data_ptr(), ds.data_ptr(),
                         lnp.data_ptr(), None)
    assert rc == 0, mg.mg_last_error()
    torch.cuda.synchronize()
    st = ctypes.c_int(0)
    assert mg.mg_device_status(1, ctypes.byref(st)) == 0 and st.value == 0, st.value
    for got, ref in ((head, head_ref), (dz, dz_ref), (stats, stats_ref), (ds, ds_ref), (lnp, lnp_ref), (hp, hp_ref)):
        assert torch.equal(bits(got), bits(ref))
