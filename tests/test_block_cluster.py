"""One residual block per kernel on 4-CTA clusters (embed 128, hidden 512)
against the kernels it replaces: the up GEMM (ReLU) followed by the
down-projection row kernel (forward), and the dV GEMM (ReLU mask) followed
by the LayerNorm-backward row kernel and the split-K weight-gradient GEMMs
with one split per 128-row tile (backward). Every output is compared bit for
bit: the saved hidden activation V / dV, the residual stream, the LayerNorm
outputs, the dgamma / dbeta partials and the weight-gradient partials.
"""
import ctypes

import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

E, H = 128, 512
ROWS = [4096, 1000, 300, 8192, 200]


def status_ok(mg):
    torch.cuda.synchronize()
    st = ctypes.c_int(0)
    assert mg.mg_device_status(1, ctypes.byref(st)) == 0 and st.value == 0, st.value


def weights(gen):
    up = (torch.randn(E, H, device="cuda", generator=gen) / E ** 0.5).bfloat16()
    dn = (torch.randn(H, E, device="cuda", generator=gen) / H ** 0.5).bfloat16()
    g = (1 + 0.1 * torch.randn(E, device="cuda", generator=gen)).bfloat16()
    b = (0.1 * torch.randn(E, device="cuda", generator=gen)).bfloat16()
    return up, dn, g, b


def bits(t):
    return t.view(torch.int16) if t.dtype == torch.bfloat16 else t


@pytest.mark.parametrize("rows", ROWS)
def test_block_cluster_forward_bit_exact(mg, rows):
    gen = torch.Generator(device="cuda").manual_seed(rows + 11)
    up, dn, g, b = weights(gen)
    ln_out = torch.randn(rows, E, device="cuda", generator=gen).bfloat16()
    h0 = torch.randn(rows, E, device="cuda", generator=gen).bfloat16()
    # the separate kernels
    v_ref = torch.empty(rows, H, device="cuda", dtype=torch.bfloat16)
    assert mg.mg_gemm_bf16(ln_out.data_ptr(), 0, E, up.data_ptr(), 1, H, rows, H, E, 1, v_ref.data_ptr(), H, None, H,
                           1, None) == 0, mg.mg_last_error()
    h_ref = h0.clone()
    xn_ref, y_ref = torch.empty_like(h0), torch.empty_like(h0)
    sd_ref = torch.empty(rows, device="cuda")
    assert mg.mg_gemm_rows_resid_layernorm(v_ref.data_ptr(), H, dn.data_ptr(), 1, E, rows, H, h_ref.data_ptr(),
                                           g.data_ptr(), b.data_ptr(), xn_ref.data_ptr(), y_ref.data_ptr(),
                                           sd_ref.data_ptr(), None) == 0, mg.mg_last_error()
    # one kernel
    h = h0.clone()
    v = torch.full_like(v_ref, float("nan"))
    xn, y = torch.full_like(h0, float("nan")), torch.full_like(h0, float("nan"))
    sd = torch.full_like(sd_ref, float("nan"))
    rc = mg.mg_block_cluster_forward(ln_out.data_ptr(), up.data_ptr(), dn.data_ptr(), h.data_ptr(), v.data_ptr(),
                                     g.data_ptr(), b.data_ptr(), xn.data_ptr(), y.data_ptr(), sd.data_ptr(), rows, None)
    assert rc == 0, mg.mg_last_error()
    status_ok(mg)
    for got, ref in ((v, v_ref), (h, h_ref), (xn, xn_ref), (y, y_ref), (sd, sd_ref)):
        assert torch.equal(bits(got), bits(ref))


@pytest.mark.parametrize("rows", ROWS)
def test_block_cluster_backward_bit_exact(mg, rows):
    gen = torch.Generator(device="cuda").manual_seed(3 * rows + 5)
    up, dn, g, _ = weights(gen)
    dS1 = torch.randn(rows, E, device="cuda", generator=gen).bfloat16()
    v = torch.relu(torch.randn(rows, H, device="cuda", generator=gen)).bfloat16()
    xn = torch.randn(rows, E, device="cuda", generator=gen).bfloat16()
    ln_out = torch.randn(rows, E, device="cuda", generator=gen).bfloat16()
    sd = 0.5 + torch.rand(rows, device="cuda", generator=gen)
    nparts = mg.mg_layernorm_backward_num_partials(rows)
    # the separate kernels
    dv_ref = torch.empty(rows, H, device="cuda", dtype=torch.bfloat16)
    assert mg.mg_gemm_bf16(dS1.data_ptr(), 0, E, dn.data_ptr(), 0, E, rows, H, E, 3, dv_ref.data_ptr(), H,
                           v.data_ptr(), H, 1, None) == 0, mg.mg_last_error()
    out_ref = torch.empty_like(dS1)
    part_ref = torch.empty(nparts, 2 * E, device="cuda")
    assert mg.mg_gemm_rows_layernorm_backward(dv_ref.data_ptr(), H, up.data_ptr(), 0, H, rows, H, xn.data_ptr(),
                                              g.data_ptr(), sd.data_ptr(), dS1.data_ptr(), out_ref.data_ptr(),
                                              part_ref.data_ptr(), None) == 0, mg.mg_last_error()
    # the weight-gradient partials: split-K GEMMs with one split per 128 rows
    tiles = (rows + 127) // 128
    up_ref = torch.empty(tiles, E, H, device="cuda")
    assert mg.mg_gemm_bf16(ln_out.data_ptr(), 1, E, dv_ref.data_ptr(), 1, H, E, H, rows, 4, up_ref.data_ptr(), H,
                           None, 0, tiles, None) == 0, mg.mg_last_error()
    dn_ref = torch.empty(tiles, H, E, device="cuda")
    assert mg.mg_gemm_bf16(v.data_ptr(), 1, H, dS1.data_ptr(), 1, E, H, E, rows, 4, dn_ref.data_ptr(), E,
                           None, 0, tiles, None) == 0, mg.mg_last_error()
    # the input layer's gradient partials of the output rows (first block), where
    # the separate kernel also takes 16 rows per partial
    O = 4
    obs = torch.randn(rows, O, device="cuda", generator=gen)
    fuse_input = mg.mg_input_backward_num_partials(rows, O, E) == (rows + 15) // 16
    in_ref = in_part = None
    if fuse_input:
        in_ref = torch.empty((rows + 15) // 16, O + 1, E, device="cuda")
        assert mg.mg_input_backward_partials(obs.data_ptr(), out_ref.data_ptr(), in_ref.data_ptr(), rows, O, E,
                                             None) == 0, mg.mg_last_error()
        in_part = torch.full_like(in_ref, float("nan"))
    # one kernel
    dv = torch.full_like(dv_ref, float("nan"))
    out = torch.full_like(dS1, float("nan"))
    part = torch.full_like(part_ref, float("nan"))
    up_part = torch.full_like(up_ref, float("nan"))
    dn_part = torch.full_like(dn_ref, float("nan"))
    rc = mg.mg_block_cluster_backward(dS1.data_ptr(), dn.data_ptr(), v.data_ptr(), up.data_ptr(), dv.data_ptr(),
                                      ln_out.data_ptr(), up_part.data_ptr(), dn_part.data_ptr(), xn.data_ptr(),
                                      g.data_ptr(), sd.data_ptr(), dS1.data_ptr(), out.data_ptr(), part.data_ptr(),
                                      obs.data_ptr() if fuse_input else None, O,
                                      in_part.data_ptr() if fuse_input else None, rows, None)
    assert rc == 0, mg.mg_last_error()
    status_ok(mg)
    for got, ref in ((dv, dv_ref), (out, out_ref), (part, part_ref), (up_part, up_ref), (dn_part, dn_ref)):
        assert torch.equal(bits(got), bits(ref))
    if fuse_input:
        assert torch.equal(in_part, in_ref)


@pytest.mark.parametrize("rows", ROWS)
def test_block_cluster_forward_with_input_layer_bit_exact(mg, rows):
    """The first block's kernel computing the input layer and the first
    LayerNorm itself, against the input kernel, the LayerNorm kernel and the
    block kernel."""
    O = 4
    gen = torch.Generator(device="cuda").manual_seed(rows + 29)
    up, dn, g, b = weights(gen)
    g0 = (1 + 0.1 * torch.randn(E, device="cuda", generator=gen)).bfloat16()
    b0 = (0.1 * torch.randn(E, device="cuda", generator=gen)).bfloat16()
    w_in = (torch.randn(O, E, device="cuda", generator=gen) / 2).bfloat16()
    b_in = (0.1 * torch.randn(E, device="cuda", generator=gen)).bfloat16()
    obs = torch.randn(rows, O, device="cuda", generator=gen)
    # the separate kernels
    h_ref = torch.empty(rows, E, device="cuda", dtype=torch.bfloat16)
    assert mg.mg_input_forward(obs.data_ptr(), w_in.data_ptr(), b_in.data_ptr(), h_ref.data_ptr(), rows, O, E,
                               None) == 0, mg.mg_last_error()
    xn0_ref, lo0_ref = torch.empty_like(h_ref), torch.empty_like(h_ref)
    sd0_ref = torch.empty(rows, device="cuda")
    assert mg.mg_layernorm_forward(h_ref.data_ptr(), xn0_ref.data_ptr(), lo0_ref.data_ptr(), g0.data_ptr(),
                                   b0.data_ptr(), sd0_ref.data_ptr(), rows, E, None) == 0
    v_ref = torch.empty(rows, H, device="cuda", dtype=torch.bfloat16)
    xn_ref, y_ref = torch.empty_like(h_ref), torch.empty_like(h_ref)
    sd_ref = torch.empty(rows, device="cuda")
    assert mg.mg_block_cluster_forward(lo0_ref.data_ptr(), up.data_ptr(), dn.data_ptr(), h_ref.data_ptr(),
                                       v_ref.data_ptr(), g.data_ptr(), b.data_ptr(), xn_ref.data_ptr(),
                                       y_ref.data_ptr(), sd_ref.data_ptr(), rows, None) == 0, mg.mg_last_error()
    # one kernel
    nan = lambda t: torch.full_like(t, float("nan"))  # noqa: E731
    h, xn0, lo0, sd0, v, xn, y, sd = (nan(t) for t in (h_ref, xn0_ref, lo0_ref, sd0_ref, v_ref, xn_ref, y_ref,
                                                       sd_ref))
    rc = mg.mg_block_cluster_forward_input(obs.data_ptr(), O, w_in.data_ptr(), b_in.data_ptr(), g0.data_ptr(),
                                           b0.data_ptr(), xn0.data_ptr(), lo0.data_ptr(), sd0.data_ptr(),
                                           up.data_ptr(), dn.data_ptr(), h.data_ptr(), v.data_ptr(), g.data_ptr(),
                                           b.data_ptr(), xn.data_ptr(), y.data_ptr(), sd.data_ptr(), rows, None)
    assert rc == 0, mg.mg_last_error()
    status_ok(mg)
    for got, ref in ((xn0, xn0_ref), (lo0, lo0_ref), (sd0, sd0_ref), (v, v_ref), (h, h_ref), (xn, xn_ref),
                     (y, y_ref), (sd, sd_ref)):
        assert torch.equal(bits(got), bits(ref))
