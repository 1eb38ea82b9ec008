"""Fused residual-block kernels against the unfused chain of the same
kernels (LayerNorm, up GEMM with ReLU, down GEMM with residual add).

All outputs must be bit-identical: the LayerNorm sums run in the same order,
and V and the updated residual stream come from the same tcgen05 products in
the same K order with the same roundings.
"""
import ctypes

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def unfused(mg, h, g, b, up, dn, rows, E, H):
    xn = torch.empty(rows, E, device="cuda", dtype=torch.bfloat16)
    lo = torch.empty_like(xn)
    sd = torch.empty(rows, device="cuda", dtype=torch.float32)
    v = torch.empty(rows, H, device="cuda", dtype=torch.bfloat16)
    hh = h.clone()
    assert mg.mg_layernorm_forward(hh.data_ptr(), xn.data_ptr(), lo.data_ptr(), g.data_ptr(), b.data_ptr(),
                                   sd.data_ptr(), rows, E, None) == 0, mg.mg_last_error()
    assert mg.mg_gemm_bf16(lo.data_ptr(), 0, E, up.data_ptr(), 1, H, rows, H, E, 1, v.data_ptr(), H, None, H, 1,
                           None) == 0, mg.mg_last_error()
    assert mg.mg_gemm_bf16(v.data_ptr(), 0, H, dn.data_ptr(), 1, E, rows, E, H, 2, hh.data_ptr(), E, hh.data_ptr(),
                           E, 1, None) == 0, mg.mg_last_error()
    torch.cuda.synchronize()
    return hh, xn, lo, sd, v


@pytest.mark.parametrize("rows,E,H", [(4096, 128, 512), (1000, 128, 256), (8192, 64, 256), (300, 64, 128)])
def test_block_forward_matches_unfused(mg, rows, E, H):
    gen = torch.Generator(device="cuda").manual_seed(rows + E + H)
    h = torch.randn(rows, E, device="cuda", generator=gen).bfloat16()
    g = (1 + 0.1 * torch.randn(E, device="cuda", generator=gen)).bfloat16()
    b = (0.1 * torch.randn(E, device="cuda", generator=gen)).bfloat16()
    up = (torch.randn(E, H, device="cuda", generator=gen) / E ** 0.5).bfloat16()
    dn = (torch.randn(H, E, device="cuda", generator=gen) / H ** 0.5).bfloat16()
    ref_h, ref_xn, ref_lo, ref_sd, ref_v = unfused(mg, h, g, b, up, dn, rows, E, H)
    hh = h.clone()
    xn = torch.full((rows, E), float("nan"), device="cuda", dtype=torch.bfloat16)
    lo = torch.full_like(xn, float("nan"))
    sd = torch.full((rows,), float("nan"), device="cuda", dtype=torch.float32)
    v = torch.full((rows, H), float("nan"), device="cuda", dtype=torch.bfloat16)
    rc = mg.mg_block_forward(hh.data_ptr(), g.data_ptr(), b.data_ptr(), up.data_ptr(), dn.data_ptr(), xn.data_ptr(),
                             lo.data_ptr(), sd.data_ptr(), v.data_ptr(), rows, E, H, None)
    assert rc == 0, mg.mg_last_error()
    torch.cuda.synchronize()
    st = ctypes.c_int(0)
    assert mg.mg_device_status(1, ctypes.byref(st)) == 0 and st.value == 0
    assert torch.equal(xn.view(torch.int16), ref_xn.view(torch.int16))
    assert torch.equal(lo.view(torch.int16), ref_lo.view(torch.int16))
    assert torch.equal(sd, ref_sd)
    assert torch.equal(v.view(torch.int16), ref_v.view(torch.int16))
    assert torch.equal(hh.view(torch.int16), ref_h.view(torch.int16))


@pytest.mark.parametrize("rows,E,H", [(32768, 256, 1024), (4096, 128, 512), (1000, 256, 512), (300, 128, 256)])
def test_down_projection_with_layernorm_matches_unfused(mg, rows, E, H):
    """The down-projection GEMM that ends with the next LayerNorm (persistent
    kernel, staged epilogue) against the residual GEMM followed by the
    LayerNorm kernel: every output bit-identical."""
    gen = torch.Generator(device="cuda").manual_seed(rows + E + H + 1)
    v = torch.relu(torch.randn(rows, H, device="cuda", generator=gen)).bfloat16()
    dn = (torch.randn(H, E, device="cuda", generator=gen) / H ** 0.5).bfloat16()
    h0 = torch.randn(rows, E, device="cuda", generator=gen).bfloat16()
    g = (1 + 0.1 * torch.randn(E, device="cuda", generator=gen)).bfloat16()
    b = (0.1 * torch.randn(E, device="cuda", generator=gen)).bfloat16()
    # unfused: persistent residual GEMM with the same tile width, then LayerNorm
    h_ref = h0.clone()
    assert mg.mg_gemm_bf16_tiled(v.data_ptr(), 0, H, dn.data_ptr(), 1, E, rows, E, H, 2, h_ref.data_ptr(), E,
                                 h_ref.data_ptr(), E, 1, E, 1, None) == 0, mg.mg_last_error()
    xn_ref = torch.empty(rows, E, device="cuda", dtype=torch.bfloat16)
    y_ref = torch.empty_like(xn_ref)
    sd_ref = torch.empty(rows, device="cuda", dtype=torch.float32)
    assert mg.mg_layernorm_forward(h_ref.data_ptr(), xn_ref.data_ptr(), y_ref.data_ptr(), g.data_ptr(), b.data_ptr(),
                                   sd_ref.data_ptr(), rows, E, None) == 0
    h = h0.clone()
    xn = torch.full_like(xn_ref, float("nan"))
    y = torch.full_like(xn_ref, float("nan"))
    sd = torch.full_like(sd_ref, float("nan"))
    rc = mg.mg_gemm_bf16_resid_layernorm(v.data_ptr(), H, dn.data_ptr(), 1, E, rows, E, H, h.data_ptr(), g.data_ptr(),
                                         b.data_ptr(), xn.data_ptr(), y.data_ptr(), sd.data_ptr(), None)
    assert rc == 0, mg.mg_last_error()
    torch.cuda.synchronize()
    st = ctypes.c_int(0)
    assert mg.mg_device_status(1, ctypes.byref(st)) == 0 and st.value == 0
    assert torch.equal(h.view(torch.int16), h_ref.view(torch.int16))
    assert torch.equal(xn.view(torch.int16), xn_ref.view(torch.int16))
    assert torch.equal(y.view(torch.int16), y_ref.view(torch.int16))
    assert torch.equal(sd, sd_ref)
