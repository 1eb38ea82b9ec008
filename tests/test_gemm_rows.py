"""The row-complete GEMM (K split over a thread-block cluster, partial tiles
summed through distributed shared memory, one warp per output row) against
the same arithmetic in separate kernels: the split-K GEMM's fp32 partials
(same K ranges), summed in split order, then the residual add and the
LayerNorm kernel (forward), or bf16 rounding and the LayerNorm backward
kernel with the residual gradient (backward). Every output is compared bit
for bit, including the dgamma / dbeta partials.
"""
import ctypes

import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def split_k_sum(mg, A, B, b_mn, rows, K):
    """fp32 A B as the cluster computes it: split-K partials, summed in order."""
    ks = mg.mg_gemm_rows_splits(K)
    parts = torch.empty(ks, rows, 128, device="cuda", dtype=torch.float32)
    ldb = 128 if b_mn else K
    assert mg.mg_gemm_bf16(A.data_ptr(), 0, K, B.data_ptr(), int(b_mn), ldb, rows, 128, K, 4, parts.data_ptr(), 128,
                           None, 128, ks, None) == 0, mg.mg_last_error()
    acc = parts[0].clone()
    for r in range(1, ks):
        acc = acc + parts[r]
    return acc


def operands(rows, K, b_mn, seed):
    gen = torch.Generator(device="cuda").manual_seed(seed)
    A = torch.relu(torch.randn(rows, K, device="cuda", generator=gen)).bfloat16()
    B = (torch.randn(K, 128, device="cuda", generator=gen) / K ** 0.5).bfloat16()
    if not b_mn:
        B = B.t().contiguous()  # [N][K]
    return gen, A, B


def status_ok(mg):
    torch.cuda.synchronize()
    st = ctypes.c_int(0)
    assert mg.mg_device_status(1, ctypes.byref(st)) == 0 and st.value == 0, st.value


CASES = [(4096, 512, True), (4096, 512, False), (1000, 512, True), (300, 256, False), (8192, 1024, True),
         (200, 256, True)]


@pytest.mark.parametrize("rows,K,b_mn", CASES)
def test_rows_residual_layernorm_bit_exact(mg, rows, K, b_mn):
    gen, A, B = operands(rows, K, b_mn, rows + K)
    h0 = torch.randn(rows, 128, device="cuda", generator=gen).bfloat16()
    g = (1 + 0.1 * torch.randn(128, device="cuda", generator=gen)).bfloat16()
    b = (0.1 * torch.randn(128, device="cuda", generator=gen)).bfloat16()
    acc = split_k_sum(mg, A, B, b_mn, rows, K)
    h_ref = (h0.float() + acc.bfloat16().float()).bfloat16()
    xn_ref = torch.empty_like(h0)
    y_ref = torch.empty_like(h0)
    sd_ref = torch.empty(rows, device="cuda", dtype=torch.float32)
    assert mg.mg_layernorm_forward(h_ref.data_ptr(), xn_ref.data_ptr(), y_ref.data_ptr(), g.data_ptr(), b.data_ptr(),
                                   sd_ref.data_ptr(), rows, 128, None) == 0
    h = h0.clone()
    xn = torch.full_like(h0, float("nan"))
    y = torch.full_like(h0, float("nan"))
    sd = torch.full_like(sd_ref, float("nan"))
    rc = mg.mg_gemm_rows_resid_layernorm(A.data_ptr(), K, B.data_ptr(), int(b_mn), 128 if b_mn else K, rows, K,
                                         h.data_ptr(), g.data_ptr(), b.data_ptr(), xn.data_ptr(), y.data_ptr(),
                                         sd.data_ptr(), None)
    assert rc == 0, mg.mg_last_error()
    status_ok(mg)
    assert torch.equal(h.view(torch.int16), h_ref.view(torch.int16))
    assert torch.equal(xn.view(torch.int16), xn_ref.view(torch.int16))
    assert torch.equal(y.view(torch.int16), y_ref.view(torch.int16))
    assert torch.equal(sd, sd_ref)


@pytest.mark.parametrize("rows,K,b_mn", [c for c in CASES if c[0] <= 9472])
def test_rows_layernorm_backward_bit_exact(mg, rows, K, b_mn):
    gen, A, B = operands(rows, K, b_mn, 7 * rows + K)
    xn = torch.randn(rows, 128, device="cuda", generator=gen).bfloat16()
    g = (1 + 0.1 * torch.randn(128, device="cuda", generator=gen)).bfloat16()
    sd = 0.5 + torch.rand(rows, device="cuda", generator=gen)
    resid = torch.randn(rows, 128, device="cuda", generator=gen).bfloat16()
    nparts = mg.mg_layernorm_backward_num_partials(rows)
    dz = split_k_sum(mg, A, B, b_mn, rows, K).bfloat16()
    out_ref = resid.clone()  # with a residual, mg_layernorm_backward adds into it in place
    part_ref = torch.empty(nparts, 256, device="cuda", dtype=torch.float32)
    assert mg.mg_layernorm_backward(dz.data_ptr(), xn.data_ptr(), g.data_ptr(), sd.data_ptr(), out_ref.data_ptr(),
                                    part_ref.data_ptr(), rows, 128, None) == 0, mg.mg_last_error()
    out = torch.full_like(resid, float("nan"))
    part = torch.full_like(part_ref, float("nan"))
    rc = mg.mg_gemm_rows_layernorm_backward(A.data_ptr(), K, B.data_ptr(), int(b_mn), 128 if b_mn else K, rows, K,
                                            xn.data_ptr(), g.data_ptr(), sd.data_ptr(), resid.data_ptr(),
                                            out.data_ptr(), part.data_ptr(), None)
    assert rc == 0, mg.mg_last_error()
    status_ok(mg)
    assert torch.equal(out.view(torch.int16), out_ref.view(torch.int16))
    assert torch.equal(part, part_ref)


def test_rows_layernorm_backward_rejects_unsupported_grouping(mg):
    """Row counts whose LayerNorm-backward partial groups do not divide 32 rows
    are refused on the host (the engine keeps the two kernels there)."""
    rows = 16384  # 56 rows per partial
    assert mg.mg_layernorm_backward_num_partials(rows) > 0
    t = torch.zeros(1, device="cuda")
    rc = mg.mg_gemm_rows_layernorm_backward(t.data_ptr(), 512, t.data_ptr(), 1, 128, rows, 512, t.data_ptr(),
                                            t.data_ptr(), t.data_ptr(), t.data_ptr(), t.data_ptr(), t.data_ptr(), None)
    assert rc != 0
