"""mg_weight_grad_noalloc: the weight gradient for callers that cannot
allocate device memory, checked through the C ABI against the existing
entry points (mg_gemm_bf16 split-K partials + mg_reduce_partials, whose
workspace the caller allocates) on two calls in a row, with the tolerance the
other weight-gradient tests use (rtol 1e-5), and against an independent
fp64 product x^T dz of the same bf16 inputs with the GEMM tests' tolerances
(bf16-rounded output: rtol 1e-2, atol 1e-2 x scale; fp32 output: rtol 2e-3,
atol 1e-3 x scale). Collected last on purpose."""
import ctypes

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def reference_path(mg, x, dz, rows, M, N, splits, round_bf16):
    kps = ((rows + splits - 1) // splits + 63) // 64 * 64
    nsplit = (rows + kps - 1) // kps
    part = torch.zeros(nsplit, M, N, dtype=torch.float32, device="cuda")
    assert mg.mg_gemm_bf16(x.data_ptr(), 1, M, dz.data_ptr(), 1, N, M, N, rows, 4, part.data_ptr(), N, None, 0,
                           nsplit, None) == 0, mg.mg_last_error()
    out = torch.zeros(M, N, dtype=torch.float32, device="cuda")
    norms = torch.zeros(mg.mg_reduce_partials_num_norm_partials(M * N), dtype=torch.float32, device="cuda")
    assert mg.mg_reduce_partials(part.data_ptr(), M * N, nsplit, M * N, out.data_ptr(), round_bf16,
                                 norms.data_ptr(), None) == 0, mg.mg_last_error()
    return out


@pytest.mark.parametrize("rows,M,N,splits,round_bf16", [(4096, 128, 512, 16, 1), (4096, 512, 128, 16, 0),
                                                         (1000, 128, 64, 4, 1)])
def test_noalloc_matches_existing_entry_points_twice(mg, rows, M, N, splits, round_bf16):
    g = torch.Generator(device="cuda").manual_seed(rows + M + N)
    for call in range(2):  # two calls in a row share (and overwrite) the scratch
        x = torch.randn(rows, M, device="cuda", generator=g).bfloat16()
        dz = torch.randn(rows, N, device="cuda", generator=g).bfloat16()
        out = torch.full((M, N), float("nan"), dtype=torch.float32, device="cuda")
        rc = mg.mg_weight_grad_noalloc(x.data_ptr(), dz.data_ptr(), rows, M, N, splits, round_bf16, out.data_ptr(),
                                       None)
        assert rc == 0, mg.mg_last_error()
        ref = reference_path(mg, x, dz, rows, M, N, splits, round_bf16)
        torch.cuda.synchronize()
        st = ctypes.c_int(0)
        assert mg.mg_device_status(1, ctypes.byref(st)) == 0 and st.value == 0
        torch.testing.assert_close(out, ref, rtol=1e-5, atol=1e-6, msg=f"call {call}")
        exact = (x.double().t() @ dz.double()).float()
        scale = exact.abs().max().item()
        if round_bf16:
            torch.testing.assert_close(out, exact, rtol=1e-2, atol=1e-2 * scale, msg=f"call {call} vs fp64")
        else:
            torch.testing.assert_close(out, exact, rtol=2e-3, atol=1e-3 * scale, msg=f"call {call} vs fp64")


def test_noalloc_rejects_sizes_beyond_the_scratch(mg):
    x = torch.zeros(64, 1024, device="cuda").bfloat16()
    dz = torch.zeros(64, 4096, device="cuda").bfloat16()
    out = torch.zeros(1024, 4096, dtype=torch.float32, device="cuda")
    rc = mg.mg_weight_grad_noalloc(x.data_ptr(), dz.data_ptr(), 64, 1024, 4096, 1, 0, out.data_ptr(), None)
    assert rc == 1  # MG_ERR_ARGUMENT: 16 MiB of partials + norm partials > 16 MiB
    assert b"maximum" in mg.mg_last_error()
