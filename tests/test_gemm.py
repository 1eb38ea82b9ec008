"""tcgen05 GEMM engine vs a PyTorch fp32 reference of the same product.

Operands are bf16; the reference multiplies the same bf16 values in fp64 and
applies the epilogue in fp32. Tolerances: bf16 outputs within one bf16
rounding of the reference (rtol 1e-2, atol 1e-2 * scale); fp32 outputs within
accumulation-order noise (rtol 2e-3, atol 1e-3 * scale).
"""
import ctypes

import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

EPI = {"bf16": 0, "relu": 1, "resid": 2, "mask": 3, "f32": 4}


def run_gemm(mg, A, a_mn, B, b_mn, M, N, K, epi, aux=None, splits=1, tile_n=None, persistent=0):
    """A, B are the logical [M,K] and [K,N] bf16 matrices; stores them in the requested major."""
    Ast = (A.t().contiguous() if a_mn else A.contiguous())
    Bst = (B.contiguous() if b_mn else B.t().contiguous())
    lda = M if a_mn else K
    ldb = N if b_mn else K
    if EPI[epi] == 4:
        out = torch.full((splits, M, N), float("nan"), device="cuda", dtype=torch.float32)
    else:
        out = torch.full((M, N), float("nan"), device="cuda", dtype=torch.bfloat16)
    auxp = aux.data_ptr() if aux is not None else None
    if tile_n is None:
        rc = mg.mg_gemm_bf16(Ast.data_ptr(), int(a_mn), lda, Bst.data_ptr(), int(b_mn), ldb, M, N, K, EPI[epi],
                             out.data_ptr(), N, auxp, N, splits, None)
    else:
        rc = mg.mg_gemm_bf16_tiled(Ast.data_ptr(), int(a_mn), lda, Bst.data_ptr(), int(b_mn), ldb, M, N, K,
                                   EPI[epi], out.data_ptr(), N, auxp, N, splits, tile_n, persistent, None)
    assert rc == 0, mg.mg_last_error()
    torch.cuda.synchronize()
    st = ctypes.c_int(0)
    assert mg.mg_device_status(1, ctypes.byref(st)) == 0 and st.value == 0
    return out


def reference(A, B, epi, aux=None):
    acc = (A.double() @ B.double()).float()
    if epi == "f32":
        return acc
    r = acc.bfloat16().float()
    if epi == "relu":
        r = torch.where(r > 0, r, r * 0)
    elif epi == "resid":
        r = (aux.float() + r).bfloat16().float()
    elif epi == "mask":
        r = r * (aux.float() > 0).float()
    return r


SHAPES = [
    (256, 128, 128),
    (4096, 512, 128),   # MLP up-projection at the CartPole config
    (4096, 128, 512),   # MLP down-projection
    (4096, 64, 128),    # policy head
    (200, 96, 96),      # ragged M, N and K tails
]


@pytest.mark.parametrize("a_mn,b_mn", [(0, 0), (0, 1), (1, 0), (1, 1)])
@pytest.mark.parametrize("shape", SHAPES)
def test_gemm_bf16_out(mg, a_mn, b_mn, shape):
    M, N, K = shape
    g = torch.Generator(device="cuda").manual_seed(M * 7 + N * 3 + K)
    A = torch.randn(M, K, device="cuda", generator=g).bfloat16()
    B = torch.randn(K, N, device="cuda", generator=g).bfloat16()
    out = run_gemm(mg, A, a_mn, B, b_mn, M, N, K, "bf16")
    ref = reference(A, B, "bf16")
    scale = ref.abs().max().item()
    torch.testing.assert_close(out.float(), ref, rtol=1e-2, atol=1e-2 * scale)


@pytest.mark.parametrize("epi", ["relu", "resid", "mask"])
def test_gemm_epilogues(mg, epi):
    M, N, K = 512, 256, 128
    g = torch.Generator(device="cuda").manual_seed(11)
    A = torch.randn(M, K, device="cuda", generator=g).bfloat16()
    B = torch.randn(K, N, device="cuda", generator=g).bfloat16()
    aux = torch.randn(M, N, device="cuda", generator=g).bfloat16()
    out = run_gemm(mg, A, 0, B, 1, M, N, K, epi, aux=aux)
    ref = reference(A, B, epi, aux)
    scale = ref.abs().max().item()
    torch.testing.assert_close(out.float(), ref, rtol=1e-2, atol=1e-2 * scale)


@pytest.mark.parametrize("shape,splits", [((128, 512, 4096), 16), ((512, 128, 4096), 8), ((128, 64, 4096), 1),
                                          ((128, 128, 1000), 4)])
def test_gemm_weight_grad_splitk(mg, shape, splits):
    """X^T dZ with K = rows: both operands MN-major, fp32 split-K partials."""
    M, N, K = shape
    g = torch.Generator(device="cuda").manual_seed(5)
    X = torch.randn(K, M, device="cuda", generator=g).bfloat16()   # rows x features
    dZ = torch.randn(K, N, device="cuda", generator=g).bfloat16()  # rows x outputs
    kps = ((K + splits - 1) // splits + 63) // 64 * 64
    real_splits = (K + kps - 1) // kps
    out = run_gemm(mg, X.t(), 1, dZ, 1, M, N, K, "f32", splits=real_splits)
    total = out.sum(0)
    ref = reference(X.t(), dZ, "f32")
    scale = ref.abs().max().item()
    torch.testing.assert_close(total, ref, rtol=2e-3, atol=1e-3 * scale)


def test_gemm_down_projection_single_launch(mg):
    """One launch of the policy's down-projection with the fused residual add
    (rows x embed x hidden = 4096 x 128 x 512): the kernel the profiles
    capture (ncu -k regex:gemm_tc_kernel -c 1 on this test)."""
    M, N, K = 4096, 128, 512
    g = torch.Generator(device="cuda").manual_seed(21)
    V = torch.relu(torch.randn(M, K, device="cuda", generator=g)).bfloat16()
    Dp = (torch.randn(K, N, device="cuda", generator=g) / 16).bfloat16()
    h = torch.randn(M, N, device="cuda", generator=g).bfloat16()
    out = run_gemm(mg, V, 0, Dp, 1, M, N, K, "resid", aux=h)
    ref = reference(V, Dp, "resid", h)
    torch.testing.assert_close(out.float(), ref, rtol=1e-2, atol=1e-2 * ref.abs().max().item())


# The persistent kernel (one CTA per SM over the tiles, double-buffered
# accumulator) and the 256-wide one-CTA-per-tile kernel, on shapes with more
# tiles than SMs (so each CTA walks several units and reuses both
# accumulators), ragged M / N / K and every epilogue.
KERNELS = [(128, 1), (256, 1), (256, 0)]


@pytest.mark.parametrize("epi", ["bf16", "resid", "mask"])
@pytest.mark.parametrize("shape", [(4096, 128, 512), (1000, 96, 200)])
def test_gemm_32_wide_tiles(mg, epi, shape):
    """32-wide output tiles (K-major B), used for small-N products such as
    dBranch = dV Up^T at 4096 rows."""
    M, N, K = shape
    g = torch.Generator(device="cuda").manual_seed(M + N + K + len(epi))
    A = torch.randn(M, K, device="cuda", generator=g).bfloat16()
    B = torch.randn(K, N, device="cuda", generator=g).bfloat16()
    aux = torch.randn(M, N, device="cuda", generator=g).bfloat16()
    out = run_gemm(mg, A, 0, B, 0, M, N, K, epi, aux=aux, tile_n=32, persistent=0)
    ref = reference(A, B, epi, aux)
    torch.testing.assert_close(out.float(), ref, rtol=1e-2, atol=1e-2 * ref.abs().max().item())
BIG_SHAPES = [
    (8192, 1024, 256),   # up-projection at the scale-out widths (train minibatch 8192 rows)
    (4096, 256, 1024),   # down-projection
    (1000, 288, 200),    # ragged M, N and K tails
]


@pytest.mark.parametrize("tile_n,persistent", KERNELS)
@pytest.mark.parametrize("a_mn,b_mn", [(0, 0), (0, 1), (1, 1)])
@pytest.mark.parametrize("shape", BIG_SHAPES)
def test_gemm_tiled_kernels(mg, tile_n, persistent, a_mn, b_mn, shape):
    M, N, K = shape
    g = torch.Generator(device="cuda").manual_seed(M + N + K + tile_n)
    A = torch.randn(M, K, device="cuda", generator=g).bfloat16()
    B = torch.randn(K, N, device="cuda", generator=g).bfloat16()
    out = run_gemm(mg, A, a_mn, B, b_mn, M, N, K, "bf16", tile_n=tile_n, persistent=persistent)
    ref = reference(A, B, "bf16")
    torch.testing.assert_close(out.float(), ref, rtol=1e-2, atol=1e-2 * ref.abs().max().item())


@pytest.mark.parametrize("tile_n,persistent", KERNELS)
@pytest.mark.parametrize("epi", ["relu", "resid", "mask"])
def test_gemm_tiled_epilogues(mg, tile_n, persistent, epi):
    M, N, K = 8192, 512, 256
    g = torch.Generator(device="cuda").manual_seed(17)
    A = torch.randn(M, K, device="cuda", generator=g).bfloat16()
    B = torch.randn(K, N, device="cuda", generator=g).bfloat16()
    aux = torch.randn(M, N, device="cuda", generator=g).bfloat16()
    out = run_gemm(mg, A, 0, B, 1, M, N, K, epi, aux=aux, tile_n=tile_n, persistent=persistent)
    ref = reference(A, B, epi, aux)
    torch.testing.assert_close(out.float(), ref, rtol=1e-2, atol=1e-2 * ref.abs().max().item())


@pytest.mark.parametrize("tile_n,persistent", KERNELS)
def test_gemm_tiled_splitk(mg, tile_n, persistent):
    M, N, K, splits = 256, 1024, 8192, 8
    g = torch.Generator(device="cuda").manual_seed(23)
    X = torch.randn(K, M, device="cuda", generator=g).bfloat16()
    dZ = torch.randn(K, N, device="cuda", generator=g).bfloat16()
    out = run_gemm(mg, X.t(), 1, dZ, 1, M, N, K, "f32", splits=splits, tile_n=tile_n, persistent=persistent)
    ref = reference(X.t(), dZ, "f32")
    torch.testing.assert_close(out.sum(0), ref, rtol=2e-3, atol=1e-3 * ref.abs().max().item())


def test_gemm_default_choice_is_persistent_for_large_problems(mg):
    """The library's own choice on a large shape (persistent, 256-wide)
    matches the reference too, in place (out aliases aux, as the residual
    stream update does)."""
    M, N, K = 32768, 256, 1024
    g = torch.Generator(device="cuda").manual_seed(29)
    V = torch.relu(torch.randn(M, K, device="cuda", generator=g)).bfloat16()
    Dp = (torch.randn(K, N, device="cuda", generator=g) / 16).bfloat16()
    h = torch.randn(M, N, device="cuda", generator=g).bfloat16()
    ref = reference(V, Dp, "resid", h)
    rc = mg.mg_gemm_bf16(V.data_ptr(), 0, K, Dp.data_ptr(), 1, N, M, N, K, EPI["resid"], h.data_ptr(), N,
                         h.data_ptr(), N, 1, None)
    assert rc == 0, mg.mg_last_error()
    torch.cuda.synchronize()
    st = ctypes.c_int(0)
    assert mg.mg_device_status(1, ctypes.byref(st)) == 0 and st.value == 0
    torch.testing.assert_close(h.float(), ref, rtol=1e-2, atol=1e-2 * ref.abs().max().item())
