// Host launcher for the tcgen05 GEMM engine (gemm_tc.cuh) and its C ABI.
#include "gemm.h"
#include "gemm_tc.cuh"
#include "gemm_tc_persist.cuh"
#include "runtime.h"

namespace mg {

namespace {

template <int BN, bool AMN, bool BMN, int EPI>
int launch_one(const CUtensorMap& ta, const CUtensorMap& tb, const GemmParams& p, int splits, cudaStream_t st) {
    using S = GemmShape<BN>;
    auto kern = gemm_tc_kernel<BN, AMN, BMN, EPI>;
    static std::atomic<uint64_t> attr_done{0};
    if (int rc = smem_limit_once(kern, S::SMEM_BYTES, attr_done)) return rc;
    dim3 grid((p.M + S::BM - 1) / S::BM, (p.N + BN - 1) / BN, splits);
    MG_CUDA_TRY(mg_launch(kern, grid, dim3(128), (size_t)S::SMEM_BYTES, st, ta, tb, p));
    return check_launch("gemm_tc_kernel");
}

// The persistent kernel: one CTA per SM (or fewer when there are fewer units).
template <int BN, bool AMN, bool BMN, int EPI>
int launch_persistent(const CUtensorMap& ta, const CUtensorMap& tb, const GemmParams& p, int splits,
                      cudaStream_t st) {
    using S = PersistShape<BN, EPI>;
    // output / aux maps of the staged epilogue: boxes of 64 columns x 32 rows
    EpiMaps em{};
    if (S::STAGED) {
        int rc = make_tmap_bf16(&em.out, p.out, p.N, p.M, p.ldo, 32);
        if (rc) return rc;
        if (EPI == kEpiBf16Resid || EPI == kEpiBf16Mask || EPI == kEpiResidLN) {
            rc = make_tmap_bf16(&em.aux, p.aux, p.N, p.M, p.ldaux, 32);
            if (rc) return rc;
        }
        if (EPI == kEpiResidLN) {
            rc = make_tmap_bf16(&em.ln, p.ln.out, p.N, p.M, p.N, 32);
            if (rc) return rc;
        }
    }
    auto kern = gemm_tc_persistent<BN, AMN, BMN, EPI>;
    static std::atomic<uint64_t> attr_done{0};
    if (int rc = smem_limit_once(kern, S::SMEM_BYTES, attr_done)) return rc;
    const int units = p.tilesM * p.tilesN * splits;
    const int grid = std::min(units, num_sms());
    MG_CUDA_TRY(mg_launch(kern, dim3(grid), dim3(S::THREADS), (size_t)S::SMEM_BYTES, st, ta, tb, em, p));
    return check_launch("gemm_tc_persistent");
}

template <int BN, bool AMN, bool BMN>
int by_epi(int epi, bool persist, const CUtensorMap& ta, const CUtensorMap& tb, const GemmParams& p, int splits,
           cudaStream_t st) {
    if constexpr (BN >= 128) {
        if (persist) {
        switch (epi) {
            case kEpiBf16: return launch_persistent<BN, AMN, BMN, kEpiBf16>(ta, tb, p, splits, st);
            case kEpiBf16Relu: return launch_persistent<BN, AMN, BMN, kEpiBf16Relu>(ta, tb, p, splits, st);
            case kEpiBf16Resid: return launch_persistent<BN, AMN, BMN, kEpiBf16Resid>(ta, tb, p, splits, st);
            case kEpiBf16Mask: return launch_persistent<BN, AMN, BMN, kEpiBf16Mask>(ta, tb, p, splits, st);
            case kEpiF32: return launch_persistent<BN, AMN, BMN, kEpiF32>(ta, tb, p, splits, st);
            case kEpiResidLN: return launch_persistent<BN, AMN, BMN, kEpiResidLN>(ta, tb, p, splits, st);
        }
        return fail(MG_ERR_ARGUMENT, "unknown GEMM epilogue");
        }
    }
    switch (epi) {
        case kEpiBf16: return launch_one<BN, AMN, BMN, kEpiBf16>(ta, tb, p, splits, st);
        case kEpiBf16Relu: return launch_one<BN, AMN, BMN, kEpiBf16Relu>(ta, tb, p, splits, st);
        case kEpiBf16Resid: return launch_one<BN, AMN, BMN, kEpiBf16Resid>(ta, tb, p, splits, st);
        case kEpiBf16Mask: return launch_one<BN, AMN, BMN, kEpiBf16Mask>(ta, tb, p, splits, st);
        case kEpiF32: return launch_one<BN, AMN, BMN, kEpiF32>(ta, tb, p, splits, st);
        case kEpiPolicyLoss:
            if constexpr (BN == 64) return launch_one<64, AMN, BMN, kEpiPolicyLoss>(ta, tb, p, splits, st);
            break;
    }
    return fail(MG_ERR_ARGUMENT, "unknown GEMM epilogue");
}

template <int BN>
int by_major(bool amn, bool bmn, int epi, bool persist, const CUtensorMap& ta, const CUtensorMap& tb,
             const GemmParams& p, int splits, cudaStream_t st) {
    if (!amn && !bmn) return by_epi<BN, false, false>(epi, persist, ta, tb, p, splits, st);
    if (!amn && bmn) return by_epi<BN, false, true>(epi, persist, ta, tb, p, splits, st);
    if (amn && !bmn) return by_epi<BN, true, false>(epi, persist, ta, tb, p, splits, st);
    return by_epi<BN, true, true>(epi, persist, ta, tb, p, splits, st);
}

// 32-wide tiles: K-major B only (a 32-column MN-major B box would be 64
// bytes wide, not the 128-byte swizzle atom).
int by_major32(bool amn, int epi, const CUtensorMap& ta, const CUtensorMap& tb, const GemmParams& p, int splits,
               cudaStream_t st) {
    return amn ? by_epi<32, true, false>(epi, false, ta, tb, p, splits, st)
               : by_epi<32, false, false>(epi, false, ta, tb, p, splits, st);
}

}  // namespace

int gemm_bf16(const GemmCall& c, cudaStream_t st) {
    MG_CHECK_ARG(c.A && c.B && c.out, "gemm: null pointer");
    MG_CHECK_ARG(c.M > 0 && c.N > 0 && c.K > 0, "gemm: empty shape");
    MG_CHECK_ARG(c.N % 32 == 0, "gemm: N must be a multiple of 32");
    MG_CHECK_ARG(c.lda % 8 == 0 && c.ldb % 8 == 0 && c.ldo % 8 == 0, "gemm: leading dimensions must be multiples of 8");
    MG_CHECK_ARG(c.lda >= (c.a_mn ? c.M : c.K) && c.ldb >= (c.b_mn ? c.N : c.K) && c.ldo >= c.N,
                 "gemm: leading dimension smaller than the matrix");
    MG_CHECK_ARG(c.splits >= 1, "gemm: splits must be >= 1");
    MG_CHECK_ARG(c.splits == 1 || c.epilogue == kEpiF32, "gemm: split-K needs the fp32 epilogue");
    MG_CHECK_ARG(!(c.epilogue == kEpiBf16Resid || c.epilogue == kEpiBf16Mask) || (c.aux && c.ldaux % 8 == 0),
                 "gemm: this epilogue needs aux with ldaux a multiple of 8");
    MG_CHECK_ARG(c.epilogue != kEpiPolicyLoss || (c.N == 64 && c.ldo == 64 && c.splits == 1 && c.loss),
                 "gemm: the policy-loss epilogue needs the 64-column head and its loss arguments");
    MG_CHECK_ARG(c.epilogue != kEpiResidLN ||
                     ((c.N == 128 || c.N == 256) && c.ldo == c.N && c.ldaux == c.N && c.splits == 1 && c.ln),
                 "gemm: the LayerNorm epilogue needs 128 or 256 dense columns and its LayerNorm arguments");
    int kPerSplit = (c.K + c.splits - 1) / c.splits;
    kPerSplit = (kPerSplit + 63) / 64 * 64;
    const int splits = (c.K + kPerSplit - 1) / kPerSplit;

    int bn = c.bn;
    bool persist = c.persistent == 1;
    if (bn == 0) {
        const int sms = num_sms();
        const int tiles128 = ((c.M + 127) / 128) * ((c.N + 127) / 128) * splits;
        const int tiles256 = ((c.M + 127) / 128) * ((c.N + 255) / 256) * splits;
        // split-K weight gradients: one wave of 256-wide tiles on most SMs beats
        // two waves of 128-wide ones (fewer operand bytes through L2)
        const int min256 = c.epilogue == kEpiF32 ? sms * 3 / 4 : sms;
        if (c.persistent != 0 && c.N >= 256 && (c.K >= 1024 || c.N >= 1024) && tiles256 >= min256) {
            // long K: persistent with 256-wide tiles (half the shared-memory
            // traffic per MMA of 128-wide ones); wide N: the operand bytes a
            // tile pulls through L2 per output byte drop by a quarter (at
            // 32768 x 1024 x 256: 23.7 against 28.2 us with ReLU, 38.9 against
            // 48.4 us with the mask)
            bn = 256;
            persist = true;
        } else if (c.persistent != 0 && c.N >= 128 && tiles128 >= sms) {
            // at least a tile per SM: persistent, epilogue of one tile
            // overlapped with the main loop of the next
            bn = 128;
            persist = true;
        } else {
            // one CTA per tile: 128-wide output tiles, or 64-wide ones when
            // 128-wide tiles would leave most of the SMs idle (small row
            // counts), or 32-wide ones (K-major B) when even 64-wide ones would
            const int tiles64 = ((c.M + 127) / 128) * ((c.N + 63) / 64) * splits;
            bn = (c.N >= 128 && tiles128 >= sms) ? 128 : (!c.b_mn && tiles64 < sms / 2) ? 32 : 64;
            persist = false;
        }
    }
    if (c.epilogue == kEpiPolicyLoss) {
        bn = 64;  // one tile spans the head row
        persist = false;
    }
    if (c.epilogue == kEpiResidLN) {
        bn = c.N;  // one tile spans the row; persistent, staged epilogue
        persist = true;
    }
    MG_CHECK_ARG(bn == 32 || bn == 64 || bn == 128 || bn == 256, "gemm: tile N must be 32, 64, 128 or 256");
    MG_CHECK_ARG(bn != 32 || !c.b_mn, "gemm: 32-wide tiles need a K-major B");
    MG_CHECK_ARG(!persist || bn >= 128, "gemm: the persistent kernel needs tile N 128 or 256");

    CUtensorMap ta, tb;
    int rc = c.a_mn ? make_tmap_bf16(&ta, c.A, c.M, c.K, c.lda, 64) : make_tmap_bf16(&ta, c.A, c.K, c.M, c.lda, 128);
    if (rc) return rc;
    rc = c.b_mn ? make_tmap_bf16(&tb, c.B, c.N, c.K, c.ldb, 64) : make_tmap_bf16(&tb, c.B, c.K, c.N, c.ldb, bn);
    if (rc) return rc;

    GemmParams p;
    p.M = c.M;
    p.N = c.N;
    p.K = c.K;
    p.kPerSplit = kPerSplit;
    p.out = c.out;
    p.ldo = c.ldo;
    p.aux = static_cast<const __nv_bfloat16*>(c.aux);
    p.ldaux = c.ldaux;
    p.status = status_ptr();
    if (c.loss) p.loss = *c.loss;
    if (c.ln) p.ln = *c.ln;
    p.tilesM = (c.M + 127) / 128;
    p.tilesN = (c.N + bn - 1) / bn;
    p.splits = splits;
    switch (bn) {
        case 32: return by_major32(c.a_mn, c.epilogue, ta, tb, p, splits, st);
        case 64: return by_major<64>(c.a_mn, c.b_mn, c.epilogue, false, ta, tb, p, splits, st);
        case 128: return by_major<128>(c.a_mn, c.b_mn, c.epilogue, persist, ta, tb, p, splits, st);
        default: return by_major<256>(c.a_mn, c.b_mn, c.epilogue, persist, ta, tb, p, splits, st);
    }
}

}  // namespace mg

extern "C" int mg_gemm_bf16(const void* A_dev, int a_mn_major, int lda, const void* B_dev, int b_mn_major, int ldb,
                            int M, int N, int K, int epilogue, void* out_dev, int ldo, const void* aux_dev, int ldaux,
                            int splits, mg_stream_t stream) {
    mg::GemmCall c;
    c.A = A_dev;
    c.a_mn = a_mn_major != 0;
    c.lda = lda;
    c.B = B_dev;
    c.b_mn = b_mn_major != 0;
    c.ldb = ldb;
    c.M = M;
    c.N = N;
    c.K = K;
    c.epilogue = epilogue;
    c.out = out_dev;
    c.ldo = ldo;
    c.aux = aux_dev;
    c.ldaux = ldaux;
    c.splits = splits;
    return mg::gemm_bf16(c, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int mg_gemm_bf16_tiled(const void* A_dev, int a_mn_major, int lda, const void* B_dev, int b_mn_major,
                                  int ldb, int M, int N, int K, int epilogue, void* out_dev, int ldo,
                                  const void* aux_dev, int ldaux, int splits, int tile_n, int persistent,
                                  mg_stream_t stream) {
    mg::GemmCall c;
    c.A = A_dev;
    c.a_mn = a_mn_major != 0;
    c.lda = lda;
    c.B = B_dev;
    c.b_mn = b_mn_major != 0;
    c.ldb = ldb;
    c.M = M;
    c.N = N;
    c.K = K;
    c.epilogue = epilogue;
    c.out = out_dev;
    c.ldo = ldo;
    c.aux = aux_dev;
    c.ldaux = ldaux;
    c.splits = splits;
    c.bn = tile_n;
    c.persistent = tile_n == 0 ? (persistent ? -1 : 0) : (persistent ? 1 : 0);
    return mg::gemm_bf16(c, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int mg_gemm_bf16_resid_layernorm(const void* A_dev, int lda, const void* B_dev, int b_mn_major, int ldb,
                                            int M, int N, int K, void* h_dev, const void* gamma, const void* beta,
                                            void* x_norm, void* ln_out, float* stdev, mg_stream_t stream) {
    MG_CHECK_ARG(h_dev && gamma && beta && x_norm && ln_out && stdev, "mg_gemm_bf16_resid_layernorm: null argument");
    mg::LnOutputs ln{static_cast<const __nv_bfloat16*>(gamma), static_cast<const __nv_bfloat16*>(beta),
                     static_cast<__nv_bfloat16*>(x_norm), static_cast<__nv_bfloat16*>(ln_out), stdev};
    mg::GemmCall c;
    c.A = A_dev;
    c.lda = lda;
    c.B = B_dev;
    c.b_mn = b_mn_major != 0;
    c.ldb = ldb;
    c.M = M;
    c.N = N;
    c.K = K;
    c.epilogue = mg::kEpiResidLN;
    c.out = h_dev;
    c.ldo = N;
    c.aux = h_dev;
    c.ldaux = N;
    c.ln = &ln;
    return mg::gemm_bf16(c, reinterpret_cast<cudaStream_t>(stream));
}
