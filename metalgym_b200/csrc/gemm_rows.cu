// Row-complete GEMM for 128-wide outputs with the row epilogue of the layer
// that follows it:
//
//   out[M x 128] = A[M x K] B[K x 128]   (A K-major; B K- or MN-major)
//
// The K dimension is split over a cluster of 4 CTAs (K a multiple of 256), and
// the 4 fp32 partial tiles are summed through distributed shared memory, so a
// 4096-row product runs on 128 CTAs while every output row still ends in one
// warp, which applies a row epilogue needing the whole row:
//
//   kRowsResidLN     h = bf16(h + bf16(acc)) in place, then the LayerNorm of
//                    h: the down projection of a residual block followed by
//                    the next block's (or the final) LayerNorm
//                    (model/mlp.metal:60-86, model/elementwise.metal:4-13,
//                    model/layernorm.metal:10-71), in the arithmetic of
//                    k_layernorm_forward (lane l: columns 4l..4l+3)
//   kRowsLNBackward  dz = bf16(acc), then the LayerNorm backward of dz with
//                    the residual gradient added: the branch gradient of a
//                    residual block followed by its LayerNorm backward
//                    (model/mlp.metal:131-153, model/layernorm.metal:74-127,
//                    model/ppo.h:851-852), in the arithmetic of
//                    k_layernorm_backward, including its dgamma / dbeta
//                    partial sums over groups of RPC rows
//
// CTA q of a cluster computes the K range [q kPer, (q + 1) kPer) of one
// 128 x 128 tile (TMA ring, tcgen05.mma into TMEM, one thread per row reads
// the accumulator), writes its fp32 tile into its own shared memory, and
// after a cluster barrier owns tile rows [32 q, 32 q + 32): lane l of a warp
// sums columns 4l..4l+3 of a row over the cluster's partial tiles in split
// order. That is the split-K product (kEpiF32 partials with the same kPer)
// followed by an ordered fp32 reduction, bit for bit. Every wait is bounded;
// the cluster barriers are reached by every thread on every path.
#include "gemm.h"
#include "gemm_tc.cuh"
#include "policy.h"
#include "policy_kernels.cuh"
#include "rows_epilogue.cuh"
#include "runtime.h"

namespace mg {

namespace {

constexpr int kRowsStages = 2;
constexpr int kRowsA = kRowsBM * 64 * 2;  // 16 KB per 64-wide K block
constexpr int kRowsB = kRowsBN * 64 * 2;
constexpr int kRowsStage = kRowsA + kRowsB;
constexpr int kRowsRing = kRowsStages * kRowsStage;  // 64 KB
// after the MMAs the ring holds the fp32 partial tile (64 KB, read by the
// whole cluster); the LayerNorm-backward column sums (32 KB, this CTA) follow
// it. About 97 KB in all: two CTAs fit on an SM, so the next kernel's CTAs
// can start (programmatic dependent launch) beside this one's.
constexpr int kRowsRedOff = kRowsRing;
constexpr int kRowsSmem = kRowsRing + kRowsRedBytes + 256 + 1024;
static_assert(kRowsTile <= kRowsRing, "the partial tile must fit in the ring");
constexpr int kRowsSmemOnePerSm = 120 * 1024;  // more than half an SM's 228 KB
static_assert(kRowsSmemOnePerSm >= kRowsSmem, "");

struct RowsParams {
    int M, K, kPer;
    RowsEpi e;
    int* status;
};

template <bool B_MN, int EPI, int RPC>
__global__ void __launch_bounds__(kRowsThreads, 2)
    k_gemm_rows(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, const RowsParams p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + kRowsRing + kRowsRedBytes);
    uint64_t* empty = full + kRowsStages;
    uint64_t* done = empty + kRowsStages;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);

    mg_pdl_trigger();
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t q = cluster_ctarank();
    const int m0 = (int)(blockIdx.x / kRowsCluster) * kRowsBM;
    const int kBegin = (int)q * p.kPer;
    const int kEnd = min(p.K, kBegin + p.kPer);
    const int nk = kEnd > kBegin ? (kEnd - kBegin + 63) / 64 : 0;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kRowsStages; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(done, 1);
        fence_barrier_init();
        prefetch_tensormap(&tmA);
        prefetch_tensormap(&tmB);
    }
    if (warp == 2) {
        tmem_alloc(tmem_slot, kRowsBN);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    mg_pdl_wait();  // operands and the row inputs come from earlier kernels

    if (warp == 0 && lane == 0) {
        // ---- TMA producer
        int issued = 0;
        for (int kb = 0; kb < nk; kb++) {
            const int s = kb % kRowsStages;
            if (!mbar_wait(&empty[s], ((kb / kRowsStages) & 1) ^ 1, p.status, kDevTimeoutEmpty)) break;
            issued = kb + 1;
            uint8_t* sA = smem + s * kRowsStage;
            uint8_t* sB = sA + kRowsA;
            const int k0 = kBegin + kb * 64;
            mbar_arrive_expect_tx(&full[s], kRowsStage);
            tma_load_2d(sA, &tmA, k0, m0, &full[s]);
            if (B_MN) {
                tma_load_2d(sB, &tmB, 0, k0, &full[s]);
                tma_load_2d(sB + 8192, &tmB, 64, k0, &full[s]);
            } else {
                tma_load_2d(sB, &tmB, k0, 0, &full[s]);
            }
        }
        for (int kb = issued - kRowsStages < 0 ? 0 : issued - kRowsStages; kb < issued; kb++)
            mbar_wait(&full[kb % kRowsStages], (kb / kRowsStages) & 1, p.status, kDevTimeoutFull);
    } else if (warp == 1 && lane == 0) {
        // ---- MMA issuer
        constexpr uint32_t idesc = idesc_bf16_f32(kRowsBN, false, B_MN);
        for (int kb = 0; kb < nk; kb++) {
            const int s = kb % kRowsStages;
            if (!mbar_wait(&full[s], (kb / kRowsStages) & 1, p.status, kDevTimeoutFull)) break;
            tc_fence_after();
            const uint32_t aBase = smem_u32(smem + s * kRowsStage);
            const uint32_t bBase = aBase + kRowsA;
#pragma unroll
            for (int kk = 0; kk < 4; kk++) {
                const uint64_t ad = smem_desc_sw128(aBase + kk * 32, 16, 1024);
                const uint64_t bd = B_MN ? smem_desc_sw128(bBase + kk * 2048, 8192, 1024)
                                         : smem_desc_sw128(bBase + kk * 32, 16, 1024);
                tc_mma_bf16(tmem, ad, bd, idesc, (kb > 0 || kk > 0) ? 1u : 0u);
            }
            tc_commit(&empty[s]);
        }
        tc_commit(done);
    }

    // ---- this CTA's fp32 partial tile into shared memory (the ring is free
    // once `done` fired: every MMA, and so every read of the ring, completed).
    // Warp w reads TMEM lanes 32 (w % 4) .. (its quadrant), columns 32 (w / 4) ..
    __syncwarp();
    const bool ready = (nk == 0) || mbar_wait_warp(done, 0, p.status, kDevTimeoutDone);
    tc_fence_after();
    rows_tmem_to_tile(smem, tmem, ready && nk > 0);
    tc_fence_before();
    __syncthreads();
    if (warp == 2) {
        if (!ready) mbar_wait(done, 0, p.status, kDevTimeoutDone);  // no MMA runs on freed TMEM
        tc_fence_after();
        tmem_dealloc(tmem, kRowsBN);
    }
    cluster_sync();  // every partial tile of the cluster is complete

    rows_cluster_epilogue<EPI, RPC>(smem, reinterpret_cast<float*>(smem + kRowsRedOff), q, m0, p.e);
    cluster_sync();  // no CTA leaves while another still reads its partial tile
}

template <bool BMN, int EPI, int RPC>
int launch_rows(const CUtensorMap& ta, const CUtensorMap& tb, const RowsParams& p, int ks, cudaStream_t st) {
    auto kern = k_gemm_rows<BMN, EPI, RPC>;
    static std::atomic<uint64_t> attr_done{0};
    if (int rc = smem_limit_once(kern, kRowsSmemOnePerSm, attr_done)) return rc;
    const int grid = ((p.M + kRowsBM - 1) / kRowsBM) * ks;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)grid);
    cfg.blockDim = dim3(kRowsThreads);
    // a grid that fits the SMs one CTA each asks for more shared memory than
    // two CTAs could share, so that every CTA gets an SM of its own (packed
    // two to an SM, half the SMs would idle: 8.7 against 6.7 us at 4096 rows)
    cfg.dynamicSmemBytes = grid <= num_sms() ? kRowsSmemOnePerSm : kRowsSmem;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = (unsigned)ks;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    MG_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, ta, tb, p));
    return check_launch("k_gemm_rows");
}

int rows_maps(CUtensorMap* ta, CUtensorMap* tb, const void* A, int lda, const void* B, bool b_mn, int ldb, int M,
              int K) {
    int rc = make_tmap_bf16(ta, A, K, M, lda, 128);
    if (rc) return rc;
    return b_mn ? make_tmap_bf16(tb, B, kRowsBN, K, ldb, 64) : make_tmap_bf16(tb, B, K, kRowsBN, ldb, 128);
}

}  // namespace

int gemm_rows_splits(int) { return (int)kRowsCluster; }

bool gemm_rows_supported(int N, int K) { return N == kRowsBN && K > 0 && K % (64 * (int)kRowsCluster) == 0; }

int gemm_rows_resid_layernorm(const void* A, int lda, const void* B, bool b_mn, int ldb, int M, int K, void* h,
                              const LnOutputs& ln, cudaStream_t st) {
    MG_CHECK_ARG(A && B && h && ln.gamma && ln.beta && ln.xNorm && ln.out && ln.stdev, "gemm_rows: null argument");
    MG_CHECK_ARG(M > 0 && gemm_rows_supported(kRowsBN, K), "gemm_rows: needs M > 0, K a multiple of 256");
    const int ks = gemm_rows_splits(K);
    CUtensorMap ta, tb;
    if (int rc = rows_maps(&ta, &tb, A, lda, B, b_mn, ldb, M, K)) return rc;
    RowsParams p{};
    p.M = M;
    p.K = K;
    p.kPer = K / ks;
    p.e.M = M;
    p.e.resid = static_cast<const __nv_bfloat16*>(h);
    p.e.out = static_cast<__nv_bfloat16*>(h);
    p.e.ln = ln;
    p.status = status_ptr();
    return b_mn ? launch_rows<true, kRowsResidLN, 32>(ta, tb, p, ks, st)
                : launch_rows<false, kRowsResidLN, 32>(ta, tb, p, ks, st);
}

bool gemm_rows_ln_backward_supported(int M) {
    const int rpc = layernorm_rows_per_part(M);
    return rpc == 8 || rpc == 16 || rpc == 32;
}

int gemm_rows_layernorm_backward(const void* A, int lda, const void* B, bool b_mn, int ldb, int M, int K,
                                 const void* xNorm, const void* gamma, const float* stdev, const void* resid,
                                 void* residOut, float* partial, cudaStream_t st) {
    MG_CHECK_ARG(A && B && xNorm && gamma && stdev && resid && residOut && partial, "gemm_rows: null argument");
    MG_CHECK_ARG(M > 0 && gemm_rows_supported(kRowsBN, K), "gemm_rows: needs M > 0, K a multiple of 256");
    MG_CHECK_ARG(gemm_rows_ln_backward_supported(M),
                 "gemm_rows: the LayerNorm backward partial groups at this row count do not divide 32 rows");
    const int ks = gemm_rows_splits(K);
    CUtensorMap ta, tb;
    if (int rc = rows_maps(&ta, &tb, A, lda, B, b_mn, ldb, M, K)) return rc;
    RowsParams p{};
    p.M = M;
    p.K = K;
    p.kPer = K / ks;
    p.e.M = M;
    p.e.resid = static_cast<const __nv_bfloat16*>(resid);
    p.e.out = static_cast<__nv_bfloat16*>(residOut);
    p.e.gamma = static_cast<const __nv_bfloat16*>(gamma);
    p.e.xNorm = static_cast<const __nv_bfloat16*>(xNorm);
    p.e.stdev = stdev;
    p.e.partial = partial;
    p.status = status_ptr();
    switch (layernorm_rows_per_part(M)) {
        case 8:
            return b_mn ? launch_rows<true, kRowsLNBackward, 8>(ta, tb, p, ks, st)
                        : launch_rows<false, kRowsLNBackward, 8>(ta, tb, p, ks, st);
        case 16:
            return b_mn ? launch_rows<true, kRowsLNBackward, 16>(ta, tb, p, ks, st)
                        : launch_rows<false, kRowsLNBackward, 16>(ta, tb, p, ks, st);
        default:
            return b_mn ? launch_rows<true, kRowsLNBackward, 32>(ta, tb, p, ks, st)
                        : launch_rows<false, kRowsLNBackward, 32>(ta, tb, p, ks, st);
    }
}

}  // namespace mg

extern "C" int mg_gemm_rows_resid_layernorm(const void* A_dev, int lda, const void* B_dev, int b_mn_major, int ldb,
                                            int M, int K, void* h_dev, const void* gamma, const void* beta,
                                            void* x_norm, void* ln_out, float* stdev, mg_stream_t stream) {
    const mg::LnOutputs ln{static_cast<const __nv_bfloat16*>(gamma), static_cast<const __nv_bfloat16*>(beta),
                           static_cast<__nv_bfloat16*>(x_norm), static_cast<__nv_bfloat16*>(ln_out), stdev};
    return mg::gemm_rows_resid_layernorm(A_dev, lda, B_dev, b_mn_major != 0, ldb, M, K, h_dev, ln,
                                         reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int mg_gemm_rows_layernorm_backward(const void* A_dev, int lda, const void* B_dev, int b_mn_major, int ldb,
                                               int M, int K, const void* x_norm, const void* gamma,
                                               const float* stdev, const void* resid, void* resid_out,
                                               float* partial, mg_stream_t stream) {
    return mg::gemm_rows_layernorm_backward(A_dev, lda, B_dev, b_mn_major != 0, ldb, M, K, x_norm, gamma, stdev,
                                            resid, resid_out, partial, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int mg_gemm_rows_splits(int K) { return mg::gemm_rows_splits(K); }
