// The end of a training minibatch's forward and the start of its backward in
// one kernel, for 128-wide embeddings and the categorical head:
//
//   logits = bf16(fOut W_head)                  model/linear.metal:17-37
//   PPO loss of each row -> dZ, statistics      model/policy.metal:14-69
//   dS = bf16(dZ W_head^T)                      model/linear.metal:40-60
//   dS = LayerNorm backward of dS (the final
//        LayerNorm; no skip path)               model/layernorm.metal:74-127
//   the 128-row tile's partial of dW_head = fOut^T dZ   model/linear.metal:71-93
//
// Four CTAs per 128-row tile, no cluster: the products are small (K = 128 and
// 64), so every CTA computes them for the whole tile, and the loss of all 128
// rows too (the tile's dZ is the A operand of the second product); CTA q
// writes only the outputs of rows 32q .. 32q + 31 (head row, dZ, statistics,
// dS, its LayerNorm-backward partials) and CTA 0 the weight-gradient partial.
// Three launches and a side-stream GEMM become one kernel on 128 CTAs at 4096
// rows. Every value is the one the separate kernels compute (the same
// products in the same K order, the shared per-row loss and LayerNorm
// code), bit for bit.
#include "gemm.h"
#include "gemm_tc.cuh"
#include "policy.h"
#include "rows_epilogue.cuh"
#include "runtime.h"

namespace mg {

namespace {

// shared memory: F fOut tile (32 KB) | W head weights (16 KB) | D dZ tile
// (16 KB) | H head rows (128 x 66 bf16) | barriers; after the products the fp32
// dS tile reuses [0, 64 KB) and the LayerNorm-backward column sums [64, 96 KB)
constexpr int kHtF = 0, kHtW = 32768, kHtD = 49152, kHtH = 65536;
constexpr int kHtHStride = 66;  // bf16 per head row: 33 words, so the rows of a warp fall in distinct banks
constexpr int kHtRed = 65536, kHtBar = 98304;
constexpr int kHtSmem = kHtBar + 256 + 1024;
static_assert(kHtH + 128 * kHtHStride * 2 <= kHtBar && kRowsTile <= kHtRed && kHtRed + kRowsRedBytes <= kHtBar, "");

struct HeadTailParams {
    int M;
    PolicyLossRows loss;
    __nv_bfloat16* head;  // [M][64] logits + value, as the head GEMM stores them
    float* headPart;      // [tile][128][64] fp32
    RowsEpi e;            // the final LayerNorm's backward: out = dS, no resid
    int* status;
};

template <int RPC>
__global__ void __launch_bounds__(kRowsThreads, 1)
    k_head_tail(const __grid_constant__ CUtensorMap tmF, const __grid_constant__ CUtensorMap tmW,
                const HeadTailParams p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + kHtBar);
    uint64_t* mma1 = full + 1;
    uint64_t* mma2 = full + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(full + 3);
    __nv_bfloat16* hs = reinterpret_cast<__nv_bfloat16*>(smem + kHtH);

    mg_pdl_trigger();
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int q = (int)(blockIdx.x & 3);
    const int tile = (int)(blockIdx.x >> 2);
    const int m0 = tile * kRowsBM;

    if (threadIdx.x == 0) {
        for (int i = 0; i < 3; i++) mbar_init(&full[i], 1);
        fence_barrier_init();
        prefetch_tensormap(&tmF);
        prefetch_tensormap(&tmW);
    }
    if (warp == 2) {
        tmem_alloc(tmem_slot, 256);  // logits 0..63, dW_head 64..127, dS 128..255
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    mg_pdl_wait();

    if (threadIdx.x == 0) {
        mbar_arrive_expect_tx(full, 32768 + 16384);
        for (int kb = 0; kb < 2; kb++) tma_load_2d(smem + kHtF + kb * 16384, &tmF, 64 * kb, m0, full);
        tma_load_2d(smem + kHtW, &tmW, 0, 0, full);  // W_head [128][64]: one 64 x 128 box
    } else if (warp == 1 && lane == 0) {
        if (mbar_wait(full, 0, p.status, kDevTimeoutFull)) {
            tc_fence_after();
            // logits = fOut W_head: A K-major (fOut rows), B = W_head as [K = 128][N = 64], MN-major
            constexpr uint32_t idesc = idesc_bf16_f32(64, false, true);
            const uint32_t a = smem_u32(smem + kHtF), b = smem_u32(smem + kHtW);
#pragma unroll
            for (int s = 0; s < 8; s++)
                tc_mma_bf16(tmem, smem_desc_sw128(a + (s >> 2) * 16384 + (s & 3) * 32, 16, 1024),
                            smem_desc_sw128(b + s * 2048, 8192, 1024), idesc, s > 0 ? 1u : 0u);
        }
        tc_commit(mma1);
    }

    // ---- the loss of every row of the tile (threads 0..127: row = thread)
    __syncwarp();
    const bool ok1 = mbar_wait_warp(mma1, 0, p.status, kDevTimeoutDone);
    tc_fence_after();
    if (warp < 4) {
        const int r = warp * 32 + lane;
        const int row = m0 + r;
        float v[64];
        if (ok1) {
            tmem_ld32(tmem + ((uint32_t)(warp * 32) << 16), v);
            tmem_ld32(tmem + ((uint32_t)(warp * 32) << 16) + 32, v + 32);
        } else {
#pragma unroll
            for (int i = 0; i < 64; i++) v[i] = 0.0f;
        }
        uint32_t hw[32];
#pragma unroll
        for (int i = 0; i < 32; i++) {
            __nv_bfloat162 h2 = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
            hw[i] = *reinterpret_cast<uint32_t*>(&h2);
            reinterpret_cast<uint32_t*>(hs + r * kHtHStride)[i] = hw[i];
        }
        const bool own = warp == q && row < p.M;
        if (own) {
            uint4* dst = reinterpret_cast<uint4*>(p.head + (size_t)row * kLossHeadDim);
#pragma unroll
            for (int i = 0; i < 8; i++) dst[i] = make_uint4(hw[4 * i], hw[4 * i + 1], hw[4 * i + 2], hw[4 * i + 3]);
        }
        uint32_t packed[kLossHeadDim / 2];
        float st[5];
        bool lossOk = false;
        if (row < p.M) lossOk = policy_loss_compute(p.loss, row, hs + r * kHtHStride, own ? p.status : nullptr,
                                                    packed, st);
        if (!lossOk) {
#pragma unroll
            for (int i = 0; i < kLossHeadDim / 2; i++) packed[i] = 0;
        }
        // dZ row into the A tile of the second product (64 bf16: 128-byte swizzled row)
#pragma unroll
        for (int c = 0; c < 8; c++)
            *reinterpret_cast<uint4*>(smem + kHtD + r * 128 + ((c ^ (r & 7)) << 4)) =
                make_uint4(packed[4 * c], packed[4 * c + 1], packed[4 * c + 2], packed[4 * c + 3]);
        if (own && lossOk) {
            uint4* dz = reinterpret_cast<uint4*>(p.loss.dZ + (size_t)row * kLossHeadDim);
#pragma unroll
            for (int c = 0; c < 8; c++)
                dz[c] = make_uint4(packed[4 * c], packed[4 * c + 1], packed[4 * c + 2], packed[4 * c + 3]);
            float* so = p.loss.stats + (size_t)row * 5;
#pragma unroll
            for (int i = 0; i < 5; i++) so[i] = st[i];
        }
    }
    fence_async_smem();  // the dZ tile -> the tensor core
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1 && lane == 0) {
        if (ok1) {
            // dS = dZ W_head^T: A = dZ (K = 64, K-major), B = W_head as [N = 128][K = 64], K-major
            constexpr uint32_t idesc2 = idesc_bf16_f32(128, false, false);
            const uint32_t d = smem_u32(smem + kHtD), w = smem_u32(smem + kHtW), f = smem_u32(smem + kHtF);
#pragma unroll
            for (int s = 0; s < 4; s++)
                tc_mma_bf16(tmem + 128, smem_desc_sw128(d + s * 32, 16, 1024), smem_desc_sw128(w + s * 32, 16, 1024),
                            idesc2, s > 0 ? 1u : 0u);
            if (q == 0) {
                // dW_head partial = fOut^T dZ over the tile's rows: both operands MN-major
                constexpr uint32_t idesc3 = idesc_bf16_f32(64, true, true);
#pragma unroll
                for (int s = 0; s < 8; s++)
                    tc_mma_bf16(tmem + 64, smem_desc_sw128(f + s * 2048, 16384, 1024),
                                smem_desc_sw128(d + s * 2048, 8192, 1024), idesc3, s > 0 ? 1u : 0u);
            }
        }
        tc_commit(mma2);
    }

    // ---- this CTA's 32 rows of dS into the fp32 tile; CTA 0: the dW_head partial
    __syncwarp();
    const bool ok2 = mbar_wait_warp(mma2, 0, p.status, kDevTimeoutDone) && ok1;
    tc_fence_after();
    {
        const int qd = warp & 3, cc = warp >> 2;
        if (qd == q) {
            float v[32];
            if (ok2) {
                tmem_ld32(tmem + 128 + ((uint32_t)(qd * 32) << 16) + (uint32_t)(cc * 32), v);
            } else {
#pragma unroll
                for (int i = 0; i < 32; i++) v[i] = 0.0f;
            }
            const int tr = qd * 32 + lane;
#pragma unroll
            for (int k = 0; k < 8; k++)
                *reinterpret_cast<float4*>(smem + tile_offset(tr, cc * 8 + k)) =
                    make_float4(v[4 * k], v[4 * k + 1], v[4 * k + 2], v[4 * k + 3]);
        }
        if (q == 0 && cc < 2) {
            float v[32];
            if (ok2) {
                tmem_ld32(tmem + 64 + ((uint32_t)(qd * 32) << 16) + (uint32_t)(cc * 32), v);
            } else {
#pragma unroll
                for (int i = 0; i < 32; i++) v[i] = 0.0f;
            }
            float4* o = reinterpret_cast<float4*>(p.headPart + (size_t)tile * kRowsBN * kLossHeadDim +
                                                  (size_t)(qd * 32 + lane) * kLossHeadDim + cc * 32);
#pragma unroll
            for (int i = 0; i < 8; i++) o[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 2) {
        if (!ok2) {
            mbar_wait(mma1, 0, p.status, kDevTimeoutDone);
            mbar_wait(mma2, 0, p.status, kDevTimeoutDone);
        }
        tc_fence_after();
        tmem_dealloc(tmem, 256);
    }
    if (!ok1 && threadIdx.x == 0) mbar_wait(full, 0, p.status, kDevTimeoutFull);  // let the loads land

    rows_cluster_epilogue<kRowsLNBackward, RPC, 1>(smem, reinterpret_cast<float*>(smem + kHtRed), (uint32_t)q, m0,
                                                   p.e);
}

template <int RPC>
int launch_ht(const CUtensorMap& tf, const CUtensorMap& tw, const HeadTailParams& p, cudaStream_t st) {
    auto kern = k_head_tail<RPC>;
    static std::atomic<uint64_t> attr_done{0};
    if (int rc = smem_limit_once(kern, kHtSmem, attr_done)) return rc;
    const int grid = ((p.M + kRowsBM - 1) / kRowsBM) * 4;
    MG_CUDA_TRY(mg_launch(kern, dim3(grid), dim3(kRowsThreads), (size_t)kHtSmem, st, tf, tw, p));
    return check_launch("k_head_tail");
}

}  // namespace

bool head_tail_supported(int E, int M) { return E == kRowsBN && M > 0 && gemm_rows_ln_backward_supported(M); }

int head_tail(const void* fOut, const void* wHead, void* head, const PolicyLossRows& loss, float* headPart,
              const void* gammaF, const void* xNormF, const float* stdevF, void* dS, float* lnPart, int M,
              cudaStream_t st) {
    MG_CHECK_ARG(fOut && wHead && head && headPart && gammaF && xNormF && stdevF && dS && lnPart && loss.dZ &&
                     loss.stats,
                 "head_tail: null argument");
    MG_CHECK_ARG(M > 0 && M == loss.rows && loss.actDim >= 1 && loss.actDim < kLossHeadDim,
                 "head_tail: bad shape");
    MG_CHECK_ARG(gemm_rows_ln_backward_supported(M),
                 "head_tail: the LayerNorm backward partial groups at this row count do not divide 32 rows");
    CUtensorMap tf, tw;
    int rc = make_tmap_bf16(&tf, fOut, kRowsBN, M, kRowsBN, 128);
    if (!rc) rc = make_tmap_bf16(&tw, wHead, kLossHeadDim, kRowsBN, kLossHeadDim, 128);
    if (rc) return rc;
    HeadTailParams p{};
    p.M = M;
    p.loss = loss;
    p.head = static_cast<__nv_bfloat16*>(head);
    p.headPart = headPart;
    p.e.M = M;
    p.e.resid = nullptr;
    p.e.out = static_cast<__nv_bfloat16*>(dS);
    p.e.gamma = static_cast<const __nv_bfloat16*>(gammaF);
    p.e.xNorm = static_cast<const __nv_bfloat16*>(xNormF);
    p.e.stdev = stdevF;
    p.e.partial = lnPart;
    p.status = status_ptr();
    switch (layernorm_rows_per_part(M)) {
        case 8: return launch_ht<8>(tf, tw, p, st);
        case 16: return launch_ht<16>(tf, tw, p, st);
        default: return launch_ht<32>(tf, tw, p, st);
    }
}

}  // namespace mg

extern "C" int mg_head_tail(const void* f_out, const void* w_head, void* head, const int32_t* action,
                            const float* adv, const float* adv_stats, const float* ret, const float* old_log_prob,
                            void* dZ, float* stats, int rows, int act_dim, float clip, float value_coef,
                            float entropy_coef, float* head_part, const void* gamma_f, const void* x_norm_f,
                            const float* stdev_f, void* dS, float* ln_partial, mg_stream_t stream) {
    const mg::PolicyLossRows L = mg::policy_loss_rows(action, adv, adv_stats, ret, old_log_prob, dZ, stats, rows,
                                                      act_dim, mg::LossHyper{clip, value_coef, entropy_coef},
                                                      mg::RowMap{nullptr, 0, 0});
    return mg::head_tail(f_out, w_head, head, L, head_part, gamma_f, x_norm_f, stdev_f, dS, ln_partial, rows,
                         reinterpret_cast<cudaStream_t>(stream));
}
