// tcgen05 GEMM engine: D[M x N] = op(A)[M x K] * op(B)[K x N], bf16 operands,
// fp32 accumulation in tensor memory, fused epilogues.
//
// This is the dense-product engine behind every policy layer of the PPO path
// (the products the reference computes with MetalPerformancePrimitives
// matmul2d in model/mlp.metal and model/linear.metal). One CTA computes one
// 128 x BN output tile of one K-split:
//   warp 0 lane 0  TMA producer: 64-wide K blocks of A and B, 128-byte
//                  swizzled, into a STAGES-deep shared-memory ring;
//   warp 1 lane 0  MMA issuer: four tcgen05.mma (128 x BN x 16) per K block,
//                  tcgen05.commit releases the ring slot;
//   warp 2         allocates / frees the TMEM accumulator (BN fp32 columns);
//   warps 0-3      epilogue: warp w reads accumulator lanes 32w..32w+31
//                  (one output row per thread) and applies the fused op.
// Operands may be K-major (rows of K contiguous) or MN-major (K rows of M or N
// contiguous), which covers X W, dZ W^T and X^T dZ without transposes.
// No cluster launch: every CTA loads its own tiles.
#pragma once

#include "gemm.h"
#include "row_epilogues.cuh"
#include "metalgym/detail/tile.cuh"
#include "metalgym/pdl.cuh"
#include "metalgym/detail/ptx.cuh"

namespace mg {


struct GemmParams {
    int M, N, K;
    int kPerSplit;  // multiple of 64
    int tilesM, tilesN, splits;  // work units of the persistent kernel
    PolicyLossRows loss;         // kEpiPolicyLoss: the loss of each output row
    LnOutputs ln;                // kEpiResidLN: the LayerNorm of each output row
    void* out;
    int ldo;
    const __nv_bfloat16* aux;
    int ldaux;
    int* status;
};

template <int BN>
struct GemmShape {
    static constexpr int BM = 128;
    static constexpr int BK = 64;
    static constexpr int STAGES = 4;
    static constexpr int A_BYTES = BM * BK * 2;  // 16 KB
    static constexpr int B_BYTES = BN * BK * 2;
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
    static constexpr int TMEM_COLS = BN < 32 ? 32 : BN;
    static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 /*align*/ + 256 /*barriers*/;
};

__device__ __forceinline__ void store_bf16x32(__nv_bfloat16* dst, const float* v) {
    uint4 w[4];
    uint32_t* u = reinterpret_cast<uint32_t*>(w);
#pragma unroll
    for (int i = 0; i < 16; i++) {
        __nv_bfloat162 h = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
        u[i] = *reinterpret_cast<uint32_t*>(&h);
    }
    uint4* d = reinterpret_cast<uint4*>(dst);
#pragma unroll
    for (int i = 0; i < 4; i++) d[i] = w[i];
}

__device__ __forceinline__ void load_bf16x32(const __nv_bfloat16* src, float* v) {
    const uint4* s = reinterpret_cast<const uint4*>(src);
#pragma unroll
    for (int i = 0; i < 4; i++) {
        uint4 w = s[i];
        const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&w);
#pragma unroll
        for (int j = 0; j < 4; j++) {
            float2 f = __bfloat1622float2(h[j]);
            v[i * 8 + 2 * j] = f.x;
            v[i * 8 + 2 * j + 1] = f.y;
        }
    }
}

template <int BN, bool A_MN, bool B_MN, int EPI>
__global__ void __launch_bounds__(128, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const GemmParams p) {
    using S = GemmShape<BN>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + S::STAGES * S::STAGE_BYTES);
    uint64_t* empty = full + S::STAGES;
    uint64_t* done = empty + S::STAGES;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);

    mg_pdl_trigger();
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int m0 = blockIdx.x * S::BM;
    const int n0 = blockIdx.y * BN;
    const int kBegin = blockIdx.z * p.kPerSplit;
    const int kEnd = min(p.K, kBegin + p.kPerSplit);
    const int nk = kEnd > kBegin ? (kEnd - kBegin + S::BK - 1) / S::BK : 0;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S::STAGES; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(done, 1);
        fence_barrier_init();
        prefetch_tensormap(&tmA);
        prefetch_tensormap(&tmB);
    }
    if (warp == 2) {
        tmem_alloc(tmem_slot, S::TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    mg_pdl_wait();  // operands and aux come from the previous kernel

    if (warp == 0 && lane == 0) {
        // ---- TMA producer
        int issued = 0;
        for (int kb = 0; kb < nk; kb++) {
            const int s = kb % S::STAGES;
            const uint32_t ph = (kb / S::STAGES) & 1;
            if (!mbar_wait(&empty[s], ph ^ 1, p.status, kDevTimeoutEmpty)) break;
            issued = kb + 1;
            uint8_t* sA = smem + s * S::STAGE_BYTES;
            uint8_t* sB = sA + S::A_BYTES;
            const int k0 = kBegin + kb * S::BK;
            mbar_arrive_expect_tx(&full[s], S::STAGE_BYTES);
            if (A_MN) {
                tma_load_2d(sA, &tmA, m0, k0, &full[s]);
                tma_load_2d(sA + 8192, &tmA, m0 + 64, k0, &full[s]);
            } else {
                tma_load_2d(sA, &tmA, k0, m0, &full[s]);
            }
            if (B_MN) {
#pragma unroll
                for (int j = 0; j < BN / 64; j++) tma_load_2d(sB + j * 8192, &tmB, n0 + 64 * j, k0, &full[s]);
            } else {
                tma_load_2d(sB, &tmB, k0, n0, &full[s]);
            }
        }
        // Drain: every issued copy has landed before this CTA can exit (a no-op
        // on the normal path, where the MMA issuer already consumed them all).
        for (int kb = issued - S::STAGES < 0 ? 0 : issued - S::STAGES; kb < issued; kb++)
            mbar_wait(&full[kb % S::STAGES], (kb / S::STAGES) & 1, p.status, kDevTimeoutFull);
    } else if (warp == 1 && lane == 0) {
        // ---- MMA issuer
        constexpr uint32_t idesc = idesc_bf16_f32(BN, A_MN, B_MN);
        for (int kb = 0; kb < nk; kb++) {
            const int s = kb % S::STAGES;
            const uint32_t ph = (kb / S::STAGES) & 1;
            if (!mbar_wait(&full[s], ph, p.status, kDevTimeoutFull)) break;
            tc_fence_after();
            const uint32_t aBase = smem_u32(smem + s * S::STAGE_BYTES);
            const uint32_t bBase = aBase + S::A_BYTES;
#pragma unroll
            for (int kk = 0; kk < 4; kk++) {
                const uint64_t ad = A_MN ? smem_desc_sw128(aBase + kk * 2048, 8192, 1024)
                                         : smem_desc_sw128(aBase + kk * 32, 16, 1024);
                const uint64_t bd = B_MN ? smem_desc_sw128(bBase + kk * 2048, 8192, 1024)
                                         : smem_desc_sw128(bBase + kk * 32, 16, 1024);
                tc_mma_bf16(tmem, ad, bd, idesc, (kb > 0 || kk > 0) ? 1u : 0u);
            }
            tc_commit(&empty[s]);
        }
        // Always commit: `done` then also covers MMAs issued before a timeout,
        // so TMEM is never freed under a running MMA.
        tc_commit(done);
    }

    // ---- epilogue: thread (warp, lane) owns output row m0 + 32 warp + lane
    __syncwarp();
    const bool ready = (nk == 0) || mbar_wait_warp(done, 0, p.status, kDevTimeoutDone);
    tc_fence_after();
    const int row = m0 + warp * 32 + lane;
    if (ready) {
#pragma unroll 1
        for (int c = 0; c < BN / 32; c++) {
            const int col = n0 + c * 32;
            float v[32];
            if (nk > 0) {
                tmem_ld32(tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)(c * 32), v);
            } else {
#pragma unroll
                for (int i = 0; i < 32; i++) v[i] = 0.0f;
            }
            if (row >= p.M || col >= p.N) continue;
            if (EPI == kEpiF32) {
                float* o = static_cast<float*>(p.out) + (size_t)blockIdx.z * p.M * p.ldo + (size_t)row * p.ldo + col;
                float4* o4 = reinterpret_cast<float4*>(o);
#pragma unroll
                for (int i = 0; i < 8; i++) o4[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
            } else {
                __nv_bfloat16* o = static_cast<__nv_bfloat16*>(p.out) + (size_t)row * p.ldo + col;
                if (EPI == kEpiBf16Relu) {
#pragma unroll
                    for (int i = 0; i < 32; i++) {
                        const float r = round_bf16(v[i]);
                        v[i] = r > 0.0f ? r : r * 0.0f;
                    }
                } else if (EPI == kEpiBf16Resid) {
                    float a[32];
                    load_bf16x32(p.aux + (size_t)row * p.ldaux + col, a);
#pragma unroll
                    for (int i = 0; i < 32; i++) v[i] = a[i] + round_bf16(v[i]);
                } else if (EPI == kEpiBf16Mask) {
                    float a[32];
                    load_bf16x32(p.aux + (size_t)row * p.ldaux + col, a);
#pragma unroll
                    for (int i = 0; i < 32; i++) v[i] = round_bf16(v[i]) * (a[i] > 0.0f ? 1.0f : 0.0f);
                }
                store_bf16x32(o, v);
            }
        }
        // the thread's whole head row is stored (one tile spans the 64 columns)
        if (EPI == kEpiPolicyLoss && row < p.M)
            policy_loss_row(p.loss, row, static_cast<const __nv_bfloat16*>(p.out) + (size_t)row * p.ldo, p.status);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 2) {
        tc_fence_after();
        tmem_dealloc(tmem, S::TMEM_COLS);
    }
}

}  // namespace mg
