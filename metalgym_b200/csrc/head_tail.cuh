// The end of a training minibatch's forward and the start of its backward
// over one 128-row tile, for 128-wide embeddings and the categorical head, as
// a pass (tile_pass.cuh): run once by k_head_tail (head_tail.cu) and between
// the block passes by the minibatch kernel (minibatch_tiles.cu):
//
//   logits = bf16(fOut W_head)                  model/linear.metal:17-37
//   PPO loss of each row -> dZ, statistics      model/policy.metal:14-69
//   dS = bf16(dZ W_head^T)                      model/linear.metal:40-60
//   dS = LayerNorm backward of dS (the final
//        LayerNorm; no skip path)               model/layernorm.metal:74-127
//   the 128-row tile's partial of dW_head = fOut^T dZ   model/linear.metal:71-93
//
// Four CTAs per 128-row tile, no exchange between them: the products are
// small (K = 128 and 64), so every CTA computes them for the whole tile, and
// the loss of all 128 rows too (the tile's dZ is the A operand of the second
// product); CTA q writes only the outputs of rows 32q .. 32q + 31 (head row,
// dZ, statistics, dS, its LayerNorm-backward partials) and CTA 0 the
// weight-gradient partial. Every value is the one the separate kernels
// compute (the same products in the same K order, the shared per-row loss and
// LayerNorm code), bit for bit.
#pragma once

#include "gemm.h"
#include "gemm_tc.cuh"
#include "policy.h"
#include "rows_epilogue.cuh"
#include "tile_pass.cuh"

namespace mg {

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
    uint64_t* trace;      // phase trace (tile_pass.cuh); null: off
};


// The maps and parameters of the pass, checked on the host (head_tail.cu;
// the arguments of head_tail, policy.h), without a launch.
int head_tail_args(const void* fOut, const void* wHead, void* head, const PolicyLossRows& loss, float* headPart,
                   const void* gammaF, const void* xNormF, const float* stdevF, void* dS, float* lnPart, int M,
                   CUtensorMap& tf, CUtensorMap& tw, HeadTailParams& p);

// The pass over tile blockIdx.x / 4 as CTA q = blockIdx.x % 4 of the tile;
// AD > 0: the head has AD actions (the loss with its loops unrolled).
// Standalone (!t.merged): frees its 256 TMEM columns (logits 0..63, dW_head
// 64..127, dS 128..255) before the epilogue. Merged: ends at a pass boundary.
template <int RPC, int AD = 0>
__device__ __forceinline__ void ht_pass(uint8_t* smem, const CUtensorMap& tmF, const CUtensorMap& tmW,
                                        const HeadTailParams& p, TilePass& t) {
    __nv_bfloat16* hs = reinterpret_cast<__nv_bfloat16*>(smem + kHtH);
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int q = (int)(blockIdx.x & 3);
    const int tile = (int)(blockIdx.x >> 2);
    const int m0 = tile * kRowsBM;
    const uint32_t tmem = t.tmem;
    t.trace = p.trace;
    tp_mark(t);  // pass start

    if (threadIdx.x == 0) {
        if (t.ok()) {
            t.issuing(kTbFull1);
            mbar_arrive_expect_tx(t.bar(kTbFull1), 32768 + 16384);
            for (int kb = 0; kb < 2; kb++) tma_load_2d(smem + kHtF + kb * 16384, &tmF, 64 * kb, m0, t.bar(kTbFull1));
            tma_load_2d(smem + kHtW, &tmW, 0, 0, t.bar(kTbFull1));  // W_head [128][64]: one 64 x 128 box
        }
    } else if (warp == 1 && lane == 0) {
        if (tp_wait(t, kTbFull1, p.status, kDevTimeoutFull)) {
            tc_fence_after();
            // logits = fOut W_head: A K-major (fOut rows), B = W_head as [K = 128][N = 64], MN-major
            constexpr uint32_t idesc = idesc_bf16_f32(64, false, true);
            const uint32_t a = smem_u32(smem + kHtF), b = smem_u32(smem + kHtW);
#pragma unroll
            for (int s = 0; s < 8; s++)
                tc_mma_bf16(tmem, smem_desc_sw128(a + (s >> 2) * 16384 + (s & 3) * 32, 16, 1024),
                            smem_desc_sw128(b + s * 2048, 8192, 1024), idesc, s > 0 ? 1u : 0u);
        }
        tc_commit(t.bar(kTbMma1));
    }

    // ---- the loss of every row of the tile (threads 0..127: row = thread)
    __syncwarp();
    const bool ok1 = tp_wait_warp(t, kTbMma1, p.status, kDevTimeoutDone);
    tc_fence_after();
    tp_mark(t);  // head product done (warp 0)
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
        if (row < p.M)
            lossOk = policy_loss_compute<AD>(p.loss, row, hs + r * kHtHStride, own ? p.status : nullptr, packed, st);
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
    tp_mark(t);  // loss and dZ tile done
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
        tc_commit(t.bar(kTbMma2));
    }

    // ---- this CTA's 32 rows of dS into the fp32 tile; CTA 0: the dW_head partial
    __syncwarp();
    const bool ok2 = tp_wait_warp(t, kTbMma2, p.status, kDevTimeoutDone) && ok1;
    tc_fence_after();
    tp_mark(t);  // head dX and dW_head products done (warp 0)
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
    if (!t.merged) {
        if (warp == 2) {
            if (!ok2) {
                mbar_wait(t.bar(kTbMma1), 0, p.status, kDevTimeoutDone);
                mbar_wait(t.bar(kTbMma2), 0, p.status, kDevTimeoutDone);
            }
            tc_fence_after();
            tmem_dealloc(tmem, 256);
        }
        if (!ok1 && threadIdx.x == 0) mbar_wait(t.bar(kTbFull1), 0, p.status, kDevTimeoutFull);  // let the loads land
    }

    tp_mark(t);  // dS tile written
    rows_cluster_epilogue<kRowsLNBackward, RPC, 1>(smem, reinterpret_cast<float*>(smem + kHtRed), (uint32_t)q, m0,
                                                   p.e);
    tp_mark(t);  // row epilogue done
    t.flip(kTbFull1);
    t.flip(kTbMma1);
    t.flip(kTbMma2);
    if (t.merged) tp_pass_boundary();
}

}  // namespace mg
