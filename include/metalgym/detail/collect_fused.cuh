// collect() (model/ppo.h:716-751) as one persistent kernel for the
// CartPole-sized policy (embed 128, hidden 512, 1..4 residual blocks):
// every forward, sample and environment step of the T-step rollout, the
// bootstrap forward and the GAE scan (model/gae.metal:14-36) of 128
// environments run in one 4-CTA cluster that never leaves the SMs.
//
// A cluster owns environment rows m0 .. m0 + 127 for the whole rollout. CTA
// q of the cluster owns hidden columns 128q .. 128q + 127 of every block and
// environment rows m0 + 32q .. m0 + 32q + 31; its warp q keeps those
// environments' State, RNG word and done flag in registers (one lane per
// environment, rollout.h:31-54) across all T steps. Per step:
//
//   input layer + LayerNorm 0 of the CTA's 32 rows    model/input.metal:11-27,
//     (observations from the previous step, in          model/layernorm.metal:10-71
//     shared memory), h kept in registers; the LayerNorm output is written
//     into the A tile of every CTA of the cluster (distributed shared memory)
//   per block l:
//     V_q = relu(bf16(X W_up[:, 128q..]))           tcgen05, K = 128, TMEM
//     P_q = V_q W_down[128q.., :]                   tcgen05, K = 128 (partial)
//     h = bf16(h + bf16(P_0 + P_1 + P_2 + P_3))     model/mlp.metal:18-86,
//     X = LayerNorm_{l+1}(h) into every CTA's A tile   model/elementwise.metal:4-13
//   logits | value = bf16(X W_head)                 model/linear.metal:17-37
//   warp q: sample (model/sample.metal:18-47 or model/gaussian.metal:42-71),
//     reset-if-done and step its environments, record the slots
//     (model/ppo.h:727-733); the new observations feed the next step
//
// The weight slices of the next block are loaded by TMA (from L2) while the
// current block's epilogue runs. Every product and every row epilogue is the
// one the per-step path computes (block_cluster.cu's K split and CTA-order
// partial sums, the head product of head_tail.cu, the samplers and
// environment code of register_env.cuh), so the rollout is bit-identical to
// the captured per-step graph of the engine at the row counts where that
// graph uses the cluster block kernels (up to 4096 rows).
//
// The environment is a template argument: MG_REGISTER_ENV instantiates the
// kernel in the environment's own translation unit (compiled with
// --fmad=false like every environment translation unit; the policy
// arithmetic here uses explicitly rounded operations and is unaffected) and
// registers collect_fused_launch<Env> in its mg_env_ops. The library builds
// the tensor maps and parameters (metalgym_b200/csrc/collect_fused.cu).
//
// Every wait is bounded (ptx.cuh); after a wait gives up, the CTA stops
// issuing copies and products, still takes part in every cluster barrier,
// lets its copies and products in flight complete before it frees TMEM, and
// the host sees the error in the device status word.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../metalgym_b200.h"
#include "../env_traits.cuh"
#include "../pdl.cuh"
#include "ptx.cuh"
#include "tile.cuh"

namespace mg {

constexpr int kCollectFusedMaxBlocks = 4;
constexpr int kCollectFusedMaxInputDim = 32;

constexpr int kCfE = kRowsBN;                       // 128
constexpr int kCfH = kRowsBN * (int)kRowsCluster;   // 512
constexpr int kCfTile = 128 * 128 * 2;              // one bf16 operand tile (32 KB)
constexpr int kCfHeadCols = kHeadDim;               // 64
constexpr int kCfHStride = 66;                      // bf16 per staged head row (33 words: distinct banks per lane)
// shared memory (offsets from the 1024-aligned base)
constexpr int kCfX = 0;                             // A operand: LayerNorm output of the tile's 128 rows
constexpr int kCfWU = kCfX + kCfTile;               // W_up[:, 128q ..] of the current block (MN-major)
constexpr int kCfWD = kCfWU + kCfTile;              // W_down[128q .., :] of the current block (MN-major)
constexpr int kCfV = kCfWD + kCfTile;               // relu(X W_up) slice: the A operand of the down product
constexpr int kCfP = kCfV + kCfTile;                // fp32 partial of the down product (64 KB)
constexpr int kCfWH = kCfP + kRowsTile;             // W_head [128][64] (MN-major, 16 KB)
constexpr int kCfHS = kCfWH + kCfE * kCfHeadCols * 2;  // head rows of this CTA's 32 environments (bf16)
constexpr int kCfIn = kCfHS + 32 * kCfHStride * 2;  // input weights [inDim][128] bf16
constexpr int kCfObs = kCfIn + kCollectFusedMaxInputDim * kCfE * 2;  // observations [32][inDim] fp32
constexpr int kCfBar = kCfObs + 32 * kCollectFusedMaxInputDim * 4;
constexpr int kCfSmem = kCfBar + 128 + 1024;
static_assert(kCfWH % 1024 == 0 && kCfIn % 16 == 0 && kCfObs % 16 == 0 && kCfBar % 8 == 0, "");
static_assert(kCfSmem <= 232448, "the fused collect kernel's shared memory exceeds 227 KB");
constexpr uint32_t kCfTmemCols = 512;  // up 0..127 | down partial 128..255 | head 256..319

struct CfMaps {
    CUtensorMap up[kCollectFusedMaxBlocks];    // W_up [128][512], boxes 64 x 64
    CUtensorMap down[kCollectFusedMaxBlocks];  // W_down [512][128], boxes 64 x 64
    CUtensorMap head;                          // W_head [128][64], one 64 x 128 box
};

struct CfParams {
    int R, T, L;
    const __nv_bfloat16* wIn;
    const __nv_bfloat16* bIn;
    const __nv_bfloat16* lnG[kCollectFusedMaxBlocks + 1];
    const __nv_bfloat16* lnB[kCollectFusedMaxBlocks + 1];
    const __nv_bfloat16* logStd;
    void* states;
    uint8_t* done;
    uint32_t* rng;
    float* obsSlots;
    void* actionSlots;
    float *logpSlots, *valueSlots, *rewardSlots;
    uint8_t* doneSlots;
    float *advSlots, *retSlots;
    __nv_bfloat16* bootHead;
    float gamma, lambda;
    int* status;
};

// A warp-uniform bounded wait that is skipped (false) once the CTA gave up.
__device__ __forceinline__ bool cf_wait_warp(uint64_t* bar, uint32_t parity, volatile int* sOk, int* status,
                                             int code) {
    const int go = __shfl_sync(0xffffffffu, *sOk, 0);
    if (!go) return false;
    const bool r = mbar_wait_warp(bar, parity, status, code);
    if (!r && (threadIdx.x & 31) == 0) *sOk = 0;
    return r;
}

// The LayerNorm of this thread's two rows (tile rows 32q + warp + 16t;
// lane l: columns 4l..4l+3) whose values v are already bf16, with the
// arithmetic and summation order of k_layernorm_forward, and its output
// written into the A tile of every CTA of the cluster (rows past R: zeros).
__device__ __forceinline__ void cf_layernorm_to_tiles(uint8_t* smem, uint32_t q, const float (&v)[2][4],
                                                      const bool (&live)[2], const __nv_bfloat16* gamma,
                                                      const __nv_bfloat16* beta) {
    constexpr float kInvE = 1.0f / kCfE;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int c0 = lane * 4;
    const float4 gm = bf4_load(gamma + c0), bt = bf4_load(beta + c0);
    const float g[4] = {gm.x, gm.y, gm.z, gm.w}, bb[4] = {bt.x, bt.y, bt.z, bt.w};
    float ms[4];
#pragma unroll
    for (int t = 0; t < 2; t++) {
        float sm = 0.0f;
#pragma unroll
        for (int i = 0; i < 4; i++) sm = __fadd_rn(sm, v[t][i]);
        ms[t] = sm;
    }
    warp_sum_n<2>(ms);
#pragma unroll
    for (int t = 0; t < 2; t++) {
        ms[t] = __fmul_rn(ms[t], kInvE);
        float sq = 0.0f;
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const float d = __fsub_rn(v[t][i], ms[t]);
            sq = __fadd_rn(sq, __fmul_rn(d, d));
        }
        ms[2 + t] = sq;
    }
    warp_sum_n<2>(ms + 2);
#pragma unroll
    for (int t = 0; t < 2; t++) {
        const int r = 32 * (int)q + warp + 16 * t;  // row of the tile
        const float sd = __fsqrt_rn(__fadd_rn(__fmul_rn(ms[2 + t], kInvE), 1e-5f));
        const float rstd = __frcp_rn(sd);
        float y[4];
#pragma unroll
        for (int i = 0; i < 4; i++) y[i] = __fadd_rn(__fmul_rn(g[i], __fmul_rn(__fsub_rn(v[t][i], ms[t]), rstd)), bb[i]);
        __nv_bfloat162 y01 = __floats2bfloat162_rn(y[0], y[1]), y23 = __floats2bfloat162_rn(y[2], y[3]);
        uint2 yw = make_uint2(*reinterpret_cast<uint32_t*>(&y01), *reinterpret_cast<uint32_t*>(&y23));
        if (!live[t]) yw = make_uint2(0u, 0u);
        // columns 4 lane .. of tile row r in the 128-byte swizzled K-major A tile
        const uint32_t off = sw128_offset(r, lane >> 1) + (uint32_t)(lane & 1) * 8u;
#pragma unroll
        for (uint32_t dst = 0; dst < kRowsCluster; dst++)
            *reinterpret_cast<uint2*>(__cluster_map_shared_rank(smem + kCfX + off, dst)) = yw;
    }
    // the A tiles are read by the tensor core (async proxy) after the next cluster barrier
    asm volatile("fence.proxy.async.shared::cluster;" ::: "memory");
}

// The input layer of this thread's two rows (h = bf16(b + sum_k obs[k] W[k][:])
// in k_input_forward's order), from the observations and weights staged in
// shared memory.
template <int IN>
__device__ __forceinline__ void cf_input_layer(const uint8_t* smem, const float4 bias, float (&h)[2][4]) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int c0 = lane * 4;
    const __nv_bfloat16* sW = reinterpret_cast<const __nv_bfloat16*>(smem + kCfIn);
    const float* sObs = reinterpret_cast<const float*>(smem + kCfObs);
#pragma unroll
    for (int t = 0; t < 2; t++) {
        const float* ob = sObs + (warp + 16 * t) * IN;
        float acc[4] = {bias.x, bias.y, bias.z, bias.w};
#pragma unroll
        for (int k = 0; k < IN; k++) {
            const float o = ob[k];
            const float4 wk = bf4_load(sW + k * kCfE + c0);
            acc[0] = __fadd_rn(acc[0], __fmul_rn(o, wk.x));
            acc[1] = __fadd_rn(acc[1], __fmul_rn(o, wk.y));
            acc[2] = __fadd_rn(acc[2], __fmul_rn(o, wk.z));
            acc[3] = __fadd_rn(acc[3], __fmul_rn(o, wk.w));
        }
#pragma unroll
        for (int i = 0; i < 4; i++) h[t][i] = round_bf16(acc[i]);
    }
}

// The residual add of the down projection for this thread's two rows: the
// cluster's four partial tiles summed in CTA order, h = bf16(h + bf16(sum))
// (rows_cluster_epilogue<kRowsResidLN>'s arithmetic).
__device__ __forceinline__ void cf_residual(const uint8_t* smem, uint32_t q, float (&h)[2][4]) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
#pragma unroll
    for (int t = 0; t < 2; t++) {
        const int tr = 32 * (int)q + warp + 16 * t;
        const uint8_t* cell = smem + kCfP + tile_offset(tr, lane);
        float4 a = *reinterpret_cast<const float4*>(__cluster_map_shared_rank(cell, 0));
#pragma unroll
        for (uint32_t r = 1; r < kRowsCluster; r++) {
            const float4 b = *reinterpret_cast<const float4*>(__cluster_map_shared_rank(cell, r));
            a = make_float4(__fadd_rn(a.x, b.x), __fadd_rn(a.y, b.y), __fadd_rn(a.z, b.z), __fadd_rn(a.w, b.w));
        }
        h[t][0] = round_bf16(h[t][0] + round_bf16(a.x));
        h[t][1] = round_bf16(h[t][1] + round_bf16(a.y));
        h[t][2] = round_bf16(h[t][2] + round_bf16(a.z));
        h[t][3] = round_bf16(h[t][3] + round_bf16(a.w));
    }
}

// W_up[:, 128q ..] (K rows 64 kb .., N boxes 128q + 64 j) and W_down[128q .., :]
// (K rows 128q + 64 kb .., N boxes 64 j) of one block, as block_cluster.cu's
// forward loads them.
__device__ __forceinline__ void cf_load_up(uint8_t* smem, const CUtensorMap* map, int h0, uint64_t* bar) {
    mbar_arrive_expect_tx(bar, kCfTile);
    for (int kb = 0; kb < 2; kb++)
        for (int j = 0; j < 2; j++) tma_load_2d(smem + kCfWU + kb * 16384 + j * 8192, map, h0 + 64 * j, 64 * kb, bar);
}
__device__ __forceinline__ void cf_load_down(uint8_t* smem, const CUtensorMap* map, int h0, uint64_t* bar) {
    mbar_arrive_expect_tx(bar, kCfTile);
    for (int kb = 0; kb < 2; kb++)
        for (int j = 0; j < 2; j++) tma_load_2d(smem + kCfWD + kb * 16384 + j * 8192, map, 64 * j, h0 + 64 * kb, bar);
}

template <class Env>
__global__ void __launch_bounds__(kRowsThreads, 1) k_collect_fused(const __grid_constant__ CfMaps tm, const CfParams p) {
    using State = typename Env::State;
    using Action = typename Env::Action;
    using Obs = typename Env::Obs;
    constexpr int IN = (int)Env::OBS_DIM;
    constexpr int A = (int)Env::ACT_DIM;
    static_assert(IN <= kCollectFusedMaxInputDim, "");
    static_assert(!EnvTraits<Env>::kInPlace, "the fused collect keeps the State in registers");

    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kCfBar);
    uint64_t* fullU = bars;
    uint64_t* fullD = bars + 1;
    uint64_t* fullH = bars + 2;
    uint64_t* mma1 = bars + 3;
    uint64_t* mma2 = bars + 4;
    uint64_t* mmaH = bars + 5;
    uint64_t* fin = bars + 6;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 7);
    volatile int* sOk = reinterpret_cast<volatile int*>(bars + 8);
    __nv_bfloat16* hs = reinterpret_cast<__nv_bfloat16*>(smem + kCfHS);
    float* sObs = reinterpret_cast<float*>(smem + kCfObs);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t q = cluster_ctarank();
    const int m0 = (int)(blockIdx.x / kRowsCluster) * kRowsBM;
    const int h0 = (int)q * kRowsBN;
    const int R = p.R, T = p.T, L = p.L;
    const int nUses = (T + 1) * L;  // block-weight uses of the whole rollout

    if (threadIdx.x == 0) {
        for (int i = 0; i < 7; i++) mbar_init(&bars[i], 1);
        *sOk = 1;
        fence_barrier_init();
        for (int l = 0; l < L; l++) {
            prefetch_tensormap(&tm.up[l]);
            prefetch_tensormap(&tm.down[l]);
        }
        prefetch_tensormap(&tm.head);
    }
    if (warp == 2) {
        tmem_alloc(tmem_slot, kCfTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    cluster_arrive_relaxed();  // this CTA has started (waited on before any peer's tile is written)
    mg_pdl_wait();

    // producer state (thread 0): parities of the outstanding up / down loads
    uint32_t prodU = 0, prodD = 0;
    if (threadIdx.x == 0) {
        cf_load_up(smem, &tm.up[0], h0, fullU);
        cf_load_down(smem, &tm.down[0], h0, fullD);
        mbar_arrive_expect_tx(fullH, kCfE * kCfHeadCols * 2);
        tma_load_2d(smem + kCfWH, &tm.head, 0, 0, fullH);
    }
    // input weights and the observations of step 0 (this CTA's 32 rows)
    {
        const uint4* src = reinterpret_cast<const uint4*>(p.wIn);
        uint4* dst = reinterpret_cast<uint4*>(smem + kCfIn);
        for (int i = threadIdx.x; i < IN * kCfE / 8; i += blockDim.x) dst[i] = src[i];
        for (int i = threadIdx.x; i < 32 * IN; i += blockDim.x) {
            const int row = m0 + 32 * (int)q + i / IN;
            sObs[i] = row < R ? p.obsSlots[(size_t)row * IN + i % IN] : 0.0f;
        }
    }
    // warp q: this CTA's 32 environments, one per lane, in registers
    const int envRow = m0 + 32 * (int)q + lane;
    const bool envWarp = warp == (int)q;
    const bool envLive = envWarp && envRow < R;
    State s{};
    uint32_t w = 0;
    uint8_t d = 0;
    if (envLive) {
        s = static_cast<const State*>(p.states)[envRow];
        w = p.rng[envRow];
        d = p.done[envRow];
    }
    const float4 bias = bf4_load(p.bIn + lane * 4);
    bool live[2];
#pragma unroll
    for (int t = 0; t < 2; t++) live[t] = m0 + 32 * (int)q + warp + 16 * t < R;
    __syncthreads();  // staged weights and observations
    cluster_wait();   // every CTA of the cluster has started

    float h[2][4];
    uint32_t pU = 0, pD = 0, p1 = 0, p2 = 0, pH = 0;
    bool headReady = false;
    float bootValue = 0.0f;
    int use = 0;
    for (int t = 0; t <= T; t++) {
        // ---- input layer and LayerNorm 0 into every CTA's A tile
        cf_input_layer<IN>(smem, bias, h);
        cf_layernorm_to_tiles(smem, q, h, live, p.lnG[0], p.lnB[0]);
        tc_fence_before();
        cluster_sync();
        tc_fence_after();
        for (int l = 0; l < L; l++, use++) {
            const int next = use + 1 < nUses ? (use + 1) % L : -1;  // block of the next weight use
            // ---- V_q = relu(bf16(X W_up[:, h0 ..]))
            if (warp == 1 && lane == 0) {
                if (*sOk && mbar_wait(fullU, pU, p.status, kDevTimeoutFull)) {
                    tc_fence_after();
                    bc_mma<true>(tmem, smem_u32(smem + kCfX), smem_u32(smem + kCfWU));
                } else {
                    *sOk = 0;
                }
                tc_commit(mma1);  // always: covers whatever was issued
            }
            pU ^= 1;
            __syncwarp();
            const bool ok1 = cf_wait_warp(mma1, p1, sOk, p.status, kDevTimeoutDone);
            p1 ^= 1;
            tc_fence_after();
            if (threadIdx.x == 0 && next >= 0 && ok1) {
                // the up slice has been consumed: load the next block's (its
                // previous load has completed: the product above read it)
                if (mbar_wait(fullU, prodU, p.status, kDevTimeoutFull)) {
                    prodU ^= 1;
                    cf_load_up(smem, &tm.up[next], h0, fullU);
                } else {
                    *sOk = 0;
                }
            }
            __syncwarp();
            bc_hidden_tile<false>(smem, kCfV, 0, tmem, ok1);
            fence_async_smem();  // generic writes of V -> visible to the tensor core
            tc_fence_before();
            __syncthreads();
            tc_fence_after();
            // ---- P_q = V_q W_down[h0 .., :]
            if (warp == 1 && lane == 0) {
                if (*sOk && mbar_wait(fullD, pD, p.status, kDevTimeoutFull)) {
                    tc_fence_after();
                    bc_mma<true>(tmem + 128, smem_u32(smem + kCfV), smem_u32(smem + kCfWD));
                } else {
                    *sOk = 0;
                }
                tc_commit(mma2);
            }
            pD ^= 1;
            __syncwarp();
            const bool ok2 = cf_wait_warp(mma2, p2, sOk, p.status, kDevTimeoutDone);
            p2 ^= 1;
            tc_fence_after();
            if (threadIdx.x == 0 && next >= 0 && ok2) {
                if (mbar_wait(fullD, prodD, p.status, kDevTimeoutFull)) {
                    prodD ^= 1;
                    cf_load_down(smem, &tm.down[next], h0, fullD);
                } else {
                    *sOk = 0;
                }
            }
            __syncwarp();
            rows_tmem_to_tile(smem + kCfP, tmem + 128, ok1 && ok2);
            tc_fence_before();
            cluster_sync();  // every CTA's partial tile is complete
            tc_fence_after();
            // ---- h += sum of the partials; the next LayerNorm (block l + 1's,
            // or the final one) into every CTA's A tile
            cf_residual(smem, q, h);
            cf_layernorm_to_tiles(smem, q, h, live, p.lnG[l + 1], p.lnB[l + 1]);
            tc_fence_before();
            cluster_sync();  // the A tiles are complete; no CTA still reads a partial tile
            tc_fence_after();
        }
        // ---- logits | value = bf16(X W_head) (head_tail.cu's product)
        if (warp == 1 && lane == 0) {
            bool ok = *sOk != 0;
            if (ok && !headReady) {
                ok = mbar_wait(fullH, 0, p.status, kDevTimeoutFull);
                headReady = ok;
            }
            if (ok) {
                tc_fence_after();
                constexpr uint32_t idesc = idesc_bf16_f32(kCfHeadCols, false, true);
                const uint32_t a = smem_u32(smem + kCfX), b = smem_u32(smem + kCfWH);
#pragma unroll
                for (int k = 0; k < 8; k++)
                    tc_mma_bf16(tmem + 256, smem_desc_sw128(a + (k >> 2) * 16384 + (k & 3) * 32, 16, 1024),
                                smem_desc_sw128(b + k * 2048, 8192, 1024), idesc, k > 0 ? 1u : 0u);
            } else {
                *sOk = 0;
            }
            tc_commit(mmaH);
        }
        __syncwarp();
        if (envWarp) {
            const bool okh = cf_wait_warp(mmaH, pH, sOk, p.status, kDevTimeoutDone);
            tc_fence_after();
            float v[kCfHeadCols];
            if (okh) {
                tmem_ld32(tmem + 256 + ((uint32_t)(q * 32) << 16), v);
                tmem_ld32(tmem + 256 + ((uint32_t)(q * 32) << 16) + 32, v + 32);
            } else {
#pragma unroll
                for (int i = 0; i < kCfHeadCols; i++) v[i] = 0.0f;
            }
            __nv_bfloat16* hrow = hs + lane * kCfHStride;
            uint32_t hw[kCfHeadCols / 2];
#pragma unroll
            for (int i = 0; i < kCfHeadCols / 2; i++) {
                __nv_bfloat162 h2 = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
                hw[i] = *reinterpret_cast<uint32_t*>(&h2);
                reinterpret_cast<uint32_t*>(hrow)[i] = hw[i];
            }
            if (t == T) {
                // the bootstrap forward: its head rows (the GEMM's bf16 output) and value
                if (envLive) {
                    uint4* dst = reinterpret_cast<uint4*>(p.bootHead + (size_t)envRow * kCfHeadCols);
#pragma unroll
                    for (int i = 0; i < kCfHeadCols / 8; i++)
                        dst[i] = make_uint4(hw[4 * i], hw[4 * i + 1], hw[4 * i + 2], hw[4 * i + 3]);
                }
                bootValue = __bfloat162float(hrow[A]);
            } else if (envLive) {
                // sample from the head row, then reset-if-done and step (env_collect_step_kernel)
                const size_t k = (size_t)t * R + envRow;
                float lp, val;
                const Action act = draw_policy_action<Env>(hrow, p.logStd, w, lp, val);
                static_cast<Action*>(p.actionSlots)[k] = act;
                p.logpSlots[k] = lp;
                p.valueSlots[k] = val;
                Obs o;
                float r;
                if (d) Env::reset(s, w);
                Env::step(s, act, o, r, d);
                reinterpret_cast<Obs*>(p.obsSlots)[(size_t)(t + 1) * R + envRow] = o;
                p.rewardSlots[k] = r;
                p.doneSlots[k] = d;
                const float* of = reinterpret_cast<const float*>(&o);
#pragma unroll
                for (int i = 0; i < IN; i++) sObs[lane * IN + i] = of[i];
            }
        }
        pH ^= 1;
        __syncwarp();  // the env lanes diverged (padding rows, the sampler's early exit): reconverge
        tc_fence_before();
        cluster_sync();  // every CTA's head product has read its A tile; the observations are staged
        tc_fence_after();
    }

    // ---- GAE over each environment's column (model/gae.metal:14-36, k_gae's
    // arithmetic), then the environment state back to the gym's buffers
    if (envLive) {
        float lastAdv = 0.0f;
        float nextValue = bootValue;
        const float gl = __fmul_rn(p.gamma, p.lambda);
        // slots in chunks of 8, newest first, each chunk's loads issued
        // together before its part of the (unchanged) serial recurrence
        constexpr int kChunk = 8;
        for (int t = T - 1; t >= 0; t -= kChunk) {
            float rw[kChunk], vl[kChunk];
            uint8_t dn[kChunk];
#pragma unroll
            for (int j = 0; j < kChunk; j++) {
                if (t - j < 0) break;
                const size_t k = (size_t)(t - j) * R + envRow;
                rw[j] = p.rewardSlots[k];
                vl[j] = p.valueSlots[k];
                dn[j] = p.doneSlots[k];
            }
#pragma unroll
            for (int j = 0; j < kChunk; j++) {
                if (t - j < 0) break;
                const size_t k = (size_t)(t - j) * R + envRow;
                const float nonTerminal = dn[j] ? 0.0f : 1.0f;
                const float val = vl[j];
                const float delta =
                    __fsub_rn(__fadd_rn(rw[j], __fmul_rn(__fmul_rn(p.gamma, nextValue), nonTerminal)), val);
                lastAdv = __fadd_rn(delta, __fmul_rn(__fmul_rn(gl, nonTerminal), lastAdv));
                p.advSlots[k] = lastAdv;
                p.retSlots[k] = __fadd_rn(lastAdv, val);
                nextValue = val;
            }
        }
        static_cast<State*>(p.states)[envRow] = s;
        p.rng[envRow] = w;
        p.done[envRow] = d;
    }

    // ---- teardown: every product and copy of this CTA has completed before TMEM is freed
    if (warp == 1 && lane == 0) {
        tc_commit(fin);
        mbar_wait(fin, 0, p.status, kDevTimeoutDone);
    }
    if (threadIdx.x == 0) {
        // the last up / down loads (normally observed by the products already)
        mbar_wait(fullU, prodU, p.status, kDevTimeoutFull);
        mbar_wait(fullD, prodD, p.status, kDevTimeoutFull);
        mbar_wait(fullH, 0, p.status, kDevTimeoutFull);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 2) {
        __syncwarp();  // warp 2 may have been an env warp (per-lane GAE loops)
        tc_fence_after();
        tmem_dealloc(tmem, kCfTmemCols);
    }
}

// Launches the kernel for Env with the tensor maps and parameters the library
// prepared (maps: CfMaps, params: CfParams). The mg_env_ops entry
// collect_fused of environments that keep their State in registers.
template <class Env>
int collect_fused_launch(const void* maps, const void* params, mg_stream_t stream) {
    if (!maps || !params) return MG_ERR_ARGUMENT;
    const CfMaps& tm = *static_cast<const CfMaps*>(maps);
    const CfParams& p = *static_cast<const CfParams*>(params);
    if (p.R <= 0 || p.T <= 0 || p.L < 1 || p.L > kCollectFusedMaxBlocks) return MG_ERR_ARGUMENT;
    auto kern = k_collect_fused<Env>;
    // a per-device attribute: set on every launch (cheap, and safe from any thread)
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kCfSmem) != cudaSuccess)
        return MG_ERR_CUDA;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(((p.R + kRowsBM - 1) / kRowsBM) * kRowsCluster));
    cfg.blockDim = dim3(kRowsThreads);
    cfg.dynamicSmemBytes = kCfSmem;
    cfg.stream = reinterpret_cast<cudaStream_t>(stream);
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = kRowsCluster;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaLaunchKernelEx(&cfg, kern, tm, p) != cudaSuccess) return MG_ERR_CUDA;
    return cudaGetLastError() == cudaSuccess ? MG_OK : MG_ERR_CUDA;
}

// Whether Env can run in the fused kernel: its State fits in registers and
// its observation in the input layer's staging.
template <class Env>
constexpr bool collect_fused_eligible() {
    return !EnvTraits<Env>::kInPlace && Env::OBS_DIM <= (uint32_t)kCollectFusedMaxInputDim;
}

}  // namespace mg
