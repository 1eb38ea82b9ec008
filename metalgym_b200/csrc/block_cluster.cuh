// One residual block of the CartPole-sized policy (embed 128, hidden 512) over
// a 128-row tile on a cluster of 4 CTAs, forward and backward, as a pass
// (tile_pass.cuh): run once by the block kernels of block_cluster.cu and back
// to back with the other layers' passes by the minibatch kernel
// (minibatch_tiles.cu).
//
// forward (model/mlp.metal:18-86, model/elementwise.metal:4-13, then the
// LayerNorm that follows, model/layernorm.metal:10-71):
//   CTA q   V_q = relu(bf16(lnOut W_up[:, 128q : 128q + 128]))   (tcgen05, K = 128)
//           V_q -> global V (kept for the backward) and, swizzled, into
//           shared memory as the A operand of
//           P_q = V_q W_down[128q : 128q + 128, :]                (tcgen05, K = 128)
//   cluster h = bf16(h + bf16(P_0 + P_1 + P_2 + P_3)), then the next
//           LayerNorm (rows_epilogue.cuh; CTA q ends rows 32q .. 32q + 31)
//
// backward (model/mlp.metal:88-153, model/layernorm.metal:74-127,
// model/ppo.h:851-852):
//   CTA q   dV_q = bf16(dS W_down[128q : 128q + 128, :]^T) * (V_q > 0)
//           dV_q -> global dV and into shared memory
//           Q_q = dV_q W_up[:, 128q : 128q + 128]^T
//           the tile's weight-gradient partials (model/mlp.metal:155-208):
//           dW_up[:, 128q..] += lnOut^T dV_q, dW_down[128q.., :] += V_q^T dS
//           (sums over the tile's 128 rows, one fp32 partial per row tile;
//           the gradient finalisation adds the tiles in order)
//   cluster dz = bf16(Q_0 + .. + Q_3), LayerNorm backward of dz plus the skip
//           gradient, dgamma / dbeta partials
//
// Every product is the one the separate kernels compute (the same K order per
// output element; the down / branch products split K as the row kernels of
// gemm_rows.cu do), so the outputs are bit-identical to the up or dV GEMM
// followed by the row kernel. Every wait is bounded; every cluster barrier is
// reached by every thread on every path.
#pragma once

#include "block.h"
#include "gemm.h"
#include "gemm_tc.cuh"
#include "policy.h"
#include "rows_epilogue.cuh"
#include "tile_pass.cuh"

namespace mg {

constexpr int kBcHidden = kRowsBN * (int)kRowsCluster;  // 512: CTA q owns hidden columns 128q ..
constexpr int kBcTile = 128 * 128 * 2;                  // one bf16 operand tile, 32 KB (two 64-wide K blocks)
// shared memory (offsets from the 1024-aligned base)
//   forward:  A1 lnOut | B1 W_up slice | B2 W_down slice | A2 V_q      | barriers
//   backward: A1 dS    | B1 W_down sl. | B2 W_up slice   | M  V_q      | A2 dV_q | LN lnOut | barriers
// after the second product the fp32 tile (64 KB) reuses A1 + B1, and the
// LayerNorm-backward column sums (32 KB) reuse M
constexpr int kBcA1 = 0, kBcB1 = kBcTile, kBcB2 = 2 * kBcTile;
constexpr int kBcFwdA2 = 3 * kBcTile, kBcFwdBar = 4 * kBcTile;
constexpr int kBcBwdM = 3 * kBcTile, kBcBwdA2 = 4 * kBcTile, kBcBwdLn = 5 * kBcTile, kBcBwdBar = 6 * kBcTile;
static_assert(kRowsTile <= 2 * kBcTile && kRowsRedBytes <= kBcTile && kBcBwdM == kBcB2 + kBcTile, "");
static_assert((32 * kRowsBN + 32 * kRowsInputMaxDim) * 4 <= kBcTile, "the input-gradient staging fits the lnOut tile");
static_assert(kBlockClusterMaxInputDim == kRowsInputMaxDim, "");
static_assert((kRowsInputMaxDim * kRowsBN + 32 * kRowsInputMaxDim) * 4 <= kBcTile, "the input staging fits A2");
constexpr int kBcFwdSmem = kBcFwdBar + 256 + 1024;
constexpr int kBcBwdSmem = kBcBwdBar + 256 + 1024;

// The input layer and the first LayerNorm computed in the first block's
// forward kernel (model/input.metal:11-27, model/layernorm.metal:10-71): h =
// bf16(b + sum_k obs[k] W[k][:]) in k_input_forward's order, then its LayerNorm
// (ln: x-hat, out, sigma), whose output is the block's A operand.
struct BcInput {
    const float* obs;       // [*][inDim] fp32
    const MgMinibatch* mb;  // row map (null: row r reads observation r)
    uint64_t envRows, total;
    int inDim;              // <= kRowsInputMaxDim
    const __nv_bfloat16* w;  // [inDim][128]
    const __nv_bfloat16* b;  // [128]
    __nv_bfloat16* h;        // [M][128]
    LnOutputs ln;
    // the observation rows may be staged before the kernel's PDL wait: they
    // come through a training minibatch's schedule from rollout slots that
    // collect() filled before the train work began (never the output of the
    // preceding kernel, as the env step's is for a collect-step forward)
    bool earlyObs;
};

struct BcParams {
    int M;
    BcInput in;
    __nv_bfloat16* vOut;  // forward: V [M][512]; backward: dV [M][512]
    float* upPart;        // backward: [tile][128][512] partial sums of dW_up over each 128-row tile
    float* downPart;      // backward: [tile][512][128] partial sums of dW_down
    RowsEpi e;
    int* status;
    uint64_t* trace;  // phase trace (tile_pass.cuh); null: off
    // standalone kernel: issue the loads of everything but the A operand
    // before the programmatic-dependency wait. Only where the preceding
    // kernel is a tile kernel that signals its dependents after its own wait
    // (block_cluster.cu, head_tail.cu): this kernel's pre-wait code then runs
    // after every kernel before that one completed, and the weights, the
    // ReLU mask and the LayerNorm output all come from those.
    bool prefetch;
};

// Maps (all SW128, 64-wide boxes):
//   forward:  a = lnOut [M][128] (box 64 x 128 rows), b1 = W_up [128][512]
//             (MN-major, box 64 x 64), b2 = W_down [512][128] (MN-major,
//             box 64 x 64), v = V [M][512] (box 64 x 128, TMA store)
//   backward: a = dS [M][128], b1 = W_down [512][128] as [N][K] (box 64 x 128
//             rows), b2 = W_up [128][512] as [N][K] (box 64 x 128 rows),
//             v = V [M][512] (load: the mask), dv = dV [M][512] (store)
struct BcMaps {
    CUtensorMap a, b1, b2, v, dv, ln;
};

// A 128 x 128 product over the tile's 128 rows (K) with both operands
// MN-major: A^T B for A [K][M] and B [K][N] tiles as TMA writes them (two
// 64-wide column blocks of 128 rows, 16 KB apart).
__device__ __forceinline__ void bc_mma_tn(uint32_t d, uint32_t aBase, uint32_t bBase) {
    constexpr uint32_t idesc = idesc_bf16_f32(128, true, true);
#pragma unroll
    for (int kk = 0; kk < 8; kk++) {
        const uint64_t ad = smem_desc_sw128(aBase + kk * 2048, 16384, 1024);
        const uint64_t bd = smem_desc_sw128(bBase + kk * 2048, 16384, 1024);
        tc_mma_bf16(d, ad, bd, idesc, kk > 0 ? 1u : 0u);
    }
}

// A 128 x 128 fp32 accumulator to global rows of `ld` floats through the
// swizzled staging tile `stage` (64 KB of free shared memory): TMEM -> stage
// (rows_tmem_to_tile), then each warp writes whole 512-byte rows, lane l the
// 16 bytes of columns 4l..4l+3. Every thread of the CTA takes part.
__device__ __forceinline__ void bc_tmem_to_global(uint8_t* stage, float* dst, int ld, uint32_t acc, bool valid) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    rows_tmem_to_tile(stage, acc, valid);
    __syncthreads();
#pragma unroll
    for (int i = 0; i < 8; i++) {
        const int r = warp + 16 * i;
        *reinterpret_cast<float4*>(dst + (size_t)r * ld + lane * 4) =
            *reinterpret_cast<const float4*>(stage + tile_offset(r, lane));
    }
    __syncthreads();  // the stage may be reused
}

// The input layer and the first LayerNorm of this CTA's 32 rows (two per
// warp, lane l: columns 4l..4l+3), their LayerNorm output written into the A
// tile of every CTA of the cluster. `stage`: free shared memory for the input
// weights (fp32) and the rows' observations.
// The observation rows of this CTA's 32 rows into the staging area after the
// input weights (stage + inDim x 128 floats), read through the row map.
__device__ __forceinline__ void bc_input_stage_obs(float* stage, uint32_t q, int m0, int M, const BcInput& in) {
    float* sObs = stage + in.inDim * kRowsBN;  // [32][inDim]
    for (int i = threadIdx.x; i < 32 * in.inDim; i += blockDim.x) {
        const int row = m0 + 32 * (int)q + i / in.inDim;
        float o = 0.0f;
        if (row < M) {
            const uint64_t g = in.mb ? mg_minibatch_row(*in.mb, row, in.envRows, in.total) : (uint64_t)row;
            o = in.obs[g * in.inDim + i % in.inDim];
        }
        sObs[i] = o;
    }
}

__device__ __forceinline__ void bc_input_prologue(uint8_t* smem, float* stage, uint32_t q, int m0, int M,
                                                  const BcInput& in) {
    constexpr int E = kRowsBN;
    constexpr float kInvE = 1.0f / E;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int c0 = lane * 4;
    float* sW = stage;                    // [inDim][128]
    float* sObs = stage + in.inDim * E;   // [32][inDim]
    // the bias and LayerNorm parameters in flight with the weights' loads
    const float4 bias = bf4_load(in.b + c0);
    const float4 gm = bf4_load(in.ln.gamma + c0), bt = bf4_load(in.ln.beta + c0);
    for (int i = threadIdx.x; i < in.inDim * E; i += blockDim.x) sW[i] = __bfloat162float(in.w[i]);
    if (!in.earlyObs) bc_input_stage_obs(stage, q, m0, M, in);  // else staged before the PDL wait
    __syncthreads();
    const float g[4] = {gm.x, gm.y, gm.z, gm.w}, bb[4] = {bt.x, bt.y, bt.z, bt.w};
    float v[2][4], ms[4];
#pragma unroll
    for (int t = 0; t < 2; t++) {
        const int tl = warp + 16 * t;
        const float* ob = sObs + tl * in.inDim;
        float acc[4] = {bias.x, bias.y, bias.z, bias.w};
        for (int k = 0; k < in.inDim; k++) {
            const float o = ob[k];
            const float4 wk = *reinterpret_cast<const float4*>(sW + k * E + c0);
            acc[0] = __fadd_rn(acc[0], __fmul_rn(o, wk.x));
            acc[1] = __fadd_rn(acc[1], __fmul_rn(o, wk.y));
            acc[2] = __fadd_rn(acc[2], __fmul_rn(o, wk.z));
            acc[3] = __fadd_rn(acc[3], __fmul_rn(o, wk.w));
        }
        float sm = 0.0f;
#pragma unroll
        for (int i = 0; i < 4; i++) {
            v[t][i] = round_bf16(acc[i]);
            sm = __fadd_rn(sm, v[t][i]);
        }
        ms[t] = sm;
        const int row = m0 + 32 * (int)q + tl;
        if (row < M) bf4_store(in.h + (size_t)row * E + c0, v[t][0], v[t][1], v[t][2], v[t][3]);
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
        const int tl = warp + 16 * t;
        const int r = 32 * (int)q + tl;  // row of the tile
        const int row = m0 + r;
        const float sd = __fsqrt_rn(__fadd_rn(__fmul_rn(ms[2 + t], kInvE), 1e-5f));
        const float rstd = __frcp_rn(sd);
        float xn[4], y[4];
#pragma unroll
        for (int i = 0; i < 4; i++) {
            xn[i] = __fmul_rn(__fsub_rn(v[t][i], ms[t]), rstd);
            y[i] = __fadd_rn(__fmul_rn(g[i], xn[i]), bb[i]);
        }
        __nv_bfloat162 y01 = __floats2bfloat162_rn(y[0], y[1]), y23 = __floats2bfloat162_rn(y[2], y[3]);
        uint2 yw = make_uint2(*reinterpret_cast<uint32_t*>(&y01), *reinterpret_cast<uint32_t*>(&y23));
        if (row < M) {
            if (lane == 0) in.ln.stdev[row] = sd;
            bf4_store(in.ln.xNorm + (size_t)row * E + c0, xn[0], xn[1], xn[2], xn[3]);
            *reinterpret_cast<uint2*>(in.ln.out + (size_t)row * E + c0) = yw;
        } else {
            yw = make_uint2(0u, 0u);
        }
        if (t == 0) cluster_wait();  // every CTA of the cluster has started
        // columns 4 lane .. of tile row r in the 128-byte swizzled K-major A tile
        const uint32_t off = sw128_offset(r, lane >> 1) + (uint32_t)(lane & 1) * 8u;
#pragma unroll
        for (uint32_t dst = 0; dst < kRowsCluster; dst++)
            *reinterpret_cast<uint2*>(__cluster_map_shared_rank(smem + kBcA1 + off, dst)) = yw;
    }
    // the A tiles are read by the tensor core (async proxy) after the cluster barrier
    asm volatile("fence.proxy.async.shared::cluster;" ::: "memory");
}


// The maps and parameters of one block pass (block_cluster.cu), checked on
// the host: the forward of block_cluster_forward and the backward of
// block_cluster_backward (block.h), without a launch.
int block_cluster_forward_args(const void* lnOut, const void* wUp, const void* wDown, void* h, void* v,
                               const LnOutputs& next, int M, const BlockClusterForwardInput* in, BcMaps& tm,
                               BcParams& p);
int block_cluster_backward_args(const void* dS, const void* wDown, const void* v, const void* wUp, void* dV,
                                const void* lnOut, float* upPart, float* downPart, const void* xNorm,
                                const void* gamma, const float* stdev, const void* resid, void* residOut,
                                float* partial, int M, const BlockClusterInput* in, BcMaps& tm, BcParams& p);

// Prefetch of the pass's tensor maps (thread 0).
__device__ __forceinline__ void bc_prefetch_maps(const BcMaps& tm, bool bwd) {
    prefetch_tensormap(&tm.a);
    prefetch_tensormap(&tm.b1);
    prefetch_tensormap(&tm.b2);
    prefetch_tensormap(&tm.v);
    if (bwd) {
        prefetch_tensormap(&tm.dv);
        prefetch_tensormap(&tm.ln);
    }
}

// Thread 0: the pass's loads other than the A operand (the weight slices;
// backward: the ReLU mask and the LayerNorm output), with the byte counts of
// both full barriers, the A operand's included (its loads follow, before or
// after the programmatic-dependency wait).
template <bool BWD, bool INPUT>
__device__ __forceinline__ void bc_issue_static(uint8_t* smem, const BcMaps& tm, TilePass& t) {
    const int m0 = (int)(blockIdx.x / kRowsCluster) * kRowsBM;
    const int h0 = (int)cluster_ctarank() * kRowsBN;
    t.issuing(kTbFull1);
    mbar_arrive_expect_tx(t.bar(kTbFull1), (INPUT ? 1 : 2) * kBcTile + (BWD ? kBcTile : 0));
    if (!BWD) {
        // W_up[k][h0 + n]: K rows 64 kb.., N boxes h0 + 64 j
        for (int kb = 0; kb < 2; kb++)
            for (int j = 0; j < 2; j++)
                tma_load_2d(smem + kBcB1 + kb * 16384 + j * 8192, &tm.b1, h0 + 64 * j, 64 * kb, t.bar(kTbFull1));
    } else {
        // W_down rows h0 .. h0 + 127 as [N][K = 128]; the mask V[m0.., h0..]
        for (int kb = 0; kb < 2; kb++) tma_load_2d(smem + kBcB1 + kb * 16384, &tm.b1, 64 * kb, h0, t.bar(kTbFull1));
        for (int kb = 0; kb < 2; kb++) tma_load_2d(smem + kBcBwdM + kb * 16384, &tm.v, h0 + 64 * kb, m0, t.bar(kTbFull1));
    }
    t.issuing(kTbFull2);
    mbar_arrive_expect_tx(t.bar(kTbFull2), kBcTile * (BWD ? 2 : 1));
    if (BWD)  // the block's LayerNorm output, for dW_up
        for (int kb = 0; kb < 2; kb++) tma_load_2d(smem + kBcBwdLn + kb * 16384, &tm.ln, 64 * kb, m0, t.bar(kTbFull2));
    if (!BWD) {
        // W_down[h0 + k][n]: K rows h0 + 64 kb.., N boxes 64 j
        for (int kb = 0; kb < 2; kb++)
            for (int j = 0; j < 2; j++)
                tma_load_2d(smem + kBcB2 + kb * 16384 + j * 8192, &tm.b2, 64 * j, h0 + 64 * kb, t.bar(kTbFull2));
    } else {
        // W_up as [N = 128][K = 512], K columns h0 + 64 kb ..
        for (int kb = 0; kb < 2; kb++) tma_load_2d(smem + kBcB2 + kb * 16384, &tm.b2, h0 + 64 * kb, 0, t.bar(kTbFull2));
    }
}

// One block pass over the tile m0 = 128 (blockIdx.x / 4) of this CTA's
// cluster. On entry: the barriers and TMEM of `t` are set up, every CTA of
// the cluster is running (or, with INPUT, has arrived on the cluster barrier
// after its setup) and the pass's inputs are visible. Standalone (!t.merged):
// frees the pass's TMEM (BWD ? 512 : 256 columns) before the epilogue, as
// the kernel's last use of it. Merged: leaves TMEM allocated and ends at a
// pass boundary.
// staticIssued: bc_issue_static already ran (before the kernel's wait).
template <bool BWD, int RPC, bool INPUT>
__device__ __forceinline__ void bc_pass(uint8_t* smem, const BcMaps& tm, const BcParams& p, TilePass& t,
                                        bool staticIssued = false) {
    constexpr int A2 = BWD ? kBcBwdA2 : kBcFwdA2;
    constexpr uint32_t kTmemCols = BWD ? 512 : 256;
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t q = cluster_ctarank();
    const int m0 = (int)(blockIdx.x / kRowsCluster) * kRowsBM;
    const int h0 = (int)q * kRowsBN;  // this CTA's hidden columns
    const uint32_t tmem = t.tmem;
    t.trace = p.trace;
    tp_mark(t);  // pass start

    if (threadIdx.x == 0 && t.ok()) {
        if (!staticIssued) bc_issue_static<BWD, INPUT>(smem, tm, t);
        if (!INPUT)
            for (int kb = 0; kb < 2; kb++) tma_load_2d(smem + kBcA1 + kb * 16384, &tm.a, 64 * kb, m0, t.bar(kTbFull1));
    }
    if (INPUT) {
        // the A tile is computed here: the input layer and the first LayerNorm
        bc_input_prologue(smem, reinterpret_cast<float*>(smem + A2), q, m0, p.M, p.in);
        cluster_sync();  // every CTA's rows are in every CTA's A tile
        tc_fence_after();
    }
    if (warp == 1 && lane == 0) {
        if (tp_wait(t, kTbFull1, p.status, kDevTimeoutFull)) {
            tc_fence_after();
            bc_mma<!BWD>(tmem, smem_u32(smem + kBcA1), smem_u32(smem + kBcB1));
            tc_commit(t.bar(kTbMma1));
            // dW_down partial = V_q^T dS (TMEM columns 384..511), covered by mma2's commit
            if (BWD) bc_mma_tn(tmem + 384, smem_u32(smem + kBcBwdM), smem_u32(smem + kBcA1));
        } else {
            tc_commit(t.bar(kTbMma1));  // always: covers whatever was issued
        }
    }

    // ---- the hidden tile: ReLU (forward) or mask (backward) into A2
    __syncwarp();
    bool ok = tp_wait_warp(t, kTbMma1, p.status, kDevTimeoutDone);
    // the mask tile arrived with full1: observe that phase before reading it
    if (BWD && ok) ok = tp_wait_warp(t, kTbFull1, p.status, kDevTimeoutFull);
    tc_fence_after();
    tp_mark(t);  // first product done (warp 0)
    bc_hidden_tile<BWD>(smem, A2, kBcBwdM, tmem, ok);
    fence_async_smem();  // generic writes of A2 -> visible to the tensor core and TMA
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    tp_mark(t);  // hidden tile in shared memory
    if (threadIdx.x == 0) {
        // V_q / dV_q to global memory (the backward reads V, the weight gradient reads dV)
        for (int kb = 0; kb < 2; kb++)
            if (m0 < p.M) tma_store_2d(BWD ? &tm.dv : &tm.v, h0 + 64 * kb, m0, smem + A2 + kb * 16384);
        bulk_commit();
    } else if (warp == 1 && lane == 0) {
        if (tp_wait(t, kTbFull2, p.status, kDevTimeoutFull)) {
            tc_fence_after();
            bc_mma<!BWD ? true : false>(tmem + 128, smem_u32(smem + A2), smem_u32(smem + kBcB2));
            // dW_up partial = lnOut^T dV_q (TMEM columns 256..383)
            if (BWD) bc_mma_tn(tmem + 256, smem_u32(smem + kBcBwdLn), smem_u32(smem + A2));
        }
        tc_commit(t.bar(kTbMma2));
    }

    // ---- the second product's partial tile into shared memory (reusing A1 + B1)
    __syncwarp();
    const bool ok2 = tp_wait_warp(t, kTbMma2, p.status, kDevTimeoutDone);
    tc_fence_after();
    tp_mark(t);  // second product done (warp 0)
    rows_tmem_to_tile(smem, tmem + 128, ok && ok2);
    if (BWD) {
        // this tile's weight-gradient partial sums: dW_up[:, h0..], dW_down[h0.., :]
        const size_t tile = (size_t)(m0 / kRowsBM);
        // (staged in B2 + M: both free once the products completed; M holds
        // the LayerNorm-backward column sums only after the cluster barrier)
        uint8_t* stage = smem + kBcB2;
        bc_tmem_to_global(stage, p.upPart + tile * kRowsBN * kBcHidden + h0, kBcHidden, tmem + 256, ok && ok2);
        bc_tmem_to_global(stage, p.downPart + tile * kBcHidden * kRowsBN + (size_t)h0 * kRowsBN, kRowsBN, tmem + 384,
                          ok && ok2);
    }
    tc_fence_before();
    __syncthreads();
    if (!t.merged) {
        if (warp == 2) {
            if (!(ok && ok2)) {  // no MMA may run on freed TMEM
                mbar_wait(t.bar(kTbMma1), 0, p.status, kDevTimeoutDone);
                mbar_wait(t.bar(kTbMma2), 0, p.status, kDevTimeoutDone);
            }
            tc_fence_after();
            tmem_dealloc(tmem, kTmemCols);
        }
        if (!ok) {
            // a product that timed out may leave its TMA loads in flight: let them land
            if (threadIdx.x == 0) {
                mbar_wait(t.bar(kTbFull1), 0, p.status, kDevTimeoutFull);
                mbar_wait(t.bar(kTbFull2), 0, p.status, kDevTimeoutFull);
            }
        }
    }
    tp_mark(t);  // partial tile (and weight-gradient partials) written
    cluster_sync();  // every partial tile of the cluster is complete
    tp_mark(t);  // cluster barrier passed

    RowsEpi e = p.e;
    if (BWD) e.inStage = reinterpret_cast<float*>(smem + kBcBwdLn);  // the lnOut tile is no longer needed
    rows_cluster_epilogue<BWD ? kRowsLNBackward : kRowsResidLN, RPC>(smem, reinterpret_cast<float*>(smem + kBcBwdM),
                                                                    q, m0, e);

    tp_mark(t);  // row epilogue done
    if (threadIdx.x == 0) bulk_wait<0>();  // the V / dV store is complete
    t.flip(kTbFull1);
    t.flip(kTbFull2);
    t.flip(kTbMma1);
    t.flip(kTbMma2);
    if (t.merged)
        tp_pass_boundary();  // also: no CTA leaves while another still reads its partial tile
    else
        cluster_sync();  // no CTA leaves while another still reads its partial tile
}

}  // namespace mg
