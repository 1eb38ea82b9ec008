// The row epilogues of the cluster kernels (gemm_rows.cu, block_cluster.cu):
// a 128-row tile of a 128-wide output is computed by a cluster of 4 CTAs, each
// holding an fp32 tile in shared memory (a K-split partial, summed here in
// split order through distributed shared memory); after a cluster barrier
// CTA q owns tile rows [32 q, 32 q + 32), two per warp (16 warps), and ends
// them with
//   kRowsResidLN     h = bf16(h + bf16(acc)), then the LayerNorm of h (the
//                    arithmetic and summation order of k_layernorm_forward,
//                    lane l: columns 4l..4l+3)
//   kRowsLNBackward  dz = bf16(acc), then the LayerNorm backward of dz, with
//                    the skip gradient added when resid is given (the
//                    arithmetic of k_layernorm_backward, including its dgamma
//                    / dbeta partial sums over groups of RPC rows)
#pragma once

#include "gemm_tc.cuh"
#include "policy_kernels.cuh"

namespace mg {

constexpr int kRowsRedBytes = 4 * 8 * 2 * kRowsBN * 4;  // LayerNorm-backward column sums, 32 KB

enum RowsEpilogue : int { kRowsResidLN = 0, kRowsLNBackward = 1 };

struct RowsEpi {
    int M;
    const __nv_bfloat16* resid;  // h before the residual add / the skip gradient (may be null: none)
    __nv_bfloat16* out;          // h after it (may equal resid) / dS = resid + LayerNorm backward
    LnOutputs ln;                // kRowsResidLN
    const __nv_bfloat16* gamma;  // kRowsLNBackward: the LayerNorm's gamma, x-hat and sigma
    const __nv_bfloat16* xNorm;
    const float* stdev;
    float* partial;  // [M / RPC][dgamma (128) | dbeta (128)]
    // kRowsLNBackward, optional (inPartial set): the input layer's gradient
    // partials of the output rows (the rows are then the input layer's dZ), as
    // k_input_backward computes them with 16 rows per partial:
    // inPartial[row / 16][(inDim + 1) x 128], dW rows then db. Row r of the
    // minibatch reads observation mg_minibatch_row(*inMb, r, ..) (row r
    // without inMb). inStage: 32 x 128 + 32 x inDim floats of shared memory.
    const float* inObs;
    const MgMinibatch* inMb;
    uint64_t inEnvRows, inTotal;
    int inDim;
    float* inPartial;
    float* inStage;
};
constexpr int kRowsInputMaxDim = 32;

// After the cluster barrier that completes every CTA's tile: this CTA's 32
// rows of the tile (tile rows of the cluster at the same offset `smem` in
// every CTA), the sum of the 4 tiles in CTA order, then the epilogue. `red`:
// kRowsRedBytes of this CTA's shared memory, unused by the tiles.
// NSUM = 1: the tile is this CTA's own and complete (no cluster).
template <int EPI, int RPC, int NSUM = (int)kRowsCluster>
__device__ __forceinline__ void rows_cluster_epilogue(uint8_t* smem, float* red, uint32_t q, int m0,
                                                      const RowsEpi& e) {
    constexpr int E = kRowsBN;
    // x / E as x * (1 / E): exact for a power of two; 1 / x as the correctly
    // rounded reciprocal: the same values as the LayerNorm kernels' divisions
    constexpr float kInvE = 1.0f / E;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // ---- rows [32 q, 32 q + 32) of the tile, NR per warp, computed side by
    // side (their warp sums interleave); loads and stores of rows past M are
    // skipped, their values unused. LayerNorm backward row order (that of
    // k_layernorm_backward with RPC rows per CTA and 8 warps): per group g of
    // RPC rows, virtual warp v takes rows v, v + 8, .. and sums its dgamma /
    // dbeta over them in that order; virtual warp (g, v) is warp 8 g + v (mod
    // 16) here.
    constexpr int G = 32 / RPC;
    constexpr int J = RPC / 8;
    constexpr int NR = EPI == kRowsResidLN ? 2 : (RPC == 32 ? 4 : 2);
    const bool active = EPI == kRowsResidLN || RPC != 32 || warp < 8;
    const int c0 = lane * 4;
    int rows[NR];
    bool live[NR];
    float4 acc[NR];
    // the cluster's partial tiles: every row's four loads (distributed shared
    // memory) issued before the first add, then the sums in rank order
    float4 part[NR][NSUM];
#pragma unroll
    for (int t = 0; t < NR; t++) {
        int tl;  // row within this CTA's 32
        if (EPI == kRowsResidLN) {
            tl = warp + 16 * t;
        } else {
            const int pr = warp + 16 * (t / J), j = t % J;
            tl = (pr / 8) * RPC + (pr % 8) + 8 * j;
        }
        const int tr = 32 * (int)q + tl;
        rows[t] = m0 + tr;
        live[t] = active && rows[t] < e.M;
        const uint8_t* cell = smem + tile_offset(tr & 127, lane);
#pragma unroll
        for (int r = 0; r < NSUM; r++) {
            part[t][r] = make_float4(0, 0, 0, 0);
            if (active)
                part[t][r] = NSUM == 1 ? *reinterpret_cast<const float4*>(cell)
                                       : ld_f4_generic_now(__cluster_map_shared_rank(cell, (uint32_t)r));
        }
    }
#pragma unroll
    for (int t = 0; t < NR; t++) {
        float4 a = part[t][0];
#pragma unroll
        for (int r = 1; r < NSUM; r++)
            a = make_float4(__fadd_rn(a.x, part[t][r].x), __fadd_rn(a.y, part[t][r].y), __fadd_rn(a.z, part[t][r].z),
                            __fadd_rn(a.w, part[t][r].w));
        acc[t] = a;
    }

    if (EPI == kRowsResidLN) {
        const float4 gm = bf4_load(e.ln.gamma + c0), bt = bf4_load(e.ln.beta + c0);
        const float g[4] = {gm.x, gm.y, gm.z, gm.w}, b[4] = {bt.x, bt.y, bt.z, bt.w};
        float v[NR][4], ms[2 * NR];  // ms: row sums (0..NR-1), sums of squares (NR..)
#pragma unroll
        for (int t = 0; t < NR; t++) {
            const float4 hin = live[t] ? bf4_load(e.resid + (size_t)rows[t] * E + c0) : make_float4(0, 0, 0, 0);
            // the residual add of the down projection (kEpiBf16Resid), then h as bf16
            v[t][0] = round_bf16(hin.x + round_bf16(acc[t].x));
            v[t][1] = round_bf16(hin.y + round_bf16(acc[t].y));
            v[t][2] = round_bf16(hin.z + round_bf16(acc[t].z));
            v[t][3] = round_bf16(hin.w + round_bf16(acc[t].w));
            if (live[t]) bf4_store(e.out + (size_t)rows[t] * E + c0, v[t][0], v[t][1], v[t][2], v[t][3]);
            float sm = 0.0f;
#pragma unroll
            for (int i = 0; i < 4; i++) sm = __fadd_rn(sm, v[t][i]);
            ms[t] = sm;
        }
        warp_sum_n<NR>(ms);
#pragma unroll
        for (int t = 0; t < NR; t++) {
            ms[t] = __fmul_rn(ms[t], kInvE);
            float sq = 0.0f;
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const float d = __fsub_rn(v[t][i], ms[t]);
                sq = __fadd_rn(sq, __fmul_rn(d, d));
            }
            ms[NR + t] = sq;
        }
        warp_sum_n<NR>(ms + NR);
#pragma unroll
        for (int t = 0; t < NR; t++) {
            const float sd = __fsqrt_rn(__fadd_rn(__fmul_rn(ms[NR + t], kInvE), 1e-5f));
            const float rstd = __frcp_rn(sd);
            if (!live[t]) continue;
            if (lane == 0) e.ln.stdev[rows[t]] = sd;
            float xn[4], y[4];
#pragma unroll
            for (int i = 0; i < 4; i++) {
                xn[i] = __fmul_rn(__fsub_rn(v[t][i], ms[t]), rstd);
                y[i] = __fadd_rn(__fmul_rn(g[i], xn[i]), b[i]);
            }
            bf4_store(e.ln.xNorm + (size_t)rows[t] * E + c0, xn[0], xn[1], xn[2], xn[3]);
            bf4_store(e.ln.out + (size_t)rows[t] * E + c0, y[0], y[1], y[2], y[3]);
        }
    } else {
        // red: [G][8 virtual warps][dgamma | dbeta]
        const float4 gm = bf4_load(e.gamma + c0);
        const float g[4] = {gm.x, gm.y, gm.z, gm.w};
        float xn[NR][4], dxn[NR][4], s12[2 * NR], rdev[NR];  // s12: sums of dxn (0..NR-1), of dxn x-hat (NR..)
        float dg[4], db[4];
#pragma unroll
        for (int t = 0; t < NR; t++) {
            const float4 x4 = live[t] ? bf4_load(e.xNorm + (size_t)rows[t] * E + c0) : make_float4(0, 0, 0, 0);
            rdev[t] = __frcp_rn(live[t] ? e.stdev[rows[t]] : 1.0f);
            xn[t][0] = x4.x;
            xn[t][1] = x4.y;
            xn[t][2] = x4.z;
            xn[t][3] = x4.w;
            const float dz[4] = {round_bf16(acc[t].x), round_bf16(acc[t].y), round_bf16(acc[t].z),
                                 round_bf16(acc[t].w)};
            if (t % J == 0) {
#pragma unroll
                for (int i = 0; i < 4; i++) dg[i] = db[i] = 0.0f;
            }
            s12[t] = 0.0f;
            s12[NR + t] = 0.0f;
#pragma unroll
            for (int i = 0; i < 4; i++) {
                if (live[t]) {
                    dg[i] = __fadd_rn(dg[i], rbf(__fmul_rn(xn[t][i], dz[i])));
                    db[i] = __fadd_rn(db[i], dz[i]);
                }
                dxn[t][i] = rbf(__fmul_rn(dz[i], g[i]));
                s12[t] = __fadd_rn(s12[t], dxn[t][i]);
                s12[NR + t] = __fadd_rn(s12[NR + t], rbf(__fmul_rn(dxn[t][i], xn[t][i])));
            }
            if (t % J == J - 1 && active) {
                const int pr = warp + 16 * (t / J);  // virtual warp (pr / 8, pr % 8)
                float* dst = red + (size_t)pr * 2 * E;
                *reinterpret_cast<float4*>(dst + c0) = make_float4(dg[0], dg[1], dg[2], dg[3]);
                *reinterpret_cast<float4*>(dst + E + c0) = make_float4(db[0], db[1], db[2], db[3]);
            }
        }
        warp_sum_n<2 * NR>(s12);
#pragma unroll
        for (int t = 0; t < 2 * NR; t++) s12[t] = __fmul_rn(s12[t], kInvE);
#pragma unroll
        for (int t = 0; t < NR; t++) {
            if (!live[t]) continue;
            float o[4];
#pragma unroll
            for (int i = 0; i < 4; i++)
                o[i] = __fmul_rn(rdev[t], __fsub_rn(__fsub_rn(dxn[t][i], s12[t]), __fmul_rn(xn[t][i], s12[NR + t])));
            if (e.resid) {  // the skip add: bf16(bf16(dx) + resid)
                const float4 rs = bf4_load(e.resid + (size_t)rows[t] * E + c0);
                o[0] = __fadd_rn(rbf(o[0]), rs.x);
                o[1] = __fadd_rn(rbf(o[1]), rs.y);
                o[2] = __fadd_rn(rbf(o[2]), rs.z);
                o[3] = __fadd_rn(rbf(o[3]), rs.w);
            }
            bf4_store(e.out + (size_t)rows[t] * E + c0, o[0], o[1], o[2], o[3]);
            if (e.inPartial)  // the stored (bf16) values, for the input layer's gradient
                *reinterpret_cast<float4*>(e.inStage + (rows[t] - m0 - 32 * (int)q) * E + c0) =
                    make_float4(rbf(o[0]), rbf(o[1]), rbf(o[2]), rbf(o[3]));
        }
        if (e.inPartial) {
            float* sObs = e.inStage + 32 * E;
            for (int i = threadIdx.x; i < 32 * e.inDim; i += blockDim.x) {
                const int row = m0 + 32 * (int)q + i / e.inDim;
                if (row >= e.M) continue;
                const uint64_t g = e.inMb ? mg_minibatch_row(*e.inMb, row, e.inEnvRows, e.inTotal) : (uint64_t)row;
                sObs[i] = e.inObs[g * e.inDim + i % e.inDim];
            }
        }
        __syncthreads();
        if (e.inPartial) {
            // k_input_backward's sums over each 16 rows, in row order
            const float* sObs = e.inStage + 32 * E;
            for (int i = threadIdx.x; i < 2 * E; i += blockDim.x) {
                const int half = i / E, c = i % E;
                const int first = m0 + 32 * (int)q + 16 * half;
                if (first >= e.M) continue;
                const int nr = min(16, e.M - first);
                const float* d = e.inStage + (16 * half) * E + c;
                const float* ob = sObs + (16 * half) * e.inDim;
                float* part = e.inPartial + (size_t)(first / 16) * (e.inDim + 1) * E;
                float accB = 0.0f;
                for (int r = 0; r < nr; r++) accB = __fadd_rn(accB, d[r * E]);
                part[(size_t)e.inDim * E + c] = accB;
                for (int k0 = 0; k0 < e.inDim; k0 += 8) {
                    float acc[8];
#pragma unroll
                    for (int k = 0; k < 8; k++) acc[k] = 0.0f;
                    for (int r = 0; r < nr; r++) {
                        const float dv = d[r * E];
#pragma unroll
                        for (int k = 0; k < 8; k++)
                            if (k0 + k < e.inDim) acc[k] = __fmaf_rn(ob[r * e.inDim + k0 + k], dv, acc[k]);
                    }
#pragma unroll
                    for (int k = 0; k < 8; k++)
                        if (k0 + k < e.inDim) part[(size_t)(k0 + k) * E + c] = acc[k];
                }
            }
        }
        // one partial per group of RPC rows: its virtual warps' sums in order
        for (int i = threadIdx.x; i < G * 2 * E; i += blockDim.x) {
            const int grp = i / (2 * E), c = i % (2 * E);
            const int first = m0 + 32 * (int)q + grp * RPC;
            if (first >= e.M) continue;
            float sacc = 0.0f;
#pragma unroll
            for (int v = 0; v < 8; v++) sacc = __fadd_rn(sacc, red[((size_t)grp * 8 + v) * 2 * E + c]);
            e.partial[(size_t)(first / RPC) * 2 * E + c] = sacc;
        }
    }
}

}  // namespace mg
