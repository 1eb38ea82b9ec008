// Row-wise kernels of the PPO hot path and their C-ABI entry points.
// The dense products live in gemm.cu; everything else lives here.
#include <algorithm>

#include "row_epilogues.cuh"
#include "policy.h"
#include "policy_kernels.cuh"
#include "runtime.h"

namespace mg {

namespace {

constexpr int kMaxRowParts = 296;       // row-reduction kernels: at most two partial sums per SM
constexpr int64_t kInputPartialBudget = 32 << 20;  // bytes of input-backward partials at most
constexpr int kInputSmemBudget = 96 * 1024;        // bytes of staged rows per input-backward CTA
constexpr int kGaussRowsPerCta = 256;  // Gaussian loss: rows per CTA

// ------------------------------------------------------------------ input

// model/input.metal:11-27: out[r, c] = bf16(b[c] + sum_k obs[r, k] * W[k, c]),
// summed in k order with separate roundings. W sits in shared memory as
// fp32; each warp computes RPW rows at a time (their observations staged in
// shared memory), lane l owning the column pairs 2l + 64j, so every weight
// read serves RPW rows and the shared-memory reads are conflict-free.
//
// With LN, the first block's LayerNorm of each output row follows in the same
// kernel (k_layernorm_forward's arithmetic and summation order exactly: the
// row's bf16 values pass through shared memory so that lane l reads columns
// l*VPT .. l*VPT + VPT - 1).
template <int VPT, int RPW, bool LN>
__global__ void __launch_bounds__(256) k_input_forward(const float* __restrict__ obs, const __nv_bfloat16* __restrict__ w,
                                                       const __nv_bfloat16* __restrict__ bias,
                                                       __nv_bfloat16* __restrict__ out, int rows, int inDim, int outDim,
                                                       RowMap rm, LnOutputs ln) {
    constexpr int NP = VPT / 2;  // column pairs per lane
    mg_pdl_trigger();
    mg_pdl_wait();
    // inDim x outDim weights as fp32, then per warp RPW x inDim observations,
    // then (LN) per warp RPW x outDim bf16 output rows
    extern __shared__ float s_w[];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
    float* s_obs = s_w + inDim * outDim + warp * RPW * inDim;
    __nv_bfloat16* s_row = reinterpret_cast<__nv_bfloat16*>(s_w + inDim * outDim + nwarps * RPW * inDim) +
                           (size_t)warp * RPW * outDim;
    float g[VPT], bt[VPT];
    if (LN) {
#pragma unroll
        for (int j = 0; j < VPT; j++) {
            g[j] = bf(ln.gamma[lane * VPT + j]);
            bt[j] = bf(ln.beta[lane * VPT + j]);
        }
    }
    for (int i = threadIdx.x; i < inDim * outDim; i += blockDim.x) s_w[i] = bf(w[i]);
    __syncthreads();
    float2 b[NP];
#pragma unroll
    for (int j = 0; j < NP; j++) b[j] = make_float2(bf(bias[2 * lane + 64 * j]), bf(bias[2 * lane + 64 * j + 1]));
    for (int r0 = (blockIdx.x * nwarps + warp) * RPW; r0 < rows; r0 += gridDim.x * nwarps * RPW) {
        // each row's rollout index once (lane q for row r0 + q), then its observations
        uint64_t gq = 0;
        if (lane < RPW && r0 + lane < rows)
            gq = rm.mb ? mg_minibatch_row(*rm.mb, r0 + lane, rm.envRows, rm.total) : (uint64_t)(r0 + lane);
        uint64_t gr[RPW];
#pragma unroll
        for (int q = 0; q < RPW; q++) gr[q] = __shfl_sync(0xffffffffu, gq, q);
        for (int i = lane; i < RPW * inDim; i += 32) {
            const int qi = i / inDim;
            const int r = r0 + qi;
            float v = 0.0f;
            if (r < rows) {
                uint64_t g = gr[0];
#pragma unroll
                for (int q = 1; q < RPW; q++)
                    if (qi == q) g = gr[q];
                v = obs[g * inDim + i % inDim];
            }
            s_obs[i] = v;
        }
        __syncwarp();
        float2 acc[RPW][NP];
#pragma unroll
        for (int q = 0; q < RPW; q++)
#pragma unroll
            for (int j = 0; j < NP; j++) acc[q][j] = b[j];
        for (int k = 0; k < inDim; k++) {
            float2 wk[NP];
#pragma unroll
            for (int j = 0; j < NP; j++) wk[j] = *reinterpret_cast<const float2*>(s_w + k * outDim + 2 * lane + 64 * j);
#pragma unroll
            for (int q = 0; q < RPW; q++) {
                const float o = s_obs[q * inDim + k];
#pragma unroll
                for (int j = 0; j < NP; j++) {
                    acc[q][j].x = __fadd_rn(acc[q][j].x, __fmul_rn(o, wk[j].x));
                    acc[q][j].y = __fadd_rn(acc[q][j].y, __fmul_rn(o, wk[j].y));
                }
            }
        }
#pragma unroll
        for (int q = 0; q < RPW; q++) {
            if (r0 + q >= rows) break;
            __nv_bfloat16* dst = out + (size_t)(r0 + q) * outDim + 2 * lane;
#pragma unroll
            for (int j = 0; j < NP; j++) {
                const __nv_bfloat162 hv = __floats2bfloat162_rn(acc[q][j].x, acc[q][j].y);
                *reinterpret_cast<__nv_bfloat162*>(dst + 64 * j) = hv;
                if (LN) *reinterpret_cast<__nv_bfloat162*>(s_row + q * outDim + 2 * lane + 64 * j) = hv;
            }
        }
        if (LN) {
            __syncwarp();
#pragma unroll
            for (int q = 0; q < RPW; q++) {
                const int r = r0 + q;
                if (r >= rows) break;
                // k_layernorm_forward on the row (lane l: columns l*VPT ..)
                float v[VPT];
#pragma unroll
                for (int j = 0; j < VPT; j++) v[j] = bf(s_row[q * outDim + lane * VPT + j]);
                float sum = 0.0f;
#pragma unroll
                for (int j = 0; j < VPT; j++) sum = __fadd_rn(sum, v[j]);
                const float mean = __fdiv_rn(warp_sum(sum), (float)outDim);
                float sq = 0.0f;
#pragma unroll
                for (int j = 0; j < VPT; j++) {
                    const float d = __fsub_rn(v[j], mean);
                    sq = __fadd_rn(sq, __fmul_rn(d, d));
                }
                const float var = __fdiv_rn(warp_sum(sq), (float)outDim);
                const float sd = __fsqrt_rn(__fadd_rn(var, 1e-5f));
                const float rstd = __fdiv_rn(1.0f, sd);
                if (lane == 0) ln.stdev[r] = sd;
                __nv_bfloat16* xo = ln.xNorm + (size_t)r * outDim + lane * VPT;
                __nv_bfloat16* yo = ln.out + (size_t)r * outDim + lane * VPT;
#pragma unroll
                for (int j = 0; j < VPT; j += 2) {
                    const float x0 = __fmul_rn(__fsub_rn(v[j], mean), rstd);
                    const float x1 = __fmul_rn(__fsub_rn(v[j + 1], mean), rstd);
                    *reinterpret_cast<__nv_bfloat162*>(xo + j) = __floats2bfloat162_rn(x0, x1);
                    *reinterpret_cast<__nv_bfloat162*>(yo + j) = __floats2bfloat162_rn(
                        __fadd_rn(__fmul_rn(g[j], x0), bt[j]), __fadd_rn(__fmul_rn(g[j + 1], x1), bt[j + 1]));
                }
            }
        }
        __syncwarp();
    }
}

// model/input.metal:38-60: per-CTA partial sums over a contiguous range of
// rowsPerCta rows of dW[k, c] = sum_r obs[r, k] dZ[r, c] and db[c] = sum_r
// dZ[r, c]; partial[blockIdx] = [(inDim + 1) x outDim]: rows 0..inDim-1 dW,
// row inDim db, each summed in row order with fused multiply-adds (the
// reference's order of these sums is unspecified: fp32 atomics). The CTA's
// dZ rows (bf16) and observation rows (fp32, gathered through the row map)
// are staged in shared memory; a thread owns a column and sweeps k in
// chunks of 8 registers.
__global__ void __launch_bounds__(256) k_input_backward(const float* __restrict__ obs, const __nv_bfloat16* __restrict__ dZ,
                                                        float* __restrict__ partial, int rows, int inDim, int outDim,
                                                        int rowsPerCta, RowMap rm) {
    mg_pdl_trigger();
    mg_pdl_wait();
    extern __shared__ float s_obs[];  // rowsPerCta x inDim fp32, rowsPerCta x outDim bf16, rowsPerCta x u64
    const int r0 = blockIdx.x * rowsPerCta;
    const int nr = min(rowsPerCta, rows - r0);
    __nv_bfloat16* s_dz = reinterpret_cast<__nv_bfloat16*>(s_obs + rowsPerCta * inDim);
    // each row's rollout index once, then its observations
    uint64_t* s_g = reinterpret_cast<uint64_t*>(s_dz + rowsPerCta * outDim);
    for (int i = threadIdx.x; i < nr; i += blockDim.x)
        s_g[i] = rm.mb ? mg_minibatch_row(*rm.mb, r0 + i, rm.envRows, rm.total) : (uint64_t)(r0 + i);
    __syncthreads();
    for (int i = threadIdx.x; i < nr * inDim; i += blockDim.x) s_obs[i] = obs[s_g[i / inDim] * inDim + i % inDim];
    {
        // dZ rows r0 .. r0 + nr are contiguous: 16-byte copies
        const uint4* src = reinterpret_cast<const uint4*>(dZ + (size_t)r0 * outDim);
        uint4* dst = reinterpret_cast<uint4*>(s_dz);
        const int n16 = nr * outDim / 8;
        for (int i = threadIdx.x; i < n16; i += blockDim.x) dst[i] = src[i];
    }
    __syncthreads();
    float* part = partial + (size_t)blockIdx.x * (inDim + 1) * outDim;
    for (int c = threadIdx.x; c < outDim; c += blockDim.x) {
        float accB = 0.0f;
        for (int r = 0; r < nr; r++) accB = __fadd_rn(accB, bf(s_dz[r * outDim + c]));
        part[(size_t)inDim * outDim + c] = accB;
        for (int k0 = 0; k0 < inDim; k0 += 8) {
            float acc[8];
#pragma unroll
            for (int k = 0; k < 8; k++) acc[k] = 0.0f;
            if (k0 + 8 <= inDim) {
                for (int r = 0; r < nr; r++) {
                    const float d = bf(s_dz[r * outDim + c]);
                    const float2 d2 = make_float2(d, d);
                    const float* o = s_obs + r * inDim + k0;
#pragma unroll
                    for (int k = 0; k < 8; k += 2) {
                        const float2 a = f2fma_rn(make_float2(o[k], o[k + 1]), d2, make_float2(acc[k], acc[k + 1]));
                        acc[k] = a.x;
                        acc[k + 1] = a.y;
                    }
                }
            } else {
                for (int r = 0; r < nr; r++) {
                    const float d = bf(s_dz[r * outDim + c]);
                    const float* o = s_obs + r * inDim + k0;
#pragma unroll
                    for (int k = 0; k < 8; k++)
                        if (k0 + k < inDim) acc[k] = __fmaf_rn(o[k], d, acc[k]);
                }
            }
#pragma unroll
            for (int k = 0; k < 8; k++)
                if (k0 + k < inDim) part[(size_t)(k0 + k) * outDim + c] = acc[k];
        }
    }
}

// The same sums with every observation column's accumulator in registers
// (inDim <= KMAX): rows outer, so each row's dZ value and observations are
// read from shared memory once (four at a time with VEC4) instead of once per
// chunk of 8 columns; the additions per accumulator run in the same row order,
// so the partials are bit-identical to k_input_backward's.
template <int KMAX, bool VEC4>
__global__ void __launch_bounds__(256) k_input_backward_regs(const float* __restrict__ obs,
                                                             const __nv_bfloat16* __restrict__ dZ,
                                                             float* __restrict__ partial, int rows, int inDim,
                                                             int outDim, int rowsPerCta, RowMap rm) {
    mg_pdl_trigger();
    mg_pdl_wait();
    extern __shared__ float s_obs[];  // rowsPerCta x inDim fp32, rowsPerCta x outDim bf16, rowsPerCta x u64
    const int r0 = blockIdx.x * rowsPerCta;
    const int nr = min(rowsPerCta, rows - r0);
    __nv_bfloat16* s_dz = reinterpret_cast<__nv_bfloat16*>(s_obs + rowsPerCta * inDim);
    // each row's rollout index once, then its observations
    uint64_t* s_g = reinterpret_cast<uint64_t*>(s_dz + rowsPerCta * outDim);
    for (int i = threadIdx.x; i < nr; i += blockDim.x)
        s_g[i] = rm.mb ? mg_minibatch_row(*rm.mb, r0 + i, rm.envRows, rm.total) : (uint64_t)(r0 + i);
    __syncthreads();
    for (int i = threadIdx.x; i < nr * inDim; i += blockDim.x) s_obs[i] = obs[s_g[i / inDim] * inDim + i % inDim];
    {
        const uint4* src = reinterpret_cast<const uint4*>(dZ + (size_t)r0 * outDim);
        uint4* dst = reinterpret_cast<uint4*>(s_dz);
        const int n16 = nr * outDim / 8;
        for (int i = threadIdx.x; i < n16; i += blockDim.x) dst[i] = src[i];
    }
    __syncthreads();
    float* part = partial + (size_t)blockIdx.x * (inDim + 1) * outDim;
    for (int c = threadIdx.x; c < outDim; c += blockDim.x) {
        float acc[KMAX];
#pragma unroll
        for (int k = 0; k < KMAX; k++) acc[k] = 0.0f;
        float accB = 0.0f;
        for (int r = 0; r < nr; r++) {
            const float d = bf(s_dz[r * outDim + c]);
            accB = __fadd_rn(accB, d);
            const float2 d2 = make_float2(d, d);
            const float* o = s_obs + r * inDim;
#pragma unroll
            for (int k = 0; k < KMAX; k += 4) {
                if (k >= inDim) break;
                float4 ov;
                if (VEC4) {
                    ov = *reinterpret_cast<const float4*>(o + k);
                } else {
                    ov = make_float4(o[k], k + 1 < inDim ? o[k + 1] : 0.0f, k + 2 < inDim ? o[k + 2] : 0.0f,
                                     k + 3 < inDim ? o[k + 3] : 0.0f);
                }
                const float2 a = f2fma_rn(make_float2(ov.x, ov.y), d2, make_float2(acc[k], acc[k + 1]));
                const float2 b = f2fma_rn(make_float2(ov.z, ov.w), d2, make_float2(acc[k + 2], acc[k + 3]));
                acc[k] = a.x;
                acc[k + 1] = a.y;
                acc[k + 2] = b.x;
                acc[k + 3] = b.y;
            }
        }
        part[(size_t)inDim * outDim + c] = accB;
#pragma unroll
        for (int k = 0; k < KMAX; k++)
            if (k < inDim) part[(size_t)k * outDim + c] = acc[k];
    }
}

// -------------------------------------------------------------- layernorm

// model/layernorm.metal:10-71. One warp per row; lane l owns VPT consecutive
// columns. Two-pass mean / population variance, sigma = sqrt(var + 1e-5).
template <int VPT>
__global__ void k_layernorm_forward(const __nv_bfloat16* __restrict__ x, __nv_bfloat16* __restrict__ xNorm,
                                    __nv_bfloat16* __restrict__ out, const __nv_bfloat16* __restrict__ gamma,
                                    const __nv_bfloat16* __restrict__ beta, float* __restrict__ stdev, int rows) {
    mg_pdl_trigger();
    mg_pdl_wait();
    constexpr int E = VPT * 32;
    const int lane = threadIdx.x & 31;
    const int c0 = lane * VPT;
    float g[VPT], b[VPT];
#pragma unroll
    for (int j = 0; j < VPT; j++) {
        g[j] = bf(gamma[c0 + j]);
        b[j] = bf(beta[c0 + j]);
    }
    for (int r = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); r < rows; r += gridDim.x * (blockDim.x >> 5)) {
        float v[VPT];
        const __nv_bfloat16* xr = x + (size_t)r * E + c0;
#pragma unroll
        for (int j = 0; j < VPT; j += 2) {
            const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(xr + j));
            v[j] = f.x;
            v[j + 1] = f.y;
        }
        float s = 0.0f;
#pragma unroll
        for (int j = 0; j < VPT; j++) s = __fadd_rn(s, v[j]);
        const float mean = __fdiv_rn(warp_sum(s), (float)E);
        float q = 0.0f;
#pragma unroll
        for (int j = 0; j < VPT; j++) {
            const float d = __fsub_rn(v[j], mean);
            q = __fadd_rn(q, __fmul_rn(d, d));
        }
        const float var = __fdiv_rn(warp_sum(q), (float)E);
        const float sd = __fsqrt_rn(__fadd_rn(var, 1e-5f));
        const float rstd = __fdiv_rn(1.0f, sd);
        if (lane == 0) stdev[r] = sd;
        __nv_bfloat16* xn_out = xNorm + (size_t)r * E + c0;
        __nv_bfloat16* y_out = out + (size_t)r * E + c0;
#pragma unroll
        for (int j = 0; j < VPT; j += 2) {
            const float xn0 = __fmul_rn(__fsub_rn(v[j], mean), rstd);
            const float xn1 = __fmul_rn(__fsub_rn(v[j + 1], mean), rstd);
            *reinterpret_cast<__nv_bfloat162*>(xn_out + j) = __floats2bfloat162_rn(xn0, xn1);
            *reinterpret_cast<__nv_bfloat162*>(y_out + j) = __floats2bfloat162_rn(
                __fadd_rn(__fmul_rn(g[j], xn0), b[j]), __fadd_rn(__fmul_rn(g[j + 1], xn1), b[j + 1]));
        }
    }
}

// model/layernorm.metal:74-127 (+ model/elementwise.metal:4-13 when resid is
// given). Per row: dxhat = bf16(dz * gamma); dx = bf16((dxhat - mean(dxhat)
// - xhat * mean(bf16(dxhat * xhat))) / sigma). Without resid dx overwrites dZ;
// with resid, residOut = bf16(dx + resid) (residOut may be resid) and dZ is
// left as is. dgamma
// (sum of bf16(xhat * dz)) and dbeta (sum of dz) are summed over this CTA's
// rows into partial[blockIdx] = [dgamma (E) | dbeta (E)].
template <int VPT>
__global__ void __launch_bounds__(256) k_layernorm_backward(__nv_bfloat16* __restrict__ dZ,
                                                            const __nv_bfloat16* __restrict__ xNorm,
                                                            const __nv_bfloat16* __restrict__ gamma,
                                                            const float* __restrict__ stdev,
                                                            const __nv_bfloat16* resid, __nv_bfloat16* residOut,
                                                            float* __restrict__ partial, int rows, int rowsPerCta) {
    mg_pdl_trigger();
    mg_pdl_wait();
    constexpr int E = VPT * 32;
    __shared__ float s_red[8][2 * E];
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int c0 = lane * VPT;
    float g[VPT], dg[VPT], db[VPT];
#pragma unroll
    for (int j = 0; j < VPT; j++) {
        g[j] = bf(gamma[c0 + j]);
        dg[j] = 0.0f;
        db[j] = 0.0f;
    }
    const int r0 = blockIdx.x * rowsPerCta;
    const int r1 = min(rows, r0 + rowsPerCta);
    // rows r, r + 8, r + 16, r + 24 of the warp per step: all four rows' loads
    // (kept as packed bf16 pairs) are issued before any row is computed; the
    // sums run over the rows in the same order as one row at a time
    constexpr int RIF = 4;
    constexpr int W = VPT / 2;  // bf16 pairs per lane and row
    auto unpack = [](uint32_t w, float& a, float& b) {
        a = __uint_as_float(w << 16);
        b = __uint_as_float(w & 0xffff0000u);
    };
    for (int r = r0 + warp; r < r1; r += 8 * RIF) {
        uint32_t wdz[RIF][W], wxn[RIF][W], wrs[RIF][W];
        float sdv[RIF];
#pragma unroll
        for (int k = 0; k < RIF; k++) {
            if (r + 8 * k >= r1) break;
            const size_t base = (size_t)(r + 8 * k) * E + c0;
#pragma unroll
            for (int j = 0; j < W; j++) {
                wdz[k][j] = *reinterpret_cast<const uint32_t*>(dZ + base + 2 * j);
                wxn[k][j] = *reinterpret_cast<const uint32_t*>(xNorm + base + 2 * j);
                if (resid) wrs[k][j] = *reinterpret_cast<const uint32_t*>(resid + base + 2 * j);
            }
            sdv[k] = stdev[r + 8 * k];
        }
#pragma unroll
        for (int k = 0; k < RIF; k++) {
            if (r + 8 * k >= r1) break;
            const size_t base = (size_t)(r + 8 * k) * E + c0;
            float dz[VPT], xn[VPT];
#pragma unroll
            for (int j = 0; j < W; j++) {
                unpack(wdz[k][j], dz[2 * j], dz[2 * j + 1]);
                unpack(wxn[k][j], xn[2 * j], xn[2 * j + 1]);
            }
            float dxn[VPT];
            float s1 = 0.0f, s2 = 0.0f;
#pragma unroll
            for (int j = 0; j < VPT; j++) {
                dg[j] = __fadd_rn(dg[j], rbf(__fmul_rn(xn[j], dz[j])));
                db[j] = __fadd_rn(db[j], dz[j]);
                dxn[j] = rbf(__fmul_rn(dz[j], g[j]));
                s1 = __fadd_rn(s1, dxn[j]);
                s2 = __fadd_rn(s2, rbf(__fmul_rn(dxn[j], xn[j])));
            }
            const float m1 = __fdiv_rn(warp_sum(s1), (float)E);
            const float m2 = __fdiv_rn(warp_sum(s2), (float)E);
            const float rdev = __fdiv_rn(1.0f, sdv[k]);
            float dx[VPT];
#pragma unroll
            for (int j = 0; j < VPT; j++)
                dx[j] = __fmul_rn(rdev, __fsub_rn(__fsub_rn(dxn[j], m1), __fmul_rn(xn[j], m2)));
            if (resid) {
#pragma unroll
                for (int j = 0; j < W; j++) {
                    float r0f, r1f;
                    unpack(wrs[k][j], r0f, r1f);
                    *reinterpret_cast<__nv_bfloat162*>(residOut + base + 2 * j) = __floats2bfloat162_rn(
                        __fadd_rn(rbf(dx[2 * j]), r0f), __fadd_rn(rbf(dx[2 * j + 1]), r1f));
                }
            } else {
#pragma unroll
                for (int j = 0; j < VPT; j += 2)
                    *reinterpret_cast<__nv_bfloat162*>(dZ + base + j) = __floats2bfloat162_rn(dx[j], dx[j + 1]);
            }
        }
    }
#pragma unroll
    for (int j = 0; j < VPT; j++) {
        s_red[warp][c0 + j] = dg[j];
        s_red[warp][E + c0 + j] = db[j];
    }
    __syncthreads();
    for (int i = threadIdx.x; i < 2 * E; i += blockDim.x) {
        float acc = 0.0f;
#pragma unroll
        for (int w2 = 0; w2 < 8; w2++) acc = __fadd_rn(acc, s_red[w2][i]);
        partial[(size_t)blockIdx.x * 2 * E + i] = acc;
    }
}

// ------------------------------------------------------- sampling / losses

__global__ void k_sample_categorical(const __nv_bfloat16* __restrict__ head, uint32_t* __restrict__ rng,
                                     int32_t* __restrict__ action, float* __restrict__ logProb,
                                     float* __restrict__ value, int rows, int actDim) {
    mg_pdl_trigger();
    mg_pdl_wait();
    const int r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= rows) return;
    uint32_t s = rng[r];
    float lp, v;
    action[r] = sample_categorical_row(head + (size_t)r * kHeadDim, actDim, s, lp, v);
    rng[r] = s;
    logProb[r] = lp;
    value[r] = v;
}

__global__ void k_sample_gaussian(const __nv_bfloat16* __restrict__ head, const __nv_bfloat16* __restrict__ logStd,
                                  uint32_t* __restrict__ rng, float* __restrict__ action, float* __restrict__ logProb,
                                  float* __restrict__ value, int rows, int actDim) {
    mg_pdl_trigger();
    mg_pdl_wait();
    const int r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= rows) return;
    uint32_t s = rng[r];
    float lp, v;
    sample_gaussian_row(head + (size_t)r * kHeadDim, logStd, actDim, s, action + (size_t)r * actDim, lp, v);
    rng[r] = s;
    logProb[r] = lp;
    value[r] = v;
}

__device__ __forceinline__ float norm_adv(const float* adv, const float* advStats, int r) {
    // model/gae.metal:76: (a - mean) * inv, inv = 1 / (sigma + 1e-8)
    return advStats ? __fmul_rn(__fsub_rn(adv[r], advStats[0]), advStats[1]) : adv[r];
}

// model/policy.metal:14-69. One thread per row (policy_loss_row).
__global__ void k_policy_loss(const __nv_bfloat16* __restrict__ head, const PolicyLossRows L, int* status) {
    mg_pdl_trigger();
    mg_pdl_wait();
    const int r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= L.rows) return;
    policy_loss_row(L, r, head + (size_t)r * kHeadDim, status);
}

// model/gaussian.metal:76-135. One thread per row; the log-std gradient is a
// batch sum, summed per CTA into partial[blockIdx][k].
__global__ void __launch_bounds__(kGaussRowsPerCta) k_gaussian_loss(
    const __nv_bfloat16* __restrict__ head, const float* __restrict__ action, const float* __restrict__ adv,
    const float* __restrict__ advStats, const float* __restrict__ ret, const float* __restrict__ oldLogProb,
    __nv_bfloat16* __restrict__ dZ, float* __restrict__ stats, const __nv_bfloat16* __restrict__ logStd,
    float* __restrict__ partial, int rows, int actDim, LossHyper hp, RowMap rm) {
    mg_pdl_trigger();
    mg_pdl_wait();
    __shared__ float s_gls[kGaussRowsPerCta];
    if (rm.mb && rm.mb->slot >= 0 && advStats) advStats += 2 * rm.mb->slot;  // per-slot statistics
    const int r = blockIdx.x * blockDim.x + threadIdx.x;
    const int64_t g = (r < rows && rm.mb) ? (int64_t)mg_minibatch_row(*rm.mb, r, rm.envRows, rm.total) : r;
    const bool live = r < rows;
    const float scale = __fdiv_rn(1.0f, (float)rows);
    float gLogp = 0.0f;
    if (live) {
        const __nv_bfloat16* h = head + (size_t)r * kHeadDim;
        const float* act = action + (size_t)g * actDim;
        float logp = 0.0f, entropy = 0.0f;
        for (int k = 0; k < actDim; k++) {
            const float ls = bf(logStd[k]);
            const float d = __fmul_rn(__fsub_rn(act[k], bf(h[k])), mg_expf(-ls));
            logp = __fadd_rn(logp, __fsub_rn(__fsub_rn(__fmul_rn(__fmul_rn(-0.5f, d), d), ls), kLogSqrt2Pi));
            entropy = __fadd_rn(entropy, __fadd_rn(__fadd_rn(ls, kLogSqrt2Pi), 0.5f));
        }
        const float A = norm_adv(adv, advStats, g);
        const float ratio = mg_expf(__fsub_rn(logp, oldLogProb[g]));
        const float surr1 = __fmul_rn(ratio, A);
        const float surr2 = __fmul_rn(fminf(fmaxf(ratio, __fsub_rn(1.0f, hp.clip)), __fadd_rn(1.0f, hp.clip)), A);
        const float policyLoss = -fminf(surr1, surr2);
        gLogp = (surr1 <= surr2) ? __fmul_rn(-A, ratio) : 0.0f;
        uint32_t packed[kHeadDim / 2];
#pragma unroll
        for (int i = 0; i < kHeadDim / 2; i++) packed[i] = 0;
        __nv_bfloat16* pz = reinterpret_cast<__nv_bfloat16*>(packed);
        for (int k = 0; k < actDim; k++) {
            const float ls = bf(logStd[k]);
            const float invStd = mg_expf(-ls);
            const float d = __fmul_rn(__fsub_rn(act[k], bf(h[k])), invStd);
            pz[k] = tobf(__fmul_rn(__fmul_rn(__fmul_rn(gLogp, d), invStd), scale));
        }
        const float vErr = __fsub_rn(bf(h[actDim]), ret[g]);
        pz[actDim] = tobf(__fmul_rn(__fmul_rn(hp.valueCoef, vErr), scale));
        uint4* dst = reinterpret_cast<uint4*>(dZ + (size_t)r * kHeadDim);
        const uint4* src = reinterpret_cast<const uint4*>(packed);
#pragma unroll
        for (int i = 0; i < kHeadDim / 8; i++) dst[i] = src[i];
        float* st = stats + (size_t)r * 5;
        st[0] = policyLoss;
        st[1] = __fmul_rn(__fmul_rn(__fmul_rn(0.5f, hp.valueCoef), vErr), vErr);
        st[2] = entropy;
        st[3] = __fsub_rn(oldLogProb[g], logp);
        st[4] = (fabsf(__fsub_rn(ratio, 1.0f)) > hp.clip) ? 1.0f : 0.0f;
    }
    for (int k = 0; k < actDim; k++) {
        float gls = 0.0f;
        if (live) {
            const float ls = bf(logStd[k]);
            const float invStd = mg_expf(-ls);
            const float d = __fmul_rn(__fsub_rn(action[(size_t)g * actDim + k], bf(head[(size_t)r * kHeadDim + k])),
                                      invStd);
            gls = __fmul_rn(__fsub_rn(__fmul_rn(gLogp, __fsub_rn(__fmul_rn(d, d), 1.0f)), hp.entropyCoef), scale);
        }
        s_gls[threadIdx.x] = gls;
        __syncthreads();
        for (int w = blockDim.x >> 1; w > 0; w >>= 1) {
            if (threadIdx.x < w) s_gls[threadIdx.x] = __fadd_rn(s_gls[threadIdx.x], s_gls[threadIdx.x + w]);
            __syncthreads();
        }
        if (threadIdx.x == 0) partial[(size_t)blockIdx.x * actDim + k] = s_gls[0];
        __syncthreads();
    }
}

// --------------------------------------------------------------------- GAE

// model/gae.metal:14-36: one thread per env, reverse scan over the T slots of
// the slot-major buffers [t * rows + i]; the bootstrap value is column actDim
// of the last forward's head. Operation order as the reference (no FMA).
constexpr int kGaeChunk = 8;

__global__ void k_gae(const float* __restrict__ reward, const uint8_t* __restrict__ done,
                      const float* __restrict__ value, const __nv_bfloat16* __restrict__ bootHead,
                      float* __restrict__ advantage, float* __restrict__ ret, int rows, int horizon, int actDim,
                      float gamma, float lambda) {
    mg_pdl_trigger();
    mg_pdl_wait();
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= rows) return;
    float lastAdv = 0.0f;
    float nextValue = bf(bootHead[(size_t)i * kHeadDim + actDim]);
    const float gl = __fmul_rn(gamma, lambda);
    // slots in chunks of kGaeChunk, newest first: a chunk's loads do not depend
    // on the recurrence, so they are issued together before it runs (the
    // arithmetic, and so every bit, is that of the one-slot-at-a-time scan)
    for (int t = horizon - 1; t >= 0; t -= kGaeChunk) {
        float rw[kGaeChunk], vl[kGaeChunk];
        uint8_t dn[kGaeChunk];
#pragma unroll
        for (int j = 0; j < kGaeChunk; j++) {
            if (t - j < 0) break;
            const size_t k = (size_t)(t - j) * rows + i;
            rw[j] = reward[k];
            vl[j] = value[k];
            dn[j] = done[k];
        }
#pragma unroll
        for (int j = 0; j < kGaeChunk; j++) {
            if (t - j < 0) break;
            const size_t k = (size_t)(t - j) * rows + i;
            const float nonTerminal = dn[j] ? 0.0f : 1.0f;
            const float v = vl[j];
            const float delta = __fsub_rn(__fadd_rn(rw[j], __fmul_rn(__fmul_rn(gamma, nextValue), nonTerminal)), v);
            lastAdv = __fadd_rn(delta, __fmul_rn(__fmul_rn(gl, nonTerminal), lastAdv));
            advantage[k] = lastAdv;
            ret[k] = __fadd_rn(lastAdv, v);
            nextValue = v;
        }
    }
}

// model/gae.metal:42-77 statistics: for minibatch (slot) s, mean and
// inv = 1 / (population std + 1e-8) of adv[s * rows .. s * rows + rows).
__global__ void __launch_bounds__(1024) k_adv_stats(const float* __restrict__ adv, float* __restrict__ out, int rows) {
    mg_pdl_trigger();
    mg_pdl_wait();
    __shared__ float s_part[32];
    __shared__ float s_mean;
    const float* a = adv + (size_t)blockIdx.x * rows;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    float s = 0.0f;
    for (int i = threadIdx.x; i < rows; i += blockDim.x) s = __fadd_rn(s, a[i]);
    s = warp_sum(s);
    if (lane == 0) s_part[warp] = s;
    __syncthreads();
    if (warp == 0) {
        float t = lane < nw ? s_part[lane] : 0.0f;
        t = warp_sum(t);
        if (lane == 0) s_mean = __fdiv_rn(t, (float)rows);
    }
    __syncthreads();
    const float mean = s_mean;
    float q = 0.0f;
    for (int i = threadIdx.x; i < rows; i += blockDim.x) {
        const float d = __fsub_rn(a[i], mean);
        q = __fadd_rn(q, __fmul_rn(d, d));
    }
    q = warp_sum(q);
    __syncthreads();
    if (lane == 0) s_part[warp] = q;
    __syncthreads();
    if (warp == 0) {
        float t = lane < nw ? s_part[lane] : 0.0f;
        t = warp_sum(t);
        if (lane == 0) {
            const float var = __fdiv_rn(t, (float)rows);
            out[2 * blockIdx.x] = mean;
            out[2 * blockIdx.x + 1] = __fdiv_rn(1.0f, __fadd_rn(__fsqrt_rn(var), 1e-8f));
        }
    }
}

// The same statistics over the rows of one row-mode minibatch, gathered
// through its row map: every CTA sums its rows' values and squares in fp64,
// the last CTA to finish adds the CTA sums in index order (deterministic)
// and writes {mean, 1/(std + 1e-8)}.
__global__ void __launch_bounds__(256) k_adv_stats_rows(const float* __restrict__ adv, RowMap rm, int rows,
                                                        float* __restrict__ out, double* __restrict__ part,
                                                        unsigned int* __restrict__ counter) {
    mg_pdl_trigger();
    mg_pdl_wait();
    __shared__ double s_a[8], s_b[8];
    __shared__ bool s_last;
    double a = 0.0, b = 0.0;
    for (int q = blockIdx.x * blockDim.x + threadIdx.x; q < rows; q += gridDim.x * blockDim.x) {
        const double v = adv[mg_minibatch_row(*rm.mb, q, rm.envRows, rm.total)];
        a += v;
        b += v * v;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        a += __shfl_xor_sync(0xffffffffu, a, o);
        b += __shfl_xor_sync(0xffffffffu, b, o);
    }
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (lane == 0) {
        s_a[warp] = a;
        s_b[warp] = b;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        double ta = 0.0, tb = 0.0;
        for (int w = 0; w < (int)(blockDim.x >> 5); w++) {
            ta += s_a[w];
            tb += s_b[w];
        }
        part[2 * blockIdx.x] = ta;
        part[2 * blockIdx.x + 1] = tb;
        __threadfence();
        s_last = atomicAdd(counter, 1u) == gridDim.x - 1;
        if (s_last) {
            __threadfence();
            double sa = 0.0, sb = 0.0;
            for (int k = 0; k < (int)gridDim.x; k++) {
                sa += __ldcg(&part[2 * k]);
                sb += __ldcg(&part[2 * k + 1]);
            }
            const double mean = sa / rows;
            const double var = fmax(sb / rows - mean * mean, 0.0);
            out[0] = (float)mean;
            out[1] = __fdiv_rn(1.0f, __fadd_rn(__fsqrt_rn((float)var), 1e-8f));
            *counter = 0u;  // ready for the next launch
        }
    }
}

// ------------------------------------------------------ gradients and Adam

// Element i of the destination: fp32 at grad[i], or, from element bf16From
// on, packed bf16 after the fp32 elements (the exchange buffer of the
// peer-memory all-reduce, where the bf16-rounded sums travel as bf16).
__device__ __forceinline__ void grad_store(float* grad, int64_t bf16From, int64_t i, float v) {
    if (i < bf16From)
        grad[i] = v;
    else
        reinterpret_cast<__nv_bfloat16*>(grad + bf16From)[i - bf16From] = __float2bfloat16_rn(v);
}

// Virtual block b of the finalisation (k_grad_finalize's CTA b): its
// gradient elements summed over their partials into grad, the block's sum of
// squares into normPartial[b]. Every thread of the CTA calls it. Elements
// from bf16From on are stored packed as bf16 (grad_store); they belong to
// bf16-rounded segments, so the values are exact.
__device__ __forceinline__ void grad_finalize_block(const GradSegmentTable& tab, int b, float* __restrict__ grad,
                                                    float* __restrict__ normPartial, int64_t bf16From) {
    __shared__ float s_red[8];
    int si = 0;
    while (si < tab.n - 1 && b >= tab.seg[si].blockEnd) si++;
    const GradSegment& sg = tab.seg[si];
    const int blockBase = si == 0 ? 0 : tab.seg[si - 1].blockEnd;
    const int64_t st = sg.partStride;
    float sq = 0.0f;
    if (sg.deep) {
        // many partials: 128 elements per CTA, warp w sums partials w, w + 8,
        // ...; warp 0 adds the eight warp sums in warp order
        __shared__ float4 s_dp[8][32];
        const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
        const int64_t i = (int64_t)(b - blockBase) * kGradPerCtaDeep + lane * 4;
        float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        if (i < sg.count) {
            const bool v4 = sg.vec4 && i + 3 < sg.count;
            int p = warp;
            // thirty-two loads in flight per thread while they last (the 256
            // partials of a 4096-row minibatch in one round trip), then
            // sixteen, then four
            for (; p + 248 < sg.nparts && v4; p += 256) {
                float4 v[32];
#pragma unroll
                for (int q = 0; q < 32; q++) v[q] = ld_f4_now(sg.src + (int64_t)(p + 8 * q) * st + i);
#pragma unroll
                for (int q = 0; q < 32; q++) {
                    acc.x = __fadd_rn(acc.x, v[q].x);
                    acc.y = __fadd_rn(acc.y, v[q].y);
                    acc.z = __fadd_rn(acc.z, v[q].z);
                    acc.w = __fadd_rn(acc.w, v[q].w);
                }
            }
            for (; p + 120 < sg.nparts && v4; p += 128) {
                float4 v[16];
#pragma unroll
                for (int q = 0; q < 16; q++) v[q] = ld_f4_now(sg.src + (int64_t)(p + 8 * q) * st + i);
#pragma unroll
                for (int q = 0; q < 16; q++) {
                    acc.x = __fadd_rn(acc.x, v[q].x);
                    acc.y = __fadd_rn(acc.y, v[q].y);
                    acc.z = __fadd_rn(acc.z, v[q].z);
                    acc.w = __fadd_rn(acc.w, v[q].w);
                }
            }
            for (; p + 24 < sg.nparts && v4; p += 32) {
                float4 v[4];
#pragma unroll
                for (int q = 0; q < 4; q++) v[q] = ld_f4_now(sg.src + (int64_t)(p + 8 * q) * st + i);
#pragma unroll
                for (int q = 0; q < 4; q++) {
                    acc.x = __fadd_rn(acc.x, v[q].x);
                    acc.y = __fadd_rn(acc.y, v[q].y);
                    acc.z = __fadd_rn(acc.z, v[q].z);
                    acc.w = __fadd_rn(acc.w, v[q].w);
                }
            }
            for (; p < sg.nparts; p += 8) {
                const float* src = sg.src + (int64_t)p * st + i;
                acc.x = __fadd_rn(acc.x, src[0]);
                if (i + 1 < sg.count) acc.y = __fadd_rn(acc.y, src[1]);
                if (i + 2 < sg.count) acc.z = __fadd_rn(acc.z, src[2]);
                if (i + 3 < sg.count) acc.w = __fadd_rn(acc.w, src[3]);
            }
        }
        s_dp[warp][lane] = acc;
        __syncthreads();
        if (warp == 0 && i < sg.count) {
            float4 t = s_dp[0][lane];
            for (int w = 1; w < 8; w++) {
                const float4 u = s_dp[w][lane];
                t.x = __fadd_rn(t.x, u.x);
                t.y = __fadd_rn(t.y, u.y);
                t.z = __fadd_rn(t.z, u.z);
                t.w = __fadd_rn(t.w, u.w);
            }
            if (sg.roundBf16) t = make_float4(rbf(t.x), rbf(t.y), rbf(t.z), rbf(t.w));
            const float tv[4] = {t.x, t.y, t.z, t.w};
            for (int e = 0; e < 4 && i + e < sg.count; e++) {
                grad_store(grad, bf16From, sg.dstOffset + i + e, tv[e]);
                sq = __fadd_rn(sq, __fmul_rn(tv[e], tv[e]));
            }
        }
    } else if (sg.vec4 && (int64_t)(b - blockBase) * kGradPerCta + threadIdx.x * 4 + 3 < sg.count) {
        // each thread sums 4 consecutive elements over the partials, in increasing p
        const int64_t i = (int64_t)(b - blockBase) * kGradPerCta + threadIdx.x * 4;
        const float* src = sg.src + i;
        float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        int p = 0;
        // thirty-two loads in flight per thread (one round trip to L2 for the
        // 32 tile partials of a 4096-row minibatch), then sixteen, then eight
        for (; p + 32 <= sg.nparts; p += 32) {
            float4 v[32];
#pragma unroll
            for (int q = 0; q < 32; q++) v[q] = ld_f4_now(src + (int64_t)(p + q) * st);
#pragma unroll
            for (int q = 0; q < 32; q++) {
                acc.x = __fadd_rn(acc.x, v[q].x);
                acc.y = __fadd_rn(acc.y, v[q].y);
                acc.z = __fadd_rn(acc.z, v[q].z);
                acc.w = __fadd_rn(acc.w, v[q].w);
            }
        }
        for (; p + 16 <= sg.nparts; p += 16) {
            float4 v[16];
#pragma unroll
            for (int q = 0; q < 16; q++) v[q] = ld_f4_now(src + (int64_t)(p + q) * st);
#pragma unroll
            for (int q = 0; q < 16; q++) {
                acc.x = __fadd_rn(acc.x, v[q].x);
                acc.y = __fadd_rn(acc.y, v[q].y);
                acc.z = __fadd_rn(acc.z, v[q].z);
                acc.w = __fadd_rn(acc.w, v[q].w);
            }
        }
        for (; p + 8 <= sg.nparts; p += 8) {
            float4 v[8];
#pragma unroll
            for (int q = 0; q < 8; q++) v[q] = ld_f4_now(src + (int64_t)(p + q) * st);
#pragma unroll
            for (int q = 0; q < 8; q++) {
                acc.x = __fadd_rn(acc.x, v[q].x);
                acc.y = __fadd_rn(acc.y, v[q].y);
                acc.z = __fadd_rn(acc.z, v[q].z);
                acc.w = __fadd_rn(acc.w, v[q].w);
            }
        }
        for (; p < sg.nparts; p++) {
            const float4 v = *reinterpret_cast<const float4*>(src + (int64_t)p * st);
            acc.x = __fadd_rn(acc.x, v.x);
            acc.y = __fadd_rn(acc.y, v.y);
            acc.z = __fadd_rn(acc.z, v.z);
            acc.w = __fadd_rn(acc.w, v.w);
        }
        if (sg.roundBf16) acc = make_float4(rbf(acc.x), rbf(acc.y), rbf(acc.z), rbf(acc.w));
        if (sg.dstOffset + i < bf16From) {
            *reinterpret_cast<float4*>(grad + sg.dstOffset + i) = acc;
        } else {  // four packed bf16 (8 bytes: bf16From and the offset are multiples of 4)
            const __nv_bfloat162 lo = __floats2bfloat162_rn(acc.x, acc.y), hi = __floats2bfloat162_rn(acc.z, acc.w);
            *reinterpret_cast<uint2*>(reinterpret_cast<__nv_bfloat16*>(grad + bf16From) + (sg.dstOffset + i - bf16From)) =
                make_uint2(*reinterpret_cast<const uint32_t*>(&lo), *reinterpret_cast<const uint32_t*>(&hi));
        }
        sq = __fadd_rn(__fadd_rn(__fmul_rn(acc.x, acc.x), __fmul_rn(acc.y, acc.y)),
                       __fadd_rn(__fmul_rn(acc.z, acc.z), __fmul_rn(acc.w, acc.w)));
    } else {
        const int64_t i = (int64_t)(b - blockBase) * kGradPerCta + threadIdx.x * 4;
        for (int e = 0; e < 4; e++) {
            if (i + e >= sg.count) break;
            const float* src = sg.src + i + e;
            float acc = 0.0f;
            for (int p = 0; p < sg.nparts; p++) acc = __fadd_rn(acc, src[(int64_t)p * st]);
            if (sg.roundBf16) acc = rbf(acc);
            grad_store(grad, bf16From, sg.dstOffset + i + e, acc);
            sq = __fadd_rn(sq, __fmul_rn(acc, acc));
        }
    }
    sq = warp_sum(sq);
    if ((threadIdx.x & 31) == 0) s_red[threadIdx.x >> 5] = sq;
    __syncthreads();
    if (threadIdx.x == 0) {
        float t = 0.0f;
        for (int w = 0; w < 8; w++) t = __fadd_rn(t, s_red[w]);
        normPartial[b] = t;
    }
}

// Sums the partials of every gradient segment into the flat fp32 gradient
// arena (model/elementwise.metal:21-31 for the GEMM weights, whose sum is
// rounded to bf16 as the reference's bf16 gradient arena stores it; the
// LayerNorm / input / log-std sums stay fp32) and writes one partial sum of
// squares per CTA for the global norm (model/optimizer.metal:23-34).
__global__ void __launch_bounds__(256) k_grad_finalize(const __grid_constant__ GradSegmentTable tab,
                                                       float* gradA, float* gradB, const unsigned int* sel,
                                                       float* __restrict__ normPartial,
                                                       unsigned int* __restrict__ counter,
                                                       float* __restrict__ normSqOut, int64_t bf16From,
                                                       bool earlyOk) {
    mg_pdl_trigger();
    // a CTA of a segment whose partials were written before the preceding
    // kernel runs beside that kernel (earlyOk: it signalled this launch only
    // after every kernel before it had completed); the others wait for it
    bool wait = true;
    if (earlyOk) {
        int si = 0;
        while (si < tab.n - 1 && (int)blockIdx.x >= tab.seg[si].blockEnd) si++;
        wait = !tab.seg[si].early;
    }
    if (wait) mg_pdl_wait();
    // with sel (the peer all-reduce's minibatch counter): gradB when the next
    // count is odd, else gradA; without it: gradA
    float* __restrict__ grad = (sel && ((*sel + 1u) & 1u)) ? gradB : gradA;
    __shared__ float s_red[8];
    __shared__ bool s_last;
    grad_finalize_block(tab, blockIdx.x, grad, normPartial, bf16From);
    if (threadIdx.x == 0) {
        s_last = false;
        if (counter) {
            __threadfence();
            s_last = atomicAdd(counter, 1u) == gridDim.x - 1;
        }
    }
    __syncthreads();
    // the last CTA to finish sums every CTA's partial in index order
    if (counter && s_last) {
        __threadfence();
        float t = 0.0f;
        for (int k = threadIdx.x; k < (int)gridDim.x; k += 256) t = __fadd_rn(t, __ldcg(&normPartial[k]));
        t = warp_sum(t);
        if ((threadIdx.x & 31) == 0) s_red[threadIdx.x >> 5] = t;
        __syncthreads();
        if (threadIdx.x == 0) {
            float u = 0.0f;
            for (int w = 0; w < 8; w++) u = __fadd_rn(u, s_red[w]);
            *normSqOut = u;
            *counter = 0u;  // ready for the next launch
        }
    }
}

// Sum of squares of grad[0..count) in fixed-size CTA partials (used after a
// cross-GPU all-reduce, which also rescales the sum to a mean).
__global__ void __launch_bounds__(256) k_grad_scale_norm(float* __restrict__ grad, int64_t count, float scale,
                                                         float* __restrict__ normPartial,
                                                         unsigned int* __restrict__ counter,
                                                         float* __restrict__ normSqOut) {
    mg_pdl_trigger();
    mg_pdl_wait();
    __shared__ float s_red[8];
    float sq = 0.0f;
    const int64_t i0 = (int64_t)blockIdx.x * 1024;
    for (int j = 0; j < 4; j++) {
        const int64_t i = i0 + j * 256 + threadIdx.x;
        if (i < count) {
            const float g = __fmul_rn(grad[i], scale);
            grad[i] = g;
            sq = __fadd_rn(sq, __fmul_rn(g, g));
        }
    }
    sq = warp_sum(sq);
    if ((threadIdx.x & 31) == 0) s_red[threadIdx.x >> 5] = sq;
    __syncthreads();
    __shared__ bool s_last;
    if (threadIdx.x == 0) {
        float t = 0.0f;
        for (int w = 0; w < 8; w++) t = __fadd_rn(t, s_red[w]);
        normPartial[blockIdx.x] = t;
        s_last = false;
        if (counter) {
            __threadfence();
            s_last = atomicAdd(counter, 1u) == gridDim.x - 1;
        }
    }
    __syncthreads();
    if (counter && s_last) {
        __threadfence();
        float t = 0.0f;
        for (int k = threadIdx.x; k < (int)gridDim.x; k += 256) t = __fadd_rn(t, __ldcg(&normPartial[k]));
        t = warp_sum(t);
        if ((threadIdx.x & 31) == 0) s_red[threadIdx.x >> 5] = t;
        __syncthreads();
        if (threadIdx.x == 0) {
            float u = 0.0f;
            for (int w = 0; w < 8; w++) u = __fadd_rn(u, s_red[w]);
            *normSqOut = u;
            *counter = 0u;
        }
    }
}

// model/optimizer.metal:36-60 for one element: gRaw the unclipped gradient,
// `scale` the clip factor, c1 = 1 - beta1^t, c2 = 1 - beta2^t; m, v, x the
// moments and the master weight, updated in place.
__device__ __forceinline__ void adam_math(float gRaw, float scale, float lr, float c1, float c2, float& m, float& v,
                                          float& x) {
    const float b1 = 0.9f, b2 = 0.999f, eps = 1e-8f;
    const float g = __fmul_rn(gRaw, scale);
    m = __fadd_rn(__fmul_rn(b1, m), __fmul_rn(__fsub_rn(1.0f, b1), g));
    v = __fadd_rn(__fmul_rn(b2, v), __fmul_rn(__fmul_rn(__fsub_rn(1.0f, b2), g), g));
    const float mHat = __fdiv_rn(m, c1);
    const float vHat = __fdiv_rn(v, c2);
    x = __fsub_rn(x, __fdiv_rn(__fmul_rn(lr, mHat), __fadd_rn(__fsqrt_rn(vHat), eps)));
}

// model/optimizer.metal:36-60 with the host bias-correction powers of
// model/ppo.h:879-880 (from betaPow[0..1] if given, else the scalars).
// Every CTA first sums the norm partials in the same order, so all agree.
// model/optimizer.metal:36-60 on elements i0, i0 + stride, .. of [0, count),
// the gradient scaled by the clip factor.
__device__ __forceinline__ void adam_range(float* __restrict__ param, const float* __restrict__ grad,
                                           float* __restrict__ mom, float* __restrict__ var,
                                           __nv_bfloat16* __restrict__ weights, int64_t count, const AdamHyper& hp,
                                           const float* __restrict__ betaPow, float scale, int64_t i0, int64_t stride) {
    const float b1p = betaPow ? betaPow[0] : hp.beta1Pow;
    const float b2p = betaPow ? betaPow[1] : hp.beta2Pow;
    const float c1 = __fsub_rn(1.0f, b1p), c2 = __fsub_rn(1.0f, b2p);
    for (int64_t i = i0; i < count; i += stride) {
        float m = mom[i], v = var[i], x = param[i];
        adam_math(grad[i], scale, hp.lr, c1, c2, m, v, x);
        mom[i] = m;
        var[i] = v;
        param[i] = x;
        weights[i] = tobf(x);
    }
}

__global__ void __launch_bounds__(256) k_adam(float* __restrict__ param, const float* __restrict__ grad,
                                              float* __restrict__ mom, float* __restrict__ var,
                                              __nv_bfloat16* __restrict__ weights,
                                              const float* __restrict__ normPartial, int nNorm, int64_t count,
                                              AdamHyper hp, const float* __restrict__ betaPow,
                                              float* __restrict__ normSqOut, const float* __restrict__ normSqIn) {
    mg_pdl_trigger();
    mg_pdl_wait();
    __shared__ float s_scale;
    // the first element's operands and the bias corrections in flight while
    // the clip factor is formed (one memory round trip instead of two)
    const int64_t i0 = (int64_t)blockIdx.x * blockDim.x + threadIdx.x, stride = (int64_t)gridDim.x * blockDim.x;
    float g0 = 0.0f, m0 = 0.0f, v0 = 0.0f, x0 = 0.0f;
    if (i0 < count) {
        g0 = grad[i0];
        m0 = mom[i0];
        v0 = var[i0];
        x0 = param[i0];
    }
    const float c1 = __fsub_rn(1.0f, betaPow ? betaPow[0] : hp.beta1Pow);
    const float c2 = __fsub_rn(1.0f, betaPow ? betaPow[1] : hp.beta2Pow);
    if (threadIdx.x < 32) {
        float s = 0.0f;
        if (normSqIn) {
            s = *normSqIn;
        } else {
            for (int i = threadIdx.x; i < nNorm; i += 32) s = __fadd_rn(s, normPartial[i]);
            s = warp_sum(s);
        }
        if (threadIdx.x == 0) {
            const float norm = __fsqrt_rn(s);
            s_scale = (hp.maxGradNorm > 0.0f && norm > hp.maxGradNorm)
                          ? __fdiv_rn(hp.maxGradNorm, __fadd_rn(norm, 1e-6f))
                          : 1.0f;
            if (blockIdx.x == 0 && normSqOut && !normSqIn) *normSqOut = s;
        }
    }
    __syncthreads();
    if (i0 < count) {
        adam_math(g0, s_scale, hp.lr, c1, c2, m0, v0, x0);
        mom[i0] = m0;
        var[i0] = v0;
        param[i0] = x0;
        weights[i0] = tobf(x0);
    }
    adam_range(param, grad, mom, var, weights, count, hp, betaPow, s_scale, i0 + stride, stride);
}

// LossStats (model/ppo.h:925-943): column means of the rows x 5 stats.
__global__ void __launch_bounds__(256) k_stats_mean(const float* __restrict__ stats, int rows, float* __restrict__ out) {
    mg_pdl_trigger();
    mg_pdl_wait();
    __shared__ float s_red[8][5];
    float acc[5] = {0, 0, 0, 0, 0};
    for (int r = threadIdx.x; r < rows; r += blockDim.x)
        for (int k = 0; k < 5; k++) acc[k] = __fadd_rn(acc[k], stats[(size_t)r * 5 + k]);
    for (int k = 0; k < 5; k++) {
        const float s = warp_sum(acc[k]);
        if ((threadIdx.x & 31) == 0) s_red[threadIdx.x >> 5][k] = s;
    }
    __syncthreads();
    if (threadIdx.x < 5) {
        float t = 0.0f;
        for (int w = 0; w < 8; w++) t = __fadd_rn(t, s_red[w][threadIdx.x]);
        out[threadIdx.x] = __fmul_rn(t, __fdiv_rn(1.0f, (float)rows));
    }
}

int grid_rows(int rows, int rowsPerCta) { return (rows + rowsPerCta - 1) / rowsPerCta; }

}  // namespace

// ------------------------------------------------------------ host launchers

int input_forward(const float* obs, const void* w, const void* b, void* out, int rows, int inDim, int outDim,
                  cudaStream_t st, RowMap rm, const LnOutputs* ln) {
    MG_CHECK_ARG(rows > 0 && inDim > 0 && outDim % 64 == 0 && outDim <= 1024, "input_forward: bad shape");
    MG_CHECK_ARG(inDim * outDim * 4 <= 160 * 1024, "input_forward: weight too large for shared memory");
    auto W = static_cast<const __nv_bfloat16*>(w);
    auto B = static_cast<const __nv_bfloat16*>(b);
    auto O = static_cast<__nv_bfloat16*>(out);
    const LnOutputs lno = ln ? *ln : LnOutputs{};
#define MG_IN_FWD(V, RPW)                                                                                     \
    case V: {                                                                                                 \
        const size_t sm = ((size_t)inDim * outDim + 8 * RPW * inDim) * 4 + (ln ? (size_t)8 * RPW * outDim * 2 : 0); \
        const int blocks = std::min(grid_rows(rows, 8 * RPW), 148 * 4);                                       \
        auto kern = ln ? &k_input_forward<V, RPW, true> : &k_input_forward<V, RPW, false>;                    \
        if (sm > 48 * 1024)                                                                                   \
            MG_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm));    \
        MG_LAUNCH(kern, blocks, 256, sm, st, obs, W, B, O, rows, inDim, outDim, rm, lno);                     \
        break;                                                                                                \
    }
    switch (outDim / 32) {
        MG_IN_FWD(2, 4) MG_IN_FWD(4, 4) MG_IN_FWD(8, 4) MG_IN_FWD(16, 2) MG_IN_FWD(32, 1)
        default: return fail(MG_ERR_ARGUMENT, "input_forward: out_dim must be 64, 128, 256, 512 or 1024");
    }
#undef MG_IN_FWD
    return check_launch("k_input_forward");
}

// Rows per CTA of the input backward: at least 16, a multiple of 8, enough
// to keep the partial sums at kMaxRowParts or fewer and within
// kInputPartialBudget bytes, as far as kInputSmemBudget bytes of staged rows
// allow.
static int input_rows_per_cta(int rows, int inDim, int outDim) {
    const int64_t perPart = (int64_t)(inDim + 1) * outDim * 4;
    const int64_t maxParts = std::max<int64_t>(1, std::min<int64_t>(kMaxRowParts, kInputPartialBudget / perPart));
    const int perRowSmem = inDim * 4 + outDim * 2 + 8;
    const int maxRpc = std::max(8, (int)(kInputSmemBudget / perRowSmem) / 8 * 8);
    int rpc = std::max<int64_t>(16, (rows + maxParts - 1) / maxParts);
    rpc = (rpc + 7) / 8 * 8;
    return std::min(rpc, maxRpc);
}

int input_backward_parts(int rows, int inDim, int outDim) {
    return grid_rows(rows, input_rows_per_cta(rows, inDim, outDim));
}

int input_backward(const float* obs, const void* dZ, float* partial, int rows, int inDim, int outDim,
                   cudaStream_t st, RowMap rm) {
    MG_CHECK_ARG(rows > 0 && inDim > 0 && inDim <= 256 && outDim > 0 && outDim <= 1024 && outDim % 8 == 0,
                 "input_backward: bad shape");
    MG_CHECK_ARG((reinterpret_cast<uintptr_t>(dZ) & 15) == 0, "input_backward: dZ must be 16-byte aligned");
    const int rpc = input_rows_per_cta(rows, inDim, outDim);
    // observations, dZ rows, the rows' rollout indices (8-byte aligned: rows per
    // CTA a multiple of 8, outDim % 8 == 0)
    const size_t sm = (size_t)rpc * inDim * 4 + (size_t)rpc * outDim * 2 + (size_t)rpc * 8;
    MG_CHECK_ARG(sm <= 200 * 1024, "input_backward: rows per CTA x widths too large for shared memory");
    const auto* DZ = static_cast<const __nv_bfloat16*>(dZ);
    const int blocks = grid_rows(rows, rpc), threads = std::min(outDim, 256);
    // the register-accumulator kernel for the observation widths of the
    // built-in environments and their kin (rows outer), else the chunked one
    auto regs = [&](auto kern) -> int {
        if (sm > 48 * 1024) MG_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm));
        MG_LAUNCH(kern, blocks, threads, sm, st, obs, DZ, partial, rows, inDim, outDim, rpc, rm);
        return check_launch("k_input_backward_regs");
    };
    const bool v4 = inDim % 4 == 0;
    if (inDim <= 8) return v4 ? regs(k_input_backward_regs<8, true>) : regs(k_input_backward_regs<8, false>);
    if (inDim <= 16) return v4 ? regs(k_input_backward_regs<16, true>) : regs(k_input_backward_regs<16, false>);
    if (inDim <= 48) return v4 ? regs(k_input_backward_regs<48, true>) : regs(k_input_backward_regs<48, false>);
    if (sm > 48 * 1024)
        MG_CUDA_TRY(cudaFuncSetAttribute(k_input_backward, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm));
    MG_LAUNCH(k_input_backward, blocks, threads, sm, st, obs, DZ, partial, rows, inDim, outDim, rpc, rm);
    return check_launch("k_input_backward");
}

int layernorm_forward(const void* x, void* xNorm, void* out, const void* gamma, const void* beta, float* stdev,
                      int rows, int cols, cudaStream_t st) {
    MG_CHECK_ARG(rows > 0, "layernorm_forward: rows must be > 0");
    const int blocks = std::min(grid_rows(rows, 8), 148 * 16);
    auto X = static_cast<const __nv_bfloat16*>(x);
    auto XN = static_cast<__nv_bfloat16*>(xNorm);
    auto Y = static_cast<__nv_bfloat16*>(out);
    auto G = static_cast<const __nv_bfloat16*>(gamma);
    auto Bt = static_cast<const __nv_bfloat16*>(beta);
    switch (cols) {
        case 64: MG_LAUNCH(k_layernorm_forward<2>, blocks, 256, 0, st, X, XN, Y, G, Bt, stdev, rows); break;
        case 128: MG_LAUNCH(k_layernorm_forward<4>, blocks, 256, 0, st, X, XN, Y, G, Bt, stdev, rows); break;
        case 256: MG_LAUNCH(k_layernorm_forward<8>, blocks, 256, 0, st, X, XN, Y, G, Bt, stdev, rows); break;
        case 512: MG_LAUNCH(k_layernorm_forward<16>, blocks, 256, 0, st, X, XN, Y, G, Bt, stdev, rows); break;
        case 1024: MG_LAUNCH(k_layernorm_forward<32>, blocks, 256, 0, st, X, XN, Y, G, Bt, stdev, rows); break;
        default: return fail(MG_ERR_ARGUMENT, "layernorm: cols must be 64, 128, 256, 512 or 1024");
    }
    return check_launch("k_layernorm_forward");
}

// Rows per CTA of the LayerNorm backward: a multiple of 8 (one row per warp
// at a time) that keeps the partial sums at kMaxRowParts or fewer.
static int ln_rows_per_cta(int rows) {
    const int rpc = std::max(8, (rows + kMaxRowParts - 1) / kMaxRowParts);
    return (rpc + 7) / 8 * 8;
}

int layernorm_backward_parts(int rows) { return grid_rows(rows, ln_rows_per_cta(rows)); }
int layernorm_rows_per_part(int rows) { return ln_rows_per_cta(rows); }

int layernorm_backward(void* dZ, const void* xNorm, const void* gamma, const float* stdev, const void* resid,
                       float* partial, int rows, int cols, cudaStream_t st, void* residOut) {
    MG_CHECK_ARG(rows > 0, "layernorm_backward: rows must be > 0");
    const int rpc = ln_rows_per_cta(rows);
    const int blocks = grid_rows(rows, rpc);
    auto DZ = static_cast<__nv_bfloat16*>(dZ);
    auto XN = static_cast<const __nv_bfloat16*>(xNorm);
    auto G = static_cast<const __nv_bfloat16*>(gamma);
    auto R = static_cast<const __nv_bfloat16*>(resid);
    auto RO = static_cast<__nv_bfloat16*>(residOut ? residOut : const_cast<void*>(resid));
    switch (cols) {
        case 64: MG_LAUNCH(k_layernorm_backward<2>, blocks, 256, 0, st, DZ, XN, G, stdev, R, RO, partial, rows, rpc); break;
        case 128: MG_LAUNCH(k_layernorm_backward<4>, blocks, 256, 0, st, DZ, XN, G, stdev, R, RO, partial, rows, rpc); break;
        case 256: MG_LAUNCH(k_layernorm_backward<8>, blocks, 256, 0, st, DZ, XN, G, stdev, R, RO, partial, rows, rpc); break;
        case 512: MG_LAUNCH(k_layernorm_backward<16>, blocks, 256, 0, st, DZ, XN, G, stdev, R, RO, partial, rows, rpc); break;
        default: return fail(MG_ERR_ARGUMENT, "layernorm_backward: cols must be 64, 128, 256 or 512");
    }
    return check_launch("k_layernorm_backward");
}

int sample_categorical(const void* head, uint32_t* rng, int32_t* action, float* logProb, float* value, int rows,
                       int actDim, cudaStream_t st) {
    MG_CHECK_ARG(rows > 0 && actDim >= 1 && actDim < kHeadDim, "sample_categorical: bad shape");
    MG_LAUNCH(k_sample_categorical, grid_rows(rows, 256), 256, 0, st, static_cast<const __nv_bfloat16*>(head), rng, action,
                                                                logProb, value, rows, actDim);
    return check_launch("k_sample_categorical");
}

int sample_gaussian(const void* head, const void* logStd, uint32_t* rng, float* action, float* logProb,
                    float* value, int rows, int actDim, cudaStream_t st) {
    MG_CHECK_ARG(rows > 0 && actDim >= 1 && actDim < kHeadDim, "sample_gaussian: bad shape");
    MG_LAUNCH(k_sample_gaussian, grid_rows(rows, 256), 256, 0, st, static_cast<const __nv_bfloat16*>(head),
                                                             static_cast<const __nv_bfloat16*>(logStd), rng, action,
                                                             logProb, value, rows, actDim);
    return check_launch("k_sample_gaussian");
}

PolicyLossRows policy_loss_rows(const int32_t* action, const float* adv, const float* advStats, const float* ret,
                                const float* oldLogProb, void* dZ, float* stats, int rows, int actDim, LossHyper hp,
                                RowMap rm) {
    PolicyLossRows L{};
    L.action = action;
    L.adv = adv;
    L.advStats = advStats;
    L.ret = ret;
    L.oldLogProb = oldLogProb;
    L.dZ = static_cast<__nv_bfloat16*>(dZ);
    L.stats = stats;
    L.mb = rm.mb;
    L.envRows = rm.envRows;
    L.total = rm.total;
    L.rows = rows;
    L.actDim = actDim;
    L.clip = hp.clip;
    L.valueCoef = hp.valueCoef;
    L.entropyCoef = hp.entropyCoef;
    return L;
}

int policy_loss(const void* head, const int32_t* action, const float* adv, const float* advStats, const float* ret,
                const float* oldLogProb, void* dZ, float* stats, int rows, int actDim, LossHyper hp,
                cudaStream_t st, RowMap rm) {
    MG_CHECK_ARG(rows > 0 && actDim >= 1 && actDim < kHeadDim, "policy_loss: bad shape");
    const PolicyLossRows L = policy_loss_rows(action, adv, advStats, ret, oldLogProb, dZ, stats, rows, actDim, hp, rm);
    MG_LAUNCH(k_policy_loss, grid_rows(rows, 64), 64, 0, st, static_cast<const __nv_bfloat16*>(head), L, status_ptr());
    return check_launch("k_policy_loss");
}

int gaussian_loss_parts(int rows) { return grid_rows(rows, kGaussRowsPerCta); }

int gaussian_loss(const void* head, const float* action, const float* adv, const float* advStats, const float* ret,
                  const float* oldLogProb, void* dZ, float* stats, const void* logStd, float* partial, int rows,
                  int actDim, LossHyper hp, cudaStream_t st, RowMap rm) {
    MG_CHECK_ARG(rows > 0 && actDim >= 1 && actDim < kHeadDim, "gaussian_loss: bad shape");
    MG_LAUNCH(k_gaussian_loss, gaussian_loss_parts(rows), kGaussRowsPerCta, 0, st, 
        static_cast<const __nv_bfloat16*>(head), action, adv, advStats, ret, oldLogProb,
        static_cast<__nv_bfloat16*>(dZ), stats, static_cast<const __nv_bfloat16*>(logStd), partial, rows, actDim, hp,
        rm);
    return check_launch("k_gaussian_loss");
}

int gae(const float* reward, const uint8_t* done, const float* value, const void* bootHead, float* adv, float* ret,
        int rows, int horizon, int actDim, float gamma, float lambda, cudaStream_t st) {
    MG_CHECK_ARG(rows > 0 && horizon > 0, "gae: bad shape");
    MG_LAUNCH(k_gae, grid_rows(rows, 128), 128, 0, st, reward, done, value, static_cast<const __nv_bfloat16*>(bootHead), adv,
                                                 ret, rows, horizon, actDim, gamma, lambda);
    return check_launch("k_gae");
}

int advantage_stats_rows(const float* adv, RowMap rm, int rows, float* out, double* partial,
                         unsigned int* counter, cudaStream_t st) {
    MG_CHECK_ARG(rm.mb && rows > 0 && partial && counter, "advantage_stats_rows: needs a row map and scratch");
    const int blocks = std::min(kAdvStatsMaxCtas, (rows + 255) / 256);
    MG_LAUNCH(k_adv_stats_rows, blocks, 256, 0, st, adv, rm, rows, out, partial, counter);
    return check_launch("k_adv_stats_rows");
}

int advantage_stats(const float* adv, float* out, int rows, int slots, cudaStream_t st) {
    MG_CHECK_ARG(rows > 0 && slots > 0, "advantage_stats: bad shape");
    MG_LAUNCH(k_adv_stats, slots, 1024, 0, st, adv, out, rows);
    return check_launch("k_adv_stats");
}

int grad_table_layout(GradSegmentTable& tab, bool allowDeep) {
    int b = 0;
    for (int i = 0; i < tab.n; i++) {
        GradSegment& g = tab.seg[i];
        g.deep = allowDeep && g.nparts > kGradDeepParts ? 1 : 0;
        const int per = g.deep ? kGradPerCtaDeep : kGradPerCta;
        b += (int)((g.count + per - 1) / per);
        g.blockEnd = b;
    }
    return b;
}

int grad_finalize(const GradSegmentTable& table, float* grad, float* normPartial, cudaStream_t st,
                  unsigned int* counter, float* normSqOut, float* grad2, const unsigned int* sel, int64_t bf16From,
                  bool earlyOk) {
    MG_CHECK_ARG(table.n > 0 && table.n <= kMaxGradSegments, "grad_finalize: bad segment count");
    const int nblocks = table.seg[table.n - 1].blockEnd;
    MG_CHECK_ARG(nblocks > 0, "grad_finalize: empty");
    // 16-byte loads and stores where every address of the segment allows them
    GradSegmentTable tab = table;
    for (int k = 0; k < tab.n; k++) {
        GradSegment& g = tab.seg[k];
        g.vec4 = (reinterpret_cast<uintptr_t>(g.src) % 16 == 0) && g.partStride % 4 == 0 && g.dstOffset % 4 == 0 &&
                 (reinterpret_cast<uintptr_t>(grad) % 16 == 0);
    }
    if (bf16From != INT64_MAX) {
        MG_CHECK_ARG(bf16From % 4 == 0, "grad_finalize: the bf16 part must start at a multiple of 4 elements");
        for (int k = 0; k < tab.n; k++)
            MG_CHECK_ARG(tab.seg[k].dstOffset + tab.seg[k].count <= bf16From ||
                             (tab.seg[k].roundBf16 && tab.seg[k].dstOffset >= bf16From),
                         "grad_finalize: only bf16-rounded segments may lie in the bf16 part");
    }
    MG_LAUNCH(k_grad_finalize, nblocks, 256, 0, st, tab, grad, grad2, sel, normPartial, counter, normSqOut, bf16From,
              earlyOk);
    return check_launch("k_grad_finalize");
}

int grad_scale_norm_blocks(int64_t count) { return (int)((count + 1023) / 1024); }

int grad_scale_norm(float* grad, int64_t count, float scale, float* normPartial, cudaStream_t st,
                    unsigned int* counter, float* normSqOut) {
    MG_LAUNCH(k_grad_scale_norm, grad_scale_norm_blocks(count), 256, 0, st, grad, count, scale, normPartial, counter,
              normSqOut);
    return check_launch("k_grad_scale_norm");
}

int adam(float* param, const float* grad, float* mom, float* var, void* weights, const float* normPartial, int nNorm,
         int64_t count, AdamHyper hp, const float* betaPow, float* normSqOut, cudaStream_t st, const float* normSqIn) {
    MG_CHECK_ARG(count > 0 && (nNorm > 0 || normSqIn), "adam: bad shape");
    const int blocks = (int)std::min<int64_t>((count + 255) / 256, 148 * 8);
    MG_LAUNCH(k_adam, blocks, 256, 0, st, param, grad, mom, var, static_cast<__nv_bfloat16*>(weights), normPartial, nNorm,
                                   count, hp, betaPow, normSqOut, normSqIn);
    return check_launch("k_adam");
}

int stats_mean(const float* stats, int rows, float* out, cudaStream_t st) {
    MG_LAUNCH(k_stats_mean, 1, 256, 0, st, stats, rows, out);
    return check_launch("k_stats_mean");
}

// actGreedy (model/ppo.h:688-702) on the device, one thread per row of the
// head [rows][64] (bf16): a categorical head's action is the index of the
// largest logit (the first of equal ones: the reference's strict >), a
// Gaussian head's the ACT_DIM means as floats.
__global__ void k_act_greedy(const __nv_bfloat16* __restrict__ head, int rows, int actDim, int continuous,
                             void* __restrict__ actions) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= rows) return;
    const __nv_bfloat16* h = head + (size_t)i * kHeadDim;
    if (continuous) {
        float* a = static_cast<float*>(actions) + (size_t)i * actDim;
        for (int k = 0; k < actDim; k++) a[k] = bf(h[k]);
    } else {
        int best = 0;
        for (int a = 1; a < actDim; a++)
            if (bf(h[a]) > bf(h[best])) best = a;
        static_cast<int32_t*>(actions)[i] = best;
    }
}

int act_greedy(const void* head, int rows, int actDim, bool continuous, void* actions, cudaStream_t st) {
    MG_CHECK_ARG(head && actions && rows > 0 && actDim >= 1 && actDim < kHeadDim, "act_greedy: bad arguments");
    MG_LAUNCH(k_act_greedy, grid_rows(rows, 256), 256, 0, st, static_cast<const __nv_bfloat16*>(head), rows, actDim,
              continuous ? 1 : 0, actions);
    return check_launch("k_act_greedy");
}

}  // namespace mg

// ------------------------------------------------------------------ C ABI

using mg::LossHyper;
using mg::AdamHyper;

#define MG_STREAM(s) reinterpret_cast<cudaStream_t>(s)

extern "C" {

int mg_input_forward(const float* obs, const void* w, const void* b, void* out, int rows, int in_dim, int out_dim,
                     mg_stream_t s) {
    MG_CHECK_ARG(obs && w && b && out, "input_forward: null argument");
    return mg::input_forward(obs, w, b, out, rows, in_dim, out_dim, MG_STREAM(s));
}

int mg_input_forward_layernorm(const float* obs, const void* w, const void* b, void* out, const void* gamma,
                               const void* beta, void* x_norm, void* ln_out, float* stdev, int rows, int in_dim,
                               int out_dim, mg_stream_t s) {
    MG_CHECK_ARG(obs && w && b && out, "input_forward_layernorm: null argument");
    MG_CHECK_ARG(gamma && beta && x_norm && ln_out && stdev, "input_forward_layernorm: null LayerNorm argument");
    mg::LnOutputs ln{static_cast<const __nv_bfloat16*>(gamma), static_cast<const __nv_bfloat16*>(beta),
                     static_cast<__nv_bfloat16*>(x_norm), static_cast<__nv_bfloat16*>(ln_out), stdev};
    return mg::input_forward(obs, w, b, out, rows, in_dim, out_dim, MG_STREAM(s), mg::RowMap{nullptr, 0, 0}, &ln);
}

int mg_input_backward_partials(const float* obs, const void* dZ, float* partial, int rows, int in_dim, int out_dim,
                               mg_stream_t s) {
    MG_CHECK_ARG(obs && dZ && partial, "input_backward: null argument");
    return mg::input_backward(obs, dZ, partial, rows, in_dim, out_dim, MG_STREAM(s));
}

int mg_input_backward_num_partials(int rows, int in_dim, int out_dim) {
    return mg::input_backward_parts(rows, in_dim, out_dim);
}

int mg_layernorm_forward(const void* x, void* x_norm, void* out, const void* gamma, const void* beta, float* stdev,
                         int rows, int cols, mg_stream_t s) {
    MG_CHECK_ARG(x && x_norm && out && gamma && beta && stdev, "layernorm_forward: null argument");
    return mg::layernorm_forward(x, x_norm, out, gamma, beta, stdev, rows, cols, MG_STREAM(s));
}

int mg_layernorm_backward(void* dZ, const void* x_norm, const void* gamma, const float* stdev, void* resid,
                          float* partial, int rows, int cols, mg_stream_t s) {
    MG_CHECK_ARG(dZ && x_norm && gamma && stdev && partial, "layernorm_backward: null argument");
    return mg::layernorm_backward(dZ, x_norm, gamma, stdev, resid, partial, rows, cols, MG_STREAM(s));
}

int mg_layernorm_backward_num_partials(int rows) { return mg::layernorm_backward_parts(rows); }

int mg_sample_categorical(const void* head, uint32_t* rng, int32_t* action, float* log_prob, float* value, int rows,
                          int act_dim, mg_stream_t s) {
    MG_CHECK_ARG(head && rng && action && log_prob && value, "sample_categorical: null argument");
    return mg::sample_categorical(head, rng, action, log_prob, value, rows, act_dim, MG_STREAM(s));
}

int mg_sample_gaussian(const void* head, const void* log_std, uint32_t* rng, float* action, float* log_prob,
                       float* value, int rows, int act_dim, mg_stream_t s) {
    MG_CHECK_ARG(head && log_std && rng && action && log_prob && value, "sample_gaussian: null argument");
    return mg::sample_gaussian(head, log_std, rng, action, log_prob, value, rows, act_dim, MG_STREAM(s));
}

int mg_policy_loss(const void* head, const int32_t* action, const float* adv, const float* adv_stats,
                   const float* ret, const float* old_log_prob, void* dZ, float* stats, int rows, int act_dim,
                   float clip, float value_coef, float entropy_coef, mg_stream_t s) {
    MG_CHECK_ARG(head && action && adv && ret && old_log_prob && dZ && stats, "policy_loss: null argument");
    LossHyper hp{clip, value_coef, entropy_coef};
    return mg::policy_loss(head, action, adv, adv_stats, ret, old_log_prob, dZ, stats, rows, act_dim, hp,
                           MG_STREAM(s));
}

int mg_gaussian_loss(const void* head, const float* action, const float* adv, const float* adv_stats,
                     const float* ret, const float* old_log_prob, void* dZ, float* stats, const void* log_std,
                     float* dlogstd_partial, int rows, int act_dim, float clip, float value_coef, float entropy_coef,
                     mg_stream_t s) {
    MG_CHECK_ARG(head && action && adv && ret && old_log_prob && dZ && stats && log_std && dlogstd_partial,
                 "gaussian_loss: null argument");
    LossHyper hp{clip, value_coef, entropy_coef};
    return mg::gaussian_loss(head, action, adv, adv_stats, ret, old_log_prob, dZ, stats, log_std, dlogstd_partial,
                             rows, act_dim, hp, MG_STREAM(s));
}

int mg_gaussian_loss_num_partials(int rows) { return mg::gaussian_loss_parts(rows); }

int mg_gae(const float* reward, const uint8_t* done, const float* value, const void* bootstrap_head, float* adv,
           float* ret, int rows, int horizon, int act_dim, float gamma, float lambda, mg_stream_t s) {
    MG_CHECK_ARG(reward && done && value && bootstrap_head && adv && ret, "gae: null argument");
    MG_CHECK_ARG(act_dim >= 1 && act_dim < mg::kHeadDim, "gae: act_dim must be in [1, 64)");
    return mg::gae(reward, done, value, bootstrap_head, adv, ret, rows, horizon, act_dim, gamma, lambda, MG_STREAM(s));
}

int mg_advantage_stats(const float* adv, float* stats_out, int rows, int slots, mg_stream_t s) {
    MG_CHECK_ARG(adv && stats_out, "advantage_stats: null argument");
    return mg::advantage_stats(adv, stats_out, rows, slots, MG_STREAM(s));
}

int mg_reduce_partials(const float* partial, int64_t part_stride, int nparts, int64_t count, float* out,
                       int round_bf16, float* norm_partial, mg_stream_t s) {
    MG_CHECK_ARG(partial && out && norm_partial && nparts > 0 && count > 0, "reduce_partials: bad arguments");
    mg::GradSegmentTable tab{};
    tab.n = 1;
    tab.seg[0].src = partial;
    tab.seg[0].partStride = part_stride;
    tab.seg[0].nparts = nparts;
    tab.seg[0].count = count;
    tab.seg[0].dstOffset = 0;
    tab.seg[0].roundBf16 = round_bf16;
    mg::grad_table_layout(tab, false);  // one norm partial per 1024 elements
    return mg::grad_finalize(tab, out, norm_partial, MG_STREAM(s));
}

int mg_reduce_partials_num_norm_partials(int64_t count) { return (int)((count + mg::kGradPerCta - 1) / mg::kGradPerCta); }

int mg_adam_step(float* master, const float* grad, float* momentum, float* variance, void* weights,
                 const float* norm_partial, int n_norm_partials, int64_t count, float lr, float beta1_pow,
                 float beta2_pow, float max_grad_norm, float* norm_sq_out, mg_stream_t s) {
    MG_CHECK_ARG(master && grad && momentum && variance && weights && norm_partial, "adam_step: null argument");
    AdamHyper hp{lr, max_grad_norm, beta1_pow, beta2_pow};
    return mg::adam(master, grad, momentum, variance, weights, norm_partial, n_norm_partials, count, hp, nullptr,
                    norm_sq_out, MG_STREAM(s));
}

int mg_stats_mean(const float* stats, int rows, float* out5, mg_stream_t s) {
    MG_CHECK_ARG(stats && out5 && rows > 0, "stats_mean: null argument or no rows");
    return mg::stats_mean(stats, rows, out5, MG_STREAM(s));
}

}  // extern "C"
