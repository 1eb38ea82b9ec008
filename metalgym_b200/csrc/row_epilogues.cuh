// Row computations shared by standalone row kernels and fused GEMM
// epilogues, so that both give the same bits: the categorical PPO loss of one
// row (model/policy.metal:14-69) and the arguments of a LayerNorm that ends a
// kernel.
#pragma once

#include <cuda_bf16.h>
#include <stdint.h>

#include "metalgym/mathf.h"
#include "metalgym/rowmap.h"
#include "metalgym/detail/ptx.cuh"

namespace mg {

constexpr int kLossHeadDim = 64;  // head columns (model/ppo.h:116)

// LayerNorm outputs of a kernel that ends with the next LayerNorm of its rows.
struct LnOutputs {
    const __nv_bfloat16* gamma;
    const __nv_bfloat16* beta;
    __nv_bfloat16* xNorm;
    __nv_bfloat16* out;
    float* stdev;
};

// Inputs and outputs of the loss of a minibatch's rows. Minibatch row r
// reads rollout row mg_minibatch_row(*mb, r, envRows, total) of action / adv
// / ret / oldLogProb (row r itself without mb); advStats holds {mean, 1 /
// (std + 1e-8)} (per slot when mb is a slot minibatch) or is null.
struct PolicyLossRows {
    const int32_t* action;
    const float* adv;
    const float* advStats;
    const float* ret;
    const float* oldLogProb;
    __nv_bfloat16* dZ;  // rows x 64
    float* stats;       // rows x 5
    const MgMinibatch* mb;
    uint64_t envRows, total;
    int rows, actDim;
    float clip, valueCoef, entropyCoef;
};

__device__ __forceinline__ float loss_bf(__nv_bfloat16 x) { return __bfloat162float(x); }
__device__ __forceinline__ __nv_bfloat16 loss_tobf(float x) { return __float2bfloat16_rn(x); }

// Row r of the minibatch, its head row h (64 bf16): the row's dZ (64 bf16,
// packed in pairs) and its 5 statistics. Returns false (and records
// kDevBadAction) for an action outside [0, actDim). AD > 0: the caller
// guarantees L.actDim == AD, and every loop over the actions has a known trip
// count (the same operations in the same order, so the same bits, in far
// less code: the loss runs once per kernel launch, from a cold instruction
// cache).
template <int AD = 0>
__device__ inline bool policy_loss_compute(const PolicyLossRows& L, int r, const __nv_bfloat16* h, int* status,
                                           uint32_t* packed, float* st) {
    static_assert(AD >= 0 && AD <= 8, "AD: 0 (the actions known at run time) or 1..8");
    const int64_t g = L.mb ? (int64_t)mg_minibatch_row(*L.mb, r, L.envRows, L.total) : r;
    const float* advStats = L.advStats;
    if (L.mb && L.mb->slot >= 0 && advStats) advStats += 2 * L.mb->slot;  // per-slot statistics
    const int actDim = AD > 0 ? AD : L.actDim;
    // the row's inputs first, so that their loads overlap the exponentials
    const int a = L.action[g];
    const float advG = L.adv[g], oldLogProb = L.oldLogProb[g], retG = L.ret[g];
    const float adv0 = advStats ? advStats[0] : 0.0f, adv1 = advStats ? advStats[1] : 0.0f;
    const float scale = __fdiv_rn(1.0f, (float)L.rows);
    // exp(logp_j) is needed twice (entropy, gradient): keep up to kCache of them
    constexpr int kCache = 8;
    float probCache[kCache];
    float rowMax = -INFINITY;
    for (int j = 0; j < actDim; j++) rowMax = fmaxf(rowMax, loss_bf(h[j]));
    float sum = 0.0f;
    for (int j = 0; j < actDim; j++) sum = __fadd_rn(sum, mg_expf(__fsub_rn(loss_bf(h[j]), rowMax)));
    const float lse = __fadd_rn(rowMax, mg_logf(sum));
    // the ratio's exponential beside the probabilities' (the action is
    // checked below; index 0 stands in for an invalid one until then)
    const float logpA = __fsub_rn(loss_bf(h[(a >= 0 && a < actDim) ? a : 0]), lse);
    const float ratio = mg_expf(__fsub_rn(logpA, oldLogProb));
    float entropy = 0.0f;
#pragma unroll
    for (int j = 0; j < kCache; j++) {
        if (j < actDim) {
            const float logp = __fsub_rn(loss_bf(h[j]), lse);
            probCache[j] = mg_expf(logp);
            entropy = __fsub_rn(entropy, __fmul_rn(probCache[j], logp));
        }
    }
    for (int j = kCache; j < actDim; j++) {
        const float logp = __fsub_rn(loss_bf(h[j]), lse);
        entropy = __fsub_rn(entropy, __fmul_rn(mg_expf(logp), logp));
    }
    if (a < 0 || a >= actDim) {  // never index the head with an invalid action
        record_error(status, kDevBadAction);
        return false;
    }
    // model/gae.metal:76: (a - mean) * inv, inv = 1 / (sigma + 1e-8)
    const float A = advStats ? __fmul_rn(__fsub_rn(advG, adv0), adv1) : advG;
    const float surr1 = __fmul_rn(ratio, A);
    const float surr2 = __fmul_rn(fminf(fmaxf(ratio, __fsub_rn(1.0f, L.clip)), __fadd_rn(1.0f, L.clip)), A);
    const float policyLoss = -fminf(surr1, surr2);
    const float gLogp = (surr1 <= surr2) ? __fmul_rn(-A, ratio) : 0.0f;
#pragma unroll
    for (int i = 0; i < kLossHeadDim / 2; i++) packed[i] = 0;
    __nv_bfloat16* pz = reinterpret_cast<__nv_bfloat16*>(packed);
    for (int j = 0; j < actDim; j++) {
        const float logp = __fsub_rn(loss_bf(h[j]), lse);
        float prob;
        if (j < kCache) {
#pragma unroll
            for (int q = 0; q < kCache; q++)
                if (q == j) prob = probCache[q];
        } else {
            prob = mg_expf(logp);
        }
        const float gr = __fadd_rn(__fmul_rn(gLogp, __fsub_rn(j == a ? 1.0f : 0.0f, prob)),
                                   __fmul_rn(__fmul_rn(L.entropyCoef, prob), __fadd_rn(logp, entropy)));
        pz[j] = loss_tobf(__fmul_rn(gr, scale));
    }
    const float vErr = __fsub_rn(loss_bf(h[actDim]), retG);
    pz[actDim] = loss_tobf(__fmul_rn(__fmul_rn(L.valueCoef, vErr), scale));
    st[0] = policyLoss;
    st[1] = __fmul_rn(__fmul_rn(__fmul_rn(0.5f, L.valueCoef), vErr), vErr);
    st[2] = entropy;
    st[3] = __fsub_rn(oldLogProb, logpA);
    st[4] = (fabsf(__fsub_rn(ratio, 1.0f)) > L.clip) ? 1.0f : 0.0f;
    return true;
}

// The loss of row r written to L.dZ and L.stats.
__device__ inline bool policy_loss_row(const PolicyLossRows& L, int r, const __nv_bfloat16* h, int* status) {
    uint32_t packed[kLossHeadDim / 2];
    float st[5];
    if (!policy_loss_compute(L, r, h, status, packed, st)) return false;
    uint4* dst = reinterpret_cast<uint4*>(L.dZ + (size_t)r * kLossHeadDim);
    const uint4* src = reinterpret_cast<const uint4*>(packed);
#pragma unroll
    for (int i = 0; i < kLossHeadDim / 8; i++) dst[i] = src[i];
    float* so = L.stats + (size_t)r * 5;
#pragma unroll
    for (int i = 0; i < 5; i++) so[i] = st[i];
    return true;
}

}  // namespace mg
