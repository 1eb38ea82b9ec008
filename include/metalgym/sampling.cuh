// Device-side action samplers shared by the policy kernels and the fused
// collect step of every registered environment.
//
// Both draw from the env's own xorshift word, so policy sampling and env
// resets share one stream as in the reference (model/ppo.h:706). Arithmetic
// is written with __fmul_rn / __fadd_rn (no contraction) and the
// project-owned transcendentals, so a draw is bit-identical to the reference
// kernel compiled as host C++ given the same head row.
#pragma once

#include <cuda_bf16.h>
#include <stdint.h>

#include "mathf.h"
#include "rng.h"

namespace mg {

constexpr int kHeadDim = 64;  // model/ppo.h:116: logits | value | zero pad
constexpr float kLogSqrt2Pi = 0.9189385332046727f;

__device__ __forceinline__ float bf(const __nv_bfloat16 x) { return __bfloat162float(x); }

// ---- categorical draw (model/sample.metal:18-47) on one head row.
// Advances the env's xorshift word by one draw. Returns the chosen action.
__device__ __forceinline__ int sample_categorical_row(const __nv_bfloat16* head, int actDim, uint32_t& rng,
                                                      float& logProb, float& value) {
    float rowMax = -INFINITY;
    for (int a = 0; a < actDim; a++) rowMax = fmaxf(rowMax, bf(head[a]));
    float sum = 0.0f;
    for (int a = 0; a < actDim; a++) sum = __fadd_rn(sum, mg_expf(__fsub_rn(bf(head[a]), rowMax)));
    const float lse = __fadd_rn(rowMax, mg_logf(sum));
    const float u = __fmul_rn(__fmul_rn((float)(rngNext(rng) >> 8), 1.0f / 16777216.0f), sum);
    int chosen = actDim - 1;
    float acc = 0.0f;
    for (int a = 0; a < actDim; a++) {
        acc = __fadd_rn(acc, mg_expf(__fsub_rn(bf(head[a]), rowMax)));
        if (u < acc) {
            chosen = a;
            break;
        }
    }
    logProb = __fsub_rn(bf(head[chosen]), lse);
    value = bf(head[actDim]);
    return chosen;
}

// ---- Gaussian draw (model/gaussian.metal:32-71): Box-Muller pairs, u1 in (0, 1].
__device__ __forceinline__ void sample_gaussian_row(const __nv_bfloat16* head, const __nv_bfloat16* logStd,
                                                    int actDim, uint32_t& rng, float* action, float& logProb,
                                                    float& value) {
    float lp = 0.0f, zx = 0.0f, zy = 0.0f;
    for (int k = 0; k < actDim; k++) {
        if ((k & 1) == 0) {
            const float u1 = __fsub_rn(1.0f, __fmul_rn((float)(rngNext(rng) >> 8), 1.0f / 16777216.0f));
            const float u2 = __fmul_rn((float)(rngNext(rng) >> 8), 1.0f / 16777216.0f);
            const float r = __fsqrt_rn(__fmul_rn(-2.0f, mg_logf(u1)));
            const float theta = __fmul_rn(__fmul_rn(2.0f, 3.14159265358979323846f), u2);
            float st, ct;
            mg_sincosf(theta, &st, &ct);
            zx = __fmul_rn(r, ct);
            zy = __fmul_rn(r, st);
        }
        const float zk = (k & 1) ? zy : zx;
        const float ls = bf(logStd[k]);
        const float mu = bf(head[k]);
        const float a = __fadd_rn(mu, __fmul_rn(mg_expf(ls), zk));
        const float d = __fmul_rn(__fsub_rn(a, mu), mg_expf(-ls));
        action[k] = a;
        lp = __fadd_rn(lp, __fsub_rn(__fsub_rn(__fmul_rn(__fmul_rn(-0.5f, d), d), ls), kLogSqrt2Pi));
    }
    logProb = lp;
    value = bf(head[actDim]);
}

// Zero-logit categorical draw: the sampler above with every logit 0, i.e.
// u = U[0,1) * A and the first a with u < a + 1 (the random policy of the raw
// environment benchmark). One draw from the env's word.
__device__ __forceinline__ int uniform_action(uint32_t& rng, int actDim) {
    const float sum = (float)actDim;
    const float u = __fmul_rn(__fmul_rn((float)(rngNext(rng) >> 8), 1.0f / 16777216.0f), sum);
    float acc = 0.0f;
    for (int a = 0; a < actDim; a++) {
        acc = __fadd_rn(acc, 1.0f);
        if (u < acc) return a;
    }
    return actDim - 1;
}

}  // namespace mg
