// Internal host interface of the row-wise policy kernels (policy.cu).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "row_epilogues.cuh"
#include "metalgym/rowmap.h"

namespace mg {

// PPO loss coefficients (model/policy.metal:5-12).
struct LossHyper {
    float clip;
    float valueCoef;
    float entropyCoef;
};

// Adam settings (model/optimizer.metal:5-15); betas (0.9, 0.999), eps 1e-8 fixed.
struct AdamHyper {
    float lr;
    float maxGradNorm;
    float beta1Pow;  // used when no device beta-power pointer is given
    float beta2Pow;
};

// One parameter's gradient: `nparts` partial sums, `partStride` floats apart,
// each `count` long, summed into grad[dstOffset ...].
struct GradSegment {
    const float* src;
    int64_t partStride;
    int64_t count;
    int64_t dstOffset;
    int nparts;
    int roundBf16;  // 1: round the sum to bf16 (GEMM weight gradients)
    int blockEnd;   // filled by grad_table_layout
    int deep;       // filled by grad_table_layout: nparts > kGradDeepParts
    int vec4;       // set by grad_finalize: 16-byte aligned addresses and strides
    // the partials come from kernels before the one that precedes the
    // finalisation (grad_finalize's earlyOk: those CTAs skip the dependency wait)
    int early;
};

// Gradient elements per CTA of the finalisation (one norm partial each):
// kGradPerCta for segments of few partials (a thread sums 4 elements over
// all partials), kGradPerCtaDeep for segments of more than kGradDeepParts
// partials (the CTA's 8 warps split the partials of 128 elements).
constexpr int kGradPerCta = 1024;
constexpr int kGradPerCtaDeep = 128;
constexpr int kGradDeepParts = 32;

constexpr int kMaxGradSegments = 40;
struct GradSegmentTable {
    GradSegment seg[kMaxGradSegments];
    int n;
};

// Where the rows of a training minibatch come from: with mb (a device
// pointer to the minibatch's schedule entry), row q of the kernel reads
// rollout row mg_minibatch_row(*mb, q, envRows, total) of the slot-major
// buffers; without it, row q reads row q.
struct RowMap {
    const MgMinibatch* mb;
    uint64_t envRows;  // R, rows per slot
    uint64_t total;    // T * R
};

// With ln, the LayerNorm of the output rows (as layernorm_forward computes
// it, bit-identical) is written too.
int input_forward(const float* obs, const void* w, const void* b, void* out, int rows, int inDim, int outDim,
                  cudaStream_t st, RowMap rm = RowMap{nullptr, 0, 0}, const LnOutputs* ln = nullptr);
int input_backward_parts(int rows, int inDim, int outDim);
int input_backward(const float* obs, const void* dZ, float* partial, int rows, int inDim, int outDim,
                   cudaStream_t st, RowMap rm = RowMap{nullptr, 0, 0});
int layernorm_forward(const void* x, void* xNorm, void* out, const void* gamma, const void* beta, float* stdev,
                      int rows, int cols, cudaStream_t st);
int layernorm_backward_parts(int rows);
int layernorm_rows_per_part(int rows);  // rows per dgamma / dbeta partial of layernorm_backward
int layernorm_backward(void* dZ, const void* xNorm, const void* gamma, const float* stdev, const void* resid,
                       float* partial, int rows, int cols, cudaStream_t st, void* residOut = nullptr);
int sample_categorical(const void* head, uint32_t* rng, int32_t* action, float* logProb, float* value, int rows,
                       int actDim, cudaStream_t st);
int sample_gaussian(const void* head, const void* logStd, uint32_t* rng, float* action, float* logProb,
                    float* value, int rows, int actDim, cudaStream_t st);
// The loss arguments as the fused head-GEMM epilogue takes them.
PolicyLossRows policy_loss_rows(const int32_t* action, const float* adv, const float* advStats, const float* ret,
                                const float* oldLogProb, void* dZ, float* stats, int rows, int actDim, LossHyper hp,
                                RowMap rm);
int policy_loss(const void* head, const int32_t* action, const float* adv, const float* advStats, const float* ret,
                const float* oldLogProb, void* dZ, float* stats, int rows, int actDim, LossHyper hp,
                cudaStream_t st, RowMap rm = RowMap{nullptr, 0, 0});
int gaussian_loss_parts(int rows);
int gaussian_loss(const void* head, const float* action, const float* adv, const float* advStats, const float* ret,
                  const float* oldLogProb, void* dZ, float* stats, const void* logStd, float* partial, int rows,
                  int actDim, LossHyper hp, cudaStream_t st, RowMap rm = RowMap{nullptr, 0, 0});
int gae(const float* reward, const uint8_t* done, const float* value, const void* bootHead, float* adv, float* ret,
        int rows, int horizon, int actDim, float gamma, float lambda, cudaStream_t st);
int advantage_stats(const float* adv, float* out, int rows, int slots, cudaStream_t st);
// {mean, 1/(std + 1e-8)} of adv over the rows of one row-mode minibatch;
// scratch: 2 x kAdvStatsMaxCtas doubles and a zeroed counter (left zeroed).
constexpr int kAdvStatsMaxCtas = 296;
int advantage_stats_rows(const float* adv, RowMap rm, int rows, float* out, double* partial,
                         unsigned int* counter, cudaStream_t st);
// Fills blockEnd (and deep, when allowDeep) of every segment; returns the
// number of CTAs (= norm partials).
int grad_table_layout(GradSegmentTable& tab, bool allowDeep = true);
// With counter (a zeroed device word) and normSqOut, the last CTA also sums
// the per-CTA partials into *normSqOut and re-zeroes the counter.
// With sel (a device counter): the sums go to grad2 when *sel + 1 is odd, else
// to grad (the two exchange buffers of the peer all-reduce).
// bf16From: elements from this index on are stored packed as bf16 after the
// fp32 ones (only bf16-rounded segments may lie there; the exchange buffer of
// the peer-memory all-reduce); INT64_MAX: every element fp32.
// earlyOk: the kernel preceding the finalisation on st signals its dependents
// only after its own dependency wait, so the CTAs of segments marked early
// (their partials written before that kernel) start without waiting.
int grad_finalize(const GradSegmentTable& tab, float* grad, float* normPartial, cudaStream_t st,
                  unsigned int* counter = nullptr, float* normSqOut = nullptr, float* grad2 = nullptr,
                  const unsigned int* sel = nullptr, int64_t bf16From = INT64_MAX, bool earlyOk = false);
int grad_scale_norm_blocks(int64_t count);
int grad_scale_norm(float* grad, int64_t count, float scale, float* normPartial, cudaStream_t st,
                    unsigned int* counter = nullptr, float* normSqOut = nullptr);
// normSqIn (optional): the squared gradient norm, instead of summing normPartial.
int adam(float* param, const float* grad, float* mom, float* var, void* weights, const float* normPartial, int nNorm,
         int64_t count, AdamHyper hp, const float* betaPow, float* normSqOut, cudaStream_t st,
         const float* normSqIn = nullptr);
int stats_mean(const float* stats, int rows, float* out, cudaStream_t st);
// actGreedy (model/ppo.h:688-702): per row of head [rows][64] bf16 the argmax
// action (int32) or, continuous, the actDim means (float) into actions.
int act_greedy(const void* head, int rows, int actDim, bool continuous, void* actions, cudaStream_t st);

}  // namespace mg
