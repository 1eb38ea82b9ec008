// Internal interface of the GEMM engine (host side).
#pragma once

#include <cuda_runtime.h>

#include "row_epilogues.cuh"

namespace mg {

// Epilogues of the bf16 GEMMs (gemm_tc.cuh, gemm_tc_persist.cuh).
enum GemmEpilogue : int {
    kEpiBf16 = 0,       // out_bf16 = bf16(acc)
    kEpiBf16Relu = 1,   // v = bf16(acc); out = v > 0 ? v : v * 0          (model/mlp.metal:49-56)
    kEpiBf16Resid = 2,  // out = bf16(aux + bf16(acc))                     (mlp.metal:85 + elementwise.metal:4-13)
    kEpiBf16Mask = 3,   // out = bf16(acc) * (aux > 0)                     (model/mlp.metal:119-126)
    kEpiF32 = 4,        // out_f32 = acc (split z writes slice z of M x N)
    kEpiPolicyLoss = 5, // out_bf16 = bf16(acc) (the policy head), then the categorical PPO loss of each row
    kEpiResidLN = 6,    // as kEpiBf16Resid, then the next LayerNorm of each output row (persistent kernel,
                        // one tile spanning the row)
};

struct GemmCall {
    const void* A = nullptr;
    bool a_mn = false;
    int lda = 0;
    const void* B = nullptr;
    bool b_mn = false;
    int ldb = 0;
    int M = 0, N = 0, K = 0;
    int epilogue = 0;
    void* out = nullptr;
    int ldo = 0;
    const void* aux = nullptr;
    int ldaux = 0;
    int splits = 1;
    int bn = 0;  // output tile width (64 / 128 / 256); 0 = choose
    int persistent = -1;  // 1: persistent kernel (bn 128 / 256), 0: one CTA per tile, -1: choose
    const PolicyLossRows* loss = nullptr;  // epilogue 5 (policy loss)
    const LnOutputs* ln = nullptr;         // epilogue 6 (residual, then LayerNorm)
};

int gemm_bf16(const GemmCall& c, cudaStream_t st);

// Row-complete products of 128-wide outputs, K split over a thread-block
// cluster and reduced through distributed shared memory, with the row
// epilogue of the layer that follows (gemm_rows.cu). A K-major [M][lda].
int gemm_rows_splits(int K);  // CTAs per cluster
bool gemm_rows_supported(int N, int K);
bool gemm_rows_ln_backward_supported(int M);
// h = bf16(h + bf16(A B)) in place, then the LayerNorm of h into ln
int gemm_rows_resid_layernorm(const void* A, int lda, const void* B, bool b_mn, int ldb, int M, int K, void* h,
                              const LnOutputs& ln, cudaStream_t st);
// The head of the training minibatch in one kernel (head_tail.cu), embed 128,
// categorical: head = bf16(fOut wHead), the PPO loss (dZ, statistics), dS =
// LayerNorm-F backward of bf16(dZ wHead^T) and the dW_head partial of each
// 128-row tile (headPart [tile][128][64]); bit-identical to the separate
// kernels.
bool head_tail_supported(int E, int M);
int head_tail(const void* fOut, const void* wHead, void* head, const PolicyLossRows& loss, float* headPart,
              const void* gammaF, const void* xNormF, const float* stdevF, void* dS, float* lnPart, int M,
              cudaStream_t st);
// dz = bf16(A B); residOut = resid + LayerNorm backward of dz; dgamma / dbeta
// partials exactly as layernorm_backward writes them
int gemm_rows_layernorm_backward(const void* A, int lda, const void* B, bool b_mn, int ldb, int M, int K,
                                 const void* xNorm, const void* gamma, const float* stdev, const void* resid,
                                 void* residOut, float* partial, cudaStream_t st);

// Number of K-splits gemm_bf16 actually launches when asked for `splits`
// (each split covers a multiple of 64 of K).
inline int gemm_effective_splits(int K, int splits) {
    int kps = (K + splits - 1) / splits;
    kps = (kps + 63) / 64 * 64;
    return (K + kps - 1) / kps;
}

}  // namespace mg
