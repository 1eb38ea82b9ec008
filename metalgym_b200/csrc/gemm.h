// Internal interface of the GEMM engine (host side).
#pragma once

#include <cuda_runtime.h>

#include "loss_row.cuh"

namespace mg {

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
};

int gemm_bf16(const GemmCall& c, cudaStream_t st);

// Number of K-splits gemm_bf16 actually launches when asked for `splits`
// (each split covers a multiple of 64 of K).
inline int gemm_effective_splits(int K, int splits) {
    int kps = (K + splits - 1) / splits;
    kps = (kps + 63) / 64 * 64;
    return (K + kps - 1) / kps;
}

}  // namespace mg
