// Internal interface of the GEMM engine (host side).
#pragma once

#include <cuda_runtime.h>

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
};

int gemm_bf16(const GemmCall& c, cudaStream_t st);

}  // namespace mg
