// Fused residual-block kernels of the policy (block_fwd.cu).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>

namespace mg {

// One residual MLP block forward over `rows` rows: LayerNorm of h (saved in
// xNorm, lnOut, stdev), V = relu(lnOut Up) (saved), h += V Dp in place.
struct BlockFwdArgs {
    __nv_bfloat16* h;              // rows x E, in / out
    const __nv_bfloat16* gamma;    // E
    const __nv_bfloat16* beta;     // E
    __nv_bfloat16* xNorm;          // rows x E
    __nv_bfloat16* lnOut;          // rows x E
    float* stdev;                  // rows
    __nv_bfloat16* V;              // rows x H
    int rows, E, H;
    int* status;
};

bool block_forward_supported(int E, int H);
// up: Up [E][H], down: Dp [H][E] (row-major bf16).
int block_forward(const BlockFwdArgs& a, const void* up, const void* down, cudaStream_t st);

}  // namespace mg
