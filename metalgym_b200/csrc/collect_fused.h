// collect() as one persistent kernel: the host side (collect_fused.cu) that
// prepares the launch of the kernel an environment registered
// (include/metalgym/detail/collect_fused.cuh, mg_env_ops::collect_fused).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "metalgym/detail/collect_fused.cuh"
#include "metalgym_b200.h"

namespace mg {

// The rollout of model/ppo.h:716-751 for the policy shape embed 128, hidden
// 512, 1..4 blocks. Device pointers; weights bf16 in the layouts of the
// parameter arena.
struct CollectFusedArgs {
    int R, T, L, inDim;
    const void* wIn;  // [inDim][128]
    const void* bIn;  // [128]
    // LayerNorm n (n < L: block n's; n == L: the final LayerNorm)
    const void* lnGamma[kCollectFusedMaxBlocks + 1];
    const void* lnBeta[kCollectFusedMaxBlocks + 1];
    const void* wUp[kCollectFusedMaxBlocks];    // [128][512]
    const void* wDown[kCollectFusedMaxBlocks];  // [512][128]
    const void* wHead;                          // [128][64]
    const void* logStd;                         // [act_dim] (continuous environments)
    // the gym's environment buffers (read at the start, written at the end)
    void* states;
    uint8_t* done;
    uint32_t* rng;
    // rollout slots, slot-major (model/ppo.h:336-345); obs slot 0 is the input
    float* obsSlots;  // [T + 1][R][inDim]
    void* actionSlots;
    float *logpSlots, *valueSlots, *rewardSlots;
    uint8_t* doneSlots;
    float *advSlots, *retSlots;
    void* bootHead;  // [R][64] bf16: the head rows of the bootstrap forward
    float gamma, lambda;
};

// True when the environment registered a fused kernel (its State fits in
// registers, its observation in 32 floats) and the policy has the kernel's
// shape (embed 128, hidden 512, 1..4 blocks).
bool collect_fused_supported(const mg_env_ops* ops, int E, int H, int L, int inDim);
int collect_fused(const mg_env_ops* ops, const CollectFusedArgs& a, cudaStream_t st);

}  // namespace mg
