// Fused residual-block kernels of the policy (block_fwd.cu, block_cluster.cu).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "metalgym/rowmap.h"

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

// One residual block per kernel on 4-CTA clusters (block_cluster.cu), embed
// 128 and hidden 512. Forward: V = relu(lnOut Up) (saved), h += V Dp in place,
// then the LayerNorm `next` of h. Backward: dV = bf16(dS Dp^T) * (V > 0)
// (saved), dz = bf16(dV Up^T), residOut = resid + LayerNorm backward of dz
// (xNorm, gamma, stdev of the block's LayerNorm) with the dgamma / dbeta
// partials of layernorm_backward. Bit-identical to the separate kernels.
struct LnOutputs;
constexpr int kBlockClusterMaxInputDim = 32;
bool block_cluster_supported(int E, int H);
// With `in` (the first block), the kernel first computes the input layer
// (h = b + obs W, written to h) and the first LayerNorm (x-hat, sigma; its
// output written to lnOut) itself, exactly as input_forward and
// layernorm_forward do; lnOut is then an output.
struct BlockClusterForwardInput {
    const float* obs;       // [*][inDim] fp32
    const MgMinibatch* mb;  // row map (null: row r reads observation r)
    uint64_t envRows, total;
    int inDim;              // <= kBlockClusterMaxInputDim
    const void* w;          // [inDim][128] bf16
    const void* b;          // [128] bf16
    const void* gamma;      // the first LayerNorm
    const void* beta;
    void* xNorm;
    float* stdev;
};
// prefetch: the preceding kernel on st is one of these block kernels or the
// head kernel (head_tail), which signal their dependents only after their
// own dependency wait; the weights (and the backward's other operands but the
// A tile) are then loaded before this kernel's wait (BcParams::prefetch).
int block_cluster_forward(const void* lnOut, const void* wUp, const void* wDown, void* h, void* v,
                          const LnOutputs& next, int M, cudaStream_t st,
                          const BlockClusterForwardInput* in = nullptr, bool prefetch = false);
// It also writes the weight-gradient partial sums of each 128-row tile t:
// upPart[t] = lnOut_t^T dV_t ([128][512]), downPart[t] = V_t^T dS_t ([512][128]).
// With `in` (the first block), the rows written are the input layer's dZ,
// and the kernel also writes its gradient partials as input_backward does at
// 16 rows per partial (the caller checks that input_backward partitions so).
struct BlockClusterInput {
    const float* obs;          // observations [*][inDim] fp32
    const MgMinibatch* mb;     // minibatch row map (null: row r reads observation r)
    uint64_t envRows, total;
    int inDim;                 // <= kBlockClusterMaxInputDim
    float* partial;            // [rows / 16][(inDim + 1) x 128]
};
int block_cluster_backward(const void* dS, const void* wDown, const void* v, const void* wUp, void* dV,
                           const void* lnOut, float* upPart, float* downPart, const void* xNorm, const void* gamma,
                           const float* stdev, const void* resid, void* residOut, float* partial, int M,
                           cudaStream_t st, const BlockClusterInput* in = nullptr, bool prefetch = false);

// The per-tile part of one training minibatch in one kernel
// (minibatch_tiles.cu): the passes of block_cluster_forward (block 0 with the
// input layer, then blocks 1 .. L-1), head_tail and block_cluster_backward
// (blocks L-1 .. 0), recorded with the same arguments as those calls, then
// launched as one kernel of 4-CTA clusters; bit-identical to the separate
// kernels. Embed 128, hidden 512, categorical head, 1..kMaxBlocks blocks.
struct PolicyLossRows;
class MinibatchTiles {
   public:
    static constexpr int kMaxBlocks = 2;
    MinibatchTiles();
    ~MinibatchTiles();
    MinibatchTiles(const MinibatchTiles&) = delete;
    MinibatchTiles& operator=(const MinibatchTiles&) = delete;
    void reset();
    int forward(const void* lnOut, const void* wUp, const void* wDown, void* h, void* v, const LnOutputs& next, int M,
                const BlockClusterForwardInput* in);
    int headTail(const void* fOut, const void* wHead, void* head, const PolicyLossRows& loss, float* headPart,
                 const void* gammaF, const void* xNormF, const float* stdevF, void* dS, float* lnPart, int M);
    int backward(const void* dS, const void* wDown, const void* v, const void* wUp, void* dV, const void* lnOut,
                 float* upPart, float* downPart, const void* xNorm, const void* gamma, const float* stdev,
                 const void* resid, void* residOut, float* partial, int M, const BlockClusterInput* in);
    // one launch of the recorded passes (checks that they form a minibatch)
    int launch(cudaStream_t st);

   private:
    struct Plan;
    Plan* plan;
    int record(int rc);
};

}  // namespace mg
