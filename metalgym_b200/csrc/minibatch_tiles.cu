// The per-tile part of a training minibatch in one kernel (model/ppo.h:
// 753-865 for one minibatch of rows): on a 4-CTA cluster per 128-row tile,
//   block 0 forward with the input layer and the first LayerNorm,
//   blocks 1 .. L-1 forward,                       block_cluster.cuh
//   head, PPO loss, head dX, final LayerNorm backward,   head_tail.cuh
//   blocks L-1 .. 0 backward (block 0 with the input layer's gradient),
// the passes the separate kernels run (k_block_cluster, k_head_tail), back to
// back without leaving the SMs. Nothing of a minibatch crosses tiles before
// the gradient sums, so the passes need only the cluster's own barrier
// between them (tile_pass.cuh); the 2L + 1 launches of the chain become one,
// the barrier setup and the TMEM allocation happen once, and every output is
// bit-identical to the separate kernels' (the same passes, in the same
// order, on the same data). The gradient sums and Adam, which need every
// tile, stay kernels of their own.
#include <memory>

#include "block.h"
#include "block_cluster.cuh"
#include "head_tail.cuh"
#include "runtime.h"

namespace mg {

namespace {

constexpr int kMtMaxBlocks = MinibatchTiles::kMaxBlocks;
// shared memory: the block backward's layout (the largest pass), then the
// pass state
constexpr int kMtBar = kBcBwdBar;
constexpr int kMtSmem = kMtBar + 256 + 1024;
static_assert(kHtBar <= kMtBar && kBcFwdBar <= kMtBar && kTilePassBytes <= 256, "");

struct MtParams {
    int L;
    BcMaps fwdMaps[kMtMaxBlocks];
    BcMaps bwdMaps[kMtMaxBlocks];  // index n: block n's backward
    CUtensorMap headF, headW;
    BcParams fwd[kMtMaxBlocks];
    BcParams bwd[kMtMaxBlocks];
    HeadTailParams head;
};

template <int RPC, int AD>
__global__ void __launch_bounds__(kRowsThreads, 1) k_minibatch_tiles(const __grid_constant__ MtParams p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    mg_pdl_trigger();
    if (threadIdx.x == 0) {
        for (int n = 0; n < p.L; n++) {
            bc_prefetch_maps(p.fwdMaps[n], false);
            bc_prefetch_maps(p.bwdMaps[n], true);
        }
        prefetch_tensormap(&p.headF);
        prefetch_tensormap(&p.headW);
    }
    TilePass t = tp_setup(smem + kMtBar, 512, true);
    cluster_arrive_relaxed();  // this CTA has started (waited on before the peers' A tiles are written)
    if (p.fwd[0].in.earlyObs)  // the minibatch's observation rows, while the preceding kernel finishes
        bc_input_stage_obs(reinterpret_cast<float*>(smem + kBcFwdA2), cluster_ctarank(),
                           (int)(blockIdx.x / kRowsCluster) * kRowsBM, p.fwd[0].M, p.fwd[0].in);
    mg_pdl_wait();             // the weights come from earlier kernels
    bc_pass<false, 32, true>(smem, p.fwdMaps[0], p.fwd[0], t);
    for (int n = 1; n < p.L; n++) bc_pass<false, 32, false>(smem, p.fwdMaps[n], p.fwd[n], t);
    ht_pass<RPC, AD>(smem, p.headF, p.headW, p.head, t);
    for (int n = p.L - 1; n >= 0; n--) bc_pass<true, RPC, false>(smem, p.bwdMaps[n], p.bwd[n], t);
    tp_teardown(t, p.head.status);
}

template <int RPC>
int launch_mt(const MtParams& p, int M, cudaStream_t st) {
    // two actions (CartPole): the loss with its loops unrolled
    auto kern = p.head.loss.actDim == 2 ? k_minibatch_tiles<RPC, 2> : k_minibatch_tiles<RPC, 0>;
    static std::atomic<uint64_t> attr_done[2] = {};  // per kernel variant
    if (int rc = smem_limit_once(kern, kMtSmem, attr_done[p.head.loss.actDim == 2 ? 1 : 0])) return rc;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(((M + kRowsBM - 1) / kRowsBM) * kRowsCluster));
    cfg.blockDim = dim3(kRowsThreads);
    cfg.dynamicSmemBytes = kMtSmem;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = kRowsCluster;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    MG_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, p));
    return check_launch("k_minibatch_tiles");
}

}  // namespace

struct MinibatchTiles::Plan {
    MtParams p{};
    int M = 0, nFwd = 0, nBwd = 0;
    bool head = false, fwdInput = false;
    int rc = MG_OK;  // the first recording error
};

MinibatchTiles::MinibatchTiles() : plan(new Plan) {}
MinibatchTiles::~MinibatchTiles() { delete plan; }

void MinibatchTiles::reset() { *plan = Plan{}; }

int MinibatchTiles::record(int rc) {
    if (rc && !plan->rc) plan->rc = rc;
    return rc;
}

int MinibatchTiles::forward(const void* lnOut, const void* wUp, const void* wDown, void* h, void* v,
                            const LnOutputs& next, int M, const BlockClusterForwardInput* in) {
    Plan& q = *plan;
    if (q.nFwd >= kMaxBlocks || q.head || q.nBwd || (q.nFwd == 0) != (in != nullptr) || (q.M && q.M != M))
        return record(fail(MG_ERR_ARGUMENT, "minibatch tiles: forward passes out of order"));
    q.M = M;
    q.fwdInput = q.fwdInput || in;
    const int n = q.nFwd++;
    return record(block_cluster_forward_args(lnOut, wUp, wDown, h, v, next, M, in, q.p.fwdMaps[n], q.p.fwd[n]));
}

int MinibatchTiles::headTail(const void* fOut, const void* wHead, void* head, const PolicyLossRows& loss,
                             float* headPart, const void* gammaF, const void* xNormF, const float* stdevF, void* dS,
                             float* lnPart, int M) {
    Plan& q = *plan;
    if (q.nFwd == 0 || q.head || q.M != M)
        return record(fail(MG_ERR_ARGUMENT, "minibatch tiles: the head pass out of order"));
    q.head = true;
    return record(head_tail_args(fOut, wHead, head, loss, headPart, gammaF, xNormF, stdevF, dS, lnPart, M,
                                 q.p.headF, q.p.headW, q.p.head));
}

int MinibatchTiles::backward(const void* dS, const void* wDown, const void* v, const void* wUp, void* dV,
                             const void* lnOut, float* upPart, float* downPart, const void* xNorm, const void* gamma,
                             const float* stdev, const void* resid, void* residOut, float* partial, int M,
                             const BlockClusterInput* in) {
    Plan& q = *plan;
    const int n = q.nFwd - 1 - q.nBwd;  // block n: the last forward block first
    if (!q.head || n < 0 || q.M != M || (in && n != 0))
        return record(fail(MG_ERR_ARGUMENT, "minibatch tiles: backward passes out of order"));
    q.nBwd++;
    return record(block_cluster_backward_args(dS, wDown, v, wUp, dV, lnOut, upPart, downPart, xNorm, gamma, stdev,
                                              resid, residOut, partial, M, in, q.p.bwdMaps[n], q.p.bwd[n]));
}

int MinibatchTiles::launch(cudaStream_t st) {
    Plan& q = *plan;
    if (q.rc) return q.rc;
    MG_CHECK_ARG(q.nFwd >= 1 && q.fwdInput && q.head && q.nBwd == q.nFwd,
                 "minibatch tiles: launch needs L forward passes (the first with the input layer), the head "
                 "pass and L backward passes");
    q.p.L = q.nFwd;
    switch (layernorm_rows_per_part(q.M)) {
        case 8: return launch_mt<8>(q.p, q.M, st);
        case 16: return launch_mt<16>(q.p, q.M, st);
        default: return launch_mt<32>(q.p, q.M, st);
    }
}

}  // namespace mg
