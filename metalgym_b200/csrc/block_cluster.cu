// The residual-block kernels of the CartPole-sized policy (embed 128, hidden
// 512): one kernel per block forward or backward on 4-CTA clusters, one
// cluster per 128-row tile, each running the block pass of
// block_cluster.cuh once (where the arithmetic is described). The hidden
// activation of a block never makes a round trip through another kernel:
// four launches per block (LayerNorm aside) become one, on 128 CTAs at 4096
// rows, bit-identical to the up or dV GEMM followed by the row kernel.
#include "block_cluster.cuh"
#include "runtime.h"

namespace mg {

namespace {

template <bool BWD, int RPC, bool INPUT = false>
__global__ void __launch_bounds__(kRowsThreads, 1) k_block_cluster(const __grid_constant__ BcMaps tm, const BcParams p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    if (threadIdx.x == 0) bc_prefetch_maps(tm, BWD);
    // 128-column accumulators: 2 (forward), 4 (backward)
    TilePass t = tp_setup(smem + (BWD ? kBcBwdBar : kBcFwdBar), BWD ? 512 : 256, false);
    if (INPUT) cluster_arrive_relaxed();  // this CTA has started (waited on before the peers' A tiles are written)
    // a training minibatch's observation rows do not depend on the preceding
    // kernel: stage them while it finishes
    if (INPUT && p.in.earlyObs)
        bc_input_stage_obs(reinterpret_cast<float*>(smem + kBcFwdA2), cluster_ctarank(),
                           (int)(blockIdx.x / kRowsCluster) * kRowsBM, p.M, p.in);
    // the weights (and the backward's mask and LayerNorm output), where they
    // come from kernels before the preceding one (BcParams::prefetch)
    const bool early = !INPUT && p.prefetch;
    if (early && threadIdx.x == 0) bc_issue_static<BWD, INPUT>(smem, tm, t);
    mg_pdl_wait();  // activations and weights come from earlier kernels
    // dependents start only now, after this kernel's predecessor completed:
    // their pre-wait loads may read what came before this kernel
    mg_pdl_trigger();
    bc_pass<BWD, RPC, INPUT>(smem, tm, p, t, early);
}

template <bool BWD, int RPC, bool INPUT = false>
int launch_bc(const BcMaps& tm, const BcParams& p, cudaStream_t st) {
    auto kern = k_block_cluster<BWD, RPC, INPUT>;
    constexpr int smemBytes = BWD ? kBcBwdSmem : kBcFwdSmem;
    static std::atomic<uint64_t> attr_done{0};
    if (int rc = smem_limit_once(kern, smemBytes, attr_done)) return rc;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(((p.M + kRowsBM - 1) / kRowsBM) * kRowsCluster));
    cfg.blockDim = dim3(kRowsThreads);
    cfg.dynamicSmemBytes = smemBytes;
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
    MG_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, tm, p));
    return check_launch("k_block_cluster");
}

}  // namespace

bool block_cluster_supported(int E, int H) { return E == kRowsBN && H == kBcHidden; }

int block_cluster_forward_args(const void* lnOut, const void* wUp, const void* wDown, void* h, void* v,
                               const LnOutputs& next, int M, const BlockClusterForwardInput* in, BcMaps& tm,
                               BcParams& p) {
    MG_CHECK_ARG(lnOut && wUp && wDown && h && v && next.gamma && next.beta && next.xNorm && next.out && next.stdev,
                 "block_cluster_forward: null argument");
    MG_CHECK_ARG(M > 0, "block_cluster_forward: M must be > 0");
    if (in)
        MG_CHECK_ARG(in->obs && in->w && in->b && in->gamma && in->beta && in->xNorm && in->stdev && in->inDim > 0 &&
                         in->inDim <= kRowsInputMaxDim,
                     "block_cluster_forward: bad input-layer arguments");
    tm = BcMaps{};
    int rc = make_tmap_bf16(&tm.a, lnOut, kRowsBN, M, kRowsBN, 128);
    if (!rc) rc = make_tmap_bf16(&tm.b1, wUp, kBcHidden, kRowsBN, kBcHidden, 64);
    if (!rc) rc = make_tmap_bf16(&tm.b2, wDown, kRowsBN, kBcHidden, kRowsBN, 64);
    if (!rc) rc = make_tmap_bf16(&tm.v, v, kBcHidden, M, kBcHidden, 128);
    if (rc) return rc;
    p = BcParams{};
    p.M = M;
    p.vOut = static_cast<__nv_bfloat16*>(v);
    p.e.M = M;
    p.e.resid = static_cast<const __nv_bfloat16*>(h);
    p.e.out = static_cast<__nv_bfloat16*>(h);
    p.e.ln = next;
    p.status = status_ptr();
    p.trace = tile_trace();
    if (in) {
        p.in = BcInput{in->obs, in->mb, in->envRows, in->total, in->inDim,
                       static_cast<const __nv_bfloat16*>(in->w), static_cast<const __nv_bfloat16*>(in->b),
                       static_cast<__nv_bfloat16*>(h),
                       LnOutputs{static_cast<const __nv_bfloat16*>(in->gamma),
                                 static_cast<const __nv_bfloat16*>(in->beta),
                                 static_cast<__nv_bfloat16*>(in->xNorm),
                                 static_cast<__nv_bfloat16*>(const_cast<void*>(lnOut)), in->stdev},
                       in->mb != nullptr};
    }
    return MG_OK;
}

int block_cluster_forward(const void* lnOut, const void* wUp, const void* wDown, void* h, void* v, const LnOutputs& next,
                          int M, cudaStream_t st, const BlockClusterForwardInput* in, bool prefetch) {
    BcMaps tm;
    BcParams p;
    MG_TRY(block_cluster_forward_args(lnOut, wUp, wDown, h, v, next, M, in, tm, p));
    p.prefetch = prefetch && !in;
    return in ? launch_bc<false, 32, true>(tm, p, st) : launch_bc<false, 32>(tm, p, st);
}

int block_cluster_backward_args(const void* dS, const void* wDown, const void* v, const void* wUp, void* dV,
                                const void* lnOut, float* upPart, float* downPart, const void* xNorm,
                                const void* gamma, const float* stdev, const void* resid, void* residOut,
                                float* partial, int M, const BlockClusterInput* in, BcMaps& tm, BcParams& p) {
    MG_CHECK_ARG(dS && wDown && v && wUp && dV && lnOut && upPart && downPart && xNorm && gamma && stdev &&
                     residOut && partial,
                 "block_cluster_backward: null argument");
    MG_CHECK_ARG(M > 0 && gemm_rows_ln_backward_supported(M),
                 "block_cluster_backward: the LayerNorm backward partial groups at this row count do not divide 32 rows");
    tm = BcMaps{};
    int rc = make_tmap_bf16(&tm.a, dS, kRowsBN, M, kRowsBN, 128);
    if (!rc) rc = make_tmap_bf16(&tm.b1, wDown, kRowsBN, kBcHidden, kRowsBN, 128);
    if (!rc) rc = make_tmap_bf16(&tm.b2, wUp, kBcHidden, kRowsBN, kBcHidden, 128);
    if (!rc) rc = make_tmap_bf16(&tm.v, v, kBcHidden, M, kBcHidden, 128);
    if (!rc) rc = make_tmap_bf16(&tm.dv, dV, kBcHidden, M, kBcHidden, 128);
    if (!rc) rc = make_tmap_bf16(&tm.ln, lnOut, kRowsBN, M, kRowsBN, 128);
    if (rc) return rc;
    p = BcParams{};
    p.M = M;
    p.vOut = static_cast<__nv_bfloat16*>(dV);
    p.upPart = upPart;
    p.downPart = downPart;
    p.e.M = M;
    p.e.resid = static_cast<const __nv_bfloat16*>(resid);
    p.e.out = static_cast<__nv_bfloat16*>(residOut);
    p.e.gamma = static_cast<const __nv_bfloat16*>(gamma);
    p.e.xNorm = static_cast<const __nv_bfloat16*>(xNorm);
    p.e.stdev = stdev;
    p.e.partial = partial;
    if (in) {
        MG_CHECK_ARG(in->obs && in->partial && in->inDim > 0 && in->inDim <= kRowsInputMaxDim,
                     "block_cluster_backward: bad input-layer arguments");
        p.e.inObs = in->obs;
        p.e.inMb = in->mb;
        p.e.inEnvRows = in->envRows;
        p.e.inTotal = in->total;
        p.e.inDim = in->inDim;
        p.e.inPartial = in->partial;
    }
    p.status = status_ptr();
    p.trace = tile_trace();
    return MG_OK;
}

int block_cluster_backward(const void* dS, const void* wDown, const void* v, const void* wUp, void* dV,
                           const void* lnOut, float* upPart, float* downPart, const void* xNorm, const void* gamma,
                           const float* stdev, const void* resid, void* residOut, float* partial, int M,
                           cudaStream_t st, const BlockClusterInput* in, bool prefetch) {
    BcMaps tm;
    BcParams p;
    MG_TRY(block_cluster_backward_args(dS, wDown, v, wUp, dV, lnOut, upPart, downPart, xNorm, gamma, stdev, resid,
                                       residOut, partial, M, in, tm, p));
    p.prefetch = prefetch;
    switch (layernorm_rows_per_part(M)) {
        case 8: return launch_bc<true, 8>(tm, p, st);
        case 16: return launch_bc<true, 16>(tm, p, st);
        default: return launch_bc<true, 32>(tm, p, st);
    }
}

}  // namespace mg

extern "C" int mg_block_cluster_forward(const void* ln_out, const void* w_up, const void* w_down, void* h, void* v,
                                        const void* gamma, const void* beta, void* x_norm, void* next_ln_out,
                                        float* stdev, int rows, mg_stream_t stream) {
    const mg::LnOutputs ln{static_cast<const __nv_bfloat16*>(gamma), static_cast<const __nv_bfloat16*>(beta),
                           static_cast<__nv_bfloat16*>(x_norm), static_cast<__nv_bfloat16*>(next_ln_out), stdev};
    return mg::block_cluster_forward(ln_out, w_up, w_down, h, v, ln, rows, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int mg_block_cluster_forward_input(const float* obs, int in_dim, const void* w_in, const void* b_in,
                                              const void* gamma0, const void* beta0, void* x_norm0, void* ln_out0,
                                              float* stdev0, const void* w_up, const void* w_down, void* h, void* v,
                                              const void* gamma, const void* beta, void* x_norm, void* next_ln_out,
                                              float* stdev, int rows, mg_stream_t stream) {
    const mg::LnOutputs ln{static_cast<const __nv_bfloat16*>(gamma), static_cast<const __nv_bfloat16*>(beta),
                           static_cast<__nv_bfloat16*>(x_norm), static_cast<__nv_bfloat16*>(next_ln_out), stdev};
    const mg::BlockClusterForwardInput in{obs, nullptr, 0, 0, in_dim, w_in, b_in, gamma0, beta0, x_norm0, stdev0};
    return mg::block_cluster_forward(ln_out0, w_up, w_down, h, v, ln, rows, reinterpret_cast<cudaStream_t>(stream),
                                     &in);
}

extern "C" int mg_block_cluster_backward(const void* dS, const void* w_down, const void* v, const void* w_up, void* dV,
                                         const void* ln_out, float* up_part, float* down_part, const void* x_norm,
                                         const void* gamma, const float* stdev, const void* resid, void* resid_out,
                                         float* partial, const float* obs, int in_dim, float* in_partial, int rows,
                                         mg_stream_t stream) {
    const mg::BlockClusterInput in{obs, nullptr, 0, 0, in_dim, in_partial};
    return mg::block_cluster_backward(dS, w_down, v, w_up, dV, ln_out, up_part, down_part, x_norm, gamma, stdev,
                                      resid, resid_out, partial, rows, reinterpret_cast<cudaStream_t>(stream),
                                      obs ? &in : nullptr);
}
