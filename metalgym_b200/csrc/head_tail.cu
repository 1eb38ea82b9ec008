// The head kernel of a training minibatch (128-wide embeddings, categorical
// head): the head GEMM, the PPO loss, the head dX, the final LayerNorm
// backward and the dW_head tile partials in one kernel, four CTAs per 128-row
// tile, each running the pass of head_tail.cuh once (where the arithmetic is
// described). Three launches and a side-stream GEMM become one kernel on 128
// CTAs at 4096 rows, bit-identical to them.
#include "head_tail.cuh"
#include "runtime.h"

namespace mg {

namespace {

template <int RPC, int AD>
__global__ void __launch_bounds__(kRowsThreads, 1)
    k_head_tail(const __grid_constant__ CUtensorMap tmF, const __grid_constant__ CUtensorMap tmW,
                const HeadTailParams p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    if (threadIdx.x == 0) {
        prefetch_tensormap(&tmF);
        prefetch_tensormap(&tmW);
    }
    TilePass t = tp_setup(smem + kHtBar, 256, false);
    mg_pdl_wait();
    // dependents start only now, after this kernel's predecessor completed
    // (the block backward kernels load their weights before their own wait)
    mg_pdl_trigger();
    ht_pass<RPC, AD>(smem, tmF, tmW, p, t);
}

template <int RPC>
int launch_ht(const CUtensorMap& tf, const CUtensorMap& tw, const HeadTailParams& p, cudaStream_t st) {
    // two actions (CartPole): the loss with its loops unrolled
    auto kern = p.loss.actDim == 2 ? k_head_tail<RPC, 2> : k_head_tail<RPC, 0>;
    static std::atomic<uint64_t> attr_done[2] = {};  // per kernel variant
    if (int rc = smem_limit_once(kern, kHtSmem, attr_done[p.loss.actDim == 2 ? 1 : 0])) return rc;
    const int grid = ((p.M + kRowsBM - 1) / kRowsBM) * 4;
    MG_CUDA_TRY(mg_launch(kern, dim3(grid), dim3(kRowsThreads), (size_t)kHtSmem, st, tf, tw, p));
    return check_launch("k_head_tail");
}

}  // namespace

bool head_tail_supported(int E, int M) { return E == kRowsBN && M > 0 && gemm_rows_ln_backward_supported(M); }

int head_tail_args(const void* fOut, const void* wHead, void* head, const PolicyLossRows& loss, float* headPart,
                   const void* gammaF, const void* xNormF, const float* stdevF, void* dS, float* lnPart, int M,
                   CUtensorMap& tf, CUtensorMap& tw, HeadTailParams& p) {
    MG_CHECK_ARG(fOut && wHead && head && headPart && gammaF && xNormF && stdevF && dS && lnPart && loss.dZ &&
                     loss.stats,
                 "head_tail: null argument");
    MG_CHECK_ARG(M > 0 && M == loss.rows && loss.actDim >= 1 && loss.actDim < kLossHeadDim,
                 "head_tail: bad shape");
    MG_CHECK_ARG(gemm_rows_ln_backward_supported(M),
                 "head_tail: the LayerNorm backward partial groups at this row count do not divide 32 rows");
    int rc = make_tmap_bf16(&tf, fOut, kRowsBN, M, kRowsBN, 128);
    if (!rc) rc = make_tmap_bf16(&tw, wHead, kLossHeadDim, kRowsBN, kLossHeadDim, 128);
    if (rc) return rc;
    p = HeadTailParams{};
    p.M = M;
    p.loss = loss;
    p.head = static_cast<__nv_bfloat16*>(head);
    p.headPart = headPart;
    p.e.M = M;
    p.e.resid = nullptr;
    p.e.out = static_cast<__nv_bfloat16*>(dS);
    p.e.gamma = static_cast<const __nv_bfloat16*>(gammaF);
    p.e.xNorm = static_cast<const __nv_bfloat16*>(xNormF);
    p.e.stdev = stdevF;
    p.e.partial = lnPart;
    p.status = status_ptr();
    p.trace = tile_trace();
    return MG_OK;
}

int head_tail(const void* fOut, const void* wHead, void* head, const PolicyLossRows& loss, float* headPart,
              const void* gammaF, const void* xNormF, const float* stdevF, void* dS, float* lnPart, int M,
              cudaStream_t st) {
    CUtensorMap tf, tw;
    HeadTailParams p;
    MG_TRY(head_tail_args(fOut, wHead, head, loss, headPart, gammaF, xNormF, stdevF, dS, lnPart, M, tf, tw, p));
    switch (layernorm_rows_per_part(M)) {
        case 8: return launch_ht<8>(tf, tw, p, st);
        case 16: return launch_ht<16>(tf, tw, p, st);
        default: return launch_ht<32>(tf, tw, p, st);
    }
}

}  // namespace mg

extern "C" int mg_head_tail(const void* f_out, const void* w_head, void* head, const int32_t* action,
                            const float* adv, const float* adv_stats, const float* ret, const float* old_log_prob,
                            void* dZ, float* stats, int rows, int act_dim, float clip, float value_coef,
                            float entropy_coef, float* head_part, const void* gamma_f, const void* x_norm_f,
                            const float* stdev_f, void* dS, float* ln_partial, mg_stream_t stream) {
    const mg::PolicyLossRows L = mg::policy_loss_rows(action, adv, adv_stats, ret, old_log_prob, dZ, stats, rows,
                                                      act_dim, mg::LossHyper{clip, value_coef, entropy_coef},
                                                      mg::RowMap{nullptr, 0, 0});
    return mg::head_tail(f_out, w_head, head, L, head_part, gamma_f, x_norm_f, stdev_f, dS, ln_partial, rows,
                         reinterpret_cast<cudaStream_t>(stream));
}
