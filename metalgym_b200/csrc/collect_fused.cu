// The host side of collect() as one persistent kernel: the tensor maps of
// the weight slices and the kernel parameters, handed to the launcher the
// environment registered (mg_env_ops::collect_fused, instantiated by
// MG_REGISTER_ENV from include/metalgym/detail/collect_fused.cuh, where the
// kernel and its design are described).
#include "collect_fused.h"
#include "runtime.h"

namespace mg {

bool collect_fused_supported(const mg_env_ops* ops, int E, int H, int L, int inDim) {
    return ops && ops->collect_fused && E == kCfE && H == kCfH && L >= 1 && L <= kCollectFusedMaxBlocks &&
           inDim == (int)ops->obs_dim && inDim <= kCollectFusedMaxInputDim;
}

int collect_fused(const mg_env_ops* ops, const CollectFusedArgs& a, cudaStream_t st) {
    MG_CHECK_ARG(ops && ops->collect_fused, "collect_fused: the environment registered no fused collect kernel");
    MG_CHECK_ARG(a.R > 0 && a.T > 0 && a.L >= 1 && a.L <= kCollectFusedMaxBlocks && a.inDim == (int)ops->obs_dim,
                 "collect_fused: bad shape");
    MG_CHECK_ARG(a.wIn && a.bIn && a.wHead && a.states && a.done && a.rng && a.obsSlots && a.actionSlots &&
                     a.logpSlots && a.valueSlots && a.rewardSlots && a.doneSlots && a.advSlots && a.retSlots &&
                     a.bootHead,
                 "collect_fused: null argument");
    MG_CHECK_ARG((reinterpret_cast<uintptr_t>(a.wIn) & 15) == 0 && (reinterpret_cast<uintptr_t>(a.bootHead) & 15) == 0,
                 "collect_fused: input weights and head rows must be 16-byte aligned");
    CfMaps tm{};
    CfParams p{};
    int rc = MG_OK;
    for (int l = 0; l < a.L && !rc; l++) {
        MG_CHECK_ARG(a.wUp[l] && a.wDown[l] && a.lnGamma[l] && a.lnBeta[l], "collect_fused: null block weights");
        rc = make_tmap_bf16(&tm.up[l], a.wUp[l], kCfH, kCfE, kCfH, 64);
        if (!rc) rc = make_tmap_bf16(&tm.down[l], a.wDown[l], kCfE, kCfH, kCfE, 64);
        p.lnG[l] = static_cast<const __nv_bfloat16*>(a.lnGamma[l]);
        p.lnB[l] = static_cast<const __nv_bfloat16*>(a.lnBeta[l]);
    }
    MG_CHECK_ARG(a.lnGamma[a.L] && a.lnBeta[a.L], "collect_fused: null final LayerNorm");
    if (!rc) rc = make_tmap_bf16(&tm.head, a.wHead, kCfHeadCols, kCfE, kCfHeadCols, 128);
    if (rc) return rc;
    p.lnG[a.L] = static_cast<const __nv_bfloat16*>(a.lnGamma[a.L]);
    p.lnB[a.L] = static_cast<const __nv_bfloat16*>(a.lnBeta[a.L]);
    p.R = a.R;
    p.T = a.T;
    p.L = a.L;
    p.wIn = static_cast<const __nv_bfloat16*>(a.wIn);
    p.bIn = static_cast<const __nv_bfloat16*>(a.bIn);
    p.logStd = static_cast<const __nv_bfloat16*>(a.logStd);
    p.states = a.states;
    p.done = a.done;
    p.rng = a.rng;
    p.obsSlots = a.obsSlots;
    p.actionSlots = a.actionSlots;
    p.logpSlots = a.logpSlots;
    p.valueSlots = a.valueSlots;
    p.rewardSlots = a.rewardSlots;
    p.doneSlots = a.doneSlots;
    p.advSlots = a.advSlots;
    p.retSlots = a.retSlots;
    p.bootHead = static_cast<__nv_bfloat16*>(a.bootHead);
    p.gamma = a.gamma;
    p.lambda = a.lambda;
    p.status = status_ptr();
    const int rc2 = ops->collect_fused(&tm, &p, reinterpret_cast<mg_stream_t>(st));
    if (rc2) return fail(rc2, "collect_fused: launch of the environment's fused collect kernel failed");
    return MG_OK;
}

}  // namespace mg
