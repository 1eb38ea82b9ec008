// Compile-time properties of an environment type and the action draws the
// environment kernels share (register_env.cuh, detail/collect_fused.cuh).
#pragma once

#include <cuda_bf16.h>
#include <stdint.h>

#include <type_traits>

#include "sampling.cuh"

namespace mg {

template <class Env>
struct EnvTraits {
    using State = typename Env::State;
    using Action = typename Env::Action;
    using Obs = typename Env::Obs;
    static constexpr bool kContinuous = !std::is_integral<Action>::value;
    // Large states (e.g. a 1 KB heightmap) are stepped in place in global
    // memory instead of being copied into registers / local memory.
    static constexpr bool kInPlace = sizeof(State) > 64;
    static_assert(sizeof(Obs) == Env::OBS_DIM * sizeof(float), "Env::Obs must be exactly OBS_DIM floats");
    static_assert(kContinuous || sizeof(Action) == 4, "a discrete Env::Action must be a 4-byte integer");
    static_assert(!kContinuous || sizeof(Action) == Env::ACT_DIM * sizeof(float),
                  "a continuous Env::Action must be exactly ACT_DIM floats");
    static_assert(Env::ACT_DIM + 1 <= (uint32_t)kHeadDim, "ACT_DIM + value must fit the 64-wide head");
};

// The policy-side draw of one action for env row i (sample.metal / gaussian.metal).
template <class Env>
__device__ __forceinline__ typename Env::Action draw_policy_action(const __nv_bfloat16* headRow,
                                                                   const __nv_bfloat16* logStd, uint32_t& w,
                                                                   float& lp, float& v) {
    typename Env::Action a;
    if constexpr (EnvTraits<Env>::kContinuous) {
        sample_gaussian_row(headRow, logStd, (int)Env::ACT_DIM, w, reinterpret_cast<float*>(&a), lp, v);
    } else {
        a = (typename Env::Action)sample_categorical_row(headRow, (int)Env::ACT_DIM, w, lp, v);
    }
    return a;
}

// The random policy of the raw-step benchmark: the policy draw with an
// all-zero head (mode 0), or a constant zero action (mode 1, the action the
// reference benchmark leaves in the buffer).
template <class Env>
__device__ __forceinline__ typename Env::Action draw_random_action(uint32_t& w, int mode) {
    typename Env::Action a;
    if constexpr (EnvTraits<Env>::kContinuous) {
        float* f = reinterpret_cast<float*>(&a);
        if (mode == 1) {
            for (uint32_t k = 0; k < Env::ACT_DIM; k++) f[k] = 0.0f;
        } else {
            __nv_bfloat16 zeros[Env::ACT_DIM + 1];  // head row (means, value) and log-std, all 0
            for (auto& z : zeros) z = __float2bfloat16_rn(0.0f);
            float lp, v;
            sample_gaussian_row(zeros, zeros, (int)Env::ACT_DIM, w, f, lp, v);
        }
    } else {
        a = mode == 1 ? (typename Env::Action)0 : (typename Env::Action)uniform_action(w, (int)Env::ACT_DIM);
    }
    return a;
}

}  // namespace mg
