// TEST INFRASTRUCTURE ONLY (oracle). Never linked into the product.
//
// Compiles the reference's OWN Metal sources, unmodified and in place, as
// host C++ through the shim in oracle/shim/metal_stdlib, and exports each
// per-thread kernel as a plain C function that loops over the thread grid.
// The build recipe is oracle/Makefile (target `ref`); its only output is
// oracle/_ref/libmg_ref.so. Nothing here is copied from the reference: the
// sources are #included from the reference tree given as REF to make.
//
// Threadgroup kernels (layernorm, normalizeAdvantage) are run as threadgroups
// of one thread, which is a valid execution of the same source: every strided
// loop then covers the whole row serially and the simd/threadgroup reductions
// see a single partial.
#include <cmath>
#include <cstdint>
#include <cstring>

#include "metal_stdlib"

namespace ref {
#include "examples/CartPole/cartpole.metal"
#include "examples/CartPoleContinuous/cartpole_continuous.metal"
#include "examples/VoxelNav/voxelnav.metal"
}  // namespace ref

namespace src_sample {
#include "model/sample.metal"
}
namespace src_gauss {
#include "model/gaussian.metal"
}
namespace src_policy {
#include "model/policy.metal"
}
namespace src_gae {
#include "model/gae.metal"
}
namespace src_opt {
#include "model/optimizer.metal"
}
namespace src_elem {
#include "model/elementwise.metal"
}
namespace src_input {
#include "model/input.metal"
}
namespace src_ln {
#include "model/layernorm.metal"
}

#define MG_REF_API extern "C" __attribute__((visibility("default")))

// ---- environments: rollout<Env> (rollout.h:31-54) once per thread id ----
template <typename Env>
static void run_rollout(void* states, const void* actions, void* obs, float* reward, uint8_t* done,
                        uint32_t* rng, uint32_t n, int threads) {
    auto* s = static_cast<typename Env::State*>(states);
    auto* a = static_cast<const typename Env::Action*>(actions);
    auto* o = static_cast<typename Env::Obs*>(obs);
#pragma omp parallel for num_threads(threads) schedule(static) if (threads > 1)
    for (uint32_t tid = 0; tid < n; tid++) ref::rollout<Env>(s, a, o, reward, done, rng, tid);
}

MG_REF_API int ref_env_sizes(int which, uint32_t* out4) {
    switch (which) {
        case 0: out4[0] = sizeof(ref::CartPole::State); out4[1] = sizeof(ref::CartPole::Action);
                out4[2] = sizeof(ref::CartPole::Obs); out4[3] = ref::CartPole::OBS_DIM; return 0;
        case 1: out4[0] = sizeof(ref::CartPoleContinuous::State); out4[1] = sizeof(ref::CartPoleContinuous::Action);
                out4[2] = sizeof(ref::CartPoleContinuous::Obs); out4[3] = ref::CartPoleContinuous::OBS_DIM; return 0;
        case 2: out4[0] = sizeof(ref::VoxelNav::State); out4[1] = sizeof(ref::VoxelNav::Action);
                out4[2] = sizeof(ref::VoxelNav::Obs); out4[3] = ref::VoxelNav::OBS_DIM; return 0;
    }
    return -1;
}

MG_REF_API void ref_rollout(int which, void* states, const void* actions, void* obs, float* reward,
                            uint8_t* done, uint32_t* rng, uint32_t n, int threads) {
    switch (which) {
        case 0: run_rollout<ref::CartPole>(states, actions, obs, reward, done, rng, n, threads); break;
        case 1: run_rollout<ref::CartPoleContinuous>(states, actions, obs, reward, done, rng, n, threads); break;
        case 2: run_rollout<ref::VoxelNav>(states, actions, obs, reward, done, rng, n, threads); break;
    }
}

// ---- policy sampling (model/sample.metal:18-47, model/gaussian.metal:42-71) ----
MG_REF_API void ref_sample_action(const uint16_t* head, uint32_t* rng, uint32_t* action, float* logProb,
                                  float* value, uint32_t rows, uint32_t actDim, uint32_t headDim) {
    src_sample::SampleParams p{rows, actDim, headDim};
    for (uint32_t r = 0; r < rows; r++)
        src_sample::sampleAction(reinterpret_cast<const bfloat*>(head), rng, action, logProb, value, p, r);
}

MG_REF_API void ref_sample_gaussian(const uint16_t* head, uint32_t* rng, float* action, float* logProb,
                                    float* value, uint32_t rows, uint32_t actDim, uint32_t headDim,
                                    const uint16_t* logStd) {
    src_gauss::SampleParams p{rows, actDim, headDim};
    for (uint32_t r = 0; r < rows; r++)
        src_gauss::sampleGaussian(reinterpret_cast<const bfloat*>(head), rng, action, logProb, value, p,
                                  reinterpret_cast<const bfloat*>(logStd), r);
}

// ---- PPO losses (model/policy.metal:14-69, model/gaussian.metal:76-135) ----
MG_REF_API void ref_policy_loss(const uint16_t* head, const uint32_t* action, const float* advantage,
                                const float* ret, const float* oldLogProb, uint16_t* dZ, float* stats,
                                uint32_t rows, uint32_t actDim, uint32_t headDim, float clip, float valueCoef,
                                float entropyCoef) {
    src_policy::PolicyParams p{rows, actDim, headDim, clip, valueCoef, entropyCoef};
    for (uint32_t r = 0; r < rows; r++)
        src_policy::policyLossBackward(reinterpret_cast<const bfloat*>(head), action, advantage, ret, oldLogProb,
                                       reinterpret_cast<bfloat*>(dZ), stats, p, r);
}

MG_REF_API void ref_gaussian_loss(const uint16_t* head, const float* action, const float* advantage,
                                  const float* ret, const float* oldLogProb, uint16_t* dZ, float* stats,
                                  uint32_t rows, uint32_t actDim, uint32_t headDim, float clip, float valueCoef,
                                  float entropyCoef, const uint16_t* logStd, float* dLogStd) {
    src_gauss::PolicyParams p{rows, actDim, headDim, clip, valueCoef, entropyCoef};
    for (uint32_t r = 0; r < rows; r++)
        src_gauss::gaussianLossBackward(reinterpret_cast<const bfloat*>(head), action, advantage, ret, oldLogProb,
                                        reinterpret_cast<bfloat*>(dZ), stats, p,
                                        reinterpret_cast<const bfloat*>(logStd),
                                        reinterpret_cast<metal::atomic_float*>(dLogStd), r, 0);
}

// ---- GAE and advantage normalisation (model/gae.metal:14-77) ----
MG_REF_API void ref_gae(const float* reward, const uint8_t* done, const float* value, const uint16_t* bootstrapHead,
                        float* advantage, float* ret, uint32_t rows, uint32_t horizon, uint32_t headDim,
                        uint32_t actDim, float gamma, float lambda) {
    src_gae::GaeParams p{rows, horizon, headDim, actDim, gamma, lambda};
    for (uint32_t i = 0; i < rows; i++)
        src_gae::gaeBackward(reward, done, value, reinterpret_cast<const bfloat*>(bootstrapHead), advantage, ret, p, i);
}

MG_REF_API void ref_normalize_advantage(const float* adv, float* out, uint32_t rows) {
    src_gae::NormalizeParams p{rows};
    src_gae::normalizeAdvantage(adv, out, p, 0, 1, 0, 0, 1);
}

// ---- optimizer (model/optimizer.metal:23-60) ----
MG_REF_API void ref_grad_norm_sq(const float* gradF, const uint16_t* gradB, float* normSq, uint32_t count,
                                 uint32_t floatCount) {
    src_opt::AdamParams p{};
    p.count = count;
    p.floatCount = floatCount;
    uint32_t padded = (count + 31) / 32 * 32;
    for (uint32_t t = 0; t < padded; t++)
        src_opt::gradNormSq(gradF, reinterpret_cast<const bfloat*>(gradB),
                            reinterpret_cast<metal::atomic_float*>(normSq), p, t, 0);
}

MG_REF_API void ref_adam_step(float* param, const float* gradF, const uint16_t* gradB, float* momentum,
                              float* variance, uint16_t* weights, const float* normSq, uint32_t count,
                              uint32_t floatCount, float lr, float beta1Pow, float beta2Pow, float maxGradNorm) {
    src_opt::AdamParams p{count, floatCount, lr, 0.9f, 0.999f, 1e-8f, beta1Pow, beta2Pow, maxGradNorm};
    for (uint32_t t = 0; t < count; t++)
        src_opt::adamStep(param, gradF, reinterpret_cast<const bfloat*>(gradB), momentum, variance,
                          reinterpret_cast<bfloat*>(weights), normSq, p, t);
}

// ---- elementwise (model/elementwise.metal) ----
MG_REF_API void ref_residual_add(const uint16_t* a, const uint16_t* b, uint16_t* out, uint32_t count) {
    for (uint32_t t = 0; t < count; t++)
        src_elem::residualAdd(reinterpret_cast<const bfloat*>(a), reinterpret_cast<const bfloat*>(b),
                              reinterpret_cast<bfloat*>(out), count, t);
}

MG_REF_API void ref_reduce_partials(const float* part, uint16_t* out, uint32_t len, uint32_t chunks) {
    src_elem::ReduceParams p{len, chunks};
    for (uint32_t t = 0; t < len; t++) src_elem::reducePartials(part, reinterpret_cast<bfloat*>(out), p, t);
}

// ---- input projection (model/input.metal) ----
MG_REF_API void ref_input_forward(const float* obs, const uint16_t* w, const uint16_t* bias, uint16_t* out,
                                  uint32_t rows, uint32_t inDim, uint32_t outDim) {
    src_input::InputParams p{rows, inDim, outDim};
    for (uint32_t r = 0; r < rows; r++)
        for (uint32_t c = 0; c < outDim; c++)
            src_input::inputForward(obs, reinterpret_cast<const bfloat*>(w), reinterpret_cast<const bfloat*>(bias),
                                    reinterpret_cast<bfloat*>(out), p, metal::uint2{c, r});
}

MG_REF_API void ref_input_backward(const float* obs, const uint16_t* dZ, float* dW, float* dBias, uint32_t rows,
                                   uint32_t inDim, uint32_t outDim, uint32_t chunkRows) {
    src_input::InputBackwardParams p{rows, inDim, outDim, chunkRows};
    uint32_t chunks = (rows + chunkRows - 1) / chunkRows;
    for (uint32_t y = 0; y < chunks; y++)
        for (uint32_t x = 0; x < (inDim + 1) * outDim; x++)
            src_input::inputBackward(obs, reinterpret_cast<const bfloat*>(dZ),
                                     reinterpret_cast<metal::atomic_float*>(dW),
                                     reinterpret_cast<metal::atomic_float*>(dBias), p, metal::uint2{x, y});
}

// ---- layernorm (model/layernorm.metal), one-thread threadgroups ----
MG_REF_API void ref_layernorm_forward(const uint16_t* x, uint16_t* xNorm, uint16_t* out, const uint16_t* gamma,
                                      const uint16_t* beta, float* stdev, uint32_t rows, uint32_t cols) {
    src_ln::LayernormParams p{rows, cols, 1, 1e-5f};
    for (uint32_t g = 0; g < rows; g++)
        src_ln::layernormForward(reinterpret_cast<const bfloat*>(x), reinterpret_cast<bfloat*>(xNorm),
                                 reinterpret_cast<bfloat*>(out), reinterpret_cast<const bfloat*>(gamma),
                                 reinterpret_cast<const bfloat*>(beta), stdev, p, 0, g, 0, 0, 1, 1);
}

MG_REF_API void ref_layernorm_backward(uint16_t* dZ, const uint16_t* xNorm, const uint16_t* gamma,
                                       const float* stdev, uint16_t* dxNorm, float* dGamma, float* dBeta,
                                       uint32_t rows, uint32_t cols) {
    src_ln::LayernormParams p{rows, cols, 1, 1e-5f};
    for (uint32_t g = 0; g < rows; g++)
        src_ln::layernormBackward(reinterpret_cast<bfloat*>(dZ), reinterpret_cast<const bfloat*>(xNorm),
                                  reinterpret_cast<const bfloat*>(gamma), stdev, reinterpret_cast<bfloat*>(dxNorm),
                                  reinterpret_cast<metal::atomic_float*>(dGamma),
                                  reinterpret_cast<metal::atomic_float*>(dBeta), p, 0, g, 0, 0, 1, 1);
}
