// Environment registration: the device-side replacement of the reference's
// per-environment kernel instantiation
//     template [[host_name("rollout_cartpole")]] kernel void rollout<CartPole>(...);
// (rollout.h:31-54, README.md:42-52). Compile a .cu translation unit that
// includes this header and the environment, then write
//     MG_REGISTER_ENV(CartPole)
// at file scope. That instantiates the three environment kernels below for
// the type, and (for a State of at most 64 bytes and at most 32 observation
// floats) the persistent collect() kernel of detail/collect_fused.cuh, and
// registers them, at load time, under Env::KERNEL with the metalgym_b200
// library (mg_env_register), where Gym<Env> and PPOModel<Env> find them by
// name. The translation unit is compiled for sm_100a.
//
// Compile such translation units with nvcc --fmad=false so environment
// arithmetic rounds every multiply and add separately (bit-exact with the
// same environment compiled as host C++ with -ffp-contract=off).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <type_traits>

#include "../metalgym_b200.h"
#include "detail/collect_fused.cuh"
#include "env_traits.cuh"
#include "pdl.cuh"
#include "sampling.cuh"

namespace mg {

// rollout<Env> (rollout.h:31-54): load, reset if done, step, store.
// doneCopy (optional) also receives the new done flag (the per-slot copy
// model/ppo.h:731-732 makes with a blit).
template <class Env>
__global__ void env_step_kernel(typename Env::State* states, const typename Env::Action* actions,
                                typename Env::Obs* obs, float* reward, uint8_t* done, uint8_t* doneCopy, uint32_t* rng,
                                int n) {
    mg_pdl_trigger();
    mg_pdl_wait();
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    uint32_t w = rng[i];
    uint8_t d = done[i];
    float r;
    if constexpr (EnvTraits<Env>::kInPlace) {
        typename Env::State& s = states[i];
        if (d) Env::reset(s, w);
        Env::step(s, actions[i], obs[i], r, d);
    } else {
        typename Env::State s = states[i];
        typename Env::Obs o;
        if (d) Env::reset(s, w);
        Env::step(s, actions[i], o, r, d);
        states[i] = s;
        obs[i] = o;
    }
    reward[i] = r;
    done[i] = d;
    if (doneCopy) doneCopy[i] = d;
    rng[i] = w;
}

// `steps` env steps per thread with the benchmark's random policy, drawn
// before the reset / step on the same word (the order collect() uses). Step
// k's obs / reward / done go to slot k % ring of the ring buffers.
template <class Env>
__global__ void env_run_random_kernel(typename Env::State* states, typename Env::Obs* obsRing, float* rewardRing,
                                      uint8_t* doneRing, uint8_t* done, uint32_t* rng, int n, int steps, int ring,
                                      int mode) {
    mg_pdl_trigger();
    mg_pdl_wait();
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    uint32_t w = rng[i];
    uint8_t d = done[i];
    typename Env::State local;
    typename Env::State* sp;
    if constexpr (EnvTraits<Env>::kInPlace) {
        sp = &states[i];
    } else {
        local = states[i];
        sp = &local;
    }
    for (int k = 0; k < steps; k++) {
        const typename Env::Action a = draw_random_action<Env>(w, mode);
        if (d) Env::reset(*sp, w);
        const size_t slot = (size_t)(k % ring) * n + i;
        float r;
        if constexpr (EnvTraits<Env>::kInPlace) {
            Env::step(*sp, a, obsRing[slot], r, d);
        } else {
            typename Env::Obs o;
            Env::step(*sp, a, o, r, d);
            obsRing[slot] = o;
        }
        rewardRing[slot] = r;
        doneRing[slot] = d;
    }
    if constexpr (!EnvTraits<Env>::kInPlace) states[i] = local;
    done[i] = d;
    rng[i] = w;
}

// One collect() step for env row i, fused: draw the action from this row of
// the policy head (model/sample.metal or model/gaussian.metal), record
// action / log-prob / value in slot t, then reset-if-done and step the env
// with it (rollout.h:31-54) and record obs t+1, reward t and done t
// (model/ppo.h:727-733: sample, encodeStep, done copy).
template <class Env>
__global__ void env_collect_step_kernel(const __nv_bfloat16* head, const __nv_bfloat16* logStd,
                                        typename Env::State* states, typename Env::Action* actionOut, float* logpOut,
                                        float* valueOut, typename Env::Obs* obsOut, float* rewardOut, uint8_t* done,
                                        uint8_t* doneSlot, uint32_t* rng, int n) {
    mg_pdl_trigger();
    mg_pdl_wait();
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    uint32_t w = rng[i];
    float lp, v;
    const typename Env::Action a = draw_policy_action<Env>(head + (size_t)i * kHeadDim, logStd, w, lp, v);
    actionOut[i] = a;
    logpOut[i] = lp;
    valueOut[i] = v;
    uint8_t d = done[i];
    float r;
    if constexpr (EnvTraits<Env>::kInPlace) {
        typename Env::State& s = states[i];
        if (d) Env::reset(s, w);
        Env::step(s, a, obsOut[i], r, d);
    } else {
        typename Env::State s = states[i];
        typename Env::Obs o;
        if (d) Env::reset(s, w);
        Env::step(s, a, o, r, d);
        states[i] = s;
        obsOut[i] = o;
    }
    rewardOut[i] = r;
    done[i] = d;
    doneSlot[i] = d;
    rng[i] = w;
}

template <class Env>
struct EnvLaunchers {
    using T = EnvTraits<Env>;
    static constexpr int kBlock = T::kInPlace ? 64 : 128;
    static int grid(int n) { return (n + kBlock - 1) / kBlock; }

    static int step(void* states, const void* actions, void* obs, float* reward, uint8_t* done, uint8_t* doneCopy,
                    uint32_t* rng, int n, mg_stream_t s) {
        if (n <= 0 || !states || !actions || !obs || !reward || !done || !rng) return MG_ERR_ARGUMENT;
        MG_LAUNCH(env_step_kernel<Env>, grid(n), kBlock, 0, reinterpret_cast<cudaStream_t>(s), 
            static_cast<typename T::State*>(states), static_cast<const typename T::Action*>(actions),
            static_cast<typename T::Obs*>(obs), reward, done, doneCopy, rng, n);
        return cudaGetLastError() == cudaSuccess ? MG_OK : MG_ERR_CUDA;
    }
    static int run_random(void* states, void* obsRing, float* rewardRing, uint8_t* doneRing, uint8_t* done,
                          uint32_t* rng, int n, int steps, int ring, int mode, mg_stream_t s) {
        if (n <= 0 || steps < 0 || ring <= 0 || !states || !obsRing || !rewardRing || !doneRing || !done || !rng)
            return MG_ERR_ARGUMENT;
        MG_LAUNCH(env_run_random_kernel<Env>, grid(n), kBlock, 0, reinterpret_cast<cudaStream_t>(s), 
            static_cast<typename T::State*>(states), static_cast<typename T::Obs*>(obsRing), rewardRing, doneRing,
            done, rng, n, steps, ring, mode);
        return cudaGetLastError() == cudaSuccess ? MG_OK : MG_ERR_CUDA;
    }
    static int collect_step(const void* head, const void* logStd, void* states, void* actionOut, float* logpOut,
                            float* valueOut, void* obsOut, float* rewardOut, uint8_t* done, uint8_t* doneSlot,
                            uint32_t* rng, int n, mg_stream_t s) {
        if (n <= 0 || !head || (T::kContinuous && !logStd) || !states || !actionOut || !logpOut || !valueOut ||
            !obsOut || !rewardOut || !done || !doneSlot || !rng)
            return MG_ERR_ARGUMENT;
        MG_LAUNCH(env_collect_step_kernel<Env>, grid(n), kBlock, 0, reinterpret_cast<cudaStream_t>(s), 
            static_cast<const __nv_bfloat16*>(head), static_cast<const __nv_bfloat16*>(logStd),
            static_cast<typename T::State*>(states), static_cast<typename T::Action*>(actionOut), logpOut, valueOut,
            static_cast<typename T::Obs*>(obsOut), rewardOut, done, doneSlot, rng, n);
        return cudaGetLastError() == cudaSuccess ? MG_OK : MG_ERR_CUDA;
    }
    static mg_env_ops ops() {
        mg_env_ops o{};
        o.abi_version = MG_VERSION;
        o.name = Env::KERNEL;
        o.state_bytes = (uint32_t)sizeof(typename T::State);
        o.action_bytes = (uint32_t)sizeof(typename T::Action);
        o.obs_bytes = (uint32_t)sizeof(typename T::Obs);
        o.obs_dim = Env::OBS_DIM;
        o.act_dim = Env::ACT_DIM;
        o.continuous = T::kContinuous ? 1u : 0u;
        o.step = &step;
        o.run_random = &run_random;
        o.collect_step = &collect_step;
        if constexpr (collect_fused_eligible<Env>()) o.collect_fused = &collect_fused_launch<Env>;
        return o;
    }
};

}  // namespace mg

#define MG_ENV_CONCAT_(a, b) a##b
#define MG_ENV_CONCAT(a, b) MG_ENV_CONCAT_(a, b)
#define MG_REGISTER_ENV(EnvType)                                                          \
    namespace {                                                                           \
    struct MG_ENV_CONCAT(mg_env_registrar_, __LINE__) {                                   \
        MG_ENV_CONCAT(mg_env_registrar_, __LINE__)() {                                    \
            static const mg_env_ops ops = ::mg::EnvLaunchers<EnvType>::ops();              \
            mg_env_register(&ops);                                                        \
        }                                                                                 \
    } MG_ENV_CONCAT(mg_env_registrar_instance_, __LINE__);                                \
    }
