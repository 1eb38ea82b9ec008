// Test helper: the product's environment structs (include/metalgym/envs)
// compiled for the HOST, with the reference's rollout semantics (load the
// env, reset it if done, step it with the given action, store it back;
// rollout.h:31-54). CPU tests compare this bit for bit with oracle/_ref, and
// GPU tests compare the device build with both. Not part of the product.
#include <cstdint>

#include "metalgym/envs/cartpole.h"
#include "metalgym/envs/cartpole_continuous.h"
#include "metalgym/envs/voxelnav.h"

template <typename Env>
static void run(void* states, const void* actions, void* obs, float* reward, uint8_t* done, uint32_t* rng,
                uint32_t n, int threads) {
    auto* s = static_cast<typename Env::State*>(states);
    auto* a = static_cast<const typename Env::Action*>(actions);
    auto* o = static_cast<typename Env::Obs*>(obs);
#pragma omp parallel for num_threads(threads) schedule(static) if (threads > 1)
    for (int64_t i = 0; i < (int64_t)n; i++) {
        typename Env::State st = s[i];
        uint32_t w = rng[i];
        uint8_t d = done[i];
        if (d) Env::reset(st, w);
        Env::step(st, a[i], o[i], reward[i], d);
        s[i] = st;
        rng[i] = w;
        done[i] = d;
    }
}

extern "C" __attribute__((visibility("default"))) void hostenv_rollout(int which, void* states, const void* actions,
                                                                       void* obs, float* reward, uint8_t* done,
                                                                       uint32_t* rng, uint32_t n, int threads) {
    switch (which) {
        case 0: run<CartPole>(states, actions, obs, reward, done, rng, n, threads); break;
        case 1: run<CartPoleContinuous>(states, actions, obs, reward, done, rng, n, threads); break;
        case 2: run<VoxelNav>(states, actions, obs, reward, done, rng, n, threads); break;
        case 3: run<CartPoleContinuousTanh>(states, actions, obs, reward, done, rng, n, threads); break;
    }
}

extern "C" __attribute__((visibility("default"))) float hostenv_sinf(float x) { return mg_sinf(x); }
extern "C" __attribute__((visibility("default"))) float hostenv_cosf(float x) { return mg_cosf(x); }
extern "C" __attribute__((visibility("default"))) float hostenv_expf(float x) { return mg_expf(x); }
extern "C" __attribute__((visibility("default"))) float hostenv_logf(float x) { return mg_logf(x); }
extern "C" __attribute__((visibility("default"))) float hostenv_tanhf(float x) { return mg_tanhf(x); }
