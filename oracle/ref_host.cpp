// TEST INFRASTRUCTURE ONLY. The reference's own host code (gym.h and
// model/ppo.h, included unmodified from the reference tree) compiled for the
// CPU through the metal-cpp stand-in of oracle/shim_host/, where buffers are
// host memory and GPU work is a no-op. The reference's host-side methods then
// run exactly as written on buffers the tests fill:
//   the PPOModel constructor's seeded parameter init and layout
//     (model/ppo.h:274-446),
//   act(rng) and actGreedy() on given head rows (model/ppo.h:636-702),
//   setLogStd / logStdValue (model/ppo.h:454-469),
//   lastStats() over given per-row statistics (model/ppo.h:925-943).
// Built by `make -C oracle ref-host REF=<reference tree>` into
// oracle/_ref/libmg_ref_host.so; nothing of it is linked into the product.
#include <cstdint>
#include <cstring>
#include <random>

#include "gym.h"
#include "model/ppo.h"

namespace {

// Host mirrors of the example environments (examples/*/main.cpp): the
// environment interface the reference's host code is instantiated with.
struct HostCartPole {
    struct State {
        float x, xDot, theta, thetaDot;
        uint32_t steps;
    };
    using Action = int;
    struct Obs {
        float x, xDot, theta, thetaDot;
    };
    static constexpr uint32_t OBS_DIM = 4;
    static constexpr uint32_t ACT_DIM = 2;
    static constexpr const char* KERNEL = "rollout_cartpole";
};
struct HostCartPoleContinuous {
    struct State {
        float x, xDot, theta, thetaDot;
        uint32_t steps;
    };
    struct Action {
        float force;
    };
    struct Obs {
        float x, xDot, theta, thetaDot;
    };
    static constexpr uint32_t OBS_DIM = 4;
    static constexpr uint32_t ACT_DIM = 1;
    static constexpr const char* KERNEL = "rollout_cartpole_continuous";
};

struct HandleBase {
    int kind;
    virtual ~HandleBase() = default;
};
template <class Env>
struct Handle : HandleBase {
    Gym<Env> gym;
    PPOModel<Env> model;
    Handle(int parallels, int e, int s, int layers, float lr, int T, uint32_t seed)
        : gym(parallels), model(gym, e, s, layers, lr, T, seed) {}
};

template <class Env>
Handle<Env>* as(void* h) {
    return static_cast<Handle<Env>*>(static_cast<HandleBase*>(h));
}

template <class F>
void dispatch(void* h, F&& f) {
    if (static_cast<HandleBase*>(h)->kind == 0)
        f(*as<HostCartPole>(h));
    else
        f(*as<HostCartPoleContinuous>(h));
}

}  // namespace

extern "C" {

// kind 0: CartPole (categorical head), 1: CartPoleContinuous (Gaussian head).
// The reference requires parallels a multiple of 64 and embed 128.
__attribute__((visibility("default"))) void* ref_host_create(int kind, int parallels, int e, int s, int layers,
                                                             float lr, int T, uint32_t seed) {
    HandleBase* h = nullptr;
    if (kind == 0)
        h = new Handle<HostCartPole>(parallels, e, s, layers, lr, T, seed);
    else
        h = new Handle<HostCartPoleContinuous>(parallels, e, s, layers, lr, T, seed);
    h->kind = kind;
    return h;
}

__attribute__((visibility("default"))) void ref_host_destroy(void* h) { delete static_cast<HandleBase*>(h); }

// out[0] = optCount, out[1] = optFloatCount, out[2] = number of parameters
__attribute__((visibility("default"))) void ref_host_sizes(void* h, uint64_t* out) {
    dispatch(h, [&](auto& x) {
        out[0] = x.model.optCount;
        out[1] = x.model.optFloatCount;
        out[2] = x.model.params.size();
    });
}

// The weight arena (bf16 bits) and the fp32 master after construction.
__attribute__((visibility("default"))) void ref_host_params(void* h, uint16_t* weights, float* master) {
    dispatch(h, [&](auto& x) {
        std::memcpy(weights, x.model.weightArena->contents(), x.model.optCount * 2);
        std::memcpy(master, x.model.parameterBuffer->contents(), x.model.optCount * 4);
    });
}

// Parameter i's element offset and count in the arenas.
__attribute__((visibility("default"))) void ref_host_param_info(void* h, uint32_t i, uint64_t* offset,
                                                                uint64_t* count) {
    dispatch(h, [&](auto& x) {
        *offset = x.model.params[i].offset;
        *count = x.model.params[i].count;
    });
}

// Head rows [parallels][64] (bf16 bits) into the model's logits buffer, as a
// forward() would leave them.
__attribute__((visibility("default"))) void ref_host_set_head(void* h, const uint16_t* head) {
    dispatch(h, [&](auto& x) {
        std::memcpy(x.model.logitsBuffer->contents(), head, (size_t)x.model.parallels * 64 * 2);
    });
}

// `calls` calls of act(rng) with one std::mt19937(seed); the outputs of the
// last call: actions (int32 or float), values, log-probabilities.
__attribute__((visibility("default"))) void ref_host_act(void* h, uint32_t seed, int calls, void* actions,
                                                         float* values, float* logp) {
    dispatch(h, [&](auto& x) {
        std::mt19937 rng(seed);
        for (int c = 0; c < calls; c++) x.model.act(rng);
        const uint32_t n = x.model.parallels;
        std::memcpy(actions, x.gym.actions(), n * sizeof(*x.gym.actions()));
        std::memcpy(values, x.model.values(), n * 4);
        std::memcpy(logp, x.model.logProbs(), n * 4);
    });
}

__attribute__((visibility("default"))) void ref_host_act_greedy(void* h, void* actions) {
    dispatch(h, [&](auto& x) {
        x.model.actGreedy();
        std::memcpy(actions, x.gym.actions(), x.model.parallels * sizeof(*x.gym.actions()));
    });
}

__attribute__((visibility("default"))) void ref_host_set_log_std(void* h, float v) {
    as<HostCartPoleContinuous>(h)->model.setLogStd(v);
}

__attribute__((visibility("default"))) float ref_host_log_std(void* h, int k) {
    return as<HostCartPoleContinuous>(h)->model.logStdValue((uint32_t)k);
}

// lastStats() over per-row statistics rows [parallels][5] and the squared
// gradient norm: {policy, value, entropy, approxKl, clipFrac, gradNorm}.
__attribute__((visibility("default"))) void ref_host_last_stats(void* h, const float* rows, float normSq,
                                                                float* out6) {
    dispatch(h, [&](auto& x) {
        std::memcpy(x.model.statsBuffer->contents(), rows, (size_t)x.model.parallels * 5 * 4);
        static_cast<float*>(x.model.normSqBuffer->contents())[0] = normSq;
        const LossStats s = x.model.lastStats();
        out6[0] = s.policy;
        out6[1] = s.value;
        out6[2] = s.entropy;
        out6[3] = s.approxKl;
        out6[4] = s.clipFrac;
        out6[5] = s.gradNorm;
    });
}

}  // extern "C"
