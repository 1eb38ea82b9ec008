// The host sampler of the drop-in PPOModel::act (metalgym::sample_actions_host,
// include/metalgym/ppo.h) as C functions for the tests, instantiated for the
// CartPole and CartPoleContinuous host mirrors; compared with the reference's
// own act() (oracle/ref_host.cpp) on the same head rows and generator seed.
#include <cstdint>
#include <random>

#include "metalgym/ppo.h"

namespace {

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

}  // namespace

// kind 0: CartPole, 1: CartPoleContinuous; `calls` calls with one
// std::mt19937(seed), the outputs of the last one.
extern "C" void host_act(int kind, const uint16_t* head, uint32_t parallels, const float* logStd, uint32_t seed,
                         int calls, void* actions, float* values, float* logp) {
    std::mt19937 rng(seed);
    for (int c = 0; c < calls; c++) {
        if (kind == 0)
            metalgym::sample_actions_host<HostCartPole>(head, parallels, logStd, rng, static_cast<int*>(actions),
                                                        values, logp);
        else
            metalgym::sample_actions_host<HostCartPoleContinuous>(
                head, parallels, logStd, rng, static_cast<HostCartPoleContinuous::Action*>(actions), values, logp);
    }
}
