// Continuous-force CartPole (Gaussian head with a learned log-std) through
// the drop-in API; rollout_cartpole_continuous ships with the library.
#include <cmath>
#include <cstdio>
#include <cstdlib>

#include "gym.h"
#include "model/ppo.h"

struct CartPoleContinuousHost {
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

int main(int argc, char** argv) {
    const uint32_t envs = 4096, horizon = 32;
    const int iterations = argc > 1 ? std::atoi(argv[1]) : 60;
    Gym<CartPoleContinuousHost> gym(envs);
    PPOModel<CartPoleContinuousHost> model(gym, 128, 4, 2, 3e-4f, horizon);
    for (int it = 0; it < iterations; it++) {
        model.collect();
        model.train();
        uint64_t ended = 0;
        for (uint32_t t = 0; t < horizon; t++)
            for (uint32_t i = 0; i < envs; i++) ended += model.slotDones(t)[i];
        const LossStats s = model.lastStats();
        std::printf("iter %3d  steps/done %7.1f  std %.3f  entropy %.3f  kl %.4f\n", it,
                    ended ? (double)envs * horizon / ended : (double)envs * horizon,
                    std::exp(model.logStdValue(0)), s.entropy, s.approxKl);
    }
    return 0;
}
