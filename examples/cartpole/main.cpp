// CartPole trained with PPO on the B200 through the drop-in API: the host
// side of an environment is only its description (sizes, dims and the name
// its kernels are registered under); the library ships rollout_cartpole.
//   g++ -std=c++17 -O2 -I include examples/cartpole/main.cpp
//       -L metalgym_b200 -lmetalgym_b200 -Wl,-rpath,<repo>/metalgym_b200 -o cartpole
#include <cstdio>
#include <cstdlib>
#include <cstring>

#include "gym.h"
#include "model/ppo.h"

struct CartPoleHost {
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

// usage: cartpole [iterations] [fused]   ("fused": collect() as one persistent kernel)
int main(int argc, char** argv) {
    const uint32_t envs = 4096, horizon = 32;
    const int iterations = argc > 1 ? std::atoi(argv[1]) : 40;
    Gym<CartPoleHost> gym(envs);
    PPOModel<CartPoleHost> model(gym, 128, 4, 2, 3e-4f, horizon);
    if (argc > 2 && std::strcmp(argv[2], "fused") == 0) model.setFusedCollect(true);
    for (int it = 0; it < iterations; it++) {
        model.collect();
        uint64_t ended = 0;
        for (uint32_t t = 0; t < horizon; t++)
            for (uint32_t i = 0; i < envs; i++) ended += model.slotDones(t)[i];
        model.train();
        const LossStats s = model.lastStats();
        std::printf("iter %3d  episode length %7.1f  entropy %.3f  kl %.4f  grad %.3f\n", it,
                    ended ? (double)envs * horizon / ended : (double)envs * horizon, s.entropy, s.approxKl,
                    s.gradNorm);
    }
    // manual stepping: greedy evaluation with the host-side sampler path
    model.forward();
    model.actGreedy();
    std::vector<float> reward(envs);
    gym.run(reward);
    std::printf("greedy step reward %.1f  obs[0].theta %.4f\n", reward[0], gym.obs()[0].theta);
    return 0;
}
