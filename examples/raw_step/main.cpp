// Raw environment stepping on the B200 through the drop-in Gym<Env>, two
// ways: the reference's loop (host actions in, rewards out, one blocking
// call per step: gym.run) and the batched device loop (gym.runN: every env
// draws its action from its own RNG and steps, `steps` times, without a host
// round trip). The host side of an environment is only its description: the
// sizes of State / Action / Obs and the name its kernels are registered
// under; VoxelNav's 1056-byte State is declared here as opaque bytes.
//   g++ -std=c++17 -O2 -I include examples/raw_step/main.cpp
//       -L metalgym_b200 -lmetalgym_b200 -Wl,-rpath,<repo>/metalgym_b200 -o raw_step
#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <vector>

#include "gym.h"

struct CartPoleDesc {
    struct State {
        float x, xDot, theta, thetaDot;
        uint32_t steps;
    };
    using Action = int;
    struct Obs {
        float v[4];
    };
    static constexpr uint32_t OBS_DIM = 4;
    static constexpr uint32_t ACT_DIM = 2;
    static constexpr const char* KERNEL = "rollout_cartpole";
};

struct VoxelNavDesc {
    struct State {
        unsigned char bytes[1056];
    };
    using Action = int;
    struct Obs {
        float v[40];
    };
    static constexpr uint32_t OBS_DIM = 40;
    static constexpr uint32_t ACT_DIM = 6;
    static constexpr const char* KERNEL = "rollout_voxelnav";
};

template <class Env>
void measure(const char* name, int envs, int hostSteps, int deviceSteps) {
    using clock = std::chrono::steady_clock;
    Gym<Env> gym(envs);
    std::vector<float> reward(envs);
    double ended = 0.0;
    const auto h0 = clock::now();
    for (int s = 0; s < hostSteps; s++) {
        for (int i = 0; i < envs; i++) gym.actions()[i] = (typename Env::Action)((i + s) % Env::ACT_DIM);
        gym.run(reward);
        for (int i = 0; i < envs; i++) ended += gym.done()[i];
    }
    const double hostS = std::chrono::duration<double>(clock::now() - h0).count();
    gym.runN(deviceSteps);  // warm-up
    const auto d0 = clock::now();
    gym.runN(deviceSteps);
    const double devS = std::chrono::duration<double>(clock::now() - d0).count();
    std::printf("%-9s %6d envs  gym.run %8.2f M steps/s (%.0f episodes ended)  runN(%d) %8.3f G steps/s\n", name,
                envs, (double)envs * hostSteps / hostS / 1e6, ended, deviceSteps,
                (double)envs * deviceSteps / devS / 1e9);
}

// usage: raw_step [envs]
int main(int argc, char** argv) {
    const int envs = argc > 1 ? std::atoi(argv[1]) : 4096;
    measure<CartPoleDesc>("CartPole", envs, 200, 1000);
    measure<VoxelNavDesc>("VoxelNav", envs, 50, 100);
    return 0;
}
