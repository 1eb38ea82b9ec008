// VoxelNav (heightmap navigation with a ray-marched depth camera) through the
// drop-in API; rollout_voxelnav ships with the library.
#include <cstdio>
#include <cstdlib>

#include "gym.h"
#include "model/ppo.h"

struct VoxelNavHost {
    static constexpr uint32_t W = 32;
    static constexpr uint32_t N_RAYS = 32;
    struct State {
        float x, z, yaw;
        float gx, gz;
        float prevDist;
        uint32_t steps;
        uint32_t cobble;
        uint8_t height[W * W];
    };
    using Action = int;
    struct Obs {
        float ray[N_RAYS];
        float goalForward, goalRight, goalUp, goalDist;
        float sinYaw, cosYaw, cobble, height;
    };
    static constexpr uint32_t OBS_DIM = N_RAYS + 8;
    static constexpr uint32_t ACT_DIM = 6;
    static constexpr const char* KERNEL = "rollout_voxelnav";
};

int main(int argc, char** argv) {
    const uint32_t envs = 4096, horizon = 32;
    const int iterations = argc > 1 ? std::atoi(argv[1]) : 200;
    Gym<VoxelNavHost> gym(envs);
    PPOModel<VoxelNavHost> model(gym, 128, 4, 2, 3e-4f, horizon);
    for (int it = 0; it < iterations; it++) {
        model.collect();
        model.train();
        uint64_t episodes = 0, successes = 0;
        for (uint32_t t = 0; t < horizon; t++) {
            const uint8_t* done = model.slotDones(t);
            const float* reward = model.slotRewards(t);
            for (uint32_t i = 0; i < envs; i++)
                if (done[i]) {
                    episodes++;
                    successes += reward[i] > 5.0f;
                }
        }
        const LossStats s = model.lastStats();
        if (it % 10 == 0 || it == iterations - 1)
            std::printf("iter %3d  success %.3f  episodes %6llu  entropy %.3f\n", it,
                        episodes ? (double)successes / episodes : 0.0, (unsigned long long)episodes, s.entropy);
    }
    return 0;
}
