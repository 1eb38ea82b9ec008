// Checkpoint and resume of PPO training on the B200 (save() / load(), an
// extension of the drop-in PPOModel: the parameters, Adam moments and step
// counter, the host shuffle generator, the last rollout observation and the
// gym's env states, done flags and RNG words). Two identical CartPoleContinuous
// trainings run side by side; one is saved after a few iterations and a third
// model, built with a different seed, loads that checkpoint. From there the
// resumed model must train exactly as the one that kept going.
//   g++ -std=c++17 -O2 -I include examples/checkpoint_resume/main.cpp
//       -L metalgym_b200 -lmetalgym_b200 -Wl,-rpath,<repo>/metalgym_b200 -o checkpoint_resume
#include <cstdio>
#include <cstring>

#include "gym.h"
#include "model/ppo.h"

struct CartPoleContinuousDesc {
    struct State {
        float x, xDot, theta, thetaDot;
        uint32_t steps;
    };
    struct Action {
        float force;
    };
    struct Obs {
        float v[4];
    };
    static constexpr uint32_t OBS_DIM = 4;
    static constexpr uint32_t ACT_DIM = 1;
    static constexpr const char* KERNEL = "rollout_cartpole_continuous";
};
using Env = CartPoleContinuousDesc;

// usage: checkpoint_resume [checkpoint file]
int main(int argc, char** argv) {
    const char* path = argc > 1 ? argv[1] : "checkpoint_resume.bin";
    const int envs = 2048, horizon = 16;
    Gym<Env> gymKept(envs), gymSaved(envs);
    PPOModel<Env> kept(gymKept, 128, 4, 2, 3e-4f, horizon);
    PPOModel<Env> saved(gymSaved, 128, 4, 2, 3e-4f, horizon);
    for (int it = 0; it < 3; it++) {
        kept.collect();
        kept.train();
        saved.collect();
        saved.train();
    }
    saved.save(path);

    Gym<Env> gymResumed(envs, /*seed*/ 7);
    PPOModel<Env> resumed(gymResumed, 128, 4, 2, 3e-4f, horizon, /*seed*/ 99);
    resumed.load(path);
    bool identical = true;
    for (int it = 0; it < 2; it++) {
        kept.collect();
        kept.train();
        resumed.collect();
        resumed.train();
        const LossStats a = kept.lastStats(), b = resumed.lastStats();
        identical = identical && std::memcmp(&a, &b, sizeof(LossStats)) == 0;
        std::printf("iteration %d after the checkpoint: policy %.6f / %.6f  value %.6f / %.6f  log_std %.4f / %.4f\n",
                    it, a.policy, b.policy, a.value, b.value, kept.logStdValue(0), resumed.logStdValue(0));
    }
    std::printf("resumed training %s\n", identical ? "identical" : "DIFFERENT");
    std::remove(path);
    return identical ? 0 : 1;
}
