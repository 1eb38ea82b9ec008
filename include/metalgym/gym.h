// Gym<Env>: the drop-in replacement of the reference's env runtime
// (gym.h:15-121) on the B200, over the metalgym_b200 C ABI.
//
// Same constructor, members and methods: Gym(int p), `parallels`, obs(),
// actions(), done(), run(std::vector<float>& reward). Env is the host-side
// description the reference's examples already write (State, Action, Obs,
// OBS_DIM, ACT_DIM, KERNEL); its kernels must be registered under
// Env::KERNEL (the library registers rollout_cartpole,
// rollout_cartpole_continuous and rollout_voxelnav; other environments are
// registered with MG_REGISTER_ENV, include/metalgym/register_env.cuh).
//
// Memory: the env buffers live on the GPU. obs(), actions() and done()
// return pinned host mirrors instead of views of unified memory: actions()
// is uploaded by every run(); obs() and done() are refreshed from the device
// when they are called after device work, so read them again after each
// step instead of keeping the pointer across steps.
// Errors: configuration errors print a message and exit(1), as the
// reference's constructor does (gym.h:65-69).
#pragma once

#include <algorithm>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <iostream>
#include <vector>

#include "../metalgym_b200.h"

namespace metalgym {

inline void check_or_exit(int rc, const char* what) {
    if (rc != MG_OK) {
        std::cerr << what << ": " << mg_last_error() << "\n";
        std::exit(1);
    }
}

template <typename T>
T* host_alloc(size_t count) {
    void* p = nullptr;
    check_or_exit(mg_host_alloc(count * sizeof(T), &p), "pinned host allocation");
    return static_cast<T*>(p);
}

}  // namespace metalgym

template <typename Env>
struct Gym {
    static_assert(sizeof(typename Env::Obs) == Env::OBS_DIM * sizeof(float), "Env::Obs must be exactly OBS_DIM floats");

    mg_gym_t handle = nullptr;
    uint32_t parallels;

    explicit Gym(int p, uint32_t seed = 0, uint32_t firstEnvId = 0, int device = -1) : parallels((uint32_t)p) {
        metalgym::check_or_exit(mg_gym_create(Env::KERNEL, p, seed, firstEnvId, device, &handle), Env::KERNEL);
        uint32_t info[8];
        metalgym::check_or_exit(mg_gym_info(handle, info), "gym info");
        if (info[1] != sizeof(typename Env::State) || info[2] != sizeof(typename Env::Action) ||
            info[3] != sizeof(typename Env::Obs)) {
            std::cerr << "Gym: the host struct sizes of " << Env::KERNEL
                      << " do not match the registered environment\n";
            std::exit(1);
        }
        obsHost_ = metalgym::host_alloc<typename Env::Obs>(parallels);
        actionsHost_ = metalgym::host_alloc<typename Env::Action>(parallels);
        doneHost_ = metalgym::host_alloc<uint8_t>(parallels);
    }
    ~Gym() {
        mg_host_free(obsHost_);
        mg_host_free(actionsHost_);
        mg_host_free(doneHost_);
        mg_gym_destroy(handle);
    }
    Gym(const Gym&) = delete;
    Gym& operator=(const Gym&) = delete;

    // written by the host before run(); run() uploads it
    typename Env::Action* actions() { return actionsHost_; }
    uint8_t* done() {
        if (doneStale_) {
            metalgym::check_or_exit(mg_gym_download(handle, MG_GYM_DONE, doneHost_, parallels), "gym.done");
            doneStale_ = false;
        }
        return doneHost_;
    }
    typename Env::Obs* obs() {
        if (obsStale_) {
            metalgym::check_or_exit(
                mg_gym_download(handle, MG_GYM_OBS, obsHost_, (size_t)parallels * sizeof(typename Env::Obs)), "gym.obs");
            obsStale_ = false;
        }
        return obsHost_;
    }

    // gym.h:110-121: one step of every env with actions(); blocks and copies
    // reward.size() rewards out.
    void run(std::vector<float>& reward) {
        const int n = (int)std::min<size_t>(reward.size(), parallels);
        metalgym::check_or_exit(mg_gym_run(handle, actionsHost_, reward.data(), n), "gym.run");
        invalidate();
    }

    // Extension: `steps` device-side steps with the random policy (mode 0:
    // uniform categorical / standard normal from the env's RNG; mode 1: action 0).
    void runN(int steps, int mode = 0) {
        metalgym::check_or_exit(mg_gym_run_random(handle, steps, mode), "gym.runN");
        metalgym::check_or_exit(mg_gym_synchronize(handle), "gym.runN");
        invalidate();
    }

    // The mirrors are re-read on the next obs() / done() (after device work).
    void invalidate() {
        obsStale_ = true;
        doneStale_ = true;
    }

   private:
    typename Env::Obs* obsHost_ = nullptr;
    typename Env::Action* actionsHost_ = nullptr;
    uint8_t* doneHost_ = nullptr;
    bool obsStale_ = true;
    bool doneStale_ = true;
};
