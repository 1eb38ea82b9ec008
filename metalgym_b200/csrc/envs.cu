// Environment registry and the by-name C-ABI wrappers around the kernels
// that MG_REGISTER_ENV instantiates (include/metalgym/register_env.cuh).
#include <cstring>
#include <mutex>
#include <string>

#include "collect_fused.h"
#include "metalgym/pdl.cuh"
#include "metalgym/rng.h"
#include "runtime.h"

namespace mg {
namespace {

constexpr int kMaxEnvs = 64;

struct Registry {
    std::mutex mu;
    const mg_env_ops* ops[kMaxEnvs] = {};
    int n = 0;
};

Registry& registry() {
    static Registry r;
    return r;
}

// gym.h:54-61: done = 1 (the first step resets every env), one seeded
// xorshift word per env.
__global__ void k_env_init(uint8_t* done, uint32_t* rng, int n, uint32_t seed, uint32_t first) {
    mg_pdl_trigger();
    mg_pdl_wait();
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    done[i] = 1;
    rng[i] = mgSeedWord(seed, first + (uint32_t)i);
}

const mg_env_ops* find_or_fail(const char* name) {
    const mg_env_ops* o = mg_env_find(name);
    if (!o) fail(MG_ERR_NOT_FOUND, std::string("no environment registered as '") + (name ? name : "(null)") + "'");
    return o;
}

}  // namespace
}  // namespace mg

extern "C" {

int mg_env_register(const mg_env_ops* ops) {
    if (!ops || !ops->name || ops->abi_version != MG_VERSION) return mg::fail(MG_ERR_ARGUMENT, "mg_env_register: bad ops");
    auto& r = mg::registry();
    std::lock_guard<std::mutex> lock(r.mu);
    for (int i = 0; i < r.n; i++) {
        if (std::strcmp(r.ops[i]->name, ops->name) == 0) {
            r.ops[i] = ops;
            return MG_OK;
        }
    }
    if (r.n >= mg::kMaxEnvs) return mg::fail(MG_ERR_ARGUMENT, "mg_env_register: registry full");
    r.ops[r.n++] = ops;
    return MG_OK;
}

const mg_env_ops* mg_env_find(const char* kernel_name) {
    if (!kernel_name) return nullptr;
    auto& r = mg::registry();
    std::lock_guard<std::mutex> lock(r.mu);
    for (int i = 0; i < r.n; i++)
        if (std::strcmp(r.ops[i]->name, kernel_name) == 0) return r.ops[i];
    return nullptr;
}

int mg_env_count(void) {
    auto& r = mg::registry();
    std::lock_guard<std::mutex> lock(r.mu);
    return r.n;
}

const char* mg_env_name(int i) {
    auto& r = mg::registry();
    std::lock_guard<std::mutex> lock(r.mu);
    return (i >= 0 && i < r.n) ? r.ops[i]->name : nullptr;
}

int mg_env_init(const char* kernel_name, void* states, uint8_t* done, uint32_t* rng, int n, uint32_t seed,
                uint32_t first_env_id, mg_stream_t stream) {
    const mg_env_ops* o = mg::find_or_fail(kernel_name);
    if (!o) return MG_ERR_NOT_FOUND;
    MG_CHECK_ARG(states && done && rng && n > 0, "mg_env_init: bad arguments");
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    MG_CUDA_TRY(cudaMemsetAsync(states, 0, (size_t)n * o->state_bytes, st));
    MG_LAUNCH(mg::k_env_init, (n + 255) / 256, 256, 0, st, done, rng, n, seed, first_env_id);
    return mg::check_launch("k_env_init");
}

int mg_env_step(const char* kernel_name, void* states, const void* actions, void* obs, float* reward, uint8_t* done,
                uint8_t* done_copy, uint32_t* rng, int n, mg_stream_t stream) {
    const mg_env_ops* o = mg::find_or_fail(kernel_name);
    if (!o) return MG_ERR_NOT_FOUND;
    int rc = o->step(states, actions, obs, reward, done, done_copy, rng, n, stream);
    return rc ? mg::fail(rc, rc == MG_ERR_ARGUMENT ? "mg_env_step: bad arguments" : "env step launch failed") : MG_OK;
}

int mg_env_run_random(const char* kernel_name, void* states, void* obs_ring, float* reward_ring, uint8_t* done_ring,
                      uint8_t* done, uint32_t* rng, int n, int steps, int ring, int mode, mg_stream_t stream) {
    const mg_env_ops* o = mg::find_or_fail(kernel_name);
    if (!o) return MG_ERR_NOT_FOUND;
    int rc = o->run_random(states, obs_ring, reward_ring, done_ring, done, rng, n, steps, ring, mode, stream);
    return rc ? mg::fail(rc, rc == MG_ERR_ARGUMENT ? "mg_env_run_random: bad arguments" : "env run_random launch failed")
              : MG_OK;
}

int mg_env_collect_step(const char* kernel_name, const void* head, const void* log_std, void* states,
                        void* action_out, float* logp_out, float* value_out, void* obs_out, float* reward_out,
                        uint8_t* done, uint8_t* done_slot, uint32_t* rng, int n, mg_stream_t stream) {
    const mg_env_ops* o = mg::find_or_fail(kernel_name);
    if (!o) return MG_ERR_NOT_FOUND;
    int rc = o->collect_step(head, log_std, states, action_out, logp_out, value_out, obs_out, reward_out, done,
                             done_slot, rng, n, stream);
    return rc ? mg::fail(rc, rc == MG_ERR_ARGUMENT ? "mg_env_collect_step: bad arguments"
                                                : "env collect_step launch failed")
              : MG_OK;
}

int mg_env_collect_fused(const char* kernel_name, const mg_collect_fused_args* args, mg_stream_t stream) {
    MG_CHECK_ARG(args, "mg_env_collect_fused: null arguments");
    const mg_env_ops* o = mg::find_or_fail(kernel_name);
    if (!o) return MG_ERR_NOT_FOUND;
    if (!o->collect_fused)
        return mg::fail(MG_ERR_UNSUPPORTED, std::string("mg_env_collect_fused: '") + kernel_name +
                                                "' has no fused collect kernel (State over 64 bytes or over 32 "
                                                "observations)");
    MG_CHECK_ARG(args->layers >= 1 && args->layers <= MG_COLLECT_FUSED_MAX_BLOCKS,
                 "mg_env_collect_fused: layers must be in [1, 4]");
    mg::CollectFusedArgs a{};
    a.R = args->parallels;
    a.T = args->horizon;
    a.L = args->layers;
    a.inDim = args->obs_dim;
    a.wIn = args->w_in;
    a.bIn = args->b_in;
    for (int l = 0; l <= args->layers; l++) {
        a.lnGamma[l] = args->ln_gamma[l];
        a.lnBeta[l] = args->ln_beta[l];
    }
    for (int l = 0; l < args->layers; l++) {
        a.wUp[l] = args->w_up[l];
        a.wDown[l] = args->w_down[l];
    }
    a.wHead = args->w_head;
    a.logStd = args->log_std;
    a.states = args->states;
    a.done = args->done;
    a.rng = args->rng;
    a.obsSlots = args->obs_slots;
    a.actionSlots = args->action_slots;
    a.logpSlots = args->logp_slots;
    a.valueSlots = args->value_slots;
    a.rewardSlots = args->reward_slots;
    a.doneSlots = args->done_slots;
    a.advSlots = args->adv_slots;
    a.retSlots = args->ret_slots;
    a.bootHead = args->boot_head;
    a.gamma = args->gamma;
    a.lambda = args->lambda;
    MG_CHECK_ARG(!o->continuous || a.logStd, "mg_env_collect_fused: a continuous environment needs log_std");
    return mg::collect_fused(o, a, reinterpret_cast<cudaStream_t>(stream));
}

}  // extern "C"
