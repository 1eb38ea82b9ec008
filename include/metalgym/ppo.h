// PPOModel<Env>: the drop-in replacement of the reference's PPO model
// (model/ppo.h:106-1009) on the B200, over the metalgym_b200 C ABI.
//
// Same constructor PPOModel(Gym<Env>&, e, s, layers, lr, T = 32, seed = 0),
// the public hyperparameter fields (clip, valueCoef, entropyCoef,
// maxGradNorm, gamma, lambda; read on every collect / train call), and the
// methods collect(), train(epochs = 4), trainSlot(t), forward(), act(rng),
// actGreedy(), values(), logProbs(), headValue(row, col), logStdValue(k),
// setLogStd(v), slotObs/Actions/Rewards/Dones/Values/Advantages/Returns(t)
// and lastStats(). collect / train / trainSlot / forward block until the GPU
// is done, as in the reference.
//
// The policy, sampler, GAE and PPO update run on the GPU (one CUDA graph per
// collect() and per train()); act() stays host code with the caller's RNG,
// exactly as model/ppo.h:636-686, and actGreedy() runs on the device. Slot
// accessors and headValue() read pinned host mirrors refreshed after device
// work (see gym.h). Extensions: no compile-time N_EMBED_CFG (embed 64/128/256/512),
// setComm() for data parallelism over NCCL, save() / load() checkpoints of the
// training state, and the field minibatchRows
// (0, the default, keeps the reference's one-slot minibatches; B > 0 trains
// on B rollout rows per minibatch, every row once per epoch in a random
// order).
#pragma once

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <random>
#include <type_traits>
#include <vector>

#include "gym.h"

namespace metalgym {

inline float bf16_bits_to_float(uint16_t b) {
    const uint32_t u = (uint32_t)b << 16;
    float f;
    std::memcpy(&f, &u, 4);
    return f;
}

// act(rng) of model/ppo.h:636-686 over head rows [parallels][64] (bf16
// bits): per row a categorical draw from the logits with the caller's host
// generator (std::uniform_real_distribution, inverse CDF over the softmax
// weights) or ACT_DIM Gaussian draws around the means with log-std logStd
// (std::normal_distribution), the log-probability of the drawn action and
// the value column. The same calls of the same distributions in the same
// order as the reference, so the same generator state gives the same
// actions.
template <typename Env, typename Rng>
void sample_actions_host(const uint16_t* head, uint32_t parallels, const float* logStd, Rng& rng,
                         typename Env::Action* action, float* value, float* logProb) {
    constexpr uint32_t kHead = 64;
    if constexpr (!std::is_integral_v<typename Env::Action>) {
        std::normal_distribution<float> normal(0.0f, 1.0f);
        float* actionF = reinterpret_cast<float*>(action);
        for (uint32_t row = 0; row < parallels; ++row) {
            const uint16_t* h = head + (size_t)row * kHead;
            float lp = 0.0f;
            for (uint32_t k = 0; k < Env::ACT_DIM; ++k) {
                const float ls = logStd[k];
                const float mu = bf16_bits_to_float(h[k]);
                const float a = mu + std::exp(ls) * normal(rng);
                const float d = (a - mu) * std::exp(-ls);
                actionF[(size_t)row * Env::ACT_DIM + k] = a;
                lp += -0.5f * d * d - ls - 0.9189385332046727f;
            }
            logProb[row] = lp;
            value[row] = bf16_bits_to_float(h[Env::ACT_DIM]);
        }
    } else {
        std::uniform_real_distribution<float> uniform(0.0f, 1.0f);
        float logits[Env::ACT_DIM];
        for (uint32_t row = 0; row < parallels; ++row) {
            const uint16_t* h = head + (size_t)row * kHead;
            float rowMax = -INFINITY;
            for (uint32_t a = 0; a < Env::ACT_DIM; ++a) {
                logits[a] = bf16_bits_to_float(h[a]);
                rowMax = std::max(rowMax, logits[a]);
            }
            float sum = 0.0f;
            for (uint32_t a = 0; a < Env::ACT_DIM; ++a) sum += std::exp(logits[a] - rowMax);
            const float lse = rowMax + std::log(sum);
            const float u = uniform(rng) * sum;
            uint32_t chosen = Env::ACT_DIM - 1;
            float acc = 0.0f;
            for (uint32_t a = 0; a < Env::ACT_DIM; ++a) {
                acc += std::exp(logits[a] - rowMax);
                if (u < acc) {
                    chosen = a;
                    break;
                }
            }
            action[row] = (typename Env::Action)chosen;
            logProb[row] = logits[chosen] - lse;
            value[row] = bf16_bits_to_float(h[Env::ACT_DIM]);
        }
    }
}

}  // namespace metalgym

// model/ppo.h:97-104
struct LossStats {
    float policy;
    float value;
    float entropy;
    float approxKl;
    float clipFrac;
    float gradNorm;
};

template <typename Env>
struct PPOModel {
    static_assert(sizeof(typename Env::Obs) == Env::OBS_DIM * sizeof(float), "Env::Obs must be exactly OBS_DIM floats");
    static constexpr bool CONTINUOUS = !std::is_integral_v<typename Env::Action>;
    static_assert(CONTINUOUS || sizeof(typename Env::Action) == 4, "the softmax head needs a discrete 4-byte Action");
    static_assert(!CONTINUOUS || sizeof(typename Env::Action) == Env::ACT_DIM * sizeof(float),
                  "the Gaussian head needs an Action of exactly ACT_DIM floats");
    static constexpr float INIT_LOG_STD = 0.0f;
    static constexpr uint32_t HEAD_DIM = 64;
    static_assert(Env::ACT_DIM + 1 <= HEAD_DIM, "ACT_DIM + value must fit one 64-wide tile");

    Gym<Env>& gym;
    mg_ppo_t handle = nullptr;
    uint32_t parallels;
    uint32_t horizon;
    uint32_t embedDim;
    uint32_t mlpScale;
    uint32_t nLayers;
    float lr;
    uint32_t hiddenDim;

    float clip = 0.2f;
    float valueCoef = 0.5f;
    float entropyCoef = 0.01f;
    float maxGradNorm = 0.5f;  // 0 disables clipping
    float gamma = 0.99f;
    float lambda = 0.95f;
    uint32_t minibatchRows = 0;  // extension: 0 = one time slot per minibatch

    PPOModel(Gym<Env>& g, int e, int s, int layers, float learningRate, int T = 32, uint32_t seed = 0)
        : gym(g), parallels(g.parallels), horizon((uint32_t)T), embedDim((uint32_t)e), mlpScale((uint32_t)s),
          nLayers((uint32_t)layers), lr(learningRate), hiddenDim((uint32_t)(e * s)) {
        metalgym::check_or_exit(mg_ppo_create(g.handle, e, s, layers, learningRate, T, seed, &handle), "PPOModel");
        values_.assign(parallels, 0.0f);
        logProbs_.assign(parallels, 0.0f);
        const size_t R = parallels, TT = horizon;
        obsSlots_ = metalgym::host_alloc<typename Env::Obs>((TT + 1) * R);
        actionSlots_ = metalgym::host_alloc<typename Env::Action>(TT * R);
        floatSlots_ = metalgym::host_alloc<float>(5 * TT * R);
        doneSlots_ = metalgym::host_alloc<uint8_t>(TT * R);
        head_ = metalgym::host_alloc<uint16_t>(R * HEAD_DIM);
    }
    ~PPOModel() {
        mg_host_free(obsSlots_);
        mg_host_free(actionSlots_);
        mg_host_free(floatSlots_);
        mg_host_free(doneSlots_);
        mg_host_free(head_);
        mg_ppo_destroy(handle);
    }
    PPOModel(const PPOModel&) = delete;
    PPOModel& operator=(const PPOModel&) = delete;

    // ---- the hot path (model/ppo.h:716-751, 906-923)
    void collect() {
        pushHyper();
        metalgym::check_or_exit(mg_ppo_collect(handle), "collect");
        afterDeviceWork(MG_PPO_HEAD);
    }
    void train(uint32_t epochs = 4) {
        pushHyper();
        metalgym::check_or_exit(mg_ppo_train(handle, (int)epochs), "train");
        afterDeviceWork(MG_PPO_TRAIN_HEAD);
    }
    void trainSlot(uint32_t t) {
        pushHyper();
        metalgym::check_or_exit(mg_ppo_train_slot(handle, (int)t), "trainSlot");
        afterDeviceWork(MG_PPO_TRAIN_HEAD);
    }
    // policy forward on gym.obs() (model/ppo.h:628-634)
    void forward() {
        metalgym::check_or_exit(mg_ppo_forward(handle), "forward");
        afterDeviceWork(MG_PPO_HEAD);
    }

    // ---- manual stepping (model/ppo.h:636-702). act() draws on the host from
    // the caller's generator (metalgym::sample_actions_host over the head rows
    // of the last forward); actGreedy() runs on the device (mg_ppo_act_greedy)
    // and leaves the actions in gym.actions() as the host version does.
    template <typename Rng>
    void act(Rng& rng) {
        syncHead();
        float ls[Env::ACT_DIM] = {};
        if constexpr (CONTINUOUS)
            for (uint32_t k = 0; k < Env::ACT_DIM; ++k) ls[k] = logStdValue(k);
        metalgym::sample_actions_host<Env>(head_, parallels, ls, rng, gym.actions(), values(), logProbs());
    }
    // discrete: argmax; continuous: the mean
    void actGreedy() {
        metalgym::check_or_exit(mg_ppo_act_greedy(handle, headSource_, gym.actions()), "actGreedy");
    }

    // ---- observability (model/ppo.h:448-476, 925-943)
    float* values() { return values_.data(); }
    float* logProbs() { return logProbs_.data(); }
    float headValue(uint32_t row, uint32_t col) const {
        syncHead();
        uint32_t u = (uint32_t)head_[(size_t)row * HEAD_DIM + col] << 16;
        float f;
        std::memcpy(&f, &u, 4);
        return f;
    }
    float logStdValue(uint32_t k) const {
        static_assert(CONTINUOUS, "logStdValue needs a continuous Env::Action");
        float v = 0.0f;
        metalgym::check_or_exit(mg_ppo_log_std(handle, (int)k, &v), "logStdValue");
        return v;
    }
    void setLogStd(float value) {
        static_assert(CONTINUOUS, "setLogStd needs a continuous Env::Action");
        metalgym::check_or_exit(mg_ppo_set_log_std(handle, value), "setLogStd");
    }
    typename Env::Obs* slotObs(uint32_t t) {
        sync(0, MG_PPO_OBS_SLOTS, obsSlots_, (size_t)(horizon + 1) * parallels * sizeof(typename Env::Obs));
        return obsSlots_ + (size_t)t * parallels;
    }
    typename Env::Action* slotActions(uint32_t t) {
        sync(1, MG_PPO_ACTION_SLOTS, actionSlots_, (size_t)horizon * parallels * sizeof(typename Env::Action));
        return actionSlots_ + (size_t)t * parallels;
    }
    float* slotRewards(uint32_t t) { return floatSlot(0, MG_PPO_REWARD_SLOTS, t); }
    float* slotValues(uint32_t t) { return floatSlot(1, MG_PPO_VALUE_SLOTS, t); }
    float* slotAdvantages(uint32_t t) { return floatSlot(2, MG_PPO_ADV_SLOTS, t); }
    float* slotReturns(uint32_t t) { return floatSlot(3, MG_PPO_RET_SLOTS, t); }
    uint8_t* slotDones(uint32_t t) {
        sync(7, MG_PPO_DONE_SLOTS, doneSlots_, (size_t)horizon * parallels);
        return doneSlots_ + (size_t)t * parallels;
    }
    LossStats lastStats() const {
        float v[6];
        metalgym::check_or_exit(mg_ppo_last_stats(handle, v), "lastStats");
        return LossStats{v[0], v[1], v[2], v[3], v[4], v[5]};
    }

    // ---- extension: data parallelism (ncclComm_t from mg_comm_init)
    void setComm(void* comm, int rank, int world) {
        metalgym::check_or_exit(mg_ppo_set_comm(handle, comm, rank, world), "setComm");
    }
    // Extensions of data-parallel training (mg_ppo_set_allreduce_overlap,
    // mg_ppo_set_comm_timeout): the gradient all-reduce overlapped with the
    // last backward layer; a timeout after which a failed or missing peer
    // makes train() fail with MG_ERR_COMM (printed, then exit) instead of
    // blocking for good.
    void setAllreduceOverlap(bool on) {
        metalgym::check_or_exit(mg_ppo_set_allreduce_overlap(handle, on ? 1 : 0), "setAllreduceOverlap");
    }
    void setCommTimeout(float seconds) {
        metalgym::check_or_exit(mg_ppo_set_comm_timeout(handle, seconds), "setCommTimeout");
    }
    // Extension: collect() as one persistent kernel (mg_ppo_set_collect_fused;
    // environments with a State of at most 64 bytes and at most 32
    // observations, embed 128, hidden 512): true = the kernel, false = the
    // per-step graph. Without a call the library chooses (the kernel where it
    // applies, up to 4096 parallels).
    void setFusedCollect(bool on) {
        metalgym::check_or_exit(mg_ppo_set_collect_fused(handle, on ? 1 : 0), "setFusedCollect");
    }
    // Extension: checkpoint / resume of the whole training state (mg_ppo_save).
    void save(const char* path) {
        pushHyper();
        metalgym::check_or_exit(mg_ppo_save(handle, path), "save");
    }
    void load(const char* path) {
        metalgym::check_or_exit(mg_ppo_load(handle, path), "load");
        float h[6];
        metalgym::check_or_exit(mg_ppo_get_hyper(handle, h), "load");
        clip = h[0];
        valueCoef = h[1];
        entropyCoef = h[2];
        maxGradNorm = h[3];
        gamma = h[4];
        lambda = h[5];
        int rows = 0;
        metalgym::check_or_exit(mg_ppo_minibatch_rows(handle, &rows), "load");
        minibatchRows = (uint32_t)rows;
        afterDeviceWork(MG_PPO_HEAD);
    }

   private:
    void pushHyper() {
        metalgym::check_or_exit(mg_ppo_set_hyper(handle, clip, valueCoef, entropyCoef, maxGradNorm, gamma, lambda),
                                "hyperparameters");
        metalgym::check_or_exit(mg_ppo_set_minibatch_rows(handle, (int)minibatchRows), "minibatchRows");
    }
    void afterDeviceWork(int headSource) {
        for (bool& s : stale_) s = true;
        headStale_ = true;
        headSource_ = headSource;
        gym.invalidate();
    }
    void sync(int idx, int which, void* dst, size_t bytes) {
        if (!stale_[idx]) return;
        metalgym::check_or_exit(mg_ppo_download(handle, which, -1, dst, bytes), "slot download");
        stale_[idx] = false;
    }
    float* floatSlot(int k, int which, uint32_t t) {
        float* base = floatSlots_ + (size_t)k * horizon * parallels;
        sync(2 + k, which, base, (size_t)horizon * parallels * sizeof(float));
        return base + (size_t)t * parallels;
    }
    void syncHead() const {
        if (!headStale_) return;
        metalgym::check_or_exit(mg_ppo_download(handle, headSource_, -1, head_, (size_t)parallels * HEAD_DIM * 2),
                                "head download");
        headStale_ = false;
    }

    std::vector<float> values_, logProbs_;
    typename Env::Obs* obsSlots_ = nullptr;
    typename Env::Action* actionSlots_ = nullptr;
    float* floatSlots_ = nullptr;  // reward, value, advantage, return slots
    uint8_t* doneSlots_ = nullptr;
    uint16_t* head_ = nullptr;
    bool stale_[8] = {true, true, true, true, true, true, true, true};
    mutable bool headStale_ = true;
    int headSource_ = MG_PPO_HEAD;
};
