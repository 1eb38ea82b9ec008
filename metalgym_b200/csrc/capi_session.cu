// C ABI of the gym / PPO sessions (mg_gym_*, mg_ppo_*, mg_comm_*, mg_host_*).
#include <dlfcn.h>
#include <nccl.h>

#include <cstdlib>
#include <cstring>
#include <string>

#include "engine.h"
#include "runtime.h"

using mg::GymCore;
using mg::PpoEngine;

namespace {

GymCore* G(mg_gym_t g) { return reinterpret_cast<GymCore*>(g); }
PpoEngine* P(mg_ppo_t m) { return reinterpret_cast<PpoEngine*>(m); }

int gym_buffer(GymCore* g, int which, void** p, size_t* bytes) {
    const size_t n = (size_t)g->n;
    switch (which) {
        case MG_GYM_STATES: *p = g->states; *bytes = n * g->ops->state_bytes; return MG_OK;
        case MG_GYM_ACTIONS: *p = g->actions; *bytes = n * g->ops->action_bytes; return MG_OK;
        case MG_GYM_OBS: *p = g->obs; *bytes = n * g->ops->obs_bytes; return MG_OK;
        case MG_GYM_REWARD: *p = g->reward; *bytes = n * 4; return MG_OK;
        case MG_GYM_DONE: *p = g->done; *bytes = n; return MG_OK;
        case MG_GYM_RNG: *p = g->rng; *bytes = n * 4; return MG_OK;
    }
    return mg::fail(MG_ERR_ARGUMENT, "unknown gym buffer id");
}

int ppo_buffer(PpoEngine* e, int which, int slot, void** p, size_t* bytes) {
    const size_t R = (size_t)e->R, T = (size_t)e->T;
    auto slotted = [&](void* base, size_t elemBytes, size_t nslots) -> int {
        if (slot < -1 || slot >= (int)nslots) return mg::fail(MG_ERR_ARGUMENT, "slot index out of range");
        if (slot < 0) {
            *p = base;
            *bytes = R * elemBytes * nslots;
        } else {
            *p = static_cast<char*>(base) + (size_t)slot * R * elemBytes;
            *bytes = R * elemBytes;
        }
        return MG_OK;
    };
    switch (which) {
        case MG_PPO_OBS_SLOTS: return slotted(e->obsSlots, (size_t)e->O * 4, T + 1);
        case MG_PPO_ACTION_SLOTS: return slotted(e->actionSlots, e->actBytes, T);
        case MG_PPO_LOGP_SLOTS: return slotted(e->logpSlots, 4, T);
        case MG_PPO_VALUE_SLOTS: return slotted(e->valueSlots, 4, T);
        case MG_PPO_REWARD_SLOTS: return slotted(e->rewardSlots, 4, T);
        case MG_PPO_DONE_SLOTS: return slotted(e->doneSlots, 1, T);
        case MG_PPO_ADV_SLOTS: return slotted(e->advSlots, 4, T);
        case MG_PPO_RET_SLOTS: return slotted(e->retSlots, 4, T);
        case MG_PPO_HEAD: *p = e->collectActs.head; *bytes = R * 64 * 2; return MG_OK;
        case MG_PPO_WEIGHTS: *p = e->weights; *bytes = e->optCount * 2; return MG_OK;
        case MG_PPO_MASTER: *p = e->master; *bytes = e->optCount * 4; return MG_OK;
        case MG_PPO_MOMENTUM: *p = e->mom; *bytes = e->optCount * 4; return MG_OK;
        case MG_PPO_VARIANCE: *p = e->var; *bytes = e->optCount * 4; return MG_OK;
        case MG_PPO_GRAD: *p = e->grad; *bytes = e->optCount * 4; return MG_OK;
        case MG_PPO_STATS: *p = e->stats; *bytes = (size_t)e->trainBufRows * 5 * 4; return MG_OK;
        case MG_PPO_ADV_STATS: *p = e->advStats; *bytes = T * 2 * 4; return MG_OK;
        case MG_PPO_TRAIN_HEAD: *p = e->trainActs.head; *bytes = (size_t)e->trainBufRows * 64 * 2; return MG_OK;
    }
    return mg::fail(MG_ERR_ARGUMENT, "unknown model buffer id");
}

int copy_checked(void* dst, const void* src, size_t bytes, size_t avail, cudaMemcpyKind kind, cudaStream_t st) {
    MG_CHECK_ARG(bytes <= avail, "copy larger than the buffer");
    MG_CUDA_TRY(cudaStreamSynchronize(st));
    MG_CUDA_TRY(cudaMemcpy(dst, src, bytes, kind));
    return MG_OK;
}

}  // namespace

extern "C" {

// ------------------------------------------------------------------ gym

int mg_gym_create(const char* kernel_name, int parallels, uint32_t seed, uint32_t first_env_id, int device,
                  mg_gym_t* out) {
    MG_CHECK_ARG(out, "mg_gym_create: null output");
    GymCore* g = nullptr;
    int rc = mg::gym_create(kernel_name, parallels, seed, first_env_id, device, &g);
    if (rc) return rc;
    *out = reinterpret_cast<mg_gym_t>(g);
    return MG_OK;
}

int mg_gym_destroy(mg_gym_t gym) {
    const bool busy = G(gym) && G(gym)->stillBusy();
    delete G(gym);
    if (busy)
        return mg::fail(MG_ERR_COMM, "mg_gym_destroy: the stream of an aborted all-reduce is still running; "
                                     "its device buffers were left allocated");
    return MG_OK;
}

int mg_gym_info(mg_gym_t gym, uint32_t out[8]) {
    GymCore* g = G(gym);
    MG_CHECK_ARG(g && out, "mg_gym_info: null argument");
    out[0] = (uint32_t)g->n;
    out[1] = g->ops->state_bytes;
    out[2] = g->ops->action_bytes;
    out[3] = g->ops->obs_bytes;
    out[4] = g->ops->obs_dim;
    out[5] = g->ops->act_dim;
    out[6] = g->ops->continuous;
    out[7] = (uint32_t)g->device;
    return MG_OK;
}

// gym.h:110-121: one step with the actions given by the host, rewards back.
int mg_gym_run(mg_gym_t gym, const void* actions_host, float* reward_host, int reward_count) {
    GymCore* g = G(gym);
    MG_CHECK_ARG(g && reward_count >= 0 && reward_count <= g->n, "mg_gym_run: bad arguments");
    MG_CHECK_ARG(reward_count == 0 || reward_host, "mg_gym_run: null reward buffer");
    MG_CUDA_TRY(cudaSetDevice(g->device));
    cudaStream_t st = g->stream;
    if (actions_host)
        MG_CUDA_TRY(cudaMemcpyAsync(g->actions, actions_host, (size_t)g->n * g->ops->action_bytes,
                                    cudaMemcpyHostToDevice, st));
    int rc = g->ops->step(g->states, g->actions, g->obs, g->reward, g->done, nullptr, g->rng, g->n,
                          reinterpret_cast<mg_stream_t>(st));
    if (rc) return mg::fail(rc, "env step launch failed");
    if (reward_count > 0)
        MG_CUDA_TRY(cudaMemcpyAsync(reward_host, g->reward, (size_t)reward_count * 4, cudaMemcpyDeviceToHost, st));
    MG_CUDA_TRY(cudaStreamSynchronize(st));
    return MG_OK;
}

int mg_gym_run_random(mg_gym_t gym, int steps, int mode) {
    GymCore* g = G(gym);
    MG_CHECK_ARG(g && steps >= 0 && (mode == 0 || mode == 1), "mg_gym_run_random: bad arguments");
    if (steps == 0) return MG_OK;
    MG_CUDA_TRY(cudaSetDevice(g->device));
    cudaStream_t st = g->stream;
    constexpr int kRing = 32;
    if (!g->obsRing) {
        MG_CUDA_TRY(cudaMalloc(&g->obsRing, (size_t)kRing * g->n * g->ops->obs_bytes));
        MG_CUDA_TRY(cudaMalloc(reinterpret_cast<void**>(&g->rewardRing), (size_t)kRing * g->n * 4));
        MG_CUDA_TRY(cudaMalloc(reinterpret_cast<void**>(&g->doneRing), (size_t)kRing * g->n));
        g->ringSlots = kRing;
    }
    int rc = g->ops->run_random(g->states, g->obsRing, g->rewardRing, g->doneRing, g->done, g->rng, g->n, steps,
                                g->ringSlots, mode, reinterpret_cast<mg_stream_t>(st));
    if (rc) return mg::fail(rc, "run_random launch failed");
    // the live obs / reward are those of the last step
    const size_t last = (size_t)((steps - 1) % g->ringSlots);
    MG_CUDA_TRY(cudaMemcpyAsync(g->obs, static_cast<char*>(g->obsRing) + last * g->n * g->ops->obs_bytes,
                                (size_t)g->n * g->ops->obs_bytes, cudaMemcpyDeviceToDevice, st));
    MG_CUDA_TRY(cudaMemcpyAsync(g->reward, g->rewardRing + last * g->n, (size_t)g->n * 4, cudaMemcpyDeviceToDevice,
                                st));
    return MG_OK;
}

int mg_gym_buffer(mg_gym_t gym, int which, void** dev_ptr, size_t* bytes) {
    MG_CHECK_ARG(gym && dev_ptr && bytes, "mg_gym_buffer: null argument");
    return gym_buffer(G(gym), which, dev_ptr, bytes);
}

int mg_gym_download(mg_gym_t gym, int which, void* host, size_t bytes) {
    MG_CHECK_ARG(gym && host, "mg_gym_download: null argument");
    void* p;
    size_t n;
    int rc = gym_buffer(G(gym), which, &p, &n);
    if (rc) return rc;
    MG_CUDA_TRY(cudaSetDevice(G(gym)->device));
    return copy_checked(host, p, bytes, n, cudaMemcpyDeviceToHost, G(gym)->stream);
}

int mg_gym_upload(mg_gym_t gym, int which, const void* host, size_t bytes) {
    MG_CHECK_ARG(gym && host, "mg_gym_upload: null argument");
    void* p;
    size_t n;
    int rc = gym_buffer(G(gym), which, &p, &n);
    if (rc) return rc;
    MG_CUDA_TRY(cudaSetDevice(G(gym)->device));
    return copy_checked(p, host, bytes, n, cudaMemcpyHostToDevice, G(gym)->stream);
}

int mg_gym_stream(mg_gym_t gym, mg_stream_t* out) {
    MG_CHECK_ARG(gym && out, "mg_gym_stream: null argument");
    *out = reinterpret_cast<mg_stream_t>(G(gym)->stream);
    return MG_OK;
}

int mg_gym_synchronize(mg_gym_t gym) {
    MG_CHECK_ARG(gym, "mg_gym_synchronize: null gym");
    MG_CUDA_TRY(cudaStreamSynchronize(G(gym)->stream));
    return MG_OK;
}

// ------------------------------------------------------------------ PPO

int mg_ppo_create(mg_gym_t gym, int embed, int scale, int layers, float lr, int horizon, uint32_t seed,
                  mg_ppo_t* out) {
    MG_CHECK_ARG(gym && out, "mg_ppo_create: null argument");
    PpoEngine* e = new PpoEngine(G(gym), embed, scale, layers, lr, horizon, seed);
    int rc = e->init();
    if (rc) {
        std::string msg = mg_last_error();
        delete e;
        return mg::fail(rc, msg);
    }
    *out = reinterpret_cast<mg_ppo_t>(e);
    return MG_OK;
}

int mg_ppo_destroy(mg_ppo_t model) {
    const bool busy = P(model) && P(model)->gym && P(model)->gym->stillBusy();
    delete P(model);
    if (busy)
        return mg::fail(MG_ERR_COMM, "mg_ppo_destroy: the stream of an aborted all-reduce is still running; "
                                     "the model's device buffers were left allocated");
    return MG_OK;
}

int mg_ppo_info(mg_ppo_t model, uint64_t out[12]) {
    PpoEngine* e = P(model);
    MG_CHECK_ARG(e && out, "mg_ppo_info: null argument");
    const uint64_t v[12] = {(uint64_t)e->R, (uint64_t)e->O, (uint64_t)e->A, (uint64_t)e->E, (uint64_t)e->H,
                            (uint64_t)e->L, (uint64_t)e->T, e->optCount, e->optFloatCount, e->params.size(),
                            (uint64_t)e->cont, (uint64_t)e->actBytes};
    std::memcpy(out, v, sizeof(v));
    return MG_OK;
}

int mg_ppo_param_info(mg_ppo_t model, int i, uint64_t* offset, uint32_t* count, int* grad_is_float) {
    PpoEngine* e = P(model);
    MG_CHECK_ARG(e && i >= 0 && i < (int)e->params.size(), "mg_ppo_param_info: bad index");
    if (offset) *offset = e->params[i].offset;
    if (count) *count = e->params[i].count;
    if (grad_is_float) *grad_is_float = e->params[i].gradIsFloat ? 1 : 0;
    return MG_OK;
}

int mg_ppo_collect(mg_ppo_t model) { return model ? P(model)->collect() : mg::fail(MG_ERR_ARGUMENT, "null model"); }
int mg_ppo_train(mg_ppo_t model, int epochs) {
    return model ? P(model)->train(epochs) : mg::fail(MG_ERR_ARGUMENT, "null model");
}
int mg_ppo_train_slot(mg_ppo_t model, int t) {
    return model ? P(model)->trainSlot(t) : mg::fail(MG_ERR_ARGUMENT, "null model");
}
int mg_ppo_p2p_handle(mg_ppo_t model, void* out64) {
    return model ? P(model)->p2pHandle(out64) : mg::fail(MG_ERR_ARGUMENT, "null model");
}
int mg_ppo_p2p_open(mg_ppo_t model, const void* handles, int rank, int world) {
    return model ? P(model)->p2pOpen(handles, rank, world) : mg::fail(MG_ERR_ARGUMENT, "null model");
}
int mg_ppo_save(mg_ppo_t model, const char* path) {
    return model ? P(model)->save(path) : mg::fail(MG_ERR_ARGUMENT, "null model");
}
int mg_ppo_load(mg_ppo_t model, const char* path) {
    return model ? P(model)->load(path) : mg::fail(MG_ERR_ARGUMENT, "null model");
}
int mg_ppo_set_minibatch_rows(mg_ppo_t model, int rows) {
    return model ? P(model)->setMinibatchRows(rows) : mg::fail(MG_ERR_ARGUMENT, "null model");
}
int mg_ppo_minibatch_rows(mg_ppo_t model, int* out) {
    MG_CHECK_ARG(model && out, "mg_ppo_minibatch_rows: null argument");
    *out = P(model)->mbRows;
    return MG_OK;
}
int mg_ppo_phase_ms(mg_ppo_t model, float out2[2]) {
    MG_CHECK_ARG(model && out2, "mg_ppo_phase_ms: null argument");
    out2[0] = P(model)->lastCollectMs;
    out2[1] = P(model)->lastTrainMs;
    return MG_OK;
}
int mg_ppo_set_comm_timeout(mg_ppo_t model, float seconds) {
    MG_CHECK_ARG(model && seconds >= 0.0f, "mg_ppo_set_comm_timeout: null model or negative timeout");
    P(model)->commTimeout = seconds;
    return MG_OK;
}
int mg_ppo_set_allreduce_overlap(mg_ppo_t model, int on) {
    MG_CHECK_ARG(model && (on == 0 || on == 1), "mg_ppo_set_allreduce_overlap: null model or on not 0 / 1");
    return P(model)->setAllreduceOverlap(on != 0);
}
int mg_ppo_set_collect_fused(mg_ppo_t model, int on) {
    MG_CHECK_ARG(model && on >= -1 && on <= 1, "mg_ppo_set_collect_fused: null model or on not -1 / 0 / 1");
    return P(model)->setCollectMode(on);
}
int mg_ppo_collect_fused(mg_ppo_t model, int* out) {
    MG_CHECK_ARG(model && out, "mg_ppo_collect_fused: null argument");
    *out = P(model)->useFusedCollect() ? 1 : 0;
    return MG_OK;
}
int mg_ppo_act_greedy(mg_ppo_t model, int head_source, void* actions_host) {
    MG_CHECK_ARG(model, "mg_ppo_act_greedy: null model");
    return P(model)->actGreedy(head_source, actions_host);
}
int mg_ppo_set_fused_minibatch(mg_ppo_t model, int on) {
    MG_CHECK_ARG(model && (on == 0 || on == 1), "mg_ppo_set_fused_minibatch: null model or on not 0 / 1");
    return P(model)->setFusedMinibatch(on != 0);
}
int mg_ppo_fused_minibatch(mg_ppo_t model, int* out) {
    MG_CHECK_ARG(model && out, "mg_ppo_fused_minibatch: null argument");
    *out = P(model)->fusedMinibatch ? 1 : 0;
    return MG_OK;
}
int mg_ppo_train_rows(mg_ppo_t model, const uint32_t key[4], uint32_t base) {
    MG_CHECK_ARG(model && key, "mg_ppo_train_rows: null argument");
    return P(model)->trainRows(key, base);
}
int mg_minibatch_rows(const uint32_t key[4], uint32_t base, uint32_t rows, uint64_t total, uint64_t* out) {
    MG_CHECK_ARG(key && out, "mg_minibatch_rows: null argument");
    MG_CHECK_ARG(total > 0 && (uint64_t)base + rows <= total, "mg_minibatch_rows: base + rows exceeds total");
    MgMinibatch m{};
    for (int i = 0; i < 4; i++) m.key[i] = key[i];
    m.base = base;
    m.slot = -1;
    for (uint32_t q = 0; q < rows; q++) out[q] = mg_minibatch_row(m, q, 0, total);
    return MG_OK;
}
int mg_ppo_forward(mg_ppo_t model) { return model ? P(model)->forward() : mg::fail(MG_ERR_ARGUMENT, "null model"); }
int mg_ppo_last_stats(mg_ppo_t model, float out6[6]) {
    MG_CHECK_ARG(model && out6, "mg_ppo_last_stats: null argument");
    return P(model)->lastStats(out6);
}

int mg_ppo_set_hyper(mg_ppo_t model, float clip, float value_coef, float entropy_coef, float max_grad_norm,
                     float gamma, float lambda) {
    MG_CHECK_ARG(model, "mg_ppo_set_hyper: null model");
    mg::PpoHyper& h = P(model)->hp;
    h.clip = clip;
    h.valueCoef = value_coef;
    h.entropyCoef = entropy_coef;
    h.maxGradNorm = max_grad_norm;
    h.gamma = gamma;
    h.lambda = lambda;
    return MG_OK;
}

int mg_ppo_get_hyper(mg_ppo_t model, float out6[6]) {
    MG_CHECK_ARG(model && out6, "mg_ppo_get_hyper: null argument");
    const mg::PpoHyper& h = P(model)->hp;
    out6[0] = h.clip;
    out6[1] = h.valueCoef;
    out6[2] = h.entropyCoef;
    out6[3] = h.maxGradNorm;
    out6[4] = h.gamma;
    out6[5] = h.lambda;
    return MG_OK;
}

int mg_ppo_set_log_std(mg_ppo_t model, float v) {
    MG_CHECK_ARG(model, "null model");
    return P(model)->setLogStd(v);
}
int mg_ppo_log_std(mg_ppo_t model, int k, float* out) {
    MG_CHECK_ARG(model && out, "null argument");
    return P(model)->logStd(k, out);
}
int mg_ppo_step_counter(mg_ppo_t model, float* out) {
    MG_CHECK_ARG(model && out, "null argument");
    *out = P(model)->stepCounter;
    return MG_OK;
}
int mg_ppo_set_step_counter(mg_ppo_t model, float step) {
    MG_CHECK_ARG(model, "null model");
    P(model)->stepCounter = step;
    return MG_OK;
}

int mg_ppo_buffer(mg_ppo_t model, int which, int slot, void** dev_ptr, size_t* bytes) {
    MG_CHECK_ARG(model && dev_ptr && bytes, "mg_ppo_buffer: null argument");
    return ppo_buffer(P(model), which, slot, dev_ptr, bytes);
}

int mg_ppo_download(mg_ppo_t model, int which, int slot, void* host, size_t bytes) {
    MG_CHECK_ARG(model && host, "mg_ppo_download: null argument");
    void* p;
    size_t n;
    int rc = ppo_buffer(P(model), which, slot, &p, &n);
    if (rc) return rc;
    MG_CUDA_TRY(cudaSetDevice(P(model)->gym->device));
    return copy_checked(host, p, bytes, n, cudaMemcpyDeviceToHost, P(model)->gym->stream);
}

int mg_ppo_upload(mg_ppo_t model, int which, int slot, const void* host, size_t bytes) {
    MG_CHECK_ARG(model && host, "mg_ppo_upload: null argument");
    void* p;
    size_t n;
    int rc = ppo_buffer(P(model), which, slot, &p, &n);
    if (rc) return rc;
    MG_CUDA_TRY(cudaSetDevice(P(model)->gym->device));
    return copy_checked(p, host, bytes, n, cudaMemcpyHostToDevice, P(model)->gym->stream);
}

int mg_ppo_graph_kernels(mg_ppo_t model, uint64_t out2[2]) {
    MG_CHECK_ARG(model && out2, "mg_ppo_graph_kernels: null argument");
    out2[0] = P(model)->collectKernels;
    out2[1] = P(model)->trainKernels;
    return MG_OK;
}

int mg_ppo_set_comm(mg_ppo_t model, void* comm, int rank, int world) {
    MG_CHECK_ARG(model, "null model");
    return P(model)->setComm(comm, rank, world);
}

// ------------------------------------------------------------------ NCCL

static void* nccl_handle() {
    static void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    return h;
}

int mg_comm_unique_id(void* out128) {
    MG_CHECK_ARG(out128, "mg_comm_unique_id: null output");
    void* h = nccl_handle();
    if (!h) return mg::fail(MG_ERR_COMM, "libnccl.so.2 not found");
    auto fn = reinterpret_cast<decltype(&ncclGetUniqueId)>(dlsym(h, "ncclGetUniqueId"));
    ncclUniqueId id;
    ncclResult_t r = fn(&id);
    if (r != ncclSuccess) return mg::fail(MG_ERR_COMM, "ncclGetUniqueId failed");
    std::memcpy(out128, &id, sizeof(id));
    return MG_OK;
}

int mg_comm_init(int world, int rank, const void* id128, int device, void** comm) {
    MG_CHECK_ARG(id128 && comm && world >= 1 && rank >= 0 && rank < world, "mg_comm_init: bad arguments");
    void* h = nccl_handle();
    if (!h) return mg::fail(MG_ERR_COMM, "libnccl.so.2 not found");
    if (device >= 0) MG_CUDA_TRY(cudaSetDevice(device));
    // connect every channel now, while all ranks take part: with NCCL's lazy
    // connection the first collective would handshake with every peer on the
    // host, and a peer that never joins would block the caller there, out of
    // reach of the train() watchdog (a caller's own setting is kept)
    setenv("NCCL_RUNTIME_CONNECT", "0", 0);
    auto fn = reinterpret_cast<decltype(&ncclCommInitRank)>(dlsym(h, "ncclCommInitRank"));
    ncclUniqueId id;
    std::memcpy(&id, id128, sizeof(id));
    ncclComm_t c = nullptr;
    ncclResult_t r = fn(&c, world, id, rank);
    if (r != ncclSuccess) return mg::fail(MG_ERR_COMM, "ncclCommInitRank failed: " + std::to_string((int)r));
    mg::comm_forget_aborted(c);  // a new communicator, whatever lived at this address before
    *comm = c;
    return MG_OK;
}

int mg_comm_abort(void* comm) {
    MG_CHECK_ARG(comm, "mg_comm_abort: null communicator");
    if (mg::comm_aborted(comm)) return MG_OK;  // the watchdog aborted it already
    void* h = nccl_handle();
    if (!h) return mg::fail(MG_ERR_COMM, "libnccl.so.2 not found");
    auto fn = reinterpret_cast<decltype(&ncclCommAbort)>(dlsym(h, "ncclCommAbort"));
    if (!fn) return mg::fail(MG_ERR_COMM, "ncclCommAbort not found");
    mg::comm_mark_aborted(comm);
    mg::comm_release_graphs(comm);  // NCCL's abort waits for the graphs that captured its collectives
    return fn(static_cast<ncclComm_t>(comm)) == ncclSuccess ? MG_OK : mg::fail(MG_ERR_COMM, "ncclCommAbort failed");
}

int mg_comm_destroy(void* comm) {
    if (!comm) return MG_OK;
    if (mg::comm_forget_aborted(comm)) return MG_OK;  // ncclCommAbort freed it
    void* h = nccl_handle();
    if (!h) return mg::fail(MG_ERR_COMM, "libnccl.so.2 not found");
    auto fn = reinterpret_cast<decltype(&ncclCommDestroy)>(dlsym(h, "ncclCommDestroy"));
    mg::comm_release_graphs(comm);  // as for the abort: the destroy waits for them
    return fn(static_cast<ncclComm_t>(comm)) == ncclSuccess ? MG_OK : mg::fail(MG_ERR_COMM, "ncclCommDestroy failed");
}

int mg_allreduce_sum_f32(float* data, size_t count, void* comm, mg_stream_t stream) {
    MG_CHECK_ARG(data && comm, "mg_allreduce_sum_f32: null argument");
    void* h = nccl_handle();
    if (!h) return mg::fail(MG_ERR_COMM, "libnccl.so.2 not found");
    auto fn = reinterpret_cast<decltype(&ncclAllReduce)>(dlsym(h, "ncclAllReduce"));
    ncclResult_t r = fn(data, data, count, ncclFloat, ncclSum, static_cast<ncclComm_t>(comm),
                        reinterpret_cast<cudaStream_t>(stream));
    return r == ncclSuccess ? MG_OK : mg::fail(MG_ERR_COMM, "ncclAllReduce failed");
}

// ------------------------------------------------------------------ host memory

int mg_host_alloc(size_t bytes, void** out) {
    MG_CHECK_ARG(out, "mg_host_alloc: null output");
    MG_CUDA_TRY(cudaMallocHost(out, bytes ? bytes : 1));
    std::memset(*out, 0, bytes);
    return MG_OK;
}

int mg_host_free(void* p) {
    if (p) MG_CUDA_TRY(cudaFreeHost(p));
    return MG_OK;
}

}  // extern "C"
