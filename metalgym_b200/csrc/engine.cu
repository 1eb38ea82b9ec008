// PPO engine: the orchestration of model/ppo.h (PPOModel) and gym.h (Gym)
// rebuilt on the B200 kernels of this library.
//
//   collect()  model/ppo.h:716-751  one CUDA graph: T x (forward, fused
//              sample + env step) + bootstrap forward + GAE + per-slot
//              advantage statistics
//   train(e)   model/ppo.h:918-923  one CUDA graph per epoch, replayed e
//              times; the host shuffles the slot order with the seeded
//              mt19937 (or draws the epoch's row-permutation key) and
//              computes the Adam bias-correction powers (model/ppo.h:873-880),
//              the graph reads them from device memory per minibatch
//   minibatch  model/ppo.h:906-916  forward (activations saved), loss,
//              backward (dX GEMMs with fused mask / LayerNorm-backward +
//              residual epilogues, split-K dW GEMMs into fp32 partials),
//              gradient finalisation + norm, [all-reduce], Adam
#include "engine.h"

#include <dlfcn.h>
#include <nccl.h>
#include <nvtx3/nvToolsExt.h>

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <sstream>
#include <string>
#include <thread>

#include "block.h"
#include "collect_fused.h"
#include "gemm.h"
#include "runtime.h"
#include "watchdog.h"

namespace mg {

namespace {

constexpr int kHead = 64;  // model/ppo.h:116

template <class T>
int dalloc(T** p, size_t bytes) {
    void* v = nullptr;
    cudaError_t e = cudaMalloc(&v, bytes ? bytes : 16);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc");
    *p = static_cast<T*>(v);
    return MG_OK;
}

// ---- NCCL, loaded on first use (the process may already hold torch's copy)
struct Nccl {
    decltype(&ncclGetUniqueId) getUniqueId = nullptr;
    decltype(&ncclCommInitRank) commInitRank = nullptr;
    decltype(&ncclCommDestroy) commDestroy = nullptr;
    decltype(&ncclAllReduce) allReduce = nullptr;
    decltype(&ncclGetErrorString) errorString = nullptr;
    decltype(&ncclGroupStart) groupStart = nullptr;
    decltype(&ncclGroupEnd) groupEnd = nullptr;
    decltype(&ncclCommGetAsyncError) getAsyncError = nullptr;
    decltype(&ncclCommAbort) commAbort = nullptr;
    bool ok = false;
};

Nccl& nccl() {
    static Nccl n;
    static std::once_flag once;
    std::call_once(once, [] {
        void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (h) {
            n.getUniqueId = reinterpret_cast<decltype(&ncclGetUniqueId)>(dlsym(h, "ncclGetUniqueId"));
            n.commInitRank = reinterpret_cast<decltype(&ncclCommInitRank)>(dlsym(h, "ncclCommInitRank"));
            n.commDestroy = reinterpret_cast<decltype(&ncclCommDestroy)>(dlsym(h, "ncclCommDestroy"));
            n.allReduce = reinterpret_cast<decltype(&ncclAllReduce)>(dlsym(h, "ncclAllReduce"));
            n.errorString = reinterpret_cast<decltype(&ncclGetErrorString)>(dlsym(h, "ncclGetErrorString"));
            n.groupStart = reinterpret_cast<decltype(&ncclGroupStart)>(dlsym(h, "ncclGroupStart"));
            n.groupEnd = reinterpret_cast<decltype(&ncclGroupEnd)>(dlsym(h, "ncclGroupEnd"));
            n.getAsyncError = reinterpret_cast<decltype(&ncclCommGetAsyncError)>(dlsym(h, "ncclCommGetAsyncError"));
            n.commAbort = reinterpret_cast<decltype(&ncclCommAbort)>(dlsym(h, "ncclCommAbort"));
            n.ok = n.getUniqueId && n.commInitRank && n.commDestroy && n.allReduce && n.errorString &&
                   n.groupStart && n.groupEnd && n.getAsyncError && n.commAbort;
        }
    });
    return n;
}

// An NVTX range over one public operation (collect, train, ...): profilers
// (ncu --nvtx, nsys) attribute the kernels launched inside it; without a
// profiler attached the calls do nothing.
struct NvtxRange {
    explicit NvtxRange(const char* name) { nvtxRangePushA(name); }
    ~NvtxRange() { nvtxRangePop(); }
};

int nccl_fail(ncclResult_t r, const char* what) {
    Nccl& n = nccl();
    return fail(MG_ERR_COMM, std::string(what) + ": " + (n.errorString ? n.errorString(r) : "nccl error"));
}

uint16_t host_f2bf(float f) {
    uint32_t u;
    std::memcpy(&u, &f, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u);
    return (uint16_t)((u + 0x7fffu + ((u >> 16) & 1u)) >> 16);
}
float host_bf2f(uint16_t h) {
    uint32_t u = (uint32_t)h << 16;
    float f;
    std::memcpy(&f, &u, 4);
    return f;
}

// Kernel nodes in a captured graph (the launches one replay makes).
size_t count_kernel_nodes(cudaGraph_t g) {
    size_t n = 0;
    if (cudaGraphGetNodes(g, nullptr, &n) != cudaSuccess || n == 0) return 0;
    std::vector<cudaGraphNode_t> nodes(n);
    if (cudaGraphGetNodes(g, nodes.data(), &n) != cudaSuccess) return 0;
    size_t k = 0;
    for (auto nd : nodes) {
        cudaGraphNodeType t;
        if (cudaGraphNodeGetType(nd, &t) == cudaSuccess && t == cudaGraphNodeTypeKernel) k++;
    }
    return k;
}

int alloc_acts(ActSet& a, int rows, int E, int H, int L, bool shared) {
    MG_TRY(dalloc(&a.h, (size_t)rows * E * 2));
    MG_TRY(dalloc(&a.fXn, (size_t)rows * E * 2));
    MG_TRY(dalloc(&a.fOut, (size_t)rows * E * 2));
    MG_TRY(dalloc(&a.fSd, (size_t)rows * 4));
    MG_TRY(dalloc(&a.head, (size_t)rows * kHead * 2));
    a.lnXn.assign(L, nullptr);
    a.lnOut.assign(L, nullptr);
    a.lnSd.assign(L, nullptr);
    a.v.assign(L, nullptr);
    for (int n = 0; n < L; n++) {
        if (shared && n > 0) {
            a.lnXn[n] = a.lnXn[0];
            a.lnOut[n] = a.lnOut[0];
            a.lnSd[n] = a.lnSd[0];
            a.v[n] = a.v[0];
            continue;
        }
        MG_TRY(dalloc(&a.lnXn[n], (size_t)rows * E * 2));
        MG_TRY(dalloc(&a.lnOut[n], (size_t)rows * E * 2));
        MG_TRY(dalloc(&a.lnSd[n], (size_t)rows * 4));
        MG_TRY(dalloc(&a.v[n], (size_t)rows * H * 2));
    }
    return MG_OK;
}

void free_acts(ActSet& a, bool shared) {
    cudaFree(a.h);
    cudaFree(a.fXn);
    cudaFree(a.fOut);
    cudaFree(a.fSd);
    cudaFree(a.head);
    const size_t n = shared ? std::min<size_t>(1, a.v.size()) : a.v.size();
    for (size_t i = 0; i < n; i++) {
        cudaFree(a.lnXn[i]);
        cudaFree(a.lnOut[i]);
        cudaFree(a.lnSd[i]);
        cudaFree(a.v[i]);
    }
    a = ActSet{};
}

int splits_for(int M, int N, int K, int bn) {
    const int tiles = ((M + 127) / 128) * ((N + bn - 1) / bn);
    int s = (256 + tiles - 1) / tiles;
    const int maxS = K / 256 > 1 ? K / 256 : 1;
    if (s > maxS) s = maxS;
    if (s < 1) s = 1;
    return gemm_effective_splits(K, s);
}

}  // namespace

// ------------------------------------------------------------------ gym

bool GymCore::stillBusy() const { return busy && stream && cudaStreamQuery(stream) == cudaErrorNotReady; }

GymCore::~GymCore() {
    if (stillBusy()) return;  // leaked on purpose: work that may never finish still uses the buffers
    int cur = 0;
    cudaGetDevice(&cur);
    cudaSetDevice(device);
    if (stream) cudaStreamSynchronize(stream);
    cudaFree(states);
    cudaFree(actions);
    cudaFree(obs);
    cudaFree(reward);
    cudaFree(done);
    cudaFree(rng);
    cudaFree(obsRing);
    cudaFree(rewardRing);
    cudaFree(doneRing);
    cudaFreeHost(hostActions);
    cudaFreeHost(hostReward);
    if (stream) cudaStreamDestroy(stream);
    cudaSetDevice(cur);
}

// gym.h:36-72
int gym_create(const char* name, int n, uint32_t seed, uint32_t firstEnvId, int device, GymCore** out) {
    const mg_env_ops* ops = mg_env_find(name);
    if (!ops) return fail(MG_ERR_NOT_FOUND, std::string("no environment registered as '") + (name ? name : "") + "'");
    MG_CHECK_ARG(n > 0, "gym: parallels must be > 0");
    if (device >= 0) MG_CUDA_TRY(cudaSetDevice(device));
    else MG_CUDA_TRY(cudaGetDevice(&device));
    GymCore* g = new GymCore();
    g->ops = ops;
    g->n = n;
    g->device = device;
    g->seed = seed;
    g->firstEnvId = firstEnvId;
    int rc = MG_OK;
    auto chk = [&](cudaError_t e, const char* w) {
        if (e != cudaSuccess && rc == MG_OK) rc = cuda_fail(e, w);
    };
    chk(cudaStreamCreateWithFlags(&g->stream, cudaStreamNonBlocking), "stream");
    if (!rc) rc = dalloc(&g->states, (size_t)n * ops->state_bytes);
    if (!rc) rc = dalloc(&g->actions, (size_t)n * ops->action_bytes);
    if (!rc) rc = dalloc(&g->obs, (size_t)n * ops->obs_bytes);
    if (!rc) rc = dalloc(&g->reward, (size_t)n * 4);
    if (!rc) rc = dalloc(&g->done, (size_t)n);
    if (!rc) rc = dalloc(&g->rng, (size_t)n * 4);
    if (!rc) chk(cudaMallocHost(&g->hostActions, (size_t)n * ops->action_bytes), "cudaMallocHost");
    if (!rc) chk(cudaMallocHost(reinterpret_cast<void**>(&g->hostReward), (size_t)n * 4), "cudaMallocHost");
    if (!rc) {
        std::memset(g->hostActions, 0, (size_t)n * ops->action_bytes);
        chk(cudaMemsetAsync(g->actions, 0, (size_t)n * ops->action_bytes, g->stream), "memset actions");
        chk(cudaMemsetAsync(g->obs, 0, (size_t)n * ops->obs_bytes, g->stream), "memset obs");
        chk(cudaMemsetAsync(g->reward, 0, (size_t)n * 4, g->stream), "memset reward");
    }
    if (!rc) rc = mg_env_init(name, g->states, g->done, g->rng, n, seed, firstEnvId, reinterpret_cast<mg_stream_t>(g->stream));
    if (!rc) chk(cudaStreamSynchronize(g->stream), "gym init sync");
    if (rc) {
        delete g;
        return rc;
    }
    status_ptr();  // resolve the status word before any graph capture
    *out = g;
    return MG_OK;
}

// ------------------------------------------------------------------ engine

PpoEngine::PpoEngine(GymCore* g, int embed, int scale, int layers, float learningRate, int horizon, uint32_t s)
    : gym(g), device(g->device), R(g->n), O((int)g->ops->obs_dim), A((int)g->ops->act_dim), E(embed),
      H(embed * scale), L(layers), T(horizon), cont(g->ops->continuous != 0), actBytes(g->ops->action_bytes),
      lr(learningRate), seed(s) {}

// Touches nothing of the gym, which may already be gone (a garbage collector
// can finalise a borrowed gym before the model that borrowed it).
PpoEngine::~PpoEngine() {
    comm_unbind_graph(comm, &trainExec);
    if (gym && gym->stillBusy()) return;  // leaked on purpose, as GymCore's buffers
    int cur = 0;
    cudaGetDevice(&cur);
    cudaSetDevice(device);
    cudaDeviceSynchronize();
    if (collectExec) cudaGraphExecDestroy(collectExec);
    if (trainExec) cudaGraphExecDestroy(trainExec);
    freeTrain();
    free_acts(collectActs, true);
    void* ptrs[] = {weights, master, mom, var, grad, obsSlots, actionSlots, logpSlots, valueSlots, rewardSlots,
                    advSlots, retSlots, doneSlots, advStats, mbAdvStats, advPartial, advCounter, normSq, normCounter, statsMean, sched,
                    schedBetaPow};
    for (void* p : ptrs) cudaFree(p);
    cudaFreeHost(hostSched);
    cudaFreeHost(hostSchedBetaPow);
    cudaFreeHost(hostStats);
    if (side) {
        cudaStreamSynchronize(side);
        cudaStreamDestroy(side);
    }
    for (void* q : p2pOpened) cudaIpcCloseMemHandle(q);
    if (p2pRegion) cudaFree(p2pRegion);
    cudaFree(p2pSeq);
    cudaFree(p2pCounter);
    for (auto ev : forkEv)
        if (ev) cudaEventDestroy(ev);
    if (joinEv) cudaEventDestroy(joinEv);
    for (cudaEvent_t ev : {arLateEv, arEarlyEv, arDoneEv})
        if (ev) cudaEventDestroy(ev);
    for (cudaEvent_t ev : phaseEv)
        if (ev) cudaEventDestroy(ev);
    cudaSetDevice(cur);
}

int PpoEngine::init() {
    // model/ppo.h:290-298, with the run-time width limits of this build
    // (no compile-time N_EMBED_CFG; rows need not be a multiple of 64).
    MG_CHECK_ARG(E == 64 || E == 128 || E == 256 || E == 512, "PPOModel: embedDim must be 64, 128, 256 or 512");
    MG_CHECK_ARG(H % 64 == 0 && H > 0 && H <= 8192, "PPOModel: hidden (embed * scale) must be a positive multiple of 64");
    MG_CHECK_ARG(L >= 1 && 6 + 4 * L <= kMaxGradSegments, "PPOModel: layers must be in [1, 8]");
    MG_CHECK_ARG(T >= 1, "PPOModel: horizon must be >= 1");
    MG_CHECK_ARG(A + 1 <= kHead, "PPOModel: ACT_DIM + value must fit one 64-wide head");
    MG_CHECK_ARG(O >= 1 && O <= 256, "PPOModel: OBS_DIM must be in [1, 256]");
    MG_CUDA_TRY(cudaSetDevice(gym->device));
    cudaStream_t st = gym->stream;
    fusedBlocks = block_forward_supported(E, H);
    lnEpilogue = E == 128 || E == 256;
    rowsKernels = gemm_rows_supported(E, H);
    clusterBlocks = block_cluster_supported(E, H);

    // ---- parameters: model/ppo.h:375-445 (seeded normal init rounded to bf16)
    std::vector<std::vector<uint16_t>> init;
    auto add = [&](uint32_t count, bool gf) {
        params.push_back(ParamSpec{count, gf, 0});
        init.emplace_back(count, (uint16_t)0);
        return (uint32_t)(params.size() - 1);
    };
    std::mt19937 rng(seed);
    auto normal = [&](uint32_t p, float sd) {
        std::normal_distribution<float> dist(0.0f, sd);
        for (auto& x : init[p]) x = host_f2bf(dist(rng));
    };
    auto constant = [&](uint32_t p, float v) { std::fill(init[p].begin(), init[p].end(), host_f2bf(v)); };
    pInW = add((uint32_t)(O * E), true);
    normal(pInW, 1.0f / std::sqrt((float)O));
    pInB = add((uint32_t)E, true);
    constant(pInB, 0.0f);
    for (int n = 0; n < L; n++) {
        pLnG.push_back(add((uint32_t)E, true));
        constant(pLnG.back(), 1.0f);
        pLnB.push_back(add((uint32_t)E, true));
        constant(pLnB.back(), 0.0f);
        pUp.push_back(add((uint32_t)(E * H), false));
        normal(pUp.back(), std::sqrt(2.0f / (float)E));
        pDown.push_back(add((uint32_t)(H * E), false));
        normal(pDown.back(), 1.0f / std::sqrt((float)H) / std::sqrt((float)L));
    }
    pLnFg = add((uint32_t)E, true);
    constant(pLnFg, 1.0f);
    pLnFb = add((uint32_t)E, true);
    constant(pLnFb, 0.0f);
    pHead = add((uint32_t)(E * kHead), false);
    {
        std::normal_distribution<float> policyDist(0.0f, 0.01f);
        std::normal_distribution<float> valueDist(0.0f, 1.0f / std::sqrt((float)E));
        for (int k = 0; k < E; k++)
            for (int n = 0; n < kHead; n++) {
                float x = 0.0f;
                if (n < A) x = policyDist(rng);
                else if (n == A) x = valueDist(rng);
                init[pHead][(size_t)k * kHead + n] = host_f2bf(x);
            }
    }
    pLogStd = UINT32_MAX;
    if (cont) {
        pLogStd = add((uint32_t)A, true);
        constant(pLogStd, 0.0f);  // INIT_LOG_STD (model/ppo.h:115)
    }
    uint64_t total = 0;
    for (int pass = 0; pass < 2; pass++) {
        for (auto& sp : params) {
            if (sp.gradIsFloat != (pass == 0)) continue;
            sp.offset = total;
            total += (sp.count + 127) / 128 * 128;
        }
        if (pass == 0) optFloatCount = total;
    }
    optCount = total;
    {
        std::vector<uint16_t> w(optCount, 0);
        std::vector<float> m(optCount, 0.0f);
        for (size_t p = 0; p < params.size(); p++)
            for (uint32_t i = 0; i < params[p].count; i++) {
                w[params[p].offset + i] = init[p][i];
                m[params[p].offset + i] = host_bf2f(init[p][i]);
            }
        MG_TRY(dalloc(&weights, optCount * 2));
        MG_TRY(dalloc(&master, optCount * 4));
        MG_TRY(dalloc(&mom, optCount * 4));
        MG_TRY(dalloc(&var, optCount * 4));
        MG_TRY(dalloc(&grad, optCount * 4));
        MG_CUDA_TRY(cudaMemcpy(weights, w.data(), optCount * 2, cudaMemcpyHostToDevice));
        MG_CUDA_TRY(cudaMemcpy(master, m.data(), optCount * 4, cudaMemcpyHostToDevice));
        MG_CUDA_TRY(cudaMemset(mom, 0, optCount * 4));
        MG_CUDA_TRY(cudaMemset(var, 0, optCount * 4));
        MG_CUDA_TRY(cudaMemset(grad, 0, optCount * 4));
    }

    // ---- rollout slots (model/ppo.h:336-348)
    const size_t slotCount = (size_t)T * R;
    MG_TRY(dalloc(&obsSlots, (size_t)(T + 1) * R * O * 4));
    MG_TRY(dalloc(&actionSlots, slotCount * actBytes));
    MG_TRY(dalloc(&logpSlots, slotCount * 4));
    MG_TRY(dalloc(&valueSlots, slotCount * 4));
    MG_TRY(dalloc(&rewardSlots, slotCount * 4));
    MG_TRY(dalloc(&doneSlots, slotCount));
    MG_TRY(dalloc(&advSlots, slotCount * 4));
    MG_TRY(dalloc(&retSlots, slotCount * 4));
    MG_TRY(dalloc(&advStats, (size_t)T * 2 * 4));
    MG_CUDA_TRY(cudaStreamCreateWithFlags(&side, cudaStreamNonBlocking));
    forkEv.assign(L + 1, nullptr);
    for (auto& ev : forkEv) MG_CUDA_TRY(cudaEventCreateWithFlags(&ev, cudaEventDisableTiming));
    MG_CUDA_TRY(cudaEventCreateWithFlags(&joinEv, cudaEventDisableTiming));
    for (cudaEvent_t* ev : {&arLateEv, &arEarlyEv, &arDoneEv})
        MG_CUDA_TRY(cudaEventCreateWithFlags(ev, cudaEventDisableTiming));
    for (cudaEvent_t& ev : phaseEv) MG_CUDA_TRY(cudaEventCreate(&ev));
    MG_TRY(dalloc(&mbAdvStats, 2 * 4));
    MG_TRY(dalloc(&advPartial, (size_t)2 * kAdvStatsMaxCtas * 8));
    MG_TRY(dalloc(&advCounter, 4));
    MG_CUDA_TRY(cudaMemset(advCounter, 0, 4));
    MG_CUDA_TRY(cudaMemset(actionSlots, 0, slotCount * actBytes));
    MG_CUDA_TRY(cudaMemset(obsSlots, 0, (size_t)(T + 1) * R * O * 4));
    slotOrder.resize(T);
    for (int t = 0; t < T; t++) slotOrder[t] = (uint32_t)t;
    hostRng.seed(seed);

    // ---- activations: collect shares one set across blocks; the training
    // buffers (every block's activations, partials) follow the minibatch rows
    MG_TRY(alloc_acts(collectActs, R, E, H, L, true));
    MG_CUDA_TRY(cudaMemset(collectActs.head, 0, (size_t)R * kHead * 2));
    MG_TRY(allocTrain(R));
    MG_TRY(dalloc(&normSq, 4));
    MG_TRY(dalloc(&normCounter, 4));
    MG_CUDA_TRY(cudaMemset(normCounter, 0, 4));
    MG_TRY(dalloc(&statsMean, 8 * 4));
    MG_CUDA_TRY(cudaMemset(normSq, 0, 4));
    MG_CUDA_TRY(cudaMallocHost(reinterpret_cast<void**>(&hostStats), 8 * 4));
    MG_TRY(ensureSchedule(T, 4 * T));
    MG_CUDA_TRY(cudaStreamSynchronize(st));
    return MG_OK;
}

// Training buffers for minibatches of `rows` rows: every block's saved
// activations, the backward temporaries, per-row statistics, the gradient
// partials and the finalisation table (split counts follow the row count).
int PpoEngine::allocTrain(int rows) {
    MG_CUDA_TRY(cudaStreamSynchronize(gym->stream));
    freeTrain();
    if (trainExec) {  // a captured graph holds the old pointers
        cudaGraphExecDestroy(trainExec);
        trainExec = nullptr;
    }
    MG_TRY(alloc_acts(trainActs, rows, E, H, L, false));
    MG_TRY(dalloc(&dLogits, (size_t)rows * kHead * 2));
    MG_TRY(dalloc(&dBranch, (size_t)rows * E * 2));
    dS.assign(L + 1, nullptr);
    dVs.assign(L, nullptr);
    for (int n = 0; n <= L; n++) MG_TRY(dalloc(&dS[n], (size_t)rows * E * 2));
    for (int n = 0; n < L; n++) MG_TRY(dalloc(&dVs[n], (size_t)rows * H * 2));
    MG_TRY(dalloc(&stats, (size_t)rows * 5 * 4));
    MG_CUDA_TRY(cudaMemset(stats, 0, (size_t)rows * 5 * 4));
    upSplits = splits_for(E, H, rows, H >= 128 ? 128 : 64);
    downSplits = splits_for(H, E, rows, E >= 128 ? 128 : 64);
    if (useBlockClusterBackward(rows)) {
        // the block kernels write one weight-gradient partial per 128-row tile
        upSplits = downSplits = (rows + 127) / 128;
    }
    headSplits = splits_for(E, kHead, rows, 64);
    if (!cont && useHeadTail(rows)) headSplits = (rows + 127) / 128;  // one dW_head partial per 128-row tile
    upPart.assign(L, nullptr);
    downPart.assign(L, nullptr);
    lnPart.assign(L, nullptr);
    const int pLn = layernorm_backward_parts(rows);
    const int pIn = input_backward_parts(rows, O, E);
    const int pGs = gaussian_loss_parts(rows);
    for (int n = 0; n < L; n++) {
        MG_TRY(dalloc(&upPart[n], (size_t)upSplits * E * H * 4));
        MG_TRY(dalloc(&downPart[n], (size_t)downSplits * H * E * 4));
        MG_TRY(dalloc(&lnPart[n], (size_t)pLn * 2 * E * 4));
    }
    MG_TRY(dalloc(&headPart, (size_t)headSplits * E * kHead * 4));
    MG_TRY(dalloc(&lnFPart, (size_t)pLn * 2 * E * 4));
    MG_TRY(dalloc(&inPart, (size_t)pIn * (O + 1) * E * 4));
    MG_TRY(dalloc(&lsPart, (size_t)pGs * (A > 0 ? A : 1) * 4));
    GradSegmentTable& tb = gradTable;
    tb = GradSegmentTable{};
    gradTableEarly = GradSegmentTable{};
    gradTableLate = GradSegmentTable{};
    auto seg = [&](const float* src, int64_t stride, int nparts, int64_t count, uint32_t p, int round) {
        GradSegment s{};
        s.src = src;
        s.partStride = stride;
        s.nparts = nparts;
        s.count = count;
        s.dstOffset = (int64_t)params[p].offset;
        s.roundBf16 = round;
        // written before the last backward kernel (block 0's): the other
        // blocks', the final LayerNorm's and the head's partials
        bool block0 = p == pInW || p == pInB;
        for (uint32_t q : {pLnG[0], pLnB[0], pUp[0], pDown[0]}) block0 = block0 || p == q;
        s.early = L > 0 && !block0 && p != pLogStd ? 1 : 0;
        tb.seg[tb.n++] = s;
        // the overlapped all-reduce: block 0 and the input layer (the last
        // backward layer), and everything before them in backward order
        const bool early = p == pInW || p == pInB || p == pLnG[0] || p == pLnB[0] || p == pUp[0] || p == pDown[0];
        GradSegmentTable& part = early ? gradTableEarly : gradTableLate;
        part.seg[part.n++] = s;
    };
    seg(inPart, (int64_t)(O + 1) * E, pIn, (int64_t)O * E, pInW, 0);
    seg(inPart + (size_t)O * E, (int64_t)(O + 1) * E, pIn, E, pInB, 0);
    for (int n = 0; n < L; n++) {
        seg(lnPart[n], 2 * E, pLn, E, pLnG[n], 0);
        seg(lnPart[n] + E, 2 * E, pLn, E, pLnB[n], 0);
        seg(upPart[n], (int64_t)E * H, upSplits, (int64_t)E * H, pUp[n], 1);
        seg(downPart[n], (int64_t)H * E, downSplits, (int64_t)H * E, pDown[n], 1);
    }
    seg(lnFPart, 2 * E, pLn, E, pLnFg, 0);
    seg(lnFPart + E, 2 * E, pLn, E, pLnFb, 0);
    seg(headPart, (int64_t)E * kHead, headSplits, (int64_t)E * kHead, pHead, 1);
    if (cont) seg(lsPart, A, pGs, A, pLogStd, 0);
    nNorm = grad_table_layout(tb);
    const int nNormAll = std::max(std::max(nNorm, grad_scale_norm_blocks((int64_t)optCount)), p2p_blocks());
    MG_TRY(dalloc(&normPartial, (size_t)nNormAll * 4));
    // the two halves of the overlapped all-reduce's sums (their norm partials
    // are unused: the norm is taken after the all-reduce); the late half runs
    // on the side stream, so it writes its own partials
    grad_table_layout(gradTableEarly);
    MG_TRY(dalloc(&normPartialLate, (size_t)std::max(1, grad_table_layout(gradTableLate)) * 4));
    trainBufRows = rows;
    return MG_OK;
}

void PpoEngine::freeTrain() {
    free_acts(trainActs, false);
    float** fs[] = {&stats, &headPart, &lnFPart, &inPart, &lsPart, &normPartial, &normPartialLate};
    for (float** p : fs) {
        cudaFree(*p);
        *p = nullptr;
    }
    void** vs[] = {&dLogits, &dBranch};
    for (void** p : vs) {
        cudaFree(*p);
        *p = nullptr;
    }
    for (void* p : dS) cudaFree(p);
    for (void* p : dVs) cudaFree(p);
    dS.clear();
    dVs.clear();
    for (auto* p : upPart) cudaFree(p);
    for (auto* p : downPart) cudaFree(p);
    for (auto* p : lnPart) cudaFree(p);
    upPart.clear();
    downPart.clear();
    lnPart.clear();
    trainBufRows = 0;
}

// Device schedule of `device` minibatches (one epoch) and its pinned host
// staging of `host` minibatches (all epochs of a train call).
int PpoEngine::ensureSchedule(int device, int host) {
    if (host > maxHostSchedule) {
        cudaStreamSynchronize(gym->stream);
        cudaFreeHost(hostSched);
        cudaFreeHost(hostSchedBetaPow);
        hostSched = nullptr;
        hostSchedBetaPow = nullptr;
        MG_CUDA_TRY(cudaMallocHost(reinterpret_cast<void**>(&hostSched), (size_t)host * sizeof(MgMinibatch)));
        MG_CUDA_TRY(cudaMallocHost(reinterpret_cast<void**>(&hostSchedBetaPow), (size_t)host * 2 * 4));
        maxHostSchedule = host;
    }
    if (device > maxSchedule) {
        cudaStreamSynchronize(gym->stream);
        cudaFree(sched);
        cudaFree(schedBetaPow);
        sched = nullptr;
        schedBetaPow = nullptr;
        MG_TRY(dalloc(&sched, (size_t)device * sizeof(MgMinibatch)));
        MG_TRY(dalloc(&schedBetaPow, (size_t)device * 2 * 4));
        maxSchedule = device;
        if (trainExec) {  // a captured graph holds the old pointers
            cudaGraphExecDestroy(trainExec);
            trainExec = nullptr;
        }
    }
    return MG_OK;
}

// Waits for the work on the gym's stream. With an NCCL communicator and a
// timeout (setCommTimeout), the wait watches the communicator (watchdog.h):
// a peer's asynchronous error or the deadline aborts it and fails with
// MG_ERR_COMM instead of blocking for good.
int PpoEngine::waitStream(const char* what) {
    cudaStream_t st = gym->stream;
    if (!(world > 1 && comm && !p2pOn && commTimeout > 0.0f)) {
        MG_CUDA_TRY(cudaStreamSynchronize(st));
        return MG_OK;
    }
    struct Ctx {
        cudaStream_t st;
        ncclComm_t comm;
        Nccl* nc;
        cudaError_t err;
    } c{st, static_cast<ncclComm_t>(comm), &nccl(), cudaSuccess};
    WatchOps o{};
    o.ctx = &c;
    o.done = [](void* p) -> int {
        Ctx* x = static_cast<Ctx*>(p);
        const cudaError_t e = cudaStreamQuery(x->st);
        if (e == cudaSuccess) return 1;
        if (e == cudaErrorNotReady) return 0;
        x->err = e;
        return -1;
    };
    o.peerError = [](void* p) -> int {
        Ctx* x = static_cast<Ctx*>(p);
        ncclResult_t a = ncclSuccess;
        if (x->nc->getAsyncError(x->comm, &a) != ncclSuccess) return 1;
        return a != ncclSuccess && a != ncclInProgress;
    };
    o.release = [](void* p) { comm_release_graphs(static_cast<Ctx*>(p)->comm); };
    o.abort = [](void* p) {
        Ctx* x = static_cast<Ctx*>(p);
        x->nc->commAbort(x->comm);
    };
    o.now = [](void*) -> double {
        return std::chrono::duration<double>(std::chrono::steady_clock::now().time_since_epoch()).count();
    };
    // a short sleep, not a spin: the wait lasts the whole step and must leave
    // the host cores to the NCCL proxy and gloo threads
    o.pause = [](void*) { std::this_thread::sleep_for(std::chrono::microseconds(100)); };
    bool drained = false;
    const int r = watch_wait(o, (double)commTimeout, 30.0, &drained);
    if (r == kWatchDone) return MG_OK;
    if (r == kWatchCudaError) return cuda_fail(c.err, what);
    comm_mark_aborted(comm);
    if (!drained) gym->busy = true;
    std::ostringstream m;
    m << what << ": the gradient all-reduce "
      << (r == kWatchPeerError ? "failed on a peer" : "did not finish within the communication timeout (")
      << (r == kWatchPeerError ? "" : std::to_string(commTimeout) + " s)")
      << "; the communicator was aborted" << (drained ? "" : ", and the stream has not drained");
    return fail(MG_ERR_COMM, m.str());
}

int PpoEngine::checkStatus(const char* what) {
    MG_TRY(waitStream(what));
    int st = 0;
    MG_CUDA_TRY(cudaMemcpy(&st, status_ptr(), sizeof(int), cudaMemcpyDeviceToHost));
    if (st != 0) {
        cudaMemset(status_ptr(), 0, sizeof(int));
        return fail(MG_ERR_DEVICE, std::string(what) + ": device status " + std::to_string(st));
    }
    return MG_OK;
}

// Arguments of the fused block kernel for block n over an activation set.
BlockFwdArgs PpoEngine::blockArgs(ActSet& a, int n, int rows) {
    BlockFwdArgs b{};
    b.h = static_cast<__nv_bfloat16*>(a.h);
    b.gamma = reinterpret_cast<const __nv_bfloat16*>(weights + params[pLnG[n]].offset);
    b.beta = reinterpret_cast<const __nv_bfloat16*>(weights + params[pLnB[n]].offset);
    b.xNorm = static_cast<__nv_bfloat16*>(a.lnXn[n]);
    b.lnOut = static_cast<__nv_bfloat16*>(a.lnOut[n]);
    b.stdev = a.lnSd[n];
    b.V = static_cast<__nv_bfloat16*>(a.v[n]);
    b.rows = rows;
    b.E = E;
    b.H = H;
    return b;
}

// The input layer, the residual blocks and the final LayerNorm of a forward
// pass (model/ppo.h:575-615). Per block either
// the fused block kernel, or LayerNorm + up GEMM (ReLU) + down GEMM (+ skip);
// with the LayerNorm epilogue the down GEMM of block n also computes the
// LayerNorm that follows it (block n + 1's, or the final one), which then has
// no kernel of its own.
int PpoEngine::blocksForward(const float* obs, const RowMap& rm, ActSet& a, int rows, cudaStream_t st,
                             MinibatchTiles* mt) {
    auto w = [&](uint32_t p) { return static_cast<const void*>(weights + params[p].offset); };
    auto bw = [&](uint32_t p) { return reinterpret_cast<const __nv_bfloat16*>(weights + params[p].offset); };
    const bool cluster = useBlockClusterForward(rows);
    const bool rowsK = !cluster && useRowsForward(rows);
    const bool fused = !cluster && !rowsK && useFusedBlock(rows);
    const bool lnEpi = !fused && (cluster || rowsK || useLnEpilogue(rows));
    // the first block's kernel also computes the input layer and the first LayerNorm
    const bool inputInBlock = cluster && L > 0 && O <= kBlockClusterMaxInputDim;
    // model/input.metal:11-27 (the input gathers the minibatch's observation rows through rm)
    if (!inputInBlock) MG_TRY(input_forward(obs, w(pInW), w(pInB), a.h, rows, O, E, st, rm));
    for (int n = 0; n < L; n++) {
        if (fused) {
            MG_TRY(block_forward(blockArgs(a, n, rows), w(pUp[n]), w(pDown[n]), st));
            continue;
        }
        if ((n == 0 && !inputInBlock) || !lnEpi)
            MG_TRY(layernorm_forward(a.h, a.lnXn[n], a.lnOut[n], w(pLnG[n]), w(pLnB[n]), a.lnSd[n], rows, E, st));
        if (cluster) {
            // up (ReLU), down (+ skip) and the next LayerNorm in one kernel
            const LnOutputs next =
                n + 1 < L ? LnOutputs{bw(pLnG[n + 1]), bw(pLnB[n + 1]), static_cast<__nv_bfloat16*>(a.lnXn[n + 1]),
                                      static_cast<__nv_bfloat16*>(a.lnOut[n + 1]), a.lnSd[n + 1]}
                          : LnOutputs{bw(pLnFg), bw(pLnFb), static_cast<__nv_bfloat16*>(a.fXn),
                                      static_cast<__nv_bfloat16*>(a.fOut), a.fSd};
            const BlockClusterForwardInput in{obs, rm.mb, rm.envRows, rm.total, O, w(pInW), w(pInB), w(pLnG[0]),
                                              w(pLnB[0]), a.lnXn[0], a.lnSd[0]};
            if (mt)
                MG_TRY(mt->forward(a.lnOut[n], w(pUp[n]), w(pDown[n]), a.h, a.v[n], next, rows,
                                   n == 0 && inputInBlock ? &in : nullptr));
            else
                // blocks after the first follow the previous block's kernel
                MG_TRY(block_cluster_forward(a.lnOut[n], w(pUp[n]), w(pDown[n]), a.h, a.v[n], next, rows, st,
                                             n == 0 && inputInBlock ? &in : nullptr, n > 0));
            continue;
        }
        GemmCall up;
        up.A = a.lnOut[n]; up.lda = E;
        up.B = w(pUp[n]); up.b_mn = true; up.ldb = H;
        up.M = rows; up.N = H; up.K = E;
        up.epilogue = kEpiBf16Relu;
        up.out = a.v[n]; up.ldo = H;
        MG_TRY(gemm_bf16(up, st));
        GemmCall down;
        down.A = a.v[n]; down.lda = H;
        down.B = w(pDown[n]); down.b_mn = true; down.ldb = E;
        down.M = rows; down.N = E; down.K = H;
        down.epilogue = kEpiBf16Resid;  // + skip, in place on the stream
        down.aux = a.h; down.ldaux = E;
        down.out = a.h; down.ldo = E;
        LnOutputs ln;
        if (lnEpi) {
            ln = n + 1 < L ? LnOutputs{bw(pLnG[n + 1]), bw(pLnB[n + 1]), static_cast<__nv_bfloat16*>(a.lnXn[n + 1]),
                                       static_cast<__nv_bfloat16*>(a.lnOut[n + 1]), a.lnSd[n + 1]}
                           : LnOutputs{bw(pLnFg), bw(pLnFb), static_cast<__nv_bfloat16*>(a.fXn),
                                       static_cast<__nv_bfloat16*>(a.fOut), a.fSd};
            down.epilogue = kEpiResidLN;
            down.ln = &ln;
        }
        if (rowsK) {
            MG_TRY(gemm_rows_resid_layernorm(a.v[n], H, w(pDown[n]), true, E, rows, H, a.h, ln, st));
            continue;
        }
        MG_TRY(gemm_bf16(down, st));
    }
    if (!lnEpi || L == 0) MG_TRY(layernorm_forward(a.h, a.fXn, a.fOut, w(pLnFg), w(pLnFb), a.fSd, rows, E, st));
    return 0;
}

// model/ppo.h:575-626: input -> L x [LN -> up (ReLU) -> down (+ skip)] -> LN -> head.
int PpoEngine::forwardOn(const float* obs, int rows, ActSet& a, cudaStream_t st) {
    const uint16_t* W = weights;
    auto w = [&](uint32_t p) { return static_cast<const void*>(W + params[p].offset); };
    // (input_forward can also end with block 0's LayerNorm; measured in a
    // CUDA graph at 4096 rows the two kernels are faster: 5.25 against 5.87 µs)
    MG_TRY(blocksForward(obs, RowMap{nullptr, 0, 0}, a, rows, st));
    GemmCall hd;
    hd.A = a.fOut; hd.lda = E;
    hd.B = w(pHead); hd.b_mn = true; hd.ldb = kHead;
    hd.M = rows; hd.N = kHead; hd.K = E;
    hd.epilogue = 0;
    hd.out = a.head; hd.ldo = kHead;
    return gemm_bf16(hd, st);
}

// One minibatch (model/ppo.h:906-916): one time slot, or in row mode B
// permuted rollout rows; which rows, and the Adam bias-correction powers,
// are read from the device schedule at j.
int PpoEngine::minibatch(int j, bool rowMode, cudaStream_t st) {
    const int rows = trainBufRows;
    const RowMap rm{sched + j, (uint64_t)R, (uint64_t)T * R};
    ActSet& a = trainActs;
    auto w = [&](uint32_t p) { return static_cast<const void*>(weights + params[p].offset); };
    const bool overlapAr = world > 1 && !p2pOn && overlapAllreduce;
    // every per-tile pass as a cluster kernel: record them, then one launch
    MinibatchTiles* mt = nullptr;
    if (fusedMinibatch && !cont && !overlapAr && L >= 1 && L <= MinibatchTiles::kMaxBlocks &&
        useBlockClusterForward(rows) && O <= kBlockClusterMaxInputDim && useHeadTail(rows) &&
        useBlockClusterBackward(rows)) {
        mt = &tilesPlan;
        mt->reset();
    }
    // forward with activations saved (the input gathers the minibatch's obs rows)
    MG_TRY(blocksForward(obsSlots, rm, a, rows, st, mt));
    // loss (model/ppo.h:753-781): per-slot advantage statistics from
    // collect(), or in row mode the statistics of this minibatch's rows
    const LossHyper lh{hp.clip, hp.valueCoef, hp.entropyCoef};
    const float* as = advStats;
    if (rowMode) {
        MG_TRY(advantage_stats_rows(advSlots, rm, rows, mbAdvStats, advPartial, advCounter, st));
        as = mbAdvStats;
    }
    // the whole head of the minibatch in one kernel (head_tail.cu): head GEMM,
    // loss, head dX, final LayerNorm backward and the dW_head tile partials
    const bool headTail = !cont && useHeadTail(rows);
    if (headTail) {
        const PolicyLossRows pl = policy_loss_rows(static_cast<const int32_t*>(actionSlots), advSlots, as, retSlots,
                                                   logpSlots, dLogits, stats, rows, A, lh, rm);
        if (mt)
            MG_TRY(mt->headTail(a.fOut, w(pHead), a.head, pl, headPart, w(pLnFg), a.fXn, a.fSd, dS[L], lnFPart, rows));
        else
            MG_TRY(head_tail(a.fOut, w(pHead), a.head, pl, headPart, w(pLnFg), a.fXn, a.fSd, dS[L], lnFPart, rows,
                             st));
    } else {
        GemmCall hd;
        hd.A = a.fOut; hd.lda = E;
        hd.B = w(pHead); hd.b_mn = true; hd.ldb = kHead;
        hd.M = rows; hd.N = kHead; hd.K = E;
        hd.out = a.head; hd.ldo = kHead;
        // the categorical loss runs in the head GEMM's epilogue (each epilogue
        // thread holds a whole head row); the Gaussian loss, whose log-std
        // gradient is a batch sum, has its own kernel
        PolicyLossRows pl{};
        if (!cont) {
            pl = policy_loss_rows(static_cast<const int32_t*>(actionSlots), advSlots, as, retSlots, logpSlots, dLogits,
                                  stats, rows, A, lh, rm);
            hd.epilogue = 5;  // bf16 head + policy loss
            hd.loss = &pl;
        }
        MG_TRY(gemm_bf16(hd, st));
    }
    if (cont)
        MG_TRY(gaussian_loss(a.head, static_cast<const float*>(actionSlots), advSlots, as, retSlots, logpSlots,
                             dLogits, stats, w(pLogStd), lsPart, rows, A, lh, st, rm));
    // backward (model/ppo.h:793-865). The input-gradient chain runs on st;
    // each weight-gradient GEMM is forked to the side stream as soon as its
    // operands exist (they are never overwritten within the minibatch) and
    // the side stream is joined before the gradient finalisation.
    bool forked = false;  // the side stream joins the capture only through a fork
    auto fork = [&](int k) -> int {
        MG_CUDA_TRY(cudaEventRecord(forkEv[k], st));
        MG_CUDA_TRY(cudaStreamWaitEvent(side, forkEv[k], 0));
        forked = true;
        return MG_OK;
    };
    if (!headTail) {
        MG_TRY(fork(L));
        GemmCall dw;  // dW_head = X_F^T dLogits (model/linear.metal:71-93)
        dw.A = a.fOut; dw.a_mn = true; dw.lda = E;
        dw.B = dLogits; dw.b_mn = true; dw.ldb = kHead;
        dw.M = E; dw.N = kHead; dw.K = rows;
        dw.epilogue = 4; dw.splits = headSplits;
        dw.out = headPart; dw.ldo = kHead;
        MG_TRY(gemm_bf16(dw, side));
        GemmCall dx;  // dS[L] = dLogits W_head^T (model/linear.metal:40-60)
        dx.A = dLogits; dx.lda = kHead;
        dx.B = w(pHead); dx.ldb = kHead;  // [E][64] = [N][K], K-major
        dx.M = rows; dx.N = E; dx.K = kHead;
        dx.out = dS[L]; dx.ldo = E;
        MG_TRY(gemm_bf16(dx, st));
        MG_TRY(layernorm_backward(dS[L], a.fXn, w(pLnFg), a.fSd, nullptr, lnFPart, rows, E, st));
    }
    const bool clusterBwd = useBlockClusterBackward(rows);
    // the first block's kernel also sums the input layer's gradient partials
    // (the same 16-row partials input_backward writes at these row counts)
    const bool inputFused = clusterBwd && inputGradFusable(rows);
    for (int n = L - 1; n >= 0; n--) {
        if (overlapAr && n == 0) {
            // every gradient but block 0's and the input layer's is complete:
            // sum and all-reduce them on the side stream while the last
            // backward layer runs here (after the side stream's own work)
            MG_CUDA_TRY(cudaEventRecord(arLateEv, st));
            MG_CUDA_TRY(cudaStreamWaitEvent(side, arLateEv, 0));
            forked = true;
            MG_TRY(grad_finalize(gradTableLate, grad, normPartialLate, side));
            MG_TRY(allreduceRanges(arLate, side));
        }
        if (clusterBwd) {
            // dV, dBranch, the LayerNorm backward with the skip add and both
            // weight-gradient partials in one kernel
            const BlockClusterInput in{obsSlots, rm.mb, rm.envRows, rm.total, O, inPart};
            if (mt)
                MG_TRY(mt->backward(dS[n + 1], w(pDown[n]), a.v[n], w(pUp[n]), dVs[n], a.lnOut[n], upPart[n],
                                    downPart[n], a.lnXn[n], w(pLnG[n]), a.lnSd[n], dS[n + 1], dS[n], lnPart[n], rows,
                                    n == 0 && inputFused ? &in : nullptr));
            else
                // the kernel before is the next block's backward kernel, or the
                // head kernel for the last block
                MG_TRY(block_cluster_backward(dS[n + 1], w(pDown[n]), a.v[n], w(pUp[n]), dVs[n], a.lnOut[n],
                                              upPart[n], downPart[n], a.lnXn[n], w(pLnG[n]), a.lnSd[n], dS[n + 1],
                                              dS[n], lnPart[n], rows, st, n == 0 && inputFused ? &in : nullptr,
                                              n < L - 1 || headTail));
            continue;
        } else {
            GemmCall g1;  // dV = bf16(dS Dp^T) * (V > 0) (model/mlp.metal:88-127)
            g1.A = dS[n + 1]; g1.lda = E;
            g1.B = w(pDown[n]); g1.ldb = E;  // Dp [H][E] = [N][K]
            g1.M = rows; g1.N = H; g1.K = E;
            g1.epilogue = 3; g1.aux = a.v[n]; g1.ldaux = H;
            g1.out = dVs[n]; g1.ldo = H;
            MG_TRY(gemm_bf16(g1, st));
        }
        MG_TRY(fork(n));
        GemmCall g2;  // dUp = X^T dV (model/mlp.metal:167-208)
        g2.A = a.lnOut[n]; g2.a_mn = true; g2.lda = E;
        g2.B = dVs[n]; g2.b_mn = true; g2.ldb = H;
        g2.M = E; g2.N = H; g2.K = rows;
        g2.epilogue = 4; g2.splits = upSplits;
        g2.out = upPart[n]; g2.ldo = H;
        MG_TRY(gemm_bf16(g2, side));
        GemmCall g3;  // dDp = V^T dS
        g3.A = a.v[n]; g3.a_mn = true; g3.lda = H;
        g3.B = dS[n + 1]; g3.b_mn = true; g3.ldb = E;
        g3.M = H; g3.N = E; g3.K = rows;
        g3.epilogue = 4; g3.splits = downSplits;
        g3.out = downPart[n]; g3.ldo = E;
        MG_TRY(gemm_bf16(g3, side));
        if (useRowsBackward(rows) && gemm_rows_ln_backward_supported(rows)) {
            // dBranch and the LayerNorm backward with the skip add in one kernel
            MG_TRY(gemm_rows_layernorm_backward(dVs[n], H, w(pUp[n]), false, H, rows, H, a.lnXn[n], w(pLnG[n]),
                                                a.lnSd[n], dS[n + 1], dS[n], lnPart[n], st));
            continue;
        }
        GemmCall g4;  // dBranch = dV Up^T (model/mlp.metal:131-153)
        g4.A = dVs[n]; g4.lda = H;
        g4.B = w(pUp[n]); g4.ldb = H;  // Up [E][H] = [N][K]
        g4.M = rows; g4.N = E; g4.K = H;
        g4.out = dBranch; g4.ldo = E;
        MG_TRY(gemm_bf16(g4, st));
        // LayerNorm backward, then dS[n] = dS[n + 1] + dBranch (model/ppo.h:851-852)
        MG_TRY(layernorm_backward(dBranch, a.lnXn[n], w(pLnG[n]), a.lnSd[n], dS[n + 1], lnPart[n], rows, E, st,
                                  dS[n]));
    }
    if (mt) MG_TRY(mt->launch(st));
    if (!inputFused) MG_TRY(input_backward(obsSlots, dS[0], inPart, rows, O, E, st, rm));
    if (forked) {
        MG_CUDA_TRY(cudaEventRecord(joinEv, side));
        MG_CUDA_TRY(cudaStreamWaitEvent(st, joinEv, 0));
    }
    // gradient sums + norm (model/ppo.h:873-890), [all-reduce], Adam (:891-903)
    if (p2pOn) {
        // sums into this minibatch's exchange buffer, then the all-reduce over
        // peer memory leaves the averaged gradient in grad and its norm in normSq
        float* x0 = reinterpret_cast<float*>(static_cast<unsigned char*>(p2pRegion) + p2pTable.xOff[0]);
        float* x1 = reinterpret_cast<float*>(static_cast<unsigned char*>(p2pRegion) + p2pTable.xOff[1]);
        MG_TRY(grad_finalize(gradTable, x0, normPartial, st, nullptr, nullptr, x1, p2pSeq, (int64_t)optFloatCount));
        MG_TRY(p2p_allreduce(p2pTable, (int64_t)optCount, grad, p2pSeq, p2pCounter, normPartial, normSq, st));
        const AdamHyper ah{lr, hp.maxGradNorm, 0.0f, 0.0f};
        return adam(master, grad, mom, var, weights, normPartial, 0, (int64_t)optCount, ah, schedBetaPow + 2 * j,
                    nullptr, st, normSq);
    }
    if (overlapAr) {
        // the early half: sums here, then its all-reduce after the late one
        // on the side stream (one stream keeps the communicator's order)
        MG_TRY(grad_finalize(gradTableEarly, grad, normPartial, st));
        MG_CUDA_TRY(cudaEventRecord(arEarlyEv, st));
        MG_CUDA_TRY(cudaStreamWaitEvent(side, arEarlyEv, 0));
        MG_TRY(allreduceRanges(arEarly, side));
        MG_CUDA_TRY(cudaEventRecord(arDoneEv, side));
        MG_CUDA_TRY(cudaStreamWaitEvent(st, arDoneEv, 0));
        MG_TRY(grad_scale_norm(grad, (int64_t)optCount, 1.0f / (float)world, normPartial, st, normCounter, normSq));
        const AdamHyper ah{lr, hp.maxGradNorm, 0.0f, 0.0f};
        return adam(master, grad, mom, var, weights, normPartial, 0, (int64_t)optCount, ah, schedBetaPow + 2 * j,
                    nullptr, st, normSq);
    }
    // the finalisation's last CTA leaves the squared norm in normSq. When the
    // kernel before it is block 0's cluster backward (which signals its
    // dependents after its own wait, with the input layer's gradient inside
    // it and no join in between), the other blocks' and the head's sums start
    // beside it.
    const bool earlyOk = world == 1 && clusterBwd && !mt && inputFused && !forked;
    MG_TRY(grad_finalize(gradTable, grad, normPartial, st, normCounter, normSq, nullptr, nullptr, INT64_MAX, earlyOk));
    if (world > 1) {
        Nccl& nc = nccl();
        ncclResult_t r = nc.allReduce(grad, grad, (size_t)optCount, ncclFloat, ncclSum, static_cast<ncclComm_t>(comm), st);
        if (r != ncclSuccess) return nccl_fail(r, "ncclAllReduce");
        MG_TRY(grad_scale_norm(grad, (int64_t)optCount, 1.0f / (float)world, normPartial, st, normCounter, normSq));
    }
    const AdamHyper ah{lr, hp.maxGradNorm, 0.0f, 0.0f};
    return adam(master, grad, mom, var, weights, normPartial, 0, (int64_t)optCount, ah, schedBetaPow + 2 * j, nullptr,
                st, normSq);
}

int PpoEngine::captureCollect() {
    std::lock_guard<std::mutex> lock(capture_mutex());
    for (int attempt = 0;; attempt++) {
        bool invalidated = false;
        const int rc = captureCollectOnce(&invalidated);
        if (rc == MG_OK || !invalidated || attempt == 2) return rc;
        cudaGetLastError();  // another thread's module load ended the capture: capture again
    }
}

int PpoEngine::captureCollectOnce(bool* invalidated) {
    cudaStream_t st = gym->stream;
    if (collectExec) {
        cudaGraphExecDestroy(collectExec);
        collectExec = nullptr;
    }
    MG_CUDA_TRY(cudaStreamBeginCapture(st, cudaStreamCaptureModeRelaxed));
    int rc = MG_OK;
    const void* logStd = cont ? static_cast<const void*>(weights + params[pLogStd].offset) : nullptr;
    const mg_env_ops* ops = gym->ops;
    const bool fusedCollect = useFusedCollect();
    if (fusedCollect) {
        // every step, the bootstrap forward and GAE in one kernel; the
        // advantage statistics need every environment's column
        CollectFusedArgs a{};
        a.R = R;
        a.T = T;
        a.L = L;
        a.inDim = O;
        auto w = [&](uint32_t p) { return static_cast<const void*>(weights + params[p].offset); };
        a.wIn = w(pInW);
        a.bIn = w(pInB);
        for (int n = 0; n < L; n++) {
            a.lnGamma[n] = w(pLnG[n]);
            a.lnBeta[n] = w(pLnB[n]);
            a.wUp[n] = w(pUp[n]);
            a.wDown[n] = w(pDown[n]);
        }
        a.lnGamma[L] = w(pLnFg);
        a.lnBeta[L] = w(pLnFb);
        a.wHead = w(pHead);
        a.logStd = logStd;
        a.states = gym->states;
        a.done = gym->done;
        a.rng = gym->rng;
        a.obsSlots = obsSlots;
        a.actionSlots = actionSlots;
        a.logpSlots = logpSlots;
        a.valueSlots = valueSlots;
        a.rewardSlots = rewardSlots;
        a.doneSlots = doneSlots;
        a.advSlots = advSlots;
        a.retSlots = retSlots;
        a.bootHead = collectActs.head;
        a.gamma = hp.gamma;
        a.lambda = hp.lambda;
        rc = collect_fused(ops, a, st);
    }
    for (int t = 0; t < T && !rc && !fusedCollect; t++) {
        rc = forwardOn(obsSlots + (size_t)t * R * O, R, collectActs, st);
        if (!rc)
            rc = ops->collect_step(collectActs.head, logStd, gym->states,
                                   static_cast<char*>(actionSlots) + (size_t)t * R * actBytes, logpSlots + (size_t)t * R,
                                   valueSlots + (size_t)t * R, obsSlots + (size_t)(t + 1) * R * O,
                                   rewardSlots + (size_t)t * R, gym->done, doneSlots + (size_t)t * R, gym->rng, R,
                                   reinterpret_cast<mg_stream_t>(st));
    }
    if (!rc && !fusedCollect) rc = forwardOn(obsSlots + (size_t)T * R * O, R, collectActs, st);
    if (!rc && !fusedCollect)
        rc = gae(rewardSlots, doneSlots, valueSlots, collectActs.head, advSlots, retSlots, R, T, A, hp.gamma,
                 hp.lambda, st);
    if (!rc) rc = advantage_stats(advSlots, advStats, R, T, st);
    cudaGraph_t graph = nullptr;
    cudaError_t e = cudaStreamEndCapture(st, &graph);
    *invalidated = e == cudaErrorStreamCaptureInvalidated;
    if (rc) {
        if (graph) cudaGraphDestroy(graph);
        return rc;
    }
    if (e != cudaSuccess) return cuda_fail(e, "collect capture");
    collectKernels = count_kernel_nodes(graph);
    e = cudaGraphInstantiate(&collectExec, graph, 0);
    cudaGraphDestroy(graph);
    if (e != cudaSuccess) return cuda_fail(e, "collect graph instantiate");
    collectHp = hp;
    collectExecFused = fusedCollect;
    return MG_OK;
}

int PpoEngine::captureTrain(int minibatches, bool rowMode) {
    std::lock_guard<std::mutex> lock(capture_mutex());
    for (int attempt = 0;; attempt++) {
        bool invalidated = false;
        const int rc = captureTrainOnce(minibatches, rowMode, &invalidated);
        if (rc == MG_OK || !invalidated || attempt == 2) return rc;
        cudaGetLastError();  // another thread's module load ended the capture: capture again
    }
}

int PpoEngine::captureTrainOnce(int minibatches, bool rowMode, bool* invalidated) {
    cudaStream_t st = gym->stream;
    MG_CUDA_TRY(cudaStreamBeginCapture(st, cudaStreamCaptureModeRelaxed));
    int rc = MG_OK;
    for (int j = 0; j < minibatches && !rc; j++) rc = minibatch(j, rowMode, st);
    cudaGraph_t graph = nullptr;
    cudaError_t e = cudaStreamEndCapture(st, &graph);
    *invalidated = e == cudaErrorStreamCaptureInvalidated;
    if (rc) {
        if (graph) cudaGraphDestroy(graph);
        return rc;
    }
    if (e != cudaSuccess) return cuda_fail(e, "train capture");
    // this library's kernels: the NCCL all-reduce adds one NCCL kernel per
    // minibatch (two, one per grouped half, when overlapped)
    const size_t ncclPerMinibatch = world > 1 && !p2pOn ? (overlapAllreduce ? 2 : 1) : 0;
    trainKernels = count_kernel_nodes(graph) - ncclPerMinibatch * (size_t)minibatches;
    cudaGraphExec_t exec = nullptr;
    e = cudaGraphInstantiate(&exec, graph, 0);
    cudaGraphDestroy(graph);
    if (e != cudaSuccess) return cuda_fail(e, "train graph instantiate");
    if (trainExec) cudaGraphExecDestroy(trainExec);
    trainExec = exec;
    trainExecMinibatches = minibatches;
    trainExecRowMode = rowMode;
    trainHp = hp;
    return MG_OK;
}

// model/ppo.h:716-751
int PpoEngine::collect() {
    NvtxRange range("mg.collect");
    MG_CUDA_TRY(cudaSetDevice(gym->device));
    cudaStream_t st = gym->stream;
    if (!rolloutStarted) {
        int rc = gym->ops->step(gym->states, actionSlots, obsSlots, rewardSlots, gym->done, nullptr, gym->rng, R,
                                reinterpret_cast<mg_stream_t>(st));
        if (rc) return fail(rc, "collect: first env step failed");
        rolloutStarted = true;
    } else {
        MG_CUDA_TRY(cudaMemcpyAsync(obsSlots, obsSlots + (size_t)T * R * O, (size_t)R * O * 4,
                                    cudaMemcpyDeviceToDevice, st));
    }
    if (!collectExec || !(collectHp == hp)) MG_TRY(captureCollect());
    MG_CUDA_TRY(cudaEventRecord(phaseEv[0], st));
    MG_CUDA_TRY(cudaGraphLaunch(collectExec, st));
    MG_CUDA_TRY(cudaEventRecord(phaseEv[1], st));
    MG_TRY(checkStatus("collect"));
    MG_CUDA_TRY(cudaEventElapsedTime(&lastCollectMs, phaseEv[0], phaseEv[1]));
    return MG_OK;
}

// Host schedule entry k: the minibatch's rows (a slot, model/ppo.h:918-923,
// or a row-permutation key and base) and the beta powers of its Adam step
// (model/ppo.h:874-880).
static void schedule_step(PpoEngine& e, int k, const MgMinibatch& mb) {
    e.stepCounter += 1.0f;
    e.hostSched[k] = mb;
    e.hostSchedBetaPow[2 * k] = std::pow(0.9f, e.stepCounter);
    e.hostSchedBetaPow[2 * k + 1] = std::pow(0.999f, e.stepCounter);
}

static MgMinibatch slot_minibatch(uint32_t t) {
    MgMinibatch m{};
    m.slot = (int32_t)t;
    return m;
}

static MgMinibatch row_minibatch(const uint32_t key[4], uint32_t base) {
    MgMinibatch m{};
    for (int i = 0; i < 4; i++) m.key[i] = key[i];
    m.base = base;
    m.slot = -1;
    return m;
}

bool PpoEngine::collectFusedApplies() const { return collect_fused_supported(gym->ops, E, H, L, O); }

int PpoEngine::setFusedMinibatch(bool on) {
    if (on != fusedMinibatch && trainExec) {
        cudaGraphExecDestroy(trainExec);  // recaptured by the next train()
        trainExec = nullptr;
    }
    fusedMinibatch = on;
    return MG_OK;
}

bool PpoEngine::useFusedCollect() const {
    if (collectMode >= 0) return collectMode == 1;
    return collectFusedApplies() && R <= kFusedCollectAutoRows;
}

int PpoEngine::setCollectMode(int mode) {
    MG_CHECK_ARG(mode >= -1 && mode <= 1, "setCollectMode: mode must be -1 (automatic), 0 (graph) or 1 (fused)");
    if (mode == 1 && !collectFusedApplies())
        return fail(MG_ERR_UNSUPPORTED,
                    "setCollectMode: no fused collect kernel for this environment and policy shape (an "
                    "environment with a State of at most 64 bytes and at most 32 observations; embed 128, hidden "
                    "512, 1-4 blocks)");
    collectMode = mode;
    if (collectExec && collectExecFused != useFusedCollect()) {
        cudaGraphExecDestroy(collectExec);  // recaptured by the next collect()
        collectExec = nullptr;
    }
    return MG_OK;
}

int PpoEngine::setMinibatchRows(int rows) {
    MG_CHECK_ARG(rows >= 0, "minibatchRows must be >= 0");
    if (rows > 0) {
        const int64_t total = (int64_t)T * R;
        MG_CHECK_ARG(rows <= total && total % rows == 0,
                     "minibatchRows must divide horizon x parallels (" + std::to_string(total) + ")");
        MG_CHECK_ARG(total < (int64_t)1 << 31, "row-mode minibatches need horizon x parallels < 2^31");
    }
    mbRows = rows;
    return MG_OK;
}

// A communicator the watchdog aborted is gone: no further training with it.
int PpoEngine::commUsable(const char* what) {
    if (world > 1 && comm && !p2pOn && comm_aborted(comm))
        return fail(MG_ERR_COMM, std::string(what) + ": the communicator was aborted after a failed all-reduce");
    return MG_OK;
}

int PpoEngine::train(int epochs) {
    MG_CHECK_ARG(epochs >= 0, "train: epochs must be >= 0");
    if (epochs == 0) return MG_OK;
    NvtxRange range("mg.train");
    MG_TRY(commUsable("train"));
    MG_CUDA_TRY(cudaSetDevice(gym->device));
    cudaStream_t st = gym->stream;
    const bool rowMode = mbRows > 0;
    const int rows = rowMode ? mbRows : R;
    if (trainBufRows != rows) MG_TRY(allocTrain(rows));
    const int nmb = rowMode ? (int)((int64_t)T * R / mbRows) : T;
    MG_TRY(ensureSchedule(nmb, epochs * nmb));
    int k = 0;
    for (int e = 0; e < epochs; e++) {
        if (rowMode) {
            // every epoch visits the T x R rows once, in a new keyed order
            uint32_t key[4];
            for (auto& w : key) w = (uint32_t)hostRng();
            for (int m = 0; m < nmb; m++) schedule_step(*this, k++, row_minibatch(key, (uint32_t)m * (uint32_t)rows));
        } else {
            std::shuffle(slotOrder.begin(), slotOrder.end(), hostRng);
            for (uint32_t t : slotOrder) schedule_step(*this, k++, slot_minibatch(t));
        }
    }
    if (!trainExec || trainExecMinibatches != nmb || trainExecRowMode != rowMode || !(trainHp == hp))
        MG_TRY(captureTrain(nmb, rowMode));
    MG_CUDA_TRY(cudaEventRecord(phaseEv[2], st));
    for (int e = 0; e < epochs; e++) {
        MG_CUDA_TRY(cudaMemcpyAsync(sched, hostSched + (size_t)e * nmb, (size_t)nmb * sizeof(MgMinibatch),
                                    cudaMemcpyHostToDevice, st));
        MG_CUDA_TRY(cudaMemcpyAsync(schedBetaPow, hostSchedBetaPow + (size_t)e * nmb * 2, (size_t)nmb * 8,
                                    cudaMemcpyHostToDevice, st));
        MG_CUDA_TRY(cudaGraphLaunch(trainExec, st));
    }
    MG_CUDA_TRY(cudaEventRecord(phaseEv[3], st));
    MG_TRY(checkStatus("train"));
    MG_CUDA_TRY(cudaEventElapsedTime(&lastTrainMs, phaseEv[2], phaseEv[3]));
    return MG_OK;
}

int PpoEngine::trainSlot(int t) {
    MG_CHECK_ARG(t >= 0 && t < T, "trainSlot: slot out of range");
    NvtxRange range("mg.trainSlot");
    MG_TRY(commUsable("trainSlot"));
    MG_CUDA_TRY(cudaSetDevice(gym->device));
    cudaStream_t st = gym->stream;
    if (trainBufRows != R) MG_TRY(allocTrain(R));
    MG_TRY(ensureSchedule(1, 1));
    schedule_step(*this, 0, slot_minibatch((uint32_t)t));
    MG_CUDA_TRY(cudaMemcpyAsync(sched, hostSched, sizeof(MgMinibatch), cudaMemcpyHostToDevice, st));
    MG_CUDA_TRY(cudaMemcpyAsync(schedBetaPow, hostSchedBetaPow, 8, cudaMemcpyHostToDevice, st));
    // single minibatches run eagerly (no graph): trainSlot is the manual path
    MG_TRY(minibatch(0, false, st));
    return checkStatus("trainSlot");
}

int PpoEngine::trainRows(const uint32_t key[4], uint32_t base) {
    MG_CHECK_ARG(mbRows > 0, "trainRows: set minibatchRows first");
    MG_CHECK_ARG((int64_t)base + mbRows <= (int64_t)T * R, "trainRows: base + minibatchRows exceeds the rollout");
    MG_TRY(commUsable("trainRows"));
    MG_CUDA_TRY(cudaSetDevice(gym->device));
    cudaStream_t st = gym->stream;
    if (trainBufRows != mbRows) MG_TRY(allocTrain(mbRows));
    MG_TRY(ensureSchedule(1, 1));
    schedule_step(*this, 0, row_minibatch(key, base));
    MG_CUDA_TRY(cudaMemcpyAsync(sched, hostSched, sizeof(MgMinibatch), cudaMemcpyHostToDevice, st));
    MG_CUDA_TRY(cudaMemcpyAsync(schedBetaPow, hostSchedBetaPow, 8, cudaMemcpyHostToDevice, st));
    MG_TRY(minibatch(0, true, st));
    return checkStatus("trainRows");
}

int PpoEngine::forward() {
    NvtxRange range("mg.forward");
    MG_CUDA_TRY(cudaSetDevice(gym->device));
    MG_TRY(forwardOn(static_cast<const float*>(gym->obs), R, collectActs, gym->stream));
    return checkStatus("forward");
}

// model/ppo.h:688-702
int PpoEngine::actGreedy(int source, void* hostOut) {
    MG_CHECK_ARG(source == MG_PPO_HEAD || source == MG_PPO_TRAIN_HEAD,
                 "actGreedy: the head is MG_PPO_HEAD or MG_PPO_TRAIN_HEAD");
    const void* head = source == MG_PPO_HEAD ? collectActs.head : trainActs.head;
    const int rows = source == MG_PPO_HEAD ? R : trainBufRows;
    MG_CHECK_ARG(head && rows >= R, "actGreedy: that head does not hold a row per environment");
    MG_CUDA_TRY(cudaSetDevice(gym->device));
    cudaStream_t st = gym->stream;
    MG_TRY(act_greedy(head, R, A, cont, gym->actions, st));
    if (hostOut) MG_CUDA_TRY(cudaMemcpyAsync(hostOut, gym->actions, (size_t)R * actBytes, cudaMemcpyDeviceToHost, st));
    MG_CUDA_TRY(cudaStreamSynchronize(st));
    return MG_OK;
}

// model/ppo.h:925-943 (means on the device; gradNorm is the pre-clip norm)
int PpoEngine::lastStats(float out6[6]) {
    MG_CUDA_TRY(cudaSetDevice(gym->device));
    cudaStream_t st = gym->stream;
    MG_TRY(stats_mean(stats, trainBufRows, statsMean, st));
    MG_CUDA_TRY(cudaMemcpyAsync(hostStats, statsMean, 5 * 4, cudaMemcpyDeviceToHost, st));
    MG_CUDA_TRY(cudaMemcpyAsync(hostStats + 5, normSq, 4, cudaMemcpyDeviceToHost, st));
    MG_CUDA_TRY(cudaStreamSynchronize(st));
    for (int i = 0; i < 5; i++) out6[i] = hostStats[i];
    out6[5] = std::sqrt(hostStats[5]);
    return MG_OK;
}

// model/ppo.h:460-469
int PpoEngine::setLogStd(float v) {
    MG_CHECK_ARG(cont, "setLogStd needs a continuous Env::Action");
    std::vector<float> m(A, v);
    std::vector<uint16_t> w(A, host_f2bf(v));
    const size_t off = params[pLogStd].offset;
    MG_CUDA_TRY(cudaSetDevice(gym->device));
    MG_CUDA_TRY(cudaStreamSynchronize(gym->stream));
    MG_CUDA_TRY(cudaMemcpy(master + off, m.data(), A * 4, cudaMemcpyHostToDevice));
    MG_CUDA_TRY(cudaMemcpy(weights + off, w.data(), A * 2, cudaMemcpyHostToDevice));
    return MG_OK;
}

int PpoEngine::logStd(int k, float* out) {
    MG_CHECK_ARG(cont, "logStdValue needs a continuous Env::Action");
    MG_CHECK_ARG(k >= 0 && k < A, "logStdValue: index out of range");
    uint16_t h = 0;
    MG_CUDA_TRY(cudaSetDevice(gym->device));
    MG_CUDA_TRY(cudaStreamSynchronize(gym->stream));
    MG_CUDA_TRY(cudaMemcpy(&h, weights + params[pLogStd].offset + k, 2, cudaMemcpyDeviceToHost));
    *out = host_bf2f(h);
    return MG_OK;
}

// ------------------------------------------------------------ checkpoints

namespace {

constexpr char kCkptMagic[8] = {'M', 'G', 'C', 'K', 'P', 'T', '0', '1'};

struct CkptHeader {
    char magic[8];
    uint32_t rows, obsDim, actDim, embed, hidden, layers, horizon, continuous;
    uint32_t stateBytes, obsBytes, actionBytes, paramCount;
    uint64_t optCount;
    float stepCounter, lr;
    int32_t minibatchRows, rolloutStarted;
    float hyper[6];  // clip, valueCoef, entropyCoef, maxGradNorm, gamma, lambda
    uint32_t rngTextBytes;
};

struct File {
    FILE* f = nullptr;
    ~File() {
        if (f) fclose(f);
    }
};

// Device buffer <-> file through a host staging vector.
int write_dev(FILE* f, const void* dev, size_t bytes) {
    std::vector<char> h(bytes);
    MG_CUDA_TRY(cudaMemcpy(h.data(), dev, bytes, cudaMemcpyDeviceToHost));
    if (fwrite(h.data(), 1, bytes, f) != bytes) return fail(MG_ERR_ARGUMENT, "checkpoint: write failed");
    return MG_OK;
}
int read_dev(FILE* f, void* dev, size_t bytes) {
    std::vector<char> h(bytes);
    if (fread(h.data(), 1, bytes, f) != bytes) return fail(MG_ERR_ARGUMENT, "checkpoint: file truncated");
    MG_CUDA_TRY(cudaMemcpy(dev, h.data(), bytes, cudaMemcpyHostToDevice));
    return MG_OK;
}

}  // namespace

int PpoEngine::save(const char* path) {
    MG_CHECK_ARG(path && *path, "save: empty path");
    MG_CUDA_TRY(cudaSetDevice(gym->device));
    MG_CUDA_TRY(cudaStreamSynchronize(gym->stream));
    File file;
    file.f = fopen(path, "wb");
    if (!file.f) return fail(MG_ERR_ARGUMENT, std::string("save: cannot open ") + path);
    std::ostringstream rs;
    rs << hostRng;
    const std::string rng = rs.str();
    CkptHeader h{};
    std::memcpy(h.magic, kCkptMagic, 8);
    h.rows = R; h.obsDim = O; h.actDim = A; h.embed = E; h.hidden = H; h.layers = L; h.horizon = T;
    h.continuous = cont ? 1 : 0;
    h.stateBytes = (uint32_t)gym->ops->state_bytes;
    h.obsBytes = (uint32_t)gym->ops->obs_bytes;
    h.actionBytes = (uint32_t)actBytes;
    h.paramCount = (uint32_t)params.size();
    h.optCount = optCount;
    h.stepCounter = stepCounter;
    h.lr = lr;
    h.minibatchRows = mbRows;
    h.rolloutStarted = rolloutStarted ? 1 : 0;
    const float hy[6] = {hp.clip, hp.valueCoef, hp.entropyCoef, hp.maxGradNorm, hp.gamma, hp.lambda};
    std::memcpy(h.hyper, hy, sizeof(hy));
    h.rngTextBytes = (uint32_t)rng.size();
    FILE* f = file.f;
    if (fwrite(&h, sizeof(h), 1, f) != 1 || fwrite(rng.data(), 1, rng.size(), f) != rng.size() ||
        fwrite(slotOrder.data(), 4, slotOrder.size(), f) != slotOrder.size())
        return fail(MG_ERR_ARGUMENT, "save: write failed");
    MG_TRY(write_dev(f, weights, optCount * 2));
    MG_TRY(write_dev(f, master, optCount * 4));
    MG_TRY(write_dev(f, mom, optCount * 4));
    MG_TRY(write_dev(f, var, optCount * 4));
    MG_TRY(write_dev(f, obsSlots + (size_t)T * R * O, (size_t)R * O * 4));  // next collect's first obs
    MG_TRY(write_dev(f, gym->states, (size_t)R * h.stateBytes));
    MG_TRY(write_dev(f, gym->done, (size_t)R));
    MG_TRY(write_dev(f, gym->rng, (size_t)R * 4));
    MG_TRY(write_dev(f, gym->obs, (size_t)R * h.obsBytes));
    return MG_OK;
}

int PpoEngine::load(const char* path) {
    MG_CHECK_ARG(path && *path, "load: empty path");
    MG_CUDA_TRY(cudaSetDevice(gym->device));
    MG_CUDA_TRY(cudaStreamSynchronize(gym->stream));
    File file;
    file.f = fopen(path, "rb");
    if (!file.f) return fail(MG_ERR_ARGUMENT, std::string("load: cannot open ") + path);
    FILE* f = file.f;
    CkptHeader h{};
    if (fread(&h, sizeof(h), 1, f) != 1 || std::memcmp(h.magic, kCkptMagic, 8) != 0)
        return fail(MG_ERR_ARGUMENT, "load: not a metalgym_b200 checkpoint");
    const bool same = h.rows == (uint32_t)R && h.obsDim == (uint32_t)O && h.actDim == (uint32_t)A &&
                      h.embed == (uint32_t)E && h.hidden == (uint32_t)H && h.layers == (uint32_t)L &&
                      h.horizon == (uint32_t)T && h.continuous == (cont ? 1u : 0u) &&
                      h.stateBytes == gym->ops->state_bytes && h.obsBytes == gym->ops->obs_bytes &&
                      h.actionBytes == actBytes && h.paramCount == params.size() && h.optCount == optCount;
    if (!same) return fail(MG_ERR_ARGUMENT, "load: checkpoint of a different model or environment shape");
    std::string rng(h.rngTextBytes, '\0');
    std::vector<uint32_t> order(T);
    if (fread(&rng[0], 1, rng.size(), f) != rng.size() || fread(order.data(), 4, order.size(), f) != order.size())
        return fail(MG_ERR_ARGUMENT, "load: file truncated");
    MG_TRY(read_dev(f, weights, optCount * 2));
    MG_TRY(read_dev(f, master, optCount * 4));
    MG_TRY(read_dev(f, mom, optCount * 4));
    MG_TRY(read_dev(f, var, optCount * 4));
    MG_TRY(read_dev(f, obsSlots + (size_t)T * R * O, (size_t)R * O * 4));
    MG_TRY(read_dev(f, gym->states, (size_t)R * h.stateBytes));
    MG_TRY(read_dev(f, gym->done, (size_t)R));
    MG_TRY(read_dev(f, gym->rng, (size_t)R * 4));
    MG_TRY(read_dev(f, gym->obs, (size_t)R * h.obsBytes));
    std::istringstream rs(rng);
    rs >> hostRng;
    if (rs.fail()) return fail(MG_ERR_ARGUMENT, "load: bad generator state");
    slotOrder = order;
    stepCounter = h.stepCounter;
    lr = h.lr;
    rolloutStarted = h.rolloutStarted != 0;
    hp.clip = h.hyper[0];
    hp.valueCoef = h.hyper[1];
    hp.entropyCoef = h.hyper[2];
    hp.maxGradNorm = h.hyper[3];
    hp.gamma = h.hyper[4];
    hp.lambda = h.hyper[5];
    MG_TRY(setMinibatchRows(h.minibatchRows));
    // a captured train graph holds lr in its Adam launches
    if (trainExec) {
        cudaGraphExecDestroy(trainExec);
        trainExec = nullptr;
    }
    return MG_OK;
}

// ------------------------------------------------------------ peer all-reduce

// Allocates this rank's exchange region (zeroed: flags, buffers and their
// padding) and returns its CUDA IPC handle (64 bytes).
int PpoEngine::p2pHandle(void* out64) {
    MG_CHECK_ARG(out64, "p2pHandle: null output");
    MG_CUDA_TRY(cudaSetDevice(gym->device));
    if (!p2pRegion) {
        const size_t bytes = p2p_region_bytes((int64_t)optCount, (int64_t)optFloatCount);
        MG_CUDA_TRY(cudaMalloc(&p2pRegion, bytes));
        MG_CUDA_TRY(cudaMemset(p2pRegion, 0, bytes));
        MG_TRY(dalloc(&p2pSeq, 4));
        MG_TRY(dalloc(&p2pCounter, 4));
        MG_CUDA_TRY(cudaMemset(p2pSeq, 0, 4));
        MG_CUDA_TRY(cudaMemset(p2pCounter, 0, 4));
        MG_CUDA_TRY(cudaDeviceSynchronize());
    }
    cudaIpcMemHandle_t h;
    MG_CUDA_TRY(cudaIpcGetMemHandle(&h, p2pRegion));
    std::memcpy(out64, &h, sizeof(h));
    return MG_OK;
}

// Opens the other ranks' regions (handles: world x 64 bytes, rank order) and
// switches train() to the peer all-reduce. Every rank must have called
// p2pHandle before any rank trains; the caller synchronises the ranks after
// this call (a host barrier) before the first train().
int PpoEngine::p2pOpen(const void* handles, int r, int w) {
    MG_CHECK_ARG(handles && w >= 2 && w <= kP2PMaxRanks && r >= 0 && r < w, "p2pOpen: bad rank / world size");
    MG_CHECK_ARG(p2pRegion, "p2pOpen: call p2pHandle first");
    MG_CHECK_ARG(!p2pOn, "p2pOpen: already open");
    MG_CUDA_TRY(cudaSetDevice(gym->device));
    P2PTable t{};
    for (int p = 0; p < w; p++) {
        if (p == r) {
            t.base[p] = static_cast<unsigned char*>(p2pRegion);
            continue;
        }
        cudaIpcMemHandle_t h;
        std::memcpy(&h, static_cast<const char*>(handles) + (size_t)p * sizeof(h), sizeof(h));
        void* ptr = nullptr;
        cudaError_t e = cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess) {
            for (void* q : p2pOpened) cudaIpcCloseMemHandle(q);
            p2pOpened.clear();
            return cuda_fail(e, "cudaIpcOpenMemHandle");
        }
        p2pOpened.push_back(ptr);
        t.base[p] = static_cast<unsigned char*>(ptr);
    }
    p2p_layout(t, (int64_t)optCount, (int64_t)optFloatCount);
    t.rank = r;
    t.world = w;
    p2pTable = t;
    p2pOn = true;
    rank = r;
    world = w;
    if (trainExec) {
        cudaGraphExecDestroy(trainExec);
        trainExec = nullptr;
    }
    return MG_OK;
}

// The two gradient-arena ranges of each half of the overlapped all-reduce:
// the float-gradient parameters come first in the arena, then the GEMM
// weights, each group in parameter order, so block 0 and the input layer own
// a prefix of both groups and the later blocks, final LayerNorm, head and
// log-std the suffixes.
void PpoEngine::overlapRanges() {
    const uint64_t lateF = L > 1 ? params[pLnG[1]].offset : params[pLnFg].offset;
    const uint64_t lateB = L > 1 ? params[pUp[1]].offset : params[pHead].offset;
    arEarly = {{{0, lateF}, {optFloatCount, lateB}}};
    arLate = {{{lateF, optFloatCount}, {lateB, optCount}}};
}

int PpoEngine::allreduceRanges(const ArRanges& rg, cudaStream_t s) {
    Nccl& nc = nccl();
    ncclResult_t r = nc.groupStart();
    for (int i = 0; i < 2 && r == ncclSuccess; i++) {
        const uint64_t b = rg.r[i][0], e = rg.r[i][1];
        if (e > b) r = nc.allReduce(grad + b, grad + b, (size_t)(e - b), ncclFloat, ncclSum, static_cast<ncclComm_t>(comm), s);
    }
    const ncclResult_t r2 = nc.groupEnd();
    if (r != ncclSuccess) return nccl_fail(r, "ncclAllReduce (overlapped)");
    if (r2 != ncclSuccess) return nccl_fail(r2, "ncclGroupEnd");
    return MG_OK;
}

int PpoEngine::setAllreduceOverlap(bool on) {
    overlapRanges();
    if (on != overlapAllreduce && trainExec) {
        cudaGraphExecDestroy(trainExec);  // recaptured by the next train()
        trainExec = nullptr;
    }
    overlapAllreduce = on;
    return MG_OK;
}

int PpoEngine::setComm(void* c, int r, int w) {
    MG_CHECK_ARG(w >= 1 && r >= 0 && r < w, "setComm: bad rank / world size");
    MG_CHECK_ARG(w == 1 || c, "setComm: a communicator is needed for world size > 1");
    if (c && comm_aborted(c)) return fail(MG_ERR_COMM, "setComm: the communicator was aborted");
    if (w > 1 && !nccl().ok) return fail(MG_ERR_COMM, "NCCL (libnccl.so.2) could not be loaded");
    if (trainExec) {
        cudaGraphExecDestroy(trainExec);
        trainExec = nullptr;
    }
    comm_unbind_graph(comm, &trainExec);
    comm = c;
    rank = r;
    world = w;
    if (w > 1) comm_bind_graph(comm, &trainExec);
    return MG_OK;
}

}  // namespace mg
