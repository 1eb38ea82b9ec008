// The runtime behind the drop-in Gym<Env> / PPOModel<Env> API: a gym core
// (env buffers, stream, RNG) and a PPO engine (parameters, rollout slots,
// activations, CUDA graphs), both sized at run time from the registered
// environment's mg_env_ops. Exposed through the mg_gym_* / mg_ppo_* C ABI.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <random>
#include <vector>

#include "../../include/metalgym_b200.h"
#include "block.h"
#include "gemm.h"
#include "p2p.h"
#include "policy.h"

namespace mg {

// gym.h:15-121: device, stream, and the six per-env buffers.
struct GymCore {
    const mg_env_ops* ops = nullptr;
    int n = 0;
    int device = 0;
    uint32_t seed = 0;
    uint32_t firstEnvId = 0;
    cudaStream_t stream = nullptr;
    void* states = nullptr;
    void* actions = nullptr;
    void* obs = nullptr;
    float* reward = nullptr;
    uint8_t* done = nullptr;
    uint32_t* rng = nullptr;
    // pinned staging for run(): actions in, rewards out
    void* hostActions = nullptr;
    float* hostReward = nullptr;
    // rings for run_random (allocated on first use)
    void* obsRing = nullptr;
    float* rewardRing = nullptr;
    uint8_t* doneRing = nullptr;
    int ringSlots = 0;
    int steps_rng_reserved = 0;
    // Set when a data-parallel train() aborted its communicator and the
    // stream had not drained within the watchdog's limit: its kernels may
    // still run, so teardown leaves every device and pinned buffer allocated
    // (freeing them would block without limit or free memory in use).
    bool busy = false;
    bool stillBusy() const;

    ~GymCore();
};

int gym_create(const char* name, int n, uint32_t seed, uint32_t firstEnvId, int device, GymCore** out);

struct PpoHyper {
    float clip = 0.2f, valueCoef = 0.5f, entropyCoef = 0.01f, maxGradNorm = 0.5f, gamma = 0.99f, lambda = 0.95f;
    bool operator==(const PpoHyper& o) const {
        return clip == o.clip && valueCoef == o.valueCoef && entropyCoef == o.entropyCoef &&
               maxGradNorm == o.maxGradNorm && gamma == o.gamma && lambda == o.lambda;
    }
};

// Per-forward activation pointers (collect shares one set across blocks).
struct ActSet {
    void* h = nullptr;        // residual stream, R x E bf16 (updated in place)
    std::vector<void*> lnXn;  // per block, R x E
    std::vector<void*> lnOut;
    std::vector<float*> lnSd;
    std::vector<void*> v;     // per block, R x H (post-ReLU)
    void* fXn = nullptr;
    void* fOut = nullptr;
    float* fSd = nullptr;
    void* head = nullptr;  // R x 64
};

struct ParamSpec {
    uint32_t count;
    bool gradIsFloat;
    uint64_t offset;
};

class PpoEngine {
   public:
    PpoEngine(GymCore* gym, int embed, int scale, int layers, float lr, int horizon, uint32_t seed);
    ~PpoEngine();
    int init();  // allocation + seeded init; returns MG_OK or an error

    int collect();
    int train(int epochs);
    int trainSlot(int t);
    // Minibatch rows of train(): 0 = one time slot per minibatch (the
    // reference); B > 0 = B rollout rows drawn without replacement per epoch.
    int setMinibatchRows(int rows);
    // collect() as one persistent kernel (collect_fused.cu) or as the
    // captured per-step graph: mode 1 = the kernel (MG_ERR_UNSUPPORTED where
    // the environment or the policy shape has none), 0 = the graph, -1 =
    // automatic, the default: the kernel where it applies and the rollout has
    // at most kFusedCollectAutoRows parallels (one wave of clusters; there the
    // two paths give identical rollouts).
    int setCollectMode(int mode);
    bool collectFusedApplies() const;
    bool useFusedCollect() const;
    static constexpr int kFusedCollectAutoRows = 4096;
    // With an NCCL communicator (world > 1): all-reduce the gradients of
    // everything but the last backward layer (block 0 and the input layer) on
    // the side stream while that layer's backward runs, then the rest. Off by
    // default; the sums and the averaged gradient are those of the single
    // all-reduce.
    int setAllreduceOverlap(bool on);
    // One row-mode minibatch with explicit permutation key and base (tests).
    int trainRows(const uint32_t key[4], uint32_t base);
    int forward();  // on the gym's live obs; head in the collect activations
    int lastStats(float out6[6]);
    // actGreedy on the device from the collect head (source MG_PPO_HEAD) or
    // the last training forward's (MG_PPO_TRAIN_HEAD) into the gym's actions,
    // copied to hostOut too when it is given; blocks.
    int actGreedy(int source, void* hostOut);
    int setLogStd(float v);
    int logStd(int k, float* out);
    int setComm(void* comm, int rank, int world);
    // Checkpoint of the whole training state: parameters and Adam moments,
    // step counter, the host shuffle generator, the last rollout observation
    // and the gym's env states / done flags / RNG words, so that training
    // resumed from it continues exactly as it would have.
    int save(const char* path);
    int load(const char* path);

    GymCore* gym;
    int device;  // the gym's device, kept for the destructor
    int R, O, A, E, H, L, T;
    bool cont;
    size_t actBytes;
    float lr;
    uint32_t seed;
    PpoHyper hp;
    bool rolloutStarted = false;
    int collectMode = -1;          // setCollectMode
    bool collectExecFused = false;  // the path collectExec was captured with
    float stepCounter = 0.0f;  // model/ppo.h:265 (float, as the reference)
    std::mt19937 hostRng;      // slot shuffle (model/ppo.h:349, 920), row-mode keys
    int mbRows = 0;            // 0: slot mode; > 0: rows per row-mode minibatch
    int trainBufRows = 0;      // rows the training buffers are sized for
    std::vector<uint32_t> slotOrder;

    std::vector<ParamSpec> params;
    uint32_t pInW, pInB, pLnFg, pLnFb, pHead, pLogStd;
    std::vector<uint32_t> pLnG, pLnB, pUp, pDown;
    uint64_t optCount = 0, optFloatCount = 0;

    // parameter state (device)
    uint16_t* weights = nullptr;
    float *master = nullptr, *mom = nullptr, *var = nullptr, *grad = nullptr;
    // rollout slots (device), layouts of model/ppo.h:336-345
    float* obsSlots = nullptr;
    void* actionSlots = nullptr;
    float *logpSlots = nullptr, *valueSlots = nullptr, *rewardSlots = nullptr, *advSlots = nullptr,
          *retSlots = nullptr;
    uint8_t* doneSlots = nullptr;
    float* advStats = nullptr;    // T x {mean, inv}
    float* mbAdvStats = nullptr;  // {mean, inv} of the current row-mode minibatch
    double* advPartial = nullptr;           // its per-CTA sums
    unsigned int* advCounter = nullptr;     // last-CTA detection
    // activations
    ActSet collectActs, trainActs;
    void *dLogits = nullptr, *dBranch = nullptr;
    std::vector<void*> dS;   // L + 1: dS[n + 1] = gradient at the output of block n, dS[L] from the head
    std::vector<void*> dVs;  // L: masked gradient of each block's hidden layer
    // the weight-gradient GEMMs run on a side stream, forked from the
    // input-gradient chain when their operands are ready and joined before
    // the gradient finalisation
    cudaStream_t side = nullptr;
    std::vector<cudaEvent_t> forkEv;  // L + 1
    cudaEvent_t joinEv = nullptr;
    float* stats = nullptr;  // R x 5
    // gradient partials
    std::vector<float*> upPart, downPart, lnPart;
    float *headPart = nullptr, *lnFPart = nullptr, *inPart = nullptr, *lsPart = nullptr;
    int upSplits = 1, downSplits = 1, headSplits = 1;
    GradSegmentTable gradTable{};
    int nNorm = 0;  // CTAs of the finalize kernel = norm partials
    float* normPartial = nullptr;
    float* normSq = nullptr;
    unsigned int* normCounter = nullptr;  // last-CTA detection of the norm reduction
    float* statsMean = nullptr;  // 5 floats
    // per-minibatch schedule: rows (slot or permutation key) and the Adam
    // bias-correction powers; the device holds one epoch, the host all epochs
    int maxSchedule = 0, maxHostSchedule = 0;
    MgMinibatch* sched = nullptr;       // device
    float* schedBetaPow = nullptr;      // device, 2 per minibatch
    MgMinibatch* hostSched = nullptr;   // pinned
    float* hostSchedBetaPow = nullptr;
    // host-side LossStats readback
    float* hostStats = nullptr;  // pinned, 6 floats

    // graphs
    cudaGraphExec_t collectExec = nullptr;
    cudaGraphExec_t trainExec = nullptr;
    size_t collectKernels = 0, trainKernels = 0;  // kernel nodes of the captured graphs
    int trainExecMinibatches = 0;  // per replay (one epoch)
    bool trainExecRowMode = false;
    PpoHyper collectHp, trainHp;

    // one fused kernel per residual block forward (block_fwd.cu) where the
    // widths allow it and there are enough row tiles to fill the GPU (with
    // few tiles the chain of LayerNorm + two GEMMs, spread over more CTAs,
    // is faster), else LayerNorm + two GEMMs
    bool fusedBlocks = false;
    bool useFusedBlock(int rows) const { return fusedBlocks && rows >= kFusedBlockMinRows; }
    static constexpr int kFusedBlockMinRows = 8192;
    // the down GEMM of the unfused chain ends with the next LayerNorm
    // (gemm_tc_persist.cuh, kEpiResidLN) where the embedding width is one
    // output tile (128 or 256)
    bool lnEpilogue = false;
    bool useLnEpilogue(int rows) const { return lnEpilogue && rows >= kLnEpilogueMinRows; }
    static constexpr int kLnEpilogueMinRows = 16384;
    // the down projection and the branch gradient as cluster split-K products
    // that end with the LayerNorm forward / backward (gemm_rows.cu): at 4096
    // rows of width 128 (128 CTAs) faster than the GEMM + LayerNorm pairs
    // they replace (in CUDA graphs: 6.6 against 8.2 us forward, 7.4 against
    // 8.5 us backward). The forward one takes precedence over the fused block
    // kernel up to 4096 rows; the backward one applies up to 8192 rows
    // (10.9 against 11.1 us there).
    bool rowsKernels = false;
    bool useRowsForward(int rows) const { return rowsKernels && rows <= kRowsForwardMaxRows; }
    bool useRowsBackward(int rows) const { return rowsKernels && rows <= kRowsBackwardMaxRows; }
    static constexpr int kRowsForwardMaxRows = 4096;
    static constexpr int kRowsBackwardMaxRows = 8192;
    // a whole residual block per kernel on 4-CTA clusters (block_cluster.cu),
    // embed 128 and hidden 512; where it applies it replaces the row kernels,
    // the up / dV GEMMs before them and (backward) the two weight-gradient
    // GEMMs of the side stream. In CUDA graphs at 4096 rows: 8.3 against 11.0
    // us forward; at 8192 rows no faster than the kernels it replaces
    bool clusterBlocks = false;
    bool useBlockClusterForward(int rows) const { return clusterBlocks && rows <= kClusterForwardMaxRows; }
    bool useBlockClusterBackward(int rows) const {
        return clusterBlocks && rows <= kClusterBackwardMaxRows && gemm_rows_ln_backward_supported(rows);
    }
    // the head GEMM, loss, head dX, final LayerNorm backward and dW_head
    // partials in one kernel (head_tail.cu), categorical head, embed 128
    bool useHeadTail(int rows) const { return E == 128 && rows <= kHeadTailMaxRows && head_tail_supported(E, rows); }
    static constexpr int kHeadTailMaxRows = 4096;
    bool inputGradFusable(int rows) const {
        return O <= kBlockClusterMaxInputDim && input_backward_parts(rows, O, E) == (rows + 15) / 16;
    }
    static constexpr int kClusterForwardMaxRows = 4096;
    static constexpr int kClusterBackwardMaxRows = 4096;
    // the block forwards, the head and the block backwards of a minibatch in
    // one kernel (minibatch_tiles.cu) where each of them would run as a
    // cluster kernel of its own (block_cluster.cu, head_tail.cu). Off by
    // default: in the train graph the separate kernels, chained by
    // programmatic dependent launch, measured 2 % faster (9.84 against 10.05
    // ms per train(4) at 4096 rows); setFusedMinibatch
    bool fusedMinibatch = false;
    MinibatchTiles tilesPlan;
    int setFusedMinibatch(bool on);

    // multi-GPU: NCCL all-reduce (setComm) or the all-reduce over NVLink peer
    // memory (p2p.cu: p2pHandle on every rank, exchange, p2pOpen)
    void* comm = nullptr;
    int rank = 0, world = 1;
    void* p2pRegion = nullptr;           // this rank's exchange region (IPC-shared)
    std::vector<void*> p2pOpened;        // peers' regions opened here
    P2PTable p2pTable{};
    bool p2pOn = false;
    bool overlapAllreduce = false;  // setAllreduceOverlap
    // device time of the last collect() and train() (CUDA events around their
    // graph launches, read after the blocking wait)
    cudaEvent_t phaseEv[4] = {};
    float lastCollectMs = 0.0f, lastTrainMs = 0.0f;
    float commTimeout = 0.0f;  // seconds; > 0: train() waits through the watchdog (watchdog.h)
    struct ArRanges {
        uint64_t r[2][2];  // [begin, end) element ranges of the gradient arena
    };
    ArRanges arEarly{}, arLate{};
    GradSegmentTable gradTableEarly{}, gradTableLate{};
    float* normPartialLate = nullptr;
    cudaEvent_t arLateEv = nullptr, arEarlyEv = nullptr, arDoneEv = nullptr;
    void overlapRanges();
    int allreduceRanges(const ArRanges& rg, cudaStream_t s);
    unsigned int* p2pSeq = nullptr;      // device minibatch counter of the exchange
    unsigned int* p2pCounter = nullptr;  // last-CTA detection of the gather
    int p2pHandle(void* out64);
    int p2pOpen(const void* handles, int rank, int world);

   private:
    int forwardOn(const float* obs, int rows, ActSet& a, cudaStream_t st);
    // mt: record the cluster block passes there instead of launching them
    int blocksForward(const float* obs, const RowMap& rm, ActSet& a, int rows, cudaStream_t st,
                      MinibatchTiles* mt = nullptr);
    BlockFwdArgs blockArgs(ActSet& a, int n, int rows);
    int minibatch(int j, bool rowMode, cudaStream_t st);  // reads sched[j], schedBetaPow[2j..]
    int captureCollect();
    int captureTrain(int minibatches, bool rowMode);
    // one capture attempt; *invalidated: the capture ended invalidated (capture_mutex)
    int captureCollectOnce(bool* invalidated);
    int captureTrainOnce(int minibatches, bool rowMode, bool* invalidated);
    int ensureSchedule(int device, int host);
    int allocTrain(int rows);
    void freeTrain();
    int checkStatus(const char* what);
    int waitStream(const char* what);
    int commUsable(const char* what);
};

}  // namespace mg
