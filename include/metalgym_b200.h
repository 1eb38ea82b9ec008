/*
 * metalgym_b200 C ABI: the boundary between host code (the C++ drop-in
 * headers in include/metalgym/, Python via ctypes, or any FFI) and the
 * sm_100a CUDA kernels of the MetalGym hot path.
 *
 * Conventions
 *   - every function returns MG_OK (0) or an MG_ERR_* code; mg_last_error()
 *     gives the message of the last failure on the calling thread;
 *   - pointers named *_dev are device pointers owned by the caller, unless a
 *     function says it allocates; bf16 data is passed as void* (2-byte
 *     elements, round-to-nearest-even storage);
 *   - every launch takes a stream (a cudaStream_t; NULL = legacy default
 *     stream) and is asynchronous unless documented otherwise;
 *   - device-side waits are bounded; a kernel that gives up records a code in
 *     the device status word (mg_device_status) instead of hanging.
 *
 * Each entry point names the reference interface it replaces, as
 * file:line inside the MetalGym source tree. The reference binds kernels by
 * name through Metal pipelines (model/ppo.h:311-330, gym.h:43-64); here the
 * same kernels are plain C functions.
 */
#ifndef METALGYM_B200_H
#define METALGYM_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MG_VERSION 2

typedef struct CUstream_st* mg_stream_t;

enum mg_status_code {
    MG_OK = 0,
    MG_ERR_ARGUMENT = 1,       /* invalid size, alignment or pointer */
    MG_ERR_CUDA = 2,           /* a CUDA runtime / driver call failed */
    MG_ERR_UNSUPPORTED = 3,    /* configuration not supported by this build */
    MG_ERR_DEVICE = 4,         /* a kernel recorded a device-side error (timeout) */
    MG_ERR_NOT_FOUND = 5,      /* unknown environment kernel name */
    MG_ERR_COMM = 6            /* NCCL failure, or a collective that timed out */
};

/* ---------------------------------------------------------------- runtime */

/* Message of the last failing call on this thread ("" if none). */
const char* mg_last_error(void);
/* ABI version (MG_VERSION). */
int mg_version(void);
/* Reads the device status word of the current device into *status (0 = no
 * error; otherwise the first device-side error code recorded) and clears it
 * if `clear` is non-zero. Synchronous. Replaces the command-buffer error check
 * of model/ppo.h:507-515. */
int mg_device_status(int clear, int* status);
/* Phase trace of the 4-CTA cluster tile kernels (block, head and minibatch
 * tile kernels; no counterpart in the reference): with a device buffer of
 * uint64 [CTAs of the launch][64], thread 0 of every CTA writes %globaltimer
 * (ns) at each phase boundary of its passes into its row, in order, for the
 * kernels launched or captured afterwards; NULL (the default) turns it off.
 * For profiling only: one buffer serves every launch, so the last kernel's
 * stamps remain. */
int mg_set_tile_trace(uint64_t* buffer);

/* ---------------------------------------------------------------- GEMM */

enum mg_gemm_epilogue {
    MG_EPI_BF16 = 0,       /* out = bf16(acc) */
    MG_EPI_BF16_RELU = 1,  /* v = bf16(acc); out = v > 0 ? v : v * 0 */
    MG_EPI_BF16_RESID = 2, /* out = bf16(aux + bf16(acc)) */
    MG_EPI_BF16_MASK = 3,  /* out = bf16(acc) * (aux > 0) */
    MG_EPI_F32 = 4         /* out (fp32) = acc; with splits > 1, split z writes
                              out + z * M * ldo (partial sums) */
};

/* out[M x N] = opA(A) * opB(B) with bf16 operands and fp32 accumulation on
 * the tcgen05 tensor cores. A is K-major ([M][lda], K contiguous) or, with
 * a_mn_major, MN-major ([K][lda], M contiguous); B is K-major ([N][ldb]) or
 * MN-major ([K][ldb], N contiguous). Leading dimensions are in elements and
 * multiples of 8; bases 16-byte aligned; N a multiple of 32; K split into
 * `splits` contiguous ranges (MG_EPI_F32 only). aux is bf16 [M][ldaux].
 * Replaces the MetalPerformancePrimitives matmul2d kernels mlpForwardOne/Two,
 * mlpBackwardOne/Two/Weights (model/mlp.metal:18-208), linearForward,
 * linearBackward, linearBackwardDw (model/linear.metal:17-93). */
int mg_gemm_bf16(const void* A_dev, int a_mn_major, int lda, const void* B_dev, int b_mn_major, int ldb, int M,
                 int N, int K, int epilogue, void* out_dev, int ldo, const void* aux_dev, int ldaux, int splits,
                 mg_stream_t stream);
/* mg_gemm_bf16 with the kernel chosen by the caller (no counterpart in the
 * reference): tile_n = output tile width 32 (K-major B only), 64, 128 or 256 (0 = the library's
 * choice, persistent then only allows the persistent kernel); persistent = 1
 * selects the persistent kernel (one CTA per SM walking the tiles with the
 * accumulator double-buffered in tensor memory; tile_n 128 or 256), 0 the
 * one-CTA-per-tile kernel. Same results. */
/* The residual down-projection followed, in the same kernel, by the next
 * LayerNorm of every output row (no single counterpart in the reference:
 * mlpForwardTwo, model/mlp.metal:60-86, residualAdd, model/elementwise.
 * metal:4-13, then layernormForward, model/layernorm.metal:10-71):
 * h = bf16(h + bf16(A B)) in place ([M][N], N = 128 or 256), then x_norm,
 * ln_out, stdev exactly as mg_layernorm_forward computes them from h. A is
 * K-major [M][lda]; B as in mg_gemm_bf16. Persistent kernel, one output tile
 * per 128 rows x N. */
int mg_gemm_bf16_resid_layernorm(const void* A_dev, int lda, const void* B_dev, int b_mn_major, int ldb, int M,
                                 int N, int K, void* h_dev, const void* gamma, const void* beta, void* x_norm,
                                 void* ln_out, float* stdev, mg_stream_t stream);
/* The same two layers for 128-wide rows at few rows (CartPole's 4096): K is
 * split over a cluster of mg_gemm_rows_splits(K) CTAs whose fp32 partial
 * tiles are summed in split order through distributed shared memory, then
 * one warp per row applies the epilogue. h = bf16(h + bf16(A B)) in place
 * ([M][128]) followed by x_norm, ln_out, stdev exactly as
 * mg_layernorm_forward computes them from h. */
int mg_gemm_rows_resid_layernorm(const void* A_dev, int lda, const void* B_dev, int b_mn_major, int ldb, int M,
                                 int K, void* h_dev, const void* gamma, const void* beta, void* x_norm, void* ln_out,
                                 float* stdev, mg_stream_t stream);
/* The branch gradient of a residual block and its LayerNorm backward in one
 * kernel (model/mlp.metal:131-153, then layernormBackward, model/layernorm.
 * metal:74-127, and the skip add, model/ppo.h:851-852): dz = bf16(A B)
 * ([M][128], K split as above), then resid_out and the dgamma / dbeta
 * partials exactly as mg_layernorm_backward computes them from dz with
 * resid. Rows per partial (8, 16 or 32) must divide 32. */
int mg_gemm_rows_layernorm_backward(const void* A_dev, int lda, const void* B_dev, int b_mn_major, int ldb, int M,
                                    int K, const void* x_norm, const void* gamma, const float* stdev,
                                    const void* resid, void* resid_out, float* partial, mg_stream_t stream);
int mg_gemm_rows_splits(int K);
/* One residual block per kernel for embed 128, hidden 512 (model/mlp.metal:
 * 18-86 and the skip add, model/elementwise.metal:4-13, then the LayerNorm that
 * follows, model/layernorm.metal:10-71): v = relu(ln_out w_up) ([rows][512],
 * saved), h += v w_down in place ([rows][128]), then x_norm, next_ln_out,
 * stdev of h under gamma, beta. A 4-CTA cluster per 128 rows, CTA q owning
 * hidden columns 128q..; bit-identical to mg_gemm_bf16 (ReLU) followed by
 * mg_gemm_rows_resid_layernorm. */
int mg_block_cluster_forward(const void* ln_out, const void* w_up, const void* w_down, void* h, void* v,
                             const void* gamma, const void* beta, void* x_norm, void* next_ln_out, float* stdev,
                             int rows, mg_stream_t stream);
/* The first block's forward with the input layer and the first LayerNorm in
 * the same kernel (inputForward, model/input.metal:11-27; layernormForward,
 * model/layernorm.metal:10-71): h = bf16(b_in + obs w_in) ([rows][128], obs
 * [rows][in_dim] fp32, in_dim <= 32), then x_norm0, ln_out0, stdev0 of h,
 * then mg_block_cluster_forward on ln_out0. Bit-identical to
 * mg_input_forward, mg_layernorm_forward and mg_block_cluster_forward. */
int mg_block_cluster_forward_input(const float* obs, int in_dim, const void* w_in, const void* b_in,
                                   const void* gamma0, const void* beta0, void* x_norm0, void* ln_out0,
                                   float* stdev0, const void* w_up, const void* w_down, void* h, void* v,
                                   const void* gamma, const void* beta, void* x_norm, void* next_ln_out,
                                   float* stdev, int rows, mg_stream_t stream);
/* Its backward (model/mlp.metal:88-208, model/layernorm.metal:74-127,
 * model/ppo.h:851-852): dV = bf16(dS w_down^T) * (v > 0) (saved), then
 * resid_out and the dgamma / dbeta partials as mg_gemm_rows_layernorm_backward
 * computes them from dV w_up^T, and the weight-gradient partial sums of each
 * 128-row tile t: up_part[t] = ln_out_t^T dV_t ([128][512] fp32), down_part[t]
 * = v_t^T dS_t ([512][128] fp32) — what mg_gemm_bf16 writes as split-K
 * partials with one split per 128 rows. Bit-identical to those kernels. With
 * obs (the first block: resid_out is then the input layer's dZ), also the
 * input layer's gradient partials (inputBackward, model/input.metal:38-60)
 * as mg_input_backward_partials writes them when it takes 16 rows per
 * partial (in_dim <= 32). */
/* The head of a training minibatch in one kernel (embed 128, categorical
 * head): head = bf16(f_out w_head) (linearForward, model/linear.metal:17-37),
 * the PPO loss of every row (policyLossBackward, model/policy.metal:14-69:
 * dZ, stats, as mg_policy_loss), dS = the final LayerNorm's backward
 * (model/layernorm.metal:74-127) of bf16(dZ w_head^T) (linearBackward,
 * model/linear.metal:40-60) with its dgamma / dbeta partials as
 * mg_layernorm_backward writes them, and head_part[t] = f_out_t^T dZ_t
 * ([128][64] fp32) for every 128-row tile t (linearBackwardDw,
 * model/linear.metal:71-93, one split per tile). Bit-identical to those
 * kernels. Rows per LayerNorm partial (8, 16 or 32) must divide 32. */
int mg_head_tail(const void* f_out, const void* w_head, void* head, const int32_t* action, const float* adv,
                 const float* adv_stats, const float* ret, const float* old_log_prob, void* dZ, float* stats, int rows,
                 int act_dim, float clip, float value_coef, float entropy_coef, float* head_part,
                 const void* gamma_f, const void* x_norm_f, const float* stdev_f, void* dS, float* ln_partial,
                 mg_stream_t stream);
int mg_block_cluster_backward(const void* dS, const void* w_down, const void* v, const void* w_up, void* dV,
                              const void* ln_out, float* up_part, float* down_part, const void* x_norm,
                              const void* gamma, const float* stdev, const void* resid, void* resid_out,
                              float* partial, const float* obs, int in_dim, float* in_partial, int rows,
                              mg_stream_t stream);
int mg_gemm_bf16_tiled(const void* A_dev, int a_mn_major, int lda, const void* B_dev, int b_mn_major, int ldb,
                       int M, int N, int K, int epilogue, void* out_dev, int ldo, const void* aux_dev, int ldaux,
                       int splits, int tile_n, int persistent, mg_stream_t stream);

/* ---------------------------------------------------------------- environments */

/* The kernels of one environment type, registered by MG_REGISTER_ENV
 * (include/metalgym/register_env.cuh). Replaces the per-environment Metal
 * kernel instantiation rollout<Env> with [[host_name(KERNEL)]]
 * (rollout.h:31-54, examples/CartPole/cartpole.metal:78-87) and the pipeline
 * lookup by Env::KERNEL in Gym (gym.h:43-44, 64-69). All buffers are device
 * memory of n elements (AoS State / Action / Obs as declared by the Env). */
typedef struct mg_env_ops {
    uint32_t abi_version;
    const char* name; /* Env::KERNEL, e.g. "rollout_cartpole" */
    uint32_t state_bytes, action_bytes, obs_bytes, obs_dim, act_dim, continuous;
    /* rollout<Env> once: reset if done, step with actions, write obs/reward/done
     * (done_copy, if not NULL, gets the done flags too). */
    int (*step)(void* states, const void* actions, void* obs, float* reward, uint8_t* done, uint8_t* done_copy,
                uint32_t* rng, int n, mg_stream_t stream);
    /* `steps` steps with the random policy (mode 0: zero-logit categorical or
     * standard-normal draw from the env's word before each step; mode 1:
     * constant action 0); step k writes slot k % ring of the ring buffers. */
    int (*run_random)(void* states, void* obs_ring, float* reward_ring, uint8_t* done_ring, uint8_t* done,
                      uint32_t* rng, int n, int steps, int ring, int mode, mg_stream_t stream);
    /* One fused collect step: sample from head rows (bf16 [n][64]; log_std
     * bf16 [act_dim] for continuous envs), write action/logp/value, then
     * reset-if-done + step, writing obs_out / reward_out / done and done_slot. */
    int (*collect_step)(const void* head, const void* log_std, void* states, void* action_out, float* logp_out,
                        float* value_out, void* obs_out, float* reward_out, uint8_t* done, uint8_t* done_slot,
                        uint32_t* rng, int n, mg_stream_t stream);
    /* The whole of collect() in one persistent kernel instantiated for this
     * environment (include/metalgym/detail/collect_fused.cuh), launched with
     * the tensor maps and parameters the library prepares; NULL for
     * environments whose State does not fit in registers (over 64 bytes) or
     * whose observation has more than 32 floats. Added in ABI version 2. */
    int (*collect_fused)(const void* maps, const void* params, mg_stream_t stream);
} mg_env_ops;

/* Registers an environment (called by MG_REGISTER_ENV at load time). A later
 * registration of the same name replaces the earlier one. */
int mg_env_register(const mg_env_ops* ops);
/* The registered environment named `kernel_name`, or NULL. */
const mg_env_ops* mg_env_find(const char* kernel_name);
/* Number of registered environments and the name of the i-th. */
int mg_env_count(void);
const char* mg_env_name(int i);
/* Gym construction state (gym.h:46-61): zero states, done = 1 so the first
 * step resets every env, rng[i] = (seed + first_env_id + i) * 2654435761 + 1
 * (a word of 0 becomes 1; at seed 0 this is the reference's i * 2654435761 + 1). */
int mg_env_init(const char* kernel_name, void* states, uint8_t* done, uint32_t* rng, int n, uint32_t seed,
                uint32_t first_env_id, mg_stream_t stream);
/* By-name forms of the mg_env_ops entries. */
int mg_env_step(const char* kernel_name, void* states, const void* actions, void* obs, float* reward, uint8_t* done,
                uint8_t* done_copy, uint32_t* rng, int n, mg_stream_t stream);
int mg_env_run_random(const char* kernel_name, void* states, void* obs_ring, float* reward_ring, uint8_t* done_ring,
                      uint8_t* done, uint32_t* rng, int n, int steps, int ring, int mode, mg_stream_t stream);
int mg_env_collect_step(const char* kernel_name, const void* head, const void* log_std, void* states,
                        void* action_out, float* logp_out, float* value_out, void* obs_out, float* reward_out,
                        uint8_t* done, uint8_t* done_slot, uint32_t* rng, int n, mg_stream_t stream);

/* One whole collect() in the environment's persistent kernel
 * (mg_env_ops.collect_fused), on caller-owned device buffers in the layouts of
 * the PPO session (mg_ppo_buffer). Replaces the ~460 dispatches of collect()
 * (model/ppo.h:716-751): horizon steps of forward, sample, reset-if-done and
 * step, the bootstrap forward (its head rows into boot_head) and GAE
 * (model/gae.metal:14-36); not the advantage statistics (mg_advantage_stats).
 * Policy: embed 128, hidden 512, 1..MG_COLLECT_FUSED_MAX_BLOCKS blocks, bf16
 * weights. MG_ERR_UNSUPPORTED for an environment without the kernel. */
#define MG_COLLECT_FUSED_MAX_BLOCKS 4
typedef struct mg_collect_fused_args {
    int parallels, horizon, layers, obs_dim;
    const void* w_in;                                         /* [obs_dim][128] */
    const void* b_in;                                         /* [128] */
    const void* ln_gamma[MG_COLLECT_FUSED_MAX_BLOCKS + 1];    /* blocks 0..layers-1, then the final one */
    const void* ln_beta[MG_COLLECT_FUSED_MAX_BLOCKS + 1];
    const void* w_up[MG_COLLECT_FUSED_MAX_BLOCKS];            /* [128][512] */
    const void* w_down[MG_COLLECT_FUSED_MAX_BLOCKS];          /* [512][128] */
    const void* w_head;                                       /* [128][64] */
    const void* log_std;                                      /* [act_dim], continuous environments */
    void* states;                                             /* the environment buffers: read, then */
    uint8_t* done;                                            /* written back after the last step */
    uint32_t* rng;
    float* obs_slots;                                         /* [horizon + 1][parallels][obs_dim]; slot 0 in */
    void* action_slots;                                       /* [horizon][parallels] actions */
    float *logp_slots, *value_slots, *reward_slots;           /* [horizon][parallels] */
    uint8_t* done_slots;
    float *adv_slots, *ret_slots;
    void* boot_head;                                          /* [parallels][64] bf16 */
    float gamma, lambda;
} mg_collect_fused_args;
int mg_env_collect_fused(const char* kernel_name, const mg_collect_fused_args* args, mg_stream_t stream);

/* ---------------------------------------------------------------- policy kernels */

/* out[r][c] = bf16(b[c] + sum_k obs[r][k] * W[k][c]); W bf16 [in_dim][out_dim].
 * Replaces inputForward (model/input.metal:11-27). */
int mg_input_forward(const float* obs, const void* w, const void* b, void* out, int rows, int in_dim, int out_dim,
                     mg_stream_t stream);
/* mg_input_forward followed, in the same kernel, by the first block's
 * LayerNorm of every output row (x_norm, ln_out, stdev exactly as
 * mg_layernorm_forward computes them). No single counterpart in the
 * reference: inputForward (model/input.metal:11-27) then layernormForward
 * (model/layernorm.metal:10-71). */
int mg_input_forward_layernorm(const float* obs, const void* w, const void* b, void* out, const void* gamma,
                               const void* beta, void* x_norm, void* ln_out, float* stdev, int rows, int in_dim,
                               int out_dim, mg_stream_t stream);
/* Per-row-range partial sums of dW = obs^T dZ and db = sum_r dZ: partial holds
 * mg_input_backward_num_partials(rows, in_dim, out_dim) blocks of (in_dim + 1) x out_dim fp32
 * (rows 0..in_dim-1: dW, row in_dim: db). Replaces inputBackward
 * (model/input.metal:38-60), whose chunk sums go to fp32 atomics. */
int mg_input_backward_partials(const float* obs, const void* dZ, float* partial, int rows, int in_dim, int out_dim,
                               mg_stream_t stream);
int mg_input_backward_num_partials(int rows, int in_dim, int out_dim);
/* Row LayerNorm, eps 1e-5: x_norm = bf16(x-hat), out = bf16(gamma x-hat + beta),
 * stdev = sqrt(var + eps); cols in {64, 128, 256, 512, 1024}.
 * Replaces layernormForward (model/layernorm.metal:10-71). */
int mg_layernorm_forward(const void* x, void* x_norm, void* out, const void* gamma, const void* beta, float* stdev,
                         int rows, int cols, mg_stream_t stream);
/* LayerNorm backward. Without resid: dZ is overwritten with dX. With resid:
 * resid = bf16(bf16(dX) + resid) (the residual add of the stream) and dZ is
 * kept. partial gets mg_layernorm_backward_num_partials(rows) blocks of
 * [dgamma (cols) | dbeta (cols)]. Replaces layernormBackward
 * (model/layernorm.metal:74-127) and residualAdd (model/elementwise.metal:4-13). */
int mg_layernorm_backward(void* dZ, const void* x_norm, const void* gamma, const float* stdev, void* resid,
                          float* partial, int rows, int cols, mg_stream_t stream);
int mg_layernorm_backward_num_partials(int rows);
/* One residual MLP block forward in one kernel (no single counterpart in the
 * reference: it fuses layernormForward, model/layernorm.metal:10-71,
 * mlpForwardOne/Two, model/mlp.metal:18-86, and residualAdd,
 * model/elementwise.metal:4-13): x_norm, ln_out, stdev = LayerNorm(h) as
 * mg_layernorm_forward computes them (bit-identical), v = relu(bf16(ln_out
 * up)) ([rows][hidden]), h = bf16(h + bf16(v down)) in place. up: [embed]
 * [hidden], down: [hidden][embed], row-major bf16; embed 64 or 128, hidden a
 * multiple of 128. */
int mg_block_forward(void* h, const void* gamma, const void* beta, const void* up, const void* down, void* x_norm,
                     void* ln_out, float* stdev, void* v, int rows, int embed, int hidden, mg_stream_t stream);
/* Categorical draw per head row (bf16 [rows][64]; logits in 0..act_dim-1,
 * value at act_dim), advancing rng once. Replaces sampleAction
 * (model/sample.metal:18-47). */
int mg_sample_categorical(const void* head, uint32_t* rng, int32_t* action, float* log_prob, float* value, int rows,
                          int act_dim, mg_stream_t stream);
/* Gaussian draw (Box-Muller) with a shared log-std (bf16 [act_dim]).
 * Replaces sampleGaussian (model/gaussian.metal:42-71). */
int mg_sample_gaussian(const void* head, const void* log_std, uint32_t* rng, float* action, float* log_prob,
                       float* value, int rows, int act_dim, mg_stream_t stream);
/* Clipped PPO loss + value + entropy for a discrete head: dZ bf16 [rows][64]
 * (gradient / rows), stats fp32 [rows][5] = policy, value, entropy, approx-KL,
 * clipped. adv_stats (nullable) = {mean, 1/(std + 1e-8)} normalises adv.
 * Replaces normalizeAdvantage + policyLossBackward (model/gae.metal:42-77,
 * model/policy.metal:14-69). */
int mg_policy_loss(const void* head, const int32_t* action, const float* adv, const float* adv_stats,
                   const float* ret, const float* old_log_prob, void* dZ, float* stats, int rows, int act_dim,
                   float clip, float value_coef, float entropy_coef, mg_stream_t stream);
/* Gaussian-head PPO loss; the log-std gradient goes to
 * mg_gaussian_loss_num_partials(rows) x act_dim per-block partial sums.
 * Replaces gaussianLossBackward (model/gaussian.metal:76-135). */
int mg_gaussian_loss(const void* head, const float* action, const float* adv, const float* adv_stats,
                     const float* ret, const float* old_log_prob, void* dZ, float* stats, const void* log_std,
                     float* dlogstd_partial, int rows, int act_dim, float clip, float value_coef, float entropy_coef,
                     mg_stream_t stream);
int mg_gaussian_loss_num_partials(int rows);
/* GAE over slot-major buffers [t * rows + i], bootstrap value from column
 * act_dim of the bf16 head. Replaces gaeBackward (model/gae.metal:14-36). */
int mg_gae(const float* reward, const uint8_t* done, const float* value, const void* bootstrap_head, float* adv,
           float* ret, int rows, int horizon, int act_dim, float gamma, float lambda, mg_stream_t stream);
/* Per-slot advantage statistics {mean, 1/(population std + 1e-8)} for `slots`
 * consecutive slots of `rows` values (the statistics of normalizeAdvantage,
 * model/gae.metal:42-77). */
int mg_advantage_stats(const float* adv, float* stats_out, int rows, int slots, mg_stream_t stream);
/* out[i] = sum_p partial[p * part_stride + i] (rounded to bf16 if round_bf16),
 * and per-1024-element sums of squares into norm_partial
 * (mg_reduce_partials_num_norm_partials(count) floats). Replaces
 * reducePartials (model/elementwise.metal:21-31) and gradNormSq
 * (model/optimizer.metal:23-34). */
int mg_reduce_partials(const float* partial, int64_t part_stride, int nparts, int64_t count, float* out,
                       int round_bf16, float* norm_partial, mg_stream_t stream);
int mg_reduce_partials_num_norm_partials(int64_t count);
/* Global-norm clip + Adam (0.9, 0.999, 1e-8) on fp32 master / moments,
 * writing the bf16 weights; the squared norm is the sum of norm_partial and is
 * stored to norm_sq_out (nullable). Replaces adamStep (model/optimizer.metal:36-60). */
int mg_adam_step(float* master, const float* grad, float* momentum, float* variance, void* weights,
                 const float* norm_partial, int n_norm_partials, int64_t count, float lr, float beta1_pow,
                 float beta2_pow, float max_grad_norm, float* norm_sq_out, mg_stream_t stream);
/* Column means of the [rows][5] loss statistics (model/ppo.h:925-943). */
int mg_stats_mean(const float* stats, int rows, float* out5, mg_stream_t stream);

/* ---------------------------------------------------------------- sessions */

/* A gym session: the env buffers of gym.h:15-121 on one device, with its
 * own stream. Replaces Gym<Env>'s Metal device, queue and shared buffers. */
typedef struct mg_gym_s* mg_gym_t;
/* A PPO session borrowing a gym (model/ppo.h:145-147): parameters, rollout
 * slots, activations and the collect / train CUDA graphs. */
typedef struct mg_ppo_s* mg_ppo_t;

enum mg_gym_buffer { MG_GYM_STATES = 0, MG_GYM_ACTIONS = 1, MG_GYM_OBS = 2, MG_GYM_REWARD = 3, MG_GYM_DONE = 4,
                     MG_GYM_RNG = 5 };
enum mg_ppo_buffer {
    MG_PPO_OBS_SLOTS = 0,    /* (T+1) x rows x OBS_DIM fp32   (model/ppo.h:470) */
    MG_PPO_ACTION_SLOTS = 1, /* T x rows x Action              (model/ppo.h:471) */
    MG_PPO_LOGP_SLOTS = 2,   /* T x rows fp32 */
    MG_PPO_VALUE_SLOTS = 3,  /* T x rows fp32                   (model/ppo.h:474) */
    MG_PPO_REWARD_SLOTS = 4, /* T x rows fp32                   (model/ppo.h:472) */
    MG_PPO_DONE_SLOTS = 5,   /* T x rows uint8                  (model/ppo.h:473) */
    MG_PPO_ADV_SLOTS = 6,    /* T x rows fp32                   (model/ppo.h:475) */
    MG_PPO_RET_SLOTS = 7,    /* T x rows fp32                   (model/ppo.h:476) */
    MG_PPO_HEAD = 8,         /* rows x 64 bf16: head of the last collect / forward (model/ppo.h:450-452) */
    MG_PPO_WEIGHTS = 9,      /* opt_count bf16 weight arena     (model/ppo.h:266) */
    MG_PPO_MASTER = 10,      /* opt_count fp32 master           (model/ppo.h:269) */
    MG_PPO_MOMENTUM = 11,    /* opt_count fp32 Adam m */
    MG_PPO_VARIANCE = 12,    /* opt_count fp32 Adam v */
    MG_PPO_GRAD = 13,        /* opt_count fp32 gradient of the last minibatch */
    MG_PPO_STATS = 14,       /* rows x 5 fp32 loss statistics of the last minibatch */
    MG_PPO_ADV_STATS = 15,   /* T x {mean, 1/(std + 1e-8)} per-slot advantage statistics */
    MG_PPO_TRAIN_HEAD = 16   /* rows x 64 bf16: head of the last minibatch forward */
};

/* Gym(int p) of gym.h:36-72 (+ optional seed, first env id for sharded
 * multi-GPU gyms, device; -1 = current). done starts at 1, rng per
 * mg_env_init. */
int mg_gym_create(const char* kernel_name, int parallels, uint32_t seed, uint32_t first_env_id, int device,
                  mg_gym_t* gym);
int mg_gym_destroy(mg_gym_t gym);
/* parallels, state/action/obs bytes, obs_dim, act_dim, continuous, device. */
int mg_gym_info(mg_gym_t gym, uint32_t out[8]);
/* gym.run (gym.h:110-121): uploads parallels actions from host memory
 * (skipped if actions_host is NULL), steps every env once, copies the first
 * reward_count rewards back and waits. */
int mg_gym_run(mg_gym_t gym, const void* actions_host, float* reward_host, int reward_count);
/* `steps` device-side steps with the random policy of mg_env_ops.run_random
 * (obs / reward of the last step are left in the live buffers). Asynchronous. */
int mg_gym_run_random(mg_gym_t gym, int steps, int mode);
int mg_gym_buffer(mg_gym_t gym, int which, void** dev_ptr, size_t* bytes);
/* Synchronous copies of a whole gym buffer (at most `bytes`). */
int mg_gym_download(mg_gym_t gym, int which, void* host, size_t bytes);
int mg_gym_upload(mg_gym_t gym, int which, const void* host, size_t bytes);
int mg_gym_stream(mg_gym_t gym, mg_stream_t* stream);
int mg_gym_synchronize(mg_gym_t gym);

/* PPOModel(gym, e, s, layers, lr, T, seed) of model/ppo.h:274-446: seeded
 * init, parameter layout, slots. Fails (instead of exit(1)) on bad sizes. */
int mg_ppo_create(mg_gym_t gym, int embed, int scale, int layers, float lr, int horizon, uint32_t seed,
                  mg_ppo_t* model);
int mg_ppo_destroy(mg_ppo_t model);
/* rows, obs_dim, act_dim, embed, hidden, layers, horizon, opt_count,
 * opt_float_count, parameter count, continuous, action bytes. */
int mg_ppo_info(mg_ppo_t model, uint64_t out[12]);
/* Parameter i in creation order (inW, inB, {ln.g, ln.b, up, down} x L,
 * lnF.g, lnF.b, head, [logStd]): element offset, count, gradient kind. */
int mg_ppo_param_info(mg_ppo_t model, int i, uint64_t* offset, uint32_t* count, int* grad_is_float);
/* collect() (model/ppo.h:716-751); blocks until done. */
int mg_ppo_collect(mg_ppo_t model);
/* train(epochs) (model/ppo.h:918-923); blocks until done. */
int mg_ppo_train(mg_ppo_t model, int epochs);
/* trainSlot(t) (model/ppo.h:906-916); blocks until done. */
int mg_ppo_train_slot(mg_ppo_t model, int t);
/* Gradient all-reduce over NVLink peer memory instead of NCCL (no counterpart
 * in the reference). Every rank calls mg_ppo_p2p_handle (allocates its
 * exchange region, returns its 64-byte CUDA IPC handle), the host exchanges
 * the handles, every rank calls mg_ppo_p2p_open with all of them in rank
 * order, and the host synchronises the ranks once before the first train().
 * train() then reduces each minibatch's gradient with one kernel that reads
 * the other ranks' regions over NVLink (every rank sums in rank order: the
 * ranks' weights stay bit-identical). world <= 16, one GPU per rank. */
int mg_ppo_p2p_handle(mg_ppo_t model, void* out64);
int mg_ppo_p2p_open(mg_ppo_t model, const void* handles, int rank, int world);
/* Checkpoint of the training state (no counterpart in the reference, which
 * has none): weights, fp32 master, Adam moments, step counter, learning rate,
 * hyperparameters, minibatch rows, the host shuffle generator and the
 * rollout position (last observation, env states, done flags, RNG words of
 * the model's gym). mg_ppo_load restores it into a model of the same shapes
 * and environment; training then continues exactly as from the saved model.
 * Blocks until done. */
int mg_ppo_save(mg_ppo_t model, const char* path);
int mg_ppo_load(mg_ppo_t model, const char* path);
/* Rows per training minibatch (no counterpart in the reference, whose
 * minibatch is always one time slot, model/ppo.h:906-923). 0 (the default)
 * keeps the reference's slot minibatches; B > 0 makes every epoch of
 * train() visit the horizon x parallels rollout rows once, in a keyed random
 * order (a 4-round Feistel permutation, include/metalgym/rowmap.h), B rows
 * per minibatch, each minibatch normalising advantages over its own rows.
 * B must divide horizon x parallels. */
int mg_ppo_set_minibatch_rows(mg_ppo_t model, int rows);
int mg_ppo_minibatch_rows(mg_ppo_t model, int* out);
/* collect() as one persistent kernel (no counterpart in the reference, whose
 * collect() encodes about 460 dispatches, model/ppo.h:716-751): on = 1 runs
 * every step of the rollout (policy forward on the tensor cores, sampling,
 * reset-if-done and env step, with each env's state and RNG word kept in
 * registers), the bootstrap forward and GAE in one launch of 4-CTA clusters,
 * 128 envs per cluster. MG_REGISTER_ENV instantiates the kernel for every
 * environment whose State has at most 64 bytes and whose observation at most
 * 32 floats (mg_env_ops.collect_fused; CartPole and CartPoleContinuous among
 * the built-ins, not VoxelNav); the policy must be embed 128, hidden 512, 1
 * to 4 blocks. Other configurations return MG_ERR_UNSUPPORTED. on = 0 runs
 * the captured per-step graph. on = -1 (the default) chooses: the kernel
 * where it applies and parallels <= 4096 (one wave of clusters), else the
 * graph. Up to 4096 parallels the two produce identical rollouts.
 * mg_ppo_collect_fused reports the path the next collect() takes. */
int mg_ppo_set_collect_fused(mg_ppo_t model, int on);
int mg_ppo_collect_fused(mg_ppo_t model, int* out);
/* One training minibatch's per-tile work as one kernel (no counterpart in the
 * reference, which encodes every layer of a minibatch as its own dispatches,
 * model/ppo.h:753-865): on = 1 runs the block forwards, the
 * head with the PPO loss and the block backwards of a minibatch in one launch
 * of 4-CTA clusters, one per 128-row tile, where each of them would run as a
 * cluster kernel of its own (embed 128, hidden 512, 1 or 2 blocks, categorical
 * head, minibatches of at most 4096 rows, no overlapped all-reduce); the
 * results are bit-identical to the separate kernels (on = 0, the default:
 * chained by programmatic dependent launch in the train graph they measured
 * 2 % faster at 4096 rows). The gradient sums and Adam stay kernels of their
 * own. mg_ppo_fused_minibatch reads the setting. */
int mg_ppo_set_fused_minibatch(mg_ppo_t model, int on);
int mg_ppo_fused_minibatch(mg_ppo_t model, int* out);
/* One row-mode minibatch over rollout rows perm(base .. base + B - 1) of the
 * permutation keyed by key[4], with an Adam step; blocks (the manual path
 * of row mode, as mg_ppo_train_slot is of slot mode). */
int mg_ppo_train_rows(mg_ppo_t model, const uint32_t key[4], uint32_t base);
/* Host evaluation of that permutation: out[q] = flat slot-major rollout row
 * (t * parallels + env) read by minibatch row q, q < rows. */
int mg_minibatch_rows(const uint32_t key[4], uint32_t base, uint32_t rows, uint64_t total, uint64_t* out);
/* forward() on the gym's live obs (model/ppo.h:628-634); blocks. */
int mg_ppo_forward(mg_ppo_t model);
/* actGreedy() (model/ppo.h:688-702) on the device: from the head rows of the
 * last forward (head_source MG_PPO_HEAD: forward() or collect();
 * MG_PPO_TRAIN_HEAD: the last training minibatch, which must hold a row per
 * environment), per environment the index of the largest logit (the first of
 * equal ones) or, for a Gaussian head, the means, written to the gym's
 * action buffer and, when actions_host is not NULL, to actions_host
 * (parallels Actions); blocks. */
int mg_ppo_act_greedy(mg_ppo_t model, int head_source, void* actions_host);
/* lastStats() (model/ppo.h:925-943): policy, value, entropy, approxKl,
 * clipFrac, gradNorm (pre-clip). */
int mg_ppo_last_stats(mg_ppo_t model, float out6[6]);
/* The public hyperparameter fields of model/ppo.h:186-191 (read on every
 * collect / train call): clip, valueCoef, entropyCoef, maxGradNorm, gamma, lambda. */
int mg_ppo_set_hyper(mg_ppo_t model, float clip, float value_coef, float entropy_coef, float max_grad_norm,
                     float gamma, float lambda);
int mg_ppo_get_hyper(mg_ppo_t model, float out6[6]);
/* setLogStd / logStdValue (model/ppo.h:454-469), continuous envs only. */
int mg_ppo_set_log_std(mg_ppo_t model, float v);
int mg_ppo_log_std(mg_ppo_t model, int k, float* out);
/* Adam step counter (model/ppo.h:265, 874). */
int mg_ppo_step_counter(mg_ppo_t model, float* out);
int mg_ppo_set_step_counter(mg_ppo_t model, float step);
/* Device pointer / synchronous copies of a model buffer (mg_ppo_buffer);
 * slot selects one slot of a slotted buffer, -1 the whole buffer. */
int mg_ppo_buffer(mg_ppo_t model, int which, int slot, void** dev_ptr, size_t* bytes);
int mg_ppo_download(mg_ppo_t model, int which, int slot, void* host, size_t bytes);
int mg_ppo_upload(mg_ppo_t model, int which, int slot, const void* host, size_t bytes);
/* Kernel launches in one replay of the captured collect() and train() graphs
 * (0 before the first call); no counterpart in the reference. */
int mg_ppo_graph_kernels(mg_ppo_t model, uint64_t out2[2]);
/* Device time in ms of the last collect() and the last train() call (CUDA
 * events around their graph launches; 0 before the first). Each public
 * operation is also an NVTX range ("mg.collect", "mg.train", "mg.trainSlot",
 * "mg.forward") for profilers. No counterpart in the reference. */
int mg_ppo_phase_ms(mg_ppo_t model, float out2[2]);
/* Data parallelism (no counterpart in the reference): with world > 1 each
 * minibatch's gradient is summed over the ranks of `comm` (an ncclComm_t)
 * and divided by world before the norm clip and Adam. */
int mg_ppo_set_comm(mg_ppo_t model, void* comm, int rank, int world);
/* With an NCCL communicator (world > 1): on = 1 all-reduces the gradients of
 * everything but the last backward layer (block 0 and the input layer) on a
 * side stream while that layer's backward runs, then the rest, instead of one
 * all-reduce of the whole gradient after the backward pass. The same sums,
 * in two grouped pairs of calls over the gradient arena's ranges. 0 (the
 * default): one all-reduce. No counterpart in the reference (one GPU). */
int mg_ppo_set_allreduce_overlap(mg_ppo_t model, int on);
/* Failure detection for data-parallel train() with an NCCL communicator (no
 * counterpart in the reference): with seconds > 0, train() / trainSlot()
 * wait for their work by polling the stream and the communicator's
 * asynchronous error instead of blocking. When a peer reports an error, or
 * the work has not finished after `seconds`, the communicator is aborted
 * (ncclCommAbort: the all-reduce kernels in flight return) and the call
 * returns MG_ERR_COMM; every later call with that communicator returns
 * MG_ERR_COMM too. 0 (the default): block until done. If the stream has
 * still not drained 30 s after the abort, mg_ppo_destroy and mg_gym_destroy
 * leave the device buffers allocated (freeing them could block without limit
 * or free memory a running kernel uses) and return MG_ERR_COMM. */
int mg_ppo_set_comm_timeout(mg_ppo_t model, float seconds);

/* ---------------------------------------------------------------- NCCL / host memory */

/* NCCL communicator helpers (libnccl.so.2 is loaded on first use).
 * mg_comm_init connects every channel when the communicator is created
 * (it sets NCCL_RUNTIME_CONNECT=0 unless the caller set it): with NCCL's lazy
 * connection the first collective would handshake with every peer on the
 * host, and a peer that never joins would block the caller there, where the
 * train() watchdog (mg_ppo_set_comm_timeout) cannot see it. */
int mg_comm_unique_id(void* out128);
int mg_comm_init(int world, int rank, const void* id128, int device, void** comm);
/* Destroy and abort first release the train graphs of every model bound to
 * the communicator (mg_ppo_set_comm): NCCL waits until each graph that
 * captured its collectives is gone, so a graph kept alive would block the
 * call for good. Those models recapture at their next train(). */
int mg_comm_destroy(void* comm);
/* Aborts the communicator and its operations in flight (ncclCommAbort), for
 * a rank that leaves a data-parallel job. The handle is freed: later
 * mg_comm_destroy calls on it do nothing. */
int mg_comm_abort(void* comm);
int mg_allreduce_sum_f32(float* data, size_t count, void* comm, mg_stream_t stream);
/* Pinned host memory for the host mirrors of the drop-in API (zeroed). */
int mg_host_alloc(size_t bytes, void** out);
int mg_host_free(void* p);

/* ---------------------------------------------------------------- no-allocation variant */

/* Scratch held by mg_weight_grad_noalloc: 16 MiB of device memory per GPU. */
#define MG_WEIGHT_GRAD_NOALLOC_SCRATCH_BYTES (16u << 20)

/* No counterpart in the reference. The weight gradient of the PPO backward
 * pass, dw_out[m][n] = sum_r x[r][m] * dz[r][n] (x bf16 [rows][in_features],
 * dz bf16 [rows][out_features], dw_out fp32 [in_features][out_features],
 * rounded to bf16 values if round_bf16), for callers that cannot allocate
 * device memory: code inside a framework that owns all device memory (a
 * custom call or plugin that must not allocate while enqueuing) or a program
 * that allocates nothing after start-up. It computes what mg_gemm_bf16 with
 * MG_EPI_F32 and `splits` followed by mg_reduce_partials computes, but keeps
 * the split-K partials in a fixed scratch array inside the library
 * (MG_WEIGHT_GRAD_NOALLOC_SCRATCH_BYTES on every GPU that loads it, held
 * until the process exits) and calls no allocator. Sizes whose scratch need
 * (effective splits x in_features x out_features x 4 bytes, plus 4 bytes
 * per 1024 outputs) exceeds that are rejected with MG_ERR_ARGUMENT. The
 * first call on a device looks up the scratch address on that device; make
 * that first call before any stream capture. All calls share the scratch and
 * it keeps the last call's contents (every call overwrites what it reads), so
 * calls that overlap on the GPU race. Asynchronous on `stream`. */
int mg_weight_grad_noalloc(const void* x, const void* dz, int rows, int in_features, int out_features, int splits,
                           int round_bf16, float* dw_out, mg_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* METALGYM_B200_H */
