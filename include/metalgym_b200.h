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

#define MG_VERSION 1

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

/* ---------------------------------------------------------------- policy kernels */

/* out[r][c] = bf16(b[c] + sum_k obs[r][k] * W[k][c]); W bf16 [in_dim][out_dim].
 * Replaces inputForward (model/input.metal:11-27). */
int mg_input_forward(const float* obs, const void* w, const void* b, void* out, int rows, int in_dim, int out_dim,
                     mg_stream_t stream);
/* Per-128-row partial sums of dW = obs^T dZ and db = sum_r dZ: partial holds
 * mg_input_backward_num_partials(rows) blocks of (in_dim + 1) x out_dim fp32
 * (rows 0..in_dim-1: dW, row in_dim: db). Replaces inputBackward
 * (model/input.metal:38-60), whose chunk sums go to fp32 atomics. */
int mg_input_backward_partials(const float* obs, const void* dZ, float* partial, int rows, int in_dim, int out_dim,
                               mg_stream_t stream);
int mg_input_backward_num_partials(int rows);
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

#ifdef __cplusplus
}
#endif

#endif /* METALGYM_B200_H */
