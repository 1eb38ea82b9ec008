// TEST INFRASTRUCTURE ONLY (oracle): a CPU restatement of the reference's
// PPO arithmetic, used by tests/, __graft_entry__.smoke() and bench.py's CPU
// baseline as the checker. The product library never links or calls it.
//
// bf16 values cross this interface as raw uint16_t bit patterns. Every
// function cites the reference kernel or host code it restates.
#pragma once

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

// ---- elementwise helpers ----
uint16_t orc_f2bf(float x);
float orc_bf2f(uint16_t x);

// ---- kernels (one call = one reference dispatch over all rows) ----
void orc_input_forward(const float* obs, const uint16_t* w, const uint16_t* bias, uint16_t* out, uint32_t rows,
                       uint32_t inDim, uint32_t outDim);
void orc_input_backward(const float* obs, const uint16_t* dZ, float* dW, float* dBias, uint32_t rows, uint32_t inDim,
                        uint32_t outDim);
void orc_layernorm_forward(const uint16_t* x, uint16_t* xNorm, uint16_t* out, const uint16_t* gamma,
                           const uint16_t* beta, float* stdev, uint32_t rows, uint32_t cols);
void orc_layernorm_backward(uint16_t* dZ, const uint16_t* xNorm, const uint16_t* gamma, const float* stdev,
                            float* dGamma, float* dBeta, uint32_t rows, uint32_t cols);
// C[M][N] = sum_k opA(A)[m][k] * opB(B)[k][n]; transA: A stored [K][M]; transB: B stored [N][K].
void orc_gemm_f32acc(const uint16_t* A, const uint16_t* B, float* C, uint32_t M, uint32_t N, uint32_t K, int transA,
                     int transB);
void orc_sample_action(const uint16_t* head, uint32_t* rng, int32_t* action, float* logProb, float* value,
                       uint32_t rows, uint32_t actDim, uint32_t headDim);
void orc_sample_gaussian(const uint16_t* head, uint32_t* rng, float* action, float* logProb, float* value,
                         uint32_t rows, uint32_t actDim, uint32_t headDim, const uint16_t* logStd);
void orc_policy_loss(const uint16_t* head, const int32_t* action, const float* adv, const float* ret,
                     const float* oldLogProb, uint16_t* dZ, float* stats, uint32_t rows, uint32_t actDim,
                     uint32_t headDim, float clip, float valueCoef, float entropyCoef);
void orc_gaussian_loss(const uint16_t* head, const float* action, const float* adv, const float* ret,
                       const float* oldLogProb, uint16_t* dZ, float* stats, uint32_t rows, uint32_t actDim,
                       uint32_t headDim, float clip, float valueCoef, float entropyCoef, const uint16_t* logStd,
                       float* dLogStd);
void orc_gae(const float* reward, const uint8_t* done, const float* value, const float* bootstrapValue,
             float* advantage, float* ret, uint32_t rows, uint32_t horizon, float gamma, float lambda);
void orc_normalize_advantage(const float* adv, float* out, uint32_t rows);
double orc_grad_norm_sq(const float* grad, uint32_t count);
void orc_adam_step(float* param, const float* grad, float* m, float* v, uint16_t* weights, float normSq,
                   uint32_t count, float lr, float beta1Pow, float beta2Pow, float maxGradNorm);

// ---- the model (model/ppo.h PPOModel restated without Metal) ----
typedef struct OrcModel OrcModel;

// Builds the parameter layout and the seeded initial weights of
// model/ppo.h:375-445. rows = parallels (forward batch), T = horizon.
OrcModel* orc_model_create(uint32_t rows, uint32_t obsDim, uint32_t actDim, int continuous, uint32_t embed,
                           uint32_t scale, uint32_t layers, float lr, uint32_t horizon, uint32_t seed);
void orc_model_destroy(OrcModel* m);
// Parameter layout: total elements, float-grad prefix, and per-parameter offsets
// in creation order (inW, inB, {ln.g, ln.b, up, down} x L, lnF.g, lnF.b, head, [logStd]).
uint32_t orc_model_opt_count(const OrcModel* m);
uint32_t orc_model_opt_float_count(const OrcModel* m);
uint32_t orc_model_param_count(const OrcModel* m);
void orc_model_param_info(const OrcModel* m, uint32_t i, uint32_t* offset, uint32_t* count, int* gradIsFloat);
// Raw state arrays (length opt_count): bf16 weights, fp32 master, Adam m and v, fp32 grads.
uint16_t* orc_model_weights(OrcModel* m);
float* orc_model_master(OrcModel* m);
float* orc_model_momentum(OrcModel* m);
float* orc_model_variance(OrcModel* m);
float* orc_model_grad(OrcModel* m);
float orc_model_step_counter(const OrcModel* m);
void orc_model_set_step_counter(OrcModel* m, float step);
void orc_model_set_hparams(OrcModel* m, float clip, float valueCoef, float entropyCoef, float maxGradNorm,
                           float gamma, float lambda);

// Forward on `rows` observation rows (model/ppo.h:575-626); head is rows x 64 bf16.
void orc_model_forward(OrcModel* m, const float* obs, uint32_t rows, uint16_t* head);
// One minibatch (model/ppo.h:906-916 with the minibatch given explicitly):
// forward, zero grads, normalise the advantages, loss, backward, grad norm,
// Adam. Writes per-row stats (rows x 5) and the pre-clip squared grad norm.
void orc_model_train_minibatch(OrcModel* m, const float* obs, const void* actions, const float* advantages,
                               const float* returns, const float* oldLogProb, uint32_t rows, float* stats,
                               float* normSq);
// Same, but stops after the gradient (no Adam step, step counter unchanged).
void orc_model_gradient(OrcModel* m, const float* obs, const void* actions, const float* advantages,
                        const float* returns, const float* oldLogProb, uint32_t rows, float* stats, float* normSq);

// train(epochs) (model/ppo.h:918-923) over caller-owned slot buffers: per epoch
// the slot order is shuffled with the model's mt19937 (seeded with the model
// seed) and each slot is one minibatch. lastStats (optional, 6 floats): mean
// LossStats of the last minibatch.
void orc_model_train(OrcModel* m, const float* obsSlots, const void* actionSlots, const float* logProbSlots,
                     const float* advSlots, const float* retSlots, uint32_t epochs, float* lastStats);

// Environment step callback with the signature of oracle/_ref's ref_rollout
// (or any host build of an Environment): steps n envs once.
typedef void (*orc_env_fn)(int which, void* states, const void* actions, void* obs, float* reward, uint8_t* done,
                           uint32_t* rng, uint32_t n, int threads);

// collect() of model/ppo.h:716-751 over `rows` envs with caller-owned env
// buffers (states, done, rng) and slot buffers laid out as in the reference:
// obsSlots (T+1) x rows x obsDim, actions T x rows, logp/value/reward/adv/ret
// T x rows, done T x rows. *started carries rolloutStarted between calls.
void orc_model_collect(OrcModel* m, orc_env_fn env, int which, void* states, uint8_t* done, uint32_t* rng,
                       float* obsSlots, void* actionSlots, float* logProbSlots, float* valueSlots,
                       float* rewardSlots, uint8_t* doneSlots, float* advSlots, float* retSlots, int* started,
                       uint16_t* headOut, int threads);

#ifdef __cplusplus
}
#endif
