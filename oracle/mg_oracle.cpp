// TEST INFRASTRUCTURE ONLY (oracle). A CPU restatement of the reference's
// PPO arithmetic; the product never links or calls it. Built by
// oracle/Makefile (target `port`) with -ffp-contract=off.
//
// Every function names the reference file:line it restates. Rounding points
// follow the reference: activations, logits, dZ and GEMM-weight gradients
// are stored as bf16 (round to nearest even); accumulation, LayerNorm
// statistics, the input/LayerNorm/log-std gradients and the Adam state are
// fp32. Transcendentals are the project's mg_expf / mg_logf / mg_sincosf,
// the same functions the CUDA kernels and the reference shim use.
//
// Parity of this restatement is pinned against oracle/_ref (the reference's
// own Metal sources compiled as host C++) for every per-thread kernel and the
// LayerNorm kernels; the GEMMs (Apple MetalPerformancePrimitives matmul2d in
// the reference, not available here) are plain loops with bf16 operands and
// fp32 accumulation, which is unpinned at the accumulation-order level.
#include "mg_oracle.h"

#include <algorithm>
#include <cmath>
#include <cstring>
#include <random>
#include <vector>

#include "metalgym/mathf.h"
#include "metalgym/rng.h"

#define ORC_API extern "C" __attribute__((visibility("default")))

static inline float bf2f(uint16_t h) {
    uint32_t u = (uint32_t)h << 16;
    float f;
    std::memcpy(&f, &u, 4);
    return f;
}
static inline uint16_t f2bf(float f) {
    uint32_t u;
    std::memcpy(&u, &f, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u);  // quiet NaN
    const uint32_t rounding = 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t)((u + rounding) >> 16);
}
static inline float rbf(float f) { return bf2f(f2bf(f)); }

ORC_API uint16_t orc_f2bf(float x) { return f2bf(x); }
ORC_API float orc_bf2f(uint16_t x) { return bf2f(x); }

static constexpr uint32_t HEAD_DIM = 64;  // model/ppo.h:116
static constexpr float LOG_SQRT_2PI = 0.9189385332046727f;  // model/gaussian.metal:20

// ---------------------------------------------------------------- kernels

// model/input.metal:11-27
ORC_API void orc_input_forward(const float* obs, const uint16_t* w, const uint16_t* bias, uint16_t* out,
                               uint32_t rows, uint32_t inDim, uint32_t outDim) {
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < (int64_t)rows; r++) {
        for (uint32_t c = 0; c < outDim; c++) {
            float acc = bf2f(bias[c]);
            for (uint32_t k = 0; k < inDim; k++) acc += obs[r * inDim + k] * bf2f(w[(size_t)k * outDim + c]);
            out[(size_t)r * outDim + c] = f2bf(acc);
        }
    }
}

// model/input.metal:38-60 (sum over all rows; the reference sums row chunks and adds them atomically)
ORC_API void orc_input_backward(const float* obs, const uint16_t* dZ, float* dW, float* dBias, uint32_t rows,
                                uint32_t inDim, uint32_t outDim) {
#pragma omp parallel for schedule(static)
    for (int64_t c = 0; c < (int64_t)outDim; c++) {
        float accB = 0.0f;
        for (uint32_t r = 0; r < rows; r++) accB += bf2f(dZ[(size_t)r * outDim + c]);
        dBias[c] += accB;
        for (uint32_t k = 0; k < inDim; k++) {
            float acc = 0.0f;
            for (uint32_t r = 0; r < rows; r++) acc += obs[(size_t)r * inDim + k] * bf2f(dZ[(size_t)r * outDim + c]);
            dW[(size_t)k * outDim + c] += acc;
        }
    }
}

// model/layernorm.metal:10-71: two-pass mean and population variance, eps 1e-5;
// saves x-hat (bf16) and sigma (fp32); out = gamma * x-hat + beta (x-hat unrounded).
ORC_API void orc_layernorm_forward(const uint16_t* x, uint16_t* xNorm, uint16_t* out, const uint16_t* gamma,
                                   const uint16_t* beta, float* stdev, uint32_t rows, uint32_t cols) {
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < (int64_t)rows; r++) {
        const uint16_t* xr = x + (size_t)r * cols;
        float sum = 0.0f;
        for (uint32_t c = 0; c < cols; c++) sum += bf2f(xr[c]);
        const float mean = sum / (float)cols;
        float var = 0.0f;
        for (uint32_t c = 0; c < cols; c++) {
            const float d = bf2f(xr[c]) - mean;
            var += d * d;
        }
        var /= (float)cols;
        const float sd = std::sqrt(var + 1e-5f);
        const float rstd = 1.0f / sd;
        stdev[r] = sd;
        for (uint32_t c = 0; c < cols; c++) {
            const float xn = (bf2f(xr[c]) - mean) * rstd;
            xNorm[(size_t)r * cols + c] = f2bf(xn);
            out[(size_t)r * cols + c] = f2bf(bf2f(gamma[c]) * xn + bf2f(beta[c]));
        }
    }
}

// model/layernorm.metal:74-127: dgamma += bf16(xhat*dz), dbeta += dz, dxhat = bf16(dz*gamma),
// dx = bf16((dxhat - mean(dxhat) - xhat * mean(bf16(dxhat*xhat))) / sigma), in place.
ORC_API void orc_layernorm_backward(uint16_t* dZ, const uint16_t* xNorm, const uint16_t* gamma, const float* stdev,
                                    float* dGamma, float* dBeta, uint32_t rows, uint32_t cols) {
    std::vector<float> dg(cols, 0.0f), db(cols, 0.0f);
    for (uint32_t r = 0; r < rows; r++) {
        for (uint32_t c = 0; c < cols; c++) {
            const size_t i = (size_t)r * cols + c;
            dg[c] += rbf(bf2f(xNorm[i]) * bf2f(dZ[i]));
            db[c] += bf2f(dZ[i]);
        }
    }
    for (uint32_t c = 0; c < cols; c++) {
        dGamma[c] += dg[c];
        dBeta[c] += db[c];
    }
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < (int64_t)rows; r++) {
        std::vector<float> dxn(cols);
        float s1 = 0.0f, s2 = 0.0f;
        for (uint32_t c = 0; c < cols; c++) {
            const size_t i = (size_t)r * cols + c;
            dxn[c] = rbf(bf2f(dZ[i]) * bf2f(gamma[c]));
            s1 += dxn[c];
            s2 += rbf(dxn[c] * bf2f(xNorm[i]));
        }
        const float m1 = s1 / (float)cols, m2 = s2 / (float)cols;
        const float rdev = 1.0f / stdev[r];
        for (uint32_t c = 0; c < cols; c++) {
            const size_t i = (size_t)r * cols + c;
            dZ[i] = f2bf(rdev * (dxn[c] - m1 - bf2f(xNorm[i]) * m2));
        }
    }
}

// The dense products of model/mlp.metal and model/linear.metal with bf16
// operands and fp32 accumulation in increasing k order.
ORC_API void orc_gemm_f32acc(const uint16_t* A, const uint16_t* B, float* C, uint32_t M, uint32_t N, uint32_t K,
                             int transA, int transB) {
    std::vector<float> a((size_t)M * K), b((size_t)K * N);
    for (uint32_t m = 0; m < M; m++)
        for (uint32_t k = 0; k < K; k++)
            a[(size_t)m * K + k] = bf2f(transA ? A[(size_t)k * M + m] : A[(size_t)m * K + k]);
    for (uint32_t k = 0; k < K; k++)
        for (uint32_t n = 0; n < N; n++)
            b[(size_t)k * N + n] = bf2f(transB ? B[(size_t)n * K + k] : B[(size_t)k * N + n]);
#pragma omp parallel for schedule(static)
    for (int64_t m = 0; m < (int64_t)M; m++) {
        float* c = C + (size_t)m * N;
        for (uint32_t n = 0; n < N; n++) c[n] = 0.0f;
        for (uint32_t k = 0; k < K; k++) {
            const float av = a[(size_t)m * K + k];
            const float* br = &b[(size_t)k * N];
            for (uint32_t n = 0; n < N; n++) c[n] += av * br[n];
        }
    }
}

// model/sample.metal:18-47: inverse-CDF draw with u scaled by the softmax denominator.
ORC_API void orc_sample_action(const uint16_t* head, uint32_t* rng, int32_t* action, float* logProb, float* value,
                               uint32_t rows, uint32_t actDim, uint32_t headDim) {
    for (uint32_t row = 0; row < rows; row++) {
        const uint16_t* h = head + (size_t)row * headDim;
        float rowMax = -INFINITY;
        for (uint32_t a = 0; a < actDim; a++) rowMax = std::fmax(rowMax, bf2f(h[a]));
        float sum = 0.0f;
        for (uint32_t a = 0; a < actDim; a++) sum += mg_expf(bf2f(h[a]) - rowMax);
        const float lse = rowMax + mg_logf(sum);
        uint32_t s = rng[row];
        const float u = (float)(rngNext(s) >> 8) * (1.0f / 16777216.0f) * sum;
        rng[row] = s;
        uint32_t chosen = actDim - 1;
        float acc = 0.0f;
        for (uint32_t a = 0; a < actDim; a++) {
            acc += mg_expf(bf2f(h[a]) - rowMax);
            if (u < acc) {
                chosen = a;
                break;
            }
        }
        action[row] = (int32_t)chosen;
        logProb[row] = bf2f(h[chosen]) - lse;
        value[row] = bf2f(h[actDim]);
    }
}

// model/gaussian.metal:32-71: Box-Muller pairs, u1 in (0, 1].
ORC_API void orc_sample_gaussian(const uint16_t* head, uint32_t* rng, float* action, float* logProb, float* value,
                                 uint32_t rows, uint32_t actDim, uint32_t headDim, const uint16_t* logStd) {
    for (uint32_t row = 0; row < rows; row++) {
        const uint16_t* h = head + (size_t)row * headDim;
        uint32_t s = rng[row];
        float lp = 0.0f, zx = 0.0f, zy = 0.0f;
        for (uint32_t k = 0; k < actDim; k++) {
            if ((k & 1u) == 0u) {
                const float u1 = 1.0f - (float)(rngNext(s) >> 8) * (1.0f / 16777216.0f);
                const float u2 = (float)(rngNext(s) >> 8) * (1.0f / 16777216.0f);
                const float r = std::sqrt(-2.0f * mg_logf(u1));
                const float theta = 2.0f * 3.14159265358979323846f * u2;
                float st, ct;
                mg_sincosf(theta, &st, &ct);
                zx = r * ct;
                zy = r * st;
            }
            const float zk = (k & 1u) ? zy : zx;
            const float ls = bf2f(logStd[k]);
            const float mu = bf2f(h[k]);
            const float a = mu + mg_expf(ls) * zk;
            const float d = (a - mu) * mg_expf(-ls);
            action[(size_t)row * actDim + k] = a;
            lp += -0.5f * d * d - ls - LOG_SQRT_2PI;
        }
        rng[row] = s;
        logProb[row] = lp;
        value[row] = bf2f(h[actDim]);
    }
}

// model/policy.metal:14-69: clipped surrogate, value and entropy terms; dZ = grad / rows.
ORC_API void orc_policy_loss(const uint16_t* head, const int32_t* action, const float* adv, const float* ret,
                             const float* oldLogProb, uint16_t* dZ, float* stats, uint32_t rows, uint32_t actDim,
                             uint32_t headDim, float clip, float valueCoef, float entropyCoef) {
    const float scale = 1.0f / (float)rows;
#pragma omp parallel for schedule(static)
    for (int64_t row = 0; row < (int64_t)rows; row++) {
        const uint16_t* h = head + (size_t)row * headDim;
        uint16_t* dz = dZ + (size_t)row * headDim;
        float rowMax = -INFINITY;
        for (uint32_t j = 0; j < actDim; j++) rowMax = std::fmax(rowMax, bf2f(h[j]));
        float sum = 0.0f;
        for (uint32_t j = 0; j < actDim; j++) sum += mg_expf(bf2f(h[j]) - rowMax);
        const float lse = rowMax + mg_logf(sum);
        float entropy = 0.0f;
        for (uint32_t j = 0; j < actDim; j++) {
            const float logp = bf2f(h[j]) - lse;
            entropy -= mg_expf(logp) * logp;
        }
        const uint32_t a = (uint32_t)action[row];
        if (a >= actDim) {  // invalid action: no gradient, NaN statistics
            for (uint32_t j = 0; j < headDim; j++) dz[j] = 0;
            for (int k = 0; k < 5; k++) stats[(size_t)row * 5 + k] = NAN;
            continue;
        }
        const float A = adv[row];
        const float logpA = bf2f(h[a]) - lse;
        const float ratio = mg_expf(logpA - oldLogProb[row]);
        const float surr1 = ratio * A;
        const float surr2 = std::fmin(std::fmax(ratio, 1.0f - clip), 1.0f + clip) * A;
        const float policyLoss = -std::fmin(surr1, surr2);
        const float gLogp = (surr1 <= surr2) ? -A * ratio : 0.0f;
        for (uint32_t j = 0; j < actDim; j++) {
            const float logp = bf2f(h[j]) - lse;
            const float prob = mg_expf(logp);
            const float g = gLogp * ((j == a ? 1.0f : 0.0f) - prob) + entropyCoef * prob * (logp + entropy);
            dz[j] = f2bf(g * scale);
        }
        const float vErr = bf2f(h[actDim]) - ret[row];
        dz[actDim] = f2bf(valueCoef * vErr * scale);
        for (uint32_t j = actDim + 1; j < headDim; j++) dz[j] = 0;
        float* st = stats + (size_t)row * 5;
        st[0] = policyLoss;
        st[1] = 0.5f * valueCoef * vErr * vErr;
        st[2] = entropy;
        st[3] = oldLogProb[row] - logpA;
        st[4] = (std::fabs(ratio - 1.0f) > clip) ? 1.0f : 0.0f;
    }
}

// model/gaussian.metal:76-135: Gaussian PPO loss; dlogStd is a batch sum (added to dLogStd).
ORC_API void orc_gaussian_loss(const uint16_t* head, const float* action, const float* adv, const float* ret,
                               const float* oldLogProb, uint16_t* dZ, float* stats, uint32_t rows, uint32_t actDim,
                               uint32_t headDim, float clip, float valueCoef, float entropyCoef,
                               const uint16_t* logStd, float* dLogStd) {
    const float scale = 1.0f / (float)rows;
    std::vector<float> gls((size_t)rows * actDim);
#pragma omp parallel for schedule(static)
    for (int64_t row = 0; row < (int64_t)rows; row++) {
        const uint16_t* h = head + (size_t)row * headDim;
        const float* act = action + (size_t)row * actDim;
        uint16_t* dz = dZ + (size_t)row * headDim;
        float logp = 0.0f, entropy = 0.0f;
        for (uint32_t k = 0; k < actDim; k++) {
            const float ls = bf2f(logStd[k]);
            const float d = (act[k] - bf2f(h[k])) * mg_expf(-ls);
            logp += -0.5f * d * d - ls - LOG_SQRT_2PI;
            entropy += ls + LOG_SQRT_2PI + 0.5f;
        }
        const float A = adv[row];
        const float ratio = mg_expf(logp - oldLogProb[row]);
        const float surr1 = ratio * A;
        const float surr2 = std::fmin(std::fmax(ratio, 1.0f - clip), 1.0f + clip) * A;
        const float policyLoss = -std::fmin(surr1, surr2);
        const float gLogp = (surr1 <= surr2) ? -A * ratio : 0.0f;
        for (uint32_t k = 0; k < actDim; k++) {
            const float ls = bf2f(logStd[k]);
            const float invStd = mg_expf(-ls);
            const float d = (act[k] - bf2f(h[k])) * invStd;
            dz[k] = f2bf(gLogp * d * invStd * scale);
            gls[(size_t)row * actDim + k] = (gLogp * (d * d - 1.0f) - entropyCoef) * scale;
        }
        const float vErr = bf2f(h[actDim]) - ret[row];
        dz[actDim] = f2bf(valueCoef * vErr * scale);
        for (uint32_t j = actDim + 1; j < headDim; j++) dz[j] = 0;
        float* st = stats + (size_t)row * 5;
        st[0] = policyLoss;
        st[1] = 0.5f * valueCoef * vErr * vErr;
        st[2] = entropy;
        st[3] = oldLogProb[row] - logp;
        st[4] = (std::fabs(ratio - 1.0f) > clip) ? 1.0f : 0.0f;
    }
    for (uint32_t k = 0; k < actDim; k++) {
        float acc = 0.0f;
        for (uint32_t r = 0; r < rows; r++) acc += gls[(size_t)r * actDim + k];
        dLogStd[k] += acc;
    }
}

// model/gae.metal:14-36: reverse scan per env over slot-major buffers [t * rows + i].
ORC_API void orc_gae(const float* reward, const uint8_t* done, const float* value, const float* bootstrapValue,
                     float* advantage, float* ret, uint32_t rows, uint32_t horizon, float gamma, float lambda) {
    for (uint32_t i = 0; i < rows; i++) {
        float lastAdv = 0.0f;
        float nextValue = bootstrapValue[i];
        for (int t = (int)horizon - 1; t >= 0; t--) {
            const size_t k = (size_t)t * rows + i;
            const float nonTerminal = done[k] ? 0.0f : 1.0f;
            const float delta = reward[k] + gamma * nextValue * nonTerminal - value[k];
            lastAdv = delta + gamma * lambda * nonTerminal * lastAdv;
            advantage[k] = lastAdv;
            ret[k] = lastAdv + value[k];
            nextValue = value[k];
        }
    }
}

// model/gae.metal:42-77: (a - mean) / (population std + 1e-8) over one minibatch.
ORC_API void orc_normalize_advantage(const float* adv, float* out, uint32_t rows) {
    double sum = 0.0;
    for (uint32_t i = 0; i < rows; i++) sum += adv[i];
    const float mean = (float)(sum / rows);
    double var = 0.0;
    for (uint32_t i = 0; i < rows; i++) {
        const double d = (double)adv[i] - mean;
        var += d * d;
    }
    const float inv = 1.0f / (std::sqrt((float)(var / rows)) + 1e-8f);
    for (uint32_t i = 0; i < rows; i++) out[i] = (adv[i] - mean) * inv;
}

// model/optimizer.metal:23-34 (accumulated in double here: the checker's value)
ORC_API double orc_grad_norm_sq(const float* grad, uint32_t count) {
    double acc = 0.0;
    for (uint32_t i = 0; i < count; i++) acc += (double)grad[i] * grad[i];
    return acc;
}

// model/optimizer.metal:36-60: global-norm clip, Adam (0.9, 0.999, 1e-8), bf16 shadow.
ORC_API void orc_adam_step(float* param, const float* grad, float* m, float* v, uint16_t* weights, float normSq,
                           uint32_t count, float lr, float beta1Pow, float beta2Pow, float maxGradNorm) {
    const float beta1 = 0.9f, beta2 = 0.999f, eps = 1e-8f;
    const float norm = std::sqrt(normSq);
    const float scale = (maxGradNorm > 0.0f && norm > maxGradNorm) ? maxGradNorm / (norm + 1e-6f) : 1.0f;
    for (uint32_t i = 0; i < count; i++) {
        const float g = grad[i] * scale;
        const float mi = beta1 * m[i] + (1.0f - beta1) * g;
        const float vi = beta2 * v[i] + (1.0f - beta2) * g * g;
        m[i] = mi;
        v[i] = vi;
        const float mHat = mi / (1.0f - beta1Pow);
        const float vHat = vi / (1.0f - beta2Pow);
        const float x = param[i] - lr * mHat / (std::sqrt(vHat) + eps);
        param[i] = x;
        weights[i] = f2bf(x);
    }
}

// ------------------------------------------------------------------ model

struct ParamSpec {
    uint32_t count;
    bool gradIsFloat;
    uint32_t offset;
};

struct OrcModel {
    uint32_t rows, obsDim, actDim, E, H, L, T;
    bool continuous;
    float lr;
    float clip = 0.2f, valueCoef = 0.5f, entropyCoef = 0.01f, maxGradNorm = 0.5f, gamma = 0.99f, lambda = 0.95f;
    float stepCounter = 0.0f;
    std::vector<ParamSpec> params;  // creation order
    uint32_t optCount = 0, optFloatCount = 0;
    std::vector<uint16_t> weights;
    std::vector<float> master, mom, var, grad;
    // parameter indices
    uint32_t pInW, pInB, pLnFg, pLnFb, pHead, pLogStd;
    std::vector<uint32_t> pLnG, pLnB, pUp, pDown;

    std::mt19937 hostRng;            // slot shuffle (model/ppo.h:349, 920), seeded with the model seed
    std::vector<uint32_t> slotOrder;

    const uint16_t* W(uint32_t p) const { return weights.data() + params[p].offset; }
    float* G(uint32_t p) { return grad.data() + params[p].offset; }
};

// model/ppo.h:375-445: seeded normal init rounded to bf16, float-grad params
// first, then bf16-grad params, each padded to 128 elements.
ORC_API OrcModel* orc_model_create(uint32_t rows, uint32_t obsDim, uint32_t actDim, int continuous, uint32_t embed,
                                   uint32_t scale, uint32_t layers, float lr, uint32_t horizon, uint32_t seed) {
    OrcModel* m = new OrcModel();
    m->rows = rows;
    m->obsDim = obsDim;
    m->actDim = actDim;
    m->continuous = continuous != 0;
    m->E = embed;
    m->H = embed * scale;
    m->L = layers;
    m->T = horizon;
    m->lr = lr;
    m->hostRng.seed(seed);
    m->slotOrder.resize(horizon);
    for (uint32_t t = 0; t < horizon; t++) m->slotOrder[t] = t;
    std::vector<std::vector<uint16_t>> init;
    auto add = [&](uint32_t count, bool gf) {
        m->params.push_back(ParamSpec{count, gf, 0});
        init.emplace_back(count, (uint16_t)0);
        return (uint32_t)(m->params.size() - 1);
    };
    std::mt19937 rng(seed);
    auto normal = [&](uint32_t p, float sd) {
        std::normal_distribution<float> dist(0.0f, sd);
        for (auto& x : init[p]) x = f2bf(dist(rng));
    };
    auto constant = [&](uint32_t p, float v) { std::fill(init[p].begin(), init[p].end(), f2bf(v)); };
    const uint32_t E = m->E, H = m->H;
    m->pInW = add(obsDim * E, true);
    normal(m->pInW, 1.0f / std::sqrt((float)obsDim));
    m->pInB = add(E, true);
    constant(m->pInB, 0.0f);
    for (uint32_t n = 0; n < layers; n++) {
        m->pLnG.push_back(add(E, true));
        constant(m->pLnG.back(), 1.0f);
        m->pLnB.push_back(add(E, true));
        constant(m->pLnB.back(), 0.0f);
        m->pUp.push_back(add(E * H, false));
        normal(m->pUp.back(), std::sqrt(2.0f / (float)E));
        m->pDown.push_back(add(H * E, false));
        normal(m->pDown.back(), 1.0f / std::sqrt((float)H) / std::sqrt((float)layers));
    }
    m->pLnFg = add(E, true);
    constant(m->pLnFg, 1.0f);
    m->pLnFb = add(E, true);
    constant(m->pLnFb, 0.0f);
    m->pHead = add(E * HEAD_DIM, false);
    {
        std::normal_distribution<float> policyDist(0.0f, 0.01f);
        std::normal_distribution<float> valueDist(0.0f, 1.0f / std::sqrt((float)E));
        for (uint32_t k = 0; k < E; k++)
            for (uint32_t n = 0; n < HEAD_DIM; n++) {
                float x = 0.0f;
                if (n < actDim) x = policyDist(rng);
                else if (n == actDim) x = valueDist(rng);
                init[m->pHead][(size_t)k * HEAD_DIM + n] = f2bf(x);
            }
    }
    m->pLogStd = UINT32_MAX;
    if (m->continuous) {
        m->pLogStd = add(actDim, true);
        constant(m->pLogStd, 0.0f);
    }
    uint32_t total = 0;
    for (int pass = 0; pass < 2; pass++) {
        for (auto& s : m->params) {
            if (s.gradIsFloat != (pass == 0)) continue;
            s.offset = total;
            total += (s.count + 127) / 128 * 128;
        }
        if (pass == 0) m->optFloatCount = total;
    }
    m->optCount = total;
    m->weights.assign(total, 0);
    m->master.assign(total, 0.0f);
    m->mom.assign(total, 0.0f);
    m->var.assign(total, 0.0f);
    m->grad.assign(total, 0.0f);
    for (size_t p = 0; p < m->params.size(); p++) {
        const uint32_t off = m->params[p].offset;
        for (uint32_t i = 0; i < m->params[p].count; i++) {
            m->weights[off + i] = init[p][i];
            m->master[off + i] = bf2f(init[p][i]);
        }
    }
    return m;
}

ORC_API void orc_model_destroy(OrcModel* m) { delete m; }
ORC_API uint32_t orc_model_opt_count(const OrcModel* m) { return m->optCount; }
ORC_API uint32_t orc_model_opt_float_count(const OrcModel* m) { return m->optFloatCount; }
ORC_API uint32_t orc_model_param_count(const OrcModel* m) { return (uint32_t)m->params.size(); }
ORC_API void orc_model_param_info(const OrcModel* m, uint32_t i, uint32_t* offset, uint32_t* count, int* gradIsFloat) {
    *offset = m->params[i].offset;
    *count = m->params[i].count;
    *gradIsFloat = m->params[i].gradIsFloat ? 1 : 0;
}
ORC_API uint16_t* orc_model_weights(OrcModel* m) { return m->weights.data(); }
ORC_API float* orc_model_master(OrcModel* m) { return m->master.data(); }
ORC_API float* orc_model_momentum(OrcModel* m) { return m->mom.data(); }
ORC_API float* orc_model_variance(OrcModel* m) { return m->var.data(); }
ORC_API float* orc_model_grad(OrcModel* m) { return m->grad.data(); }
ORC_API float orc_model_step_counter(const OrcModel* m) { return m->stepCounter; }
ORC_API void orc_model_set_step_counter(OrcModel* m, float step) { m->stepCounter = step; }
ORC_API void orc_model_set_hparams(OrcModel* m, float clip, float valueCoef, float entropyCoef, float maxGradNorm,
                                   float gamma, float lambda) {
    m->clip = clip;
    m->valueCoef = valueCoef;
    m->entropyCoef = entropyCoef;
    m->maxGradNorm = maxGradNorm;
    m->gamma = gamma;
    m->lambda = lambda;
}

namespace {

// Saved activations of one forward (model/ppo.h:351-373 buffers).
struct Acts {
    std::vector<uint16_t> input;                  // R x E
    std::vector<std::vector<uint16_t>> lnIn;      // block input h_n, R x E
    std::vector<std::vector<uint16_t>> lnXn;      // x-hat, R x E
    std::vector<std::vector<float>> lnSd;         // sigma, R
    std::vector<std::vector<uint16_t>> lnOut;     // R x E
    std::vector<std::vector<uint16_t>> v;         // relu(up), R x H
    std::vector<uint16_t> fXn, fOut, head;        // final LN and head
    std::vector<float> fSd;
};

void gemm_to_bf16(const uint16_t* A, const uint16_t* B, uint16_t* out, uint32_t M, uint32_t N, uint32_t K, int tA,
                  int tB) {
    std::vector<float> c((size_t)M * N);
    orc_gemm_f32acc(A, B, c.data(), M, N, K, tA, tB);
    for (size_t i = 0; i < c.size(); i++) out[i] = f2bf(c[i]);
}

// model/ppo.h:575-626
void forward(OrcModel* m, const float* obs, uint32_t R, Acts& a) {
    const uint32_t E = m->E, H = m->H;
    a.input.resize((size_t)R * E);
    orc_input_forward(obs, m->W(m->pInW), m->W(m->pInB), a.input.data(), R, m->obsDim, E);
    a.lnIn.assign(m->L, {});
    a.lnXn.assign(m->L, {});
    a.lnSd.assign(m->L, {});
    a.lnOut.assign(m->L, {});
    a.v.assign(m->L, {});
    std::vector<uint16_t> h = a.input, mlpOut((size_t)R * E);
    for (uint32_t n = 0; n < m->L; n++) {
        a.lnIn[n] = h;
        a.lnXn[n].resize((size_t)R * E);
        a.lnOut[n].resize((size_t)R * E);
        a.lnSd[n].resize(R);
        orc_layernorm_forward(h.data(), a.lnXn[n].data(), a.lnOut[n].data(), m->W(m->pLnG[n]), m->W(m->pLnB[n]),
                              a.lnSd[n].data(), R, E);
        // model/mlp.metal:18-58: V = bf16(X Up), mask = V > 0, V *= mask
        a.v[n].resize((size_t)R * H);
        gemm_to_bf16(a.lnOut[n].data(), m->W(m->pUp[n]), a.v[n].data(), R, H, E, 0, 0);
        for (auto& x : a.v[n])
            if (!(bf2f(x) > 0.0f)) x = f2bf(bf2f(x) * 0.0f);
        // model/mlp.metal:60-86 then model/elementwise.metal:4-13
        gemm_to_bf16(a.v[n].data(), m->W(m->pDown[n]), mlpOut.data(), R, E, H, 0, 0);
        for (size_t i = 0; i < h.size(); i++) h[i] = f2bf(bf2f(h[i]) + bf2f(mlpOut[i]));
    }
    a.fXn.resize((size_t)R * E);
    a.fOut.resize((size_t)R * E);
    a.fSd.resize(R);
    orc_layernorm_forward(h.data(), a.fXn.data(), a.fOut.data(), m->W(m->pLnFg), m->W(m->pLnFb), a.fSd.data(), R, E);
    // model/linear.metal:17-37
    a.head.resize((size_t)R * HEAD_DIM);
    gemm_to_bf16(a.fOut.data(), m->W(m->pHead), a.head.data(), R, HEAD_DIM, E, 0, 0);
}

// GEMM-weight gradient: fp32 sum over rows rounded to bf16 (model/linear.metal:71-93,
// model/mlp.metal:167-208 + model/elementwise.metal:21-31), stored as fp32.
void weight_grad(const uint16_t* A, const uint16_t* B, float* g, uint32_t M, uint32_t N, uint32_t K) {
    std::vector<float> c((size_t)M * N);
    orc_gemm_f32acc(A, B, c.data(), M, N, K, 1, 0);
    for (size_t i = 0; i < c.size(); i++) g[i] = rbf(c[i]);
}

// model/ppo.h:753-865 (+ the grad norm of :888): loss, then backward into m->grad.
void gradient(OrcModel* m, const float* obs, const void* actions, const float* advantages, const float* returns,
              const float* oldLogProb, uint32_t R, float* stats, float* normSq, Acts& a) {
    const uint32_t E = m->E, H = m->H;
    std::fill(m->grad.begin(), m->grad.end(), 0.0f);
    forward(m, obs, R, a);
    std::vector<float> advN(R);
    orc_normalize_advantage(advantages, advN.data(), R);
    std::vector<uint16_t> dLogits((size_t)R * HEAD_DIM);
    if (m->continuous)
        orc_gaussian_loss(a.head.data(), static_cast<const float*>(actions), advN.data(), returns, oldLogProb,
                          dLogits.data(), stats, R, m->actDim, HEAD_DIM, m->clip, m->valueCoef, m->entropyCoef,
                          m->W(m->pLogStd), m->G(m->pLogStd));
    else
        orc_policy_loss(a.head.data(), static_cast<const int32_t*>(actions), advN.data(), returns, oldLogProb,
                        dLogits.data(), stats, R, m->actDim, HEAD_DIM, m->clip, m->valueCoef, m->entropyCoef);

    std::vector<uint16_t> dStream((size_t)R * E), dBranch((size_t)R * E), dV((size_t)R * H);
    // model/linear.metal:40-60 and :71-93
    gemm_to_bf16(dLogits.data(), m->W(m->pHead), dStream.data(), R, E, HEAD_DIM, 0, 1);
    weight_grad(a.fOut.data(), dLogits.data(), m->G(m->pHead), E, HEAD_DIM, R);
    orc_layernorm_backward(dStream.data(), a.fXn.data(), m->W(m->pLnFg), a.fSd.data(), m->G(m->pLnFg),
                           m->G(m->pLnFb), R, E);
    for (int n = (int)m->L - 1; n >= 0; n--) {
        // model/mlp.metal:88-127: dV = bf16(dZ Dp^T) * mask
        gemm_to_bf16(dStream.data(), m->W(m->pDown[n]), dV.data(), R, H, E, 0, 1);
        for (size_t i = 0; i < dV.size(); i++)
            if (!(bf2f(a.v[n][i]) > 0.0f)) dV[i] = f2bf(bf2f(dV[i]) * 0.0f);
        // model/mlp.metal:167-208
        weight_grad(a.lnOut[n].data(), dV.data(), m->G(m->pUp[n]), E, H, R);
        weight_grad(a.v[n].data(), dStream.data(), m->G(m->pDown[n]), H, E, R);
        // model/mlp.metal:131-153
        gemm_to_bf16(dV.data(), m->W(m->pUp[n]), dBranch.data(), R, E, H, 0, 1);
        orc_layernorm_backward(dBranch.data(), a.lnXn[n].data(), m->W(m->pLnG[n]), a.lnSd[n].data(),
                               m->G(m->pLnG[n]), m->G(m->pLnB[n]), R, E);
        for (size_t i = 0; i < dStream.size(); i++) dStream[i] = f2bf(bf2f(dBranch[i]) + bf2f(dStream[i]));
    }
    // model/input.metal:38-60
    orc_input_backward(obs, dStream.data(), m->G(m->pInW), m->G(m->pInB), R, m->obsDim, E);
    *normSq = (float)orc_grad_norm_sq(m->grad.data(), m->optCount);
}

}  // namespace

ORC_API void orc_model_forward(OrcModel* m, const float* obs, uint32_t rows, uint16_t* head) {
    Acts a;
    forward(m, obs, rows, a);
    std::memcpy(head, a.head.data(), a.head.size() * sizeof(uint16_t));
}

ORC_API void orc_model_gradient(OrcModel* m, const float* obs, const void* actions, const float* advantages,
                                const float* returns, const float* oldLogProb, uint32_t rows, float* stats,
                                float* normSq) {
    Acts a;
    gradient(m, obs, actions, advantages, returns, oldLogProb, rows, stats, normSq, a);
}

// model/ppo.h:873-904 after the gradient: host beta powers, then Adam.
ORC_API void orc_model_train_minibatch(OrcModel* m, const float* obs, const void* actions, const float* advantages,
                                       const float* returns, const float* oldLogProb, uint32_t rows, float* stats,
                                       float* normSq) {
    Acts a;
    gradient(m, obs, actions, advantages, returns, oldLogProb, rows, stats, normSq, a);
    m->stepCounter += 1.0f;
    const float b1p = std::pow(0.9f, m->stepCounter);
    const float b2p = std::pow(0.999f, m->stepCounter);
    orc_adam_step(m->master.data(), m->grad.data(), m->mom.data(), m->var.data(), m->weights.data(), *normSq,
                  m->optCount, m->lr, b1p, b2p, m->maxGradNorm);
}

// model/ppo.h:918-923 over caller-owned slot buffers (layouts of
// orc_model_collect): per epoch the slot order is shuffled with the model's
// mt19937 and every slot is one minibatch (orc_model_train_minibatch).
// lastStats (optional) gets the mean LossStats of the last minibatch
// (policy, value, entropy, approxKl, clipFrac, gradNorm).
ORC_API void orc_model_train(OrcModel* m, const float* obsSlots, const void* actionSlots, const float* logProbSlots,
                             const float* advSlots, const float* retSlots, uint32_t epochs, float* lastStats) {
    const uint32_t R = m->rows, O = m->obsDim;
    const size_t actBytes = m->continuous ? (size_t)m->actDim * 4 : 4;
    std::vector<float> stats((size_t)R * 5);
    float nsq = 0.0f;
    for (uint32_t e = 0; e < epochs; e++) {
        std::shuffle(m->slotOrder.begin(), m->slotOrder.end(), m->hostRng);
        for (uint32_t t : m->slotOrder)
            orc_model_train_minibatch(m, obsSlots + (size_t)t * R * O,
                                      static_cast<const char*>(actionSlots) + (size_t)t * R * actBytes,
                                      advSlots + (size_t)t * R, retSlots + (size_t)t * R,
                                      logProbSlots + (size_t)t * R, R, stats.data(), &nsq);
    }
    if (lastStats) {
        for (int k = 0; k < 5; k++) {
            double acc = 0.0;
            for (uint32_t r = 0; r < R; r++) acc += stats[(size_t)r * 5 + k];
            lastStats[k] = (float)(acc / R);
        }
        lastStats[5] = std::sqrt(nsq);
    }
}

// model/ppo.h:716-751
ORC_API void orc_model_collect(OrcModel* m, orc_env_fn env, int which, void* states, uint8_t* done, uint32_t* rng,
                               float* obsSlots, void* actionSlots, float* logProbSlots, float* valueSlots,
                               float* rewardSlots, uint8_t* doneSlots, float* advSlots, float* retSlots, int* started,
                               uint16_t* headOut, int threads) {
    const uint32_t R = m->rows, O = m->obsDim, T = m->T;
    const size_t actBytes = m->continuous ? (size_t)m->actDim * 4 : 4;
    char* acts = static_cast<char*>(actionSlots);
    if (!*started) {
        env(which, states, acts, obsSlots, rewardSlots, done, rng, R, threads);
        *started = 1;
    } else {
        std::memcpy(obsSlots, obsSlots + (size_t)T * R * O, (size_t)R * O * sizeof(float));
    }
    std::vector<uint16_t> head((size_t)R * HEAD_DIM);
    for (uint32_t t = 0; t < T; t++) {
        orc_model_forward(m, obsSlots + (size_t)t * R * O, R, head.data());
        if (m->continuous)
            orc_sample_gaussian(head.data(), rng, reinterpret_cast<float*>(acts + (size_t)t * R * actBytes),
                                logProbSlots + (size_t)t * R, valueSlots + (size_t)t * R, R, m->actDim, HEAD_DIM,
                                m->W(m->pLogStd));
        else
            orc_sample_action(head.data(), rng, reinterpret_cast<int32_t*>(acts + (size_t)t * R * actBytes),
                              logProbSlots + (size_t)t * R, valueSlots + (size_t)t * R, R, m->actDim, HEAD_DIM);
        env(which, states, acts + (size_t)t * R * actBytes, obsSlots + (size_t)(t + 1) * R * O,
            rewardSlots + (size_t)t * R, done, rng, R, threads);
        std::memcpy(doneSlots + (size_t)t * R, done, R);
    }
    orc_model_forward(m, obsSlots + (size_t)T * R * O, R, head.data());
    std::vector<float> boot(R);
    for (uint32_t i = 0; i < R; i++) boot[i] = bf2f(head[(size_t)i * HEAD_DIM + m->actDim]);
    orc_gae(rewardSlots, doneSlots, valueSlots, boot.data(), advSlots, retSlots, R, T, m->gamma, m->lambda);
    if (headOut) std::memcpy(headOut, head.data(), head.size() * sizeof(uint16_t));
}
