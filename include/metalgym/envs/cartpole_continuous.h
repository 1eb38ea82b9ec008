// CartPole with a continuous force: Action is one float, which step() clamps
// to [-1, 1] and scales by the force magnitude
// (examples/CartPoleContinuous/cartpole_continuous.metal:55-78). Because the
// Action is a struct of ACT_DIM floats, PPOModel selects the Gaussian head.
// The reset and the Euler step are those of CartPole.
#pragma once

#include "cartpole.h"

struct CartPoleContinuous {
    using State = CartPole::State;
    struct Action {
        float force;  // Gaussian sample, unbounded; clamped in step()
    };
    using Obs = CartPole::Obs;

    static constexpr uint32_t OBS_DIM = 4;
    static constexpr uint32_t ACT_DIM = 1;
    static constexpr const char* KERNEL = "rollout_cartpole_continuous";

    MG_HD static void reset(State& s, uint32_t& rng) { CartPole::reset(s, rng); }

    MG_HD static void step(State& s, Action action, Obs& obs, float& reward, uint8_t& done) {
        const float f = fminf(fmaxf(action.force, -1.0f), 1.0f);
        CartPole::integrate(s, f * CartPole::FORCE_MAG, obs, reward, done);
    }
};

// The BASELINE text's variant of CartPoleContinuous (its config 4: the action
// tanh-squashed to +-10 force inside step()); the reference code clamps, and
// CartPoleContinuous follows the code. tanh is the project's own (mathf.h),
// so host and device give the same float. With action a it steps exactly as
// CartPoleContinuous stepped with action tanh(a) (|tanh a| < 1: the clamp
// changes nothing).
struct CartPoleContinuousTanh {
    using State = CartPole::State;
    using Action = CartPoleContinuous::Action;
    using Obs = CartPole::Obs;

    static constexpr uint32_t OBS_DIM = 4;
    static constexpr uint32_t ACT_DIM = 1;
    static constexpr const char* KERNEL = "rollout_cartpole_continuous_tanh";

    MG_HD static void reset(State& s, uint32_t& rng) { CartPole::reset(s, rng); }

    MG_HD static void step(State& s, Action action, Obs& obs, float& reward, uint8_t& done) {
        CartPole::integrate(s, mg_tanhf(action.force) * CartPole::FORCE_MAG, obs, reward, done);
    }
};
