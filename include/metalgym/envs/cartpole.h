// CartPole with a discrete push left / push right action.
//
// The environment contract of the reference (README.md:19-53) with
// __host__ __device__ statics: State / Action / Obs, OBS_DIM, ACT_DIM,
// reset(State&, rng) and step(State&, Action, Obs&, reward, done), plus the
// host-side KERNEL name (examples/CartPole/main.cpp:5-18).
//
// Dynamics follow examples/CartPole/cartpole.metal:36-75 operation for
// operation, because trajectories are compared bit for bit with that file
// compiled as host C++: Euler cart-pole (gravity 9.8, cart 1.0, pole 0.1,
// half length 0.5, force 10, tau 0.02), semi-implicit update order, done on
// |x| > 2.4, |theta| > 12 degrees or 500 steps, reward 1 on every step.
// Compile translation units that instantiate it with nvcc --fmad=false (and
// g++ -ffp-contract=off on the host) so no expression is fused into an FMA.
#pragma once

#include "../config.h"
#include "../mathf.h"
#include "../rng.h"

struct CartPole {
    struct State {
        float x;
        float xDot;
        float theta;
        float thetaDot;
        uint32_t steps;
    };
    using Action = int;  // 0 = push left, 1 = push right
    struct Obs {
        float x;
        float xDot;
        float theta;
        float thetaDot;
    };

    static constexpr uint32_t OBS_DIM = 4;
    static constexpr uint32_t ACT_DIM = 2;
    static constexpr const char* KERNEL = "rollout_cartpole";

    static constexpr float GRAVITY = 9.8f;
    static constexpr float MASS_CART = 1.0f;
    static constexpr float MASS_POLE = 0.1f;
    static constexpr float TOTAL_MASS = MASS_CART + MASS_POLE;
    static constexpr float LENGTH = 0.5f;  // half the pole length
    static constexpr float POLE_MASS_LENGTH = MASS_POLE * LENGTH;
    static constexpr float FORCE_MAG = 10.0f;
    static constexpr float TAU = 0.02f;
    static constexpr float PI_F = 3.14159265358979323846f;
    static constexpr float THETA_THRESHOLD = 12.0f * 2.0f * PI_F / 360.0f;
    static constexpr float X_THRESHOLD = 2.4f;
    static constexpr uint32_t MAX_STEPS = 500;

    MG_HD static void reset(State& s, uint32_t& rng) {
        s.x = rngUniform(rng, -0.05f, 0.05f);
        s.xDot = rngUniform(rng, -0.05f, 0.05f);
        s.theta = rngUniform(rng, -0.05f, 0.05f);
        s.thetaDot = rngUniform(rng, -0.05f, 0.05f);
        s.steps = 0;
    }

    // Shared by both CartPole variants: one Euler step under `force`.
    MG_HD static void integrate(State& s, float force, Obs& obs, float& reward, uint8_t& done) {
        float sinTheta, cosTheta;
        mg_sincosf(s.theta, &sinTheta, &cosTheta);
        const float temp = (force + POLE_MASS_LENGTH * s.thetaDot * s.thetaDot * sinTheta) / TOTAL_MASS;
        const float thetaAcc = (GRAVITY * sinTheta - cosTheta * temp) /
                               (LENGTH * (4.0f / 3.0f - MASS_POLE * cosTheta * cosTheta / TOTAL_MASS));
        const float xAcc = temp - POLE_MASS_LENGTH * thetaAcc * cosTheta / TOTAL_MASS;

        s.x += TAU * s.xDot;
        s.xDot += TAU * xAcc;
        s.theta += TAU * s.thetaDot;
        s.thetaDot += TAU * thetaAcc;
        s.steps += 1;

        const bool terminated = fabsf(s.x) > X_THRESHOLD || fabsf(s.theta) > THETA_THRESHOLD;
        const bool truncated = s.steps >= MAX_STEPS;

        obs.x = s.x;
        obs.xDot = s.xDot;
        obs.theta = s.theta;
        obs.thetaDot = s.thetaDot;
        reward = 1.0f;
        done = (terminated || truncated) ? 1 : 0;
    }

    MG_HD static void step(State& s, Action action, Obs& obs, float& reward, uint8_t& done) {
        integrate(s, action == 1 ? FORCE_MAG : -FORCE_MAG, obs, reward, done);
    }
};
