// VoxelNav: goal-conditioned navigation over a generated 32 x 32 heightmap
// with one chasm. Six actions (forward, back, turn left, turn right, jump
// forward, place cobble); the observation is a depth camera of 8 x 4 rays
// marched through the heightmap plus the goal in the agent's frame.
//
// The generator, camera, moves and shaped reward follow
// examples/VoxelNav/voxelnav.metal:49-162 operation for operation, because
// trajectories are compared bit for bit with that file compiled as host C++:
//   reset   5 x 5 knots U[3,9) blended bilinearly (x + (y - x) * t), rounded
//           to whole cells; chasm 2-5 wide starting at x in [12, 18), far side
//           lifted by 0-2 (max 15); spawn left of it, goal right of it, yaw
//           U[-pi, pi); 33 draws from the env's word per reset;
//   observe rays at yaw + (c/7 - 1/2) * 90 deg and pitches -45/-20/0/15 deg,
//           sampled every 0.5 up to 24 cells; goal forward/right/up/distance;
//   step    moves up at most one block, falling into the void ends the episode
//           with -5, reaching within 1.5 cells gives +10, -0.05 per step plus
//           0.2 * clamp(progress, -1.5, 1.5), 250-step limit.
// Compile with nvcc --fmad=false / g++ -ffp-contract=off (see cartpole.h).
#pragma once

#include "../config.h"
#include "../mathf.h"
#include "../rng.h"

struct VoxelNav {
    static constexpr uint32_t W = 32;
    static constexpr uint32_t RAY_COLS = 8;
    static constexpr uint32_t RAY_ROWS = 4;
    static constexpr uint32_t N_RAYS = RAY_COLS * RAY_ROWS;
    static constexpr uint32_t OBS_DIM = N_RAYS + 8;
    static constexpr uint32_t ACT_DIM = 6;
    static constexpr uint32_t MAX_STEPS = 250;
    static constexpr float PI_F = 3.14159265358979323846f;
    static constexpr float FOV = 90.0f * PI_F / 180.0f;
    static constexpr float MAX_DEPTH = 24.0f;
    static constexpr float EYE = 1.6f;
    static constexpr float GOAL_RADIUS = 1.5f;
    static constexpr uint32_t START_COBBLE = 16;
    static constexpr const char* KERNEL = "rollout_voxelnav";

    struct State {
        float x, z, yaw;
        float gx, gz;
        float prevDist;
        uint32_t steps;
        uint32_t cobble;
        uint8_t height[W * W];  // terrain height per cell, 0 = void
    };
    using Action = int;
    struct Obs {
        float ray[N_RAYS];
        float goalForward, goalRight, goalUp, goalDist;
        float sinYaw, cosYaw, cobble, height;
    };

    MG_HD static uint32_t cell(int cx, int cz) { return (uint32_t)cx * W + (uint32_t)cz; }
    MG_HD static bool inside(int cx, int cz) { return cx >= 0 && cz >= 0 && cx < (int)W && cz < (int)W; }
    MG_HD static float lerp(float a, float b, float t) { return a + (b - a) * t; }
    MG_HD static float heightAt(const State& s, float x, float z) {
        const int cx = (int)floorf(x), cz = (int)floorf(z);
        return inside(cx, cz) ? (float)s.height[cell(cx, cz)] : 0.0f;
    }
    MG_HD static float dist(const State& s) {
        const float dx = s.gx - s.x, dz = s.gz - s.z;
        return sqrtf(dx * dx + dz * dz);
    }

    MG_HD static void reset(State& s, uint32_t& rng) {
        float knot[25];
        for (uint32_t i = 0; i < 25; i++) knot[i] = rngUniform(rng, 3.0f, 9.0f);
        for (uint32_t cx = 0; cx < W; cx++) {
            const float fx = (float)cx / (float)(W - 1) * 4.0f;
            const uint32_t ix = (uint32_t)fx < 3u ? (uint32_t)fx : 3u;
            const float tx = fx - (float)ix;
            for (uint32_t cz = 0; cz < W; cz++) {
                const float fz = (float)cz / (float)(W - 1) * 4.0f;
                const uint32_t iz = (uint32_t)fz < 3u ? (uint32_t)fz : 3u;
                const float tz = fz - (float)iz;
                const float near = lerp(knot[ix * 5 + iz], knot[(ix + 1) * 5 + iz], tx);
                const float far = lerp(knot[ix * 5 + iz + 1], knot[(ix + 1) * 5 + iz + 1], tx);
                s.height[cell((int)cx, (int)cz)] = (uint8_t)roundf(lerp(near, far, tz));
            }
        }
        const uint32_t width = 2 + rngInt(rng, 4);
        const uint32_t left = 12 + rngInt(rng, 6);
        const uint32_t lift = rngInt(rng, 3);
        for (uint32_t cx = 0; cx < W; cx++) {
            for (uint32_t cz = 0; cz < W; cz++) {
                const uint32_t k = cell((int)cx, (int)cz);
                if (cx >= left && cx < left + width) {
                    s.height[k] = 0;
                } else if (cx >= left + width) {
                    const uint32_t h = (uint32_t)s.height[k] + lift;
                    s.height[k] = (uint8_t)(h < 15u ? h : 15u);
                }
            }
        }
        s.x = 2.5f + rngUniform(rng) * (float)(left - 4);
        s.z = 2.5f + rngUniform(rng) * (float)(W - 5);
        s.gx = (float)(left + width) + 2.5f + rngUniform(rng) * (float)(W - 5 - (left + width));
        s.gz = 2.5f + rngUniform(rng) * (float)(W - 5);
        s.yaw = rngUniform(rng, -PI_F, PI_F);
        s.prevDist = dist(s);
        s.steps = 0;
        s.cobble = START_COBBLE;
    }

    // Depth of one camera ray: first sample below the terrain or off the map.
    MG_HD static float march(const State& s, float ey, float dx, float dy, float dz) {
        for (float t = 0.5f; t < MAX_DEPTH; t += 0.5f) {
            const float px = s.x + t * dx, py = ey + t * dy, pz = s.z + t * dz;
            const int cx = (int)floorf(px), cz = (int)floorf(pz);
            if (!inside(cx, cz)) return t;
            if (py <= (float)s.height[cell(cx, cz)]) return t;
        }
        return MAX_DEPTH;
    }

    MG_HD static void observe(const State& s, Obs& o) {
        const float pitchDeg[RAY_ROWS] = {-45.0f, -20.0f, 0.0f, 15.0f};
        const float h = heightAt(s, s.x, s.z);
        const float ey = h + EYE;
        for (uint32_t c = 0; c < RAY_COLS; c++) {
            const float a = s.yaw + ((float)c / (float)(RAY_COLS - 1) - 0.5f) * FOV;
            float sinA, cosA;
            mg_sincosf(a, &sinA, &cosA);
            for (uint32_t r = 0; r < RAY_ROWS; r++) {
                const float p = pitchDeg[r] * PI_F / 180.0f;
                float sinP, cosP;
                mg_sincosf(p, &sinP, &cosP);
                const float depth = march(s, ey, cosP * cosA, sinP, cosP * sinA);
                o.ray[c * RAY_ROWS + r] = depth / MAX_DEPTH;
            }
        }
        const float gx = s.gx - s.x, gz = s.gz - s.z;
        float sa, ca;
        mg_sincosf(s.yaw, &sa, &ca);
        o.goalForward = (gx * ca + gz * sa) / (float)W;
        o.goalRight = (-gx * sa + gz * ca) / (float)W;
        o.goalUp = (heightAt(s, s.gx, s.gz) - h) / 8.0f;
        o.goalDist = sqrtf(gx * gx + gz * gz) / (float)W;
        o.sinYaw = sa;
        o.cosYaw = ca;
        o.cobble = (float)s.cobble / (float)START_COBBLE;
        o.height = h / 16.0f;
    }

    // Move to (nx, nz) if that cell is on the map and at most one block up.
    // Returns true if the move ended in the void.
    MG_HD static bool tryMove(State& s, float nx, float nz) {
        const int cx = (int)floorf(nx), cz = (int)floorf(nz);
        if (!inside(cx, cz)) return false;
        const float here = heightAt(s, s.x, s.z);
        const float there = (float)s.height[cell(cx, cz)];
        if (there == 0.0f) {
            s.x = nx;
            s.z = nz;
            return true;
        }
        if (there > here + 1.0f) return false;
        s.x = nx;
        s.z = nz;
        return false;
    }

    MG_HD static void step(State& s, Action action, Obs& obs, float& reward, uint8_t& done) {
        float sa, ca;
        mg_sincosf(s.yaw, &sa, &ca);
        bool fell = false;
        switch (action) {
            case 0: fell = tryMove(s, s.x + ca, s.z + sa); break;
            case 1: fell = tryMove(s, s.x - ca, s.z - sa); break;
            case 2: s.yaw -= PI_F / 6.0f; break;
            case 3: s.yaw += PI_F / 6.0f; break;
            case 4: fell = tryMove(s, s.x + 2.0f * ca, s.z + 2.0f * sa); break;
            case 5: {
                const int cx = (int)floorf(s.x + ca), cz = (int)floorf(s.z + sa);
                if (s.cobble > 0 && inside(cx, cz)) {
                    const uint32_t k = cell(cx, cz);
                    const uint32_t here = (uint32_t)heightAt(s, s.x, s.z);
                    if (s.height[k] == 0) {
                        s.height[k] = (uint8_t)here;
                        s.cobble--;
                    } else if ((uint32_t)s.height[k] <= here) {
                        s.height[k]++;
                        s.cobble--;
                    }
                }
                break;
            }
            default: break;
        }
        if (s.yaw > PI_F) s.yaw -= 2.0f * PI_F;
        if (s.yaw < -PI_F) s.yaw += 2.0f * PI_F;
        s.steps++;

        const float d = dist(s);
        reward = -0.05f + 0.2f * fminf(fmaxf(s.prevDist - d, -1.5f), 1.5f);
        s.prevDist = d;
        const bool success = d < GOAL_RADIUS;
        if (success) reward += 10.0f;
        if (fell) reward -= 5.0f;
        done = (success || fell || s.steps >= MAX_STEPS) ? 1 : 0;
        observe(s, obs);
    }
};
