// Per-environment random numbers: one xorshift32 word per env.
//
// Same names, arguments and results as the helpers environments call in the
// reference (rollout.h:9-29): rngNext advances the word with shifts
// (13, 17, 5); rngUniform returns the top 24 bits scaled by 2^-24 (a float in
// [0, 1)); the two-argument form maps that to [lo, hi) as lo + (hi - lo) * u
// with two roundings (no FMA); rngInt is the raw word modulo n.
// The policy sampler draws from the same word (model/sample.metal:11-16,
// model/gaussian.metal:24-29), so sampling and env resets share one stream.
#pragma once

#include "config.h"

MG_HD inline uint32_t rngNext(uint32_t& s) {
    s ^= s << 13;
    s ^= s >> 17;
    s ^= s << 5;
    return s;
}

MG_HD inline float rngUniform(uint32_t& s) {
    return (float)(rngNext(s) >> 8) * (1.0f / 16777216.0f);
}

MG_HD inline float rngUniform(uint32_t& s, float lo, float hi) {
    return mg_fadd(lo, mg_fmul(hi - lo, rngUniform(s)));
}

MG_HD inline uint32_t rngInt(uint32_t& s, uint32_t n) {
    return rngNext(s) % n;
}

// Seed of env `globalId` for a gym seeded with `seed` (gym.h:57-61 with the
// seed folded into the env index): (seed + id) * 2654435761 + 1 mod 2^32.
// At seed 0 this is the reference's rng[i] = i * 2654435761u + 1u exactly.
// xorshift32 stays at 0 forever, so the one index that hashes to 0 gets 1.
MG_HD inline uint32_t mgSeedWord(uint32_t seed, uint32_t globalId) {
    uint32_t w = (seed + globalId) * 2654435761u + 1u;
    return w == 0u ? 1u : w;
}
