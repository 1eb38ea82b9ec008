// Minibatch row maps of the PPO update.
//
// Slot mode (the reference, model/ppo.h:906-923): minibatch j is one whole
// time slot t, so row q of the minibatch is rollout row t * R + q.
// Row mode (minibatches smaller than the env count, e.g. 8192 of 16384 envs):
// every epoch visits the T * R rollout rows in a random order without
// replacement; minibatch j of the epoch is rows perm(j * B + q), q < B, where
// perm is a keyed bijection of [0, T * R): a 4-round Feistel network on the
// smallest even number of bits covering T * R, with cycle walking (values
// that fall outside the domain are permuted again until they land inside).
// The permutation is computed where a row is read, so no index buffer is
// stored; the same function is compiled for the host for tests and tools.
#pragma once

#include <stdint.h>

#include "config.h"

struct MgMinibatch {
    uint32_t key[4];  // Feistel round keys of the epoch (row mode)
    uint32_t base;    // first permuted position of the minibatch (row mode)
    int32_t slot;     // time slot (slot mode), -1 in row mode
};

MG_HD inline uint32_t mg_mix32(uint32_t x) {
    x ^= x >> 16;
    x *= 0x7feb352du;
    x ^= x >> 15;
    x *= 0x846ca68bu;
    x ^= x >> 16;
    return x;
}

// Bijection of [0, 2^(2*half)) for half-width `half` bits.
MG_HD inline uint64_t mg_feistel(uint64_t x, int half, const uint32_t key[4]) {
    const uint64_t mask = (1ull << half) - 1ull;
    uint64_t l = x >> half, r = x & mask;
    for (int round = 0; round < 4; round++) {
        const uint64_t f = mg_mix32((uint32_t)r ^ key[round]) & mask;
        const uint64_t nl = r;
        r = l ^ f;
        l = nl;
    }
    return (l << half) | r;
}

// Position `pos` of the keyed permutation of [0, n), n >= 1.
MG_HD inline uint64_t mg_permute(uint64_t pos, uint64_t n, const uint32_t key[4]) {
    int half = 1;
    while ((1ull << (2 * half)) < n) half++;
    uint64_t y = mg_feistel(pos, half, key);
    // at most 4 expected walks (the domain is < 4 n); the walk always ends
    // because the Feistel network is a permutation of a finite set
    while (y >= n) y = mg_feistel(y, half, key);
    return y;
}

// Rollout row (flat slot-major index t * rows + i) of minibatch row q.
MG_HD inline uint64_t mg_minibatch_row(const MgMinibatch& m, uint32_t q, uint64_t rows, uint64_t total) {
    if (m.slot >= 0) return (uint64_t)m.slot * rows + q;
    return mg_permute((uint64_t)m.base + q, total, m.key);
}
