// Gradient all-reduce over NVLink peer memory (p2p.cu).
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace mg {

constexpr int kP2PMaxRanks = 16;
constexpr int kP2PFlagStride = 32;  // uint32 per rank slot: one 128-byte line
constexpr size_t kP2PFlagsA = 0;  // "exchange buffer complete" flags
constexpr size_t kP2PData = (size_t)kP2PMaxRanks * kP2PFlagStride * 4;  // buffers start here

// Every rank's region (own and peers', opened through CUDA IPC) and the
// buffer offsets inside a region.
// An exchange buffer holds the gradient arena's first floatCount elements as
// fp32 and the rest (the GEMM weights' gradients, rounded to bf16 by the
// finalisation) packed as bf16: exact, and half the bytes over NVLink.
struct P2PTable {
    unsigned char* base[kP2PMaxRanks];
    size_t xOff[2];
    int64_t floatCount;
    int rank, world;
};

// CTAs of the exchange kernel: few enough to be resident together (CTA 0
// announces for all of them), enough to keep NVLink busy: one per SM.
inline int p2p_blocks() { return 148; }

// Bytes of one rank's region for a gradient of `count` elements whose first
// floatCount are fp32 in the exchange buffers (both multiples of 8), and the
// buffer offsets within it.
size_t p2p_region_bytes(int64_t count, int64_t floatCount);
void p2p_layout(P2PTable& t, int64_t count, int64_t floatCount);

// The exchange kernel: grad = (sum over ranks of xbuf[b], in rank order) /
// world, normSqOut = |grad|^2; seq is the device minibatch counter that
// selects b (the gradient finalisation writes xbuf[b] with the same rule,
// its elements from t.floatCount on packed as bf16).
int p2p_allreduce(const P2PTable& t, int64_t count, float* grad, unsigned int* seq, unsigned int* counter,
                  float* normPartial, float* normSqOut, cudaStream_t st);

}  // namespace mg
