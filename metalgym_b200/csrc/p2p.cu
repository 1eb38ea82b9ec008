// Gradient all-reduce over NVLink peer memory (data parallelism, one process
// per GPU). Replaces the NCCL all-reduce of each minibatch's flat gradient:
//
//   finalize    each rank sums its split-K partials into its exchange buffer
//               xbuf[b] (k_grad_finalize, buffer chosen on the device)
//   all-reduce  k_p2p_allreduce: every rank announces xbuf[b] complete (a
//               flag written into every rank's memory), waits for all
//               announcements, then reads every rank's xbuf[b] over NVLink,
//               sums in rank order, scales by 1 / world into the gradient
//               arena and computes the squared norm for the clip (last CTA)
//
// One synchronisation round per minibatch; each GPU reads (world - 1) peer
// buffers. b alternates per minibatch (a device counter), so a rank never
// overwrites a buffer that another rank may still read: it rewrites buffer b
// two minibatches later, after every rank has announced the minibatch in
// between, which it does only after its reads of buffer b ended. Every rank
// sums in the same order, so the ranks' gradients, and hence their weights,
// stay bit-identical. Waits on flags are bounded (2 s); a wait that gives up
// records kDevTimeoutPeer in the status word, which the host reports.
//
// Memory of one rank (one allocation, shared with the others through CUDA IPC):
//   [flags: kP2PMaxRanks x 128 B][xbuf0][xbuf1]
#include "p2p.h"

#include "metalgym/pdl.cuh"
#include "policy_kernels.cuh"
#include "metalgym/detail/ptx.cuh"
#include "runtime.h"

namespace mg {

namespace {

__device__ __forceinline__ void store_release_sys(unsigned int* p, unsigned int v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned int load_acquire_sys(const unsigned int* p) {
    unsigned int v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Thread t < world of every CTA waits (acquire, system scope) until rank t's
// flag in this rank's region reaches seq; the CTA barrier then orders the
// other threads' reads of peer data after those acquires.
__device__ void wait_flags(const unsigned int* flags, int world, unsigned int seq, int* status) {
    if ((int)threadIdx.x < world) {
        const unsigned int* f = flags + threadIdx.x * kP2PFlagStride;
        if (load_acquire_sys(f) < seq) {
            const uint64_t t0 = globaltimer();
            while (load_acquire_sys(f) < seq) {
                if (globaltimer() - t0 > kWaitLimitNs) {
                    record_error(status, kDevTimeoutPeer);
                    break;
                }
            }
        }
    }
    __syncthreads();
}

// Thread 0 of CTA 0 writes seq into slot `rank` of the flag array at byte
// `flagOff` of every rank's region (its own included). The data the flag
// announces was written by an earlier kernel, complete before this one
// started; the release makes it visible to the ranks that acquire the flag.
__device__ void announce(const P2PTable& t, size_t flagOff, unsigned int seq) {
    if (blockIdx.x == 0 && threadIdx.x == 0) {
        __threadfence_system();
        for (int p = 0; p < t.world; p++)
            store_release_sys(reinterpret_cast<unsigned int*>(t.base[p] + flagOff) + t.rank * kP2PFlagStride, seq);
    }
}

// One exchange: announce this rank's exchange buffer complete, wait for every
// rank's, then each thread sums its float4 groups over the ranks' buffers in
// rank order (peer memory read over NVLink), scales by 1 / world and writes
// the gradient arena; CTA partial sums of squares, the last CTA adds them in
// CTA order and advances the minibatch counter.
__global__ void __launch_bounds__(256) k_p2p_allreduce(const __grid_constant__ P2PTable t, int64_t count,
                                                       float scale, float* __restrict__ grad,
                                                       unsigned int* __restrict__ seqPtr,
                                                       unsigned int* __restrict__ counter,
                                                       float* __restrict__ normPartial, float* __restrict__ normSqOut,
                                                       int* status) {
    __shared__ float s_red[8];
    __shared__ bool s_last;
    const unsigned int seq = *seqPtr + 1;
    const int b = seq & 1;
    announce(t, kP2PFlagsA, seq);
    wait_flags(reinterpret_cast<const unsigned int*>(t.base[t.rank] + kP2PFlagsA), t.world, seq, status);
    const size_t xOff = t.xOff[b];
    float4* gd = reinterpret_cast<float4*>(grad);
    float sq = 0.0f;
    for (int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; g < count / 4; g += (int64_t)gridDim.x * blockDim.x) {
        // every rank's values in flight at once (one NVLink round trip), then
        // the sum in rank order
        float4 v[kP2PMaxRanks];
#pragma unroll
        for (int p = 0; p < kP2PMaxRanks; p++)
            if (p < t.world) v[p] = __ldcg(reinterpret_cast<const float4*>(t.base[p] + xOff) + g);
        float4 acc = v[0];
#pragma unroll
        for (int p = 1; p < kP2PMaxRanks; p++) {
            if (p < t.world) {
                acc.x = __fadd_rn(acc.x, v[p].x);
                acc.y = __fadd_rn(acc.y, v[p].y);
                acc.z = __fadd_rn(acc.z, v[p].z);
                acc.w = __fadd_rn(acc.w, v[p].w);
            }
        }
        acc = make_float4(__fmul_rn(acc.x, scale), __fmul_rn(acc.y, scale), __fmul_rn(acc.z, scale),
                          __fmul_rn(acc.w, scale));
        gd[g] = acc;
        sq = __fadd_rn(sq, __fadd_rn(__fadd_rn(__fmul_rn(acc.x, acc.x), __fmul_rn(acc.y, acc.y)),
                                     __fadd_rn(__fmul_rn(acc.z, acc.z), __fmul_rn(acc.w, acc.w))));
    }
    sq = warp_sum(sq);
    if ((threadIdx.x & 31) == 0) s_red[threadIdx.x >> 5] = sq;
    __syncthreads();
    if (threadIdx.x == 0) {
        float u = 0.0f;
        for (int w = 0; w < 8; w++) u = __fadd_rn(u, s_red[w]);
        normPartial[blockIdx.x] = u;
        __threadfence();
        s_last = atomicAdd(counter, 1u) == gridDim.x - 1;
    }
    __syncthreads();
    if (s_last) {
        __threadfence();
        float u = 0.0f;
        for (int k = threadIdx.x; k < (int)gridDim.x; k += 256) u = __fadd_rn(u, __ldcg(&normPartial[k]));
        u = warp_sum(u);
        if ((threadIdx.x & 31) == 0) s_red[threadIdx.x >> 5] = u;
        __syncthreads();
        if (threadIdx.x == 0) {
            float v = 0.0f;
            for (int w = 0; w < 8; w++) v = __fadd_rn(v, s_red[w]);
            *normSqOut = v;
            *counter = 0u;
            *seqPtr = seq;  // the next minibatch uses the other buffer
        }
    }
}

}  // namespace

size_t p2p_region_bytes(int64_t count) {
    const size_t xb = ((size_t)count * 4 + 255) / 256 * 256;
    return kP2PData + 2 * xb;
}

void p2p_layout(P2PTable& t, int64_t count) {
    const size_t xb = ((size_t)count * 4 + 255) / 256 * 256;
    t.xOff[0] = kP2PData;
    t.xOff[1] = kP2PData + xb;
}

int p2p_allreduce(const P2PTable& t, int64_t count, float* grad, unsigned int* seq, unsigned int* counter,
                  float* normPartial, float* normSqOut, cudaStream_t st) {
    MG_CHECK_ARG(t.world >= 2 && t.world <= kP2PMaxRanks && t.rank >= 0 && t.rank < t.world,
                 "p2p all-reduce: bad rank / world size");
    MG_CHECK_ARG(count % 4 == 0, "p2p all-reduce: count must be a multiple of 4");
    // a plain launch: this kernel waits on other GPUs, not on earlier kernels of this stream
    k_p2p_allreduce<<<p2p_blocks(), 256, 0, st>>>(t, count, 1.0f / (float)t.world, grad, seq, counter, normPartial,
                                                  normSqOut, status_ptr());
    return check_launch("k_p2p_allreduce");
}

}  // namespace mg
