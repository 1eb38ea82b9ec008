// Gradient all-reduce over NVLink peer memory (data parallelism, one process
// per GPU). Replaces the NCCL all-reduce of each minibatch's flat gradient:
//
//   finalize    each rank sums its split-K partials into its exchange buffer
//               xbuf[b] (k_grad_finalize, buffer chosen on the device; the
//               bf16-rounded GEMM-weight sums packed as bf16, exact)
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

// A 16-byte load of peer memory, cached in L2 only, issued where it stands:
// every rank's load of a work item goes out before the first add (one NVLink
// round trip per item, not one per rank).
__device__ __forceinline__ uint4 ld_u4_cg_now(const void* p) {
    uint4 v;
    asm volatile("ld.global.cg.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
    return v;
}

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
// announces was written by an earlier kernel, complete once this kernel's
// dependency wait returned; the release makes it visible to the ranks that
// acquire the flag.
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
    // launched as a programmatic dependent of the finalisation: its buffer
    // (and the counter) are complete once the wait returns
    mg_pdl_wait();
    mg_pdl_trigger();
    const unsigned int seq = *seqPtr + 1;
    const int b = seq & 1;
    announce(t, kP2PFlagsA, seq);
    wait_flags(reinterpret_cast<const unsigned int*>(t.base[t.rank] + kP2PFlagsA), t.world, seq, status);
    const size_t xOff = t.xOff[b];
    float4* gd = reinterpret_cast<float4*>(grad);
    float sq = 0.0f;
    // work items: the fp32 part in groups of 4 elements, then the bf16 part
    // in groups of 8 (16 bytes per rank either way)
    const int64_t nf = t.floatCount / 4, nh = (count - t.floatCount) / 8;
    for (int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; g < nf + nh; g += (int64_t)gridDim.x * blockDim.x) {
        // every rank's 16 bytes in flight at once (one NVLink round trip),
        // then the sum in rank order
        uint4 raw[kP2PMaxRanks];
        const int64_t byteOff = g < nf ? g * 16 : t.floatCount * 4 + (g - nf) * 16;
#pragma unroll
        for (int p = 0; p < kP2PMaxRanks; p++)
            if (p < t.world) raw[p] = ld_u4_cg_now(t.base[p] + xOff + byteOff);
        const int ne = g < nf ? 4 : 8;
        float acc[8];
#pragma unroll
        for (int p = 0; p < kP2PMaxRanks; p++) {
            if (p < t.world) {
                float v[8];
                const uint32_t w[4] = {raw[p].x, raw[p].y, raw[p].z, raw[p].w};
                if (ne == 4) {
#pragma unroll
                    for (int e = 0; e < 4; e++) v[e] = __uint_as_float(w[e]);
                } else {
#pragma unroll
                    for (int e = 0; e < 4; e++) {
                        v[2 * e] = __uint_as_float(w[e] << 16);
                        v[2 * e + 1] = __uint_as_float(w[e] & 0xffff0000u);
                    }
                }
#pragma unroll
                for (int e = 0; e < 8; e++)
                    if (e < ne) acc[e] = p == 0 ? v[e] : __fadd_rn(acc[e], v[e]);
            }
        }
        float* dst = g < nf ? grad + g * 4 : grad + t.floatCount + (g - nf) * 8;
#pragma unroll
        for (int e = 0; e < 8; e++) {
            if (e < ne) {
                acc[e] = __fmul_rn(acc[e], scale);
                sq = __fadd_rn(sq, __fmul_rn(acc[e], acc[e]));
            }
        }
        reinterpret_cast<float4*>(dst)[0] = make_float4(acc[0], acc[1], acc[2], acc[3]);
        if (ne == 8) reinterpret_cast<float4*>(dst)[1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
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

// One exchange buffer: floatCount fp32 elements, then the rest as bf16.
static size_t xbuf_bytes(int64_t count, int64_t floatCount) {
    return ((size_t)floatCount * 4 + (size_t)(count - floatCount) * 2 + 255) / 256 * 256;
}

size_t p2p_region_bytes(int64_t count, int64_t floatCount) { return kP2PData + 2 * xbuf_bytes(count, floatCount); }

void p2p_layout(P2PTable& t, int64_t count, int64_t floatCount) {
    const size_t xb = xbuf_bytes(count, floatCount);
    t.xOff[0] = kP2PData;
    t.xOff[1] = kP2PData + xb;
    t.floatCount = floatCount;
}

int p2p_allreduce(const P2PTable& t, int64_t count, float* grad, unsigned int* seq, unsigned int* counter,
                  float* normPartial, float* normSqOut, cudaStream_t st) {
    MG_CHECK_ARG(t.world >= 2 && t.world <= kP2PMaxRanks && t.rank >= 0 && t.rank < t.world,
                 "p2p all-reduce: bad rank / world size");
    MG_CHECK_ARG(count % 8 == 0 && t.floatCount % 8 == 0 && t.floatCount <= count,
                 "p2p all-reduce: the element counts must be multiples of 8");
    MG_LAUNCH(k_p2p_allreduce, p2p_blocks(), 256, 0, st, t, count, 1.0f / (float)t.world, grad, seq, counter,
              normPartial, normSqOut, status_ptr());
    return check_launch("k_p2p_allreduce");
}

}  // namespace mg
