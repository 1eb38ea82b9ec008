// One residual MLP block of the policy, forward, fused into one kernel per
// 128-row tile (model/ppo.h:575-626 for the order; model/layernorm.metal:
// 10-71, model/mlp.metal:18-86 and model/elementwise.metal:4-13 for the
// arithmetic):
//
//   xn = LN(h) (saved: xNorm, lnOut = bf16(g xn + b), sigma)
//   V  = relu(bf16(lnOut Up))            (saved, R x H)
//   h  = bf16(h + bf16(V Dp))            (in place)
//
// The hidden layer is processed in chunks of 64 columns. Per chunk the
// tensor cores compute the up-projection into one of two TMEM accumulators,
// the row warps apply ReLU and write the chunk, in the swizzled K-major
// layout, to shared memory, from where a TMA store writes it to V and the
// tensor cores add its down-projection into a third accumulator. Every tile
// moves between global and shared memory by TMA (h in, xNorm / lnOut / V / h
// out), so global accesses are whole lines whatever the row-per-thread
// layout of the tensor-memory reads.
//
// Warp roles (224 threads): warp 0 TMA loads of h and Up, warp 6 TMA loads of
// Dp (two producers, so an Up chunk never waits behind a Dp chunk), warp 1
// MMA, warps 2-5 row work (LayerNorm, epilogues, TMA stores by one elected
// thread): thread (warp, lane) owns tile row 32 (warp % 4) + lane, the TMEM
// lane quarter its warp may access.
//
// The LayerNorm sums follow exactly the order of k_layernorm_forward (32
// partial sums of E/32 consecutive columns, combined as a butterfly over 32
// lanes), so the block's outputs are bit-identical to the unfused kernels.
#include "block.h"
#include "gemm_tc.cuh"
#include "policy_kernels.cuh"
#include "runtime.h"

namespace mg {

namespace {

constexpr int kHC = 64;  // hidden columns per chunk
constexpr int kWS = 4;   // weight-chunk ring depth (loads run up to 3 chunks ahead)

template <int E>
struct BlockFwdSmem {
    static constexpr int TILE = E * 256;           // 128 rows x E bf16 (K-major, E/64 blocks of 16 KB)
    static constexpr int WUP_BYTES = E * kHC * 2;  // E (K) x 64 (N), MN-major
    static constexpr int V_BYTES = 128 * kHC * 2;  // 128 rows x 64 (K-major, one block)
    static constexpr int WDN_BYTES = kHC * E * 2;  // 64 (K) x E (N), MN-major
    static constexpr int OFF_A = 0;                // lnOut: MMA operand and store source
    static constexpr int OFF_H = OFF_A + TILE;     // h tile in; h out
    static constexpr int OFF_V = OFF_H + TILE;     // two V chunks; xNorm staging before them
    static constexpr int OFF_WUP = OFF_V + 2 * V_BYTES;
    static constexpr int OFF_WDN = OFF_WUP + kWS * WUP_BYTES;
    static constexpr int OFF_BAR = OFF_WDN + kWS * WDN_BYTES;
    static_assert(TILE <= 2 * V_BYTES, "xNorm staging must fit the V buffers");
    static constexpr int OFF_GB = OFF_BAR + 256;             // gamma, beta as fp32
    static constexpr int BYTES = OFF_GB + 2 * E * 4 + 1024;  // + alignment slack
};

// Sum of 32 partials in the order of warp_sum (xor butterfly 16, 8, 4, 2, 1).
__device__ __forceinline__ float butterfly32(float* p) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
#pragma unroll
        for (int l = 0; l < o; l++) p[l] = __fadd_rn(p[l], p[l + o]);
    return p[0];
}

__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
}

// Barrier over the 128 row threads (warps 2-5), named barrier 1.
__device__ __forceinline__ void row_barrier() { asm volatile("bar.sync 1, 128;" ::: "memory"); }
// The same barrier, returning whether v holds on every row thread, so that
// all row warps take the same branch after a bounded wait gave up.
__device__ __forceinline__ bool row_all(bool v) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.u32 q, %1, 0;\n\t"
        "bar.red.and.pred p, 1, 128, q;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(r)
        : "r"((uint32_t)v)
        : "memory");
    return r != 0;
}

struct BlockFwdMaps {
    CUtensorMap up, dn;      // weights: Up [E][H], Dp [H][E] (K rows of N), boxes 64 x 64
    CUtensorMap h, xn, lo;   // [rows][E], boxes 64 x 128
    CUtensorMap v;           // [rows][H], box 64 x 128
};

template <int E>
__global__ void __launch_bounds__(224, 1) k_block_forward(const __grid_constant__ BlockFwdMaps maps, BlockFwdArgs args) {
    using S = BlockFwdSmem<E>;
    constexpr int VPT = E / 32;
    constexpr int KB = E / 64;  // 64-column blocks of a row tile
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sA = smem + S::OFF_A;
    uint8_t* sH = smem + S::OFF_H;
    uint8_t* sXn = smem + S::OFF_V;  // free until the first chunk epilogue
    uint64_t* bar = reinterpret_cast<uint64_t*>(smem + S::OFF_BAR);
    uint64_t* hFull = bar + 0;
    uint64_t* aReady = bar + 1;
    uint64_t* d1Full = bar + 2;    // [2]
    uint64_t* d1Empty = bar + 4;   // [2]
    uint64_t* vFull = bar + 6;     // [2]
    uint64_t* vEmpty = bar + 8;    // [2]
    uint64_t* d2Full = bar + 10;
    uint64_t* done = bar + 11;
    uint64_t* wupFull = bar + 12;  // [kWS]
    uint64_t* wupEmpty = wupFull + kWS;
    uint64_t* wdnFull = wupEmpty + kWS;
    uint64_t* wdnEmpty = wdnFull + kWS;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(wdnEmpty + kWS);
    float* s_gb = reinterpret_cast<float*>(smem + S::OFF_GB);  // gamma[E], beta[E]

    mg_pdl_trigger();
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int NC = args.H / kHC;
    const int m0 = blockIdx.x * 128;
    int* status = args.status;

    if (threadIdx.x == 0) {
        mbar_init(hFull, 1);
        mbar_init(aReady, 1);
        for (int w = 0; w < kWS; w++) {
            mbar_init(&wupFull[w], 1);
            mbar_init(&wupEmpty[w], 1);
            mbar_init(&wdnFull[w], 1);
            mbar_init(&wdnEmpty[w], 1);
        }
        for (int b = 0; b < 2; b++) {
            mbar_init(&d1Full[b], 1);
            mbar_init(&d1Empty[b], 1);
            mbar_init(&vFull[b], 1);
            mbar_init(&vEmpty[b], 1);
        }
        mbar_init(d2Full, 1);
        mbar_init(done, 1);
        fence_barrier_init();
        prefetch_tensormap(&maps.up);
        prefetch_tensormap(&maps.dn);
        prefetch_tensormap(&maps.h);
    }
    if (warp == 2) {
        tmem_alloc(tmem_slot, 256);  // D1[0], D1[1]: 64 columns each; D2: E columns at 128
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    mg_pdl_wait();  // h and the weights come from earlier kernels

    if (warp == 0) {
        if (lane == 0) {
            // ---- TMA loads: the h tile, then chunk c of Up (E x 64)
            mbar_arrive_expect_tx(hFull, S::TILE);
#pragma unroll
            for (int kb = 0; kb < KB; kb++) tma_load_2d(sH + kb * 16384, &maps.h, kb * 64, m0, hFull);
            int nu = 0;
            for (int c = 0; c < NC; c++) {
                const int w = c % kWS;
                if (!mbar_wait(&wupEmpty[w], ((c / kWS) & 1) ^ 1, status, kDevTimeoutEmpty)) break;
                uint8_t* wu = smem + S::OFF_WUP + w * S::WUP_BYTES;
                mbar_arrive_expect_tx(&wupFull[w], S::WUP_BYTES);
#pragma unroll
                for (int kb = 0; kb < KB; kb++) tma_load_2d(wu + kb * 8192, &maps.up, c * kHC, kb * 64, &wupFull[w]);
                nu++;
            }
            // drain: every copy has landed before the CTA can exit
            mbar_wait(hFull, 0, status, kDevTimeoutFull);
            for (int c = nu - kWS < 0 ? 0 : nu - kWS; c < nu; c++)
                mbar_wait(&wupFull[c % kWS], (c / kWS) & 1, status, kDevTimeoutFull);
        }
    } else if (warp == 6) {
        if (lane == 0) {
            // ---- TMA loads: chunk c of Dp (64 x E)
            int nd = 0;
            for (int c = 0; c < NC; c++) {
                const int w = c % kWS;
                if (!mbar_wait(&wdnEmpty[w], ((c / kWS) & 1) ^ 1, status, kDevTimeoutEmpty)) break;
                uint8_t* wd = smem + S::OFF_WDN + w * S::WDN_BYTES;
                mbar_arrive_expect_tx(&wdnFull[w], S::WDN_BYTES);
#pragma unroll
                for (int j = 0; j < KB; j++) tma_load_2d(wd + j * 8192, &maps.dn, 64 * j, c * kHC, &wdnFull[w]);
                nd++;
            }
            for (int c = nd - kWS < 0 ? 0 : nd - kWS; c < nd; c++)
                mbar_wait(&wdnFull[c % kWS], (c / kWS) & 1, status, kDevTimeoutFull);
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ---- MMA
            constexpr uint32_t idUp = idesc_bf16_f32(kHC, false, true);
            constexpr uint32_t idDn = idesc_bf16_f32(E, false, true);
            const uint32_t aBase = smem_u32(sA);
            const uint32_t d2 = tmem + 128;
            bool ok = mbar_wait(aReady, 0, status, kDevTimeoutFull);
            tc_fence_after();
            auto down = [&](int k) -> bool {
                const int b = k & 1;
                const uint32_t ph = (k >> 1) & 1;
                const int w = k % kWS;
                if (!mbar_wait(&vFull[b], ph, status, kDevTimeoutFull)) return false;
                if (!mbar_wait(&wdnFull[w], (k / kWS) & 1, status, kDevTimeoutFull)) return false;
                tc_fence_after();
                const uint32_t vBase = smem_u32(smem + S::OFF_V + b * S::V_BYTES);
                const uint32_t wBase = smem_u32(smem + S::OFF_WDN + w * S::WDN_BYTES);
#pragma unroll
                for (int kk = 0; kk < 4; kk++)
                    tc_mma_bf16(d2, smem_desc_sw128(vBase + kk * 32, 16, 1024),
                                smem_desc_sw128(wBase + kk * 2048, 8192, 1024), idDn, (k > 0 || kk > 0) ? 1u : 0u);
                tc_commit(&vEmpty[b]);
                tc_commit(&wdnEmpty[w]);
                return true;
            };
            // up(c + 1) is issued before down(c): it only needs the epilogue of
            // chunk c - 1, so the epilogue of chunk c + 1 can start as soon as
            // that of chunk c ends
            auto up = [&](int c) -> bool {
                const int b = c & 1;
                const uint32_t ph = (c >> 1) & 1;
                const int w = c % kWS;
                if (!mbar_wait(&wupFull[w], (c / kWS) & 1, status, kDevTimeoutFull)) return false;
                if (!mbar_wait(&d1Empty[b], ph ^ 1, status, kDevTimeoutEmpty)) return false;
                tc_fence_after();
                const uint32_t wBase = smem_u32(smem + S::OFF_WUP + w * S::WUP_BYTES);
                const uint32_t d1 = tmem + (uint32_t)(b * kHC);
#pragma unroll
                for (int kb = 0; kb < KB; kb++)
#pragma unroll
                    for (int kk = 0; kk < 4; kk++)
                        tc_mma_bf16(d1, smem_desc_sw128(aBase + kb * 16384 + kk * 32, 16, 1024),
                                    smem_desc_sw128(wBase + kb * 8192 + kk * 2048, 8192, 1024), idUp,
                                    (kb > 0 || kk > 0) ? 1u : 0u);
                tc_commit(&wupEmpty[w]);
                tc_commit(&d1Full[b]);
                return true;
            };
            if (ok) ok = up(0);
            for (int c = 0; c < NC && ok; c++) {
                if (c + 1 < NC) ok = up(c + 1);
                if (ok) ok = down(c);
            }
            if (ok) tc_commit(d2Full);
            tc_commit(done);  // covers every MMA issued, also after a timeout
        }
    } else if (warp >= 2 && warp <= 5) {
        // ---- row work: thread owns tile row tr; warp 2 lane 0 issues the stores
        const int q = warp & 3;
        const int tr = q * 32 + lane;
        const int row = m0 + tr;
        const bool valid = row < args.rows;
        const bool leader = threadIdx.x == 64;
        for (int i = threadIdx.x - 64; i < E; i += 128) {
            s_gb[i] = bf(args.gamma[i]);
            s_gb[E + i] = bf(args.beta[i]);
        }
        row_barrier();
        bool ok = row_all(mbar_wait_warp(hFull, 0, status, kDevTimeoutFull));
        // the row (zero beyond the matrix: TMA fills out-of-range rows with 0),
        // read 8 values per 16-byte load
        auto chunk8 = [&](int ch, float* f) {
            const uint4 w = *reinterpret_cast<const uint4*>(sH + sw128_offset(tr, ch));
            const uint32_t u[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
            for (int t = 0; t < 4; t++) {
                f[2 * t] = __uint_as_float(u[t] << 16);
                f[2 * t + 1] = __uint_as_float(u[t] & 0xffff0000u);
            }
        };
        // LayerNorm: the order of k_layernorm_forward (lane l: columns l*VPT ..)
        float p[32];
#pragma unroll
        for (int ch = 0; ch < E / 8; ch++) {
            float f[8];
            chunk8(ch, f);
#pragma unroll
            for (int g = 0; g < 8 / VPT; g++) {
                float s = 0.0f;
#pragma unroll
                for (int j = 0; j < VPT; j++) s = __fadd_rn(s, f[g * VPT + j]);
                p[ch * (8 / VPT) + g] = s;
            }
        }
        const float mean = __fdiv_rn(butterfly32(p), (float)E);
        asm volatile("" ::: "memory");  // re-read the row per pass rather than hold it in registers
#pragma unroll
        for (int ch = 0; ch < E / 8; ch++) {
            float f[8];
            chunk8(ch, f);
#pragma unroll
            for (int g = 0; g < 8 / VPT; g++) {
                float s = 0.0f;
#pragma unroll
                for (int j = 0; j < VPT; j++) {
                    const float d = __fsub_rn(f[g * VPT + j], mean);
                    s = __fadd_rn(s, __fmul_rn(d, d));
                }
                p[ch * (8 / VPT) + g] = s;
            }
        }
        const float var = __fdiv_rn(butterfly32(p), (float)E);
        const float sd = __fsqrt_rn(__fadd_rn(var, 1e-5f));
        const float rstd = __fdiv_rn(1.0f, sd);
        if (valid) args.stdev[row] = sd;
        asm volatile("" ::: "memory");
#pragma unroll
        for (int ch = 0; ch < E / 8; ch++) {
            float f[8];
            chunk8(ch, f);
            const float4 g0 = *reinterpret_cast<const float4*>(s_gb + ch * 8);
            const float4 g1 = *reinterpret_cast<const float4*>(s_gb + ch * 8 + 4);
            const float4 b0 = *reinterpret_cast<const float4*>(s_gb + E + ch * 8);
            const float4 b1 = *reinterpret_cast<const float4*>(s_gb + E + ch * 8 + 4);
            const float gg[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
            const float bb[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
            uint32_t xn4[4], y4[4];
#pragma unroll
            for (int t = 0; t < 4; t++) {
                const float xn0 = __fmul_rn(__fsub_rn(f[2 * t], mean), rstd);
                const float xn1 = __fmul_rn(__fsub_rn(f[2 * t + 1], mean), rstd);
                xn4[t] = pack_bf16(xn0, xn1);
                y4[t] = pack_bf16(__fadd_rn(__fmul_rn(gg[2 * t], xn0), bb[2 * t]),
                                  __fadd_rn(__fmul_rn(gg[2 * t + 1], xn1), bb[2 * t + 1]));
            }
            *reinterpret_cast<uint4*>(sXn + sw128_offset(tr, ch)) = make_uint4(xn4[0], xn4[1], xn4[2], xn4[3]);
            *reinterpret_cast<uint4*>(sA + sw128_offset(tr, ch)) = make_uint4(y4[0], y4[1], y4[2], y4[3]);
        }
        fence_async_smem();
        row_barrier();
        if (leader) {
            mbar_arrive(aReady);
#pragma unroll
            for (int kb = 0; kb < KB; kb++) {
                tma_store_2d(&maps.xn, kb * 64, m0, sXn + kb * 16384);
                tma_store_2d(&maps.lo, kb * 64, m0, sA + kb * 16384);
            }
            bulk_commit();
        }

        // hidden chunks: V = relu(bf16(D1)) into shared memory, stored by TMA
        for (int c = 0; c < NC && ok; c++) {
            const int b = c & 1;
            const uint32_t ph = (c >> 1) & 1;
            const bool got = mbar_wait_warp(&d1Full[b], ph, status, kDevTimeoutDone) &&
                             mbar_wait_warp(&vEmpty[b], ph ^ 1, status, kDevTimeoutEmpty);
            // the store of chunk c - 2 has read buffer b (before chunk 1, also the
            // xNorm store, staged in both buffers)
            if (leader) {
                if (c < 2) bulk_wait_read<0>();
                else bulk_wait_read<1>();
            }
            if (!row_all(got)) {
                ok = false;
                break;
            }
            tc_fence_after();
            uint8_t* sV = smem + S::OFF_V + b * S::V_BYTES;
            const uint32_t d1 = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(b * kHC);
            uint32_t raw[kHC];
#pragma unroll
            for (int j = 0; j < kHC / 32; j++) tmem_ld32_async(d1 + (uint32_t)(j * 32), raw + 32 * j);
            tc_wait_ld();
#pragma unroll
            for (int j = 0; j < kHC / 32; j++) {
                uint32_t w[16];
#pragma unroll
                for (int i = 0; i < 16; i++) {
                    const float r0 = round_bf16(__uint_as_float(raw[32 * j + 2 * i]));
                    const float r1 = round_bf16(__uint_as_float(raw[32 * j + 2 * i + 1]));
                    w[i] = pack_bf16(r0 > 0.0f ? r0 : r0 * 0.0f, r1 > 0.0f ? r1 : r1 * 0.0f);
                }
#pragma unroll
                for (int i = 0; i < 4; i++)
                    *reinterpret_cast<uint4*>(sV + sw128_offset(tr, j * 4 + i)) =
                        make_uint4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
            }
            tc_fence_before();
            fence_async_smem();
            row_barrier();
            if (leader) {
                mbar_arrive(&d1Empty[b]);
                mbar_arrive(&vFull[b]);
                tma_store_2d(&maps.v, c * kHC, m0, sV);
                bulk_commit();
            }
        }
        // h = bf16(h + bf16(V Dp)), written over the h tile and stored by TMA
        if (ok && row_all(mbar_wait_warp(d2Full, 0, status, kDevTimeoutDone))) {
            tc_fence_after();
            const uint32_t d2 = tmem + ((uint32_t)(q * 32) << 16) + 128u;
#pragma unroll
            for (int j = 0; j < E / 32; j++) {
                float v[32];
                tmem_ld32(d2 + (uint32_t)(j * 32), v);
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    uint4* cell = reinterpret_cast<uint4*>(sH + sw128_offset(tr, j * 4 + i));
                    const uint4 o = *cell;
                    const uint32_t ow[4] = {o.x, o.y, o.z, o.w};
                    uint32_t w[4];
#pragma unroll
                    for (int t = 0; t < 4; t++) {
                        const int k = i * 8 + 2 * t;
                        w[t] = pack_bf16(__fadd_rn(__uint_as_float(ow[t] << 16), round_bf16(v[k])),
                                         __fadd_rn(__uint_as_float(ow[t] & 0xffff0000u), round_bf16(v[k + 1])));
                    }
                    *cell = make_uint4(w[0], w[1], w[2], w[3]);
                }
            }
            fence_async_smem();
            row_barrier();
            if (leader) {
#pragma unroll
                for (int kb = 0; kb < KB; kb++) tma_store_2d(&maps.h, kb * 64, m0, sH + kb * 16384);
                bulk_commit();
            }
        }
        if (leader) bulk_wait<0>();  // every store complete before the CTA exits
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 2) {
        mbar_wait(done, 0, status, kDevTimeoutDone);
        tc_fence_after();
        tmem_dealloc(tmem, 256);
    }
}

}  // namespace

bool block_forward_supported(int E, int H) { return (E == 64 || E == 128) && H % kHC == 0 && H >= kHC; }

int block_forward(const BlockFwdArgs& a, const void* up, const void* down, cudaStream_t st) {
    MG_CHECK_ARG(block_forward_supported(a.E, a.H), "block_forward: embed must be 64 or 128 and hidden a multiple of 64");
    MG_CHECK_ARG(a.rows > 0 && a.h && a.gamma && a.beta && a.xNorm && a.lnOut && a.stdev && a.V && up && down,
                 "block_forward: null argument");
    BlockFwdMaps m;
    int rc = make_tmap_bf16(&m.up, up, a.H, a.E, a.H, 64);  // Up [E][H]: K rows of N
    if (!rc) rc = make_tmap_bf16(&m.dn, down, a.E, a.H, a.E, 64);  // Dp [H][E]: K rows of N
    if (!rc) rc = make_tmap_bf16(&m.h, a.h, a.E, a.rows, a.E, 128);
    if (!rc) rc = make_tmap_bf16(&m.xn, a.xNorm, a.E, a.rows, a.E, 128);
    if (!rc) rc = make_tmap_bf16(&m.lo, a.lnOut, a.E, a.rows, a.E, 128);
    if (!rc) rc = make_tmap_bf16(&m.v, a.V, a.H, a.rows, a.H, 128);
    if (rc) return rc;
    BlockFwdArgs args = a;
    args.status = status_ptr();
    const int grid = (a.rows + 127) / 128;
    if (a.E == 64) {
        using S = BlockFwdSmem<64>;
        static std::atomic<uint64_t> attr_done{0};
        if (int rc2 = smem_limit_once(k_block_forward<64>, S::BYTES, attr_done)) return rc2;
        MG_CUDA_TRY(mg_launch(k_block_forward<64>, dim3(grid), dim3(224), (size_t)S::BYTES, st, m, args));
    } else {
        using S = BlockFwdSmem<128>;
        static std::atomic<uint64_t> attr_done{0};
        if (int rc2 = smem_limit_once(k_block_forward<128>, S::BYTES, attr_done)) return rc2;
        MG_CUDA_TRY(mg_launch(k_block_forward<128>, dim3(grid), dim3(224), (size_t)S::BYTES, st, m, args));
    }
    return check_launch("k_block_forward");
}

}  // namespace mg

extern "C" int mg_block_forward(void* h, const void* gamma, const void* beta, const void* up, const void* down,
                                void* x_norm, void* ln_out, float* stdev, void* v, int rows, int embed, int hidden,
                                mg_stream_t stream) {
    mg::BlockFwdArgs a{};
    a.h = static_cast<__nv_bfloat16*>(h);
    a.gamma = static_cast<const __nv_bfloat16*>(gamma);
    a.beta = static_cast<const __nv_bfloat16*>(beta);
    a.xNorm = static_cast<__nv_bfloat16*>(x_norm);
    a.lnOut = static_cast<__nv_bfloat16*>(ln_out);
    a.stdev = stdev;
    a.V = static_cast<__nv_bfloat16*>(v);
    a.rows = rows;
    a.E = embed;
    a.H = hidden;
    return mg::block_forward(a, up, down, reinterpret_cast<cudaStream_t>(stream));
}
