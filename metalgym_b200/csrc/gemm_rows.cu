// Row-complete GEMM for 128-wide outputs with the row epilogue of the layer
// that follows it:
//
//   out[M x 128] = A[M x K] B[K x 128]   (A K-major; B K- or MN-major)
//
// The K dimension is split over a cluster of 4 CTAs (K a multiple of 256), and
// the 4 fp32 partial tiles are summed through distributed shared memory, so a
// 4096-row product runs on 128 CTAs while every output row still ends in one
// warp, which applies a row epilogue needing the whole row:
//
//   kRowsResidLN     h = bf16(h + bf16(acc)) in place, then the LayerNorm of
//                    h: the down projection of a residual block followed by
//                    the next block's (or the final) LayerNorm
//                    (model/mlp.metal:60-86, model/elementwise.metal:4-13,
//                    model/layernorm.metal:10-71), in the arithmetic of
//                    k_layernorm_forward (lane l: columns 4l..4l+3)
//   kRowsLNBackward  dz = bf16(acc), then the LayerNorm backward of dz with
//                    the residual gradient added: the branch gradient of a
//                    residual block followed by its LayerNorm backward
//                    (model/mlp.metal:131-153, model/layernorm.metal:74-127,
//                    model/ppo.h:851-852), in the arithmetic of
//                    k_layernorm_backward, including its dgamma / dbeta
//                    partial sums over groups of RPC rows
//
// CTA q of a cluster computes the K range [q kPer, (q + 1) kPer) of one
// 128 x 128 tile (TMA ring, tcgen05.mma into TMEM, one thread per row reads
// the accumulator), writes its fp32 tile into its own shared memory, and
// after a cluster barrier owns tile rows [32 q, 32 q + 32): lane l of a warp
// sums columns 4l..4l+3 of a row over the cluster's partial tiles in split
// order. That is the split-K product (kEpiF32 partials with the same kPer)
// followed by an ordered fp32 reduction, bit for bit. Every wait is bounded;
// the cluster barriers are reached by every thread on every path.
#include "gemm.h"
#include "gemm_tc.cuh"
#include "policy.h"
#include "policy_kernels.cuh"
#include "runtime.h"

namespace mg {

namespace {

constexpr int kRowsBM = 128;
constexpr int kRowsBN = 128;
constexpr int kRowsStages = 2;
constexpr uint32_t kRowsCluster = 4;  // CTAs per cluster = K splits; each ends 32 rows of the tile
// 16 warps: all copy the accumulator out of TMEM (quadrant w % 4, columns
// 32 (w / 4) ..), and two rows per warp give the row epilogue enough warps to
// hide its latency (four warps of eight rows each were latency bound)
constexpr int kRowsThreads = 512;
constexpr int kRowsA = kRowsBM * 64 * 2;  // 16 KB per 64-wide K block
constexpr int kRowsB = kRowsBN * 64 * 2;
constexpr int kRowsStage = kRowsA + kRowsB;
constexpr int kRowsRing = kRowsStages * kRowsStage;  // 64 KB
// after the MMAs the ring holds the fp32 partial tile (64 KB, read by the
// whole cluster); the LayerNorm-backward column sums (32 KB, this CTA) follow
// it. About 97 KB in all: two CTAs fit on an SM, so the next kernel's CTAs
// can start (programmatic dependent launch) beside this one's.
constexpr int kRowsTile = kRowsBM * kRowsBN * 4;
constexpr int kRowsRedOff = kRowsRing;
constexpr int kRowsRedBytes = 4 * 8 * 2 * kRowsBN * 4;
constexpr int kRowsSmem = kRowsRing + kRowsRedBytes + 256 + 1024;
static_assert(kRowsTile <= kRowsRing, "the partial tile must fit in the ring");
constexpr int kRowsSmemOnePerSm = 120 * 1024;  // more than half an SM's 228 KB
static_assert(kRowsSmemOnePerSm >= kRowsSmem, "");

enum RowsEpilogue : int { kRowsResidLN = 0, kRowsLNBackward = 1 };

struct RowsParams {
    int M, K, kPer;
    const __nv_bfloat16* resid;  // h before the residual add / the residual gradient
    __nv_bfloat16* out;          // h after it (may equal resid) / dS = resid + LayerNorm backward
    LnOutputs ln;                // kRowsResidLN
    const __nv_bfloat16* gamma;  // kRowsLNBackward: the LayerNorm's gamma, x-hat and sigma
    const __nv_bfloat16* xNorm;
    const float* stdev;
    float* partial;  // [M / RPC][dgamma (128) | dbeta (128)]
    int* status;
};

// Byte offset of the 16-byte column chunk k (columns 4k..4k+3) of tile row r in
// a partial tile: rows of 512 bytes, chunks XOR-swizzled by the row, so a
// warp writing chunk k of 32 rows and a warp reading a whole row are both
// free of bank conflicts.
__device__ __forceinline__ uint32_t tile_offset(int r, int k) { return (uint32_t)(r * 512 + ((k ^ (r & 31)) << 4)); }

__device__ __forceinline__ float4 bf4_load(const __nv_bfloat16* p) {
    const uint2 w = *reinterpret_cast<const uint2*>(p);
    return make_float4(__uint_as_float(w.x << 16), __uint_as_float(w.x & 0xffff0000u), __uint_as_float(w.y << 16),
                       __uint_as_float(w.y & 0xffff0000u));
}
__device__ __forceinline__ void bf4_store(__nv_bfloat16* p, float a, float b, float c, float d) {
    __nv_bfloat162 x = __floats2bfloat162_rn(a, b), y = __floats2bfloat162_rn(c, d);
    *reinterpret_cast<uint2*>(p) = make_uint2(*reinterpret_cast<uint32_t*>(&x), *reinterpret_cast<uint32_t*>(&y));
}

template <bool B_MN, int EPI, int RPC>
__global__ void __launch_bounds__(kRowsThreads, 2)
    k_gemm_rows(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, const RowsParams p) {
    constexpr int E = kRowsBN;
    // x / E as x * (1 / E): exact for a power of two; 1 / x as the correctly
    // rounded reciprocal: the same values as the LayerNorm kernels' divisions
    constexpr float kInvE = 1.0f / E;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + kRowsRing + kRowsRedBytes);
    uint64_t* empty = full + kRowsStages;
    uint64_t* done = empty + kRowsStages;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);

    mg_pdl_trigger();
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t q = cluster_ctarank();
    const int m0 = (int)(blockIdx.x / kRowsCluster) * kRowsBM;
    const int kBegin = (int)q * p.kPer;
    const int kEnd = min(p.K, kBegin + p.kPer);
    const int nk = kEnd > kBegin ? (kEnd - kBegin + 63) / 64 : 0;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kRowsStages; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(done, 1);
        fence_barrier_init();
        prefetch_tensormap(&tmA);
        prefetch_tensormap(&tmB);
    }
    if (warp == 2) {
        tmem_alloc(tmem_slot, kRowsBN);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    mg_pdl_wait();  // operands and the row inputs come from earlier kernels

    if (warp == 0 && lane == 0) {
        // ---- TMA producer
        int issued = 0;
        for (int kb = 0; kb < nk; kb++) {
            const int s = kb % kRowsStages;
            if (!mbar_wait(&empty[s], ((kb / kRowsStages) & 1) ^ 1, p.status, kDevTimeoutEmpty)) break;
            issued = kb + 1;
            uint8_t* sA = smem + s * kRowsStage;
            uint8_t* sB = sA + kRowsA;
            const int k0 = kBegin + kb * 64;
            mbar_arrive_expect_tx(&full[s], kRowsStage);
            tma_load_2d(sA, &tmA, k0, m0, &full[s]);
            if (B_MN) {
                tma_load_2d(sB, &tmB, 0, k0, &full[s]);
                tma_load_2d(sB + 8192, &tmB, 64, k0, &full[s]);
            } else {
                tma_load_2d(sB, &tmB, k0, 0, &full[s]);
            }
        }
        for (int kb = issued - kRowsStages < 0 ? 0 : issued - kRowsStages; kb < issued; kb++)
            mbar_wait(&full[kb % kRowsStages], (kb / kRowsStages) & 1, p.status, kDevTimeoutFull);
    } else if (warp == 1 && lane == 0) {
        // ---- MMA issuer
        constexpr uint32_t idesc = idesc_bf16_f32(kRowsBN, false, B_MN);
        for (int kb = 0; kb < nk; kb++) {
            const int s = kb % kRowsStages;
            if (!mbar_wait(&full[s], (kb / kRowsStages) & 1, p.status, kDevTimeoutFull)) break;
            tc_fence_after();
            const uint32_t aBase = smem_u32(smem + s * kRowsStage);
            const uint32_t bBase = aBase + kRowsA;
#pragma unroll
            for (int kk = 0; kk < 4; kk++) {
                const uint64_t ad = smem_desc_sw128(aBase + kk * 32, 16, 1024);
                const uint64_t bd = B_MN ? smem_desc_sw128(bBase + kk * 2048, 8192, 1024)
                                         : smem_desc_sw128(bBase + kk * 32, 16, 1024);
                tc_mma_bf16(tmem, ad, bd, idesc, (kb > 0 || kk > 0) ? 1u : 0u);
            }
            tc_commit(&empty[s]);
        }
        tc_commit(done);
    }

    // ---- this CTA's fp32 partial tile into shared memory (the ring is free
    // once `done` fired: every MMA, and so every read of the ring, completed).
    // Warp w reads TMEM lanes 32 (w % 4) .. (its quadrant), columns 32 (w / 4) ..
    __syncwarp();
    const bool ready = (nk == 0) || mbar_wait_warp(done, 0, p.status, kDevTimeoutDone);
    tc_fence_after();
    {
        const int qd = warp & 3, cc = warp >> 2;
        const int tr = qd * 32 + lane;
        float v[32];
        if (ready && nk > 0) {
            tmem_ld32(tmem + ((uint32_t)(qd * 32) << 16) + (uint32_t)(cc * 32), v);
        } else {
#pragma unroll
            for (int i = 0; i < 32; i++) v[i] = 0.0f;
        }
#pragma unroll
        for (int k = 0; k < 8; k++)
            *reinterpret_cast<float4*>(smem + tile_offset(tr, cc * 8 + k)) =
                make_float4(v[4 * k], v[4 * k + 1], v[4 * k + 2], v[4 * k + 3]);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 2) {
        if (!ready) mbar_wait(done, 0, p.status, kDevTimeoutDone);  // no MMA runs on freed TMEM
        tc_fence_after();
        tmem_dealloc(tmem, kRowsBN);
    }
    cluster_sync();  // every partial tile of the cluster is complete

    // ---- rows [32 q, 32 q + 32) of the tile, NR per warp, computed side by
    // side (their warp sums interleave); loads and stores of rows past M are
    // skipped, their values unused. LayerNorm backward row order (that of
    // k_layernorm_backward with RPC rows per CTA and 8 warps): per group g of
    // RPC rows, virtual warp v takes rows v, v + 8, .. and sums its dgamma /
    // dbeta over them in that order; virtual warp (g, v) is warp 8 g + v (mod
    // 16) here.
    constexpr int G = 32 / RPC;
    constexpr int J = RPC / 8;
    constexpr int NR = EPI == kRowsResidLN ? 2 : (RPC == 32 ? 4 : 2);
    const bool active = EPI == kRowsResidLN || RPC != 32 || warp < 8;
    const int c0 = lane * 4;
    int rows[NR];
    bool live[NR];
    float4 acc[NR];
#pragma unroll
    for (int t = 0; t < NR; t++) {
        int tl;  // row within this CTA's 32
        if (EPI == kRowsResidLN) {
            tl = warp + 16 * t;
        } else {
            const int pr = warp + 16 * (t / J), j = t % J;
            tl = (pr / 8) * RPC + (pr % 8) + 8 * j;
        }
        const int tr = 32 * (int)q + tl;
        rows[t] = m0 + tr;
        live[t] = active && rows[t] < p.M;
        const uint8_t* cell = smem + tile_offset(tr & 127, lane);
        float4 a = make_float4(0, 0, 0, 0);
        if (active) {
            a = *reinterpret_cast<const float4*>(__cluster_map_shared_rank(cell, 0));
#pragma unroll
            for (uint32_t r = 1; r < kRowsCluster; r++) {
                const float4 b = *reinterpret_cast<const float4*>(__cluster_map_shared_rank(cell, r));
                a = make_float4(__fadd_rn(a.x, b.x), __fadd_rn(a.y, b.y), __fadd_rn(a.z, b.z), __fadd_rn(a.w, b.w));
            }
        }
        acc[t] = a;
    }

    if (EPI == kRowsResidLN) {
        const float4 gm = bf4_load(p.ln.gamma + c0), bt = bf4_load(p.ln.beta + c0);
        const float g[4] = {gm.x, gm.y, gm.z, gm.w}, b[4] = {bt.x, bt.y, bt.z, bt.w};
        float v[NR][4], ms[2 * NR];  // ms: row sums (0..NR-1), sums of squares (NR..)
#pragma unroll
        for (int t = 0; t < NR; t++) {
            const float4 hin = live[t] ? bf4_load(p.resid + (size_t)rows[t] * E + c0) : make_float4(0, 0, 0, 0);
            // the residual add of the down projection (kEpiBf16Resid), then h as bf16
            v[t][0] = round_bf16(hin.x + round_bf16(acc[t].x));
            v[t][1] = round_bf16(hin.y + round_bf16(acc[t].y));
            v[t][2] = round_bf16(hin.z + round_bf16(acc[t].z));
            v[t][3] = round_bf16(hin.w + round_bf16(acc[t].w));
            if (live[t]) bf4_store(p.out + (size_t)rows[t] * E + c0, v[t][0], v[t][1], v[t][2], v[t][3]);
            float sm = 0.0f;
#pragma unroll
            for (int i = 0; i < 4; i++) sm = __fadd_rn(sm, v[t][i]);
            ms[t] = sm;
        }
        warp_sum_n<NR>(ms);
#pragma unroll
        for (int t = 0; t < NR; t++) {
            ms[t] = __fmul_rn(ms[t], kInvE);
            float sq = 0.0f;
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const float d = __fsub_rn(v[t][i], ms[t]);
                sq = __fadd_rn(sq, __fmul_rn(d, d));
            }
            ms[NR + t] = sq;
        }
        warp_sum_n<NR>(ms + NR);
#pragma unroll
        for (int t = 0; t < NR; t++) {
            const float sd = __fsqrt_rn(__fadd_rn(__fmul_rn(ms[NR + t], kInvE), 1e-5f));
            const float rstd = __frcp_rn(sd);
            if (!live[t]) continue;
            if (lane == 0) p.ln.stdev[rows[t]] = sd;
            float xn[4], y[4];
#pragma unroll
            for (int i = 0; i < 4; i++) {
                xn[i] = __fmul_rn(__fsub_rn(v[t][i], ms[t]), rstd);
                y[i] = __fadd_rn(__fmul_rn(g[i], xn[i]), b[i]);
            }
            bf4_store(p.ln.xNorm + (size_t)rows[t] * E + c0, xn[0], xn[1], xn[2], xn[3]);
            bf4_store(p.ln.out + (size_t)rows[t] * E + c0, y[0], y[1], y[2], y[3]);
        }
    } else {
        float* red = reinterpret_cast<float*>(smem + kRowsRedOff);  // [G][8 virtual warps][dgamma | dbeta]
        const float4 gm = bf4_load(p.gamma + c0);
        const float g[4] = {gm.x, gm.y, gm.z, gm.w};
        float xn[NR][4], dxn[NR][4], s12[2 * NR], rdev[NR];  // s12: sums of dxn (0..NR-1), of dxn x-hat (NR..)
        float dg[4], db[4];
#pragma unroll
        for (int t = 0; t < NR; t++) {
            const float4 x4 = live[t] ? bf4_load(p.xNorm + (size_t)rows[t] * E + c0) : make_float4(0, 0, 0, 0);
            rdev[t] = __frcp_rn(live[t] ? p.stdev[rows[t]] : 1.0f);
            xn[t][0] = x4.x;
            xn[t][1] = x4.y;
            xn[t][2] = x4.z;
            xn[t][3] = x4.w;
            const float dz[4] = {round_bf16(acc[t].x), round_bf16(acc[t].y), round_bf16(acc[t].z),
                                 round_bf16(acc[t].w)};
            if (t % J == 0) {
#pragma unroll
                for (int i = 0; i < 4; i++) dg[i] = db[i] = 0.0f;
            }
            s12[t] = 0.0f;
            s12[NR + t] = 0.0f;
#pragma unroll
            for (int i = 0; i < 4; i++) {
                if (live[t]) {
                    dg[i] = __fadd_rn(dg[i], rbf(__fmul_rn(xn[t][i], dz[i])));
                    db[i] = __fadd_rn(db[i], dz[i]);
                }
                dxn[t][i] = rbf(__fmul_rn(dz[i], g[i]));
                s12[t] = __fadd_rn(s12[t], dxn[t][i]);
                s12[NR + t] = __fadd_rn(s12[NR + t], rbf(__fmul_rn(dxn[t][i], xn[t][i])));
            }
            if (t % J == J - 1 && active) {
                const int pr = warp + 16 * (t / J);  // virtual warp (pr / 8, pr % 8)
                float* dst = red + (size_t)pr * 2 * E;
                *reinterpret_cast<float4*>(dst + c0) = make_float4(dg[0], dg[1], dg[2], dg[3]);
                *reinterpret_cast<float4*>(dst + E + c0) = make_float4(db[0], db[1], db[2], db[3]);
            }
        }
        warp_sum_n<2 * NR>(s12);
#pragma unroll
        for (int t = 0; t < 2 * NR; t++) s12[t] = __fmul_rn(s12[t], kInvE);
#pragma unroll
        for (int t = 0; t < NR; t++) {
            if (!live[t]) continue;
            const float4 rs = bf4_load(p.resid + (size_t)rows[t] * E + c0);
            const float r4[4] = {rs.x, rs.y, rs.z, rs.w};
            float o[4];
#pragma unroll
            for (int i = 0; i < 4; i++)
                o[i] = __fadd_rn(rbf(__fmul_rn(rdev[t], __fsub_rn(__fsub_rn(dxn[t][i], s12[t]),
                                                                   __fmul_rn(xn[t][i], s12[NR + t])))),
                                 r4[i]);
            bf4_store(p.out + (size_t)rows[t] * E + c0, o[0], o[1], o[2], o[3]);
        }
        __syncthreads();
        // one partial per group of RPC rows: its virtual warps' sums in order
        for (int i = threadIdx.x; i < G * 2 * E; i += blockDim.x) {
            const int grp = i / (2 * E), c = i % (2 * E);
            const int first = m0 + 32 * (int)q + grp * RPC;
            if (first >= p.M) continue;
            float sacc = 0.0f;
#pragma unroll
            for (int v = 0; v < 8; v++) sacc = __fadd_rn(sacc, red[((size_t)grp * 8 + v) * 2 * E + c]);
            p.partial[(size_t)(first / RPC) * 2 * E + c] = sacc;
        }
    }
    cluster_sync();  // no CTA leaves while another still reads its partial tile
}

template <bool BMN, int EPI, int RPC>
int launch_rows(const CUtensorMap& ta, const CUtensorMap& tb, const RowsParams& p, int ks, cudaStream_t st) {
    auto kern = k_gemm_rows<BMN, EPI, RPC>;
    static uint64_t attr_done = 0;  // one bit per device
    int dev = 0;
    cudaGetDevice(&dev);
    if (!(attr_done & (1ull << (dev & 63)))) {
        MG_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kRowsSmemOnePerSm));
        attr_done |= 1ull << (dev & 63);
    }
    const int grid = ((p.M + kRowsBM - 1) / kRowsBM) * ks;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)grid);
    cfg.blockDim = dim3(kRowsThreads);
    // a grid that fits the SMs one CTA each asks for more shared memory than
    // two CTAs could share, so that every CTA gets an SM of its own (packed
    // two to an SM, half the SMs would idle: 8.7 against 6.7 us at 4096 rows)
    cfg.dynamicSmemBytes = grid <= num_sms() ? kRowsSmemOnePerSm : kRowsSmem;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = (unsigned)ks;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    MG_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, ta, tb, p));
    return check_launch("k_gemm_rows");
}

int rows_maps(CUtensorMap* ta, CUtensorMap* tb, const void* A, int lda, const void* B, bool b_mn, int ldb, int M,
              int K) {
    int rc = make_tmap_bf16(ta, A, K, M, lda, 128);
    if (rc) return rc;
    return b_mn ? make_tmap_bf16(tb, B, kRowsBN, K, ldb, 64) : make_tmap_bf16(tb, B, K, kRowsBN, ldb, 128);
}

}  // namespace

int gemm_rows_splits(int) { return (int)kRowsCluster; }

bool gemm_rows_supported(int N, int K) { return N == kRowsBN && K > 0 && K % (64 * (int)kRowsCluster) == 0; }

int gemm_rows_resid_layernorm(const void* A, int lda, const void* B, bool b_mn, int ldb, int M, int K, void* h,
                              const LnOutputs& ln, cudaStream_t st) {
    MG_CHECK_ARG(A && B && h && ln.gamma && ln.beta && ln.xNorm && ln.out && ln.stdev, "gemm_rows: null argument");
    MG_CHECK_ARG(M > 0 && gemm_rows_supported(kRowsBN, K), "gemm_rows: needs M > 0, K a multiple of 256");
    const int ks = gemm_rows_splits(K);
    CUtensorMap ta, tb;
    if (int rc = rows_maps(&ta, &tb, A, lda, B, b_mn, ldb, M, K)) return rc;
    RowsParams p{};
    p.M = M;
    p.K = K;
    p.kPer = K / ks;
    p.resid = static_cast<const __nv_bfloat16*>(h);
    p.out = static_cast<__nv_bfloat16*>(h);
    p.ln = ln;
    p.status = status_ptr();
    return b_mn ? launch_rows<true, kRowsResidLN, 32>(ta, tb, p, ks, st)
                : launch_rows<false, kRowsResidLN, 32>(ta, tb, p, ks, st);
}

bool gemm_rows_ln_backward_supported(int M) {
    const int rpc = layernorm_rows_per_part(M);
    return rpc == 8 || rpc == 16 || rpc == 32;
}

int gemm_rows_layernorm_backward(const void* A, int lda, const void* B, bool b_mn, int ldb, int M, int K,
                                 const void* xNorm, const void* gamma, const float* stdev, const void* resid,
                                 void* residOut, float* partial, cudaStream_t st) {
    MG_CHECK_ARG(A && B && xNorm && gamma && stdev && resid && residOut && partial, "gemm_rows: null argument");
    MG_CHECK_ARG(M > 0 && gemm_rows_supported(kRowsBN, K), "gemm_rows: needs M > 0, K a multiple of 256");
    MG_CHECK_ARG(gemm_rows_ln_backward_supported(M),
                 "gemm_rows: the LayerNorm backward partial groups at this row count do not divide 32 rows");
    const int ks = gemm_rows_splits(K);
    CUtensorMap ta, tb;
    if (int rc = rows_maps(&ta, &tb, A, lda, B, b_mn, ldb, M, K)) return rc;
    RowsParams p{};
    p.M = M;
    p.K = K;
    p.kPer = K / ks;
    p.resid = static_cast<const __nv_bfloat16*>(resid);
    p.out = static_cast<__nv_bfloat16*>(residOut);
    p.gamma = static_cast<const __nv_bfloat16*>(gamma);
    p.xNorm = static_cast<const __nv_bfloat16*>(xNorm);
    p.stdev = stdev;
    p.partial = partial;
    p.status = status_ptr();
    switch (layernorm_rows_per_part(M)) {
        case 8:
            return b_mn ? launch_rows<true, kRowsLNBackward, 8>(ta, tb, p, ks, st)
                        : launch_rows<false, kRowsLNBackward, 8>(ta, tb, p, ks, st);
        case 16:
            return b_mn ? launch_rows<true, kRowsLNBackward, 16>(ta, tb, p, ks, st)
                        : launch_rows<false, kRowsLNBackward, 16>(ta, tb, p, ks, st);
        default:
            return b_mn ? launch_rows<true, kRowsLNBackward, 32>(ta, tb, p, ks, st)
                        : launch_rows<false, kRowsLNBackward, 32>(ta, tb, p, ks, st);
    }
}

}  // namespace mg

extern "C" int mg_gemm_rows_resid_layernorm(const void* A_dev, int lda, const void* B_dev, int b_mn_major, int ldb,
                                            int M, int K, void* h_dev, const void* gamma, const void* beta,
                                            void* x_norm, void* ln_out, float* stdev, mg_stream_t stream) {
    const mg::LnOutputs ln{static_cast<const __nv_bfloat16*>(gamma), static_cast<const __nv_bfloat16*>(beta),
                           static_cast<__nv_bfloat16*>(x_norm), static_cast<__nv_bfloat16*>(ln_out), stdev};
    return mg::gemm_rows_resid_layernorm(A_dev, lda, B_dev, b_mn_major != 0, ldb, M, K, h_dev, ln,
                                         reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int mg_gemm_rows_layernorm_backward(const void* A_dev, int lda, const void* B_dev, int b_mn_major, int ldb,
                                               int M, int K, const void* x_norm, const void* gamma,
                                               const float* stdev, const void* resid, void* resid_out,
                                               float* partial, mg_stream_t stream) {
    return mg::gemm_rows_layernorm_backward(A_dev, lda, B_dev, b_mn_major != 0, ldb, M, K, x_norm, gamma, stdev,
                                            resid, resid_out, partial, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int mg_gemm_rows_splits(int K) { return mg::gemm_rows_splits(K); }
