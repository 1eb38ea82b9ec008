// Persistent tcgen05 GEMM for large problems: one CTA per SM walks the
// output tiles (and K splits) in a fixed round-robin order, with its
// accumulator double-buffered in tensor memory so that the epilogue of one
// tile overlaps the main loop of the next.
//
// Warp roles (192 threads):
//   warp 0     TMA producer: A and B tiles into a STAGES-deep shared ring
//   warp 1     MMA issuer: 128 x BN x 16 tcgen05.mma into accumulator a
//              (columns a * BN of a 2 * BN column allocation), commit to
//              tfull[a] when the tile's K range is done
//   warps 2-5  epilogue: warp w reads TMEM lanes 32 (w % 4) .. + 31, i.e.
//              output rows 32 (w % 4) + lane of the tile, applies the
//              epilogue and arrives on tempty[a]. bf16 outputs go through a
//              per-warp shared-memory slab (32 rows x the warp's columns,
//              128-byte swizzled; half of them per round for the epilogues
//              without aux at 256-wide tiles) that one lane stores with TMA;
//              the aux operand of the residual and mask epilogues is loaded
//              into the same slab by TMA first.
//              fp32 split-K partials are stored directly.
//
// Units are numbered with the N tile fastest, so the CTAs working at the same
// time share A tiles through L2. Same operand layouts, epilogues and
// rounding as gemm_tc_kernel; every wait is bounded (ptx.cuh).
#pragma once

#include "gemm_tc.cuh"

namespace mg {

template <int BN, int EPI>
struct PersistShape {
    static constexpr int BM = 128;
    static constexpr int BK = 64;
    static constexpr bool STAGED = EPI != kEpiF32;         // bf16 output through shared memory + TMA
    // epilogue warps: 8 for the staged elementwise epilogues (two per TMEM
    // lane quadrant, each on half of the tile's columns: with four the
    // epilogue, not the tensor core, set the pace), 4 where a thread needs its
    // whole row (the LayerNorm epilogue) or stores fp32 directly
    static constexpr int EW = (STAGED && EPI != kEpiResidLN) ? 8 : 4;
    static constexpr int EPI_COLS = BN * 4 / EW;             // columns per epilogue warp
    static constexpr int THREADS = 64 + 32 * EW;
    // the elementwise epilogues without an aux operand at 256-wide tiles
    // store each warp's columns in two rounds through a half-size slab, which
    // leaves room for a fourth TMA stage (more operand bytes in flight)
    static constexpr bool HALF_SLAB = STAGED && EW == 8 && BN == 256 && (EPI == kEpiBf16 || EPI == kEpiBf16Relu);
    static constexpr int SLAB_COLS = HALF_SLAB ? EPI_COLS / 2 : EPI_COLS;  // columns the slab holds
    static constexpr int ROUNDS = EPI_COLS / SLAB_COLS;
    static constexpr int SLAB = 32 * SLAB_COLS * 2;          // per epilogue warp: 32 rows x SLAB_COLS bf16
    static constexpr int STAGES = STAGED ? (BN == 256 ? (HALF_SLAB ? 4 : 3) : 4) : (BN == 256 ? 4 : 6);
    static constexpr int A_BYTES = BM * BK * 2;
    static constexpr int B_BYTES = BN * BK * 2;
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
    static constexpr int SLAB_OFF = STAGES * STAGE_BYTES;
    static constexpr int BAR_OFF = SLAB_OFF + (STAGED ? EW * SLAB : 0);
    static constexpr int GB_OFF = BAR_OFF + 256;  // kEpiResidLN: gamma, beta as fp32
    static constexpr int TMEM_COLS = 2 * BN;      // two accumulators (256 or 512 columns)
    static constexpr int SMEM_BYTES = GB_OFF + (EPI == kEpiResidLN ? 2 * BN * 4 : 0) + 1024 /*align*/;
};

// Byte offset of 16-byte chunk k (8 bf16, 0..BN/8-1) of slab row r (0..31)
// in a slab of 64-column boxes of 32 rows x 128 bytes, 128-byte swizzled.
__device__ __forceinline__ uint32_t slab_offset(int r, int k) {
    return (uint32_t)((k >> 3) * 4096 + r * 128 + (((k & 7) ^ (r & 7)) << 4));
}

// One 32-column chunk of one output row: epilogue and store.
template <int EPI>
__device__ __forceinline__ void epilogue_chunk(const GemmParams& p, int row, int col, int z, float* v) {
    if (EPI == kEpiF32) {
        float* o = static_cast<float*>(p.out) + (size_t)z * p.M * p.ldo + (size_t)row * p.ldo + col;
        float4* o4 = reinterpret_cast<float4*>(o);
#pragma unroll
        for (int i = 0; i < 8; i++) o4[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
    } else {
        __nv_bfloat16* o = static_cast<__nv_bfloat16*>(p.out) + (size_t)row * p.ldo + col;
        if (EPI == kEpiBf16Relu) {
#pragma unroll
            for (int i = 0; i < 32; i++) {
                const float r = round_bf16(v[i]);
                v[i] = r > 0.0f ? r : r * 0.0f;
            }
        } else if (EPI == kEpiBf16Resid) {
            float a[32];
            load_bf16x32(p.aux + (size_t)row * p.ldaux + col, a);
#pragma unroll
            for (int i = 0; i < 32; i++) v[i] = a[i] + round_bf16(v[i]);
        } else if (EPI == kEpiBf16Mask) {
            float a[32];
            load_bf16x32(p.aux + (size_t)row * p.ldaux + col, a);
#pragma unroll
            for (int i = 0; i < 32; i++) v[i] = round_bf16(v[i]) * (a[i] > 0.0f ? 1.0f : 0.0f);
        }
        store_bf16x32(o, v);
    }
}

// Output, aux and LayerNorm-output tensor maps of the staged epilogue (boxes
// of 64 columns x 32 rows).
struct EpiMaps {
    CUtensorMap out, aux, ln;
};

template <int BN, bool A_MN, bool B_MN, int EPI>
__global__ void __launch_bounds__(PersistShape<BN, EPI>::THREADS, 1)
    gemm_tc_persistent(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                       const __grid_constant__ EpiMaps em, const GemmParams p) {
    using S = PersistShape<BN, EPI>;
    constexpr bool HAS_AUX = EPI == kEpiBf16Resid || EPI == kEpiBf16Mask || EPI == kEpiResidLN;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + S::BAR_OFF);
    uint64_t* empty = full + S::STAGES;
    uint64_t* tfull = empty + S::STAGES;  // [2]
    uint64_t* tempty = tfull + 2;         // [2]
    uint64_t* done = tempty + 2;
    uint64_t* auxFull = done + 1;         // [EW], one per epilogue warp
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(auxFull + S::EW);
    float* s_gb = reinterpret_cast<float*>(smem + S::GB_OFF);  // kEpiResidLN: gamma[BN], beta[BN]

    mg_pdl_trigger();
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int tilesMN = p.tilesM * p.tilesN;
    const int units = tilesMN * p.splits;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S::STAGES; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int a = 0; a < 2; a++) {
            mbar_init(&tfull[a], 1);
            mbar_init(&tempty[a], S::EW);  // one arrival per epilogue warp
        }
        mbar_init(done, 1);
        for (int w = 0; w < S::EW; w++) mbar_init(&auxFull[w], 1);
        fence_barrier_init();
        prefetch_tensormap(&tmA);
        prefetch_tensormap(&tmB);
        if (S::STAGED) prefetch_tensormap(&em.out);
        if (HAS_AUX) prefetch_tensormap(&em.aux);
        if (EPI == kEpiResidLN) prefetch_tensormap(&em.ln);
    }
    if (EPI == kEpiResidLN) {
        for (int i = threadIdx.x; i < BN; i += blockDim.x) {
            s_gb[i] = __bfloat162float(p.ln.gamma[i]);
            s_gb[BN + i] = __bfloat162float(p.ln.beta[i]);
        }
    }
    if (warp == 2) {
        tmem_alloc(tmem_slot, S::TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    mg_pdl_wait();  // operands and aux come from the previous kernel

    if (warp == 0) {
        if (lane == 0) {
            // ---- TMA producer
            int it = 0;
            bool ok = true;
            for (int u = blockIdx.x; u < units && ok; u += gridDim.x) {
                const int nt = u % p.tilesN;
                const int mt = (u / p.tilesN) % p.tilesM;
                const int z = u / tilesMN;
                const int m0 = mt * S::BM, n0 = nt * BN;
                const int kBegin = z * p.kPerSplit;
                const int kEnd = min(p.K, kBegin + p.kPerSplit);
                for (int k0 = kBegin; k0 < kEnd; k0 += S::BK) {
                    const int s = it % S::STAGES;
                    const uint32_t ph = (it / S::STAGES) & 1;
                    if (!mbar_wait(&empty[s], ph ^ 1, p.status, kDevTimeoutEmpty)) {
                        ok = false;
                        break;
                    }
                    it++;
                    uint8_t* sA = smem + s * S::STAGE_BYTES;
                    uint8_t* sB = sA + S::A_BYTES;
                    mbar_arrive_expect_tx(&full[s], S::STAGE_BYTES);
                    if (A_MN) {
                        tma_load_2d(sA, &tmA, m0, k0, &full[s]);
                        tma_load_2d(sA + 8192, &tmA, m0 + 64, k0, &full[s]);
                    } else {
                        tma_load_2d(sA, &tmA, k0, m0, &full[s]);
                    }
                    if (B_MN) {
#pragma unroll
                        for (int j = 0; j < BN / 64; j++) tma_load_2d(sB + j * 8192, &tmB, n0 + 64 * j, k0, &full[s]);
                    } else {
                        tma_load_2d(sB, &tmB, k0, n0, &full[s]);
                    }
                }
            }
            // Drain: every issued copy has landed before the CTA can exit.
            for (int k = it - S::STAGES < 0 ? 0 : it - S::STAGES; k < it; k++)
                mbar_wait(&full[k % S::STAGES], (k / S::STAGES) & 1, p.status, kDevTimeoutFull);
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ---- MMA issuer
            constexpr uint32_t idesc = idesc_bf16_f32(BN, A_MN, B_MN);
            int it = 0, t = 0;
            bool ok = true;
            for (int u = blockIdx.x; u < units && ok; u += gridDim.x, t++) {
                const int z = u / tilesMN;
                const int kBegin = z * p.kPerSplit;
                const int kEnd = min(p.K, kBegin + p.kPerSplit);
                const int a = t & 1;
                // the epilogue has emptied accumulator a (its previous use was tile t - 2)
                if (!mbar_wait(&tempty[a], ((t >> 1) & 1) ^ 1, p.status, kDevTimeoutEmpty)) break;
                tc_fence_after();
                const uint32_t acc = tmem + (uint32_t)(a * BN);
                bool first = true;
                for (int k0 = kBegin; k0 < kEnd; k0 += S::BK) {
                    const int s = it % S::STAGES;
                    const uint32_t ph = (it / S::STAGES) & 1;
                    if (!mbar_wait(&full[s], ph, p.status, kDevTimeoutFull)) {
                        ok = false;
                        break;
                    }
                    it++;
                    tc_fence_after();
                    const uint32_t aBase = smem_u32(smem + s * S::STAGE_BYTES);
                    const uint32_t bBase = aBase + S::A_BYTES;
#pragma unroll
                    for (int kk = 0; kk < 4; kk++) {
                        const uint64_t ad = A_MN ? smem_desc_sw128(aBase + kk * 2048, 8192, 1024)
                                                 : smem_desc_sw128(aBase + kk * 32, 16, 1024);
                        const uint64_t bd = B_MN ? smem_desc_sw128(bBase + kk * 2048, 8192, 1024)
                                                 : smem_desc_sw128(bBase + kk * 32, 16, 1024);
                        tc_mma_bf16(acc, ad, bd, idesc, first ? 0u : 1u);
                        first = false;
                    }
                    tc_commit(&empty[s]);
                }
                if (ok) tc_commit(&tfull[a]);
            }
            // Always commit: `done` then covers every MMA issued, also after a
            // timeout, so TMEM is never freed under a running MMA.
            tc_commit(done);
        }
    } else {
        // ---- epilogue: thread owns row 32 (warp % 4) + lane of each tile, in
        // columns [h EPI_COLS, (h + 1) EPI_COLS) (h: which of the quadrant's warps)
        const int q = warp & 3;
        const int e = warp - 2;
        const int hc = (e / 4) * S::EPI_COLS;
        uint8_t* slab = smem + S::SLAB_OFF + e * S::SLAB;
        int t = 0;
        int auxWaited = 0;  // aux loads this warp has seen land
        for (int u = blockIdx.x; u < units; u += gridDim.x, t++) {
            const int nt = u % p.tilesN;
            const int mt = (u / p.tilesN) % p.tilesM;
            const int z = u / tilesMN;
            const int a = t & 1;
            const int row0 = mt * S::BM + q * 32;  // first row of this warp's slab
            const int n0 = nt * BN;
            if (S::STAGED && lane == 0) {
                bulk_wait_read<0>();  // the previous tile's store has read the slab
                if (HAS_AUX) {
                    mbar_arrive_expect_tx(&auxFull[e], S::SLAB);
#pragma unroll
                    for (int j = 0; j < S::EPI_COLS / 64; j++)
                        tma_load_2d(slab + j * 4096, &em.aux, n0 + hc + 64 * j, row0, &auxFull[e]);
                }
            }
            __syncwarp();
            if (!mbar_wait_warp(&tfull[a], (t >> 1) & 1, p.status, kDevTimeoutDone)) break;
            if (HAS_AUX) {
                if (!mbar_wait_warp(&auxFull[e], t & 1, p.status, kDevTimeoutFull)) break;
                auxWaited = t + 1;
            }
            tc_fence_after();
            const int row = row0 + lane;
            const uint32_t acc = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(a * BN + hc);
            // TMA store of slab round r (columns hc + r SLAB_COLS ..) of the tile
            auto storeRound = [&](int r) {
                fence_async_smem();
                __syncwarp();
                if (lane == 0) {
#pragma unroll
                    for (int j = 0; j < S::SLAB_COLS / 64; j++)
                        if (n0 + hc + r * S::SLAB_COLS + 64 * j < p.N && row0 < p.M)
                            tma_store_2d(&em.out, n0 + hc + r * S::SLAB_COLS + 64 * j, row0, slab + j * 4096);
                    bulk_commit();
                }
            };
            constexpr int kChunksPerRound = S::SLAB_COLS / 32;
#pragma unroll 1
            for (int c = 0; c < S::EPI_COLS / 32; c++) {
                if (S::STAGED && S::ROUNDS > 1 && c > 0 && c % kChunksPerRound == 0) {
                    // the finished round out, and the slab free for the next one
                    storeRound(c / kChunksPerRound - 1);
                    if (lane == 0) bulk_wait_read<0>();
                    __syncwarp();
                }
                const int col = n0 + hc + c * 32;
                float v[32];
                tmem_ld32(acc + (uint32_t)(c * 32), v);
                if (c == S::EPI_COLS / 32 - 1) {
                    // the whole accumulator is in registers or stored: release it
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&tempty[a]);
                }
                if (!S::STAGED) {
                    if (row < p.M && col < p.N) epilogue_chunk<EPI>(p, row, col, z, v);
                    continue;
                }
#pragma unroll
                for (int k = 0; k < 4; k++) {
                    uint4* cell = reinterpret_cast<uint4*>(slab + slab_offset(lane, (c % kChunksPerRound) * 4 + k));
                    float x[8];
#pragma unroll
                    for (int i = 0; i < 8; i++) x[i] = v[8 * k + i];
                    if (EPI == kEpiBf16Relu) {
#pragma unroll
                        for (int i = 0; i < 8; i++) {
                            const float r = round_bf16(x[i]);
                            x[i] = r > 0.0f ? r : r * 0.0f;
                        }
                    } else if (HAS_AUX) {  // residual, LayerNorm-ending residual, mask
                        const uint4 w = *cell;
                        const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
                        float au[8];
#pragma unroll
                        for (int i = 0; i < 4; i++) {
                            au[2 * i] = __uint_as_float(ww[i] << 16);
                            au[2 * i + 1] = __uint_as_float(ww[i] & 0xffff0000u);
                        }
#pragma unroll
                        for (int i = 0; i < 8; i++)
                            x[i] = EPI == kEpiBf16Mask ? round_bf16(x[i]) * (au[i] > 0.0f ? 1.0f : 0.0f)
                                                       : au[i] + round_bf16(x[i]);
                    }
                    uint32_t o[4];
#pragma unroll
                    for (int i = 0; i < 4; i++) {
                        __nv_bfloat162 h2 = __floats2bfloat162_rn(x[2 * i], x[2 * i + 1]);
                        o[i] = *reinterpret_cast<uint32_t*>(&h2);
                    }
                    *cell = make_uint4(o[0], o[1], o[2], o[3]);
                }
            }
            if (S::STAGED) storeRound(S::ROUNDS - 1);
            if constexpr (EPI == kEpiResidLN) {
                // the LayerNorm of the warp's 32 rows now in the slab: one row
                // across the lanes at a time (lane l: columns l VPT ..), eight
                // rows side by side, in k_layernorm_forward's arithmetic and
                // summation order (bit-identical to it)
                constexpr int VPT = BN / 32;
                float g[VPT], bb[VPT];
#pragma unroll
                for (int j = 0; j < VPT; j++) {
                    g[j] = s_gb[lane * VPT + j];
                    bb[j] = s_gb[BN + lane * VPT + j];
                }
                // lane l's VPT columns of a slab row: a whole 16-byte chunk
                // (BN 256) or half of one (BN 128)
                const uint32_t cellOff = VPT == 8 ? 0u : (uint32_t)(lane & 1) * 8u;
                const int cellChunk = VPT == 8 ? lane : lane >> 1;
#pragma unroll 1
                for (int r0 = 0; r0 < 32; r0 += 8) {
                    float v[8][VPT], mean[8], sq[8];
#pragma unroll
                    for (int u = 0; u < 8; u++) {
                        const uint8_t* cell = slab + slab_offset(r0 + u, cellChunk) + cellOff;
                        uint32_t w[VPT / 2];
                        if constexpr (VPT == 8) {
                            const uint4 x = *reinterpret_cast<const uint4*>(cell);
                            w[0] = x.x;
                            w[1] = x.y;
                            w[2] = x.z;
                            w[3] = x.w;
                        } else {
                            const uint2 x = *reinterpret_cast<const uint2*>(cell);
                            w[0] = x.x;
                            w[1] = x.y;
                        }
                        float sm = 0.0f;
#pragma unroll
                        for (int i = 0; i < VPT / 2; i++) {
                            v[u][2 * i] = __uint_as_float(w[i] << 16);
                            v[u][2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
                        }
#pragma unroll
                        for (int j = 0; j < VPT; j++) sm = __fadd_rn(sm, v[u][j]);
                        mean[u] = sm;
                    }
                    warp_sum_n<8>(mean);
#pragma unroll
                    for (int u = 0; u < 8; u++) mean[u] = __fmul_rn(mean[u], 1.0f / BN);  // exact: BN is a power of two
#pragma unroll
                    for (int u = 0; u < 8; u++) {
                        sq[u] = 0.0f;
#pragma unroll
                        for (int j = 0; j < VPT; j++) {
                            const float d = __fsub_rn(v[u][j], mean[u]);
                            sq[u] = __fadd_rn(sq[u], __fmul_rn(d, d));
                        }
                    }
                    warp_sum_n<8>(sq);
                    // lnOut replaces h in the slab: the h store must have read it
                    if (r0 == 0) {
                        if (lane == 0) bulk_wait_read<0>();
                        __syncwarp();
                    }
#pragma unroll
                    for (int u = 0; u < 8; u++) {
                        const int rowU = row0 + r0 + u;
                        const float sd = __fsqrt_rn(__fadd_rn(__fmul_rn(sq[u], 1.0f / BN), 1e-5f));
                        const float rstd = __frcp_rn(sd);  // = __fdiv_rn(1, sd): both correctly rounded
                        if (lane == 0 && rowU < p.M) p.ln.stdev[rowU] = sd;
                        uint32_t xw[VPT / 2], yw[VPT / 2];
#pragma unroll
                        for (int i = 0; i < VPT / 2; i++) {
                            const float x0 = __fmul_rn(__fsub_rn(v[u][2 * i], mean[u]), rstd);
                            const float x1 = __fmul_rn(__fsub_rn(v[u][2 * i + 1], mean[u]), rstd);
                            __nv_bfloat162 xh = __floats2bfloat162_rn(x0, x1);
                            __nv_bfloat162 yh = __floats2bfloat162_rn(__fadd_rn(__fmul_rn(g[2 * i], x0), bb[2 * i]),
                                                                      __fadd_rn(__fmul_rn(g[2 * i + 1], x1), bb[2 * i + 1]));
                            xw[i] = *reinterpret_cast<uint32_t*>(&xh);
                            yw[i] = *reinterpret_cast<uint32_t*>(&yh);
                        }
                        uint8_t* cell = slab + slab_offset(r0 + u, cellChunk) + cellOff;
                        __nv_bfloat16* xdst = p.ln.xNorm + (size_t)rowU * BN + lane * VPT;
                        if constexpr (VPT == 8) {
                            if (rowU < p.M)
                                *reinterpret_cast<uint4*>(xdst) = make_uint4(xw[0], xw[1], xw[2], xw[3]);
                            *reinterpret_cast<uint4*>(cell) = make_uint4(yw[0], yw[1], yw[2], yw[3]);
                        } else {
                            if (rowU < p.M) *reinterpret_cast<uint2*>(xdst) = make_uint2(xw[0], xw[1]);
                            *reinterpret_cast<uint2*>(cell) = make_uint2(yw[0], yw[1]);
                        }
                    }
                }
                fence_async_smem();
                __syncwarp();
                if (lane == 0) {
#pragma unroll
                    for (int j = 0; j < BN / 64; j++)
                        if (row0 < p.M) tma_store_2d(&em.ln, 64 * j, row0, slab + j * 4096);
                    bulk_commit();
                }
            }
        }
        // after a timeout: the aux load issued for tile t has landed before the CTA exits
        if (HAS_AUX && lane == 0 && auxWaited < t + 1 && t < (units - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x)
            mbar_wait(&auxFull[e], t & 1, p.status, kDevTimeoutFull);
        if (S::STAGED && lane == 0) bulk_wait<0>();  // every store complete before the CTA exits
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 2) {
        mbar_wait(done, 0, p.status, kDevTimeoutDone);
        tc_fence_after();
        tmem_dealloc(tmem, S::TMEM_COLS);
    }
}

}  // namespace mg
