// Tile helpers shared by the kernels that run a residual block of the
// CartPole-sized policy (embed 128, hidden 512) on 4-CTA clusters
// (block_cluster.cu: one block per launch; collect_fused.cu: every block of
// every collect() step in one persistent launch). A 128 x 128 bf16 operand
// tile is two 64-column blocks of 16 KB, 128-byte swizzled, K-major.
#pragma once

#include "gemm_tc.cuh"

namespace mg {

// SW128 K-major byte offset of the 16-byte chunk c (columns 8c .. 8c + 7, c in
// 0..15) of row r of a 128 x 128 bf16 tile: two 64-column blocks of 16 KB.
__device__ __forceinline__ uint32_t sw128_offset(int r, int c) {
    return (uint32_t)((c >> 3) * 16384 + r * 128 + (((c & 7) ^ (r & 7)) << 4));
}

// The first product's accumulator (TMEM columns 0..127) through the ReLU
// (forward) or the V > 0 mask (backward) into the A operand of the second
// product at byte offset a2Off of `smem` (backward: the V tile at maskOff):
// warp w converts rows 32 (w % 4) .., columns 32 (w / 4) .. .
template <bool BWD>
__device__ __forceinline__ void bc_hidden_tile(uint8_t* smem, int a2Off, int maskOff, uint32_t acc, bool valid) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int qd = warp & 3, cc = warp >> 2;
    const int r = qd * 32 + lane;
    float v[32];
    if (valid) {
        tmem_ld32(acc + ((uint32_t)(qd * 32) << 16) + (uint32_t)(cc * 32), v);
    } else {
#pragma unroll
        for (int i = 0; i < 32; i++) v[i] = 0.0f;
    }
#pragma unroll
    for (int j = 0; j < 4; j++) {
        const uint32_t off = sw128_offset(r, cc * 4 + j);
        float x[8];
        if (BWD) {  // kEpiBf16Mask: bf16(acc) * (V > 0)
            const uint4 m = *reinterpret_cast<const uint4*>(smem + maskOff + off);
            const uint32_t mw[4] = {m.x, m.y, m.z, m.w};
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const float m0 = __uint_as_float(mw[i] << 16), m1 = __uint_as_float(mw[i] & 0xffff0000u);
                x[2 * i] = round_bf16(v[8 * j + 2 * i]) * (m0 > 0.0f ? 1.0f : 0.0f);
                x[2 * i + 1] = round_bf16(v[8 * j + 2 * i + 1]) * (m1 > 0.0f ? 1.0f : 0.0f);
            }
        } else {  // kEpiBf16Relu: v = bf16(acc); v > 0 ? v : v * 0
#pragma unroll
            for (int i = 0; i < 8; i++) {
                const float b = round_bf16(v[8 * j + i]);
                x[i] = b > 0.0f ? b : b * 0.0f;
            }
        }
        uint32_t o[4];
#pragma unroll
        for (int i = 0; i < 4; i++) {
            __nv_bfloat162 h2 = __floats2bfloat162_rn(x[2 * i], x[2 * i + 1]);
            o[i] = *reinterpret_cast<uint32_t*>(&h2);
        }
        *reinterpret_cast<uint4*>(smem + a2Off + off) = make_uint4(o[0], o[1], o[2], o[3]);
    }
}

// Eight tcgen05.mma (K = 128) of a 128 x 128 product into TMEM.
template <bool B_MN>
__device__ __forceinline__ void bc_mma(uint32_t d, uint32_t aBase, uint32_t bBase) {
    constexpr uint32_t idesc = idesc_bf16_f32(128, false, B_MN);
#pragma unroll
    for (int kb = 0; kb < 2; kb++)
#pragma unroll
        for (int kk = 0; kk < 4; kk++) {
            const uint64_t ad = smem_desc_sw128(aBase + kb * 16384 + kk * 32, 16, 1024);
            // MN-major B: per 64-row K block two 64-wide N boxes (8 KB apart);
            // K-major B: one 16 KB box of 128 N rows per 64-wide K block
            const uint64_t bd = B_MN ? smem_desc_sw128(bBase + kb * 16384 + kk * 2048, 8192, 1024)
                                     : smem_desc_sw128(bBase + kb * 16384 + kk * 32, 16, 1024);
            tc_mma_bf16(d, ad, bd, idesc, (kb > 0 || kk > 0) ? 1u : 0u);
        }
}

}  // namespace mg
