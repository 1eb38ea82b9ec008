// Tile helpers of the tcgen05 policy kernels, in the public device headers
// because environment translation units instantiate the fused collect kernel
// (include/metalgym/detail/collect_fused.cuh) for their own environments.
//
//   round_bf16          x rounded to bf16 and back (the reference's bf16 stores)
//   kRows*              the 128-row tile of the cluster kernels: 4 CTAs, 512
//                       threads each, a 128-wide fp32 tile of 64 KB
//   tile_offset, bf4_*, rows_tmem_to_tile   the swizzled fp32 tile in shared
//                       memory and 4-wide bf16 row access
//   sw128_offset, bc_hidden_tile, bc_mma    the 128 x 128 bf16 operand tiles of
//                       a residual block (embed 128, hidden 512) on a 4-CTA
//                       cluster: two 64-column blocks of 16 KB, 128-byte
//                       swizzled, K-major
#pragma once

#include <cuda_bf16.h>
#include <stdint.h>

#include "ptx.cuh"

namespace mg {

__device__ __forceinline__ float round_bf16(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

constexpr int kRowsBM = 128;
constexpr int kRowsBN = 128;                 // the output width (the embedding)
constexpr uint32_t kRowsCluster = 4;         // CTAs per cluster; each ends 32 rows of the tile
// 16 warps: all copy an accumulator out of TMEM (quadrant w % 4, columns
// 32 (w / 4) ..), and two rows per warp give the row epilogue enough warps to
// hide its latency (four warps of eight rows each were latency bound)
constexpr int kRowsThreads = 512;
constexpr int kRowsTile = kRowsBM * kRowsBN * 4;        // the fp32 tile, 64 KB

// Byte offset of the 16-byte column chunk k (columns 4k..4k+3) of tile row r in
// an fp32 tile: rows of 512 bytes, chunks XOR-swizzled by the row, so a warp
// writing chunk k of 32 rows and a warp reading a whole row are both free of
// bank conflicts.
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

// The 128 x 128 fp32 accumulator at TMEM address acc into the fp32 tile at
// `tile` (zeros when !valid): every one of the 16 warps copies 32 rows x 32
// columns.
__device__ __forceinline__ void rows_tmem_to_tile(uint8_t* tile, uint32_t acc, bool valid) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int qd = warp & 3, cc = warp >> 2;
    const int tr = qd * 32 + lane;
    float v[32];
    if (valid) {
        tmem_ld32(acc + ((uint32_t)(qd * 32) << 16) + (uint32_t)(cc * 32), v);
    } else {
#pragma unroll
        for (int i = 0; i < 32; i++) v[i] = 0.0f;
    }
#pragma unroll
    for (int k = 0; k < 8; k++)
        *reinterpret_cast<float4*>(tile + tile_offset(tr, cc * 8 + k)) =
            make_float4(v[4 * k], v[4 * k + 1], v[4 * k + 2], v[4 * k + 3]);
}

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
