// Row-wise policy kernels of the PPO path (everything that is not a dense
// product): input projection, LayerNorm forward/backward, the categorical and
// Gaussian samplers and PPO losses, GAE, advantage statistics, gradient
// finalisation and Adam.
//
// Rounding follows the reference's store points (bf16 activations, logits,
// dZ; fp32 statistics and accumulators). Products and sums that the reference
// evaluates as separate operations are written with __fmul_rn / __fadd_rn so
// the compiler cannot fuse them; transcendentals are the project-owned
// mg_expf / mg_logf / mg_sincosf (identical on host and device).
#pragma once

#include <cuda_bf16.h>
#include <stdint.h>

#include "metalgym/pdl.cuh"
#include "metalgym/sampling.cuh"
#include "metalgym/detail/ptx.cuh"

namespace mg {

__device__ __forceinline__ __nv_bfloat16 tobf(float x) { return __float2bfloat16_rn(x); }
__device__ __forceinline__ float rbf(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }


}  // namespace mg
