// Host-side runtime shared by the C-ABI entry points: error reporting,
// the per-device status word, TMA descriptor encoding and launch helpers.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "../../include/metalgym_b200.h"

namespace mg {

// Records a message for mg_last_error() and returns `code`.
int fail(int code, const std::string& msg);
// Converts a CUDA error into MG_ERR_CUDA with the call site in the message.
int cuda_fail(cudaError_t e, const char* what);

#define MG_CUDA_TRY(expr)                                   \
    do {                                                    \
        cudaError_t mg_e_ = (expr);                         \
        if (mg_e_ != cudaSuccess) return ::mg::cuda_fail(mg_e_, #expr); \
    } while (0)

#define MG_CHECK_ARG(cond, msg)                                  \
    do {                                                         \
        if (!(cond)) return ::mg::fail(MG_ERR_ARGUMENT, msg);    \
    } while (0)

// Device address of the status word of the current device (a __device__ int
// in runtime.cu, looked up once per device with cudaGetSymbolAddress).
int* status_ptr();
// Streaming multiprocessors of the current device (cached per device).
int num_sms();

// 2D bf16 tensor map with 128-byte swizzle: `inner` contiguous elements per
// row, `outer` rows, `row_stride` elements between rows, box of 64 x box_outer.
int make_tmap_bf16(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer, uint64_t row_stride,
                   uint32_t box_outer);

// Last launch error check (cudaGetLastError) with a message.
int check_launch(const char* what);

}  // namespace mg
