// Common macros for code that compiles both as CUDA device code and as plain
// host C++ (the CPU oracle and host-side unit tests include the same headers).
#pragma once

#include <stdint.h>

#if defined(__CUDACC__)
#define MG_HD __host__ __device__
#define MG_DEVICE_CODE 1
#else
#define MG_HD
#endif

#if defined(__CUDA_ARCH__)
#define MG_ON_DEVICE 1
#endif

// Single-precision multiply and add that the compiler may never contract into
// an FMA. Environment code uses them wherever an expression of the form
// `a + b * c` must round twice, as the Metal code it mirrors does when it is
// compiled as host C++ with -ffp-contract=off.
MG_HD inline float mg_fmul(float a, float b) {
#if defined(__CUDA_ARCH__)
    return __fmul_rn(a, b);
#else
    return a * b;
#endif
}
MG_HD inline float mg_fadd(float a, float b) {
#if defined(__CUDA_ARCH__)
    return __fadd_rn(a, b);
#else
    return a + b;
#endif
}
