/*
 * metalgym_b200 C ABI: the boundary between host code (the C++ drop-in
 * headers in include/metalgym/, Python via ctypes, or any FFI) and the
 * sm_100a CUDA kernels of the MetalGym hot path.
 *
 * Conventions
 *   - every function returns MG_OK (0) or an MG_ERR_* code; mg_last_error()
 *     gives the message of the last failure on the calling thread;
 *   - pointers named *_dev are device pointers owned by the caller, unless a
 *     function says it allocates; bf16 data is passed as void* (2-byte
 *     elements, round-to-nearest-even storage);
 *   - every launch takes a stream (a cudaStream_t; NULL = legacy default
 *     stream) and is asynchronous unless documented otherwise;
 *   - device-side waits are bounded; a kernel that gives up records a code in
 *     the device status word (mg_device_status) instead of hanging.
 *
 * Each entry point names the reference interface it replaces, as
 * file:line inside the MetalGym source tree. The reference binds kernels by
 * name through Metal pipelines (model/ppo.h:311-330, gym.h:43-64); here the
 * same kernels are plain C functions.
 */
#ifndef METALGYM_B200_H
#define METALGYM_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MG_VERSION 1

typedef struct CUstream_st* mg_stream_t;

enum mg_status_code {
    MG_OK = 0,
    MG_ERR_ARGUMENT = 1,       /* invalid size, alignment or pointer */
    MG_ERR_CUDA = 2,           /* a CUDA runtime / driver call failed */
    MG_ERR_UNSUPPORTED = 3,    /* configuration not supported by this build */
    MG_ERR_DEVICE = 4,         /* a kernel recorded a device-side error (timeout) */
    MG_ERR_NOT_FOUND = 5,      /* unknown environment kernel name */
    MG_ERR_COMM = 6            /* NCCL failure, or a collective that timed out */
};

/* ---------------------------------------------------------------- runtime */

/* Message of the last failing call on this thread ("" if none). */
const char* mg_last_error(void);
/* ABI version (MG_VERSION). */
int mg_version(void);
/* Reads the device status word of the current device into *status (0 = no
 * error; otherwise the first device-side error code recorded) and clears it
 * if `clear` is non-zero. Synchronous. Replaces the command-buffer error check
 * of model/ppo.h:507-515. */
int mg_device_status(int clear, int* status);

/* ---------------------------------------------------------------- GEMM */

enum mg_gemm_epilogue {
    MG_EPI_BF16 = 0,       /* out = bf16(acc) */
    MG_EPI_BF16_RELU = 1,  /* v = bf16(acc); out = v > 0 ? v : v * 0 */
    MG_EPI_BF16_RESID = 2, /* out = bf16(aux + bf16(acc)) */
    MG_EPI_BF16_MASK = 3,  /* out = bf16(acc) * (aux > 0) */
    MG_EPI_F32 = 4         /* out (fp32) = acc; with splits > 1, split z writes
                              out + z * M * ldo (partial sums) */
};

/* out[M x N] = opA(A) * opB(B) with bf16 operands and fp32 accumulation on
 * the tcgen05 tensor cores. A is K-major ([M][lda], K contiguous) or, with
 * a_mn_major, MN-major ([K][lda], M contiguous); B is K-major ([N][ldb]) or
 * MN-major ([K][ldb], N contiguous). Leading dimensions are in elements and
 * multiples of 8; bases 16-byte aligned; N a multiple of 32; K split into
 * `splits` contiguous ranges (MG_EPI_F32 only). aux is bf16 [M][ldaux].
 * Replaces the MetalPerformancePrimitives matmul2d kernels mlpForwardOne/Two,
 * mlpBackwardOne/Two/Weights (model/mlp.metal:18-208), linearForward,
 * linearBackward, linearBackwardDw (model/linear.metal:17-93). */
int mg_gemm_bf16(const void* A_dev, int a_mn_major, int lda, const void* B_dev, int b_mn_major, int ldb, int M,
                 int N, int K, int epilogue, void* out_dev, int ldo, const void* aux_dev, int ldaux, int splits,
                 mg_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* METALGYM_B200_H */
