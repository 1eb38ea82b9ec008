// Host-side runtime shared by the C-ABI entry points: error reporting,
// the per-device status word, TMA descriptor encoding and launch helpers.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <mutex>
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

// Returns the status of expr from the calling function when it is not MG_OK.
#define MG_TRY(expr)               \
    do {                           \
        int mg_rc_ = (expr);       \
        if (mg_rc_) return mg_rc_; \
    } while (0)

// Device address of the status word of the current device (a __device__ int
// in runtime.cu, looked up once per device with cudaGetSymbolAddress).
int* status_ptr();
// The device buffer of the tile kernels' phase trace (mg_set_tile_trace), or
// null when tracing is off (the default).
uint64_t* tile_trace();
// A unique id of the calling thread's current CUDA context (cuCtxGetId; 0
// when none is current or the driver lacks the call). Caches of per-context
// device addresses compare it so that they are looked up again after a
// device reset.
uint64_t current_context_id();
// NCCL communicators aborted by the train() watchdog (ncclCommAbort freed
// them): their handles must not be used or destroyed again. A new
// communicator at the same address is not aborted (comm_forget_aborted).
void comm_mark_aborted(const void* comm);
bool comm_aborted(const void* comm);
bool comm_forget_aborted(const void* comm);  // true if it was aborted
// Executable graphs that captured a communicator's collectives, by the
// address of the field that holds each (a model's train graph). NCCL's
// ncclCommAbort and ncclCommDestroy keep polling until every graph that
// references the communicator is gone, so comm_release_graphs destroys them
// first (a graph still in flight is freed when its launch completes, which
// the abort's flag brings about). Binding the same field again is a no-op.
void comm_bind_graph(const void* comm, cudaGraphExec_t* slot);
void comm_unbind_graph(const void* comm, cudaGraphExec_t* slot);
void comm_release_graphs(const void* comm);
// Serialises the engines' CUDA-graph captures across host threads. A capture
// open in one thread can still be invalidated by what another thread does
// meanwhile (the driver loading a kernel module on a kernel's first use under
// lazy loading, for one): the engine then captures again (at most three
// attempts), with the modules the first attempt loaded already in place.
std::mutex& capture_mutex();
// Streaming multiprocessors of the current device (cached per device).
int num_sms();

// 2D bf16 tensor map with 128-byte swizzle: `inner` contiguous elements per
// row, `outer` rows, `row_stride` elements between rows, box of 64 x box_outer.
int make_tmap_bf16(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer, uint64_t row_stride,
                   uint32_t box_outer);

// Last launch error check (cudaGetLastError) with a message.
int check_launch(const char* what);

// Raises `kern`'s dynamic shared memory limit to `bytes` the first time it is
// launched on the current device. The limit is a per-device attribute, so
// `done` keeps one bit per device (one static object per kernel); concurrent
// callers may both set it, which is harmless.
template <class K>
int smem_limit_once(K kern, int bytes, std::atomic<uint64_t>& done) {
    int dev = 0;
    MG_CUDA_TRY(cudaGetDevice(&dev));
    const uint64_t bit = 1ull << (dev & 63);
    if (done.load(std::memory_order_acquire) & bit) return 0;
    MG_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
    done.fetch_or(bit, std::memory_order_release);
    return 0;
}

}  // namespace mg
