// Programmatic dependent launch: every kernel of the hot path is launched
// with programmatic stream serialisation, so inside a CUDA graph the next
// kernel's CTAs are scheduled (and run their prologue) while the current
// kernel drains. Each kernel signals its dependents at its start
// (mg_pdl_trigger) and waits for its predecessor's memory before its first
// dependent read (mg_pdl_wait). Both are no-ops for a kernel launched
// without the attribute.
#pragma once

#include <cuda_runtime.h>

#include <utility>

__device__ __forceinline__ void mg_pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void mg_pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

template <typename... KArgs, typename... Args>
inline cudaError_t mg_launch(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                             Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

#define MG_LAUNCH(kernel, grid, block, smem, stream, ...) \
    mg_launch(kernel, dim3(grid), dim3(block), (size_t)(smem), (stream), __VA_ARGS__)
