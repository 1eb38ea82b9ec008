// State shared by the passes of the 4-CTA cluster kernels over one 128-row
// tile (block_cluster.cuh, head_tail.cuh): each pass is a device function
// that a standalone kernel runs once, and the minibatch kernel
// (minibatch_tiles.cu) runs back to back, one pass per layer, without leaving
// the SMs.
//
// A pass uses up to four mbarriers (two TMA "full" barriers, two MMA commit
// barriers), each completing exactly one phase per pass, and a TMEM
// allocation of 512 columns made once per kernel. `ph` holds the parity every
// barrier waits for next; a pass flips the bits of the barriers it used.
// Once a bounded wait has given up (the error is in the device status word),
// `alive` is cleared and later passes of a merged kernel issue no copies or
// products and wait for nothing, but still reach every barrier of the
// cluster; the kernel's teardown then waits, bounded, for the copies and
// products still in flight before it frees TMEM.
#pragma once

#include <stdint.h>

#include "metalgym/detail/ptx.cuh"

namespace mg {

enum TileBar : int { kTbFull1 = 0, kTbFull2 = 1, kTbMma1 = 2, kTbMma2 = 3, kTbFin = 4, kTbCount = 5 };

struct TilePass {
    uint64_t* bars;          // kTbCount mbarriers (count 1 each)
    uint32_t tmem;           // TMEM base of the CTA's 512-column allocation
    uint32_t ph;             // bit b: the parity barrier b waits for next
    volatile int* alive;     // shared: 0 once a wait of this CTA gave up
    bool merged;             // part of the minibatch kernel (TMEM outlives the pass)
    // thread 0, merged kernels: the parity of the last load issued on each
    // full barrier (bit b), and which barriers have a load issued at all
    uint32_t lastLoad, loaded;
    // phase trace (mg_set_tile_trace; null: off): thread 0 of each CTA
    // writes %globaltimer at every tp_mark into trace[blockIdx.x][mark]
    uint64_t* trace;
    int mark;

    __device__ __forceinline__ uint64_t* bar(int b) const { return bars + b; }
    __device__ __forceinline__ uint32_t parity(int b) const { return (ph >> b) & 1u; }
    __device__ __forceinline__ void flip(int b) { ph ^= 1u << b; }
    __device__ __forceinline__ bool ok() const { return *alive != 0; }
    // thread 0, before the copies of a full barrier's phase
    __device__ __forceinline__ void issuing(int b) {
        lastLoad = (lastLoad & ~(1u << b)) | (parity(b) << b);
        loaded |= 1u << b;
    }
};

constexpr int kTileTraceSlots = 64;

// A phase boundary of the trace: every thread counts it, thread 0 stamps it.
__device__ __forceinline__ void tp_mark(TilePass& t) {
    if (t.trace && threadIdx.x == 0 && t.mark < kTileTraceSlots)
        t.trace[(size_t)blockIdx.x * kTileTraceSlots + t.mark] = globaltimer();
    t.mark++;
}

// Bounded wait of one thread for barrier b's current phase; false once the
// CTA gave up (then without waiting).
__device__ __forceinline__ bool tp_wait(TilePass& t, int b, int* status, int code) {
    if (!t.ok()) return false;
    const bool r = mbar_wait(t.bar(b), t.parity(b), status, code);
    if (!r) *t.alive = 0;
    return r;
}

// The same for a whole warp, with a warp-uniform result.
__device__ __forceinline__ bool tp_wait_warp(TilePass& t, int b, int* status, int code) {
    const int go = __shfl_sync(0xffffffffu, t.ok() ? 1 : 0, 0);
    if (!go) return false;
    const bool r = mbar_wait_warp(t.bar(b), t.parity(b), status, code);
    if (!r && (threadIdx.x & 31) == 0) *t.alive = 0;
    return r;
}

// Between two passes of a merged kernel: this thread's global stores (and
// completed TMA stores) ordered before the async-proxy (TMA) loads of the next
// pass in any CTA of the cluster, its TMEM loads before the next products,
// then the cluster barrier.
__device__ __forceinline__ void tp_pass_boundary() {
    asm volatile("fence.proxy.async.global;" ::: "memory");
    tc_fence_before();
    cluster_sync();
    tc_fence_after();
}

// Start of a kernel over tiles: barrier init, the TMEM allocation (512
// columns in a merged kernel; a standalone kernel allocates what its one pass
// uses and frees it inside the pass).
__device__ __forceinline__ TilePass tp_setup(uint8_t* barMem, uint32_t tmemCols, bool merged) {
    TilePass t;
    t.bars = reinterpret_cast<uint64_t*>(barMem);
    t.alive = reinterpret_cast<volatile int*>(barMem + 8 * kTbCount + 8);
    uint32_t* slot = reinterpret_cast<uint32_t*>(barMem + 8 * kTbCount);
    if (threadIdx.x == 0) {
        for (int i = 0; i < kTbCount; i++) mbar_init(&t.bars[i], 1);
        *t.alive = 1;
        fence_barrier_init();
    }
    if ((threadIdx.x >> 5) == 2) {
        tmem_alloc(slot, tmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    t.tmem = *slot;
    t.ph = 0;
    t.merged = merged;
    t.lastLoad = 0;
    t.loaded = 0;
    t.trace = nullptr;
    t.mark = 0;
    return t;
}

// End of a merged kernel: every product and copy of the CTA has completed
// (waited for only when a wait gave up: otherwise each pass observed its
// own), then TMEM is freed.
__device__ __forceinline__ void tp_teardown(TilePass& t, int* status) {
    const bool dead = __syncthreads_or(t.ok() ? 0 : 1) != 0;
    if (dead) {
        if ((threadIdx.x >> 5) == 1 && (threadIdx.x & 31) == 0) {
            tc_commit(t.bar(kTbFin));
            mbar_wait(t.bar(kTbFin), 0, status, kDevTimeoutDone);
        }
        if (threadIdx.x == 0)
            for (int b = kTbFull1; b <= kTbFull2; b++)
                if (t.loaded & (1u << b)) mbar_wait(t.bar(b), (t.lastLoad >> b) & 1u, status, kDevTimeoutFull);
    }
    tc_fence_before();
    __syncthreads();
    if ((threadIdx.x >> 5) == 2) {
        tc_fence_after();
        tmem_dealloc(t.tmem, 512);
    }
}

// Shared memory the pass state takes after a kernel's tiles.
constexpr int kTilePassBytes = 8 * kTbCount + 8 + 8;

}  // namespace mg
