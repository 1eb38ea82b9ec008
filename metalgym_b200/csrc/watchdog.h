// Bounded wait for GPU work that depends on other ranks (the gradient
// all-reduce of a data-parallel train()).
//
// A rank whose peer died, or never joined the collective, would otherwise
// wait forever in cudaStreamSynchronize while the NCCL kernel spins. Instead
// the host polls: the stream's completion, the communicator's asynchronous
// error, and a deadline. On a peer error or at the deadline it releases the
// CUDA graphs that captured the communicator's collectives (NCCL's abort waits
// until every such graph is gone; one still in flight is freed when its launch
// completes), aborts the communicator's operations in flight (ncclCommAbort
// makes the spinning kernels return) and then waits, again at most a bounded
// time, for the stream to drain. Plain C++ with the operations passed as function
// pointers, so the logic is tested on the CPU with fakes.
#pragma once

namespace mg {

struct WatchOps {
    void* ctx;
    int (*done)(void* ctx);       // 1: the stream has finished; 0: not yet; < 0: a CUDA error
    int (*peerError)(void* ctx);  // non-zero: the communicator reported an asynchronous error
    void (*release)(void* ctx);   // releases the graphs that the abort would wait for
    void (*abort)(void* ctx);     // aborts the communicator and its operations in flight
    double (*now)(void* ctx);     // monotonic seconds
    void (*pause)(void* ctx);     // a short sleep between polls
};

enum WatchResult : int {
    kWatchDone = 0,       // the stream finished
    kWatchCudaError = 1,  // done() reported a CUDA error (nothing aborted)
    kWatchPeerError = 2,  // the communicator reported an error: aborted
    kWatchTimeout = 3,    // the deadline passed: aborted
};

// Waits until the stream finishes, at most `limit` seconds. After an abort,
// *drained tells whether the stream then finished within `drain` seconds.
inline int watch_wait(const WatchOps& o, double limit, double drain, bool* drained) {
    if (drained) *drained = false;
    const double t0 = o.now(o.ctx);
    int result = kWatchDone;
    for (;;) {
        const int d = o.done(o.ctx);
        if (d > 0) {
            if (drained) *drained = true;
            return kWatchDone;
        }
        if (d < 0) return kWatchCudaError;
        if (o.peerError(o.ctx)) {
            result = kWatchPeerError;
            break;
        }
        if (o.now(o.ctx) - t0 > limit) {
            result = kWatchTimeout;
            break;
        }
        o.pause(o.ctx);
    }
    o.release(o.ctx);
    o.abort(o.ctx);
    const double t1 = o.now(o.ctx);
    for (;;) {
        const int d = o.done(o.ctx);
        if (d != 0) {
            if (drained) *drained = d > 0;
            break;
        }
        if (o.now(o.ctx) - t1 > drain) break;
        o.pause(o.ctx);
    }
    return result;
}

}  // namespace mg
