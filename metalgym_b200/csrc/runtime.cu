// Host runtime: error strings, the device status word, TMA descriptors.
#include "runtime.h"

#include <atomic>
#include <map>
#include <mutex>
#include <set>
#include <string>

namespace mg {

namespace {
thread_local std::string g_last_error;

// One status word per device: kernels record wait timeouts and shape errors
// here (first error wins); mg_device_status() reads and clears it.
__device__ int g_status_word;

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    });
    return fn;
}
}  // namespace

int fail(int code, const std::string& msg) {
    g_last_error = msg;
    return code;
}

int cuda_fail(cudaError_t e, const char* what) {
    return fail(MG_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

namespace {
std::mutex g_comm_mu;
std::set<const void*>& aborted_comms() {
    static std::set<const void*> s;
    return s;
}
}  // namespace

void comm_mark_aborted(const void* comm) {
    std::lock_guard<std::mutex> g(g_comm_mu);
    aborted_comms().insert(comm);
}
bool comm_aborted(const void* comm) {
    std::lock_guard<std::mutex> g(g_comm_mu);
    return aborted_comms().count(comm) != 0;
}
bool comm_forget_aborted(const void* comm) {
    std::lock_guard<std::mutex> g(g_comm_mu);
    return aborted_comms().erase(comm) != 0;
}

namespace {
std::map<const void*, std::set<cudaGraphExec_t*>>& comm_graphs() {
    static std::map<const void*, std::set<cudaGraphExec_t*>> m;
    return m;
}
}  // namespace

void comm_bind_graph(const void* comm, cudaGraphExec_t* slot) {
    if (!comm || !slot) return;
    std::lock_guard<std::mutex> g(g_comm_mu);
    comm_graphs()[comm].insert(slot);
}

void comm_unbind_graph(const void* comm, cudaGraphExec_t* slot) {
    if (!comm || !slot) return;
    std::lock_guard<std::mutex> g(g_comm_mu);
    auto it = comm_graphs().find(comm);
    if (it == comm_graphs().end()) return;
    it->second.erase(slot);
    if (it->second.empty()) comm_graphs().erase(it);
}

void comm_release_graphs(const void* comm) {
    std::lock_guard<std::mutex> g(g_comm_mu);
    auto it = comm_graphs().find(comm);
    if (it == comm_graphs().end()) return;
    for (cudaGraphExec_t* slot : it->second)
        if (*slot) {
            cudaGraphExecDestroy(*slot);
            *slot = nullptr;
        }
}

std::mutex& capture_mutex() {
    static std::mutex m;
    return m;
}

int num_sms() {
    static std::atomic<int> cache[64] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
    int n = cache[dev].load(std::memory_order_relaxed);
    if (!n) {
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
        cache[dev].store(n, std::memory_order_relaxed);
    }
    return n;
}

uint64_t current_context_id() {
    typedef CUresult (*CtxGetCurrentFn)(CUcontext*);
    typedef CUresult (*CtxGetIdFn)(CUcontext, unsigned long long*);
    static CtxGetCurrentFn getCurrent = nullptr;
    static CtxGetIdFn getId = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            getCurrent = reinterpret_cast<CtxGetCurrentFn>(p);
        if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            getId = reinterpret_cast<CtxGetIdFn>(p);
    });
    CUcontext ctx = nullptr;
    unsigned long long id = 0;
    if (!getCurrent || !getId || getCurrent(&ctx) != CUDA_SUCCESS || !ctx || getId(ctx, &id) != CUDA_SUCCESS) return 0;
    return (uint64_t)id;
}

int* status_ptr() {
    constexpr int kMaxDevices = 64;
    // per device: the address and the id of the context it was looked up in
    // (a device reset makes a new context, with the word at a new address)
    static int* cache[kMaxDevices] = {};
    static uint64_t cacheCtx[kMaxDevices] = {};
    static std::mutex mu;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
    // 0 before the runtime made a context current: the lookup below does,
    // and the next call sees the real id and looks the address up once more
    const uint64_t ctx = current_context_id();
    std::lock_guard<std::mutex> lock(mu);
    if (!cache[dev] || cacheCtx[dev] != ctx) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_status_word) != cudaSuccess) return nullptr;
        cache[dev] = static_cast<int*>(p);
        cacheCtx[dev] = ctx;
    }
    return cache[dev];
}

namespace {
std::atomic<uint64_t*> g_tile_trace{nullptr};
}

uint64_t* tile_trace() { return g_tile_trace.load(std::memory_order_relaxed); }

int make_tmap_bf16(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer, uint64_t row_stride,
                   uint32_t box_outer) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return fail(MG_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
    if ((reinterpret_cast<uintptr_t>(base) & 15) != 0) return fail(MG_ERR_ARGUMENT, "TMA base not 16-byte aligned");
    if ((row_stride * 2) % 16 != 0) return fail(MG_ERR_ARGUMENT, "TMA row stride not a multiple of 16 bytes");
    cuuint64_t dims[2] = {inner, outer};
    cuuint64_t strides[1] = {row_stride * 2};
    cuuint32_t box[2] = {64, box_outer};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(MG_ERR_CUDA, "cuTensorMapEncodeTiled failed: " + std::to_string((int)r));
    return MG_OK;
}

int check_launch(const char* what) {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, what);
    return MG_OK;
}

}  // namespace mg

extern "C" {

const char* mg_last_error(void) { return mg::g_last_error.c_str(); }

int mg_version(void) { return MG_VERSION; }

int mg_set_tile_trace(uint64_t* buffer) {
    mg::g_tile_trace.store(buffer, std::memory_order_relaxed);
    return MG_OK;
}

int mg_device_status(int clear, int* status) {
    int* p = mg::status_ptr();
    if (!p) return mg::fail(MG_ERR_CUDA, "status word lookup failed");
    int v = 0;
    MG_CUDA_TRY(cudaMemcpy(&v, p, sizeof(int), cudaMemcpyDeviceToHost));
    if (clear) MG_CUDA_TRY(cudaMemset(p, 0, sizeof(int)));
    if (status) *status = v;
    return MG_OK;
}

}  // extern "C"
