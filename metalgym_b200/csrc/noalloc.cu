// Weight gradient dW = X^T dZ that allocates no device memory.
//
// Some callers cannot call cudaMalloc: code running inside a framework that
// owns every byte of device memory (a custom call or plugin whose enqueue
// must not allocate), or a host program that forbids allocation after
// start-up. For them this entry point keeps its split-K partial sums in a
// fixed scratch array compiled into the library instead of asking for a
// workspace. The caller still passes the inputs and the output.
//
// The array below is allocated once on every GPU that loads the library and
// is held until the process exits. Every call shares it and it keeps the last
// call's contents; each call overwrites all of the partials it reads, so
// nothing has to start at zero. Calls that overlap on the GPU (on different
// streams, or on different host threads of the same device) race on it.
#include <mutex>
#include <string>

#include "gemm.h"
#include "policy.h"
#include "runtime.h"

namespace {

constexpr size_t kScratchBytes = MG_WEIGHT_GRAD_NOALLOC_SCRATCH_BYTES;

// The scratch: split-K partials, then one sum of squares per finalisation CTA.
static __device__ __align__(256) float g_noalloc_scratch[kScratchBytes / sizeof(float)];

constexpr int kMaxDevices = 64;
float* g_scratch_addr[kMaxDevices] = {};
uint64_t g_scratch_ctx[kMaxDevices] = {};  // the context each address belongs to
std::mutex g_scratch_mu;

// Device address of the scratch on the current device, looked up on the
// first call made on that device (host code cannot use the symbol itself),
// and again when the device's context changed (after cudaDeviceReset the
// array lives at a new address in the new context).
int scratch_address(float** out) {
    int dev = 0;
    MG_CUDA_TRY(cudaGetDevice(&dev));
    if (dev < 0 || dev >= kMaxDevices) return mg::fail(MG_ERR_UNSUPPORTED, "device index out of range");
    const uint64_t ctx = mg::current_context_id();
    std::lock_guard<std::mutex> lock(g_scratch_mu);
    if (!g_scratch_addr[dev] || ctx == 0 || g_scratch_ctx[dev] != ctx) {
        void* p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess) return mg::cuda_fail(e, "cudaGetSymbolAddress(no-alloc scratch)");
        g_scratch_addr[dev] = static_cast<float*>(p);
        g_scratch_ctx[dev] = mg::current_context_id();
    }
    *out = g_scratch_addr[dev];
    return MG_OK;
}

}  // namespace

extern "C" int mg_weight_grad_noalloc(const void* x, const void* dz, int rows, int in_features, int out_features,
                                      int splits, int round_bf16, float* dw_out, mg_stream_t stream) {
    MG_CHECK_ARG(x && dz && dw_out, "mg_weight_grad_noalloc: null pointer");
    MG_CHECK_ARG(rows > 0 && in_features > 0 && out_features > 0 && splits >= 1,
                 "mg_weight_grad_noalloc: sizes must be positive");
    MG_CHECK_ARG(in_features % 8 == 0 && out_features % 32 == 0,
                 "mg_weight_grad_noalloc: in_features must be a multiple of 8 and out_features of 32");
    const int nsplit = mg::gemm_effective_splits(rows, splits);
    const size_t count = (size_t)in_features * out_features;
    const size_t normParts = (count + mg::kGradPerCta - 1) / mg::kGradPerCta;
    const size_t need = ((size_t)nsplit * count + normParts) * sizeof(float);
    if (need > kScratchBytes)
        return mg::fail(MG_ERR_ARGUMENT, "mg_weight_grad_noalloc: needs " + std::to_string(need) +
                                             " bytes of scratch (splits x in_features x out_features x 4 + norm "
                                             "partials), the maximum is " +
                                             std::to_string(kScratchBytes));
    float* scratch = nullptr;
    int rc = scratch_address(&scratch);
    if (rc) return rc;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    // split-K partials: split z = sum over its rows of x^T dz
    mg::GemmCall c;
    c.A = x;
    c.a_mn = true;
    c.lda = in_features;
    c.B = dz;
    c.b_mn = true;
    c.ldb = out_features;
    c.M = in_features;
    c.N = out_features;
    c.K = rows;
    c.epilogue = 4;
    c.out = scratch;
    c.ldo = out_features;
    c.splits = nsplit;
    rc = mg::gemm_bf16(c, st);
    if (rc) return rc;
    // sum of the partials into dw_out (rounded to bf16 if asked)
    mg::GradSegmentTable tab{};
    tab.n = 1;
    tab.seg[0].src = scratch;
    tab.seg[0].partStride = (int64_t)count;
    tab.seg[0].nparts = nsplit;
    tab.seg[0].count = (int64_t)count;
    tab.seg[0].dstOffset = 0;
    tab.seg[0].roundBf16 = round_bf16 ? 1 : 0;
    mg::grad_table_layout(tab, false);  // one norm partial per 1024 elements
    return mg::grad_finalize(tab, dw_out, scratch + (size_t)nsplit * count, st);
}
