// prefill_static.cu -- pma_prefill_no_alloc: the prefill for callers that cannot
// allocate device memory.
//
// pma_prefill asks its caller for a small scratch workspace (a status word, and
// the per-segment states when a sequence is split across SMs).  Some callers
// cannot provide one on demand: a plugin running inside a host application that
// owns all device memory through its own pool and forbids direct cudaMalloc; FFI
// callers (cgo, JNI, other runtimes) that have no device allocator of their own;
// and latency-critical loops, where cudaMalloc/cudaFree would synchronise the
// device.  This entry point takes the same arguments minus the workspace and
// uses a fixed buffer compiled into the library instead.
//
// The buffer is a file-scope __device__ array of kScratchBytes; every GPU that
// loads the library holds one copy until the process exits.  Host code cannot
// use the array's name as a device address, so the first call on each device
// (with that device current) looks the address up with cudaGetSymbolAddress and
// keeps it; make that first call before any stream capture.  The address belongs
// to the CUDA context the library's module is loaded into, so it is kept together
// with that context and looked up again when a call finds another context current
// (a host application that creates or switches contexts).  All calls on a device
// share the one buffer and it keeps the previous call's contents: the status word
// is cleared by every call, and segment states are written before they are read,
// so nothing else needs clearing; but calls that overlap on the GPU (other
// streams, other host threads) race on it and must be serialised by the caller.
// The status word sits inside the buffer, out of the caller's reach; a caller
// sees an expired wait through the fault word it registers with
// pma_set_fault_word, which every launch of this entry point also writes.
#include <cuda.h>

#include <mutex>

#include "prefill.cuh"

namespace {

constexpr size_t kScratchBytes = size_t(16) << 20;  // 16 MiB per device
static __device__ __align__(256) unsigned char g_prefill_scratch[kScratchBytes];

constexpr int kMaxDevices = 64;
struct ScratchAddr {
    CUcontext ctx;  // context the address was looked up in
    void *ptr;
};
ScratchAddr g_scratch_addr[kMaxDevices];
std::mutex g_scratch_mu;

typedef CUresult (*CtxGetCurrent)(CUcontext *);

// The driver's cuCtxGetCurrent, fetched through the runtime (the library does not link libcuda).
CtxGetCurrent ctx_get_current() {
    static CtxGetCurrent fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<CtxGetCurrent>(ptr);
    });
    return fn;
}

}  // namespace

extern "C" int pma_prefill_no_alloc(int B, int H, int L, int D, const pma_seq_tensor *q, const pma_seq_tensor *k,
                                    const pma_seq_tensor *v, const float *lambda, int64_t lambda_stride_b,
                                    const pma_state *state_in, const pma_state *state_out, float eps,
                                    const pma_seq_tensor *y, pma_stream_t stream) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return pma::cuda_fail(e);
    if (dev < 0 || dev >= kMaxDevices) return PMA_ERR_DEVICE;
    void *scratch = nullptr;
    {
        std::lock_guard<std::mutex> lk(g_scratch_mu);
        ScratchAddr &slot = g_scratch_addr[dev];
        CUcontext ctx = nullptr;
        const CtxGetCurrent get_ctx = ctx_get_current();
        if (get_ctx && get_ctx(&ctx) != CUDA_SUCCESS) ctx = nullptr;
        if (!slot.ptr || (ctx && ctx != slot.ctx)) {
            void *ptr = nullptr;
            if ((e = cudaGetSymbolAddress(&ptr, g_prefill_scratch)) != cudaSuccess) return pma::cuda_fail(e);
            if (!ptr) return pma::cuda_fail(cudaErrorInvalidSymbol);
            if (!ctx && get_ctx) get_ctx(&ctx);  // the lookup made the primary context current
            slot.ctx = ctx;
            slot.ptr = ptr;
        }
        scratch = slot.ptr;
    }
    if (!q) return PMA_ERR_ARGUMENT;
    // Same plan as pma_prefill; reject problems whose scratch exceeds the fixed buffer.
    if (pma_prefill_workspace_bytes(B, H, L, D, q->dtype) > kScratchBytes) return PMA_ERR_WORKSPACE;
    return pma_prefill(B, H, L, D, q, k, v, lambda, lambda_stride_b, state_in, state_out, eps, y, scratch,
                       kScratchBytes, stream);
}
