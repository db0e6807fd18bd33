// noalloc.cu — aos_lora_op_f32_noalloc_dev: the fp32 base + K-sparse LoRA op
// of aos_lora_op_f32_dev for callers that must not allocate device memory.
// It runs the same shrink kernel and then one single-pass base + expand
// kernel over all of K, where aos_lora_op_f32_dev sums eight fp32 K-eighth
// partials; the two entry points therefore round differently and agree
// within fp32 tolerance, not bit for bit (each is bit-identical run to run).
//
// Who needs it: a host that fixes its device-memory budget when it starts and
// forbids allocation afterwards, code that shares a device with a thread
// capturing a CUDA graph (cudaMalloc/cudaFree synchronise the device and are
// not allowed while a capture is open), and latency-critical loops where an
// allocator call would stall other streams.  aos_lora_op_f32_dev allocates
// its per-call scratch (the rank-sized shrink results) with cudaMallocAsync;
// this entry point takes that scratch from a fixed device array instead.
//
// The scratch is the file-scope array below: kNoAllocScratchFloats floats
// (512 KiB), present on every device that loads this library until the
// process exits.  A call needs T * 8 * rank floats of it (the shrink results
// of every token's 8 ring slots), so T * 8 * rank must not exceed
// kNoAllocScratchFloats; larger calls are rejected with AOS_ERR_INVALID.
//
// Host code cannot use the array's name as a device address (in host code it
// names a host-side stand-in).  The first call in each CUDA context (per
// device, and again after the context changes, e.g. after cudaDeviceReset)
// looks up the real address with cudaGetSymbolAddress while that device is
// current and caches it with the context's id; make that first call before
// any stream capture on the device.
//
// Every call shares the one array, and a call leaves its own results in it.
// The shrink kernel writes every scratch entry it later reads (zero for
// unused slots), so nothing needs clearing between calls.  Calls whose
// kernels overlap on the GPU (different streams, or a second call before the
// first has run) race on the array: serialise them, e.g. on one stream.
// Nothing here calls cudaMalloc, cudaFree or any allocating library routine.

#include <cuda.h>

#include <mutex>
#include <string>

#include "common.cuh"

namespace aos {
cudaError_t launch_lora_op_f32_small(const float* x, int T, int in_dim, int out_dim, const float* W, const float* A,
                               const float* B, int n_adapters, int rank, const float* alpha,
                               const aos_router_ring* rings, float* y, float* h_scratch, cudaStream_t stream);
int lora_op_max_rank();
}  // namespace aos

namespace {

constexpr size_t kNoAllocScratchFloats = 131072;  // 512 KiB

static __device__ __align__(256) float g_noalloc_scratch[kNoAllocScratchFloats];

constexpr int kMaxDevices = 64;
std::mutex g_addr_mutex;
struct CachedAddr {
    unsigned long long ctx_id;  // context the address belongs to (0 = unknown)
    float* addr;
};
CachedAddr g_addr[kMaxDevices] = {};

// Id of the current CUDA context (cuCtxGetId through the runtime's driver
// entry points), so that an address cached in one context is never used in
// another (a cudaDeviceReset makes a new primary context and reloads the
// module).  0 when there is no current context or the driver cannot tell.
unsigned long long current_ctx_id() {
    using GetCurrent = CUresult (*)(CUcontext*);
    using GetId = CUresult (*)(CUcontext, unsigned long long*);
    static GetCurrent get_current = nullptr;
    static GetId get_id = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            get_current = reinterpret_cast<GetCurrent>(f);
        f = nullptr;
        if (cudaGetDriverEntryPoint("cuCtxGetId", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            get_id = reinterpret_cast<GetId>(f);
    });
    CUcontext ctx = nullptr;
    unsigned long long id = 0;
    if (get_current && get_id && get_current(&ctx) == CUDA_SUCCESS && ctx && get_id(ctx, &id) == CUDA_SUCCESS)
        return id;
    return 0;
}

// Device address of g_noalloc_scratch in the current context, looked up with
// the device current the first time a context is seen (every call, should
// the driver not report context ids).
int scratch_address(float** out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
        aos::set_global_error("aos_lora_op_f32_noalloc_dev: no current CUDA device");
        return AOS_ERR_NO_DEVICE;
    }
    std::lock_guard<std::mutex> lock(g_addr_mutex);
    const unsigned long long id = current_ctx_id();
    if (id == 0 || !g_addr[dev].addr || g_addr[dev].ctx_id != id) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess || !p) {
            aos::set_global_error(std::string("aos_lora_op_f32_noalloc_dev: cudaGetSymbolAddress failed: ") +
                                  cudaGetErrorString(e));
            return AOS_ERR_CUDA;
        }
        g_addr[dev].addr = static_cast<float*>(p);
        g_addr[dev].ctx_id = current_ctx_id();  // the lookup made the context current if it was not
    }
    *out = g_addr[dev].addr;
    return AOS_OK;
}

}  // namespace

extern "C" int aos_lora_op_f32_noalloc_dev(const float* x, uint32_t T, uint32_t in_dim, uint32_t out_dim,
                                           const float* W, const float* A, const float* B, uint32_t n_adapters,
                                           uint32_t rank, const float* alpha, const aos_router_ring* rings, float* y,
                                           void* stream) {
    if (!x || !W || !A || !B || !rings || !y || rank == 0 || (int)rank > aos::lora_op_max_rank() ||
        in_dim % 4 != 0 || in_dim == 0 || out_dim == 0) {
        aos::set_global_error("aos_lora_op_f32_noalloc_dev: invalid arguments (rank in [1,64], in_dim % 4 == 0)");
        return AOS_ERR_INVALID;
    }
    // The shrink reads x and A rows with 16-byte loads.
    if (((uintptr_t)x | (uintptr_t)A) & 15u) {
        aos::set_global_error("aos_lora_op_f32_noalloc_dev: x and A must be 16-byte aligned");
        return AOS_ERR_INVALID;
    }
    if ((size_t)T * AOS_MAX_K * rank > kNoAllocScratchFloats) {
        aos::set_global_error("aos_lora_op_f32_noalloc_dev: T * 8 * rank = " +
                              std::to_string((size_t)T * AOS_MAX_K * rank) + " exceeds the fixed scratch of " +
                              std::to_string(kNoAllocScratchFloats) + " floats");
        return AOS_ERR_INVALID;
    }
    int rc = aos::require_device();
    if (rc) return rc;
    if (T == 0) return AOS_OK;
    float* h = nullptr;
    if ((rc = scratch_address(&h))) return rc;
    cudaError_t e = aos::launch_lora_op_f32_small(x, (int)T, (int)in_dim, (int)out_dim, W, A, B, (int)n_adapters, (int)rank,
                                            alpha, rings, y, h, (cudaStream_t)stream);
    if (e != cudaSuccess) {
        aos::set_global_error(std::string("aos_lora_op_f32_noalloc_dev launch: ") + cudaGetErrorString(e));
        return AOS_ERR_CUDA;
    }
    return AOS_OK;
}
