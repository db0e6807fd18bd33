// capi.cu — context-free C-ABI entry points: library info, batched router,
// fp32 LoRA op.  See include/aos_cuda.h for the contract.

#include <cstring>
#include <mutex>
#include <vector>
#include <atomic>
#include <string>

#include "common.cuh"

namespace aos {

cudaError_t launch_route(const float* priors, const uint64_t* stable_ids, const float* vw,
                         const uint8_t* allowed, const uint32_t* positions, int T, int N,
                         const aos_router_params* params, aos_router_ring* rings, float* entropy,
                         int32_t* status, cudaStream_t stream);
cudaError_t launch_lora_op_f32(const float* x, int T, int in_dim, int out_dim, const float* W,
                               const float* A, const float* B, int n_adapters, int rank,
                               const float* alpha, const aos_router_ring* rings, float* y,
                               float* h_scratch, cudaStream_t stream);
size_t lora_op_scratch_floats(int T, int out_dim, int rank);
int lora_op_max_rank();

namespace {
thread_local std::string g_error;
}

void set_global_error(const std::string& msg) { g_error = msg; }

const char* global_error() { return g_error.c_str(); }

int require_device(int device) {
    int n = 0;
    cudaError_t e = cudaGetDeviceCount(&n);
    if (e != cudaSuccess || n == 0) {
        cudaGetLastError();
        set_global_error("no CUDA device visible; this backend has no CPU fallback");
        return AOS_ERR_NO_DEVICE;
    }
    int dev = device;
    if (dev < 0) {
        if (cudaGetDevice(&dev) != cudaSuccess) return AOS_ERR_NO_DEVICE;
    }
    if (dev >= n) return AOS_ERR_NO_DEVICE;
    // Compute capability per device, queried once (a per-call property query
    // costs milliseconds of host time on the step path).
    static std::atomic<int> cc[64];
    int major = dev < 64 ? cc[dev].load(std::memory_order_relaxed) : 0;
    if (major == 0) {
        int mj = 0, mn = 0;
        if (cudaDeviceGetAttribute(&mj, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
            cudaDeviceGetAttribute(&mn, cudaDevAttrComputeCapabilityMinor, dev) != cudaSuccess)
            return AOS_ERR_NO_DEVICE;
        major = mj * 16 + mn + 1;
        if (dev < 64) cc[dev].store(major, std::memory_order_relaxed);
    }
    const int mj = (major - 1) / 16, mn = (major - 1) % 16;
    if (mj != 10) {
        set_global_error("device is sm_" + std::to_string(mj) + std::to_string(mn) + "; this build targets sm_100a only");
        return AOS_ERR_NO_DEVICE;
    }
    return AOS_OK;
}

namespace {

// Device staging buffer for the host-pointer entry points: grow-only and
// cached per thread and device, so steady-state calls never allocate.
struct DevBuf {
    void* p = nullptr;
    int slot;
    explicit DevBuf(int s) : slot(s) {}
    cudaError_t alloc(size_t n) {
        struct Cache {
            void* ptr[16] = {};
            size_t cap[16] = {};
            int dev[16] = {};
        };
        thread_local Cache cache;
        if (!n) return cudaSuccess;
        int dev = 0;
        cudaGetDevice(&dev);
        if (cache.ptr[slot] && (cache.cap[slot] < n || cache.dev[slot] != dev)) {
            cudaFree(cache.ptr[slot]);
            cache.ptr[slot] = nullptr;
        }
        if (!cache.ptr[slot]) {
            cudaError_t e = cudaMalloc(&cache.ptr[slot], n);
            if (e != cudaSuccess) return e;
            cache.cap[slot] = n;
            cache.dev[slot] = dev;
        }
        p = cache.ptr[slot];
        return cudaSuccess;
    }
};

int validate_route_args(const void* priors, const void* sids, const void* rings, uint32_t T,
                        uint32_t N) {
    if (!priors || !sids || !rings) {
        set_global_error("aos_route_batch: priors, stable_ids and rings are required");
        return AOS_ERR_INVALID;
    }
    if (N == 0 || N > 4096) {
        set_global_error("aos_route_batch: N must be in [1, 4096]");
        return AOS_ERR_INVALID;
    }
    (void)T;
    return AOS_OK;
}

}  // namespace
}  // namespace aos

using namespace aos;

extern "C" {

const char* aos_version(void) { return "adapteros-b200 0.1.0 (sm_100a)"; }

int aos_device_count(void) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    int c = 0;
    for (int d = 0; d < n; ++d) {
        cudaDeviceProp p;
        if (cudaGetDeviceProperties(&p, d) == cudaSuccess && p.major == 10) ++c;
    }
    return c;
}

int aos_route_batch_dev(const float* priors, const uint64_t* stable_ids, const float* version_weights,
                        const uint8_t* allowed, const uint32_t* positions, uint32_t T, uint32_t N,
                        const aos_router_params* params, aos_router_ring* rings, float* entropy,
                        int32_t* status, void* stream) {
    int rc = validate_route_args(priors, stable_ids, rings, T, N);
    if (rc) return rc;
    if ((rc = require_device())) return rc;
    cudaError_t e = launch_route(priors, stable_ids, version_weights, allowed, positions, (int)T,
                                 (int)N, params, rings, entropy, status, (cudaStream_t)stream);
    if (e != cudaSuccess) {
        set_global_error(std::string("route kernel launch: ") + cudaGetErrorString(e));
        return AOS_ERR_CUDA;
    }
    return AOS_OK;
}

int aos_route_batch(const float* priors, const uint64_t* stable_ids, const float* version_weights,
                    const uint8_t* allowed, const uint32_t* positions, uint32_t T, uint32_t N,
                    const aos_router_params* params, aos_router_ring* rings, float* entropy,
                    int32_t* status) {
    int rc = validate_route_args(priors, stable_ids, rings, T, N);
    if (rc) return rc;
    if ((rc = require_device())) return rc;
    if (T == 0) return AOS_OK;
    DevBuf dp(0), ds(1), dv(2), da(3), dpos(4), dr(5), de(6), dst(7);
    AOS_RETURN_IF_CUDA(dp.alloc((size_t)T * N * 4), set_global_error);
    AOS_RETURN_IF_CUDA(ds.alloc((size_t)N * 8), set_global_error);
    AOS_RETURN_IF_CUDA(dr.alloc((size_t)T * sizeof(aos_router_ring)), set_global_error);
    AOS_RETURN_IF_CUDA(de.alloc((size_t)T * 4), set_global_error);
    AOS_RETURN_IF_CUDA(dst.alloc((size_t)T * 4), set_global_error);
    AOS_RETURN_IF_CUDA(cudaMemcpy(dp.p, priors, (size_t)T * N * 4, cudaMemcpyHostToDevice), set_global_error);
    AOS_RETURN_IF_CUDA(cudaMemcpy(ds.p, stable_ids, (size_t)N * 8, cudaMemcpyHostToDevice), set_global_error);
    if (version_weights) {
        AOS_RETURN_IF_CUDA(dv.alloc((size_t)N * 4), set_global_error);
        AOS_RETURN_IF_CUDA(cudaMemcpy(dv.p, version_weights, (size_t)N * 4, cudaMemcpyHostToDevice), set_global_error);
    }
    if (allowed) {
        AOS_RETURN_IF_CUDA(da.alloc((size_t)N), set_global_error);
        AOS_RETURN_IF_CUDA(cudaMemcpy(da.p, allowed, (size_t)N, cudaMemcpyHostToDevice), set_global_error);
    }
    if (positions) {
        AOS_RETURN_IF_CUDA(dpos.alloc((size_t)T * 4), set_global_error);
        AOS_RETURN_IF_CUDA(cudaMemcpy(dpos.p, positions, (size_t)T * 4, cudaMemcpyHostToDevice), set_global_error);
    }
    cudaError_t e = launch_route((const float*)dp.p, (const uint64_t*)ds.p, (const float*)dv.p,
                                 (const uint8_t*)da.p, (const uint32_t*)dpos.p, (int)T, (int)N, params,
                                 (aos_router_ring*)dr.p, (float*)de.p, (int32_t*)dst.p, 0);
    if (e != cudaSuccess) {
        set_global_error(std::string("route kernel launch: ") + cudaGetErrorString(e));
        return AOS_ERR_CUDA;
    }
    AOS_RETURN_IF_CUDA(cudaMemcpy(rings, dr.p, (size_t)T * sizeof(aos_router_ring), cudaMemcpyDeviceToHost), set_global_error);
    std::vector<int32_t> st(T);
    AOS_RETURN_IF_CUDA(cudaMemcpy(st.data(), dst.p, (size_t)T * 4, cudaMemcpyDeviceToHost), set_global_error);
    if (entropy) AOS_RETURN_IF_CUDA(cudaMemcpy(entropy, de.p, (size_t)T * 4, cudaMemcpyDeviceToHost), set_global_error);
    if (status) memcpy(status, st.data(), (size_t)T * 4);
    for (uint32_t t = 0; t < T; ++t)
        if (st[t] != 0) {
            set_global_error("aos_route_batch: non-finite prior or score for token " + std::to_string(t));
            return AOS_ERR_NONFINITE;
        }
    return AOS_OK;
}

int aos_lora_op_f32_dev(const float* x, uint32_t T, uint32_t in_dim, uint32_t out_dim, const float* W,
                        const float* A, const float* B, uint32_t n_adapters, uint32_t rank,
                        const float* alpha, const aos_router_ring* rings, float* y, void* stream) {
    if (!x || !W || !A || !B || !rings || !y || rank == 0 || (int)rank > lora_op_max_rank() ||
        in_dim % 4 != 0 || in_dim == 0 || out_dim == 0) {
        set_global_error("aos_lora_op_f32: invalid arguments (rank in [1,64], in_dim % 4 == 0)");
        return AOS_ERR_INVALID;
    }
    // The shrink reads x and A rows with 16-byte loads (in_dim % 4 == 0 keeps
    // every row on a 16-byte boundary once the base pointer is).
    if (((uintptr_t)x | (uintptr_t)A) & 15u) {
        set_global_error("aos_lora_op_f32: x and A must be 16-byte aligned");
        return AOS_ERR_INVALID;
    }
    int rc = require_device();
    if (rc) return rc;
    if (T == 0) return AOS_OK;
    cudaStream_t s = (cudaStream_t)stream;
    float* h = nullptr;
    AOS_RETURN_IF_CUDA(cudaMallocAsync((void**)&h, lora_op_scratch_floats((int)T, (int)out_dim, (int)rank) * 4, s),
                       set_global_error);
    cudaError_t e = launch_lora_op_f32(x, (int)T, (int)in_dim, (int)out_dim, W, A, B, (int)n_adapters,
                                       (int)rank, alpha, rings, y, h, s);
    cudaFreeAsync(h, s);
    if (e != cudaSuccess) {
        set_global_error(std::string("lora op launch: ") + cudaGetErrorString(e));
        return AOS_ERR_CUDA;
    }
    return AOS_OK;
}

int aos_lora_op_f32(const float* x, uint32_t T, uint32_t in_dim, uint32_t out_dim, const float* W,
                    const float* A, const float* B, uint32_t n_adapters, uint32_t rank, const float* alpha,
                    const aos_router_ring* rings, float* y) {
    if (!x || !W || !A || !B || !rings || !y) {
        set_global_error("aos_lora_op_f32: null argument");
        return AOS_ERR_INVALID;
    }
    int rc = require_device();
    if (rc) return rc;
    if (T == 0) return AOS_OK;
    DevBuf dx(8), dw(9), da(10), db(11), dal(12), dr(13), dy(14);
    const size_t nx = (size_t)T * in_dim * 4, nw = (size_t)out_dim * in_dim * 4;
    const size_t na = (size_t)n_adapters * rank * in_dim * 4, nb = (size_t)n_adapters * out_dim * rank * 4;
    AOS_RETURN_IF_CUDA(dx.alloc(nx), set_global_error);
    AOS_RETURN_IF_CUDA(dw.alloc(nw), set_global_error);
    AOS_RETURN_IF_CUDA(da.alloc(na), set_global_error);
    AOS_RETURN_IF_CUDA(db.alloc(nb), set_global_error);
    AOS_RETURN_IF_CUDA(dr.alloc((size_t)T * sizeof(aos_router_ring)), set_global_error);
    AOS_RETURN_IF_CUDA(dy.alloc((size_t)T * out_dim * 4), set_global_error);
    AOS_RETURN_IF_CUDA(cudaMemcpy(dx.p, x, nx, cudaMemcpyHostToDevice), set_global_error);
    AOS_RETURN_IF_CUDA(cudaMemcpy(dw.p, W, nw, cudaMemcpyHostToDevice), set_global_error);
    AOS_RETURN_IF_CUDA(cudaMemcpy(da.p, A, na, cudaMemcpyHostToDevice), set_global_error);
    AOS_RETURN_IF_CUDA(cudaMemcpy(db.p, B, nb, cudaMemcpyHostToDevice), set_global_error);
    AOS_RETURN_IF_CUDA(cudaMemcpy(dr.p, rings, (size_t)T * sizeof(aos_router_ring), cudaMemcpyHostToDevice), set_global_error);
    if (alpha) {
        AOS_RETURN_IF_CUDA(dal.alloc((size_t)n_adapters * 4), set_global_error);
        AOS_RETURN_IF_CUDA(cudaMemcpy(dal.p, alpha, (size_t)n_adapters * 4, cudaMemcpyHostToDevice), set_global_error);
    }
    rc = aos_lora_op_f32_dev((const float*)dx.p, T, in_dim, out_dim, (const float*)dw.p, (const float*)da.p,
                             (const float*)db.p, n_adapters, rank, (const float*)dal.p,
                             (const aos_router_ring*)dr.p, (float*)dy.p, nullptr);
    if (rc) return rc;
    AOS_RETURN_IF_CUDA(cudaMemcpy(y, dy.p, (size_t)T * out_dim * 4, cudaMemcpyDeviceToHost), set_global_error);
    return AOS_OK;
}

}  // extern "C"
