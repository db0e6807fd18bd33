// common.cuh — shared device/host helpers for the sm_100a backend.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>
#include <utility>

#include "../../include/aos_cuda.h"

namespace aos {

// Host-side error channel for context-free entry points (thread local, like
// mlx_get_last_error's global string, wrapper.h:199-200).
void set_global_error(const std::string& msg);
const char* global_error();

#define AOS_RETURN_IF_CUDA(expr, setter)                                                     \
    do {                                                                                     \
        cudaError_t _e = (expr);                                                             \
        if (_e != cudaSuccess) {                                                             \
            setter(std::string(#expr " failed: ") + cudaGetErrorString(_e));                 \
            return AOS_ERR_CUDA;                                                             \
        }                                                                                    \
    } while (0)

// True when a usable sm_100 device is current; otherwise records why.
int require_device(int device = -1);

// ----------------------------------------------------------------- device side
__device__ __forceinline__ float bf2f(uint16_t h) { return __uint_as_float((uint32_t)h << 16); }
__device__ __forceinline__ uint16_t f2bf(float f) {
    __nv_bfloat16 b = __float2bfloat16_rn(f);
    return *reinterpret_cast<uint16_t*>(&b);
}

// f32::total_cmp key: signed-integer order equals IEEE-754 total order.
__device__ __forceinline__ int32_t total_key(float f) {
    int32_t i = __float_as_int(f);
    return i ^ (int32_t)(((uint32_t)(i >> 31)) >> 1);
}

// Upper bound for every device-side spin (~1 s at the B200's max SM clock).
constexpr long long kSpinLimitCycles = 2000000000LL;

// Programmatic dependent launch.  Every kernel of the decode step runs
//   prologue (static data, or data produced two or more launches earlier)
//   -> pdl_wait()   : the previous launch has completed and its writes are visible
//   -> pdl_trigger(): the next launch may be scheduled (it still waits for us)
//   -> main work.
// Because each kernel triggers only after its own wait, a kernel's prologue
// may read anything written by the launch before its predecessor.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Launch with the programmatic-stream-serialization attribute.  cooperative:
// also ask for every CTA of the grid to be resident at once (kernels whose
// CTAs wait on one another); the launch then fails instead of starting a grid
// that cannot be co-resident.
template <typename... KArgs, typename... Args>
cudaError_t launch_k_ex(bool cooperative, void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                        Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeCooperative;
    attr[1].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = cooperative ? 2 : 1;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}
template <typename... KArgs, typename... Args>
cudaError_t launch_k(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, Args&&... args) {
    return launch_k_ex(false, kernel, grid, block, smem, s, std::forward<Args>(args)...);
}

}  // namespace aos
