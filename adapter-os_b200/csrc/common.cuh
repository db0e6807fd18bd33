// common.cuh — shared device/host helpers for the sm_100a backend.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

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

}  // namespace aos
