// loader.cuh — host-side pieces shared by the weight loaders
// (safetensors.cu, aos_archive.cu, runtime.cu).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <string>
#include <vector>

struct aos_ctx;

namespace aos {

// One tensor of a safetensors container; [b, e) is relative to the first
// byte after the JSON header.
struct StTensor {
    std::string name, dtype;
    std::vector<int64_t> shape;
    uint64_t b = 0, e = 0;
};

// Parses a safetensors container; *base receives the first tensor byte.
int parse_safetensors(const uint8_t* d, uint64_t len, std::vector<StTensor>& out, const uint8_t** base,
                      std::string& err);
// F32 / F16 / BF16 tensor bytes -> bf16 (round to nearest even).
int tensor_to_bf16(const StTensor& t, const uint8_t* base, std::vector<uint16_t>& out, std::string& err);

// BLAKE3 digests of n_msg messages of device memory d_base + offsets[i],
// lens[i] bytes each, into host digests[32 * i].  Synchronizes s.
int blake3_many(const uint8_t* d_base, const uint64_t* offsets, const uint64_t* lens, int n_msg, uint8_t* digests,
                cudaStream_t s, std::string& err);

// One packed matrix in the canonical element stream read by
// launch_unpack_samples: elements [e0, e0 + rows * cols) are the row-major
// rows x cols matrix stored at packed rows row0.., columns col0.. of base
// (dst_cols columns, blocks of br rows x 64 columns, 128-byte swizzle).
struct UnpackSeg {
    long long e0;
    const uint16_t* base;
    int rows, cols, dst_cols, br, row0, col0;
};
// out[w * n_per + k] = element starts[w] + k (w < 3) of the stream (device arrays).
cudaError_t launch_unpack_samples(const UnpackSeg* segs, int n_segs, const long long* starts, int n_per,
                                  uint16_t* out, cudaStream_t s);

// context internals (runtime.cu)
int ctx_model_dims(const aos_ctx* c, uint32_t* n_layers, uint32_t* in_dims, uint32_t* out_dims, uint32_t* hidden,
                   uint32_t* vocab);
int ctx_fail(aos_ctx* c, int code, const std::string& msg);
cudaStream_t ctx_stream(aos_ctx* c);
int ctx_set_device(aos_ctx* c);
// aos_adapter_new with a separate scale: arena columns for storage_rank (a
// multiple of 8), LoRA scale = scale (alpha / rank of the adapter's config).
int ctx_adapter_new(aos_ctx* c, uint16_t id, uint32_t storage_rank, float alpha, float scale);

}  // namespace aos
