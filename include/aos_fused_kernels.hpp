// aos_fused_kernels.hpp — C++ host-side mirror of adapter-os's kernel API
// over the C ABI in aos_cuda.h (header only).
//
//   RouterRing    <- crates/adapteros-lora-kernel-api/src/lib.rs:58-214
//   IoBuffers     <- lib.rs:221-246
//   FusedKernels  <- lib.rs:308-716 (the trait a backend implements)
//   CudaKernels   <- the sm_100a backend (what kernel-mtl's MetalKernels,
//                    src/lib.rs:287-322, is for Metal)
//   Router        <- crates/adapteros-lora-router/src/router.rs:1517-1952,
//                    batched: one RouterRing per token
//
// Errors follow adapteros_core::AosError: every fallible call returns a
// Result with the C status and the backend's last-error text.
#pragma once

#include <cstdint>
#include <cstring>
#include <memory>
#include <stdexcept>
#include <string>
#include <utility>
#include <vector>

#include "aos_cuda.h"

namespace adapteros {

struct AosError {
    int code = AOS_OK;
    std::string message;
    bool ok() const { return code == AOS_OK; }
};

inline AosError status(int code, const aos_ctx* ctx = nullptr) {
    if (code == AOS_OK) return {};
    return AosError{code, aos_last_error(ctx)};
}

// RouterRing::set (lib.rs:140-193), release-build policy: mismatched lengths or
// an index >= max_adapter zero-fill the ring and set k = 0.
struct RouterRing {
    uint16_t indices[AOS_MAX_K] = {};
    int16_t gates_q15[AOS_MAX_K] = {};
    uint32_t position = 0;
    uint32_t k = 0;
    uint32_t dropout_seed = 0;
    float dropout_rate = 0.0f;

    void set(const std::vector<uint16_t>& idx, const std::vector<int16_t>& gates, uint16_t max_adapter = 0xFFFF) {
        std::memset(indices, 0, sizeof(indices));
        std::memset(gates_q15, 0, sizeof(gates_q15));
        k = 0;
        if (idx.size() != gates.size()) return;
        for (uint16_t i : idx)
            if (i >= max_adapter) return;
        const size_t n = idx.size() < AOS_MAX_K ? idx.size() : AOS_MAX_K;
        for (size_t j = 0; j < n; ++j) {
            indices[j] = idx[j];
            gates_q15[j] = gates[j];
        }
        k = (uint32_t)n;
    }
    aos_router_ring device_layout() const {
        aos_router_ring r{};
        r.top_k = k;
        r.position = position;
        std::memcpy(r.indices, indices, sizeof(indices));
        std::memcpy(r.gates_q15, gates_q15, sizeof(gates_q15));
        return r;
    }
};

struct IoBuffers {
    std::vector<uint32_t> input_ids;
    std::vector<float> output_logits;
    size_t position = 0;
    std::string session_id;
    explicit IoBuffers(size_t vocab = 0) : output_logits(vocab, 0.0f) {}
};

struct AdapterLoadMetadata {
    std::string adapter_id;
    uint32_t rank = 16;
    float alpha = 32.0f;
};

// One LoRA module's weights for one layer: A [rank, in], B [out, rank] (bf16 bits).
struct LoraModuleWeights {
    uint32_t layer;
    aos_module module;
    const uint16_t* A;
    const uint16_t* B;
};

class FusedKernels {
   public:
    virtual ~FusedKernels() = default;
    virtual AosError run_step(const RouterRing& ring, IoBuffers& io) = 0;
    virtual std::string device_name() const = 0;
    virtual AosError attest_determinism(aos_determinism_report* out) const = 0;
    virtual AosError load_adapter_with_metadata(uint16_t id, const std::vector<LoraModuleWeights>& weights,
                                                const AdapterLoadMetadata& meta) = 0;
    virtual AosError unload_adapter(uint16_t id) = 0;
    virtual AosError detach_adapter(uint16_t id) { return unload_adapter(id); }
    virtual AosError attach_adapter(uint16_t) { return {}; }
    virtual AosError switch_adapter(uint16_t) { return {}; }
    virtual bool supports_kv_cache() const { return false; }
    virtual void clear_session_cache(const std::string&) {}
    virtual void clear_all_caches() {}
    virtual size_t cache_memory_bytes() const { return 0; }
    virtual AosError health_check() { return {}; }
};

// The sm_100a backend.  Single-threaded per instance (the trait is used
// through &mut self).
class CudaKernels final : public FusedKernels {
   public:
    explicit CudaKernels(const aos_model_config& cfg) : cfg_(cfg), ctx_(aos_init(&cfg)) {
        if (!ctx_) throw std::runtime_error(std::string("aos_init: ") + aos_last_error(nullptr));
    }
    // FusedKernels::load(plan_bytes) (kernel-api/src/lib.rs:350): the model's
    // dimensions from the plan's tensor shapes (and `pc`, the plan crate's
    // model config, when given), the runtime sizes from `runtime`, then the
    // plan's base weights (aos_init_from_plan).  Throws with the reason.
    static std::unique_ptr<CudaKernels> from_plan(const std::vector<uint8_t>& plan, const aos_plan_config* pc,
                                                  const aos_model_config& runtime) {
        aos_model_config cfg = runtime;
        if (aos_model_config_from_plan(plan.data(), plan.size(), pc, &cfg) != AOS_OK)
            throw std::runtime_error(std::string("load: ") + aos_last_error(nullptr));
        aos_ctx* ctx = aos_init_from_plan(plan.data(), plan.size(), pc, &cfg);
        if (!ctx) throw std::runtime_error(std::string("load: ") + aos_last_error(nullptr));
        return std::unique_ptr<CudaKernels>(new CudaKernels(cfg, ctx));
    }
    ~CudaKernels() override { aos_destroy(ctx_); }
    CudaKernels(const CudaKernels&) = delete;
    CudaKernels& operator=(const CudaKernels&) = delete;

    aos_ctx* ctx() { return ctx_; }

    AosError load_weight(aos_weight_kind kind, uint32_t layer, aos_module m, const uint16_t* data, uint64_t n,
                         bool on_device = false) {
        return status(aos_load_weight(ctx_, kind, layer, m, data, n, on_device ? 1 : 0), ctx_);
    }

    AosError load_adapter_with_metadata(uint16_t id, const std::vector<LoraModuleWeights>& w,
                                        const AdapterLoadMetadata& meta) override {
        AosError e = status(aos_adapter_new(ctx_, id, meta.rank, meta.alpha), ctx_);
        if (!e.ok()) return e;
        for (const auto& m : w) {
            e = status(aos_adapter_set_module(ctx_, id, m.layer, m.module, m.A, m.B, 0), ctx_);
            if (!e.ok()) {
                aos_adapter_unload(ctx_, id);
                return e;
            }
        }
        return {};
    }
    AosError unload_adapter(uint16_t id) override { return status(aos_adapter_unload(ctx_, id), ctx_); }

    // Batched step: one decode token per (ring, token, sequence).
    AosError run_step_batch(const std::vector<RouterRing>& rings, const std::vector<uint32_t>& tokens,
                            const std::vector<uint64_t>& seqs, float* logits) {
        std::vector<aos_router_ring> r(rings.size());
        for (size_t i = 0; i < rings.size(); ++i) r[i] = rings[i].device_layout();
        return status(aos_run_step_batch(ctx_, r.data(), tokens.data(), seqs.data(), (uint32_t)r.size(), logits,
                                         nullptr),
                      ctx_);
    }

    // Prompt pass on device buffers (aos_prefill_dev): sequence i takes
    // n_tok[i] tokens from its current length on; rings / tokens are device
    // arrays concatenated over the sequences, logits device [n_seq][vocab].
    AosError prefill_dev(const std::vector<uint64_t>& seqs, const std::vector<uint32_t>& n_tok,
                         const aos_router_ring* rings_dev, const uint32_t* tokens_dev, float* logits_dev,
                         void* stream = nullptr) {
        if (seqs.size() != n_tok.size()) return AosError{AOS_ERR_INVALID, "seqs and n_tok differ in length"};
        return status(aos_prefill_dev(ctx_, (uint32_t)seqs.size(), seqs.data(), n_tok.data(), rings_dev, tokens_dev,
                                      logits_dev, stream),
                      ctx_);
    }

    // .aos archive into adapter slot id (LifecycleLoader::load_from_aos_static
    // + the MLX adapter rules); backend: "mlx", "metal", "coreml", "canonical".
    AosError load_adapter_aos(uint16_t id, const std::vector<uint8_t>& archive, const char* backend = "canonical",
                              aos_archive_load_info* info = nullptr) {
        return status(aos_adapter_load_aos(ctx_, id, archive.data(), archive.size(), backend, info), ctx_);
    }

    // FusedKernels::verify_adapter_buffers / store_gpu_fingerprint /
    // verify_gpu_fingerprint (kernel-api/src/lib.rs:440-508).
    AosError verify_adapter_buffers(uint16_t id, uint64_t* bytes, std::vector<uint8_t>& first,
                                    std::vector<uint8_t>& last, std::vector<uint8_t>& mid) {
        first.assign(4096, 0);
        last.assign(4096, 0);
        mid.assign(4096, 0);
        uint32_t n = 0;
        AosError e = status(aos_adapter_verify_buffers(ctx_, id, bytes, first.data(), last.data(), mid.data(), &n),
                            ctx_);
        first.resize(n);
        last.resize(n);
        mid.resize(n);
        return e;
    }
    AosError store_gpu_fingerprint(uint16_t id, uint64_t bytes, const std::string& hex) {
        return status(aos_store_gpu_fingerprint(ctx_, id, bytes, hex.c_str()), ctx_);
    }
    AosError verify_gpu_fingerprint(uint16_t id, uint64_t bytes, const std::string& hex, bool* matches) const {
        int m = 0;
        AosError e = status(aos_verify_gpu_fingerprint(ctx_, id, bytes, hex.c_str(), &m), ctx_);
        *matches = m != 0;
        return e;
    }

    // FusedKernels::check_memory_footprint: within 2 sigma of the adapter's
    // footprint baseline (kernel-mtl/src/vram.rs:386-407).
    AosError check_memory_footprint(uint16_t id, uint64_t bytes, bool* within, double* z_score) {
        int w = 0;
        AosError e = status(aos_check_memory_footprint(ctx_, id, bytes, &w, z_score, nullptr, nullptr, nullptr), ctx_);
        *within = w != 0;
        return e;
    }
    // FusedKernels::memory_report (kernel-api/src/lib.rs:588-593).
    AosError memory_report(aos_memory_report_data* out, std::vector<aos_adapter_allocation>* allocs = nullptr) {
        uint32_t n = 0;
        AosError e = status(aos_memory_report(ctx_, out, nullptr, 0, &n), ctx_);
        if (e.ok() && allocs) {
            allocs->resize(n);
            e = status(aos_memory_report(ctx_, out, allocs->data(), n, &n), ctx_);
        }
        return e;
    }
    // KvCache generation guards (crates/adapteros-lora-worker/src/kvcache.rs:288-402).
    AosError ensure_cache_coherence(uint64_t generation, bool* reset) {
        int r = 0;
        AosError e = status(aos_kv_ensure_coherence(ctx_, generation, &r), ctx_);
        if (reset) *reset = r != 0;
        return e;
    }
    AosError zeroize_sequence(uint64_t seq) { return status(aos_kv_zeroize(ctx_, seq), ctx_); }

    // Next tokens of device logits rows (Generator::next_token / greedy on the
    // device); u: device uniform draws, one per row (the caller's RNG).
    static AosError sample_dev(const float* logits_dev, uint32_t rows, uint32_t vocab, const aos_sample_params& p,
                               const float* u_dev, uint32_t* tokens_dev, void* stream = nullptr) {
        return status(aos_sample_dev(logits_dev, rows, vocab, vocab, &p, u_dev, tokens_dev, stream), nullptr);
    }

    // Adapter-sharded decode: join the group once (collective), then every
    // rank calls run_step_sharded_dev with the same number of home tokens.
    AosError shard_init(uint32_t rank, uint32_t world, const void* unique_id) {
        return status(aos_shard_init(ctx_, rank, world, unique_id), ctx_);
    }
    AosError run_step_sharded_dev(const aos_router_ring* rings_dev, const uint32_t* tokens_dev,
                                  const std::vector<uint64_t>& seqs, float* logits_dev, void* stream = nullptr) {
        return status(aos_run_step_sharded_dev(ctx_, rings_dev, tokens_dev, seqs.data(), (uint32_t)seqs.size(),
                                               logits_dev, nullptr, stream),
                      ctx_);
    }

    // FusedKernels::run_step: io.input_ids at io.position of the
    // io.session_id sequence -- one id is a decode token (aos_run_step_batch),
    // several are a prompt pass with causal attention (aos_prefill), the ring
    // applying to each; logits of the last token; position advances by
    // input_ids.size() (mlx-ffi/src/backend.rs:1212-1310).
    AosError run_step(const RouterRing& ring, IoBuffers& io) override {
        if (io.input_ids.empty()) return AosError{AOS_ERR_INVALID, "Input token IDs cannot be empty"};
        uint64_t seq = session(io.session_id);
        AosError e = status(aos_kv_set_len(ctx_, seq, (uint32_t)io.position), ctx_);
        if (!e.ok()) return e;
        std::vector<float> logits(cfg_.vocab);
        const aos_router_ring r = ring.device_layout();
        if (io.input_ids.size() == 1) {
            e = status(aos_run_step_batch(ctx_, &r, io.input_ids.data(), &seq, 1, logits.data(), nullptr), ctx_);
        } else {
            const std::vector<aos_router_ring> rings(io.input_ids.size(), r);
            const uint32_t n = (uint32_t)io.input_ids.size();
            e = status(aos_prefill(ctx_, 1, &seq, &n, rings.data(), io.input_ids.data(), logits.data()), ctx_);
        }
        if (!e.ok()) return e;
        const size_t n = io.output_logits.size() < logits.size() ? io.output_logits.size() : logits.size();
        std::memcpy(io.output_logits.data(), logits.data(), n * sizeof(float));
        io.position += io.input_ids.size();
        return {};
    }

    std::string device_name() const override { return aos_device_name(ctx_); }
    AosError attest_determinism(aos_determinism_report* out) const override {
        return status(aos_attest_determinism(ctx_, out), ctx_);
    }
    bool supports_kv_cache() const override { return true; }
    void clear_session_cache(const std::string& sid) override {
        for (auto it = sessions_.begin(); it != sessions_.end(); ++it)
            if (it->first == sid) {
                aos_kv_free(ctx_, it->second);
                sessions_.erase(it);
                return;
            }
    }
    void clear_all_caches() override {
        aos_kv_clear_all(ctx_);
        sessions_.clear();
    }
    size_t cache_memory_bytes() const override { return (size_t)aos_kv_memory_bytes(ctx_); }
    AosError health_check() override { return status(aos_health_check(ctx_), ctx_); }

   private:
    CudaKernels(const aos_model_config& cfg, aos_ctx* ctx) : cfg_(cfg), ctx_(ctx) {}
    uint64_t session(const std::string& sid) {
        for (auto& kv : sessions_)
            if (kv.first == sid) return kv.second;
        const uint64_t id = (1ull << 62) + sessions_.size();
        if (aos_kv_alloc(ctx_, id, cfg_.max_seq_len) != AOS_OK)
            throw std::runtime_error(aos_last_error(ctx_));
        sessions_.emplace_back(sid, id);
        return id;
    }
    aos_model_config cfg_;
    aos_ctx* ctx_;
    std::vector<std::pair<std::string, uint64_t>> sessions_;
};

// Batched router (router.rs:1517-1952): one RouterRing per token.
class Router {
   public:
    Router(uint32_t k, float tau, float eps) : p_{k, tau, eps, 1.0f} {}
    void set_routing_bias(float b) { p_.routing_bias = b; }  // router.rs:556-561 (sanitised in the kernel call)
    AosError route_batch(const float* priors, uint32_t T, uint32_t N, const uint64_t* stable_ids,
                         std::vector<RouterRing>& out, const float* version_weights = nullptr,
                         const uint8_t* allowed = nullptr) const {
        std::vector<aos_router_ring> r(T);
        AosError e =
            status(aos_route_batch(priors, stable_ids, version_weights, allowed, nullptr, T, N, &p_, r.data(), nullptr,
                                   nullptr));
        out.resize(T);
        for (uint32_t t = 0; t < T; ++t) {
            out[t].k = r[t].top_k;
            out[t].position = r[t].position;
            std::memcpy(out[t].indices, r[t].indices, sizeof(r[t].indices));
            std::memcpy(out[t].gates_q15, r[t].gates_q15, sizeof(r[t].gates_q15));
        }
        return e;
    }

   private:
    aos_router_params p_;
};

}  // namespace adapteros
