/*
 * aos_cuda.h — C ABI of the B200 (sm_100a) backend for adapter-os's per-token
 * hot path: batched K-sparse router, fused base + gathered-LoRA projections,
 * SwiGLU MLP and paged-KV decode attention.
 *
 * The ABI is what a `FusedKernels` implementation
 * (crates/adapteros-lora-kernel-api/src/lib.rs:308-716) calls through a thin
 * extern "C" FFI crate; conventions follow the MLX C wrapper
 * (crates/adapteros-lora-mlx-ffi/wrapper.h): opaque handles, int status codes
 * and a per-handle last-error string.
 *
 * Rules shared by every entry point:
 *   - Status: 0 = AOS_OK, negative = error (see aos_status); the message is in
 *     aos_last_error(ctx) (or aos_last_error(NULL) for context-free calls).
 *   - There is no CPU fallback: with no usable sm_100 device every compute
 *     entry point fails with AOS_ERR_NO_DEVICE.
 *   - `_dev` entry points take device pointers and enqueue on `stream` (a
 *     cudaStream_t, NULL = the context's stream); the others take host
 *     pointers and return when the result is in host memory.
 *   - A context is single-threaded (the Rust side serialises calls with
 *     &mut self, lib.rs:371); distinct contexts may be used concurrently.
 */
#ifndef AOS_CUDA_H
#define AOS_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define AOS_MAX_K 8             /* adapteros-core/src/defaults.rs:37 MAX_K */
#define AOS_Q15_DENOM 32767.0f  /* adapteros-lora-router/src/quantization.rs:22 */
#define AOS_NUM_MODULES 7

typedef enum aos_status {
    AOS_OK = 0,
    AOS_ERR_INVALID = -1,    /* AosError::Validation: bad argument or shape        */
    AOS_ERR_CUDA = -2,       /* AosError::Kernel: a CUDA call or kernel failed      */
    AOS_ERR_NOMEM = -3,      /* arena / KV pool / device allocation exhausted      */
    AOS_ERR_NONFINITE = -4,  /* AosError::DeterminismViolation: NaN/Inf router input */
    AOS_ERR_NOT_FOUND = -5,  /* unknown adapter id / sequence id                  */
    AOS_ERR_TIMEOUT = -6,    /* a bounded device-side wait ran out                */
    AOS_ERR_NO_DEVICE = -7,  /* no sm_100 device: there is no CPU fallback         */
    AOS_ERR_STATE = -8       /* call out of order (e.g. step before weights load)  */
} aos_status;

/* Module ids, in the order of MLXLoraLayer (mlx_cpp_wrapper_real.cpp:1248-1256). */
typedef enum aos_module {
    AOS_MOD_Q = 0, AOS_MOD_K = 1, AOS_MOD_V = 2, AOS_MOD_O = 3,
    AOS_MOD_GATE = 4, AOS_MOD_UP = 5, AOS_MOD_DOWN = 6
} aos_module;

/* Base-weight kinds for aos_load_weight. */
typedef enum aos_weight_kind {
    AOS_W_EMBED = 0,      /* [vocab, hidden]                                     */
    AOS_W_LM_HEAD = 1,    /* [vocab, hidden]                                     */
    AOS_W_FINAL_NORM = 2, /* [hidden]                                            */
    AOS_W_ATTN_NORM = 3,  /* [hidden] per layer (input_layernorm)                */
    AOS_W_MLP_NORM = 4,   /* [hidden] per layer (post_attention_layernorm)       */
    AOS_W_PROJ = 5        /* [out, in] per layer and module (q..down, nn.Linear) */
} aos_weight_kind;

/* RouterRing device layout, 40 bytes
 * (kernel-mtl/src/ring_buffer.rs:44-58; kernel-api/src/lib.rs:58-75).
 * Unused entries are zero-filled (RouterRing::set, lib.rs:188-192). */
typedef struct aos_router_ring {
    uint32_t top_k;
    uint32_t position;
    uint16_t indices[AOS_MAX_K];
    int16_t gates_q15[AOS_MAX_K];
} aos_router_ring;

/* Router parameters; sanitised like Router::new_with_weights
 * (router.rs:397-400 via sanitize_k/eps/tau, :127-187) and set_routing_bias
 * (:556-561).  Features are empty, so feature scores are 0 (router.rs:985-988). */
typedef struct aos_router_params {
    uint32_t k;          /* 0 -> 1, > 8 -> 8                                   */
    float tau;           /* non-finite or <= 0 -> 1.0                          */
    float eps;           /* non-finite or outside [0,1] -> 0.02                */
    float routing_bias;  /* non-finite or <= 0 -> 1.0                          */
} aos_router_params;

/* Decoder shape and resource sizing for a context. */
typedef struct aos_model_config {
    uint32_t hidden, n_heads, n_kv_heads, head_dim, intermediate, vocab, n_layers;
    float rms_eps;
    float rope_theta;
    uint32_t rope_mlx_as_written; /* 1: inv_freq = 1/theta^(-2i/hd) as MLX code writes it */
    uint32_t max_batch;           /* tokens per decode step (<= 256)                      */
    uint32_t kv_block_size;       /* tokens per KV page; must be 16                        */
    uint32_t kv_num_blocks;       /* KV pages per layer in the pool                        */
    uint32_t max_seq_len;         /* longest sequence (tokens)                             */
    uint32_t lora_rank_capacity;  /* rank columns in the adapter arena (rounded up to 64)   */
    uint32_t lora_max_adapters;   /* adapter ids are < this (<= 65535)                     */
    uint32_t lora_module_mask;    /* bit m: module m may carry LoRA (0 = all seven)        */
    int32_t device;               /* CUDA ordinal                                          */
} aos_model_config;

typedef struct aos_metrics {           /* BackendMetrics (kernel-api/src/lib.rs:28-39) */
    uint64_t steps, tokens, route_calls;
    uint64_t base_weight_bytes, arena_bytes, arena_used_rank_cols, kv_pool_bytes;
    uint32_t adapters_loaded, kv_blocks_used, kv_blocks_total, sequences;
    float last_step_ms;
} aos_metrics;

typedef struct aos_determinism_report { /* DeterminismReport, attestation.rs:130-160 */
    char backend[32];
    char device_name[64];
    uint32_t sm_major, sm_minor;
    uint32_t fast_math;             /* 0: built without fast-math                     */
    uint32_t float_atomics;         /* 0: no floating-point atomics on any path       */
    uint32_t fixed_reduction_order; /* 1: every split reduction has a fixed order     */
    char kernel_build_id[65];       /* kernel hash: SHA-256 (hex) of every kernel source and
                                       header plus the compiler flags, fixed at build time
                                       (the role of the Metal backend's metallib_hash) */
    char compiler_flags[512];       /* the nvcc flags, space separated                */
    char runtime_version[64];       /* CUDA runtime and driver versions               */
    char device_id[64];             /* "cuda:<ordinal> <PCI bus id>"                  */
    uint32_t rng_seed_method;       /* 0 HkdfSeeded (RngSeedingMethod)                */
    uint32_t floating_point_mode;   /* 0 Deterministic (FloatingPointMode)            */
    uint32_t determinism_level;     /* 2 BitExact (DeterminismLevel: 0 None, 1 Bounded) */
    uint32_t deterministic;         /* 1                                              */
} aos_determinism_report;

typedef struct aos_ctx aos_ctx;
/* GpuMemoryReportData (kernel-api/src/lib.rs:732-758) */
typedef struct aos_memory_report_data {
    uint64_t total_gpu_bytes, used_gpu_bytes;      /* cudaMemGetInfo of the context's device  */
    uint32_t adapter_count;
    uint64_t adapter_vram_total;                   /* arena bytes held by the loaded adapters */
    uint64_t arena_bytes, arena_used_bytes;        /* the LoRA arena (pool) and its used part */
    uint64_t kv_pool_bytes, kv_used_bytes;         /* KV pages held by sequences              */
} aos_memory_report_data;
typedef struct aos_adapter_allocation { uint32_t adapter_id; uint64_t bytes; } aos_adapter_allocation;

/* ---- library ------------------------------------------------------------ */
const char* aos_version(void);
/* Number of sm_100 devices visible (0 when none). */
int aos_device_count(void);
/* Last error of a context, or of context-free calls when ctx is NULL
 * (mlx_get_last_error, wrapper.h:199-200). */
const char* aos_last_error(const aos_ctx* ctx);

/* ---- batched router (crates/adapteros-lora-router/src/router.rs:1567-1952) ----
 * One RouterRing per token: scores = ((prior + 0) - 0) * bias * clamp(vw,0,2),
 * total-order sort DESC with stable_id ASC tie-break (:234-264), top-K,
 * f64 Kahan softmax (:1340-1411), entropy floor eps/K and f32 renormalise
 * (:1818-1842), Q15 round-half-away (quantization.rs:172-175), canonical order
 * (q15 DESC, score DESC, stable_id ASC, idx ASC; :1310-1325).  Bit-exact with
 * the reference.  priors: [T, N]; stable_ids: [N]; version_weights: [N] or
 * NULL; allowed: [N] (0/1) or NULL; positions: [T] or NULL (ring.position);
 * entropy: [T] or NULL; status: [T] or NULL (0 or AOS_ERR_NONFINITE).  A
 * token whose inputs are non-finite gets an empty ring and the call returns
 * AOS_ERR_NONFINITE.  N <= 4096. */
int aos_route_batch(const float* priors, const uint64_t* stable_ids, const float* version_weights,
                    const uint8_t* allowed, const uint32_t* positions, uint32_t T, uint32_t N,
                    const aos_router_params* params, aos_router_ring* rings, float* entropy,
                    int32_t* status);
/* Device-pointer form; enqueued on `stream`, no host synchronisation.
 * Per-token errors are only reported through `status`. */
int aos_route_batch_dev(const float* priors, const uint64_t* stable_ids,
                        const float* version_weights, const uint8_t* allowed,
                        const uint32_t* positions, uint32_t T, uint32_t N,
                        const aos_router_params* params, aos_router_ring* rings, float* entropy,
                        int32_t* status, void* stream);

/* ---- fp32 LoRA op (config 1) ---------------------------------------------
 * y[t] = W x[t] + sum over ring slots with q15 > 0 of
 *        (q15/32767 * (B_a (A_a x[t]))) * (alpha_a / rank)
 * (kernel_testing.rs:220-257 cpu_lora_forward; liquid.rs:222-250 blend loop;
 *  gate dequant mlx-ffi/src/backend.rs:405-418).  x: [T, in]; W: [out, in];
 * A: [n_adapters, rank, in]; B: [n_adapters, out, rank]; alpha: [n_adapters]
 * or NULL (alpha = rank); rings: [T]; y: [T, out].  rank <= 64, in % 4 == 0;
 * on device, x and A must be 16-byte aligned (AOS_ERR_INVALID otherwise). */
int aos_lora_op_f32(const float* x, uint32_t T, uint32_t in_dim, uint32_t out_dim,
                    const float* W, const float* A, const float* B, uint32_t n_adapters,
                    uint32_t rank, const float* alpha, const aos_router_ring* rings, float* y);
int aos_lora_op_f32_dev(const float* x, uint32_t T, uint32_t in_dim, uint32_t out_dim,
                        const float* W, const float* A, const float* B, uint32_t n_adapters,
                        uint32_t rank, const float* alpha, const aos_router_ring* rings, float* y,
                        void* stream);

/* The op of aos_lora_op_f32_dev, for callers that must not allocate device
 * memory (no counterpart in the reference).  Hosts with a device-memory budget
 * fixed at start-up, code sharing a device with an open CUDA graph capture
 * (cudaMalloc/cudaFree synchronise the device and are illegal while a capture
 * is open) and latency-critical loops can call this one: its scratch is a
 * fixed 512 KiB device array in the library (131072 floats, held on every
 * device that loads the library until exit), not an allocation.  Requires
 * T * 8 * rank <= 131072, otherwise AOS_ERR_INVALID; same argument rules as
 * aos_lora_op_f32_dev.  Its base GEMM is one single-pass kernel over all of K
 * (aos_lora_op_f32_dev sums eight K-eighth partials), so the two agree within
 * fp32 tolerance, not bit for bit; each is bit-identical run to run.  The
 * first call in each CUDA context on a device looks up the array's address
 * (cudaGetSymbolAddress) and should be made before any stream capture on that
 * device.  All calls share the array: calls that overlap on the GPU race, so
 * serialise them (one stream).  It calls no cudaMalloc, cudaFree or
 * allocating library routine. */
int aos_lora_op_f32_noalloc_dev(const float* x, uint32_t T, uint32_t in_dim, uint32_t out_dim,
                                const float* W, const float* A, const float* B, uint32_t n_adapters,
                                uint32_t rank, const float* alpha, const aos_router_ring* rings,
                                float* y, void* stream);

/* ---- context: FusedKernels::load + hot-swap arena + KV cache ------------- */
/* Create a backend on cfg->device; allocates the KV pool, adapter arena and
 * step scratch up front (kernel-mtl/src/lib.rs:1476-1537 load).
 * The decode projection GEMMs run one CTA per SM and wait on one another
 * inside the launch; init checks that every SM can hold one such CTA.  By
 * default they are plain launches, which assumes no other kernel occupies the
 * device's SMs during a step (otherwise a step ends with AOS_ERR_TIMEOUT after
 * about a second).  With AOS_GEMM_COOPERATIVE=1 in the environment at init
 * they are cooperative launches, which the driver starts only with the whole
 * grid resident (shared-device mode, about 3% slower per step: they give up
 * the overlap with the neighbouring launches).  Results are bit-identical in
 * both modes. */
aos_ctx* aos_init(const aos_model_config* cfg);
void aos_destroy(aos_ctx* ctx);
/* FusedKernels::device_name (lib.rs:374). */
const char* aos_device_name(const aos_ctx* ctx);
/* The context's CUDA stream (cudaStream_t). */
void* aos_stream(aos_ctx* ctx);

/* Load one bf16 base tensor (the plan's safetensors entries,
 * kernel-mtl/src/lib.rs:660-1135).  layer is ignored for EMBED/LM_HEAD/
 * FINAL_NORM; module is used only for AOS_W_PROJ.  data holds the tensor in
 * row-major [out, in] (nn.Linear) order; src_on_device = 1 if it is a device
 * pointer.  n_elems must match the configured shape. */
int aos_load_weight(aos_ctx* ctx, aos_weight_kind kind, uint32_t layer, aos_module module,
                    const uint16_t* data, uint64_t n_elems, int src_on_device);

/* Adapter arena (FusedKernels::load_adapter_with_metadata / unload_adapter,
 * lib.rs:388-432; MLX mlx_lora_adapter_new / _set_module, wrapper.h:383-397).
 * aos_adapter_new reserves `rank` arena columns for id (rank % 8 == 0,
 * 8 <= rank <= 256); scale = alpha / rank.  Modules that are never set stay
 * zero (contribute nothing). */
int aos_adapter_new(aos_ctx* ctx, uint16_t id, uint32_t rank, float alpha);
/* A: [rank, in] (lora_A), B: [out, rank] (lora_B), bf16, for one layer/module. */
int aos_adapter_set_module(aos_ctx* ctx, uint16_t id, uint32_t layer, aos_module module,
                           const uint16_t* A, const uint16_t* B, int src_on_device);
int aos_adapter_unload(aos_ctx* ctx, uint16_t id);
/* 1 if id is resident, else 0. */
int aos_adapter_is_loaded(const aos_ctx* ctx, uint16_t id);

/* Paged KV cache (replaces the first-fit contiguous allocator of
 * crates/adapteros-lora-worker/src/kvcache.rs:112-524 with 16-token pages). */
int aos_kv_alloc(aos_ctx* ctx, uint64_t seq_id, uint32_t max_tokens);
int aos_kv_free(aos_ctx* ctx, uint64_t seq_id);
/* Declare `len` tokens already cached for seq (their K/V written by
 * aos_kv_write or aos_kv_fill_synthetic). */
int aos_kv_set_len(aos_ctx* ctx, uint64_t seq_id, uint32_t len);
int aos_kv_get_len(const aos_ctx* ctx, uint64_t seq_id, uint32_t* len);
/* Write K/V rows [n_tokens, n_kv_heads, head_dim] bf16 for positions
 * pos0..pos0+n_tokens-1 of one layer. */
int aos_kv_write(aos_ctx* ctx, uint64_t seq_id, uint32_t layer, uint32_t pos0, uint32_t n_tokens,
                 const uint16_t* k, const uint16_t* v, int src_on_device);
int aos_kv_read(aos_ctx* ctx, uint64_t seq_id, uint32_t layer, uint32_t pos0, uint32_t n_tokens,
                uint16_t* k, uint16_t* v);
/* Fill every page of the pool with seeded synthetic bf16 values ~N(0, std). */
int aos_kv_fill_synthetic(aos_ctx* ctx, uint64_t seed, float std);
/* Sliding-window rotate (kv_cache.metal:200-236 kv_cache_rotate): drops the
 * sequence's oldest `shift` positions; position i then holds the K/V rows of
 * old position i + shift in every layer, and the length is len - shift (the
 * capacity is kept).  Rows are moved as stored: the keys keep the rotary
 * angle of their old positions, as in the shader.  shift > len is
 * AOS_ERR_INVALID; shift 0 does nothing. */
int aos_kv_rotate(aos_ctx* ctx, uint64_t seq_id, uint32_t shift);
/* FusedKernels::clear_all_caches / cache_memory_bytes (lib.rs:536-554). */
int aos_kv_clear_all(aos_ctx* ctx);
uint64_t aos_kv_memory_bytes(const aos_ctx* ctx);
/* KvCache's generation guards and zeroization (crates/adapteros-lora-worker/
 * src/kvcache.rs:288-402, 586-733).  ensure_coherence: when the generation
 * differs, every sequence is released and both pools are zeroed (reset_all),
 * *reset = 1.  alloc_guarded: ensure_coherence, then aos_kv_alloc, recording
 * the sequence's generation.  has_stale_guards: 1 when a guarded sequence was
 * allocated under another generation.  drain_guarded: releases every guarded
 * sequence.  zeroize: zeroes one sequence's K/V pages in every layer (the
 * sequence stays allocated); zeroize_all: both pools to zero, every sequence
 * released. */
int aos_kv_set_generation(aos_ctx* ctx, uint64_t generation);
uint64_t aos_kv_generation(const aos_ctx* ctx);
int aos_kv_ensure_coherence(aos_ctx* ctx, uint64_t generation, int* reset);
int aos_kv_alloc_guarded(aos_ctx* ctx, uint64_t seq_id, uint32_t max_tokens, uint64_t generation);
int aos_kv_has_stale_guards(const aos_ctx* ctx, uint64_t generation);
int aos_kv_drain_guarded(aos_ctx* ctx, uint32_t* n_drained);
int aos_kv_zeroize(aos_ctx* ctx, uint64_t seq_id);
int aos_kv_zeroize_all(aos_ctx* ctx);

/* ---- the step (FusedKernels::run_step, batched; lib.rs:371) --------------
 * One decode token per entry: rings[t] selects the adapters for token t,
 * token_ids[t] is its input id and seq_ids[t] its sequence (each at most once
 * per call).  Runs embedding -> n_layers x [RMSNorm -> q/k/v + LoRA -> RoPE ->
 * paged-KV append -> GQA attention -> o + LoRA -> residual -> RMSNorm ->
 * gate/up + LoRA -> SwiGLU -> down + LoRA -> residual] -> final RMSNorm ->
 * lm_head (mlx_cpp_wrapper_real.cpp:3338-3559) and advances each sequence
 * by one token (IoBuffers.position += 1, mlx-ffi/src/backend.rs:1292).
 * logits: [T, vocab] f32 or NULL; hidden_out: [T, hidden] bf16 (the final
 * hidden state before the final norm) or NULL. */
int aos_run_step_batch(aos_ctx* ctx, const aos_router_ring* rings, const uint32_t* token_ids,
                       const uint64_t* seq_ids, uint32_t T, float* logits, uint16_t* hidden_out);
/* Device-pointer form (rings, token_ids, logits, hidden_out on the device;
 * seq_ids stays a host array because it drives the page tables). */
int aos_run_step_batch_dev(aos_ctx* ctx, const aos_router_ring* rings, const uint32_t* token_ids,
                           const uint64_t* seq_ids, uint32_t T, float* logits,
                           uint16_t* hidden_out, void* stream);
/* One decoder layer on a caller-provided hidden state (config 2): hidden is
 * [T, hidden] bf16 on the device, updated in place; sequences advance only
 * if advance != 0. */
int aos_layer_step_dev(aos_ctx* ctx, uint32_t layer, const aos_router_ring* rings,
                       const uint64_t* seq_ids, uint32_t T, uint16_t* hidden, int advance,
                       void* stream);

/* ---- loading from safetensors bytes ------------------------------------------
 * Adapters (FusedKernels::load_adapter_with_metadata,
 * kernel-mtl/src/lib.rs:1893-2046): for every target module, the first tensor
 * name in sorted order that contains the module name and "lora_A" (resp.
 * "lora_B"); a name with ".layers.<L>." belongs to layer L, one without to
 * layer 0.  Target modules: meta->target_modules (trimmed, empty and repeated
 * names dropped) or, when absent or matching nothing, q_proj, k_proj, v_proj,
 * down_proj, up_proj.  Rank: meta->rank if > 0, else lora_A's first dimension,
 * else 16; alpha: meta->alpha if finite and > 0, else 2 * rank.  F32, F16 and
 * BF16 tensors are stored as bf16.  meta may be NULL. */
typedef struct aos_adapter_meta {
    uint32_t rank;
    float alpha;
    const char* const* target_modules;
    uint32_t n_targets;
} aos_adapter_meta;
/* Context-free: the rank / alpha the load would use and, per layer and module
 * (found[layer * 7 + module]), bit 0 = lora_A found, bit 1 = lora_B found. */
int aos_adapter_probe_safetensors(const void* data, uint64_t len, const aos_adapter_meta* meta,
                                  uint32_t n_layers, uint32_t* rank_out, float* alpha_out,
                                  uint32_t* found);
int aos_adapter_load_safetensors(aos_ctx* ctx, uint16_t id, const void* data, uint64_t len,
                                 const aos_adapter_meta* meta);
/* Base weights under the Hugging Face LLaMA names (kernel-mtl/src/lib.rs:660-1000):
 * model.embed_tokens, lm_head (tied to the embedding when absent), model.norm,
 * model.layers.<L>.{input_layernorm, post_attention_layernorm,
 * self_attn.{q,k,v,o}_proj, mlp.{gate,up,down}_proj}.weight. */
int aos_load_model_safetensors(aos_ctx* ctx, const void* data, uint64_t len);

/* ---- model plan: FusedKernels::load(plan_bytes) ---------------------------
 * The plan crate's ModelConfig (crates/adapteros-lora-plan/src/config.rs:9-62)
 * as ModelConfig::from_json reads it (required: name, architecture,
 * hidden_size, intermediate_size, num_hidden_layers, num_attention_heads,
 * num_key_value_heads, max_position_embeddings, rope_theta, vocab_size;
 * optional: rope_scaling_factor, rope_scaling {factor,
 * original_max_position_embeddings, scaling_type}; other fields ignored),
 * plus its derived values: dimensions() (:171-193), effective_context_length()
 * (:201-208) and is_qwen2_5() (:196-198). */
typedef struct aos_plan_config {
    char name[128];
    char architecture[128];
    uint32_t hidden_size, intermediate_size, num_hidden_layers;
    uint32_t num_attention_heads, num_key_value_heads, max_position_embeddings, vocab_size;
    float rope_theta;
    uint32_t has_rope_scaling_factor; /* Option<f32> rope_scaling_factor               */
    float rope_scaling_factor;
    uint32_t has_rope_scaling;        /* Option<RopeScaling> rope_scaling              */
    float scaling_factor;
    uint32_t scaling_original_max_position_embeddings;
    char scaling_type[64];
    float rms_norm_eps;               /* "rms_norm_eps" when the JSON carries it, else 0 */
    uint32_t head_dim, kv_width;      /* hidden / heads (0 when heads == 0), kv_heads * head_dim */
    uint64_t total_params;            /* dimensions().total_params                     */
    uint32_t effective_context_length;
    uint32_t is_qwen2_5;
} aos_plan_config;
/* ModelConfig::from_json (config.rs:80-86): AOS_ERR_INVALID with
 * aos_last_error(NULL) = "Failed to parse model config: ..." (missing field,
 * wrong type, malformed JSON). */
int aos_plan_config_parse(const char* json, uint64_t len, aos_plan_config* out);
/* ModelConfig::validate (config.rs:127-167) and validate_gqa (:101-124), with
 * the reference's messages in aos_last_error(NULL). */
int aos_plan_config_validate(const aos_plan_config* cfg);
int aos_plan_config_validate_gqa(const aos_plan_config* cfg);
/* validate_lora_targets (config.rs:256-277) and calculate_lora_size
 * (:212-253): fp16 bytes of a rank-`rank` adapter on `targets` over every layer. */
int aos_plan_validate_lora_targets(const char* const* targets, uint32_t n);
int aos_plan_lora_size(const aos_plan_config* cfg, uint32_t rank, const char* const* targets, uint32_t n,
                       uint64_t* bytes);
/* Dimension inference of FusedKernels::load (kernel-mtl/src/lib.rs:1476-1537,
 * validate_embedding_dimensions :790-839): vocab and hidden from the plan's
 * embedding tensor [vocab, hidden] (first of model.embed_tokens.weight,
 * transformer.wte.weight, embeddings.word_embeddings.weight,
 * embed_tokens.weight, wte.weight); layers from model.layers.<l>.*; the MLP
 * width from mlp.gate_proj; heads, KV heads, head_dim, rope_theta and
 * rms_norm_eps from `pc` when given (checked against the tensor shapes), else
 * GqaConfig::default() (head_dim 128, rope_theta 10000; fused_qkv.rs:41-54).
 * Fills those fields of *cfg and leaves its runtime fields (batch, KV pool,
 * adapter arena, device) as the caller set them.  Context-free, no device. */
int aos_model_config_from_plan(const void* plan, uint64_t len, const aos_plan_config* pc, aos_model_config* cfg);
/* FusedKernels::load(plan_bytes): the dimensions above with the runtime
 * fields of *runtime, aos_init, then aos_load_model_safetensors of the plan.
 * NULL on failure (aos_last_error(NULL)). */
aos_ctx* aos_init_from_plan(const void* plan, uint64_t len, const aos_plan_config* pc, const aos_model_config* runtime);

/* ---- .aos adapter archives -------------------------------------------------
 * Layout and validation of crates/adapteros-aos/src/writer.rs:118-135,
 * 407-558: 64-byte header, 80-byte index entries, payloads, JSON manifest. */
typedef struct aos_archive_segment {
    uint32_t segment_id;
    uint16_t backend_tag; /* 0 canonical, 1 mlx, 2 metal, 3 coreml (writer.rs:41-71) */
    uint16_t reserved;
    uint64_t offset;
    uint64_t len;
    uint8_t scope_hash[16];   /* first 16 bytes of BLAKE3(manifest metadata.scope_path) */
    uint8_t weights_hash[32]; /* BLAKE3 of the payload */
} aos_archive_segment;
typedef struct aos_archive_info {
    uint32_t flags;
    uint32_t n_segments;
    uint64_t manifest_offset;
    uint64_t manifest_size;
} aos_archive_info;
/* Context-free layout check (AosWriter::parse_header_bytes + parse_segments
 * without the hash check, same rules and messages); copies up to max_segs
 * index entries.  AOS_ERR_INVALID with aos_last_error(NULL) on a bad layout. */
int aos_archive_parse(const void* data, uint64_t len, aos_archive_info* info, aos_archive_segment* segs,
                      uint32_t max_segs);
/* BLAKE3 (B3Hash::hash, crates/adapteros-infra-common/src/hash.rs:22-27) of
 * len bytes, computed on the GPU; data is host memory, or device memory when
 * on_device != 0.  out: 32 bytes. */
int aos_blake3(aos_ctx* ctx, const void* data, uint64_t len, int on_device, uint8_t* out);
/* Layout check plus every segment's BLAKE3 against its index entry, on the
 * GPU (open_aos, writer.rs:561-585).  bad_segment: index of the first
 * mismatching entry, or -1. */
int aos_archive_verify(aos_ctx* ctx, const void* data, uint64_t len, int32_t* bad_segment);
typedef struct aos_archive_load_info {
    uint32_t rank;         /* scaling rank: manifest rank / lora_rank, else 4 */
    uint32_t tensor_rank;  /* rows of lora_A in the payload */
    uint32_t storage_rank; /* arena columns: tensor_rank rounded up to a multiple of 8 */
    float alpha;           /* manifest alpha / lora_alpha, else 16 */
    uint32_t module_mask;  /* bit m: module m (aos_module order) loaded, at every layer */
    uint32_t segment_id;
    uint16_t backend_tag;
    uint16_t reserved;
    uint8_t weights_hash[32]; /* BLAKE3 of the selected payload */
    uint8_t scope_hash[16];
} aos_archive_load_info;
/* LifecycleLoader::load_from_aos_static (crates/adapteros-lora-lifecycle/src/
 * loader.rs:931-1070) into adapter slot id: layout, segment hashes (GPU),
 * canonical segment present, scope_path required, segment chosen for
 * `backend` ("mlx", "metal", "coreml", "canonical"; anything else or NULL =
 * canonical), per_layer_hashes and weights_hash checked when present; the
 * payload's lora_a.<m> / lora_b.<m> (or <m>.lora_A / <m>.lora_B) tensors load
 * under the MLX backend's rules (mlx-ffi/src/backend.rs:1017-1200) and apply
 * at every layer; LoRA scale = alpha / rank.  info may be NULL. */
int aos_adapter_load_aos(aos_ctx* ctx, uint16_t id, const void* data, uint64_t len, const char* backend,
                         aos_archive_load_info* info);

/* ---- next-token sampling ----------------------------------------------------
 * Generator::next_token / greedy (crates/adapteros-lora-worker/src/
 * generation.rs:326-480) on the device, one token per row: logits [T][ld]
 * f32 (first V columns used), u [T] uniform draws in [0, 1) (the caller's
 * RNG; unused for greedy), tokens [T] out; all device memory, ordered on
 * `stream`.  flags pick greedy, top-k (keep the k most likely, stable order)
 * and top-p (nucleus over what top-k kept).  The temperature is applied as
 * given (the reference clamps it to >= 0.01 when it is set).  The result is
 * the reference's token for the same logits and u; the sums keep the
 * reference's sequential order, so a sampled step costs about 0.3 ms of
 * sequential adds per 128K-entry row (rows run in parallel). */
enum {
    AOS_SAMPLE_GREEDY = 1,
    AOS_SAMPLE_TOP_K = 2,
    AOS_SAMPLE_TOP_P = 4
};
typedef struct aos_sample_params {
    float temperature;
    uint32_t top_k;
    float top_p;
    uint32_t flags;
} aos_sample_params;
int aos_sample_dev(const float* logits, uint32_t T, uint32_t V, uint64_t ld, const aos_sample_params* params,
                   const float* u, uint32_t* tokens, void* stream);

/* ---- GPU buffer fingerprints (FusedKernels::verify_adapter_buffers /
 * store_gpu_fingerprint / verify_gpu_fingerprint, crates/adapteros-lora-
 * kernel-api/src/lib.rs:440-508; GpuBufferFingerprint, kernel-mtl/src/
 * vram.rs:20-80).  An adapter's buffer is, for every layer and LoRA-enabled
 * module (aos_module order), its lora_A [rank][in] then its lora_B
 * [out][rank], bf16 row-major, as read back from the arena.  Samples are the
 * first, last and middle 4 KB (the whole buffer when smaller; the middle
 * window starts at (size - window) / 2). */
int aos_adapter_verify_buffers(aos_ctx* ctx, uint16_t id, uint64_t* buffer_bytes, void* first, void* last,
                               void* mid, uint32_t* sample_bytes);
/* BLAKE3(first || last || mid) on the GPU: GpuBufferFingerprint::new's
 * checkpoint hash.  hash: 32 bytes. */
int aos_adapter_fingerprint(aos_ctx* ctx, uint16_t id, uint64_t* buffer_bytes, uint8_t* hash);
/* Baseline per adapter id (64 hex digits; stored lower-case). */
int aos_store_gpu_fingerprint(aos_ctx* ctx, uint16_t id, uint64_t buffer_bytes, const char* checkpoint_hash_hex);
/* *matches = 1 when a baseline exists with the same size and the same hex
 * string, else 0 (no baseline reads as 0, as in the reference). */
int aos_verify_gpu_fingerprint(aos_ctx* ctx, uint16_t id, uint64_t buffer_bytes, const char* checkpoint_hash_hex,
                               int* matches);
/* FusedKernels::check_memory_footprint (kernel-mtl/src/vram.rs:386-407): the
 * adapter's footprint baseline (storing a fingerprint adds a sample, window 10;
 * the first check starts a baseline of window 100) against bytes: within 2
 * population standard deviations, or equal when every sample is. */
int aos_check_memory_footprint(aos_ctx* ctx, uint16_t id, uint64_t bytes, int* within, double* z_score, double* mean,
                               double* stddev, uint32_t* n_samples);
/* FusedKernels::get_gpu_fingerprints: up to max stored baselines in id order
 * (hex65: max x 65 chars); *n receives how many there are. */
int aos_get_gpu_fingerprints(const aos_ctx* ctx, uint32_t* ids, uint64_t* buffer_bytes, char* hex65, uint32_t max,
                             uint32_t* n);

/* ---- prefill (the prompt path) ---------------------------------------------
 * InferencePipeline's prompt pass (inference_pipeline.rs:983-1154, MLX
 * forward over the prompt, mlx_cpp_wrapper_real.cpp:3338-3559 with T > 1):
 * sequence i contributes n_tok[i] tokens at positions len_i, len_i + 1, ...
 * (its current length onward) with causal attention over its cache.
 * rings / token_ids: device arrays, the concatenation over the sequences (one
 * RouterRing per token).  logits: device [n_seq][vocab] f32 of each
 * sequence's last prompt token, or NULL.  Each sequence advances by n_tok[i];
 * n_seq <= max_batch. */
int aos_prefill_dev(aos_ctx* ctx, uint32_t n_seq, const uint64_t* seq_ids, const uint32_t* n_tok,
                    const aos_router_ring* rings, const uint32_t* token_ids, float* logits, void* stream);
/* The same prompt pass with host arrays (FusedKernels::run_step with several
 * input ids, kernel-api/src/lib.rs:371): rings / token_ids are host arrays,
 * logits a host [n_seq][vocab] f32 array or NULL; returns when the step is
 * done. */
int aos_prefill(aos_ctx* ctx, uint32_t n_seq, const uint64_t* seq_ids, const uint32_t* n_tok,
                const aos_router_ring* rings, const uint32_t* token_ids, float* logits);

/* ---- adapter-sharded decode (the large-pool config) -------------------------
 * No reference counterpart: the reference keeps every adapter on one device
 * (kernel-mtl/src/lib.rs:1897-2046).  Adapters are sharded by id: rank r
 * loads only the adapters with id % world == r.  Per layer and input site
 * (normed -> q/k/v, attention output -> o, normed -> gate/up, SwiGLU ->
 * down) every rank sends its T input rows to every rank over NCCL, each rank
 * runs the LoRA of its own adapters on all world * T rows, the bf16 deltas go
 * back to the rows' home ranks, and each base GEMM adds them in owner order.
 * T must be the same on every rank and world * T <= max_batch.
 * aos_shard_get_unique_id fills AOS_SHARD_ID_BYTES bytes on one rank; the
 * caller hands them to every rank's aos_shard_init (collective: every rank
 * calls it). */
#define AOS_SHARD_ID_BYTES 128
int aos_shard_get_unique_id(void* id);
int aos_shard_init(aos_ctx* ctx, uint32_t rank, uint32_t world, const void* id);
/* One decode step of the home tokens, like aos_run_step_batch_dev
 * (collective: every rank calls it once per step, with the same T). */
int aos_run_step_sharded_dev(aos_ctx* ctx, const aos_router_ring* rings, const uint32_t* token_ids,
                             const uint64_t* seq_ids, uint32_t T, float* logits,
                             uint16_t* hidden_out, void* stream);

/* ---- per-kernel device timing (replaces Metal counter sampling,
 * crates/adapteros-lora-kernel-prof/src/lib.rs:1-21) ------------------------
 * While enabled, steps run without CUDA graphs and every launch is bracketed
 * by CUDA events on its stream; aos_profile_read sums the device time per
 * kernel class. */
typedef enum aos_kernel_class {
    AOS_K_GEMM = 0,    /* base projection + fused LoRA expand (tcgen05)      */
    AOS_K_SHRINK = 1,  /* LoRA-only launch of an adapter owner (sharded step) */
    AOS_K_ATTN = 2,    /* paged decode attention + chunk combine             */
    AOS_K_NORM = 3,    /* RMSNorm                                            */
    AOS_K_PREP = 4,    /* routing prep (touched rank groups)                 */
    AOS_K_EMBED = 5,   /* embedding gather                                   */
    AOS_K_LM_HEAD = 6, /* lm_head GEMM (tcgen05)                             */
    AOS_K_COMM = 7,    /* NCCL exchange of the adapter-sharded step          */
    AOS_K_NUM_CLASSES = 8
} aos_kernel_class;

typedef struct aos_profile {
    uint64_t launches[AOS_K_NUM_CLASSES];
    double ms[AOS_K_NUM_CLASSES];
    uint64_t steps;
    uint32_t last_touched_groups; /* 64-column rank groups the last step streamed */
} aos_profile;

int aos_profile_enable(aos_ctx* ctx, int enable);
int aos_profile_read(aos_ctx* ctx, aos_profile* out, int reset);
/* Diagnostics: with AOS_TC_TRACE=<g> set before aos_init, the GEMM launch g
 * (0..3: qkv, o, gate/up, down) of layer 0 writes per-CTA %globaltimer stamps
 * (256 slots per CTA); this copies n of them to host. */
/* FusedKernels::memory_report (kernel-api/src/lib.rs:588-593): totals, and up
 * to max_allocs per-adapter allocations (id, bytes) in id order; *n_allocs
 * receives the number of loaded adapters. */
int aos_memory_report(aos_ctx* ctx, aos_memory_report_data* out, aos_adapter_allocation* allocs, uint32_t max_allocs,
                      uint32_t* n_allocs);
int aos_debug_trace_read(aos_ctx* ctx, uint64_t* out, uint64_t n);
/* Failure-path check: runs one of the GEMM kernel's bounded waits against a
 * condition nothing satisfies (kind 0: global-counter spin, 1: mbarrier wait);
 * returns AOS_ERR_TIMEOUT after the wait's limit (about one second), with the
 * context left usable. */
int aos_debug_bounded_wait(aos_ctx* ctx, int kind);

/* ---- metrics / health / attestation (lib.rs:383, 559-593) ---------------- */
int aos_get_metrics(const aos_ctx* ctx, aos_metrics* out);
/* 0 = healthy; otherwise the first device error seen (e.g. AOS_ERR_TIMEOUT). */
int aos_health_check(aos_ctx* ctx);
int aos_attest_determinism(const aos_ctx* ctx, aos_determinism_report* out);

#ifdef __cplusplus
}
#endif
#endif /* AOS_CUDA_H */
