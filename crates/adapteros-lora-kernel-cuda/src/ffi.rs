//! Raw bindings of libaoscuda (`include/aos_cuda.h`), the C ABI the CUDA
//! backend exposes.  Layouts are `#[repr(C)]` copies of the header's structs;
//! every function returns an `aos_status` (0 = ok, < 0 = error, message in
//! `aos_last_error`) unless its signature says otherwise.

#![allow(non_camel_case_types, dead_code)]

use std::os::raw::{c_char, c_double, c_float, c_int, c_void};

pub const AOS_OK: c_int = 0;
pub const AOS_ERR_INVALID: c_int = -1;
pub const AOS_ERR_CUDA: c_int = -2;
pub const AOS_ERR_NOMEM: c_int = -3;
pub const AOS_ERR_NONFINITE: c_int = -4;
pub const AOS_ERR_NOT_FOUND: c_int = -5;
pub const AOS_ERR_TIMEOUT: c_int = -6;
pub const AOS_ERR_NO_DEVICE: c_int = -7;
pub const AOS_ERR_STATE: c_int = -8;

pub const AOS_MAX_K: usize = 8;

/// Opaque backend context (one CUDA stream; calls on it are serialised).
#[repr(C)]
pub struct AosCtx {
    _private: [u8; 0],
}

/// The 40-byte RouterRing device layout (kernel-mtl/src/ring_buffer.rs:44-58).
#[repr(C)]
#[derive(Clone, Copy, Debug, Default)]
pub struct AosRouterRing {
    pub top_k: u32,
    pub position: u32,
    pub indices: [u16; AOS_MAX_K],
    pub gates_q15: [i16; AOS_MAX_K],
}

#[repr(C)]
#[derive(Clone, Copy, Debug, Default)]
pub struct AosModelConfig {
    pub hidden: u32,
    pub n_heads: u32,
    pub n_kv_heads: u32,
    pub head_dim: u32,
    pub intermediate: u32,
    pub vocab: u32,
    pub n_layers: u32,
    pub rms_eps: c_float,
    pub rope_theta: c_float,
    pub rope_mlx_as_written: u32,
    pub max_batch: u32,
    pub kv_block_size: u32,
    pub kv_num_blocks: u32,
    pub max_seq_len: u32,
    pub lora_rank_capacity: u32,
    pub lora_max_adapters: u32,
    pub lora_module_mask: u32,
    pub device: i32,
}

/// The plan crate's ModelConfig with its derived values (aos_plan_config).
#[repr(C)]
#[derive(Clone, Copy)]
pub struct AosPlanConfig {
    pub name: [c_char; 128],
    pub architecture: [c_char; 128],
    pub hidden_size: u32,
    pub intermediate_size: u32,
    pub num_hidden_layers: u32,
    pub num_attention_heads: u32,
    pub num_key_value_heads: u32,
    pub max_position_embeddings: u32,
    pub vocab_size: u32,
    pub rope_theta: c_float,
    pub has_rope_scaling_factor: u32,
    pub rope_scaling_factor: c_float,
    pub has_rope_scaling: u32,
    pub scaling_factor: c_float,
    pub scaling_original_max_position_embeddings: u32,
    pub scaling_type: [c_char; 64],
    pub rms_norm_eps: c_float,
    pub head_dim: u32,
    pub kv_width: u32,
    pub total_params: u64,
    pub effective_context_length: u32,
    pub is_qwen2_5: u32,
}

/// AdapterLoadMetadata's rank / alpha / target modules (aos_adapter_meta).
#[repr(C)]
pub struct AosAdapterMeta {
    pub rank: u32,
    pub alpha: c_float,
    pub target_modules: *const *const c_char,
    pub n_targets: u32,
}

#[repr(C)]
#[derive(Clone, Copy, Debug, Default)]
pub struct AosMetrics {
    pub steps: u64,
    pub tokens: u64,
    pub route_calls: u64,
    pub base_weight_bytes: u64,
    pub arena_bytes: u64,
    pub arena_used_rank_cols: u64,
    pub kv_pool_bytes: u64,
    pub adapters_loaded: u32,
    pub kv_blocks_used: u32,
    pub kv_blocks_total: u32,
    pub sequences: u32,
    pub last_step_ms: c_float,
}

#[repr(C)]
#[derive(Clone, Copy)]
pub struct AosDeterminismReport {
    pub backend: [c_char; 32],
    pub device_name: [c_char; 64],
    pub sm_major: u32,
    pub sm_minor: u32,
    pub fast_math: u32,
    pub float_atomics: u32,
    pub fixed_reduction_order: u32,
    pub kernel_build_id: [c_char; 65],
    pub compiler_flags: [c_char; 512],
    pub runtime_version: [c_char; 64],
    pub device_id: [c_char; 64],
    pub rng_seed_method: u32,
    pub floating_point_mode: u32,
    pub determinism_level: u32,
    pub deterministic: u32,
}

#[repr(C)]
#[derive(Clone, Copy, Debug, Default)]
pub struct AosMemoryReportData {
    pub total_gpu_bytes: u64,
    pub used_gpu_bytes: u64,
    pub adapter_count: u32,
    pub adapter_vram_total: u64,
    pub arena_bytes: u64,
    pub arena_used_bytes: u64,
    pub kv_pool_bytes: u64,
    pub kv_used_bytes: u64,
}

#[repr(C)]
#[derive(Clone, Copy, Debug, Default)]
pub struct AosAdapterAllocation {
    pub adapter_id: u32,
    pub bytes: u64,
}

extern "C" {
    pub fn aos_last_error(ctx: *const AosCtx) -> *const c_char;
    pub fn aos_device_count() -> c_int;

    // FusedKernels::load(plan_bytes)
    pub fn aos_plan_config_parse(json: *const c_char, len: u64, out: *mut AosPlanConfig) -> c_int;
    pub fn aos_plan_config_validate(cfg: *const AosPlanConfig) -> c_int;
    pub fn aos_model_config_from_plan(plan: *const c_void, len: u64, pc: *const AosPlanConfig,
                                      cfg: *mut AosModelConfig) -> c_int;
    pub fn aos_init_from_plan(plan: *const c_void, len: u64, pc: *const AosPlanConfig,
                              runtime: *const AosModelConfig) -> *mut AosCtx;
    pub fn aos_destroy(ctx: *mut AosCtx);
    pub fn aos_device_name(ctx: *const AosCtx) -> *const c_char;

    // run_step: one decode token, or a prompt pass
    pub fn aos_run_step_batch(ctx: *mut AosCtx, rings: *const AosRouterRing, token_ids: *const u32,
                              seq_ids: *const u64, t: u32, logits: *mut c_float, hidden_out: *mut u16) -> c_int;
    pub fn aos_prefill(ctx: *mut AosCtx, n_seq: u32, seq_ids: *const u64, n_tok: *const u32,
                       rings: *const AosRouterRing, token_ids: *const u32, logits: *mut c_float) -> c_int;

    // hot-swap
    pub fn aos_adapter_load_safetensors(ctx: *mut AosCtx, id: u16, data: *const c_void, len: u64,
                                        meta: *const AosAdapterMeta) -> c_int;
    pub fn aos_adapter_unload(ctx: *mut AosCtx, id: u16) -> c_int;

    // KV cache (sessions)
    pub fn aos_kv_alloc(ctx: *mut AosCtx, seq_id: u64, max_tokens: u32) -> c_int;
    pub fn aos_kv_free(ctx: *mut AosCtx, seq_id: u64) -> c_int;
    pub fn aos_kv_set_len(ctx: *mut AosCtx, seq_id: u64, len: u32) -> c_int;
    pub fn aos_kv_clear_all(ctx: *mut AosCtx) -> c_int;
    pub fn aos_kv_rotate(ctx: *mut AosCtx, seq_id: u64, shift: u32) -> c_int;
    pub fn aos_kv_memory_bytes(ctx: *const AosCtx) -> u64;

    // GPU buffer verification and fingerprints
    pub fn aos_adapter_verify_buffers(ctx: *mut AosCtx, id: u16, buffer_bytes: *mut u64, first: *mut c_void,
                                      last: *mut c_void, mid: *mut c_void, sample_bytes: *mut u32) -> c_int;
    pub fn aos_store_gpu_fingerprint(ctx: *mut AosCtx, id: u16, buffer_bytes: u64,
                                     checkpoint_hash_hex: *const c_char) -> c_int;
    pub fn aos_verify_gpu_fingerprint(ctx: *mut AosCtx, id: u16, buffer_bytes: u64,
                                      checkpoint_hash_hex: *const c_char, matches: *mut c_int) -> c_int;
    pub fn aos_check_memory_footprint(ctx: *mut AosCtx, id: u16, bytes: u64, within: *mut c_int,
                                      z_score: *mut c_double, mean: *mut c_double, stddev: *mut c_double,
                                      n_samples: *mut u32) -> c_int;
    pub fn aos_get_gpu_fingerprints(ctx: *const AosCtx, ids: *mut u32, buffer_bytes: *mut u64, hex65: *mut c_char,
                                    max: u32, n: *mut u32) -> c_int;

    // metrics, health, memory report, attestation
    pub fn aos_get_metrics(ctx: *const AosCtx, out: *mut AosMetrics) -> c_int;
    pub fn aos_health_check(ctx: *mut AosCtx) -> c_int;
    pub fn aos_memory_report(ctx: *mut AosCtx, out: *mut AosMemoryReportData, allocs: *mut AosAdapterAllocation,
                             max_allocs: u32, n_allocs: *mut u32) -> c_int;
    pub fn aos_attest_determinism(ctx: *const AosCtx, out: *mut AosDeterminismReport) -> c_int;
}
