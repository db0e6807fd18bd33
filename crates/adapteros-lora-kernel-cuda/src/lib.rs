//! CUDA backend (B200, sm_100a) for adapterOS's `FusedKernels` trait
//! (crates/adapteros-lora-kernel-api/src/lib.rs:308-716).
//!
//! Every method is one call into libaoscuda's C ABI (`include/aos_cuda.h`);
//! the router, the fused base + LoRA projections, attention over the paged KV
//! cache, adapter loading and attestation all run there.  There is no CPU
//! fallback: without an sm_100 device every call fails with `AosError::Kernel`.
//!
//! Threading: `&mut self` serialises the calls that change state, as the trait
//! requires (lib.rs:371); the context owns one CUDA stream.

pub mod ffi;

use std::collections::HashMap;
use std::ffi::{CStr, CString};
use std::os::raw::{c_char, c_int};
use std::ptr;
use std::time::Duration;

use adapteros_core::{AosError, B3Hash, Result};
use adapteros_lora_kernel_api::attestation::{
    BackendType, DeterminismLevel, DeterminismReport, FloatingPointMode, RngSeedingMethod,
};
use adapteros_lora_kernel_api::{
    AdapterLoadMetadata, BackendHealth, BackendMetrics, BufferVerificationResult, FusedKernels,
    GpuBufferFingerprint, GpuMemoryReportData, IoBuffers, RouterRing,
};

/// Sizes the backend reserves when `load` creates its context: the KV pool,
/// the adapter arena and the decode batch (aos_model_config's runtime fields).
/// The model's own dimensions come from the plan.
#[derive(Debug, Clone)]
pub struct CudaRuntimeOptions {
    /// Tokens per decode step (<= 256).
    pub max_batch: u32,
    /// KV pages (16 positions each) per layer.
    pub kv_num_blocks: u32,
    /// Longest sequence; a new session reserves this many positions.
    pub max_seq_len: u32,
    /// Rank columns of the adapter arena.
    pub lora_rank_capacity: u32,
    /// Adapter ids are below this.
    pub lora_max_adapters: u32,
    /// Bit m: module m (q, k, v, o, gate, up, down) may carry LoRA; 0 = all.
    pub lora_module_mask: u32,
    /// CUDA device ordinal.
    pub device: i32,
    /// The plan crate's model config JSON (config.rs ModelConfig), if any:
    /// its head geometry, rope_theta and rms_norm_eps are used and checked
    /// against the plan's tensor shapes.  Without it the backend uses
    /// GqaConfig::default() (head_dim 128, rope_theta 10000), as the Metal
    /// backend does without set_gqa_config.
    pub model_config_json: Option<String>,
}

impl Default for CudaRuntimeOptions {
    fn default() -> Self {
        Self {
            max_batch: 64,
            kv_num_blocks: 16384,
            max_seq_len: 4096,
            lora_rank_capacity: 4096,
            lora_max_adapters: 128,
            lora_module_mask: 0,
            device: 0,
            model_config_json: None,
        }
    }
}

/// The CUDA implementation of `FusedKernels`.
pub struct CudaKernels {
    ctx: *mut ffi::AosCtx,
    opts: CudaRuntimeOptions,
    plan_config: Option<ffi::AosPlanConfig>,
    vocab: usize,
    name: String,
    sessions: HashMap<String, u64>,
    next_seq: u64,
}

// The context is only touched through &self / &mut self, and the library
// serialises work on the context's own stream.
unsafe impl Send for CudaKernels {}
unsafe impl Sync for CudaKernels {}

fn last_error(ctx: *const ffi::AosCtx) -> String {
    let p = unsafe { ffi::aos_last_error(ctx) };
    if p.is_null() {
        return String::new();
    }
    unsafe { CStr::from_ptr(p) }.to_string_lossy().into_owned()
}

/// aos_status -> AosError, with the library's message.
fn check(rc: c_int, ctx: *const ffi::AosCtx) -> Result<()> {
    if rc == ffi::AOS_OK {
        return Ok(());
    }
    let msg = last_error(ctx);
    Err(match rc {
        ffi::AOS_ERR_INVALID => AosError::Validation(msg),
        ffi::AOS_ERR_NONFINITE => AosError::DeterminismViolation(msg),
        ffi::AOS_ERR_NOT_FOUND => AosError::NotFound(msg),
        ffi::AOS_ERR_NOMEM => AosError::ResourceExhaustion(msg),
        _ => AosError::Kernel(format!("aos status {rc}: {msg}")),
    })
}

fn c_str(bytes: &[c_char]) -> String {
    let b: Vec<u8> = bytes.iter().take_while(|&&c| c != 0).map(|&c| c as u8).collect();
    String::from_utf8_lossy(&b).into_owned()
}

fn ring_to_c(ring: &RouterRing) -> ffi::AosRouterRing {
    ffi::AosRouterRing {
        top_k: ring.k as u32,
        position: ring.position as u32,
        indices: ring.indices,
        gates_q15: ring.gates_q15,
    }
}

impl CudaKernels {
    /// A backend with no model yet; `load(plan_bytes)` creates the device
    /// context.  A model config JSON in `opts` is parsed and validated here
    /// (ModelConfig::from_json + validate, config.rs:80-86, 127-167).
    pub fn new(opts: CudaRuntimeOptions) -> Result<Self> {
        let plan_config = match &opts.model_config_json {
            Some(json) => {
                let mut pc = std::mem::MaybeUninit::<ffi::AosPlanConfig>::zeroed();
                let c = CString::new(json.as_str())
                    .map_err(|_| AosError::Validation("model config JSON contains a NUL byte".into()))?;
                check(unsafe { ffi::aos_plan_config_parse(c.as_ptr(), json.len() as u64, pc.as_mut_ptr()) },
                      ptr::null())?;
                let pc = unsafe { pc.assume_init() };
                check(unsafe { ffi::aos_plan_config_validate(&pc) }, ptr::null())?;
                Some(pc)
            }
            None => None,
        };
        Ok(Self {
            ctx: ptr::null_mut(),
            opts,
            plan_config,
            vocab: 0,
            name: String::from("cuda (no model loaded)"),
            sessions: HashMap::new(),
            next_seq: 1,
        })
    }

    fn ctx(&self) -> Result<*mut ffi::AosCtx> {
        if self.ctx.is_null() {
            return Err(AosError::Kernel("CUDA backend: load(plan_bytes) has not been called".into()));
        }
        Ok(self.ctx)
    }

    /// The KV sequence of a session (IoBuffers::session_id; None is one
    /// default session), reserved on first use for max_seq_len positions.
    fn session(&mut self, id: Option<&str>) -> Result<u64> {
        let key = id.unwrap_or("").to_string();
        if let Some(&seq) = self.sessions.get(&key) {
            return Ok(seq);
        }
        let ctx = self.ctx()?;
        let seq = self.next_seq;
        check(unsafe { ffi::aos_kv_alloc(ctx, seq, self.opts.max_seq_len) }, ctx)?;
        self.next_seq += 1;
        self.sessions.insert(key, seq);
        Ok(seq)
    }

    /// Sliding-window rotate of a session's KV cache (kv_cache.metal:200-236):
    /// drops its oldest `shift` positions in every layer.  Not part of
    /// FusedKernels; a worker that wants a fixed-memory window calls it
    /// between steps.
    pub fn rotate_session_cache(&mut self, session_id: &str, shift: u32) -> Result<()> {
        let ctx = self.ctx()?;
        let Some(&seq) = self.sessions.get(session_id) else {
            return Err(AosError::Validation(format!("unknown session {session_id}")));
        };
        check(unsafe { ffi::aos_kv_rotate(ctx, seq, shift) }, ctx)
    }

    fn pc_ptr(&self) -> *const ffi::AosPlanConfig {
        self.plan_config.as_ref().map_or(ptr::null(), |p| p as *const _)
    }
}

impl Drop for CudaKernels {
    fn drop(&mut self) {
        if !self.ctx.is_null() {
            unsafe { ffi::aos_destroy(self.ctx) };
            self.ctx = ptr::null_mut();
        }
    }
}

impl FusedKernels for CudaKernels {
    /// The plan is the model's safetensors bytes (kernel-mtl/src/lib.rs:1476-1537):
    /// dimensions from the tensor shapes (and the model config, if given),
    /// then the base weights into a fresh context.  Loading again replaces
    /// the model and forgets every session.
    fn load(&mut self, plan_bytes: &[u8]) -> Result<()> {
        let mut cfg = ffi::AosModelConfig {
            kv_block_size: 16,
            max_batch: self.opts.max_batch,
            kv_num_blocks: self.opts.kv_num_blocks,
            max_seq_len: self.opts.max_seq_len,
            lora_rank_capacity: self.opts.lora_rank_capacity,
            lora_max_adapters: self.opts.lora_max_adapters,
            lora_module_mask: self.opts.lora_module_mask,
            device: self.opts.device,
            ..Default::default()
        };
        let pc = self.pc_ptr();
        let plan = plan_bytes.as_ptr() as *const std::ffi::c_void;
        check(unsafe { ffi::aos_model_config_from_plan(plan, plan_bytes.len() as u64, pc, &mut cfg) },
              ptr::null())?;
        if !self.ctx.is_null() {
            unsafe { ffi::aos_destroy(self.ctx) };
            self.ctx = ptr::null_mut();
            self.sessions.clear();
        }
        let ctx = unsafe { ffi::aos_init_from_plan(plan, plan_bytes.len() as u64, pc, &cfg) };
        if ctx.is_null() {
            return Err(AosError::Kernel(format!("CUDA backend load: {}", last_error(ptr::null()))));
        }
        self.ctx = ctx;
        self.vocab = cfg.vocab as usize;
        let name = unsafe { ffi::aos_device_name(ctx) };
        self.name = if name.is_null() {
            "cuda".into()
        } else {
            unsafe { CStr::from_ptr(name) }.to_string_lossy().into_owned()
        };
        Ok(())
    }

    /// One step of the session in `io`: a single input id is a decode token
    /// (aos_run_step_batch); several are a prompt pass with causal attention
    /// (aos_prefill).  The ring applies to every input token.  Logits of the
    /// last token go to io.output_logits[..vocab]; io.position advances by the
    /// number of input ids (mlx-ffi/src/backend.rs:1292).
    fn run_step(&mut self, ring: &RouterRing, io: &mut IoBuffers) -> Result<()> {
        let ctx = self.ctx()?;
        let n = io.input_ids.len();
        if n == 0 {
            return Err(AosError::Validation("run_step needs at least one input id".into()));
        }
        if io.output_logits.len() < self.vocab {
            io.output_logits.resize(self.vocab, 0.0);
        }
        let seq = self.session(io.session_id.as_deref())?;
        check(unsafe { ffi::aos_kv_set_len(ctx, seq, io.position as u32) }, ctx)?;
        let r = ring_to_c(ring);
        if n == 1 {
            check(unsafe {
                ffi::aos_run_step_batch(ctx, &r, io.input_ids.as_ptr(), &seq, 1, io.output_logits.as_mut_ptr(),
                                        ptr::null_mut())
            }, ctx)?;
        } else {
            let rings = vec![r; n];
            let n_tok = n as u32;
            check(unsafe {
                ffi::aos_prefill(ctx, 1, &seq, &n_tok, rings.as_ptr(), io.input_ids.as_ptr(),
                                 io.output_logits.as_mut_ptr())
            }, ctx)?;
        }
        io.position += n;
        Ok(())
    }

    fn device_name(&self) -> &str {
        &self.name
    }

    /// DeterminismReport of the CUDA build (attestation.rs:130-160): no fast
    /// math, no floating-point atomics, fixed-order reductions (bit-exact run
    /// to run), HKDF-seeded sampling.  The kernel hash slot carries the BLAKE3
    /// of the library's build stamp (SHA-256 of every kernel source and header
    /// plus the nvcc flags).
    fn attest_determinism(&self) -> Result<DeterminismReport> {
        let ctx = self.ctx()?;
        let mut r = std::mem::MaybeUninit::<ffi::AosDeterminismReport>::zeroed();
        check(unsafe { ffi::aos_attest_determinism(ctx, r.as_mut_ptr()) }, ctx)?;
        let r = unsafe { r.assume_init() };
        let build_id = c_str(&r.kernel_build_id);
        Ok(DeterminismReport {
            backend_type: BackendType::Cuda,
            metallib_hash: Some(B3Hash::hash(build_id.as_bytes())),
            metallib_verified: false,
            manifest: None,
            rng_seed_method: match r.rng_seed_method {
                0 => RngSeedingMethod::HkdfSeeded,
                _ => RngSeedingMethod::SystemEntropy,
            },
            floating_point_mode: match r.floating_point_mode {
                0 => FloatingPointMode::Deterministic,
                1 => FloatingPointMode::FastMath,
                _ => FloatingPointMode::Unknown,
            },
            determinism_level: match r.determinism_level {
                2 => DeterminismLevel::BitExact,
                1 => DeterminismLevel::BoundedTolerance,
                _ => DeterminismLevel::None,
            },
            compiler_flags: c_str(&r.compiler_flags).split_whitespace().map(String::from).collect(),
            deterministic: r.deterministic != 0,
            runtime_version: Some(c_str(&r.runtime_version)),
            device_id: Some(c_str(&r.device_id)),
        })
    }

    /// Safetensors bytes with no metadata: rank, alpha and target modules from
    /// the tensors and the defaults (kernel-mtl/src/lib.rs:186-251).
    fn load_adapter(&mut self, id: u16, weights: &[u8]) -> Result<()> {
        let ctx = self.ctx()?;
        check(unsafe {
            ffi::aos_adapter_load_safetensors(ctx, id, weights.as_ptr() as *const _, weights.len() as u64,
                                              ptr::null())
        }, ctx)
    }

    fn load_adapter_with_metadata(&mut self, id: u16, weights: &[u8], m: &AdapterLoadMetadata) -> Result<()> {
        let ctx = self.ctx()?;
        let names: Vec<CString> = m
            .target_modules
            .iter()
            .filter_map(|t| CString::new(t.as_str()).ok())
            .collect();
        let ptrs: Vec<*const c_char> = names.iter().map(|c| c.as_ptr()).collect();
        let meta = ffi::AosAdapterMeta {
            rank: m.rank,
            alpha: m.alpha,
            target_modules: if ptrs.is_empty() { ptr::null() } else { ptrs.as_ptr() },
            n_targets: ptrs.len() as u32,
        };
        check(unsafe {
            ffi::aos_adapter_load_safetensors(ctx, id, weights.as_ptr() as *const _, weights.len() as u64, &meta)
        }, ctx)
    }

    fn unload_adapter(&mut self, id: u16) -> Result<()> {
        let ctx = self.ctx()?;
        check(unsafe { ffi::aos_adapter_unload(ctx, id) }, ctx)
    }

    fn verify_adapter_buffers(&self, id: u16) -> Result<BufferVerificationResult> {
        let ctx = self.ctx()?;
        let (mut bytes, mut k) = (0u64, 0u32);
        let (mut f, mut l, mut mid) = (vec![0u8; 4096], vec![0u8; 4096], vec![0u8; 4096]);
        check(unsafe {
            ffi::aos_adapter_verify_buffers(ctx, id, &mut bytes, f.as_mut_ptr() as *mut _, l.as_mut_ptr() as *mut _,
                                            mid.as_mut_ptr() as *mut _, &mut k)
        }, ctx)?;
        f.truncate(k as usize);
        l.truncate(k as usize);
        mid.truncate(k as usize);
        Ok((bytes, f, l, mid))
    }

    fn store_gpu_fingerprint(&mut self, id: u16, buffer_size: u64, checkpoint_hash_hex: &str) -> Result<()> {
        let ctx = self.ctx()?;
        let h = CString::new(checkpoint_hash_hex).map_err(|_| AosError::Validation("hash contains NUL".into()))?;
        check(unsafe { ffi::aos_store_gpu_fingerprint(ctx, id, buffer_size, h.as_ptr()) }, ctx)
    }

    fn verify_gpu_fingerprint(&self, id: u16, buffer_size: u64, checkpoint_hash_hex: &str) -> Result<bool> {
        let ctx = self.ctx()?;
        let h = CString::new(checkpoint_hash_hex).map_err(|_| AosError::Validation("hash contains NUL".into()))?;
        let mut matches: c_int = 0;
        check(unsafe { ffi::aos_verify_gpu_fingerprint(ctx, id, buffer_size, h.as_ptr(), &mut matches) }, ctx)?;
        Ok(matches != 0)
    }

    fn check_memory_footprint(&self, id: u16, buffer_size: u64) -> (bool, f64, Option<(f64, f64, usize)>) {
        let Ok(ctx) = self.ctx() else { return (false, 0.0, None) };
        let (mut within, mut z, mut mean, mut sd, mut n) = (0 as c_int, 0f64, 0f64, 0f64, 0u32);
        let rc = unsafe {
            ffi::aos_check_memory_footprint(ctx, id, buffer_size, &mut within, &mut z, &mut mean, &mut sd, &mut n)
        };
        if rc != ffi::AOS_OK {
            return (false, 0.0, None);
        }
        (within != 0, z, if n > 0 { Some((mean, sd, n as usize)) } else { None })
    }

    fn supports_kv_cache(&self) -> bool {
        true
    }

    fn clear_session_cache(&mut self, session_id: &str) {
        if let Some(seq) = self.sessions.remove(session_id) {
            if let Ok(ctx) = self.ctx() {
                unsafe { ffi::aos_kv_free(ctx, seq) };
            }
        }
    }

    fn clear_all_caches(&mut self) {
        if let Ok(ctx) = self.ctx() {
            unsafe { ffi::aos_kv_clear_all(ctx) };
        }
        self.sessions.clear();
    }

    fn cache_memory_bytes(&self) -> usize {
        self.ctx().map(|ctx| unsafe { ffi::aos_kv_memory_bytes(ctx) } as usize).unwrap_or(0)
    }

    fn get_metrics(&self) -> BackendMetrics {
        let Ok(ctx) = self.ctx() else { return BackendMetrics::default() };
        let mut m = ffi::AosMetrics::default();
        if unsafe { ffi::aos_get_metrics(ctx, &mut m) } != ffi::AOS_OK {
            return BackendMetrics::default();
        }
        BackendMetrics {
            total_operations: m.steps,
            successful_operations: m.steps,
            failed_operations: 0,
            avg_latency: Duration::from_secs_f64(m.last_step_ms as f64 / 1000.0),
            memory_usage_bytes: m.base_weight_bytes + m.arena_bytes + m.kv_pool_bytes,
        }
    }

    fn health_check(&self) -> Result<BackendHealth> {
        let ctx = self.ctx()?;
        let rc = unsafe { ffi::aos_health_check(ctx) };
        Ok(if rc == ffi::AOS_OK {
            BackendHealth::Healthy
        } else {
            BackendHealth::Failed { reason: format!("aos status {rc}: {}", last_error(ctx)), recoverable: false }
        })
    }

    fn get_gpu_fingerprints(&self) -> HashMap<u32, GpuBufferFingerprint> {
        let mut out = HashMap::new();
        let Ok(ctx) = self.ctx() else { return out };
        let mut n = 0u32;
        if unsafe { ffi::aos_get_gpu_fingerprints(ctx, ptr::null_mut(), ptr::null_mut(), ptr::null_mut(), 0, &mut n) }
            != ffi::AOS_OK
        {
            return out;
        }
        let (mut ids, mut bytes, mut hex) = (vec![0u32; n as usize], vec![0u64; n as usize], vec![0 as c_char; 65 * n as usize]);
        if unsafe { ffi::aos_get_gpu_fingerprints(ctx, ids.as_mut_ptr(), bytes.as_mut_ptr(), hex.as_mut_ptr(), n, &mut n) }
            != ffi::AOS_OK
        {
            return out;
        }
        for i in 0..n as usize {
            if let Ok(h) = B3Hash::from_hex(&c_str(&hex[65 * i..65 * i + 65])) {
                out.insert(ids[i], GpuBufferFingerprint { buffer_bytes: bytes[i], checkpoint_hash: h });
            }
        }
        out
    }

    fn memory_report(&self) -> Option<GpuMemoryReportData> {
        let ctx = self.ctx().ok()?;
        let mut d = ffi::AosMemoryReportData::default();
        let mut n = 0u32;
        if unsafe { ffi::aos_memory_report(ctx, &mut d, ptr::null_mut(), 0, &mut n) } != ffi::AOS_OK {
            return None;
        }
        let mut allocs = vec![ffi::AosAdapterAllocation::default(); n as usize];
        if unsafe { ffi::aos_memory_report(ctx, &mut d, allocs.as_mut_ptr(), n, &mut n) } != ffi::AOS_OK {
            return None;
        }
        Some(GpuMemoryReportData {
            total_gpu_bytes: d.total_gpu_bytes,
            used_gpu_bytes: d.used_gpu_bytes,
            adapter_count: d.adapter_count as usize,
            adapter_vram_total: d.adapter_vram_total,
            adapter_allocations: allocs.iter().take(n as usize).map(|a| (a.adapter_id, a.bytes)).collect(),
            pool_stats: None,
        })
    }
}
