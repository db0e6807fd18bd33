"""adapter-os B200 backend: host-side mirror of the reference's kernel API.

The compute lives in ``libaoscuda.so`` (hand-written sm_100a CUDA behind the C
ABI in include/aos_cuda.h).  This module binds it with ctypes and mirrors the
names and behaviour of the reference's Rust surface:

* ``RouterRing`` / ``IoBuffers`` — crates/adapteros-lora-kernel-api/src/lib.rs:58-246
* ``route_batch`` — Router::route_with_adapter_info (crates/adapteros-lora-router/src/router.rs:1517-1952),
  batched one decision per token
* ``CudaKernels`` — a ``FusedKernels`` implementation (lib.rs:308-716)

There is no CPU fallback: importing works anywhere, but every compute call
raises ``AosError`` when the library or an sm_100 device is missing.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libaoscuda.so")
_lib = None

MAX_K = 8
Q15_DENOM = np.float32(32767.0)
MODULES = ("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj")

STATUS = {0: "OK", -1: "INVALID", -2: "CUDA", -3: "NOMEM", -4: "NONFINITE", -5: "NOT_FOUND",
          -6: "TIMEOUT", -7: "NO_DEVICE", -8: "STATE"}


class AosError(RuntimeError):
    """adapteros_core::AosError equivalent carrying the C status code."""

    def __init__(self, code, msg):
        super().__init__(f"{STATUS.get(code, code)}: {msg}")
        self.code = code


class RouterRingC(C.Structure):
    """aos_router_ring: the 40-byte RouterRing device layout (ring_buffer.rs:44-58)."""

    _fields_ = [("top_k", C.c_uint32), ("position", C.c_uint32),
                ("indices", C.c_uint16 * 8), ("gates_q15", C.c_int16 * 8)]


RING_DTYPE = np.dtype([("top_k", "<u4"), ("position", "<u4"), ("indices", "<u2", (8,)),
                       ("gates_q15", "<i2", (8,))])


class RouterParams(C.Structure):
    _fields_ = [("k", C.c_uint32), ("tau", C.c_float), ("eps", C.c_float), ("routing_bias", C.c_float)]


class ModelConfig(C.Structure):
    _fields_ = [
        ("hidden", C.c_uint32), ("n_heads", C.c_uint32), ("n_kv_heads", C.c_uint32),
        ("head_dim", C.c_uint32), ("intermediate", C.c_uint32), ("vocab", C.c_uint32),
        ("n_layers", C.c_uint32), ("rms_eps", C.c_float), ("rope_theta", C.c_float),
        ("rope_mlx_as_written", C.c_uint32), ("max_batch", C.c_uint32),
        ("kv_block_size", C.c_uint32), ("kv_num_blocks", C.c_uint32), ("max_seq_len", C.c_uint32),
        ("lora_rank_capacity", C.c_uint32), ("lora_max_adapters", C.c_uint32),
        ("lora_module_mask", C.c_uint32), ("device", C.c_int32),
    ]


class Metrics(C.Structure):
    _fields_ = [
        ("steps", C.c_uint64), ("tokens", C.c_uint64), ("route_calls", C.c_uint64),
        ("base_weight_bytes", C.c_uint64), ("arena_bytes", C.c_uint64),
        ("arena_used_rank_cols", C.c_uint64), ("kv_pool_bytes", C.c_uint64),
        ("adapters_loaded", C.c_uint32), ("kv_blocks_used", C.c_uint32),
        ("kv_blocks_total", C.c_uint32), ("sequences", C.c_uint32), ("last_step_ms", C.c_float),
    ]


KERNEL_CLASSES = ("gemm", "owner_lora", "attention", "rmsnorm", "prep", "embed", "lm_head", "comm")


class Profile(C.Structure):
    _fields_ = [("launches", C.c_uint64 * 8), ("ms", C.c_double * 8), ("steps", C.c_uint64),
                ("last_touched_groups", C.c_uint32)]


class DeterminismReport(C.Structure):
    _fields_ = [
        ("backend", C.c_char * 32), ("device_name", C.c_char * 64), ("sm_major", C.c_uint32),
        ("sm_minor", C.c_uint32), ("fast_math", C.c_uint32), ("float_atomics", C.c_uint32),
        ("fixed_reduction_order", C.c_uint32), ("kernel_build_id", C.c_char * 65),
        ("compiler_flags", C.c_char * 512), ("runtime_version", C.c_char * 64), ("device_id", C.c_char * 64),
        ("rng_seed_method", C.c_uint32), ("floating_point_mode", C.c_uint32), ("determinism_level", C.c_uint32),
        ("deterministic", C.c_uint32),
    ]


RNG_METHODS = ("HkdfSeeded", "FixedSeed", "SystemEntropy")
FP_MODES = ("Deterministic", "FastMath", "Unknown")
DET_LEVELS = ("none", "bounded_tolerance", "bit_exact")


def validate_report(rep: dict):
    """DeterminismReport::validate (kernel-api/src/attestation.rs:163-233):
    the list of violations (empty = valid)."""
    errors = []
    if not rep["deterministic"]:
        errors.append("Overall deterministic flag is false")
    if rep["deterministic"] and rep["determinism_level"] == "none":
        errors.append("Determinism level must be deterministic when deterministic=true")
    if not rep["deterministic"] and rep["determinism_level"] != "none":
        errors.append("Determinism level must be none when deterministic=false")
    if rep["rng_seed_method"] == "SystemEntropy":
        errors.append("RNG seeding method SystemEntropy is not deterministic")
    if rep["floating_point_mode"] != "Deterministic":
        errors.append(f"Floating-point mode {rep['floating_point_mode']} is not deterministic")
    for flag in rep["compiler_flags"]:
        for bad in ("-ffast-math", "-funsafe-math-optimizations"):
            if bad in flag:
                errors.append(f"Forbidden compiler flag: {flag}")
    if not rep.get("kernel_hash"):
        errors.append("the backend must provide a kernel hash")
    return errors


def attestation_hash_input(rep: dict) -> bytes:
    """The bytes DeterminismReport::to_attestation_hash hashes
    (attestation.rs:254-300): u32-LE length-prefixed components -- backend,
    RNG method, FP mode, level, kernel hash bytes (the metallib_hash slot),
    verified flag, runtime version, device id, then the compiler flags sorted."""
    comps = [rep["backend_type"].encode(), rep["rng_seed_method"].encode(), rep["floating_point_mode"].encode(),
             rep["determinism_level"].encode()]
    if rep.get("kernel_hash"):
        comps.append(bytes.fromhex(rep["kernel_hash"]))
    comps.append(bytes([1 if rep.get("kernel_verified") else 0]))
    if rep.get("runtime_version"):
        comps.append(rep["runtime_version"].encode())
    if rep.get("device_id"):
        comps.append(rep["device_id"].encode())
    comps += [f.encode() for f in sorted(rep["compiler_flags"])]
    return b"".join(len(c).to_bytes(4, "little") + c for c in comps)


def lib():
    """Load libaoscuda.so (built in-tree); raise AosError if it is missing."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise AosError(-7, f"{LIB_PATH} is not built (run adapter-os_b200/build.py); "
                               "there is no CPU fallback")
        L = C.CDLL(LIB_PATH)
        vp, u32, u64, i32, f32 = C.c_void_p, C.c_uint32, C.c_uint64, C.c_int32, C.c_float
        sig = {
            "aos_version": (C.c_char_p, []),
            "aos_device_count": (C.c_int, []),
            "aos_last_error": (C.c_char_p, [vp]),
            "aos_route_batch": (C.c_int, [vp, vp, vp, vp, vp, u32, u32, vp, vp, vp, vp]),
            "aos_route_batch_dev": (C.c_int, [vp, vp, vp, vp, vp, u32, u32, vp, vp, vp, vp, vp]),
            "aos_lora_op_f32": (C.c_int, [vp, u32, u32, u32, vp, vp, vp, u32, u32, vp, vp, vp]),
            "aos_lora_op_f32_dev": (C.c_int, [vp, u32, u32, u32, vp, vp, vp, u32, u32, vp, vp, vp, vp]),
            "aos_init": (vp, [vp]),
            "aos_destroy": (None, [vp]),
            "aos_device_name": (C.c_char_p, [vp]),
            "aos_stream": (vp, [vp]),
            "aos_load_weight": (C.c_int, [vp, C.c_int, u32, C.c_int, vp, u64, C.c_int]),
            "aos_adapter_new": (C.c_int, [vp, C.c_uint16, u32, f32]),
            "aos_adapter_set_module": (C.c_int, [vp, C.c_uint16, u32, C.c_int, vp, vp, C.c_int]),
            "aos_adapter_unload": (C.c_int, [vp, C.c_uint16]),
            "aos_adapter_is_loaded": (C.c_int, [vp, C.c_uint16]),
            "aos_kv_alloc": (C.c_int, [vp, u64, u32]),
            "aos_kv_free": (C.c_int, [vp, u64]),
            "aos_kv_set_len": (C.c_int, [vp, u64, u32]),
            "aos_kv_get_len": (C.c_int, [vp, u64, vp]),
            "aos_kv_write": (C.c_int, [vp, u64, u32, u32, u32, vp, vp, C.c_int]),
            "aos_kv_read": (C.c_int, [vp, u64, u32, u32, u32, vp, vp]),
            "aos_kv_fill_synthetic": (C.c_int, [vp, u64, f32]),
            "aos_kv_rotate": (C.c_int, [vp, u64, u32]),
            "aos_kv_clear_all": (C.c_int, [vp]),
            "aos_kv_memory_bytes": (u64, [vp]),
            "aos_run_step_batch": (C.c_int, [vp, vp, vp, vp, u32, vp, vp]),
            "aos_run_step_batch_dev": (C.c_int, [vp, vp, vp, vp, u32, vp, vp, vp]),
            "aos_layer_step_dev": (C.c_int, [vp, u32, vp, vp, u32, vp, C.c_int, vp]),
            "aos_prefill_dev": (C.c_int, [vp, u32, vp, vp, vp, vp, vp, vp]),
            "aos_adapter_probe_safetensors": (C.c_int, [vp, u64, vp, u32, vp, vp, vp]),
            "aos_adapter_load_safetensors": (C.c_int, [vp, C.c_uint16, vp, u64, vp]),
            "aos_load_model_safetensors": (C.c_int, [vp, vp, u64]),
            "aos_shard_get_unique_id": (C.c_int, [vp]),
            "aos_shard_init": (C.c_int, [vp, u32, u32, vp]),
            "aos_run_step_sharded_dev": (C.c_int, [vp, vp, vp, vp, u32, vp, vp, vp]),
            "aos_get_metrics": (C.c_int, [vp, vp]),
            "aos_profile_enable": (C.c_int, [vp, C.c_int]),
            "aos_profile_read": (C.c_int, [vp, vp, C.c_int]),
            "aos_health_check": (C.c_int, [vp]),
            "aos_attest_determinism": (C.c_int, [vp, vp]),
            "aos_sample_dev": (C.c_int, [vp, u32, u32, u64, vp, vp, vp, vp]),
            "aos_debug_bounded_wait": (C.c_int, [vp, C.c_int]),
            "aos_memory_report": (C.c_int, [vp, vp, vp, u32, vp]),
            "aos_check_memory_footprint": (C.c_int, [vp, C.c_uint16, u64, vp, vp, vp, vp, vp]),
            "aos_get_gpu_fingerprints": (C.c_int, [vp, vp, vp, vp, u32, vp]),
            "aos_kv_set_generation": (C.c_int, [vp, u64]),
            "aos_kv_generation": (u64, [vp]),
            "aos_kv_ensure_coherence": (C.c_int, [vp, u64, vp]),
            "aos_kv_alloc_guarded": (C.c_int, [vp, u64, u32, u64]),
            "aos_kv_has_stale_guards": (C.c_int, [vp, u64]),
            "aos_kv_drain_guarded": (C.c_int, [vp, vp]),
            "aos_kv_zeroize": (C.c_int, [vp, u64]),
            "aos_kv_zeroize_all": (C.c_int, [vp]),
            "aos_archive_parse": (C.c_int, [vp, u64, vp, vp, u32]),
            "aos_blake3": (C.c_int, [vp, vp, u64, C.c_int, vp]),
            "aos_archive_verify": (C.c_int, [vp, vp, u64, vp]),
            "aos_adapter_load_aos": (C.c_int, [vp, C.c_uint16, vp, u64, C.c_char_p, vp]),
            "aos_adapter_verify_buffers": (C.c_int, [vp, C.c_uint16, vp, vp, vp, vp, vp]),
            "aos_adapter_fingerprint": (C.c_int, [vp, C.c_uint16, vp, vp]),
            "aos_store_gpu_fingerprint": (C.c_int, [vp, C.c_uint16, u64, C.c_char_p]),
            "aos_verify_gpu_fingerprint": (C.c_int, [vp, C.c_uint16, u64, C.c_char_p, vp]),
            "aos_plan_config_parse": (C.c_int, [C.c_char_p, u64, vp]),
            "aos_plan_config_validate": (C.c_int, [vp]),
            "aos_plan_config_validate_gqa": (C.c_int, [vp]),
            "aos_plan_validate_lora_targets": (C.c_int, [vp, u32]),
            "aos_plan_lora_size": (C.c_int, [vp, u32, vp, u32, vp]),
            "aos_model_config_from_plan": (C.c_int, [vp, u64, vp, vp]),
            "aos_init_from_plan": (vp, [vp, u64, vp, vp]),
        }
        for name, (res, args) in sig.items():
            if not hasattr(L, name):
                continue  # tests/test_capi_symbols.py reports missing exports
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


SHARD_ID_BYTES = 128


# ------------------------------------------------------------------ model plan
class PlanConfig(C.Structure):
    """aos_plan_config: the plan crate's ModelConfig with its derived values
    (crates/adapteros-lora-plan/src/config.rs:9-62, 171-208)."""

    _fields_ = [
        ("name", C.c_char * 128), ("architecture", C.c_char * 128),
        ("hidden_size", C.c_uint32), ("intermediate_size", C.c_uint32), ("num_hidden_layers", C.c_uint32),
        ("num_attention_heads", C.c_uint32), ("num_key_value_heads", C.c_uint32),
        ("max_position_embeddings", C.c_uint32), ("vocab_size", C.c_uint32), ("rope_theta", C.c_float),
        ("has_rope_scaling_factor", C.c_uint32), ("rope_scaling_factor", C.c_float),
        ("has_rope_scaling", C.c_uint32), ("scaling_factor", C.c_float),
        ("scaling_original_max_position_embeddings", C.c_uint32), ("scaling_type", C.c_char * 64),
        ("rms_norm_eps", C.c_float), ("head_dim", C.c_uint32), ("kv_width", C.c_uint32),
        ("total_params", C.c_uint64), ("effective_context_length", C.c_uint32), ("is_qwen2_5", C.c_uint32),
    ]

    def to_dict(self):
        return {k: (v.decode() if isinstance(v, bytes) else v)
                for k, v in ((f[0], getattr(self, f[0])) for f in self._fields_)}


def plan_config_parse(json_text, validate=True) -> PlanConfig:
    """ModelConfig::from_json (config.rs:80-86), then ModelConfig::validate
    (:127-167) unless validate is False; AosError with the reference's message."""
    raw = json_text.encode() if isinstance(json_text, str) else bytes(json_text)
    cfg = PlanConfig()
    check(lib().aos_plan_config_parse(raw, len(raw), C.byref(cfg)))
    if validate:
        check(lib().aos_plan_config_validate(C.byref(cfg)))
    return cfg


def plan_config_validate(cfg: PlanConfig, gqa_only=False):
    fn = lib().aos_plan_config_validate_gqa if gqa_only else lib().aos_plan_config_validate
    check(fn(C.byref(cfg)))


def _c_strings(names):
    arr = (C.c_char_p * max(1, len(names)))(*[n.encode() for n in names])
    return C.cast(arr, C.c_void_p), arr


def plan_validate_lora_targets(targets):
    """validate_lora_targets (config.rs:256-277)."""
    p, keep = _c_strings(list(targets))
    check(lib().aos_plan_validate_lora_targets(p, len(targets)))
    del keep


def plan_lora_size(cfg: PlanConfig, rank, targets) -> int:
    """calculate_lora_size (config.rs:212-253): fp16 bytes over every layer."""
    p, keep = _c_strings(list(targets))
    out = C.c_uint64()
    check(lib().aos_plan_lora_size(C.byref(cfg), int(rank), p, len(targets), C.byref(out)))
    del keep
    return out.value


def model_config_from_plan(plan_bytes: bytes, plan_cfg: PlanConfig = None) -> dict:
    """The model dimensions FusedKernels::load infers from a plan's tensor
    shapes (kernel-mtl/src/lib.rs:790-839; aos_model_config_from_plan)."""
    buf = C.create_string_buffer(bytes(plan_bytes), max(1, len(plan_bytes)))
    mc = ModelConfig()
    check(lib().aos_model_config_from_plan(buf, len(plan_bytes), C.byref(plan_cfg) if plan_cfg else None,
                                           C.byref(mc)))
    return {k: getattr(mc, k) for k in ("hidden", "n_heads", "n_kv_heads", "head_dim", "intermediate", "vocab",
                                        "n_layers", "rms_eps", "rope_theta")}


class AdapterMeta(C.Structure):
    """aos_adapter_meta: AdapterLoadMetadata (kernel-mtl/src/lib.rs:186-220)."""
    _fields_ = [("rank", C.c_uint32), ("alpha", C.c_float), ("target_modules", C.POINTER(C.c_char_p)),
                ("n_targets", C.c_uint32)]


def _adapter_meta(rank=0, alpha=0.0, target_modules=None):
    m = AdapterMeta(int(rank), float(alpha), None, 0)
    keep = None
    if target_modules is not None:
        keep = (C.c_char_p * max(1, len(target_modules)))(*[t.encode() for t in target_modules])
        m.target_modules = C.cast(keep, C.POINTER(C.c_char_p))
        m.n_targets = len(target_modules)
    return m, keep


def adapter_probe_safetensors(data: bytes, n_layers, rank=0, alpha=0.0, target_modules=None):
    """What aos_adapter_load_safetensors would load: (rank, alpha, found) with
    found[layer][module] bit 0 = lora_A, bit 1 = lora_B (no device needed)."""
    meta, keep = _adapter_meta(rank, alpha, target_modules)
    buf = C.create_string_buffer(bytes(data), len(data))
    r, a = C.c_uint32(0), C.c_float(0.0)
    found = np.zeros((n_layers, len(MODULES)), np.uint32)
    rc = lib().aos_adapter_probe_safetensors(buf, len(data), C.byref(meta), n_layers, C.byref(r), C.byref(a),
                                             _p(found))
    del keep
    if rc != 0:
        raise AosError(rc, last_error())
    return int(r.value), float(a.value), found


class ArchiveSegment(C.Structure):
    """aos_archive_segment: one 80-byte .aos index entry (adapteros-aos/src/writer.rs:313-323)."""
    _fields_ = [("segment_id", C.c_uint32), ("backend_tag", C.c_uint16), ("reserved", C.c_uint16),
                ("offset", C.c_uint64), ("len", C.c_uint64), ("scope_hash", C.c_uint8 * 16),
                ("weights_hash", C.c_uint8 * 32)]


class ArchiveInfo(C.Structure):
    _fields_ = [("flags", C.c_uint32), ("n_segments", C.c_uint32), ("manifest_offset", C.c_uint64),
                ("manifest_size", C.c_uint64)]


class ArchiveLoadInfo(C.Structure):
    _fields_ = [("rank", C.c_uint32), ("tensor_rank", C.c_uint32), ("storage_rank", C.c_uint32),
                ("alpha", C.c_float), ("module_mask", C.c_uint32), ("segment_id", C.c_uint32),
                ("backend_tag", C.c_uint16), ("reserved", C.c_uint16), ("weights_hash", C.c_uint8 * 32),
                ("scope_hash", C.c_uint8 * 16)]


BACKEND_TAGS = ("canonical", "mlx", "metal", "coreml")


def archive_parse(data: bytes):
    """Layout of a .aos archive (AosWriter::parse_header_bytes + parse_segments
    without the hash check; no device needed): (info dict, [segment dicts])."""
    buf = C.create_string_buffer(bytes(data), max(1, len(data)))
    info = ArchiveInfo()
    rc = lib().aos_archive_parse(buf, len(data), C.byref(info), None, 0)
    if rc != 0:
        raise AosError(rc, last_error())
    segs = (ArchiveSegment * max(1, info.n_segments))()
    check(lib().aos_archive_parse(buf, len(data), C.byref(info), segs, info.n_segments))
    out = [{"segment_id": s.segment_id, "backend": BACKEND_TAGS[s.backend_tag], "offset": s.offset, "len": s.len,
            "scope_hash": bytes(s.scope_hash).hex(), "weights_hash": bytes(s.weights_hash).hex()}
           for s in segs[:info.n_segments]]
    return {"flags": info.flags, "n_segments": info.n_segments, "manifest_offset": info.manifest_offset,
            "manifest_size": info.manifest_size}, out


class SampleParams(C.Structure):
    """aos_sample_params: Generator's temperature / top_k / top_p (generation.rs:9-21)."""
    _fields_ = [("temperature", C.c_float), ("top_k", C.c_uint32), ("top_p", C.c_float), ("flags", C.c_uint32)]


SAMPLE_GREEDY, SAMPLE_TOP_K, SAMPLE_TOP_P = 1, 2, 4


def sample_dev(logits, u=None, temperature=1.0, top_k=None, top_p=None, greedy=False, out=None, stream=None):
    """Next token per row of device logits [T, V] (f32) on the GPU:
    Generator::next_token (or greedy) of lora-worker/src/generation.rs:321-490
    with u [T] (device f32) as each row's uniform draw.  Returns uint32 [T]."""
    import torch
    T, V = logits.shape
    if out is None:
        out = torch.empty(T, dtype=torch.int32, device=logits.device)
    flags = (SAMPLE_GREEDY if greedy else 0) | (SAMPLE_TOP_K if top_k is not None else 0) | \
            (SAMPLE_TOP_P if top_p is not None else 0)
    prm = SampleParams(float(temperature), int(top_k or 0), float(top_p or 0.0), flags)
    if stream is None:
        stream = torch.cuda.current_stream(logits.device).cuda_stream
    rc = lib().aos_sample_dev(logits.data_ptr(), T, V, logits.stride(0), C.byref(prm),
                              u.data_ptr() if u is not None else None, out.data_ptr(), stream)
    if rc != 0:
        raise AosError(rc, last_error())
    return out


def _hkdf_sha256(ikm: bytes, info: bytes, n=32) -> bytes:
    """HKDF-SHA256 with no salt (RFC 5869), as derive_seed uses it (adapteros-core/src/seed.rs:986-1016)."""
    import hashlib
    import hmac
    prk = hmac.new(bytes(32), ikm, hashlib.sha256).digest()
    okm, block, i = b"", b"", 1
    while len(okm) < n:
        block = hmac.new(prk, block + info + bytes([i]), hashlib.sha256).digest()
        okm += block
        i += 1
    return okm[:n]


class DeterministicRng:
    """lora-worker/src/deterministic_rng.rs: ChaCha20Rng (rand_chacha 0.3) seeded
    with derive_seed(seed, label); gen_f32 is rand 0.8's Standard f32
    ((next_u32 >> 8) * 2^-24).  The keystream comes from the `cryptography`
    package's ChaCha20 with a zero counter and nonce (rand_chacha's stream 0)."""

    def __init__(self, seed32: bytes, label: str):
        from cryptography.hazmat.primitives.ciphers import Cipher, algorithms
        self.seed = _hkdf_sha256(bytes(seed32), label.encode())
        self._enc = Cipher(algorithms.ChaCha20(self.seed, bytes(16)), mode=None).encryptor()
        self._buf = b""

    def next_u32(self) -> int:
        if len(self._buf) < 4:
            self._buf += self._enc.update(bytes(256))
        v = int.from_bytes(self._buf[:4], "little")
        self._buf = self._buf[4:]
        return v

    def gen_f32(self) -> float:
        return float(np.float32(self.next_u32() >> 8) * np.float32(1.0 / (1 << 24)))


class Generator:
    """Generator (lora-worker/src/generation.rs): temperature, top-k, top-p and a
    seeded RNG; the sampling itself runs on the GPU (sample_dev)."""

    def __init__(self, seed: bytes = bytes(32), deterministic=False):
        self.base_seed = bytes(seed)
        self.rng = DeterministicRng(self.base_seed, "sampling")
        self.temperature, self.top_k, self.top_p = 1.0, None, None
        self.deterministic = deterministic

    @staticmethod
    def new_deterministic(seed_global: bytes, context: str):
        if len(seed_global) != 32:
            raise AosError(-1, "new_deterministic: a 32-byte global seed is required here")
        g = Generator(_hkdf_sha256(seed_global, context.encode()), deterministic=True)
        return g

    def with_temperature(self, t):
        self.temperature = max(float(np.float32(t)), 0.01)
        return self

    def with_top_k(self, k):
        self.top_k = int(k)
        return self

    def with_top_p(self, p):
        self.top_p = min(max(float(p), 0.0), 1.0)
        return self

    def reseed_for_step(self, step: int):
        if self.deterministic:  # derive_seed_indexed(base, "sample", step)
            self.rng = DeterministicRng(_hkdf_sha256(self.base_seed, f"sample:{step}".encode()), "sampling")

    def next_tokens_dev(self, logits, generators=None):
        """One token per row of device logits; row r draws from generators[r] (default: self)."""
        import torch
        gens = generators or [self] * logits.shape[0]
        u = torch.tensor([g.rng.gen_f32() for g in gens], dtype=torch.float32, device=logits.device)
        return sample_dev(logits, u, self.temperature, self.top_k, self.top_p)

    def next_token(self, logits) -> int:
        import torch
        x = logits if hasattr(logits, "data_ptr") else torch.tensor(np.asarray(logits, np.float32), device="cuda")
        return int(self.next_tokens_dev(x.reshape(1, -1).float().contiguous())[0].item())

    def greedy(self, logits) -> int:
        import torch
        x = logits if hasattr(logits, "data_ptr") else torch.tensor(np.asarray(logits, np.float32), device="cuda")
        return int(sample_dev(x.reshape(1, -1).float().contiguous(), greedy=True)[0].item())


def shard_unique_id() -> bytes:
    """NCCL unique id for aos_shard_init (made on one rank, shared by the caller)."""
    buf = C.create_string_buffer(SHARD_ID_BYTES)
    rc = lib().aos_shard_get_unique_id(buf)
    if rc != 0:
        raise AosError(rc, last_error())
    return buf.raw


def shard_owner(adapter_id: int, world: int) -> int:
    """Rank that holds an adapter in the adapter-sharded step (id mod world)."""
    return int(adapter_id) % int(world)


def last_error(ctx=None) -> str:
    m = lib().aos_last_error(ctx)
    return m.decode() if m else ""


def check(rc, ctx=None):
    if rc != 0:
        raise AosError(rc, last_error(ctx))
    return rc


def device_count() -> int:
    try:
        return int(lib().aos_device_count())
    except AosError:
        return 0


def _p(a):
    """Pointer of a numpy array or torch tensor (None -> NULL)."""
    if a is None:
        return None
    if hasattr(a, "data_ptr"):
        return a.data_ptr()
    return a.ctypes.data


def _params(k, tau, eps, routing_bias):
    return RouterParams(int(k), float(tau), float(eps), float(routing_bias))


# ------------------------------------------------------------------ RouterRing / IoBuffers
class RouterRing:
    """RouterRing (kernel-api/src/lib.rs:58-193): fixed [u16; 8] indices,
    [i16; 8] Q15 gates, k <= 8; unused entries zero-filled.  ``set`` follows
    RouterRing::set's release-build policy (length mismatch or out-of-range
    index -> zero-filled, k = 0)."""

    def __init__(self, k=0):
        self.indices = np.zeros(8, np.uint16)
        self.gates_q15 = np.zeros(8, np.int16)
        self.position = 0
        self.k = min(int(k), 8)
        self.dropout_seed = 0
        self.dropout_rate = 0.0

    def set(self, indices, gates, max_adapter=0xFFFF):
        if len(indices) != len(gates) or any(int(i) >= max_adapter for i in indices):
            self.indices[:] = 0
            self.gates_q15[:] = 0
            self.k = 0
            return
        k = min(len(indices), 8)
        self.indices[:] = 0
        self.gates_q15[:] = 0
        self.indices[:k] = np.asarray(indices[:k], np.uint16)
        self.gates_q15[:k] = np.asarray(gates[:k], np.int16)
        self.k = k

    def active_indices(self):
        return self.indices[: self.k]

    def active_gates(self):
        return self.gates_q15[: self.k]

    def to_record(self):
        r = np.zeros(1, RING_DTYPE)
        r[0]["top_k"], r[0]["position"] = self.k, self.position
        r[0]["indices"], r[0]["gates_q15"] = self.indices, self.gates_q15
        return r[0]

    @staticmethod
    def from_record(rec):
        r = RouterRing(int(rec["top_k"]))
        r.indices[:] = rec["indices"]
        r.gates_q15[:] = rec["gates_q15"]
        r.position = int(rec["position"])
        return r


class IoBuffers:
    """IoBuffers (kernel-api/src/lib.rs:221-246) for one sequence."""

    def __init__(self, vocab_size):
        self.input_ids = []
        self.output_logits = np.zeros(vocab_size, np.float32)
        self.position = 0
        self.attention_entropy = None
        self.activations = None
        self.session_id = None


# ------------------------------------------------------------------ router
def route_batch(priors, stable_ids=None, k=4, tau=1.0, eps=0.02, routing_bias=1.0,
                version_weights=None, allowed=None, positions=None, raise_on_nonfinite=True):
    """Batched router on the GPU (host arrays in, host arrays out).

    Returns (rings [T] RING_DTYPE, entropy [T] f32, status [T] i32).  A
    non-finite prior raises AosError(NONFINITE) like validate_router_inputs
    (router.rs:611-625) unless raise_on_nonfinite is False."""
    pr = np.ascontiguousarray(priors, dtype=np.float32)
    if pr.ndim == 1:
        pr = pr[None, :]
    T, N = pr.shape
    sid = np.ascontiguousarray(np.arange(N) if stable_ids is None else stable_ids, dtype=np.uint64)
    vw = None if version_weights is None else np.ascontiguousarray(version_weights, np.float32)
    al = None if allowed is None else np.ascontiguousarray(allowed, np.uint8)
    pos = None if positions is None else np.ascontiguousarray(positions, np.uint32)
    rings = np.zeros(T, RING_DTYPE)
    ent = np.zeros(T, np.float32)
    st = np.zeros(T, np.int32)
    p = _params(k, tau, eps, routing_bias)
    rc = lib().aos_route_batch(_p(pr), _p(sid), _p(vw), _p(al), _p(pos), T, N, C.byref(p), _p(rings),
                               _p(ent), _p(st))
    if rc != 0 and not (rc == -4 and not raise_on_nonfinite):
        raise AosError(rc, last_error())
    return rings, ent, st


def route_batch_dev(priors, stable_ids, rings_out, k=4, tau=1.0, eps=0.02, routing_bias=1.0,
                    version_weights=None, allowed=None, positions=None, entropy=None, status=None,
                    stream=None):
    """Device form: every array is a torch CUDA tensor; enqueued on ``stream``."""
    T, N = priors.shape
    p = _params(k, tau, eps, routing_bias)
    check(lib().aos_route_batch_dev(_p(priors), _p(stable_ids), _p(version_weights), _p(allowed),
                                    _p(positions), T, N, C.byref(p), _p(rings_out), _p(entropy),
                                    _p(status), stream))


# ------------------------------------------------------------------ fp32 LoRA op
def lora_op_f32(x, W, A, B, rings, alpha=None):
    """fp32 base + K-sparse LoRA on the GPU (host arrays); see aos_lora_op_f32."""
    x = np.ascontiguousarray(x, np.float32)
    W = np.ascontiguousarray(W, np.float32)
    A = np.ascontiguousarray(A, np.float32)
    B = np.ascontiguousarray(B, np.float32)
    rings = np.ascontiguousarray(rings, RING_DTYPE)
    T, ind = x.shape
    outd = W.shape[0]
    n_ad, rank, _ = A.shape
    al = None if alpha is None else np.ascontiguousarray(alpha, np.float32)
    y = np.zeros((T, outd), np.float32)
    check(lib().aos_lora_op_f32(_p(x), T, ind, outd, _p(W), _p(A), _p(B), n_ad, rank, _p(al),
                                _p(rings), _p(y)))
    return y


def lora_op_f32_dev(x, W, A, B, rings, y, alpha=None, stream=None):
    T, ind = x.shape
    outd = W.shape[0]
    n_ad, rank, _ = A.shape
    check(lib().aos_lora_op_f32_dev(_p(x), T, ind, outd, _p(W), _p(A), _p(B), n_ad, rank, _p(alpha),
                                    _p(rings), _p(y), stream))


# ------------------------------------------------------------------ FusedKernels
MOD_INDEX = {name: i for i, name in enumerate(MODULES)}
W_EMBED, W_LM_HEAD, W_FINAL_NORM, W_ATTN_NORM, W_MLP_NORM, W_PROJ = range(6)


class CudaKernels:
    """``FusedKernels`` implementation over libaoscuda (kernel-api/src/lib.rs:308-716).

    Method names follow the trait: ``load``-time weights go through
    ``load_weight``/``load_host_model``; ``load_adapter_with_metadata``,
    ``unload_adapter``, ``run_step`` (one sequence, one RouterRing), the batched
    ``run_step_batch`` (one ring per token), the KV-cache methods and
    ``get_metrics``/``health_check``/``attest_determinism``."""

    def __init__(self, hidden, n_heads, n_kv_heads, head_dim, intermediate, vocab, n_layers,
                 rms_eps=1e-5, rope_theta=1e6, rope_mlx_as_written=False, max_batch=64,
                 kv_block_size=16, kv_num_blocks=1024, max_seq_len=4096, lora_rank_capacity=1024,
                 lora_max_adapters=128, lora_modules=MODULES, device=0):
        mask = 0
        for m in lora_modules:
            mask |= 1 << MOD_INDEX[m]
        self.cfg = ModelConfig(hidden, n_heads, n_kv_heads, head_dim, intermediate, vocab, n_layers,
                               rms_eps, rope_theta, int(bool(rope_mlx_as_written)), max_batch,
                               kv_block_size, kv_num_blocks, max_seq_len, lora_rank_capacity,
                               lora_max_adapters, mask, device)
        L = lib()
        self._L = L
        self.ctx = L.aos_init(C.byref(self.cfg))
        if not self.ctx:
            raise AosError(-2, last_error())
        self.vocab, self.hidden, self.n_layers = vocab, hidden, n_layers
        self.n_kv_heads, self.head_dim = n_kv_heads, head_dim
        self._sessions = {}

    @classmethod
    def from_plan(cls, plan_bytes: bytes, plan_config=None, rope_mlx_as_written=False, max_batch=64,
                  kv_block_size=16, kv_num_blocks=1024, max_seq_len=4096, lora_rank_capacity=1024,
                  lora_max_adapters=128, lora_modules=MODULES, device=0):
        """FusedKernels::load(plan_bytes) (kernel-api/src/lib.rs:350): the model's
        dimensions come from the plan (safetensors base weights) and, when
        given, its model config (a PlanConfig or the config JSON); the keyword
        arguments are the runtime sizes.  aos_init_from_plan."""
        if plan_config is not None and not isinstance(plan_config, PlanConfig):
            plan_config = plan_config_parse(plan_config)
        mask = 0
        for m in lora_modules:
            mask |= 1 << MOD_INDEX[m]
        rt = ModelConfig(0, 0, 0, 0, 0, 0, 0, 0.0, 0.0, int(bool(rope_mlx_as_written)), max_batch, kv_block_size,
                         kv_num_blocks, max_seq_len, lora_rank_capacity, lora_max_adapters, mask, device)
        L = lib()
        buf = C.create_string_buffer(bytes(plan_bytes), max(1, len(plan_bytes)))
        ctx = L.aos_init_from_plan(buf, len(plan_bytes), C.byref(plan_config) if plan_config else None, C.byref(rt))
        if not ctx:
            raise AosError(-1, last_error())
        self = cls.__new__(cls)
        dims = model_config_from_plan(plan_bytes, plan_config)
        for k, v in dims.items():
            setattr(rt, k, v)
        self.cfg = rt
        self._L = L
        self.ctx = ctx
        self.vocab, self.hidden, self.n_layers = dims["vocab"], dims["hidden"], dims["n_layers"]
        self.n_kv_heads, self.head_dim = dims["n_kv_heads"], dims["head_dim"]
        self._sessions = {}
        return self

    def close(self):
        if getattr(self, "ctx", None):
            self._L.aos_destroy(self.ctx)
            self.ctx = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _check(self, rc):
        if rc != 0:
            raise AosError(rc, last_error(self.ctx))
        return rc

    def _ordered(self, stream, call):
        """Runs call(stream).  With stream=None the call goes on the context's
        own (non-blocking) stream, ordered after the work already queued on
        torch's current stream and before the work queued on it later, so
        tensors made and read by torch around the call are safe."""
        if stream is not None:
            return call(stream)
        import torch
        cur = torch.cuda.current_stream(self.cfg.device)
        ext = torch.cuda.ExternalStream(self.stream(), device=cur.device)
        ext.wait_stream(cur)
        try:
            return call(None)
        finally:
            cur.wait_stream(ext)

    # -- identity -------------------------------------------------------
    def device_name(self) -> str:
        return self._L.aos_device_name(self.ctx).decode()

    def stream(self):
        return self._L.aos_stream(self.ctx)

    def attest_determinism(self) -> dict:
        """FusedKernels::attest_determinism (kernel-api/src/lib.rs:383): the
        DeterminismReport fields, its validate() result and its attestation
        hash (BLAKE3 on the GPU).  kernel_verified: the library's build stamp
        equals the stamp of the kernel sources beside it (False where the
        sources are not deployed)."""
        r = DeterminismReport()
        self._check(self._L.aos_attest_determinism(self.ctx, C.byref(r)))
        stamp = r.kernel_build_id.decode()
        try:
            from . import build as _b
            verified = _b.current_stamp() == stamp
        except Exception:
            verified = False
        rep = {"backend": r.backend.decode(), "backend_type": "Cuda", "device": r.device_name.decode(),
               "sm": (r.sm_major, r.sm_minor), "fast_math": bool(r.fast_math),
               "float_atomics": bool(r.float_atomics),
               "fixed_reduction_order": bool(r.fixed_reduction_order),
               "build": stamp, "kernel_hash": stamp if len(stamp) == 64 else "", "kernel_verified": verified,
               "compiler_flags": r.compiler_flags.decode().split(),
               "runtime_version": r.runtime_version.decode(), "device_id": r.device_id.decode(),
               "rng_seed_method": RNG_METHODS[r.rng_seed_method],
               "floating_point_mode": FP_MODES[r.floating_point_mode],
               "determinism_level": DET_LEVELS[r.determinism_level], "deterministic": bool(r.deterministic)}
        rep["violations"] = validate_report(rep)
        rep["attestation_hash"] = self.blake3(attestation_hash_input(rep))
        return rep

    def get_metrics(self) -> dict:
        m = Metrics()
        self._check(self._L.aos_get_metrics(self.ctx, C.byref(m)))
        return {f: getattr(m, f) for f, _ in Metrics._fields_}

    def memory_report(self) -> dict:
        """FusedKernels::memory_report (kernel-api/src/lib.rs:588-593, GpuMemoryReportData)."""
        class Rep(C.Structure):
            _fields_ = [("total_gpu_bytes", C.c_uint64), ("used_gpu_bytes", C.c_uint64), ("adapter_count", C.c_uint32),
                        ("adapter_vram_total", C.c_uint64), ("arena_bytes", C.c_uint64),
                        ("arena_used_bytes", C.c_uint64), ("kv_pool_bytes", C.c_uint64), ("kv_used_bytes", C.c_uint64)]

        class Alloc(C.Structure):
            _fields_ = [("adapter_id", C.c_uint32), ("bytes", C.c_uint64)]

        r, n = Rep(), C.c_uint32(0)
        allocs = (Alloc * 1024)()
        self._check(self._L.aos_memory_report(self.ctx, C.byref(r), allocs, 1024, C.byref(n)))
        out = {f: getattr(r, f) for f, _ in Rep._fields_}
        out["adapter_allocations"] = [(a.adapter_id, a.bytes) for a in allocs[:min(n.value, 1024)]]
        return out

    def health_check(self):
        return self._check(self._L.aos_health_check(self.ctx))

    def profile_enable(self, on=True):
        """Per-kernel-class CUDA-event timing of every launch (steps run without graphs)."""
        self._check(self._L.aos_profile_enable(self.ctx, int(bool(on))))

    def profile_read(self, reset=True) -> dict:
        p = Profile()
        self._check(self._L.aos_profile_read(self.ctx, C.byref(p), int(bool(reset))))
        return {"steps": p.steps, "touched_groups": p.last_touched_groups,
                "ms": {k: p.ms[i] for i, k in enumerate(KERNEL_CLASSES)},
                "launches": {k: p.launches[i] for i, k in enumerate(KERNEL_CLASSES)}}

    # -- weights (FusedKernels::load) ------------------------------------
    def load_weight(self, kind, data, layer=0, module=0, on_device=False):
        n = data.numel() if hasattr(data, "numel") else data.size
        self._check(self._L.aos_load_weight(self.ctx, kind, layer, module, _p(data), n, int(on_device)))

    def load_host_model(self, m):
        """Load a model given as per-layer/module bf16 (uint16) arrays (oracle.HostModel layout)."""
        if m.embed is not None:
            self.load_weight(W_EMBED, m.embed)
            self.load_weight(W_LM_HEAD, m.lm_head)
            self.load_weight(W_FINAL_NORM, m.final_norm)
        for l in range(m.n_layers):
            self.load_weight(W_ATTN_NORM, m.attn_norm[l], layer=l)
            self.load_weight(W_MLP_NORM, m.mlp_norm[l], layer=l)
            for mod in range(7):
                self.load_weight(W_PROJ, m.w[mod][l], layer=l, module=mod)

    # -- hot-swap (load_adapter_with_metadata / unload_adapter) ----------
    def load_adapter_with_metadata(self, adapter_id, rank, alpha, modules):
        """modules: {(layer, module_index_or_name): (A [rank, in], B [out, rank])} bf16 bits."""
        self._check(self._L.aos_adapter_new(self.ctx, adapter_id, rank, float(alpha)))
        for (layer, mod), (A, B) in modules.items():
            mi = MOD_INDEX[mod] if isinstance(mod, str) else int(mod)
            dev = hasattr(A, "data_ptr") and A.is_cuda
            A = A if hasattr(A, "data_ptr") else np.ascontiguousarray(A, np.uint16)
            B = B if hasattr(B, "data_ptr") else np.ascontiguousarray(B, np.uint16)
            self._check(self._L.aos_adapter_set_module(self.ctx, adapter_id, layer, mi, _p(A), _p(B), int(dev)))

    def unload_adapter(self, adapter_id):
        self._check(self._L.aos_adapter_unload(self.ctx, adapter_id))

    def detach_adapter(self, adapter_id):
        """FusedKernels::detach_adapter: forwards to unload_adapter (kernel-api/src/lib.rs:414-420)."""
        self.unload_adapter(adapter_id)

    def attach_adapter(self, adapter_id):
        """FusedKernels::attach_adapter: a no-op, as the trait default (lib.rs:410-412); every
        loaded adapter is selectable by the router rings."""

    def switch_adapter(self, adapter_id):
        """FusedKernels::switch_adapter: a no-op, as the trait default (lib.rs:425-427)."""

    def load_adapter(self, adapter_id, weights: bytes):
        """FusedKernels::load_adapter (lib.rs:388): safetensors bytes with no metadata
        (rank / alpha / target modules from the tensors and the defaults)."""
        self.load_adapter_safetensors(adapter_id, weights)

    def is_loaded(self, adapter_id) -> bool:
        return bool(self._L.aos_adapter_is_loaded(self.ctx, adapter_id))

    # -- KV cache --------------------------------------------------------
    def supports_kv_cache(self):
        return True

    def kv_alloc(self, seq_id, max_tokens):
        self._check(self._L.aos_kv_alloc(self.ctx, seq_id, max_tokens))

    def kv_free(self, seq_id):
        self._check(self._L.aos_kv_free(self.ctx, seq_id))

    def kv_set_len(self, seq_id, n):
        self._check(self._L.aos_kv_set_len(self.ctx, seq_id, n))

    def kv_rotate(self, seq_id, shift):
        """Sliding-window rotate (kv_cache.metal:200-236): drop the oldest
        `shift` positions of the sequence in every layer."""
        self._check(self._L.aos_kv_rotate(self.ctx, seq_id, shift))

    def kv_len(self, seq_id):
        v = C.c_uint32()
        self._check(self._L.aos_kv_get_len(self.ctx, seq_id, C.byref(v)))
        return v.value

    def kv_write(self, seq_id, layer, pos0, k, v):
        k = np.ascontiguousarray(k, np.uint16)
        v = np.ascontiguousarray(v, np.uint16)
        self._check(self._L.aos_kv_write(self.ctx, seq_id, layer, pos0, k.shape[0], _p(k), _p(v), 0))

    def kv_read(self, seq_id, layer, pos0, n):
        k = np.zeros((n, self.n_kv_heads, self.head_dim), np.uint16)
        v = np.zeros_like(k)
        self._check(self._L.aos_kv_read(self.ctx, seq_id, layer, pos0, n, _p(k), _p(v)))
        return k, v

    def kv_fill_synthetic(self, seed=0, std=1.0):
        self._check(self._L.aos_kv_fill_synthetic(self.ctx, seed, float(std)))

    def clear_session_cache(self, session_id):
        sid = self._sessions.pop(session_id, None)
        if sid is not None:
            self.kv_free(sid)

    # -- KvCache generation guards and zeroization (kvcache.rs:288-402, 586-733)
    def set_generation(self, generation):
        self._check(self._L.aos_kv_set_generation(self.ctx, int(generation)))

    def generation(self) -> int:
        return int(self._L.aos_kv_generation(self.ctx))

    def ensure_cache_coherence(self, generation) -> bool:
        r = C.c_int(0)
        self._check(self._L.aos_kv_ensure_coherence(self.ctx, int(generation), C.byref(r)))
        return bool(r.value)

    def allocate_with_guard(self, seq_id, max_tokens, generation):
        self._check(self._L.aos_kv_alloc_guarded(self.ctx, int(seq_id), int(max_tokens), int(generation)))

    def has_active_sequences_with_generation(self, generation) -> bool:
        return bool(self._L.aos_kv_has_stale_guards(self.ctx, int(generation)))

    def drain_active_sequences(self) -> int:
        n = C.c_uint32(0)
        self._check(self._L.aos_kv_drain_guarded(self.ctx, C.byref(n)))
        return int(n.value)

    def zeroize_sequence(self, seq_id):
        self._check(self._L.aos_kv_zeroize(self.ctx, int(seq_id)))

    def zeroize_all(self):
        self._check(self._L.aos_kv_zeroize_all(self.ctx))

    def clear_all_caches(self):
        self._check(self._L.aos_kv_clear_all(self.ctx))
        self._sessions.clear()

    def cache_memory_bytes(self):
        return int(self._L.aos_kv_memory_bytes(self.ctx))

    # -- the step --------------------------------------------------------
    def run_step_batch(self, rings, token_ids, seq_ids, want_logits=True, want_hidden=False):
        """One decode token per entry (host arrays); returns (logits [T,V] f32, hidden [T,H] bf16 bits)."""
        rings = np.ascontiguousarray(rings, RING_DTYPE)
        tok = np.ascontiguousarray(token_ids, np.uint32)
        sid = np.ascontiguousarray(seq_ids, np.uint64)
        T = len(tok)
        logits = np.zeros((T, self.vocab), np.float32) if want_logits else None
        hidden = np.zeros((T, self.hidden), np.uint16) if want_hidden else None
        self._check(self._L.aos_run_step_batch(self.ctx, _p(rings), _p(tok), _p(sid), T, _p(logits), _p(hidden)))
        return logits, hidden

    def run_step_batch_dev(self, rings, token_ids, seq_ids, logits=None, hidden=None, stream=None):
        """Device form: rings/token_ids/logits/hidden are torch CUDA tensors; seq_ids a host array."""
        sid = np.ascontiguousarray(seq_ids, np.uint64)
        self._ordered(stream, lambda st: self._check(self._L.aos_run_step_batch_dev(
            self.ctx, _p(rings), _p(token_ids), _p(sid), len(sid), _p(logits), _p(hidden), st)))

    # -- safetensors loading --------------------------------------------------
    def load_adapter_safetensors(self, adapter_id, data: bytes, rank=0, alpha=0.0, target_modules=None):
        """FusedKernels::load_adapter_with_metadata from safetensors bytes."""
        meta, keep = _adapter_meta(rank, alpha, target_modules)
        buf = C.create_string_buffer(bytes(data), len(data))
        self._check(self._L.aos_adapter_load_safetensors(self.ctx, int(adapter_id), buf, len(data), C.byref(meta)))
        del keep

    def load_model_safetensors(self, data: bytes):
        """Base weights under the Hugging Face LLaMA tensor names."""
        buf = C.create_string_buffer(bytes(data), len(data))
        self._check(self._L.aos_load_model_safetensors(self.ctx, buf, len(data)))

    # -- .aos archives and GPU fingerprints ---------------------------------
    def blake3(self, data) -> str:
        """BLAKE3 hex digest computed on the GPU; data: bytes, or a CUDA tensor."""
        out = C.create_string_buffer(32)
        if hasattr(data, "data_ptr"):
            n = data.numel() * data.element_size()
            self._check(self._L.aos_blake3(self.ctx, data.data_ptr(), n, 1, out))
        else:
            buf = C.create_string_buffer(bytes(data), max(1, len(data)))
            self._check(self._L.aos_blake3(self.ctx, buf, len(data), 0, out))
        return out.raw.hex()

    def archive_verify(self, data: bytes):
        """open_aos: layout plus every segment hash (on the GPU); raises on a bad archive."""
        buf = C.create_string_buffer(bytes(data), max(1, len(data)))
        bad = C.c_int32(-1)
        self._check(self._L.aos_archive_verify(self.ctx, buf, len(data), C.byref(bad)))

    def load_adapter_aos(self, adapter_id, data: bytes, backend="canonical") -> dict:
        """LifecycleLoader::load_from_aos_static into adapter slot adapter_id."""
        buf = C.create_string_buffer(bytes(data), max(1, len(data)))
        info = ArchiveLoadInfo()
        self._check(self._L.aos_adapter_load_aos(self.ctx, int(adapter_id), buf, len(data),
                                                 backend.encode() if backend else None, C.byref(info)))
        return {"rank": info.rank, "tensor_rank": info.tensor_rank, "storage_rank": info.storage_rank,
                "alpha": info.alpha, "modules": [MODULES[m] for m in range(len(MODULES)) if info.module_mask >> m & 1],
                "segment_id": info.segment_id, "backend": BACKEND_TAGS[info.backend_tag],
                "weights_hash": bytes(info.weights_hash).hex(), "scope_hash": bytes(info.scope_hash).hex()}

    def verify_adapter_buffers(self, adapter_id):
        """(buffer_bytes, first, last, mid) samples of the adapter's arena buffer."""
        size, n = C.c_uint64(0), C.c_uint32(0)
        bufs = [C.create_string_buffer(4096) for _ in range(3)]
        self._check(self._L.aos_adapter_verify_buffers(self.ctx, int(adapter_id), C.byref(size), bufs[0], bufs[1],
                                                       bufs[2], C.byref(n)))
        return int(size.value), bufs[0].raw[:n.value], bufs[1].raw[:n.value], bufs[2].raw[:n.value]

    def adapter_fingerprint(self, adapter_id):
        """(buffer_bytes, BLAKE3 hex of first || last || mid), hashed on the GPU."""
        size, h = C.c_uint64(0), C.create_string_buffer(32)
        self._check(self._L.aos_adapter_fingerprint(self.ctx, int(adapter_id), C.byref(size), h))
        return int(size.value), h.raw.hex()

    def store_gpu_fingerprint(self, adapter_id, buffer_bytes, checkpoint_hash_hex):
        self._check(self._L.aos_store_gpu_fingerprint(self.ctx, int(adapter_id), int(buffer_bytes),
                                                      checkpoint_hash_hex.encode()))

    def check_memory_footprint(self, adapter_id, buffer_bytes):
        """(within_tolerance, z_score, (mean, stddev, samples))."""
        w, z, m, sd, n = C.c_int(0), C.c_double(0), C.c_double(0), C.c_double(0), C.c_uint32(0)
        self._check(self._L.aos_check_memory_footprint(self.ctx, int(adapter_id), int(buffer_bytes), C.byref(w),
                                                       C.byref(z), C.byref(m), C.byref(sd), C.byref(n)))
        return bool(w.value), float(z.value), (float(m.value), float(sd.value), int(n.value))

    def get_gpu_fingerprints(self) -> dict:
        """{adapter id: (buffer bytes, checkpoint hash hex)} of the stored baselines."""
        n = C.c_uint32(0)
        self._check(self._L.aos_get_gpu_fingerprints(self.ctx, None, None, None, 0, C.byref(n)))
        k = n.value
        ids, nb, hx = (C.c_uint32 * max(1, k))(), (C.c_uint64 * max(1, k))(), C.create_string_buffer(65 * max(1, k))
        self._check(self._L.aos_get_gpu_fingerprints(self.ctx, ids, nb, hx, k, C.byref(n)))
        return {int(ids[i]): (int(nb[i]), hx.raw[65 * i:65 * i + 64].decode()) for i in range(k)}

    def verify_gpu_fingerprint(self, adapter_id, buffer_bytes, checkpoint_hash_hex) -> bool:
        m = C.c_int(0)
        self._check(self._L.aos_verify_gpu_fingerprint(self.ctx, int(adapter_id), int(buffer_bytes),
                                                       checkpoint_hash_hex.encode(), C.byref(m)))
        return bool(m.value)

    # -- prefill ----------------------------------------------------------
    def prefill_dev(self, seq_ids, n_tok, rings, token_ids, logits=None, stream=None):
        """Prompt pass: sequence i takes n_tok[i] tokens from its current length
        on (causal attention over its cache).  rings/token_ids/logits are torch
        CUDA tensors (the concatenation over sequences; logits [n_seq, vocab]
        for each sequence's last token, optional); seq_ids/n_tok host arrays."""
        sid = np.ascontiguousarray(seq_ids, np.uint64)
        nt = np.ascontiguousarray(n_tok, np.uint32)
        self._ordered(stream, lambda st: self._check(self._L.aos_prefill_dev(
            self.ctx, len(sid), _p(sid), _p(nt), _p(rings), _p(token_ids), _p(logits), st)))

    # -- the worker's generation loop ---------------------------------------
    def generate_tokens(self, generators, stable_ids, initial_tokens, max_tokens, eos_token, seq_ids, k=4):
        """Generator::generate_tokens (lora-worker/src/generation.rs:226-310),
        batched over sequences: each step reseeds every live sequence's
        generator for the step, routes with uniform priors 1/N over the
        adapters (ring position = current length - 1), runs one decode step for
        the live sequences' last tokens, samples on the GPU, and drops a
        sequence when it draws eos_token.  The prompt up to its last token is
        cached first (prefill), so a step's input sits at position len - 1 as
        the reference's IoBuffers.position says.  Returns the token lists."""
        import torch
        dev = torch.device("cuda", self.cfg.device)
        st = self.stream()  # routing, steps, sampling and torch's own copies all in the context's stream order
        with torch.cuda.stream(torch.cuda.ExternalStream(st, device=dev)):
            return self._generate(generators, stable_ids, initial_tokens, max_tokens, eos_token, seq_ids, k, dev, st)

    def _generate(self, generators, stable_ids, initial_tokens, max_tokens, eos_token, seq_ids, k, dev, st):
        import torch
        n, N = len(initial_tokens), len(stable_ids)
        toks = [list(map(int, t)) for t in initial_tokens]
        if any(len(t) == 0 for t in toks):
            raise AosError(-1, "Token sequence cannot be empty during generation")
        sids = torch.tensor(np.asarray(stable_ids, np.uint64).view(np.int64), device=dev)
        prior = float(np.float32(1.0) / np.float32(N))

        def rings_for(positions):
            T = len(positions)
            rings = torch.zeros((T, 40), dtype=torch.uint8, device=dev)
            route_batch_dev(torch.full((T, N), prior, dtype=torch.float32, device=dev), sids, rings, k=k,
                            positions=torch.tensor(positions, dtype=torch.int32, device=dev), stream=st)
            return rings

        for s, t in zip(seq_ids, toks):
            self.kv_alloc(int(s), len(t) + int(max_tokens))
        pre = [i for i in range(n) if len(toks[i]) > 1]
        if pre:
            pos = [p for i in pre for p in range(len(toks[i]) - 1)]
            ids = torch.tensor([x for i in pre for x in toks[i][:-1]], dtype=torch.int32, device=dev)
            self.prefill_dev([seq_ids[i] for i in pre], [len(toks[i]) - 1 for i in pre], rings_for(pos), ids,
                             stream=st)
        logits = torch.empty((n, self.vocab), dtype=torch.float32, device=dev)
        active = list(range(n))
        for step in range(int(max_tokens)):
            if not active:
                break
            for i in active:
                generators[i].reseed_for_step(step)
            T = len(active)
            rings = rings_for([len(toks[i]) - 1 for i in active])
            last = torch.tensor([toks[i][-1] for i in active], dtype=torch.int32, device=dev)
            self.run_step_batch_dev(rings, last, [seq_ids[i] for i in active], logits=logits[:T], stream=st)
            nxt = np.zeros(T, np.int64)
            groups = {}
            for j, i in enumerate(active):  # rows sharing sampling settings go in one launch
                g = generators[i]
                groups.setdefault((g.temperature, g.top_k, g.top_p), []).append(j)
            for rows in groups.values():
                sub = logits[torch.tensor(rows, device=dev)]
                lead = generators[active[rows[0]]]
                got = lead.next_tokens_dev(sub, [generators[active[j]] for j in rows]).cpu().numpy()
                nxt[rows] = got
            still = []
            for j, i in enumerate(active):
                if int(nxt[j]) == int(eos_token):
                    continue
                toks[i].append(int(nxt[j]))
                still.append(i)
            active = still
        return toks

    # -- adapter-sharded step ---------------------------------------------
    def shard_init(self, rank, world, unique_id: bytes):
        """Join the adapter-sharded group (collective over the world ranks).
        This context must hold only adapters with id % world == rank."""
        buf = C.create_string_buffer(bytes(unique_id), SHARD_ID_BYTES)
        self._check(self._L.aos_shard_init(self.ctx, int(rank), int(world), buf))
        self.shard = (int(rank), int(world))

    def run_step_sharded_dev(self, rings, token_ids, seq_ids, logits=None, hidden=None, stream=None):
        """Decode step of this rank's home tokens (collective; same T on every
        rank).  Arguments as run_step_batch_dev; rings carry global adapter ids."""
        sid = np.ascontiguousarray(seq_ids, np.uint64)
        self._ordered(stream, lambda st: self._check(self._L.aos_run_step_sharded_dev(
            self.ctx, _p(rings), _p(token_ids), _p(sid), len(sid), _p(logits), _p(hidden), st)))

    def layer_step_dev(self, layer, rings, seq_ids, hidden, advance=False, stream=None):
        sid = np.ascontiguousarray(seq_ids, np.uint64)
        self._ordered(stream, lambda st: self._check(self._L.aos_layer_step_dev(
            self.ctx, layer, _p(rings), _p(sid), len(sid), _p(hidden), int(advance), st)))

    def run_step(self, ring: RouterRing, io: IoBuffers):
        """FusedKernels::run_step for one sequence: every id in io.input_ids is
        decoded in turn at io.position; output_logits gets the last token's
        logits and io.position advances by len(input_ids)
        (mlx-ffi/src/backend.rs:1212-1310)."""
        if not io.input_ids:
            raise AosError(-1, "Input token IDs cannot be empty")
        key = io.session_id
        if key not in self._sessions:
            sid = len(self._sessions) + (1 << 62)
            self.kv_alloc(sid, int(self.cfg.max_seq_len))
            self._sessions[key] = sid
        sid = self._sessions[key]
        self.kv_set_len(sid, io.position)
        rec = np.zeros(1, RING_DTYPE)
        rec[0] = ring.to_record()
        logits = None
        for tok in io.input_ids:
            logits, _ = self.run_step_batch(rec, [tok], [sid])
        io.output_logits[: self.vocab] = logits[0][: len(io.output_logits)]
        io.position += len(io.input_ids)
