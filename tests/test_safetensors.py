"""Loading adapters and base weights from safetensors bytes
(aos_adapter_probe_safetensors / aos_adapter_load_safetensors /
aos_load_model_safetensors), following FusedKernels::load_adapter_with_metadata
(crates/adapteros-lora-kernel-mtl/src/lib.rs:186-251, 1893-2046) and the
base-weight names of kernel-mtl/src/lib.rs:660-1000.

CPU tests: tensor matching, rank / alpha resolution, target-module handling
and malformed containers, through the context-free probe.  GPU tests: an
adapter and a model loaded from safetensors (F32, F16 and BF16 tensors) decode
bit-identically to the same values loaded through the array entry points."""
import json
import struct

import numpy as np
import pytest

from tests.aos_import import aos

DT = {np.float32: "F32", np.float16: "F16"}


def st_bytes(tensors, metadata=None):
    """safetensors container: u64 header length, JSON header, tensor bytes.
    Values may be np.float32 / np.float16 arrays or ("BF16", uint16 array)."""
    header, blobs, off = {}, [], 0
    for name, v in tensors.items():
        if isinstance(v, tuple):
            dtype, arr = v
        else:
            arr = v
            dtype = DT[arr.dtype.type]
        raw = np.ascontiguousarray(arr).tobytes()
        header[name] = {"dtype": dtype, "shape": list(arr.shape), "data_offsets": [off, off + len(raw)]}
        blobs.append(raw)
        off += len(raw)
    if metadata is not None:
        header["__metadata__"] = metadata
    h = json.dumps(header).encode()
    return struct.pack("<Q", len(h)) + h + b"".join(blobs)


def peft_adapter(rng, n_layers, rank, shapes, modules, dtype=np.float32, prefix="base_model.model.model.layers"):
    t = {}
    for l in range(n_layers):
        for m in modules:
            out, inn = shapes[m]
            blk = "self_attn" if m in ("q_proj", "k_proj", "v_proj", "o_proj") else "mlp"
            t[f"{prefix}.{l}.{blk}.{m}.lora_A.weight"] = (rng.standard_normal((rank, inn)) * 0.02).astype(dtype)
            t[f"{prefix}.{l}.{blk}.{m}.lora_B.weight"] = (rng.standard_normal((out, rank)) * 0.02).astype(dtype)
    return t


SHAPES = {"q_proj": (256, 256), "k_proj": (128, 256), "v_proj": (128, 256), "o_proj": (256, 256),
          "gate_proj": (384, 256), "up_proj": (384, 256), "down_proj": (256, 384)}
ALL = list(SHAPES)


def mi(name):
    return aos.MODULES.index(name)


def test_probe_defaults_and_inference():
    rng = np.random.default_rng(0)
    data = st_bytes(peft_adapter(rng, 2, 8, SHAPES, ALL), metadata={"format": "pt"})
    rank, alpha, found = aos.adapter_probe_safetensors(data, 2)
    assert rank == 8 and alpha == 16.0  # lora_A rows; alpha = 2 * rank
    # the default target set (kernel-mtl DEFAULT_METAL_TARGET_MODULES): no o_proj / gate_proj
    for l in range(2):
        for m in ALL:
            want = 3 if m in ("q_proj", "k_proj", "v_proj", "down_proj", "up_proj") else 0
            assert found[l, mi(m)] == want, (l, m)


def test_probe_metadata_targets_rank_alpha():
    rng = np.random.default_rng(1)
    data = st_bytes(peft_adapter(rng, 2, 8, SHAPES, ALL))
    rank, alpha, found = aos.adapter_probe_safetensors(data, 2, rank=8, alpha=5.0,
                                                       target_modules=["  o_proj ", "o_proj", "", "gate_proj"])
    assert (rank, alpha) == (8, 5.0)
    assert set(zip(*np.nonzero(found))) == {(l, mi(m)) for l in range(2) for m in ("o_proj", "gate_proj")}
    # non-finite / non-positive alpha and zero rank fall back
    rank, alpha, _ = aos.adapter_probe_safetensors(data, 2, rank=0, alpha=float("nan"))
    assert (rank, alpha) == (8, 16.0)


def test_probe_unmatched_metadata_falls_back_to_defaults():
    rng = np.random.default_rng(2)
    data = st_bytes(peft_adapter(rng, 1, 16, SHAPES, ["q_proj", "up_proj"]))
    rank, alpha, found = aos.adapter_probe_safetensors(data, 1, target_modules=["c_attn"])
    assert rank == 16 and found[0, mi("q_proj")] == 3 and found[0, mi("up_proj")] == 3


def test_probe_single_layer_names_and_missing_b():
    rng = np.random.default_rng(3)
    t = {"q_proj.lora_A.weight": (rng.standard_normal((4, 256)) * 0.02).astype(np.float32),
         "k_proj.lora_A.weight": (rng.standard_normal((4, 256)) * 0.02).astype(np.float32),
         "k_proj.lora_B.weight": (rng.standard_normal((128, 4)) * 0.02).astype(np.float32)}
    rank, _, found = aos.adapter_probe_safetensors(st_bytes(t), 2)
    assert rank == 4
    assert found[0, mi("q_proj")] == 1 and found[0, mi("k_proj")] == 3 and not found[1].any()


def test_probe_errors():
    rng = np.random.default_rng(4)
    with pytest.raises(aos.AosError, match="no LoRA tensors"):
        aos.adapter_probe_safetensors(st_bytes({"model.norm.weight": np.ones(8, np.float32)}), 1)
    good = st_bytes(peft_adapter(rng, 1, 8, SHAPES, ["q_proj"]))
    with pytest.raises(aos.AosError):
        aos.adapter_probe_safetensors(good[:20], 1)  # header cut short
    with pytest.raises(aos.AosError):
        aos.adapter_probe_safetensors(b"\x01\x02", 1)
    h = json.dumps({"x.q_proj.lora_A.weight": {"dtype": "F32", "shape": [1, 4], "data_offsets": [0, 64]}}).encode()
    with pytest.raises(aos.AosError, match="past the buffer"):
        aos.adapter_probe_safetensors(struct.pack("<Q", len(h)) + h + bytes(16), 1)


# ---------------------------------------------------------------- GPU
def _small_gpu(m, n_ad):
    return aos.CudaKernels(m.hidden, m.n_heads, m.n_kv_heads, 128, m.inter, m.vocab, m.n_layers, max_batch=8,
                           kv_num_blocks=64, max_seq_len=128, lora_rank_capacity=128, lora_max_adapters=n_ad)


@pytest.mark.gpu
def test_gpu_adapter_and_model_from_safetensors_match_array_loads():
    from oracle import oracle as O
    rng = np.random.default_rng(5)
    m = O.HostModel.random(rng, 256, 2, 1, 128, 384, 512, 2)
    # adapter 0 in F32, adapter 1 in F16, adapter 2 in BF16 (values exact in bf16)
    ad = O.HostAdapters.random(rng, m, [8, 16, 8], modules=range(7))
    files = []
    for a, kind in enumerate(("F32", "F16", "BF16")):
        t = {}
        for l in range(2):
            for mod in range(7):
                name = aos.MODULES[mod]
                blk = "self_attn" if mod < 4 else "mlp"
                A, B = O.bf16_bits_to_f32(ad.A[a][l][mod]), O.bf16_bits_to_f32(ad.B[a][l][mod])
                if kind == "F16":  # keep the adapter's values where f16 holds them exactly
                    A, B = A.astype(np.float16).astype(np.float32), B.astype(np.float16).astype(np.float32)
                    ad.A[a][l][mod], ad.B[a][l][mod] = O.f32_to_bf16_bits(A), O.f32_to_bf16_bits(B)
                    A, B = A.astype(np.float16), B.astype(np.float16)
                elif kind == "BF16":
                    A, B = ("BF16", ad.A[a][l][mod]), ("BF16", ad.B[a][l][mod])
                t[f"base_model.model.model.layers.{l}.{blk}.{name}.lora_A.weight"] = A
                t[f"base_model.model.model.layers.{l}.{blk}.{name}.lora_B.weight"] = B
        files.append(st_bytes(t))
    model = {"model.embed_tokens.weight": ("BF16", m.embed), "lm_head.weight": O.bf16_bits_to_f32(m.lm_head),
             "model.norm.weight": ("BF16", m.final_norm)}
    for l in range(2):
        model[f"model.layers.{l}.input_layernorm.weight"] = ("BF16", m.attn_norm[l])
        model[f"model.layers.{l}.post_attention_layernorm.weight"] = ("BF16", m.mlp_norm[l])
        for mod in range(7):
            blk = "self_attn" if mod < 4 else "mlp"
            model[f"model.layers.{l}.{blk}.{aos.MODULES[mod]}.weight"] = ("BF16", m.w[mod][l])
    T = 5
    rings, _, _, _ = O.route_batch(rng.standard_normal((T, 3)).astype(np.float32), None, k=2)
    toks = rng.integers(0, 512, size=T).astype(np.uint32)
    outs = []
    for from_st in (False, True):
        gpu = _small_gpu(m, 3)
        if from_st:
            gpu.load_model_safetensors(st_bytes(model))
            for a in range(3):
                gpu.load_adapter_safetensors(a, files[a], target_modules=list(aos.MODULES))
        else:
            gpu.load_host_model(m)
            for a in range(3):
                gpu.load_adapter_with_metadata(a, ad.ranks[a], 2.0 * ad.ranks[a],
                                               {(l, mod): (ad.A[a][l][mod], ad.B[a][l][mod])
                                                for l in range(2) for mod in range(7)})
        sids = np.arange(T, dtype=np.uint64)
        for s in sids:
            gpu.kv_alloc(int(s), 64)
        logits, _ = gpu.run_step_batch(rings, toks, sids)
        outs.append(logits)
        gpu.close()
    assert outs[0].tobytes() == outs[1].tobytes()
