"""Model plan loading (FusedKernels::load(plan_bytes)): the plan crate's
ModelConfig (crates/adapteros-lora-plan/src/config.rs) and the dimension
inference of the Metal backend's load (crates/adapteros-lora-kernel-mtl/src/
lib.rs:1476-1537, 790-839), through aos_plan_config_* and
aos_model_config_from_plan / aos_init_from_plan.

CPU: the reference's own known answers for the Qwen2.5-7B config
(config.rs:282-389: head_dim 128, kv_width 512, is_qwen2_5, ~77 MB of rank-16
LoRA on all seven targets, hidden 3585 refused), serde's required-field and
type rules, the validation messages, and the model dimensions taken from a
plan's tensor shapes (with and without a model config, and the errors the
reference raises).  GPU: a context made from the plan decodes bit-identically
to one given the same weights through aos_init + the array loads."""
import numpy as np
import pytest

from tests.aos_import import aos
from tests.test_safetensors import st_bytes

QWEN = """{
    "name": "Qwen2.5-7B",
    "architecture": "Qwen2.5ForCausalLM",
    "hidden_size": 3584,
    "intermediate_size": 18944,
    "num_hidden_layers": 28,
    "num_attention_heads": 28,
    "num_key_value_heads": 4,
    "max_position_embeddings": 32768,
    "rope_theta": 1000000.0,
    "vocab_size": 151936
}"""
ALL = ["q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj"]


def test_qwen2_5_config_parsing():  # config.rs:286-311
    c = aos.plan_config_parse(QWEN)
    assert (c.hidden_size, c.num_attention_heads, c.num_key_value_heads) == (3584, 28, 4)
    assert c.is_qwen2_5 == 1
    assert (c.head_dim, c.kv_width) == (128, 512)
    assert c.name == b"Qwen2.5-7B" and c.vocab_size == 151936 and c.rope_theta == 1e6
    assert c.effective_context_length == 32768  # no rope_scaling
    # dimensions(): 28 layers of (4 H^2 + 3 H I) plus embedding and output
    assert c.total_params == (3584 * 3584 * 4 + 3584 * 18944 * 3) * 28 + 151936 * 3584 * 2


def test_lora_size_calculation():  # config.rs:313-345
    c = aos.plan_config_parse(QWEN)
    b = aos.plan_lora_size(c, 16, ALL)
    assert 70 <= b // (1024 * 1024) <= 85
    per_layer = 16 * ((3584 + 3584) * 2 + (3584 + 512) * 2 + (3584 + 18944) * 3)
    assert b == per_layer * 28 * 2
    with pytest.raises(aos.AosError, match="Unknown LoRA target: lm_head"):
        aos.plan_lora_size(c, 16, ["q_proj", "lm_head"])
    aos.plan_validate_lora_targets(ALL)
    with pytest.raises(aos.AosError, match=r'Invalid LoRA target: qproj\. Valid targets: \["q_proj"'):
        aos.plan_validate_lora_targets(["qproj"])


def test_config_validation():  # config.rs:347-389
    aos.plan_config_parse(QWEN)  # validates
    bad = QWEN.replace('"hidden_size": 3584', '"hidden_size": 3585')
    c = aos.plan_config_parse(bad, validate=False)  # parses, fails validation
    with pytest.raises(aos.AosError, match=r"hidden_size \(3585\) must be divisible by num_attention_heads \(28\)"):
        aos.plan_config_validate(c)
    gqa = QWEN.replace('"num_key_value_heads": 4', '"num_key_value_heads": 3')
    with pytest.raises(aos.AosError, match=r"num_attention_heads \(28\) must be divisible by num_key_value_heads \(3\)"):
        aos.plan_config_validate(aos.plan_config_parse(gqa, validate=False), gqa_only=True)
    with pytest.raises(aos.AosError, match="vocab_size must be non-zero"):
        aos.plan_config_parse(QWEN.replace('"vocab_size": 151936', '"vocab_size": 0'))
    scaled = QWEN[:-1].rstrip() + ', "rope_scaling": {"factor": 4.0, "original_max_position_embeddings": 32768, ' \
                                  '"scaling_type": "yarn"}}'
    c = aos.plan_config_parse(scaled)
    assert c.has_rope_scaling == 1 and c.effective_context_length == 131072 and c.scaling_type == b"yarn"
    with pytest.raises(aos.AosError, match="RoPE scaling factor must be positive, got -1"):
        aos.plan_config_parse(scaled.replace('"factor": 4.0', '"factor": -1.0'))
    with pytest.raises(aos.AosError, match="original_max_position_embeddings must be non-zero"):
        aos.plan_config_parse(scaled.replace('"original_max_position_embeddings": 32768',
                                             '"original_max_position_embeddings": 0'))


def test_serde_field_rules():
    with pytest.raises(aos.AosError, match="Failed to parse model config: missing field `hidden_size`"):
        aos.plan_config_parse(QWEN.replace('"hidden_size": 3584,', ""))
    with pytest.raises(aos.AosError, match="expected u32"):  # u32 fields take unsigned integers only
        aos.plan_config_parse(QWEN.replace('"num_hidden_layers": 28', '"num_hidden_layers": 28.0'))
    with pytest.raises(aos.AosError, match="expected u32"):
        aos.plan_config_parse(QWEN.replace('"num_hidden_layers": 28', '"num_hidden_layers": -28'))
    with pytest.raises(aos.AosError, match="expected a string"):
        aos.plan_config_parse(QWEN.replace('"name": "Qwen2.5-7B"', '"name": 7'))
    with pytest.raises(aos.AosError, match="Failed to parse model config"):
        aos.plan_config_parse("{not json")
    # f32 takes integers; optional fields may be null; unknown fields are kept aside
    c = aos.plan_config_parse(QWEN.replace('"rope_theta": 1000000.0', '"rope_theta": 500000') [:-1]
                              + ', "rope_scaling_factor": null, "rope_scaling": null, "rms_norm_eps": 1e-6,'
                                ' "torch_dtype": "bfloat16"}')
    assert c.rope_theta == 500000.0 and c.has_rope_scaling_factor == 0 and c.has_rope_scaling == 0
    assert abs(c.rms_norm_eps - 1e-6) < 1e-12
    assert c.is_qwen2_5 == 1
    c = aos.plan_config_parse(QWEN.replace("Qwen2.5ForCausalLM", "LlamaForCausalLM"))
    assert c.is_qwen2_5 == 0


def _plan(H=256, nh=2, nkv=1, I=384, V=512, L=2, rng=None, embed_name="model.embed_tokens.weight"):
    rng = rng or np.random.default_rng(0)
    z = lambda *s: ("BF16", np.zeros(s, np.uint16))
    t = {embed_name: z(V, H), "lm_head.weight": z(V, H), "model.norm.weight": z(H)}
    shapes = [(nh * 128, H), (nkv * 128, H), (nkv * 128, H), (H, nh * 128), (I, H), (I, H), (H, I)]
    for l in range(L):
        t[f"model.layers.{l}.input_layernorm.weight"] = z(H)
        t[f"model.layers.{l}.post_attention_layernorm.weight"] = z(H)
        for m, name in enumerate(ALL):
            blk = "self_attn" if m < 4 else "mlp"
            t[f"model.layers.{l}.{blk}.{name}.weight"] = z(*shapes[m])
    return t


def test_dimensions_from_plan_shapes():
    d = aos.model_config_from_plan(st_bytes(_plan(H=256, nh=2, nkv=1, I=384, V=512, L=3)))
    # GqaConfig::default(): head_dim 128, rope_theta 10000
    assert (d["hidden"], d["vocab"], d["n_layers"], d["intermediate"]) == (256, 512, 3, 384)
    assert (d["n_heads"], d["n_kv_heads"], d["head_dim"]) == (2, 1, 128)
    assert d["rope_theta"] == 10000.0 and abs(d["rms_eps"] - 1e-5) < 1e-12
    # another embedding name of the reference's list
    d = aos.model_config_from_plan(st_bytes(_plan(embed_name="transformer.wte.weight")))
    assert (d["vocab"], d["hidden"]) == (512, 256)
    # with the plan's model config: its heads, theta and eps, checked against the tensors
    cfg = aos.plan_config_parse('{"name": "t", "architecture": "LlamaForCausalLM", "hidden_size": 256, '
                                '"intermediate_size": 384, "num_hidden_layers": 2, "num_attention_heads": 2, '
                                '"num_key_value_heads": 1, "max_position_embeddings": 4096, "rope_theta": 1000000.0, '
                                '"vocab_size": 512, "rms_norm_eps": 1e-6}')
    d = aos.model_config_from_plan(st_bytes(_plan()), cfg)
    assert d["rope_theta"] == 1e6 and abs(d["rms_eps"] - 1e-6) < 1e-12 and d["n_kv_heads"] == 1
    cfg.hidden_size = 512
    with pytest.raises(aos.AosError, match="does not match the plan's tensors"):
        aos.model_config_from_plan(st_bytes(_plan()), cfg)


def test_dimension_inference_errors():  # kernel-mtl/src/lib.rs:805-826
    t = _plan()
    t.pop("model.embed_tokens.weight")
    with pytest.raises(aos.AosError, match="Embedding tensor not found for dimension inference. Tried: "
                                           r'\["model.embed_tokens.weight", "transformer.wte.weight"'):
        aos.model_config_from_plan(st_bytes(t))
    t["wte.weight"] = ("BF16", np.zeros(512 * 256, np.uint16))
    with pytest.raises(aos.AosError, match=r"Expected 2D embedding tensor for dimension inference, got shape: \[131072\]"):
        aos.model_config_from_plan(st_bytes(t))
    with pytest.raises(aos.AosError, match="Failed to parse SafeTensors for dimensions"):
        aos.model_config_from_plan(b"\x05\x00")
    t = _plan()
    for k in [k for k in t if k.startswith("model.layers.")]:
        t.pop(k)
    with pytest.raises(aos.AosError, match="no transformer layers"):
        aos.model_config_from_plan(st_bytes(t))


@pytest.mark.gpu
def test_gpu_context_from_plan_matches_array_loads():
    from oracle import oracle as O
    rng = np.random.default_rng(8)
    m = O.HostModel.random(rng, 256, 2, 1, 128, 384, 512, 2, rope_theta=1e6)
    plan = {"model.embed_tokens.weight": ("BF16", m.embed), "lm_head.weight": ("BF16", m.lm_head),
            "model.norm.weight": ("BF16", m.final_norm)}
    for l in range(2):
        plan[f"model.layers.{l}.input_layernorm.weight"] = ("BF16", m.attn_norm[l])
        plan[f"model.layers.{l}.post_attention_layernorm.weight"] = ("BF16", m.mlp_norm[l])
        for mod in range(7):
            blk = "self_attn" if mod < 4 else "mlp"
            plan[f"model.layers.{l}.{blk}.{ALL[mod]}.weight"] = ("BF16", m.w[mod][l])
    cfg_json = ('{"name": "t", "architecture": "LlamaForCausalLM", "hidden_size": 256, "intermediate_size": 384, '
                '"num_hidden_layers": 2, "num_attention_heads": 2, "num_key_value_heads": 1, '
                '"max_position_embeddings": 4096, "rope_theta": 1000000.0, "vocab_size": 512}')
    T = 4
    toks = rng.integers(0, 512, size=T).astype(np.uint32)
    rings = np.zeros(T, O.RING_DTYPE)
    outs = []
    for from_plan in (False, True):
        if from_plan:
            gpu = aos.CudaKernels.from_plan(st_bytes(plan), cfg_json, max_batch=8, kv_num_blocks=64, max_seq_len=128,
                                            lora_rank_capacity=64, lora_max_adapters=2)
        else:
            gpu = aos.CudaKernels(256, 2, 1, 128, 384, 512, 2, max_batch=8, kv_num_blocks=64, max_seq_len=128,
                                  lora_rank_capacity=64, lora_max_adapters=2)
            gpu.load_host_model(m)
        sids = np.arange(T, dtype=np.uint64)
        for s in sids:
            gpu.kv_alloc(int(s), 64)
        logits, _ = gpu.run_step_batch(rings, toks, sids)
        outs.append(logits)
        gpu.close()
    assert outs[0].tobytes() == outs[1].tobytes()
