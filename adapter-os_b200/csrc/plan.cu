// plan.cu — the model plan behind FusedKernels::load(plan_bytes).
//
// Two host-side pieces of the reference, restated for the CUDA backend:
//
//  * the plan crate's model configuration (crates/adapteros-lora-plan/src/
//    config.rs): ModelConfig::from_json (:80-86) with serde's field rules,
//    validate (:127-167), validate_gqa (:101-124), dimensions (:171-193),
//    is_qwen2_5 (:196-198), effective_context_length (:201-208),
//    calculate_lora_size (:212-253) and validate_lora_targets (:256-277);
//
//  * the Metal backend's load(plan_bytes) (crates/adapteros-lora-kernel-mtl/
//    src/lib.rs:1476-1537): the plan is a safetensors container of base
//    weights; vocab and hidden size come from the embedding tensor's shape
//    (validate_embedding_dimensions, :790-839), the attention geometry from a
//    set GQA config or GqaConfig::default() (fused_qkv.rs:41-54: head_dim 128,
//    rope_theta 10000).  The CUDA backend also takes the layer count and the
//    MLP width from the tensor shapes (model.layers.<l>.*, mlp.gate_proj),
//    since aos_init sizes every buffer up front.
//
// Host code only: nothing here touches the device except aos_init_from_plan,
// which creates a context and loads the plan's weights into it.

#include <cmath>
#include <cstdio>
#include <cstring>
#include <map>
#include <string>
#include <vector>

#include "common.cuh"
#include "json.cuh"
#include "loader.cuh"

namespace {

using aos::JVal;

int plan_fail(const std::string& msg) {
    aos::set_global_error(msg);
    return AOS_ERR_INVALID;
}

// serde_json's typed reads of one struct field: missing, null or mistyped
// values are errors for required fields (Rust's `u32`, `f32`, `String`).
const char* kind_name(const JVal& v) {
    switch (v.k) {
        case JVal::NUL: return "null";
        case JVal::BOOL: return "boolean";
        case JVal::NUM: return v.n_uint ? "integer" : "floating point or signed integer";
        case JVal::STR: return "string";
        case JVal::ARR: return "sequence";
        default: return "map";
    }
}

bool read_u32(const JVal& obj, const char* key, uint32_t& out, std::string& err) {
    const JVal* v = obj.get(key);
    if (!v) { err = std::string("missing field `") + key + "`"; return false; }
    if (v->k == JVal::NUM && v->n_uint) {
        if (v->u > 0xFFFFFFFFull) {
            err = "invalid value: integer `" + std::to_string(v->u) + "`, expected u32 (field `" + key + "`)";
            return false;
        }
        out = (uint32_t)v->u;
        return true;
    }
    err = std::string("invalid type: ") + kind_name(*v) + ", expected u32 (field `" + key + "`)";
    return false;
}

bool read_f32(const JVal& obj, const char* key, float& out, std::string& err, bool* present = nullptr) {
    const JVal* v = obj.get(key);
    if (present) {  // Option<f32>: missing or null is None
        *present = v && v->k != JVal::NUL;
        if (!*present) return true;
    } else if (!v) {
        err = std::string("missing field `") + key + "`";
        return false;
    }
    if (v->k != JVal::NUM) {
        err = std::string("invalid type: ") + kind_name(*v) + ", expected f32 (field `" + key + "`)";
        return false;
    }
    out = (float)v->n;
    return true;
}

bool read_str(const JVal& obj, const char* key, char* out, size_t cap, std::string& err) {
    const JVal* v = obj.get(key);
    if (!v) { err = std::string("missing field `") + key + "`"; return false; }
    if (v->k != JVal::STR) {
        err = std::string("invalid type: ") + kind_name(*v) + ", expected a string (field `" + key + "`)";
        return false;
    }
    std::strncpy(out, v->s.c_str(), cap - 1);
    out[cap - 1] = 0;
    return true;
}

// u32::is_multiple_of: rhs == 0 holds only for lhs == 0.
bool is_multiple_of(uint32_t a, uint32_t b) { return b == 0 ? a == 0 : a % b == 0; }

// Rust's saturating `f32 as u32`.
uint32_t f32_as_u32(float x) {
    if (!(x > 0.0f)) return 0;  // NaN and negatives
    if (x >= 4294967296.0f) return 0xFFFFFFFFu;
    return (uint32_t)x;
}

const char* const kTargets[7] = {"q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj"};

int target_index(const char* t) {
    for (int i = 0; i < 7; ++i)
        if (t && std::strcmp(t, kTargets[i]) == 0) return i;
    return -1;
}

}  // namespace

extern "C" {

int aos_plan_config_parse(const char* json, uint64_t len, aos_plan_config* out) {
    if (!json || !out) return plan_fail("aos_plan_config_parse: null argument");
    std::memset(out, 0, sizeof(*out));
    JVal v;
    std::string err;
    if (!aos::parse_json(reinterpret_cast<const uint8_t*>(json), len, v, err, "model config"))
        return plan_fail("Failed to parse model config: " + err);
    if (v.k != JVal::OBJ)
        return plan_fail(std::string("Failed to parse model config: invalid type: ") + kind_name(v) +
                         ", expected struct ModelConfig");
    aos_plan_config& c = *out;
    bool ok = read_str(v, "name", c.name, sizeof(c.name), err) &&
              read_str(v, "architecture", c.architecture, sizeof(c.architecture), err) &&
              read_u32(v, "hidden_size", c.hidden_size, err) &&
              read_u32(v, "intermediate_size", c.intermediate_size, err) &&
              read_u32(v, "num_hidden_layers", c.num_hidden_layers, err) &&
              read_u32(v, "num_attention_heads", c.num_attention_heads, err) &&
              read_u32(v, "num_key_value_heads", c.num_key_value_heads, err) &&
              read_u32(v, "max_position_embeddings", c.max_position_embeddings, err) &&
              read_f32(v, "rope_theta", c.rope_theta, err) && read_u32(v, "vocab_size", c.vocab_size, err);
    bool has_factor = false;
    ok = ok && read_f32(v, "rope_scaling_factor", c.rope_scaling_factor, err, &has_factor);
    c.has_rope_scaling_factor = has_factor ? 1u : 0u;
    if (ok) {  // Option<RopeScaling>: every field of the struct is required when present
        const JVal* rs = v.get("rope_scaling");
        if (rs && rs->k != JVal::NUL) {
            if (rs->k != JVal::OBJ) {
                err = std::string("invalid type: ") + kind_name(*rs) + ", expected struct RopeScaling";
                ok = false;
            } else {
                ok = read_f32(*rs, "factor", c.scaling_factor, err) &&
                     read_u32(*rs, "original_max_position_embeddings", c.scaling_original_max_position_embeddings,
                              err) &&
                     read_str(*rs, "scaling_type", c.scaling_type, sizeof(c.scaling_type), err);
                c.has_rope_scaling = ok ? 1u : 0u;
            }
        }
    }
    if (!ok) {
        std::memset(out, 0, sizeof(*out));
        return plan_fail("Failed to parse model config: " + err);
    }
    // an extra field the runtime uses when the plan carries it
    const JVal* eps = v.get("rms_norm_eps");
    if (eps && eps->k == JVal::NUM && eps->n > 0) c.rms_norm_eps = (float)eps->n;
    // dimensions(): head_dim = hidden / heads (u32), kv_width = kv_heads *
    // head_dim, the parameter estimate in Rust's u32 arithmetic per layer
    c.head_dim = c.num_attention_heads ? c.hidden_size / c.num_attention_heads : 0;
    c.kv_width = c.num_key_value_heads * c.head_dim;
    const uint32_t per_layer = (c.hidden_size * c.hidden_size) * 4u + (c.hidden_size * c.intermediate_size) * 3u;
    c.total_params = (uint64_t)per_layer * c.num_hidden_layers + ((uint64_t)c.vocab_size * c.hidden_size) * 2u;
    c.effective_context_length =
        c.has_rope_scaling ? f32_as_u32((float)c.scaling_original_max_position_embeddings * c.scaling_factor)
                           : c.max_position_embeddings;
    c.is_qwen2_5 = (std::strcmp(c.architecture, "Qwen2.5ForCausalLM") == 0 ||
                    std::strstr(c.architecture, "Qwen2.5") != nullptr)
                       ? 1u
                       : 0u;
    return AOS_OK;
}

int aos_plan_config_validate_gqa(const aos_plan_config* c) {
    if (!c) return plan_fail("aos_plan_config_validate_gqa: null argument");
    if (!is_multiple_of(c->hidden_size, c->num_attention_heads))
        return plan_fail("hidden_size (" + std::to_string(c->hidden_size) + ") must be divisible by num_attention_heads (" +
                         std::to_string(c->num_attention_heads) + ")");
    if (!is_multiple_of(c->num_attention_heads, c->num_key_value_heads))
        return plan_fail("num_attention_heads (" + std::to_string(c->num_attention_heads) +
                         ") must be divisible by num_key_value_heads (" + std::to_string(c->num_key_value_heads) + ")");
    return AOS_OK;
}

int aos_plan_config_validate(const aos_plan_config* c) {
    int rc = aos_plan_config_validate_gqa(c);
    if (rc) return rc;
    if (c->has_rope_scaling) {
        if (!(c->scaling_factor > 0.0f)) {
            char buf[64];
            std::snprintf(buf, sizeof(buf), "%g", (double)c->scaling_factor);
            return plan_fail(std::string("RoPE scaling factor must be positive, got ") + buf);
        }
        if (c->scaling_original_max_position_embeddings == 0)
            return plan_fail("RoPE scaling original_max_position_embeddings must be non-zero");
    }
    if (c->vocab_size == 0) return plan_fail("vocab_size must be non-zero");
    return AOS_OK;
}

int aos_plan_validate_lora_targets(const char* const* targets, uint32_t n) {
    if (n && !targets) return plan_fail("aos_plan_validate_lora_targets: null argument");
    for (uint32_t i = 0; i < n; ++i)
        if (target_index(targets[i]) < 0)
            return plan_fail(std::string("Invalid LoRA target: ") + (targets[i] ? targets[i] : "") +
                             ". Valid targets: [\"q_proj\", \"k_proj\", \"v_proj\", \"o_proj\", \"gate_proj\", "
                             "\"up_proj\", \"down_proj\"]");
    return AOS_OK;
}

int aos_plan_lora_size(const aos_plan_config* c, uint32_t rank, const char* const* targets, uint32_t n,
                       uint64_t* bytes) {
    if (!c || !bytes || (n && !targets)) return plan_fail("aos_plan_lora_size: null argument");
    uint64_t total = 0;
    for (uint32_t i = 0; i < n; ++i) {
        const int t = target_index(targets[i]);
        const uint64_t H = c->hidden_size, I = c->intermediate_size;
        switch (t) {
            case 0: case 3: total += (uint64_t)rank * (H + H); break;  // q / o
            case 1: case 2: {                                            // k / v: GQA width
                if (c->num_attention_heads == 0) return plan_fail("num_attention_heads is zero");
                const uint32_t kv_width = c->num_key_value_heads * (c->hidden_size / c->num_attention_heads);
                total += (uint64_t)rank * (H + kv_width);
                break;
            }
            case 4: case 5: total += (uint64_t)rank * (H + I); break;  // gate / up
            case 6: total += (uint64_t)rank * (I + H); break;          // down
            default:
                return plan_fail(std::string("Unknown LoRA target: ") + (targets[i] ? targets[i] : "") +
                                 ". Valid targets: q_proj, k_proj, v_proj, o_proj, gate_proj, up_proj, down_proj");
        }
    }
    *bytes = total * c->num_hidden_layers * 2u;  // fp16 bytes
    return AOS_OK;
}

int aos_model_config_from_plan(const void* plan, uint64_t len, const aos_plan_config* pc, aos_model_config* cfg) {
    if (!plan || !cfg) return plan_fail("aos_model_config_from_plan: null argument");
    std::vector<aos::StTensor> ts;
    const uint8_t* base = nullptr;
    std::string err;
    if (aos::parse_safetensors(static_cast<const uint8_t*>(plan), len, ts, &base, err))
        return plan_fail("Failed to parse SafeTensors for dimensions: " + err);
    std::map<std::string, const aos::StTensor*> by;
    for (const auto& t : ts) by[t.name] = &t;
    // validate_embedding_dimensions: the first embedding name present
    static const char* kEmbed[] = {"model.embed_tokens.weight", "transformer.wte.weight",
                                   "embeddings.word_embeddings.weight", "embed_tokens.weight", "wte.weight"};
    const aos::StTensor* emb = nullptr;
    for (const char* n : kEmbed)
        if (!emb && by.count(n)) emb = by[n];
    auto list = [](const std::vector<std::string>& v) {
        std::string s = "[";
        for (size_t i = 0; i < v.size(); ++i) s += (i ? ", \"" : "\"") + v[i] + "\"";
        return s + "]";
    };
    if (!emb) {
        std::vector<std::string> names;
        for (const auto& t : ts) names.push_back(t.name);
        return plan_fail("Embedding tensor not found for dimension inference. Tried: " +
                         list({kEmbed, kEmbed + 5}) + ". Available tensors: " + list(names));
    }
    if (emb->shape.size() != 2) {
        std::string sh = "[";
        for (size_t i = 0; i < emb->shape.size(); ++i) sh += (i ? ", " : "") + std::to_string(emb->shape[i]);
        return plan_fail("Expected 2D embedding tensor for dimension inference, got shape: " + sh + "]");
    }
    const int64_t V = emb->shape[0], H = emb->shape[1];
    // layers: model.layers.<l>.self_attn.q_proj.weight for l = 0, 1, ...
    auto layer_tensor = [&](int l, const char* sub) -> const aos::StTensor* {
        auto it = by.find("model.layers." + std::to_string(l) + "." + sub);
        return it == by.end() ? nullptr : it->second;
    };
    int L = 0;
    while (layer_tensor(L, "self_attn.q_proj.weight")) ++L;
    if (L == 0) return plan_fail("no transformer layers in the plan (model.layers.0.self_attn.q_proj.weight)");
    const aos::StTensor *q = layer_tensor(0, "self_attn.q_proj.weight"), *k = layer_tensor(0, "self_attn.k_proj.weight"),
                        *gate = layer_tensor(0, "mlp.gate_proj.weight");
    auto is2 = [&](const aos::StTensor* t) { return t && t->shape.size() == 2 && t->shape[1] == H; };
    if (!is2(q) || !is2(k) || !is2(gate))
        return plan_fail("layer 0: q_proj, k_proj and mlp.gate_proj must be [rows, hidden] matrices");
    const int64_t I = gate->shape[0], q_rows = q->shape[0], k_rows = k->shape[0];
    uint32_t heads, kv_heads, head_dim;
    float theta, eps = cfg->rms_eps > 0 ? cfg->rms_eps : 1e-5f;
    if (pc) {  // the plan's model config, checked against the tensors
        if ((int64_t)pc->hidden_size != H || (int64_t)pc->vocab_size != V || (int64_t)pc->num_hidden_layers != L ||
            (int64_t)pc->intermediate_size != I)
            return plan_fail("model config (hidden " + std::to_string(pc->hidden_size) + ", vocab " +
                             std::to_string(pc->vocab_size) + ", layers " + std::to_string(pc->num_hidden_layers) +
                             ", intermediate " + std::to_string(pc->intermediate_size) +
                             ") does not match the plan's tensors (hidden " + std::to_string(H) + ", vocab " +
                             std::to_string(V) + ", layers " + std::to_string(L) + ", intermediate " +
                             std::to_string(I) + ")");
        heads = pc->num_attention_heads;
        kv_heads = pc->num_key_value_heads;
        head_dim = pc->head_dim;
        theta = pc->rope_theta;
        if (pc->rms_norm_eps > 0) eps = pc->rms_norm_eps;
    } else {  // GqaConfig::default(): head_dim 128, rope_theta 10000
        head_dim = 128;
        if (q_rows % head_dim || k_rows % head_dim)
            return plan_fail("q_proj / k_proj rows are not multiples of the default head_dim 128");
        heads = (uint32_t)(q_rows / head_dim);
        kv_heads = (uint32_t)(k_rows / head_dim);
        theta = 10000.0f;
    }
    if (!heads || !kv_heads || (int64_t)heads * head_dim != q_rows || (int64_t)kv_heads * head_dim != k_rows)
        return plan_fail("attention geometry (" + std::to_string(heads) + " heads / " + std::to_string(kv_heads) +
                         " KV heads of " + std::to_string(head_dim) + ") does not match q_proj / k_proj rows (" +
                         std::to_string(q_rows) + " / " + std::to_string(k_rows) + ")");
    cfg->hidden = (uint32_t)H;
    cfg->vocab = (uint32_t)V;
    cfg->n_layers = (uint32_t)L;
    cfg->intermediate = (uint32_t)I;
    cfg->n_heads = heads;
    cfg->n_kv_heads = kv_heads;
    cfg->head_dim = head_dim;
    cfg->rope_theta = theta;
    cfg->rms_eps = eps;
    return AOS_OK;
}

aos_ctx* aos_init_from_plan(const void* plan, uint64_t len, const aos_plan_config* pc, const aos_model_config* runtime) {
    if (!plan || !runtime) {
        plan_fail("aos_init_from_plan: null argument");
        return nullptr;
    }
    aos_model_config cfg = *runtime;
    if (aos_model_config_from_plan(plan, len, pc, &cfg)) return nullptr;
    aos_ctx* c = aos_init(&cfg);
    if (!c) return nullptr;
    if (aos_load_model_safetensors(c, plan, len)) {
        aos::set_global_error(std::string("aos_init_from_plan: ") + aos_last_error(c));
        aos_destroy(c);
        return nullptr;
    }
    return c;
}

}  // extern "C"
