// safetensors.cu — adapter and base-model loading from safetensors bytes.
//
// The reference loads adapters (FusedKernels::load_adapter_with_metadata,
// crates/adapteros-lora-kernel-mtl/src/lib.rs:1893-2046) and base weights
// (FusedKernels::load, kernel-mtl/src/lib.rs:660-1135) from safetensors.
// This file restates that host path in C++ for the CUDA backend.
//
// Container: 8-byte little-endian header length N, N bytes of JSON
// {name: {"dtype", "shape", "data_offsets": [begin, end]}, "__metadata__": {..}},
// then the tensor bytes, with offsets relative to the end of the header.
//
// Adapter rules (kernel-mtl/src/lib.rs:186-251, 1893-1975):
//   * tensor names are sorted; for every target module the first name that
//     contains the module name and "lora_A" (resp. "lora_B") is used;
//   * target modules come from the metadata (trimmed, empty names dropped,
//     duplicates dropped); with none, or when the metadata's modules match no
//     tensor, the default set q_proj, k_proj, v_proj, down_proj, up_proj;
//   * rank = metadata rank (> 0), else lora_A's first dimension, else 16;
//     alpha = metadata alpha (finite, > 0), else 2 * rank;
//   * no LoRA tensor at all is an error.
// The reference's Metal path holds one layer.  Here a name containing
// ".layers.<L>." belongs to layer L, and a name without a layer index belongs
// to layer 0; the matching above runs per layer.  F32, F16 and BF16 tensors
// are accepted and stored as bf16 (round to nearest even).

#include <algorithm>
#include <cmath>
#include <cstring>
#include <map>
#include <string>
#include <vector>

#include "common.cuh"
#include "json.cuh"
#include "loader.cuh"

namespace aos {
namespace {

int st_parse(const uint8_t* d, uint64_t len, std::vector<StTensor>& out, const uint8_t** base, std::string& err) {
    if (!d || len < 8) { err = "safetensors: shorter than its 8-byte header length"; return AOS_ERR_INVALID; }
    uint64_t n = 0;
    for (int i = 7; i >= 0; --i) n = (n << 8) | d[i];
    if (n > len - 8) { err = "safetensors: header length exceeds the buffer"; return AOS_ERR_INVALID; }
    *base = d + 8 + n;
    const uint64_t data_len = len - 8 - n;
    out.clear();
    JVal h;
    if (!parse_json(d + 8, n, h, err, "safetensors header")) return AOS_ERR_INVALID;
    if (h.k != JVal::OBJ) { err = "safetensors header: not an object"; return AOS_ERR_INVALID; }
    for (const auto& kv : h.o) {
        if (kv.first == "__metadata__") continue;
        const JVal& t = kv.second;
        const JVal *dt = t.get("dtype"), *sh = t.get("shape"), *of = t.get("data_offsets");
        if (!dt || dt->k != JVal::STR || !sh || sh->k != JVal::ARR || !of || of->k != JVal::ARR) {
            err = "safetensors: tensor " + kv.first + " lacks dtype, shape or data_offsets";
            return AOS_ERR_INVALID;
        }
        StTensor x;
        x.name = kv.first;
        x.dtype = dt->s;
        for (const JVal& e : sh->a) {
            if (e.k != JVal::NUM || !e.n_uint || e.u > (uint64_t)INT64_MAX) {
                err = "safetensors: tensor " + kv.first + ": shape must list non-negative integers";
                return AOS_ERR_INVALID;
            }
            x.shape.push_back((int64_t)e.u);
        }
        if (of->a.size() != 2 || of->a[0].k != JVal::NUM || !of->a[0].n_uint || of->a[1].k != JVal::NUM ||
            !of->a[1].n_uint || of->a[1].u < of->a[0].u) {
            err = "safetensors: tensor " + kv.first + " lacks dtype, shape or data_offsets";
            return AOS_ERR_INVALID;
        }
        x.b = of->a[0].u;
        x.e = of->a[1].u;
        if (x.e > data_len) { err = "safetensors: tensor " + kv.first + " runs past the buffer"; return AOS_ERR_INVALID; }
        out.push_back(std::move(x));
    }
    return AOS_OK;
}

uint16_t f32_bf16(float f) {  // round to nearest even, NaN kept quiet
    uint32_t u;
    std::memcpy(&u, &f, 4);
    if ((u & 0x7F800000u) == 0x7F800000u && (u & 0x007FFFFFu)) return (uint16_t)((u >> 16) | 0x40);
    u += 0x7FFFu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}
float f16_f32(uint16_t h) {
    const uint32_t s = (uint32_t)(h & 0x8000u) << 16, e = (h >> 10) & 0x1F, m = h & 0x3FF;
    uint32_t u;
    if (e == 0) {
        if (m == 0) u = s;
        else {  // subnormal: normalise
            int ee = -1;
            uint32_t mm = m;
            do { ++ee; mm <<= 1; } while (!(mm & 0x400));
            u = s | ((uint32_t)(127 - 15 - ee) << 23) | ((mm & 0x3FF) << 13);
        }
    } else if (e == 31) {
        u = s | 0x7F800000u | (m << 13);
    } else {
        u = s | ((e + 112) << 23) | (m << 13);
    }
    float f;
    std::memcpy(&f, &u, 4);
    return f;
}

int64_t numel(const StTensor& t) {
    int64_t n = 1;
    for (int64_t x : t.shape) n *= x;
    return n;
}

int st_to_bf16(const StTensor& t, const uint8_t* base, std::vector<uint16_t>& out, std::string& err) {
    const int64_t n = numel(t);
    const uint8_t* p = base + t.b;
    const uint64_t bytes = t.e - t.b;
    out.resize((size_t)n);
    if (t.dtype == "BF16" && bytes == (uint64_t)n * 2) {
        std::memcpy(out.data(), p, bytes);
    } else if (t.dtype == "F16" && bytes == (uint64_t)n * 2) {
        for (int64_t i = 0; i < n; ++i) out[i] = f32_bf16(f16_f32((uint16_t)(p[2 * i] | (p[2 * i + 1] << 8))));
    } else if (t.dtype == "F32" && bytes == (uint64_t)n * 4) {
        for (int64_t i = 0; i < n; ++i) {
            float f;
            std::memcpy(&f, p + 4 * i, 4);
            out[i] = f32_bf16(f);
        }
    } else {
        err = "tensor " + t.name + ": dtype " + t.dtype + " (F32, F16 or BF16 expected) or size mismatch";
        return AOS_ERR_INVALID;
    }
    return AOS_OK;
}

// ---------------------------------------------------------------- adapters
const char* const kModuleNames[AOS_NUM_MODULES] = {"q_proj", "k_proj", "v_proj", "o_proj",
                                                   "gate_proj", "up_proj", "down_proj"};
const char* const kDefaultTargets[5] = {"q_proj", "k_proj", "v_proj", "down_proj", "up_proj"};

int layer_of(const std::string& name) {  // ".layers.<L>." (or a leading "layers.<L>.") -> L, else -1
    size_t i;
    const size_t at = name.find(".layers.");
    if (at != std::string::npos) i = at + 8;
    else if (name.compare(0, 7, "layers.") == 0) i = 7;
    else return -1;
    int L = 0, digits = 0;
    while (i < name.size() && name[i] >= '0' && name[i] <= '9') {
        L = L * 10 + (name[i++] - '0');
        if (++digits > 6) return -1;
    }
    return digits && i < name.size() && name[i] == '.' ? L : -1;
}

struct AdapterPlan {
    int rank = 0;
    float alpha = 0.f;
    // per (layer, module): indices into the tensor list (-1: none)
    std::map<std::pair<int, int>, std::pair<int, int>> ab;
};

std::vector<std::string> sanitized_targets(const aos_adapter_meta* m) {
    std::vector<std::string> out;
    if (!m || !m->target_modules) return out;
    for (uint32_t i = 0; i < m->n_targets; ++i) {
        if (!m->target_modules[i]) continue;
        std::string s = m->target_modules[i];
        const size_t a = s.find_first_not_of(" \t\r\n"), b = s.find_last_not_of(" \t\r\n");
        if (a == std::string::npos) continue;
        s = s.substr(a, b - a + 1);
        if (std::find(out.begin(), out.end(), s) == out.end()) out.push_back(s);
    }
    return out;
}

// Match per layer; returns the number of A/B tensors found and the rank
// inferred from the first lora_A found in target order.
int match_targets(const std::vector<StTensor>& ts, const std::vector<int>& order, const std::vector<std::string>& targets,
                  int n_layers, AdapterPlan& plan, int& inferred) {
    plan.ab.clear();
    inferred = 0;
    int found = 0;
    for (const std::string& mod : targets) {
        int mi = -1;
        for (int m = 0; m < AOS_NUM_MODULES; ++m)
            if (mod == kModuleNames[m]) mi = m;
        for (int L = 0; L < n_layers; ++L) {
            int a = -1, b = -1;
            for (int idx : order) {
                const std::string& nm = ts[idx].name;
                const int l = layer_of(nm);
                if ((l < 0 ? 0 : l) != L || nm.find(mod) == std::string::npos) continue;
                if (a < 0 && nm.find("lora_A") != std::string::npos) a = idx;
                if (b < 0 && nm.find("lora_B") != std::string::npos) b = idx;
            }
            if (a >= 0 && !inferred && ts[a].shape.size() >= 2) inferred = (int)ts[a].shape[0];
            found += (a >= 0) + (b >= 0);
            if (mi >= 0 && (a >= 0 || b >= 0)) plan.ab[{L, mi}] = {a, b};
        }
    }
    return found;
}

int plan_adapter(const std::vector<StTensor>& ts, const aos_adapter_meta* meta, int n_layers, AdapterPlan& plan,
                 std::string& err) {
    std::vector<int> order(ts.size());
    for (size_t i = 0; i < ts.size(); ++i) order[i] = (int)i;
    std::sort(order.begin(), order.end(), [&](int x, int y) { return ts[x].name < ts[y].name; });
    std::vector<std::string> targets = sanitized_targets(meta);
    const bool has_meta_targets = !targets.empty();
    const std::vector<std::string> defaults(kDefaultTargets, kDefaultTargets + 5);
    if (!has_meta_targets) targets = defaults;
    int inferred = 0;
    int found = match_targets(ts, order, targets, n_layers, plan, inferred);
    if (found == 0 && has_meta_targets && targets != defaults)  // metadata matched nothing: default set
        found = match_targets(ts, order, defaults, n_layers, plan, inferred);
    if (found == 0) {
        err = "no LoRA tensors found in the adapter";
        return AOS_ERR_INVALID;
    }
    plan.rank = (meta && meta->rank > 0) ? (int)meta->rank : (inferred > 0 ? inferred : 16);
    plan.alpha = (meta && std::isfinite(meta->alpha) && meta->alpha > 0.f) ? meta->alpha : (float)(plan.rank * 2);
    return AOS_OK;
}

}  // namespace

int parse_safetensors(const uint8_t* d, uint64_t len, std::vector<StTensor>& out, const uint8_t** base,
                      std::string& err) {
    return st_parse(d, len, out, base, err);
}
int tensor_to_bf16(const StTensor& t, const uint8_t* base, std::vector<uint16_t>& out, std::string& err) {
    return st_to_bf16(t, base, out, err);
}

}  // namespace aos

// context internals used here (runtime.cu)
extern "C" {
int aos_adapter_new(aos_ctx* ctx, uint16_t id, uint32_t rank, float alpha);
int aos_adapter_set_module(aos_ctx* ctx, uint16_t id, uint32_t layer, aos_module module, const uint16_t* A,
                           const uint16_t* B, int src_on_device);
int aos_adapter_unload(aos_ctx* ctx, uint16_t id);
int aos_load_weight(aos_ctx* ctx, aos_weight_kind kind, uint32_t layer, aos_module module, const uint16_t* data,
                    uint64_t n, int src_on_device);
}
using namespace aos;

extern "C" {

int aos_adapter_probe_safetensors(const void* data, uint64_t len, const aos_adapter_meta* meta, uint32_t n_layers,
                                  uint32_t* rank_out, float* alpha_out, uint32_t* found) {
    std::vector<StTensor> ts;
    const uint8_t* base = nullptr;
    std::string err;
    int rc = st_parse(static_cast<const uint8_t*>(data), len, ts, &base, err);
    if (!rc) {
        AdapterPlan plan;
        rc = plan_adapter(ts, meta, (int)std::max(1u, n_layers), plan, err);
        if (!rc) {
            if (rank_out) *rank_out = (uint32_t)plan.rank;
            if (alpha_out) *alpha_out = plan.alpha;
            if (found) {
                std::memset(found, 0, sizeof(uint32_t) * n_layers * AOS_NUM_MODULES);
                for (const auto& kv : plan.ab)
                    if (kv.first.first < (int)n_layers)
                        found[kv.first.first * AOS_NUM_MODULES + kv.first.second] =
                            (kv.second.first >= 0 ? 1u : 0u) | (kv.second.second >= 0 ? 2u : 0u);
            }
            return AOS_OK;
        }
    }
    set_global_error("aos_adapter_probe_safetensors: " + err);
    return rc;
}

int aos_adapter_load_safetensors(aos_ctx* c, uint16_t id, const void* data, uint64_t len, const aos_adapter_meta* meta) {
    if (!c) return AOS_ERR_INVALID;
    uint32_t L = 0, in[AOS_NUM_MODULES], out[AOS_NUM_MODULES], H = 0, V = 0;
    ctx_model_dims(c, &L, in, out, &H, &V);
    std::vector<StTensor> ts;
    const uint8_t* base = nullptr;
    std::string err;
    int rc = st_parse(static_cast<const uint8_t*>(data), len, ts, &base, err);
    if (rc) return ctx_fail(c, rc, err);
    AdapterPlan plan;
    if ((rc = plan_adapter(ts, meta, (int)L, plan, err))) return ctx_fail(c, rc, err);
    // validate every shape before touching the arena
    for (const auto& kv : plan.ab) {
        const int m = kv.first.second;
        const int a = kv.second.first, b = kv.second.second;
        if (a >= 0 && (ts[a].shape.size() != 2 || ts[a].shape[0] != plan.rank || ts[a].shape[1] != (int64_t)in[m]))
            return ctx_fail(c, AOS_ERR_INVALID, "tensor " + ts[a].name + ": lora_A must be [rank, in] of its module");
        if (b >= 0 && (ts[b].shape.size() != 2 || ts[b].shape[0] != (int64_t)out[m] || ts[b].shape[1] != plan.rank))
            return ctx_fail(c, AOS_ERR_INVALID, "tensor " + ts[b].name + ": lora_B must be [out, rank] of its module");
    }
    if ((rc = aos_adapter_new(c, id, (uint32_t)plan.rank, plan.alpha))) return rc;
    std::vector<uint16_t> A, B;
    for (const auto& kv : plan.ab) {
        const int L_ = kv.first.first, m = kv.first.second;
        const int a = kv.second.first, b = kv.second.second;
        A.assign((size_t)plan.rank * in[m], 0);
        B.assign((size_t)out[m] * plan.rank, 0);
        if (a >= 0 && (rc = st_to_bf16(ts[a], base, A, err))) break;
        if (b >= 0 && (rc = st_to_bf16(ts[b], base, B, err))) break;
        if ((rc = aos_adapter_set_module(c, id, (uint32_t)L_, (aos_module)m, A.data(), B.data(), 0))) {
            aos_adapter_unload(c, id);
            return rc;
        }
    }
    if (rc) {
        aos_adapter_unload(c, id);
        return ctx_fail(c, rc, err);
    }
    return AOS_OK;
}

// Base weights under the Hugging Face LLaMA names (the names the reference's
// loader tries first, kernel-mtl/src/lib.rs:660-1000): model.embed_tokens,
// lm_head (tied to the embedding when absent), model.norm, and per layer
// input_layernorm, post_attention_layernorm, self_attn.{q,k,v,o}_proj,
// mlp.{gate,up,down}_proj.  Every tensor of the model must be present.
int aos_load_model_safetensors(aos_ctx* c, const void* data, uint64_t len) {
    if (!c) return AOS_ERR_INVALID;
    uint32_t L = 0, in[AOS_NUM_MODULES], out[AOS_NUM_MODULES], H = 0, V = 0;
    ctx_model_dims(c, &L, in, out, &H, &V);
    std::vector<StTensor> ts;
    const uint8_t* base = nullptr;
    std::string err;
    int rc = st_parse(static_cast<const uint8_t*>(data), len, ts, &base, err);
    if (rc) return ctx_fail(c, rc, err);
    std::map<std::string, int> by;
    for (size_t i = 0; i < ts.size(); ++i) by[ts[i].name] = (int)i;
    std::vector<uint16_t> buf;
    auto load = [&](const std::string& name, const std::string& alt, aos_weight_kind kind, uint32_t layer, int module,
                    int64_t rows, int64_t cols) -> int {
        auto it = by.find(name);
        if (it == by.end() && !alt.empty()) it = by.find(alt);
        if (it == by.end()) return ctx_fail(c, AOS_ERR_NOT_FOUND, "tensor " + name + " not found");
        const StTensor& t = ts[it->second];
        const bool ok = cols ? (t.shape.size() == 2 && t.shape[0] == rows && t.shape[1] == cols)
                             : (t.shape.size() == 1 && t.shape[0] == rows);
        if (!ok) return ctx_fail(c, AOS_ERR_INVALID, "tensor " + t.name + ": shape does not match the model");
        int r = st_to_bf16(t, base, buf, err);
        if (r) return ctx_fail(c, r, err);
        return aos_load_weight(c, kind, layer, (aos_module)module, buf.data(), buf.size(), 0);
    };
    if ((rc = load("model.embed_tokens.weight", "", AOS_W_EMBED, 0, 0, V, H))) return rc;
    if ((rc = load("lm_head.weight", "model.embed_tokens.weight", AOS_W_LM_HEAD, 0, 0, V, H))) return rc;
    if ((rc = load("model.norm.weight", "", AOS_W_FINAL_NORM, 0, 0, H, 0))) return rc;
    const char* sub[AOS_NUM_MODULES] = {"self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj", "self_attn.o_proj",
                                        "mlp.gate_proj", "mlp.up_proj", "mlp.down_proj"};
    for (uint32_t l = 0; l < L; ++l) {
        const std::string pre = "model.layers." + std::to_string(l) + ".";
        if ((rc = load(pre + "input_layernorm.weight", "", AOS_W_ATTN_NORM, l, 0, H, 0))) return rc;
        if ((rc = load(pre + "post_attention_layernorm.weight", "", AOS_W_MLP_NORM, l, 0, H, 0))) return rc;
        for (int m = 0; m < AOS_NUM_MODULES; ++m)
            if ((rc = load(pre + sub[m] + ".weight", "", AOS_W_PROJ, l, m, out[m], in[m]))) return rc;
    }
    return AOS_OK;
}

}  // extern "C"
