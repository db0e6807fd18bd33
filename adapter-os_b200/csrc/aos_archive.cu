// aos_archive.cu — `.aos` adapter archives into the adapter arena.
//
// Layout (crates/adapteros-aos/src/writer.rs:118-135, 313-358): a 64-byte
// header {magic "AOS\0" (or the older "AOS2"), u32 flags (bit 0: index
// present), u64 index offset (= 64), u64 index size, u64 manifest offset,
// u64 manifest size, 24 zero bytes}, then 80-byte index entries {u32 segment
// id, u16 backend tag (0 canonical, 1 mlx, 2 metal, 3 coreml), 2 zero bytes,
// u64 offset, u64 length, 16-byte scope hash, 32-byte BLAKE3 of the payload,
// 8 zero bytes}, the payloads, and the JSON manifest.  All integers are
// little-endian.
//
// Validation follows AosWriter::parse_header_bytes and parse_segments
// (writer.rs:407-558) rule for rule and message for message.  The payload
// hashes are computed on the GPU (blake3.cu) over a device copy of the
// archive, together with the manifest's scope path.
//
// Loading follows LifecycleLoader::load_from_aos_static
// (crates/adapteros-lora-lifecycle/src/loader.rs:931-1070):
//   * a canonical segment must exist;
//   * metadata.scope_path is required; scope hash = first 16 bytes of its
//     BLAKE3 (writer.rs:31-37);
//   * segment choice by select_segment_for_backend (loader.rs:177-218);
//   * per_layer_hashes (BLAKE3 of each tensor's bytes, keyed by
//     canonical_layer_id, loader.rs:107-158, 1247-1292) and weights_hash
//     (BLAKE3 of the payload) are checked when the manifest has them.
// The payload's tensors then go through the MLX backend's adapter rules
// (crates/adapteros-lora-mlx-ffi/src/backend.rs:1017-1200), the canonical
// backend's: modules discovered from "lora_a.<m>" / "<m>.lora_A" names,
// config defaults rank 4, alpha 16, targets q/k/v/o_proj (mlx-ffi
// src/lora.rs:29-44), overridden by the manifest's rank / lora_rank, alpha /
// lora_alpha and target_modules (top level first, then its "metadata"
// object); a module's weights apply at every layer.  The manifest is the
// metadata object passed.  Kernel version, base-model identity and CoreML
// placement checks of the lifecycle loader are policy, not arena work, and
// are not made here.

#include <algorithm>
#include <cctype>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <string>
#include <vector>

#include "common.cuh"
#include "json.cuh"
#include "loader.cuh"

extern "C" {
int aos_adapter_set_module(aos_ctx* ctx, uint16_t id, uint32_t layer, aos_module module, const uint16_t* A,
                           const uint16_t* B, int src_on_device);
int aos_adapter_unload(aos_ctx* ctx, uint16_t id);
}

namespace aos {
namespace {

// ---------------------------------------------------------------- layout
constexpr uint64_t kHeader = 64, kEntry = 80;

uint64_t rd64(const uint8_t* p) {
    uint64_t v = 0;
    for (int i = 7; i >= 0; --i) v = v << 8 | p[i];
    return v;
}
uint32_t rd32(const uint8_t* p) { return (uint32_t)p[0] | (uint32_t)p[1] << 8 | (uint32_t)p[2] << 16 | (uint32_t)p[3] << 24; }

// parse_header_bytes + parse_segments without the hash check
int parse_layout(const uint8_t* b, uint64_t len, aos_archive_info& info, std::vector<aos_archive_segment>& segs,
                 std::string& err) {
    const std::string bad = "Corrupted / needs retrain: ";
    if (!b || len < kHeader) return err = bad + "file too small for AOS header", AOS_ERR_INVALID;
    if (memcmp(b, "AOS\0", 4) != 0 && memcmp(b, "AOS2", 4) != 0) return err = bad + "invalid AOS magic", AOS_ERR_INVALID;
    const uint32_t flags = rd32(b + 4);
    const uint64_t io = rd64(b + 8), isz = rd64(b + 16), mo = rd64(b + 24), ms = rd64(b + 32);
    if (io != kHeader) return err = bad + "invalid header layout (index offset)", AOS_ERR_INVALID;
    for (uint64_t i = 40; i < kHeader; ++i)
        if (b[i]) return err = bad + "reserved header bytes non-zero", AOS_ERR_INVALID;
    if (!(flags & 1)) return err = bad + "missing segment index", AOS_ERR_INVALID;
    if (isz > UINT64_MAX - io) return err = bad + "index overflow", AOS_ERR_INVALID;
    const uint64_t iend = io + isz;
    if (iend > len) return err = bad + "index beyond file", AOS_ERR_INVALID;
    if (isz % kEntry) return err = bad + "index size not 80-byte aligned", AOS_ERR_INVALID;
    if (ms > UINT64_MAX - mo) return err = bad + "manifest overflow", AOS_ERR_INVALID;
    if (mo + ms > len) return err = bad + "manifest beyond file", AOS_ERR_INVALID;
    if (mo < iend) return err = bad + "manifest overlaps index/segments", AOS_ERR_INVALID;
    segs.clear();
    for (uint64_t e = 0; e < isz / kEntry; ++e) {
        const uint8_t* ent = b + io + kEntry * e;
        aos_archive_segment sg;
        memset(&sg, 0, sizeof sg);
        sg.segment_id = rd32(ent);
        sg.backend_tag = (uint16_t)(ent[4] | ent[5] << 8);
        if (sg.backend_tag > 3) return err = "Unknown backend tag: " + std::to_string(sg.backend_tag), AOS_ERR_INVALID;
        sg.offset = rd64(ent + 8);
        sg.len = rd64(ent + 16);
        memcpy(sg.scope_hash, ent + 24, 16);
        memcpy(sg.weights_hash, ent + 40, 32);
        if (sg.len > UINT64_MAX - sg.offset) return err = bad + "segment overflow", AOS_ERR_INVALID;
        if (sg.offset < iend) return err = bad + "segment overlaps index", AOS_ERR_INVALID;
        if (sg.offset + sg.len > mo) return err = bad + "segment overlaps manifest", AOS_ERR_INVALID;
        if (sg.offset + sg.len > len) return err = bad + "segment beyond file", AOS_ERR_INVALID;
        segs.push_back(sg);
    }
    info.flags = flags;
    info.n_segments = (uint32_t)segs.size();
    info.manifest_offset = mo;
    info.manifest_size = ms;
    return AOS_OK;
}

// A device copy of the archive (and optional extra strings after it); the
// digests of its segments and of the extras.
struct DeviceImage {
    uint8_t* d = nullptr;
    cudaStream_t s = nullptr;
    ~DeviceImage() {
        if (d) {
            cudaFreeAsync(d, s);
            cudaStreamSynchronize(s);
        }
    }
};

int hash_archive(aos_ctx* c, const uint8_t* b, uint64_t len, const std::vector<aos_archive_segment>& segs,
                 const std::vector<std::string>& extras, DeviceImage& img, std::vector<uint8_t>& digests,
                 std::string& err) {
    img.s = ctx_stream(c);
    uint64_t total = len;
    for (const auto& x : extras) total += x.size();
    cudaError_t e = cudaMallocAsync((void**)&img.d, std::max<uint64_t>(total, 1), img.s);
    if (e == cudaSuccess) e = cudaMemcpyAsync(img.d, b, len, cudaMemcpyHostToDevice, img.s);
    std::vector<uint64_t> off, n;
    for (const auto& sg : segs) {
        off.push_back(sg.offset);
        n.push_back(sg.len);
    }
    uint64_t at = len;
    for (const auto& x : extras) {
        if (e == cudaSuccess && !x.empty()) e = cudaMemcpyAsync(img.d + at, x.data(), x.size(), cudaMemcpyHostToDevice, img.s);
        off.push_back(at);
        n.push_back(x.size());
        at += x.size();
    }
    if (e != cudaSuccess) {
        err = std::string("archive copy to the device: ") + cudaGetErrorString(e);
        return AOS_ERR_CUDA;
    }
    digests.assign(32 * off.size(), 0);
    return blake3_many(img.d, off.data(), n.data(), (int)off.size(), digests.data(), img.s, err);
}

// select_segment_for_backend (lifecycle/src/loader.rs:177-218)
int select_for_backend(const std::vector<aos_archive_segment>& segs, const char* backend, const uint8_t scope[16]) {
    std::string be = backend ? backend : "";
    for (auto& ch : be) ch = (char)std::tolower((unsigned char)ch);
    const int preferred = be == "mlx" ? 1 : be == "metal" ? 2 : be == "coreml" ? 3 : be == "canonical" ? 0 : -1;
    static const uint8_t zero[16] = {0};
    auto find = [&](int tag, const uint8_t* h) -> int {
        for (size_t i = 0; i < segs.size(); ++i)
            if (segs[i].backend_tag == tag && !memcmp(segs[i].scope_hash, h, 16)) return (int)i;
        return -1;
    };
    const bool scoped = memcmp(scope, zero, 16) != 0;
    if (preferred > 0) {
        int i = scoped ? find(preferred, scope) : -1;
        if (i < 0) i = find(preferred, zero);
        if (i >= 0) return i;
    }
    if (scoped) {
        const int i = find(0, scope);
        if (i >= 0) return i;
    }
    return find(0, zero);
}

// canonical_layer_id (lifecycle/src/loader.rs:107-158)
std::string canonical_layer_id(const std::string& name) {
    std::vector<std::string> segs, parts;
    std::string cur;
    for (char ch : name) {
        if (ch == '.' || ch == '/') {
            parts.push_back(cur);
            cur.clear();
        } else {
            cur += ch;
        }
    }
    parts.push_back(cur);
    for (size_t i = 0; i < parts.size(); ++i) {
        const std::string& seg = parts[i];
        if (seg.empty()) continue;
        std::string lower = seg;
        for (auto& ch : lower) ch = (char)std::tolower((unsigned char)ch);
        if (lower == "weight") continue;
        if (lower == "model" || lower == "transformer") {
            if (segs.empty()) segs.push_back("transformer");
            continue;
        }
        if ((lower == "layers" || lower == "layer") && i + 1 < parts.size()) {
            const std::string& nx = parts[i + 1];
            if (!nx.empty() && nx.size() <= 19 && nx.find_first_not_of("0123456789") == std::string::npos) {
                segs.push_back("layer_" + std::to_string(strtoull(nx.c_str(), nullptr, 10)));
                ++i;
                continue;
            }
        }
        segs.push_back(lower == "lora_a" ? "lora_A" : lower == "lora_b" ? "lora_B" : lower);
    }
    if (segs.empty()) return name;
    if (segs[0] != "transformer") segs.insert(segs.begin(), "transformer");
    std::string out;
    for (size_t i = 0; i < segs.size(); ++i) out += (i ? "." : "") + segs[i];
    return out;
}

std::string hex32(const uint8_t* h) {
    static const char* d = "0123456789abcdef";
    std::string s;
    for (int i = 0; i < 32; ++i) {
        s += d[h[i] >> 4];
        s += d[h[i] & 15];
    }
    return s;
}

bool parse_hex32(const std::string& s, uint8_t out[32]) {  // B3Hash::from_hex: 64 hex digits
    if (s.size() != 64) return false;
    for (int i = 0; i < 32; ++i) {
        int v = 0;
        for (int j = 0; j < 2; ++j) {
            const char h = s[2 * i + j];
            const int d = h >= '0' && h <= '9' ? h - '0' : (h >= 'a' && h <= 'f') ? h - 'a' + 10 : (h >= 'A' && h <= 'F') ? h - 'A' + 10 : -1;
            if (d < 0) return false;
            v = v * 16 + d;
        }
        out[i] = (uint8_t)v;
    }
    return true;
}

std::string trim(const std::string& s) {
    size_t a = 0, b = s.size();
    while (a < b && std::isspace((unsigned char)s[a])) ++a;
    while (b > a && std::isspace((unsigned char)s[b - 1])) --b;
    return s.substr(a, b - a);
}

// metadata_value_any (mlx-ffi backend.rs:1166-1179)
const JVal* meta_any(const JVal& m, std::initializer_list<const char*> keys) {
    for (const char* k : keys) {
        if (const JVal* v = m.get(k)) return v;
        if (const JVal* md = m.get("metadata"))
            if (const JVal* v = md->get(k)) return v;
    }
    return nullptr;
}

// parse_rank / parse_alpha / the target-module override (backend.rs:1108-1200)
bool meta_rank(const JVal& m, uint32_t& rank) {
    const JVal* v = meta_any(m, {"rank", "lora_rank"});
    if (!v) return false;
    uint64_t r = 0;
    if (v->k == JVal::NUM && v->n_uint) {
        r = v->u;
    } else if (v->k == JVal::STR) {
        const std::string t = trim(v->s);
        if (t.empty() || t.size() > 19 || t.find_first_not_of("0123456789") != std::string::npos) return false;
        r = strtoull(t.c_str(), nullptr, 10);
    } else {
        return false;
    }
    if (r == 0 || r > 0xFFFFFFFFull) return false;
    rank = (uint32_t)r;
    return true;
}

bool meta_alpha(const JVal& m, float& alpha) {
    const JVal* v = meta_any(m, {"alpha", "lora_alpha"});
    if (!v) return false;
    float a;
    if (v->k == JVal::NUM) {
        a = (float)v->n;
    } else if (v->k == JVal::STR) {
        const std::string t = trim(v->s);
        char* stop = nullptr;
        a = strtof(t.c_str(), &stop);
        if (t.empty() || !stop || *stop != 0) return false;
    } else {
        return false;
    }
    if (!std::isfinite(a) || !(a > 0.0f)) return false;
    alpha = a;
    return true;
}

bool meta_targets(const JVal& m, std::vector<std::string>& out) {
    const JVal* v = meta_any(m, {"target_modules"});
    if (!v) return false;
    std::vector<std::string> mods;
    if (v->k == JVal::ARR) {
        for (const auto& e : v->a)
            if (e.k == JVal::STR && !trim(e.s).empty()) mods.push_back(trim(e.s));
    } else if (v->k == JVal::STR) {
        const std::string t = trim(v->s);
        if (!t.empty() && t[0] == '[') {
            JVal arr;
            std::string err;
            if (!parse_json(reinterpret_cast<const uint8_t*>(t.data()), t.size(), arr, err) || arr.k != JVal::ARR)
                return false;
            for (const auto& e : arr.a) {
                if (e.k != JVal::STR) return false;  // serde would reject a non-string element
                if (!trim(e.s).empty()) mods.push_back(trim(e.s));
            }
        } else {
            std::string cur;
            for (size_t i = 0; i <= t.size(); ++i) {
                if (i == t.size() || t[i] == ',') {
                    if (!trim(cur).empty()) mods.push_back(trim(cur));
                    cur.clear();
                } else {
                    cur += t[i];
                }
            }
        }
    } else {
        return false;
    }
    if (mods.empty()) return false;
    out.clear();
    for (auto& x : mods)
        if (std::find(out.begin(), out.end(), x) == out.end()) out.push_back(x);
    return true;
}

const char* const kModuleNames[AOS_NUM_MODULES] = {"q_proj", "k_proj", "v_proj", "o_proj",
                                                   "gate_proj", "up_proj", "down_proj"};

}  // namespace
}  // namespace aos

using namespace aos;

extern "C" {

int aos_archive_parse(const void* data, uint64_t len, aos_archive_info* info, aos_archive_segment* segs,
                      uint32_t max_segs) {
    aos_archive_info inf;
    std::vector<aos_archive_segment> sg;
    std::string err;
    const int rc = parse_layout(static_cast<const uint8_t*>(data), len, inf, sg, err);
    if (rc) {
        set_global_error("aos_archive_parse: " + err);
        return rc;
    }
    if (info) *info = inf;
    if (segs)
        for (uint32_t i = 0; i < std::min<uint32_t>(max_segs, inf.n_segments); ++i) segs[i] = sg[i];
    return AOS_OK;
}

int aos_blake3(aos_ctx* c, const void* data, uint64_t len, int on_device, uint8_t* out) {
    if (!c || !out || (!data && len)) return AOS_ERR_INVALID;
    int rc = ctx_set_device(c);
    if (rc) return rc;
    std::string err;
    const uint64_t off = 0;
    if (on_device) {
        rc = blake3_many(static_cast<const uint8_t*>(data), &off, &len, 1, out, ctx_stream(c), err);
    } else {  // the host bytes as one message of a device copy
        aos_archive_segment whole;
        memset(&whole, 0, sizeof whole);
        whole.len = len;
        DeviceImage img;
        std::vector<uint8_t> dig;
        rc = hash_archive(c, static_cast<const uint8_t*>(data), len, {whole}, {}, img, dig, err);
        if (!rc) memcpy(out, dig.data(), 32);
    }
    return rc ? ctx_fail(c, rc, err) : AOS_OK;
}

int aos_archive_verify(aos_ctx* c, const void* data, uint64_t len, int32_t* bad_segment) {
    if (!c) return AOS_ERR_INVALID;
    if (bad_segment) *bad_segment = -1;
    const uint8_t* b = static_cast<const uint8_t*>(data);
    aos_archive_info inf;
    std::vector<aos_archive_segment> segs;
    std::string err;
    int rc = parse_layout(b, len, inf, segs, err);
    if (rc) return ctx_fail(c, rc, err);
    if ((rc = ctx_set_device(c))) return rc;
    DeviceImage img;
    std::vector<uint8_t> dig;
    if ((rc = hash_archive(c, b, len, segs, {}, img, dig, err))) return ctx_fail(c, rc, err);
    for (size_t i = 0; i < segs.size(); ++i)
        if (memcmp(dig.data() + 32 * i, segs[i].weights_hash, 32)) {
            if (bad_segment) *bad_segment = (int32_t)i;
            return ctx_fail(c, AOS_ERR_INVALID, "Corrupted / needs retrain: segment " +
                                                     std::to_string(segs[i].segment_id) + " hash mismatch");
        }
    return AOS_OK;
}

int aos_adapter_load_aos(aos_ctx* c, uint16_t id, const void* data, uint64_t len, const char* backend,
                         aos_archive_load_info* info) {
    if (!c) return AOS_ERR_INVALID;
    const uint8_t* b = static_cast<const uint8_t*>(data);
    aos_archive_info inf;
    std::vector<aos_archive_segment> segs;
    std::string err;
    int rc = parse_layout(b, len, inf, segs, err);
    if (rc) return ctx_fail(c, rc, err);
    // manifest and scope path (hashed with the segments)
    JVal man;
    if (!parse_json(b + inf.manifest_offset, inf.manifest_size, man, err, "manifest JSON"))
        return ctx_fail(c, AOS_ERR_INVALID, err);
    if (man.k != JVal::OBJ) return ctx_fail(c, AOS_ERR_INVALID, "manifest JSON: not an object");
    const JVal* md = man.get("metadata");
    const JVal* sp = md ? md->get("scope_path") : nullptr;
    if (!sp || sp->k != JVal::STR || sp->s.empty())
        return ctx_fail(c, AOS_ERR_INVALID, "Corrupted / needs retrain: missing scope_path in manifest metadata");
    if ((rc = ctx_set_device(c))) return rc;
    DeviceImage img;
    std::vector<uint8_t> dig;
    if ((rc = hash_archive(c, b, len, segs, {sp->s}, img, dig, err))) return ctx_fail(c, rc, err);
    for (size_t i = 0; i < segs.size(); ++i)
        if (memcmp(dig.data() + 32 * i, segs[i].weights_hash, 32))
            return ctx_fail(c, AOS_ERR_INVALID, "Corrupted / needs retrain: segment " +
                                                    std::to_string(segs[i].segment_id) + " hash mismatch");
    if (std::none_of(segs.begin(), segs.end(), [](const aos_archive_segment& s) { return s.backend_tag == 0; }))
        return ctx_fail(c, AOS_ERR_NOT_FOUND, "archive has no canonical segment");
    const uint8_t* scope = dig.data() + 32 * segs.size();  // first 16 bytes of BLAKE3(scope_path)
    const int si = select_for_backend(segs, backend, scope);
    if (si < 0)
        return ctx_fail(c, AOS_ERR_NOT_FOUND, "no segment for backend '" + std::string(backend ? backend : "") +
                                                  "' and scope_path " + sp->s);
    const aos_archive_segment& sel = segs[si];
    const uint8_t* payload = b + sel.offset;
    std::vector<StTensor> ts;
    const uint8_t* base = nullptr;
    if ((rc = parse_safetensors(payload, sel.len, ts, &base, err)))
        return ctx_fail(c, rc, "Failed to parse SafeTensors from .aos: " + err);
    // per-layer hashes: BLAKE3 of each tensor's bytes, by canonical layer id
    if (const JVal* plh = man.get("per_layer_hashes")) {
        if (plh->k == JVal::OBJ && !plh->o.empty()) {
            std::vector<uint64_t> off, n;
            std::vector<std::string> ids;
            for (const auto& t : ts) {
                off.push_back(sel.offset + (uint64_t)(base - payload) + t.b);
                n.push_back(t.e - t.b);
                ids.push_back(canonical_layer_id(t.name));
            }
            std::vector<uint8_t> th(32 * ts.size());
            if ((rc = blake3_many(img.d, off.data(), n.data(), (int)ts.size(), th.data(), img.s, err)))
                return ctx_fail(c, rc, err);
            for (const auto& kv : plh->o) {
                const JVal* hv = kv.second.k == JVal::STR ? &kv.second : kv.second.get("hash");
                uint8_t want[32];
                if (!hv || hv->k != JVal::STR || !parse_hex32(hv->s, want))
                    return ctx_fail(c, AOS_ERR_INVALID, "Invalid per-layer hash for '" + kv.first + "'");
                const std::string cid = canonical_layer_id(kv.first);
                int hit = -1;
                for (size_t i = 0; i < ids.size() && hit < 0; ++i)
                    if (ids[i] == cid) hit = (int)i;  // first tensor with this id, in container order
                if (hit < 0)
                    return ctx_fail(c, AOS_ERR_INVALID, "Per-layer hash provided for missing tensor '" + cid + "'");
                if (memcmp(th.data() + 32 * hit, want, 32))
                    return ctx_fail(c, AOS_ERR_INVALID, "adapter layer hash mismatch for " + cid);
            }
        }
    }
    if (const JVal* wh = man.get("weights_hash")) {
        if (wh->k == JVal::STR) {
            uint8_t want[32];
            if (!parse_hex32(wh->s, want)) return ctx_fail(c, AOS_ERR_INVALID, "Invalid manifest weights_hash");
            if (memcmp(want, dig.data() + 32 * si, 32))
                return ctx_fail(c, AOS_ERR_INVALID, "adapter hash mismatch: expected " + wh->s + ", actual " +
                                                        hex32(dig.data() + 32 * si));
        }
    }
    // MLX adapter rules
    std::vector<std::string> discovered;
    for (const auto& t : ts) {
        if (t.name.rfind("lora_a.", 0) == 0) discovered.push_back(t.name.substr(7));
        else if (t.name.size() > 7 && t.name.compare(t.name.size() - 7, 7, ".lora_A") == 0)
            discovered.push_back(t.name.substr(0, t.name.size() - 7));
    }
    std::sort(discovered.begin(), discovered.end());
    discovered.erase(std::unique(discovered.begin(), discovered.end()), discovered.end());
    uint32_t rank = 4;
    float alpha = 16.0f;
    std::vector<std::string> targets = discovered.empty()
                                           ? std::vector<std::string>{"q_proj", "k_proj", "v_proj", "o_proj"}
                                           : discovered;
    meta_rank(man, rank);
    meta_alpha(man, alpha);
    meta_targets(man, targets);
    auto find = [&](const std::string& name) -> int {
        for (size_t i = 0; i < ts.size(); ++i)
            if (ts[i].name == name) return (int)i;
        return -1;
    };
    uint32_t L = 0, in[AOS_NUM_MODULES], out[AOS_NUM_MODULES], H = 0, V = 0;
    ctx_model_dims(c, &L, in, out, &H, &V);
    struct Mod { int m, a, b; };
    std::vector<Mod> mods;
    int64_t tr = -1;
    for (const auto& name : targets) {
        int a = find("lora_a." + name), bb = find("lora_b." + name);
        if (a < 0 || bb < 0) {
            a = find(name + ".lora_A");
            bb = find(name + ".lora_B");
            if (a < 0 || bb < 0) continue;
        }
        int m = -1;
        for (int k = 0; k < AOS_NUM_MODULES; ++k)
            if (name == kModuleNames[k]) m = k;
        if (m < 0) continue;  // a module this model has no projection for
        if (std::any_of(mods.begin(), mods.end(), [&](const Mod& x) { return x.m == m; })) continue;
        const StTensor &A = ts[a], &B = ts[bb];
        if (A.shape.size() != 2 || A.shape[1] != (int64_t)in[m] || A.shape[0] < 1)
            return ctx_fail(c, AOS_ERR_INVALID, "tensor " + A.name + ": lora_A must be [rank, in] of its module");
        if (B.shape.size() != 2 || B.shape[0] != (int64_t)out[m] || B.shape[1] != A.shape[0])
            return ctx_fail(c, AOS_ERR_INVALID, "tensor " + B.name + ": lora_B must be [out, rank] of its module");
        if (tr >= 0 && A.shape[0] != tr)
            return ctx_fail(c, AOS_ERR_INVALID, "tensor " + A.name + ": rank differs from the other modules'");
        tr = A.shape[0];
        mods.push_back({m, a, bb});
    }
    if (mods.empty())
        return ctx_fail(c, AOS_ERR_INVALID, "no lora_a/lora_b pair in the payload for any target module of this model");
    const uint32_t store = (uint32_t)std::max<int64_t>(8, (tr + 7) / 8 * 8);
    if (store > 256) return ctx_fail(c, AOS_ERR_INVALID, "adapter rank above 256");
    if ((rc = ctx_adapter_new(c, id, store, alpha, alpha / (float)rank))) return rc;
    std::vector<uint16_t> a16, b16, A, B;
    uint32_t mask = 0;
    for (const Mod& x : mods) {
        if ((rc = tensor_to_bf16(ts[x.a], base, a16, err)) || (rc = tensor_to_bf16(ts[x.b], base, b16, err))) {
            aos_adapter_unload(c, id);
            return ctx_fail(c, rc, err);
        }
        A.assign((size_t)store * in[x.m], 0);  // rows past the tensor rank stay zero
        std::copy(a16.begin(), a16.end(), A.begin());
        B.assign((size_t)out[x.m] * store, 0);
        for (uint32_t o = 0; o < out[x.m]; ++o)
            std::copy(b16.begin() + (size_t)o * tr, b16.begin() + (size_t)(o + 1) * tr, B.begin() + (size_t)o * store);
        for (uint32_t l = 0; l < L; ++l)
            if ((rc = aos_adapter_set_module(c, id, l, (aos_module)x.m, A.data(), B.data(), 0))) {
                aos_adapter_unload(c, id);
                return rc;
            }
        mask |= 1u << x.m;
    }
    if (info) {
        memset(info, 0, sizeof *info);
        info->rank = rank;
        info->tensor_rank = (uint32_t)tr;
        info->storage_rank = store;
        info->alpha = alpha;
        info->module_mask = mask;
        info->segment_id = sel.segment_id;
        info->backend_tag = sel.backend_tag;
        memcpy(info->weights_hash, dig.data() + 32 * si, 32);
        memcpy(info->scope_hash, scope, 16);
    }
    return AOS_OK;
}

}  // extern "C"
