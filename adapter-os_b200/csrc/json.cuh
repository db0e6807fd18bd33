// json.cuh — a JSON reader for the loaders (safetensors headers, .aos
// manifests): values as a tree, numbers kept as double plus, for unsigned
// integer literals, their exact uint64 (tensor offsets need all 64 bits).
// Host code only.
#pragma once

#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <string>
#include <utility>
#include <vector>

namespace aos {

struct JVal {
    enum Kind { NUL, BOOL, NUM, STR, ARR, OBJ } k = NUL;
    bool b = false;
    double n = 0;
    bool n_uint = false;  // an integer literal without sign, fraction or exponent
    uint64_t u = 0;
    std::string s;
    std::vector<JVal> a;
    std::vector<std::pair<std::string, JVal>> o;
    const JVal* get(const char* key) const {  // a repeated key keeps its last value, as serde_json's map does
        if (k != OBJ) return nullptr;
        for (auto it = o.rbegin(); it != o.rend(); ++it)
            if (it->first == key) return &it->second;
        return nullptr;
    }
};

struct JParser {
    const char* p;
    const char* end;
    std::string err;
    int depth = 0;
    void ws() {
        while (p < end && (*p == ' ' || *p == '\n' || *p == '\r' || *p == '\t')) ++p;
    }
    bool fail(const char* m) {
        if (err.empty()) err = m;
        return false;
    }
    static void utf8(std::string& out, uint32_t v) {
        if (v < 0x80) {
            out += (char)v;
        } else if (v < 0x800) {
            out += (char)(0xC0 | (v >> 6));
            out += (char)(0x80 | (v & 63));
        } else if (v < 0x10000) {
            out += (char)(0xE0 | (v >> 12));
            out += (char)(0x80 | ((v >> 6) & 63));
            out += (char)(0x80 | (v & 63));
        } else {
            out += (char)(0xF0 | (v >> 18));
            out += (char)(0x80 | ((v >> 12) & 63));
            out += (char)(0x80 | ((v >> 6) & 63));
            out += (char)(0x80 | (v & 63));
        }
    }
    bool hex4(uint32_t& v) {
        if (end - p < 4) return fail("truncated \\u escape");
        v = 0;
        for (int i = 0; i < 4; ++i) {
            const char h = *p++;
            int d = h >= '0' && h <= '9' ? h - '0' : (h >= 'a' && h <= 'f') ? h - 'a' + 10 : (h >= 'A' && h <= 'F') ? h - 'A' + 10 : -1;
            if (d < 0) return fail("bad \\u escape");
            v = v * 16 + (uint32_t)d;
        }
        return true;
    }
    bool str(std::string& out) {
        if (p >= end || *p != '"') return fail("expected a string");
        ++p;
        out.clear();
        while (p < end && *p != '"') {
            const unsigned char ch = (unsigned char)*p;
            if (ch < 0x20) return fail("control character in a string");
            if (ch != '\\') {
                out += *p++;
                continue;
            }
            if (++p >= end) break;
            const char e = *p++;
            switch (e) {
                case '"': out += '"'; break;
                case '\\': out += '\\'; break;
                case '/': out += '/'; break;
                case 'b': out += '\b'; break;
                case 'f': out += '\f'; break;
                case 'n': out += '\n'; break;
                case 'r': out += '\r'; break;
                case 't': out += '\t'; break;
                case 'u': {
                    uint32_t v;
                    if (!hex4(v)) return false;
                    if (v >= 0xD800 && v < 0xDC00) {  // surrogate pair
                        uint32_t w;
                        if (end - p < 6 || p[0] != '\\' || p[1] != 'u') return fail("lone surrogate");
                        p += 2;
                        if (!hex4(w) || w < 0xDC00 || w >= 0xE000) return fail("lone surrogate");
                        v = 0x10000 + ((v - 0xD800) << 10) + (w - 0xDC00);
                    } else if (v >= 0xDC00 && v < 0xE000) {
                        return fail("lone surrogate");
                    }
                    utf8(out, v);
                    break;
                }
                default: return fail("bad escape");
            }
        }
        if (p >= end) return fail("unterminated string");
        ++p;
        return true;
    }
    bool value(JVal& v) {
        ws();
        if (p >= end) return fail("truncated JSON");
        if (++depth > 128) return fail("JSON nested too deeply");
        bool ok = true;
        const char c = *p;
        if (c == '{') {
            v.k = JVal::OBJ;
            ++p;
            ws();
            if (p < end && *p == '}') {
                ++p;
            } else {
                while (ok) {
                    ws();
                    std::pair<std::string, JVal> kv;
                    ok = str(kv.first);
                    ws();
                    if (ok && (p >= end || *p++ != ':')) ok = fail("expected ':'");
                    if (ok) ok = value(kv.second);
                    if (!ok) break;
                    v.o.push_back(std::move(kv));
                    ws();
                    if (p < end && *p == ',') { ++p; continue; }
                    if (p < end && *p == '}') { ++p; break; }
                    ok = fail("expected ',' or '}'");
                }
            }
        } else if (c == '[') {
            v.k = JVal::ARR;
            ++p;
            ws();
            if (p < end && *p == ']') {
                ++p;
            } else {
                while (ok) {
                    JVal e;
                    ok = value(e);
                    if (!ok) break;
                    v.a.push_back(std::move(e));
                    ws();
                    if (p < end && *p == ',') { ++p; continue; }
                    if (p < end && *p == ']') { ++p; break; }
                    ok = fail("expected ',' or ']'");
                }
            }
        } else if (c == '"') {
            v.k = JVal::STR;
            ok = str(v.s);
        } else if (end - p >= 4 && !memcmp(p, "null", 4)) {
            v.k = JVal::NUL;
            p += 4;
        } else if (end - p >= 4 && !memcmp(p, "true", 4)) {
            v.k = JVal::BOOL;
            v.b = true;
            p += 4;
        } else if (end - p >= 5 && !memcmp(p, "false", 5)) {
            v.k = JVal::BOOL;
            p += 5;
        } else if (c == '-' || (c >= '0' && c <= '9')) {
            const char* s0 = p;
            if (*p == '-') ++p;
            while (p < end && ((*p >= '0' && *p <= '9') || *p == '.' || *p == 'e' || *p == 'E' || *p == '+' || *p == '-'))
                ++p;
            const std::string lit(s0, p);
            char* stop = nullptr;
            v.k = JVal::NUM;
            v.n = strtod(lit.c_str(), &stop);
            if (!stop || *stop != 0) ok = fail("bad number");
            v.n_uint = lit.find_first_not_of("0123456789") == std::string::npos && lit.size() <= 19;
            if (v.n_uint) v.u = strtoull(lit.c_str(), nullptr, 10);
        } else {
            ok = fail("unexpected character in JSON");
        }
        --depth;
        return ok;
    }
};

// Parses d[0..n) as one JSON value; on failure err = "<what>: <reason>".
inline bool parse_json(const uint8_t* d, uint64_t n, JVal& v, std::string& err, const char* what = "JSON") {
    JParser jp{reinterpret_cast<const char*>(d), reinterpret_cast<const char*>(d) + n, {}, 0};
    if (!jp.value(v)) {
        err = std::string(what) + ": " + jp.err;
        return false;
    }
    jp.ws();
    if (jp.p != jp.end) {
        err = std::string(what) + ": trailing bytes";
        return false;
    }
    return true;
}

}  // namespace aos
