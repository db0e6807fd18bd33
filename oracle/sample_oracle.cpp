// CPU oracle for next-token sampling.  TEST INFRASTRUCTURE ONLY (tests/,
// smoke(), bench's CPU leg); the product samples on the GPU
// (adapter-os_b200/csrc/sample.cu).
//
// Restates Generator (crates/adapteros-lora-worker/src/generation.rs):
// process_logits 321-343, softmax 387-401, apply_top_k 404-422, apply_top_p
// 424-453, sample_from_distribution 456-480, greedy 483-490.  Rust semantics
// kept: Iterator::max_by keeps the later element on Equal and on a NaN
// comparison; f32 sums are sequential left folds; sort_by is stable;
// f32::exp is libm's expf (glibc here).
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <utility>
#include <vector>

namespace {

size_t fold_argmax(const std::vector<float>& x) {
    size_t best = 0;
    for (size_t i = 1; i < x.size(); ++i)
        if (!(x[best] > x[i])) best = i;
    return best;
}

float seq_sum(const std::vector<float>& x) {
    float s = 0.0f;
    for (float v : x) s += v;
    return s;
}

std::vector<std::pair<size_t, float>> sorted_desc(const std::vector<float>& p) {
    std::vector<std::pair<size_t, float>> ip(p.size());
    for (size_t i = 0; i < p.size(); ++i) ip[i] = {i, p[i]};
    std::stable_sort(ip.begin(), ip.end(), [](const std::pair<size_t, float>& a, const std::pair<size_t, float>& b) {
        return a.second > b.second;
    });
    return ip;
}

std::vector<float> renorm(std::vector<float> r) {
    const float s = seq_sum(r);
    if (s > 0.0f)
        for (auto& v : r) v = v / s;
    return r;
}

}  // namespace

extern "C" {

uint32_t oracle_greedy(const float* logits, uint32_t V) {
    return (uint32_t)fold_argmax(std::vector<float>(logits, logits + V));
}

uint32_t oracle_sample(const float* logits, uint32_t V, float temperature, int has_top_k, uint32_t top_k,
                       int has_top_p, float top_p, float u) {
    std::vector<float> x(logits, logits + V);
    if (temperature != 1.0f)
        for (auto& v : x) v = v / temperature;
    const float mx = x.empty() ? 0.0f : x[fold_argmax(x)];
    for (auto& v : x) v = expf(v - mx);
    const float sum = seq_sum(x);
    for (auto& v : x) v = v / sum;
    if (has_top_k) {
        auto ip = sorted_desc(x);
        std::vector<float> r(V, 0.0f);
        for (size_t q = 0; q < ip.size() && q < top_k; ++q) r[ip[q].first] = ip[q].second;
        x = renorm(std::move(r));
    }
    if (has_top_p) {
        auto ip = sorted_desc(x);
        float cum = 0.0f;
        size_t cut = ip.size();
        for (size_t q = 0; q < ip.size(); ++q) {
            cum += ip[q].second;
            if (cum >= top_p) {
                cut = q + 1;
                break;
            }
        }
        std::vector<float> r(V, 0.0f);
        for (size_t q = 0; q < cut; ++q) r[ip[q].first] = ip[q].second;
        x = renorm(std::move(r));
    }
    const float total = seq_sum(x);
    if (total <= 0.0f) return (uint32_t)fold_argmax(x);
    float cum = 0.0f;
    for (size_t i = 0; i < x.size(); ++i) {
        cum += x[i];
        if (u <= cum) return (uint32_t)i;
    }
    return V - 1;
}

}  // extern "C"
