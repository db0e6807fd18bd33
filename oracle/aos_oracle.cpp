// aos_oracle.cpp — CPU restatement of adapter-os's per-token hot path.
//
// TEST INFRASTRUCTURE ONLY: the checker for the CUDA library and the timed CPU
// baseline.  The product library never links or calls it.
//
// Reference citations are file:line inside the rogu3bear/adapter-os tree.
// Compile with -O3 -fno-fast-math -ffp-contract=off (see oracle/Makefile).

#include "aos_oracle.h"

#include <algorithm>
#include <cmath>
#include <cstring>
#include <vector>
#ifdef _OPENMP
#include <omp.h>
#endif

namespace {

constexpr uint32_t kMaxK = 8;               // crates/adapteros-core/src/defaults.rs:37
constexpr float kDefaultEntropyFloor = 0.02f;  // defaults.rs:24
constexpr float kQ15Denom = 32767.0f;        // quantization.rs:22
constexpr int32_t kQ15Max = 32767;           // quantization.rs:23

int threads_or_default(int n) {
#ifdef _OPENMP
    return n > 0 ? n : omp_get_max_threads();
#else
    (void)n;
    return 1;
#endif
}

// f32::total_cmp key (Rust core::f32::total_cmp): flip the magnitude bits of
// negative numbers so that signed-integer order is the IEEE total order.
inline int32_t total_key(float f) {
    int32_t i;
    std::memcpy(&i, &f, 4);
    i ^= (int32_t)(((uint32_t)(i >> 31)) >> 1);
    return i;
}

// sanitize_k / sanitize_eps / sanitize_tau (router.rs:127-187).
uint32_t sanitize_k(uint32_t k) { return k == 0 ? 1 : (k > kMaxK ? kMaxK : k); }
float sanitize_eps(float eps) {
    if (!std::isfinite(eps)) return kDefaultEntropyFloor;
    if (!(eps >= 0.0f && eps <= 1.0f)) return kDefaultEntropyFloor;
    return eps;
}
float sanitize_tau(float tau) {
    if (!std::isfinite(tau)) return 1.0f;
    if (tau <= 0.0f) return 1.0f;
    return tau;
}

// Rust `f32 as i32` is saturating with NaN -> 0.
int32_t f32_as_i32(float f) {
    if (std::isnan(f)) return 0;
    if (f >= 2147483648.0f) return INT32_MAX;
    if (f < -2147483648.0f) return INT32_MIN;
    return (int32_t)f;
}

struct Cand {
    uint32_t idx;
    float score;
};

// One token through Router::route_with_adapter_info_and_scope_with_ctx
// (router.rs:1567-1952) with empty features, no scope hint, deterministic
// (non-adaptive) tie-breaking, orthogonality off and is_moe_model = false.
int route_one(const float* priors, const uint64_t* stable_ids, const float* vw,
              const uint8_t* allowed, uint32_t N, uint32_t k, float tau, float eps,
              float bias, oracle_ring* ring, float* entropy_out) {
    std::memset(ring, 0, sizeof(*ring));
    if (entropy_out) *entropy_out = 0.0f;
    // validate_router_inputs (router.rs:611-625): any non-finite prior -> error.
    for (uint32_t i = 0; i < N; ++i)
        if (!std::isfinite(priors[i])) return ORACLE_ERR_NONFINITE;

    // Scoring loop (router.rs:1632-1690).  Features are empty, so
    // compute_adapter_feature_score returns 0.0 (router.rs:985-988); the
    // orthogonal penalty is 0.0 when disabled (router.rs:1490-1493).
    std::vector<Cand> scores;
    scores.reserve(N);
    for (uint32_t i = 0; i < N; ++i) {
        if (allowed && !allowed[i]) continue;
        const float feature_score = 0.0f;
        const float penalty = 0.0f;
        float s = ((priors[i] + feature_score) - penalty) * bias;  // scoring.rs:35-37
        float w = 1.0f;
        if (vw) {
            w = vw[i];
            if (std::isfinite(w)) {
                if (w < 0.0f) w = 0.0f;   // f32::clamp(0.0, 2.0)
                if (w > 2.0f) w = 2.0f;
            } else {
                w = 1.0f;
            }
        }
        s = s * w;
        if (!std::isfinite(s)) return ORACLE_ERR_NONFINITE;
        scores.push_back({i, s});
    }
    if (scores.empty()) return ORACLE_OK;  // empty decision (router.rs:1692-1699)

    // sort_scores_deterministic (router.rs:234-264): score DESC by total_cmp,
    // stable_id ASC; Rust's sort_by is stable, so equal keys keep index order.
    std::sort(scores.begin(), scores.end(), [&](const Cand& a, const Cand& b) {
        int32_t ka = total_key(a.score), kb = total_key(b.score);
        if (ka != kb) return ka > kb;
        if (stable_ids[a.idx] != stable_ids[b.idx]) return stable_ids[a.idx] < stable_ids[b.idx];
        return a.idx < b.idx;
    });
    const uint32_t n = std::min<uint32_t>(k, (uint32_t)scores.size());  // take(K) (:1812)

    float top_scores[kMaxK];
    for (uint32_t j = 0; j < n; ++j) top_scores[j] = scores[j].score;
    float gates[kMaxK];
    oracle_deterministic_softmax(top_scores, (int)n, tau, gates);

    // Entropy floor (router.rs:1818-1827); tau is never 0 after sanitize_tau.
    if (tau != 0.0f) {
        const uint32_t active_k = n > 0 ? n : 1;
        const float min_gate = eps / (float)active_k;
        for (uint32_t j = 0; j < n; ++j) gates[j] = std::fmax(gates[j], min_gate);
    }
    // Renormalise with a sequential f32 sum (router.rs:1830-1842).
    float sum = -0.0f;
    for (uint32_t j = 0; j < n; ++j) sum = sum + gates[j];
    if (sum <= 0.0f || n == 0) return ORACLE_OK;  // empty decision
    for (uint32_t j = 0; j < n; ++j) gates[j] = gates[j] / sum;

    // compute_entropy (router.rs:1287-1293).
    float ent = -0.0f;
    for (uint32_t j = 0; j < n; ++j)
        if (gates[j] > 0.0f) ent = ent + (-gates[j]) * std::log2(gates[j]);
    if (entropy_out) *entropy_out = ent;

    struct DC { uint16_t idx; float raw; int16_t q; };
    DC cands[kMaxK];
    for (uint32_t j = 0; j < n; ++j)
        cands[j] = {(uint16_t)scores[j].idx, scores[j].score, oracle_quantize_gate(gates[j])};
    // sort_candidates_by_quantized_gate_canonical (router.rs:1310-1325).
    std::sort(cands, cands + n, [&](const DC& a, const DC& b) {
        if (a.q != b.q) return a.q > b.q;
        int32_t ka = total_key(a.raw), kb = total_key(b.raw);
        if (ka != kb) return ka > kb;
        if (stable_ids[a.idx] != stable_ids[b.idx]) return stable_ids[a.idx] < stable_ids[b.idx];
        return a.idx < b.idx;
    });
    // Decision::to_router_ring (types.rs:699-706) -> RouterRing::set (kernel-api lib.rs:140-193).
    ring->top_k = n;
    for (uint32_t j = 0; j < n; ++j) {
        ring->indices[j] = cands[j].idx;
        ring->gates_q15[j] = cands[j].q;
    }
    return ORACLE_OK;
}

// ---------------------------------------------------------------- bf16 helpers
inline float bf(uint16_t h) {
    uint32_t u = (uint32_t)h << 16;
    float f;
    std::memcpy(&f, &u, 4);
    return f;
}
inline uint16_t to_bf(float f) {
    uint32_t u;
    std::memcpy(&u, &f, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40);  // quiet NaN
    u += 0x7fffu + ((u >> 16) & 1u);  // round to nearest even
    return (uint16_t)(u >> 16);
}
inline float rbf(float f) { return bf(to_bf(f)); }

// Dot product of a bf16 row with an f32 vector, accumulated in double with a
// fixed 4-way split (order fixed, so results are reproducible).
inline double dot_bf_f(const uint16_t* w, const float* x, uint32_t n) {
    double a0 = 0, a1 = 0, a2 = 0, a3 = 0;
    uint32_t j = 0;
    for (; j + 4 <= n; j += 4) {
        a0 += (double)bf(w[j]) * x[j];
        a1 += (double)bf(w[j + 1]) * x[j + 1];
        a2 += (double)bf(w[j + 2]) * x[j + 2];
        a3 += (double)bf(w[j + 3]) * x[j + 3];
    }
    for (; j < n; ++j) a0 += (double)bf(w[j]) * x[j];
    return (a0 + a1) + (a2 + a3);
}

struct Dims {
    uint32_t H, nq, nkv, hd, I, V;
    uint32_t out_dim[ORACLE_NUM_MODS];
    uint32_t in_dim[ORACLE_NUM_MODS];
};

Dims dims_of(const oracle_model* m) {
    Dims d;
    d.H = m->hidden; d.nq = m->n_heads; d.nkv = m->n_kv_heads; d.hd = m->head_dim;
    d.I = m->inter; d.V = m->vocab;
    const uint32_t q = d.nq * d.hd, kv = d.nkv * d.hd;
    const uint32_t outs[7] = {q, kv, kv, d.H, d.I, d.I, d.H};
    const uint32_t ins[7] = {d.H, d.H, d.H, q, d.H, d.H, d.I};
    for (int i = 0; i < 7; ++i) { d.out_dim[i] = outs[i]; d.in_dim[i] = ins[i]; }
    return d;
}

// y[t][o] = x[t] . W[o]  for all t (f32 result, double accumulation),
// parallel over output rows so W streams once for the whole batch.
void linear(const uint16_t* W, const float* x, uint32_t T, uint32_t in, uint32_t out,
            float* y, int nt) {
#pragma omp parallel for num_threads(nt) schedule(static)
    for (int64_t o = 0; o < (int64_t)out; ++o) {
        const uint16_t* w = W + (size_t)o * in;
        for (uint32_t t = 0; t < T; ++t) y[(size_t)t * out + o] = (float)dot_bf_f(w, x + (size_t)t * in, in);
    }
}

// LoRA delta for one module: MLX apply_lora (mlx_cpp_wrapper_real.cpp:3394-3419)
// with blend = q15/32767 (mlx-ffi/src/backend.rs:405-418, skip q15 <= 0) and
// scale = alpha/rank (wrapper.h:383-394).  Adds into y (f32 [T, out]).
// rounding_mode 0: h is gated and rounded to bf16 before the expand (the fused
// CUDA path's storage point).  1: MLX op-by-op bf16 rounding.
void lora_delta(const oracle_adapters* ad, uint32_t layer, uint32_t n_layers, int mod,
                const oracle_ring* rings, uint32_t T, const float* x, uint32_t in,
                uint32_t out, float* y, int rounding_mode, int nt) {
    if (!ad || ad->n_adapters == 0) return;
#pragma omp parallel for num_threads(nt) schedule(dynamic, 1)
    for (int64_t t = 0; t < (int64_t)T; ++t) {
        const oracle_ring& r = rings[t];
        std::vector<float> acc(out, 0.0f);
        bool any = false;
        for (uint32_t s = 0; s < r.top_k && s < kMaxK; ++s) {
            const int16_t q = r.gates_q15[s];
            if (q <= 0) continue;
            const uint32_t a = r.indices[s];
            if (a >= ad->n_adapters) continue;
            const size_t slot = ((size_t)a * n_layers + layer) * ORACLE_NUM_MODS + mod;
            const uint16_t* A = ad->A[slot];
            const uint16_t* B = ad->B[slot];
            if (!A || !B) continue;
            const uint32_t rank = ad->rank[a];
            const float blend = (float)q / kQ15Denom;
            const float scale = ad->alpha[a] / (float)rank;
            std::vector<float> h(rank);
            for (uint32_t j = 0; j < rank; ++j) {
                float v = (float)dot_bf_f(A + (size_t)j * in, x + (size_t)t * in, in);
                h[j] = v;
            }
            if (rounding_mode == 0) {
                const float coef = blend * scale;
                for (uint32_t j = 0; j < rank; ++j) h[j] = rbf(h[j] * coef);
                for (uint32_t o = 0; o < out; ++o) {
                    double d = 0.0;
                    for (uint32_t j = 0; j < rank; ++j) d += (double)bf(B[(size_t)o * rank + j]) * h[j];
                    acc[o] += (float)d;
                }
            } else {
                for (uint32_t j = 0; j < rank; ++j) h[j] = rbf(h[j]);
                const float coef = rbf(scale * blend);
                for (uint32_t o = 0; o < out; ++o) {
                    double d = 0.0;
                    for (uint32_t j = 0; j < rank; ++j) d += (double)bf(B[(size_t)o * rank + j]) * h[j];
                    float lo = rbf(rbf((float)d) * coef);
                    acc[o] = any ? rbf(acc[o] + lo) : lo;
                }
                any = true;
            }
            if (rounding_mode == 0) any = true;
        }
        if (!any) continue;
        float* yt = y + (size_t)t * out;
        if (rounding_mode == 0) {
            for (uint32_t o = 0; o < out; ++o) yt[o] += acc[o];
        } else {
            for (uint32_t o = 0; o < out; ++o) yt[o] = rbf(rbf(yt[o]) + acc[o]);
        }
    }
}

// RMSNorm (mlx_cpp_wrapper_real.cpp:3384-3390): x * (w / sqrt(mean(x^2) + eps)).
void rms_norm(const float* x, const uint16_t* w, uint32_t T, uint32_t H, float eps,
              float* out, int rounding_mode) {
    for (uint32_t t = 0; t < T; ++t) {
        const float* xt = x + (size_t)t * H;
        double ss = 0.0;
        for (uint32_t j = 0; j < H; ++j) {
            float sq = xt[j] * xt[j];
            if (rounding_mode == 1) sq = rbf(sq);
            ss += sq;
        }
        float ms = (float)(ss / (double)H);
        if (rounding_mode == 1) ms = rbf(ms);
        float denom = std::sqrt(ms + eps);
        if (rounding_mode == 1) denom = rbf(std::sqrt(rbf(ms + eps)));
        for (uint32_t j = 0; j < H; ++j) {
            float f = bf(w[j]) / denom;
            if (rounding_mode == 1) f = rbf(f);
            out[(size_t)t * H + j] = rbf(xt[j] * f);
        }
    }
}

inline float silu_mul(float g, float u, int rounding_mode) {
    // gate * sigmoid(gate) * up (mlx_cpp_wrapper_real.cpp:3522).
    float sg = 1.0f / (1.0f + std::exp(-g));
    if (rounding_mode == 1) {
        sg = rbf(sg);
        return rbf(rbf(g * sg) * u);
    }
    return rbf((g * sg) * u);
}

inline size_t kv_index(const oracle_kv* kv, uint32_t nkv, uint32_t hd, uint32_t layer,
                       int32_t blk, uint32_t h, uint32_t off) {
    return ((((size_t)layer * kv->num_blocks + (size_t)blk) * nkv + h) * kv->block_size + off) * hd;
}

}  // namespace

extern "C" {

float oracle_bf16_to_f32(uint16_t h) { return bf(h); }
uint16_t oracle_f32_to_bf16(float f) { return to_bf(f); }

int16_t oracle_quantize_gate(float gate) {
    // ((gate * 32767.0).round() as i32).clamp(0, 32767); Rust f32::round is
    // round-half-away-from-zero, which is C roundf.
    int32_t scaled = f32_as_i32(std::round(gate * kQ15Denom));
    if (scaled < 0) scaled = 0;
    if (scaled > kQ15Max) scaled = kQ15Max;
    return (int16_t)scaled;
}

void oracle_deterministic_softmax(const float* scores, int n, float tau, float* out) {
    // router.rs:1340-1411.
    if (n <= 0) return;
    if (tau == 0.0f) {
        for (int i = 0; i < n; ++i) out[i] = 0.0f;
        out[0] = 1.0f;
        return;
    }
    tau = sanitize_tau(tau);
    double mx = -INFINITY;
    for (int i = 0; i < n; ++i) mx = std::fmax(mx, (double)scores[i]);
    double sum = 0.0, c = 0.0;
    double e[kMaxK > 64 ? kMaxK : 64];
    std::vector<double> big;
    double* ex = e;
    if (n > 64) { big.resize(n); ex = big.data(); }
    for (int i = 0; i < n; ++i) {
        const double v = std::exp(((double)scores[i] - mx) / (double)tau);
        const double y = v - c;  // Kahan summation
        const double t = sum + y;
        c = (t - sum) - y;
        sum = t;
        ex[i] = v;
    }
    if (sum == 0.0) {
        const float u = 1.0f / (float)n;
        for (int i = 0; i < n; ++i) out[i] = u;
    } else {
        for (int i = 0; i < n; ++i) out[i] = (float)(ex[i] / sum);
    }
}

int oracle_route_batch(const float* priors, const uint64_t* stable_ids,
                       const float* version_weights, const uint8_t* allowed,
                       uint32_t T, uint32_t N, uint32_t k, float tau, float eps,
                       float routing_bias, const uint32_t* positions,
                       oracle_ring* rings, float* entropy, int32_t* status, int n_threads) {
    if (!priors || !stable_ids || !rings) return ORACLE_ERR_INVALID;
    k = sanitize_k(k);
    tau = sanitize_tau(tau);
    eps = sanitize_eps(eps);
    // set_routing_bias keeps the default 1.0 for non-finite or non-positive values (router.rs:556-561).
    if (!(std::isfinite(routing_bias) && routing_bias > 0.0f)) routing_bias = 1.0f;
    int err = 0;
    const int nt = threads_or_default(n_threads);
#pragma omp parallel for num_threads(nt) schedule(static) reduction(| : err)
    for (int64_t t = 0; t < (int64_t)T; ++t) {
        float ent = 0.0f;
        int st = route_one(priors + (size_t)t * N, stable_ids, version_weights, allowed, N, k,
                           tau, eps, routing_bias, &rings[t], &ent);
        rings[t].position = positions ? positions[t] : 0u;
        if (entropy) entropy[t] = ent;
        if (status) status[t] = st;
        if (st != 0) err |= 1;
    }
    return err ? ORACLE_ERR_NONFINITE : ORACLE_OK;
}

int oracle_lora_op_f32(const float* x, uint32_t T, uint32_t in_dim, uint32_t out_dim,
                       const float* W, const float* A, const float* B, uint32_t n_adapters,
                       uint32_t rank, const float* alpha, const oracle_ring* rings, float* y,
                       int n_threads) {
    if (!x || !W || !A || !B || !rings || !y || rank == 0) return ORACLE_ERR_INVALID;
    const int nt = threads_or_default(n_threads);
#pragma omp parallel for num_threads(nt) schedule(static)
    for (int64_t t = 0; t < (int64_t)T; ++t) {
        const float* xt = x + (size_t)t * in_dim;
        float* yt = y + (size_t)t * out_dim;
        // Base: output[i] += W[i, j] * x[j] (kernel_testing.rs:232-237).
        for (uint32_t i = 0; i < out_dim; ++i) {
            float o = 0.0f;
            const float* w = W + (size_t)i * in_dim;
            for (uint32_t j = 0; j < in_dim; ++j) o += w[j] * xt[j];
            yt[i] = o;
        }
        // Adapter loop in ring order (liquid.rs:222-250), skipping q15 <= 0
        // (mlx-ffi/src/backend.rs:405-418); coeff = q15 / 32767.
        std::vector<float> inter(rank);
        const oracle_ring& r = rings[t];
        for (uint32_t s = 0; s < r.top_k && s < kMaxK; ++s) {
            const int16_t q = r.gates_q15[s];
            if (q <= 0) continue;
            const uint32_t a = r.indices[s];
            if (a >= n_adapters) continue;
            const float coeff = (float)q / kQ15Denom;
            const float scaling = (alpha ? alpha[a] : (float)rank) / (float)rank;
            const float* Aa = A + (size_t)a * rank * in_dim;
            const float* Ba = B + (size_t)a * out_dim * rank;
            for (uint32_t rr = 0; rr < rank; ++rr) {
                float acc = 0.0f;
                for (uint32_t c = 0; c < in_dim; ++c) acc += Aa[(size_t)rr * in_dim + c] * xt[c];
                inter[rr] = acc;
            }
            for (uint32_t i = 0; i < out_dim; ++i) {
                float acc = 0.0f;
                for (uint32_t rr = 0; rr < rank; ++rr) acc += Ba[(size_t)i * rank + rr] * inter[rr];
                yt[i] += coeff * acc * scaling;
            }
        }
    }
    return ORACLE_OK;
}

int oracle_liquid_blend_f32(const float* x, uint32_t in_dim, uint32_t out_dim,
                            uint32_t n_adapters, const float* const* A, const float* const* B,
                            const uint32_t* rank, const uint32_t* b_rows, const float* alpha,
                            const float* coeff, float* y) {
    // liquid.rs:164-219: validation (LIQUID_MAX_ADAPTERS = 3).
    if (n_adapters == 0 || n_adapters > 3) return ORACLE_ERR_INVALID;
    for (uint32_t a = 0; a < n_adapters; ++a)
        if (b_rows[a] > out_dim || rank[a] == 0) return ORACLE_ERR_INVALID;
    for (uint32_t i = 0; i < out_dim; ++i) y[i] = 0.0f;  // output.fill(0.0)
    for (uint32_t a = 0; a < n_adapters; ++a) {
        const float c = coeff[a];
        if (c == 0.0f) continue;
        const uint32_t r = rank[a];
        const float scaling = alpha[a] / (float)r;
        std::vector<float> rank_buf(r);
        for (uint32_t rr = 0; rr < r; ++rr) {
            float acc = 0.0f;
            for (uint32_t cc = 0; cc < in_dim; ++cc) acc += A[a][(size_t)rr * in_dim + cc] * x[cc];
            rank_buf[rr] = acc;
        }
        for (uint32_t o = 0; o < b_rows[a]; ++o) {
            float acc = 0.0f;
            for (uint32_t rr = 0; rr < r; ++rr) acc += B[a][(size_t)o * r + rr] * rank_buf[rr];
            y[o] += c * acc * scaling;
        }
    }
    return ORACLE_OK;
}

void oracle_rope_table(uint32_t head_dim, float theta, uint32_t mlx_as_written, uint32_t max_pos,
                       float* table) {
    // Angles follow mlx_cpp_wrapper_real.cpp:3249-3282 (positions x inv_freq in
    // f32).  Standard form: inv_freq = 1/theta^(2i/hd); the MLX code as written
    // uses exponent -2i/hd (:3254-3255), reproduced when mlx_as_written = 1.
    const uint32_t half = head_dim / 2;
    std::vector<float> inv(half);
    for (uint32_t i = 0; i < half; ++i) {
        float e = mlx_as_written ? (-2.0f * (float)i / (float)head_dim)
                                 : (2.0f * (float)i / (float)head_dim);
        inv[i] = 1.0f / std::pow(theta, e);
    }
    for (uint32_t p = 0; p < max_pos; ++p)
        for (uint32_t i = 0; i < half; ++i) {
            float ang = (float)p * inv[i];
            table[((size_t)p * half + i) * 2 + 0] = std::cos(ang);
            table[((size_t)p * half + i) * 2 + 1] = std::sin(ang);
        }
}

int oracle_layer_step(const oracle_model* m, const oracle_adapters* ad, uint32_t layer,
                      const oracle_ring* rings, uint32_t T, oracle_kv* kv, uint16_t* hidden,
                      int rounding_mode, int n_threads) {
    if (!m || !rings || !kv || !hidden || layer >= m->n_layers) return ORACLE_ERR_INVALID;
    const int nt = threads_or_default(n_threads);
    const Dims d = dims_of(m);
    const uint32_t H = d.H, hd = d.hd, nq = d.nq, nkv = d.nkv, I = d.I;
    const uint32_t QD = nq * hd, KVD = nkv * hd, half = hd / 2;
    const uint32_t L = m->n_layers;
    std::vector<float> h(T * (size_t)H), normed(T * (size_t)H);
    for (size_t i = 0; i < (size_t)T * H; ++i) h[i] = bf(hidden[i]);

    // ---- attention block (mlx_cpp_wrapper_real.cpp:3441-3507)
    rms_norm(h.data(), m->attn_norm[layer], T, H, m->rms_eps, normed.data(), rounding_mode);
    std::vector<float> q(T * (size_t)QD), k(T * (size_t)KVD), v(T * (size_t)KVD);
    linear(m->w[ORACLE_MOD_Q][layer], normed.data(), T, H, QD, q.data(), nt);
    linear(m->w[ORACLE_MOD_K][layer], normed.data(), T, H, KVD, k.data(), nt);
    linear(m->w[ORACLE_MOD_V][layer], normed.data(), T, H, KVD, v.data(), nt);
    lora_delta(ad, layer, L, ORACLE_MOD_Q, rings, T, normed.data(), H, QD, q.data(), rounding_mode, nt);
    lora_delta(ad, layer, L, ORACLE_MOD_K, rings, T, normed.data(), H, KVD, k.data(), rounding_mode, nt);
    lora_delta(ad, layer, L, ORACLE_MOD_V, rings, T, normed.data(), H, KVD, v.data(), rounding_mode, nt);
    if (rounding_mode == 1) {
        for (auto& f : q) f = rbf(f);
        for (auto& f : k) f = rbf(f);
    }

    // RoPE, half-split rotation (mlx_cpp_wrapper_real.cpp:3270-3280).
    const uint32_t max_ctx = kv->max_blocks * kv->block_size;
    std::vector<float> inv(half);
    for (uint32_t i = 0; i < half; ++i) {
        float e = m->rope_mlx_as_written ? (-2.0f * (float)i / (float)hd) : (2.0f * (float)i / (float)hd);
        inv[i] = 1.0f / std::pow(m->rope_theta, e);
    }
    auto rope = [&](float* x, uint32_t pos) {
        for (uint32_t i = 0; i < half; ++i) {
            float ang = (float)pos * inv[i];
            float c = std::cos(ang), s = std::sin(ang);
            float x1 = x[i], x2 = x[i + half];
            float r1 = x1 * c - x2 * s;
            float r2 = x1 * s + x2 * c;
            if (rounding_mode == 1) {
                r1 = rbf(rbf(x1 * c) - rbf(x2 * s));
                r2 = rbf(rbf(x1 * s) + rbf(x2 * c));
            }
            x[i] = r1;
            x[i + half] = r2;
        }
    };
    for (uint32_t t = 0; t < T; ++t) {
        const uint32_t pos = (uint32_t)kv->ctx_lens[t];
        if (pos >= max_ctx) return ORACLE_ERR_INVALID;
        for (uint32_t hh = 0; hh < nq; ++hh) rope(&q[(size_t)t * QD + hh * hd], pos);
        for (uint32_t hh = 0; hh < nkv; ++hh) rope(&k[(size_t)t * KVD + hh * hd], pos);
        // append the new K/V to the paged cache
        const int32_t* bt = kv->block_tables + (size_t)t * kv->max_blocks;
        const int32_t blk = bt[pos / kv->block_size];
        const uint32_t off = pos % kv->block_size;
        for (uint32_t hh = 0; hh < nkv; ++hh) {
            const size_t base = kv_index(kv, nkv, hd, layer, blk, hh, off);
            for (uint32_t j = 0; j < hd; ++j) {
                kv->k_pool[base + j] = to_bf(k[(size_t)t * KVD + hh * hd + j]);
                kv->v_pool[base + j] = to_bf(v[(size_t)t * KVD + hh * hd + j]);
            }
        }
    }
    for (auto& f : q) f = rbf(f);

    // Attention over the cache (mlx_cpp_wrapper_real.cpp:3284-3324): GQA head
    // map h -> h / (nq/nkv), scale 1/sqrt(hd), softmax over positions 0..pos.
    std::vector<float> attn(T * (size_t)QD);
    const float scale = 1.0f / std::sqrt((float)hd);
    const uint32_t rep = nq / nkv;
#pragma omp parallel for num_threads(nt) schedule(dynamic, 1) collapse(2)
    for (int64_t t = 0; t < (int64_t)T; ++t) {
        for (int64_t hh = 0; hh < (int64_t)nq; ++hh) {
            const uint32_t pos = (uint32_t)kv->ctx_lens[t];
            const uint32_t n = pos + 1;
            const uint32_t kvh = (uint32_t)hh / rep;
            const int32_t* bt = kv->block_tables + (size_t)t * kv->max_blocks;
            const float* qv = &q[(size_t)t * QD + hh * hd];
            std::vector<double> sc(n);
            double mx = -INFINITY;
            for (uint32_t j = 0; j < n; ++j) {
                const size_t base = kv_index(kv, nkv, hd, layer, bt[j / kv->block_size], kvh, j % kv->block_size);
                double s = 0.0;
                for (uint32_t e = 0; e < hd; ++e) s += (double)qv[e] * bf(kv->k_pool[base + e]);
                float sf = (float)s * scale;
                if (rounding_mode == 1) sf = rbf(rbf((float)s) * scale);
                sc[j] = sf;
                mx = std::fmax(mx, sc[j]);
            }
            double sum = 0.0;
            for (uint32_t j = 0; j < n; ++j) { sc[j] = std::exp(sc[j] - mx); sum += sc[j]; }
            std::vector<double> o(hd, 0.0);
            for (uint32_t j = 0; j < n; ++j) {
                const size_t base = kv_index(kv, nkv, hd, layer, bt[j / kv->block_size], kvh, j % kv->block_size);
                double p = sc[j] / sum;
                if (rounding_mode == 1) p = rbf((float)p);
                for (uint32_t e = 0; e < hd; ++e) o[e] += p * bf(kv->v_pool[base + e]);
            }
            for (uint32_t e = 0; e < hd; ++e) attn[(size_t)t * QD + hh * hd + e] = rbf((float)o[e]);
        }
    }

    // o_proj + LoRA(o) on attn_raw, residual (mlx_cpp_wrapper_real.cpp:3499-3505).
    std::vector<float> o(T * (size_t)H);
    linear(m->w[ORACLE_MOD_O][layer], attn.data(), T, QD, H, o.data(), nt);
    lora_delta(ad, layer, L, ORACLE_MOD_O, rings, T, attn.data(), QD, H, o.data(), rounding_mode, nt);
    for (size_t i = 0; i < (size_t)T * H; ++i)
        h[i] = rounding_mode == 1 ? rbf(h[i] + rbf(o[i])) : rbf(h[i] + o[i]);

    // MLP block (mlx_cpp_wrapper_real.cpp:3507-3531).
    rms_norm(h.data(), m->mlp_norm[layer], T, H, m->rms_eps, normed.data(), rounding_mode);
    std::vector<float> g(T * (size_t)I), u(T * (size_t)I);
    linear(m->w[ORACLE_MOD_GATE][layer], normed.data(), T, H, I, g.data(), nt);
    linear(m->w[ORACLE_MOD_UP][layer], normed.data(), T, H, I, u.data(), nt);
    lora_delta(ad, layer, L, ORACLE_MOD_GATE, rings, T, normed.data(), H, I, g.data(), rounding_mode, nt);
    lora_delta(ad, layer, L, ORACLE_MOD_UP, rings, T, normed.data(), H, I, u.data(), rounding_mode, nt);
    std::vector<float> act(T * (size_t)I);
    for (size_t i = 0; i < (size_t)T * I; ++i) {
        float gg = g[i], uu = u[i];
        if (rounding_mode == 1) { gg = rbf(gg); uu = rbf(uu); }
        act[i] = silu_mul(gg, uu, rounding_mode);
    }
    std::vector<float> dn(T * (size_t)H);
    linear(m->w[ORACLE_MOD_DOWN][layer], act.data(), T, I, H, dn.data(), nt);
    lora_delta(ad, layer, L, ORACLE_MOD_DOWN, rings, T, act.data(), I, H, dn.data(), rounding_mode, nt);
    for (size_t i = 0; i < (size_t)T * H; ++i)
        h[i] = rounding_mode == 1 ? rbf(h[i] + rbf(dn[i])) : rbf(h[i] + dn[i]);

    for (size_t i = 0; i < (size_t)T * H; ++i) hidden[i] = to_bf(h[i]);
    return ORACLE_OK;
}

int oracle_decode_step(const oracle_model* m, const oracle_adapters* ad, const oracle_ring* rings,
                       const int32_t* token_ids, uint32_t T, oracle_kv* kv, uint32_t n_layers_run,
                       int rounding_mode, float* logits, uint16_t* hidden_out, int n_threads) {
    if (!m || !m->embed || !token_ids) return ORACLE_ERR_INVALID;
    const int nt = threads_or_default(n_threads);
    const uint32_t H = m->hidden, V = m->vocab;
    std::vector<uint16_t> hidden((size_t)T * H, 0);
    // Embedding gather; out-of-vocabulary ids give zeros
    // (metal/src/kernels/adapteros_kernels.metal:195-234).
    for (uint32_t t = 0; t < T; ++t) {
        if (token_ids[t] < 0 || (uint32_t)token_ids[t] >= V) continue;
        std::memcpy(&hidden[(size_t)t * H], m->embed + (size_t)token_ids[t] * H, H * 2);
    }
    if (n_layers_run > m->n_layers) n_layers_run = m->n_layers;
    for (uint32_t l = 0; l < n_layers_run; ++l) {
        int st = oracle_layer_step(m, ad, l, rings, T, kv, hidden.data(), rounding_mode, nt);
        if (st) return st;
    }
    if (hidden_out) std::memcpy(hidden_out, hidden.data(), hidden.size() * 2);
    if (logits && m->lm_head && m->final_norm) {
        // Final RMSNorm + lm_head (mlx_cpp_wrapper_real.cpp:3534-3545).
        std::vector<float> h(hidden.size()), hn(hidden.size());
        for (size_t i = 0; i < hidden.size(); ++i) h[i] = bf(hidden[i]);
        rms_norm(h.data(), m->final_norm, T, H, m->rms_eps, hn.data(), rounding_mode);
        linear(m->lm_head, hn.data(), T, H, V, logits, nt);
    }
    return ORACLE_OK;
}

}  // extern "C"
