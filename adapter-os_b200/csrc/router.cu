// router.cu — batched K-sparse router, one warp per token.
//
// Restates Router::route_with_adapter_info_and_scope_with_ctx
// (crates/adapteros-lora-router/src/router.rs:1567-1952) for a batch of tokens,
// bit-exact with the reference:
//   score   = ((prior + 0.0) - 0.0) * bias * clamp(version_weight, 0, 2)  (:1632-1690)
//   order   = f32::total_cmp DESC, stable_id ASC, index ASC             (:234-264)
//   softmax = f64, Kahan-summed in slot order, (e/sum) as f32           (:1340-1411)
//   floor   = max(g, eps/K), f32 sequential renormalise                 (:1818-1842)
//   q15     = clamp(round_half_away(g * 32767), 0, 32767)               (quantization.rs:172-175)
//   ring    = (q15 DESC, score DESC, stable_id ASC, idx ASC)            (:1310-1325)
// Every float/double op is an explicit round-to-nearest intrinsic so nvcc
// cannot contract or reorder it.
//
// Top-K: each lane scans a strided slice of the N adapters keeping its own
// sorted best-K list in registers, then K rounds of a warp-shuffle argmax over
// the lanes' list heads pick the global order.

#include "common.cuh"

namespace aos {
namespace {

constexpr int kK = AOS_MAX_K;

struct Cand {
    float score;
    uint32_t idx;
    uint64_t sid;
};

// a strictly before b in the sort_scores_deterministic order.
__device__ __forceinline__ bool before(float sa, uint64_t ida, uint32_t ia, float sb, uint64_t idb,
                                       uint32_t ib) {
    const int32_t ka = total_key(sa), kb = total_key(sb);
    if (ka != kb) return ka > kb;
    if (ida != idb) return ida < idb;
    return ia < ib;
}

__global__ void __launch_bounds__(256) route_kernel(
    const float* __restrict__ priors, const uint64_t* __restrict__ stable_ids,
    const float* __restrict__ version_weights, const uint8_t* __restrict__ allowed,
    const uint32_t* __restrict__ positions, int T, int N, int k, float tau, float eps, float bias,
    aos_router_ring* __restrict__ rings, float* __restrict__ entropy_out,
    int32_t* __restrict__ status_out) {
    const int warp = (int)((blockIdx.x * blockDim.x + threadIdx.x) >> 5);
    const int lane = threadIdx.x & 31;
    if (warp >= T) return;
    const float* p = priors + (size_t)warp * N;

    // ---- pass over the adapters: validate, score, keep the lane's best k.
    Cand best[kK];
    int nbest = 0;
    bool bad = false;
    int n_allowed = 0;
    for (int i = lane; i < N; i += 32) {
        const float prior = __ldg(p + i);
        if (!isfinite(prior)) bad = true;  // validate_router_inputs (:611-625)
        if (allowed && !__ldg(allowed + i)) continue;
        float s = __fsub_rn(__fadd_rn(prior, 0.0f), 0.0f);  // prior + feature(0) - penalty(0)
        s = __fmul_rn(s, bias);
        float w = 1.0f;
        if (version_weights) {
            w = __ldg(version_weights + i);
            w = isfinite(w) ? (w < 0.0f ? 0.0f : (w > 2.0f ? 2.0f : w)) : 1.0f;  // f32::clamp
        }
        s = __fmul_rn(s, w);
        if (!isfinite(s)) bad = true;
        ++n_allowed;
        const uint64_t sid = __ldg(stable_ids + i);
        // insertion into the sorted local list (length <= k)
        if (nbest < k || before(s, sid, (uint32_t)i, best[nbest - 1].score, best[nbest - 1].sid,
                                best[nbest - 1].idx)) {
            int j = nbest < k ? nbest++ : k - 1;
#pragma unroll 1
            while (j > 0 && before(s, sid, (uint32_t)i, best[j - 1].score, best[j - 1].sid, best[j - 1].idx)) {
                best[j] = best[j - 1];
                --j;
            }
            best[j] = Cand{s, (uint32_t)i, sid};
        }
    }
    const bool any_bad = __any_sync(0xffffffffu, bad);
    n_allowed = __reduce_add_sync(0xffffffffu, (unsigned)n_allowed);

    aos_router_ring* ring = rings + warp;
    if (any_bad || n_allowed == 0) {
        if (lane < 10) reinterpret_cast<uint32_t*>(ring)[lane] = 0u;
        if (lane == 0) {
            if (positions) ring->position = positions[warp];
            if (entropy_out) entropy_out[warp] = 0.0f;
            if (status_out) status_out[warp] = any_bad ? AOS_ERR_NONFINITE : AOS_OK;
        }
        return;
    }

    // ---- K rounds of warp argmax over list heads -> global top-n in order.
    const int n = min(k, n_allowed);
    float top_s[kK];
    uint32_t top_i[kK];
    uint64_t top_sid[kK];
    int head = 0;
#pragma unroll 1
    for (int r = 0; r < n; ++r) {
        const bool has = head < nbest;
        float s = has ? best[head].score : 0.0f;
        uint32_t idx = has ? best[head].idx : 0xffffffffu;
        uint64_t sid = has ? best[head].sid : 0ull;
        int owner = has ? lane : 32;
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) {
            const float s2 = __shfl_xor_sync(0xffffffffu, s, off);
            const uint32_t i2 = __shfl_xor_sync(0xffffffffu, idx, off);
            const uint64_t d2 = __shfl_xor_sync(0xffffffffu, sid, off);
            const int o2 = __shfl_xor_sync(0xffffffffu, owner, off);
            bool take;
            if (o2 == 32) take = false;
            else if (owner == 32) take = true;
            else take = before(s2, d2, i2, s, sid, idx);
            if (take) { s = s2; idx = i2; sid = d2; owner = o2; }
        }
        top_s[r] = s;
        top_i[r] = idx;
        top_sid[r] = sid;
        if (owner == lane) ++head;
    }

    if (lane != 0) return;

    // ---- deterministic_softmax (:1340-1411)
    float g[kK];
    if (tau == 0.0f) {
        for (int j = 0; j < n; ++j) g[j] = j == 0 ? 1.0f : 0.0f;
    } else {
        double mx = -INFINITY;
        for (int j = 0; j < n; ++j) mx = fmax(mx, (double)top_s[j]);
        double sum = 0.0, c = 0.0;
        double e[kK];
        for (int j = 0; j < n; ++j) {
            const double v = exp(__ddiv_rn(__dsub_rn((double)top_s[j], mx), (double)tau));
            const double y = __dsub_rn(v, c);
            const double t = __dadd_rn(sum, y);
            c = __dsub_rn(__dsub_rn(t, sum), y);
            sum = t;
            e[j] = v;
        }
        if (sum == 0.0) {
            const float u = __fdiv_rn(1.0f, (float)n);
            for (int j = 0; j < n; ++j) g[j] = u;
        } else {
            for (int j = 0; j < n; ++j) g[j] = __double2float_rn(__ddiv_rn(e[j], sum));
        }
        // entropy floor (:1818-1827)
        const float min_gate = __fdiv_rn(eps, (float)n);
        for (int j = 0; j < n; ++j) g[j] = fmaxf(g[j], min_gate);
    }
    // renormalise (:1830-1842)
    float sum32 = -0.0f;
    for (int j = 0; j < n; ++j) sum32 = __fadd_rn(sum32, g[j]);
    if (!(sum32 > 0.0f)) {
        for (int w = 0; w < 10; ++w) reinterpret_cast<uint32_t*>(ring)[w] = 0u;
        if (positions) ring->position = positions[warp];
        if (entropy_out) entropy_out[warp] = 0.0f;
        if (status_out) status_out[warp] = AOS_OK;
        return;
    }
    for (int j = 0; j < n; ++j) g[j] = __fdiv_rn(g[j], sum32);

    // compute_entropy (:1287-1293); libm log2 may differ in the last ulp.
    float ent = -0.0f;
    for (int j = 0; j < n; ++j)
        if (g[j] > 0.0f) ent = __fadd_rn(ent, __fmul_rn(-g[j], log2f(g[j])));

    // quantize_gate (quantization.rs:172-175): roundf is half-away-from-zero.
    int16_t q[kK];
    for (int j = 0; j < n; ++j) {
        const float r = roundf(__fmul_rn(g[j], AOS_Q15_DENOM));
        int32_t v = isnan(r) ? 0 : (r >= 2147483648.0f ? INT32_MAX : (r < -2147483648.0f ? INT32_MIN : (int32_t)r));
        v = v < 0 ? 0 : (v > 32767 ? 32767 : v);
        q[j] = (int16_t)v;
    }
    // canonical order (:1310-1325), insertion sort over <= 8 entries.
    int ord[kK];
    for (int j = 0; j < n; ++j) ord[j] = j;
    for (int j = 1; j < n; ++j) {
        const int cur = ord[j];
        int m = j;
        while (m > 0) {
            const int prv = ord[m - 1];
            bool cur_first;
            if (q[cur] != q[prv]) cur_first = q[cur] > q[prv];
            else cur_first = before(top_s[cur], top_sid[cur], top_i[cur], top_s[prv], top_sid[prv], top_i[prv]);
            if (!cur_first) break;
            ord[m] = prv;
            --m;
        }
        ord[m] = cur;
    }
    aos_router_ring out;
    out.top_k = (uint32_t)n;
    out.position = positions ? positions[warp] : 0u;
    for (int j = 0; j < kK; ++j) {
        out.indices[j] = j < n ? (uint16_t)top_i[ord[j]] : (uint16_t)0;
        out.gates_q15[j] = j < n ? q[ord[j]] : (int16_t)0;
    }
    *ring = out;
    if (entropy_out) entropy_out[warp] = ent;
    if (status_out) status_out[warp] = AOS_OK;
}

}  // namespace

// Sanitise like Router::new_with_weights / set_routing_bias (router.rs:127-187, 556-561).
void sanitize_router_params(const aos_router_params* in, int* k, float* tau, float* eps,
                            float* bias) {
    uint32_t kk = in ? in->k : 4u;
    *k = kk == 0 ? 1 : (kk > (uint32_t)AOS_MAX_K ? AOS_MAX_K : (int)kk);
    float t = in ? in->tau : 1.0f;
    *tau = (!isfinite(t) || t <= 0.0f) ? 1.0f : t;
    float e = in ? in->eps : 0.02f;
    *eps = (!isfinite(e) || !(e >= 0.0f && e <= 1.0f)) ? 0.02f : e;
    float b = in ? in->routing_bias : 1.0f;
    *bias = (isfinite(b) && b > 0.0f) ? b : 1.0f;
}

cudaError_t launch_route(const float* priors, const uint64_t* stable_ids, const float* vw,
                         const uint8_t* allowed, const uint32_t* positions, int T, int N,
                         const aos_router_params* params, aos_router_ring* rings, float* entropy,
                         int32_t* status, cudaStream_t stream) {
    int k;
    float tau, eps, bias;
    sanitize_router_params(params, &k, &tau, &eps, &bias);
    if (T <= 0) return cudaSuccess;
    const int threads = 256, warps_per_block = threads / 32;
    const int blocks = (T + warps_per_block - 1) / warps_per_block;
    route_kernel<<<blocks, threads, 0, stream>>>(priors, stable_ids, vw, allowed, positions, T, N, k,
                                                 tau, eps, bias, rings, entropy, status);
    return cudaGetLastError();
}

}  // namespace aos
