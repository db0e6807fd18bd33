// sample.cu — next-token sampling on the GPU, one CTA per sequence.
//
// Restates Generator::next_token / greedy (crates/adapteros-lora-worker/src/
// generation.rs:326-480) so that the chosen token is the reference's, given
// the same logits and the same uniform draw u:
//   * scaled = logit / temperature when temperature != 1.0 (f32 division);
//   * softmax: max by a left fold of max_by(partial_cmp, NaN -> Equal), exp
//     of (scaled - max) in f32, the sum as a sequential f32 left fold, then
//     e / sum;
//   * top_k: stable sort by probability descending (ties keep index order),
//     keep the first k, renormalise by the sum of the kept values in index
//     order (only when that sum > 0);
//   * top_p: stable sort of those values descending, running f32 sum in
//     sorted order, keep the elements up to the first one at which the sum
//     reaches p (all of them when it never does), renormalise as above;
//   * draw: the sum of the final values in index order; if it is <= 0 (or
//     not > 0) the fallback is the max_by fold's index, else the first index
//     whose running sum (index order) is >= u, else the last index.
//   * greedy: the max_by fold's index over the raw logits.
// The sequential f32 sums are sequential here too (thread 0 of the CTA); a
// running sum in the sampler's order cannot be reassociated without changing
// its rounding.  The sample sum and the cumulative draw are one pass: both
// are the same running sum.  The fold max_by keeps the later element on a tie
// and on any NaN comparison, so it equals: the element after the last NaN
// onwards, maximum with ties to the last index (or the last element if it is
// NaN).  exp is computed as the f32 rounding of the double-precision exp,
// which is the correctly rounded f32 exp except within one double ulp of a
// rounding boundary; the reference's f32::exp is the platform libm expf.
//
// Selection (top-k, and top-p's sorted order) works on 64-bit keys
// (value bits << 32 | ~index): the values are >= 0, so the key order is the
// stable descending order.  Keys are taken in chunks of kChunk: a radix
// select over the value bits among keys below the previous chunk's last key
// finds the threshold, an ordered block scan takes the ties in index order,
// and a bitonic sort in shared memory orders the chunk.

#include <cmath>

#include "common.cuh"

namespace aos {

struct SampleCfg {
    float temperature;
    int top_k;
    float top_p;
    int greedy, has_top_k, has_top_p;
};

namespace {

constexpr int kThreads = 1024;
constexpr int kChunk = 2048;
constexpr int kStage = 4096;  // values staged in shared memory for a sequential fold

struct SampleSmem {
    float stage[kStage];
    unsigned long long cand[kChunk];
    unsigned int hist[256];
    int scan[kThreads];
    float fval;
    int ival;
    unsigned long long kval;
    unsigned int n_cand;
    unsigned int need;
    unsigned int prefix;
};

__device__ __forceinline__ float exp_f32(float x) { return (float)exp((double)x); }

__device__ __forceinline__ unsigned long long key_of(float v, int i) {
    return ((unsigned long long)__float_as_uint(v) << 32) | (unsigned long long)(0xFFFFFFFFu - (unsigned)i);
}

// block-wide reductions (kThreads threads)
__device__ int block_max_int(int v, SampleSmem& sm) {
    for (int o = 16; o; o >>= 1) v = max(v, __shfl_xor_sync(0xffffffffu, v, o));
    __syncthreads();
    if ((threadIdx.x & 31) == 0) sm.scan[threadIdx.x >> 5] = v;
    __syncthreads();
    if (threadIdx.x < 32) {
        int w = sm.scan[threadIdx.x];
        for (int o = 16; o; o >>= 1) w = max(w, __shfl_xor_sync(0xffffffffu, w, o));
        if (threadIdx.x == 0) sm.ival = w;
    }
    __syncthreads();
    return sm.ival;
}

// max_by fold over x[0..n): index of the result (see the file comment)
__device__ int fold_argmax(const float* x, int n, SampleSmem& sm) {
    int last_nan = -1;
    for (int i = threadIdx.x; i < n; i += kThreads)
        if (isnan(x[i])) last_nan = i;
    last_nan = block_max_int(last_nan, sm);
    if (last_nan == n - 1) return n - 1;
    const int lo = last_nan + 1;
    // maximum value over [lo, n), then the last index holding it
    float best = -INFINITY;
    for (int i = lo + threadIdx.x; i < n; i += kThreads) best = fmaxf(best, x[i]);
    for (int o = 16; o; o >>= 1) best = fmaxf(best, __shfl_xor_sync(0xffffffffu, best, o));
    __syncthreads();
    if ((threadIdx.x & 31) == 0) sm.scan[threadIdx.x >> 5] = __float_as_int(best);
    __syncthreads();
    if (threadIdx.x == 0) {
        float b = __int_as_float(sm.scan[0]);
        for (int w = 1; w < kThreads / 32; ++w) b = fmaxf(b, __int_as_float(sm.scan[w]));
        sm.fval = b;
    }
    __syncthreads();
    const float m = sm.fval;
    int at = lo;  // all -inf: every element ties, the last one wins
    for (int i = lo + threadIdx.x; i < n; i += kThreads)
        if (x[i] == m) at = max(at, i);
    at = block_max_int(at, sm);
    if (m == -INFINITY) return n - 1;
    return at;
}

// Ordered compaction: list[0..count) = indices i (ascending) with pred(i).
template <class Pred>
__device__ int compact(int n, int* list, SampleSmem& sm, Pred pred) {
    const int per = (n + kThreads - 1) / kThreads;
    const int b = threadIdx.x * per, e = min(n, b + per);
    int cnt = 0;
    for (int i = b; i < e; ++i) cnt += pred(i) ? 1 : 0;
    __syncthreads();
    sm.scan[threadIdx.x] = cnt;
    __syncthreads();
    if (threadIdx.x == 0) {
        int run = 0;
        for (int t = 0; t < kThreads; ++t) {
            const int c = sm.scan[t];
            sm.scan[t] = run;
            run += c;
        }
        sm.ival = run;
    }
    __syncthreads();
    int at = sm.scan[threadIdx.x];
    for (int i = b; i < e; ++i)
        if (pred(i)) list[at++] = i;
    __syncthreads();
    return sm.ival;
}

// The next up-to-kChunk keys of v[0..n) below `below`, sorted descending into
// sm.cand[0..count).  Returns count.
__device__ int next_chunk(const float* v, int n, unsigned long long below, int remaining, SampleSmem& sm) {
    const int want = min(kChunk, remaining);
    if (want <= 0) return 0;
    if (threadIdx.x == 0) {
        sm.need = (unsigned)want;
        sm.prefix = 0;
    }
    __syncthreads();
    unsigned mask = 0;
    for (int shift = 24; shift >= 0; shift -= 8) {
        for (int i = threadIdx.x; i < 256; i += kThreads) sm.hist[i] = 0;
        __syncthreads();
        const unsigned prefix = sm.prefix;
        for (int i = threadIdx.x; i < n; i += kThreads) {
            const unsigned bits = __float_as_uint(v[i]);
            if (key_of(v[i], i) < below && (bits & mask) == prefix) atomicAdd(&sm.hist[(bits >> shift) & 255], 1u);
        }
        __syncthreads();
        if (threadIdx.x == 0) {
            unsigned above = 0, need = sm.need;
            int bin = 255;
            for (; bin > 0; --bin) {
                if (above + sm.hist[bin] >= need) break;
                above += sm.hist[bin];
            }
            sm.prefix = prefix | ((unsigned)bin << shift);
            sm.need = need - above;
        }
        mask |= 255u << shift;
        __syncthreads();
    }
    const unsigned t = sm.prefix, take_ties = sm.need;
    // everything strictly above t, plus the first take_ties elements equal to t (index order)
    if (threadIdx.x == 0) sm.n_cand = 0;
    __syncthreads();
    for (int i = threadIdx.x; i < n; i += kThreads) {
        const unsigned bits = __float_as_uint(v[i]);
        if (bits > t && key_of(v[i], i) < below) sm.cand[atomicAdd(&sm.n_cand, 1u)] = key_of(v[i], i);
    }
    {
        const int per = (n + kThreads - 1) / kThreads;
        const int b = threadIdx.x * per, e = min(n, b + per);
        int cnt = 0;
        for (int i = b; i < e; ++i) cnt += (__float_as_uint(v[i]) == t && key_of(v[i], i) < below) ? 1 : 0;
        __syncthreads();
        sm.scan[threadIdx.x] = cnt;
        __syncthreads();
        if (threadIdx.x == 0) {
            int run = 0;
            for (int q = 0; q < kThreads; ++q) {
                const int c = sm.scan[q];
                sm.scan[q] = run;
                run += c;
            }
        }
        __syncthreads();
        int rank = sm.scan[threadIdx.x];
        for (int i = b; i < e && rank < (int)take_ties; ++i)
            if (__float_as_uint(v[i]) == t && key_of(v[i], i) < below) {
                sm.cand[atomicAdd(&sm.n_cand, 1u)] = key_of(v[i], i);
                ++rank;
            }
    }
    __syncthreads();
    const int count = (int)sm.n_cand;
    int pow2 = 1;
    while (pow2 < count) pow2 <<= 1;
    for (int i = count + threadIdx.x; i < pow2; i += kThreads) sm.cand[i] = 0ull;
    __syncthreads();
    for (int size = 2; size <= pow2; size <<= 1)
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            for (int i = threadIdx.x; i < pow2; i += kThreads) {
                const int j = i ^ stride;
                if (j > i) {
                    const bool desc = (i & size) == 0;
                    const unsigned long long a = sm.cand[i], c = sm.cand[j];
                    if (desc ? (a < c) : (a > c)) {
                        sm.cand[i] = c;
                        sm.cand[j] = a;
                    }
                }
            }
            __syncthreads();
        }
    return count;
}

// the key of the k-th largest element (1-based) of v[0..n)
__device__ unsigned long long kth_key(const float* v, int n, int k, SampleSmem& sm) {
    unsigned long long below = ~0ull;
    int taken = 0;
    while (true) {
        const int c = next_chunk(v, n, below, n - taken, sm);
        if (c == 0) return 0ull;  // not reached for k <= n: keeps everything
        if (taken + c >= k) return sm.cand[k - taken - 1];
        taken += c;
        below = sm.cand[c - 1];
        __syncthreads();
    }
}

// Sequential f32 left fold of get(0), get(1), ... get(m - 1), by thread 0
// out of shared memory: the CTA stages kStage values at a time with parallel
// loads, then thread 0 adds them in order (float4 reads keep the add chain,
// not the loads, on the critical path).  With u_pick, also the first q at
// which u <= running sum (-1 if none).  Every thread returns the sum.
template <class Get>
__device__ float seq_fold(int m, Get get, SampleSmem& sm, bool want_pick = false, float u = 0.0f,
                          int* pick_q = nullptr) {
    float run = 0.0f;
    int pick = -1;
    for (int base = 0; base < m; base += kStage) {
        const int n = min(kStage, m - base);
        for (int q = threadIdx.x; q < n; q += kThreads) sm.stage[q] = get(base + q);
        for (int q = n + threadIdx.x; q < ((n + 3) & ~3); q += kThreads) sm.stage[q] = 0.0f;
        __syncthreads();
        if (threadIdx.x == 0) {
            const float4* s4 = reinterpret_cast<const float4*>(sm.stage);
            if (!want_pick || pick >= 0) {
                const int n4 = n / 4;
                for (int q = 0; q < n4; ++q) {
                    const float4 w = s4[q];
                    run += w.x;
                    run += w.y;
                    run += w.z;
                    run += w.w;
                }
                for (int q = n4 * 4; q < n; ++q) run += sm.stage[q];
            } else {  // four adds per step; the compares sit beside the add chain
                const int n4 = (n + 3) / 4;  // the padding zeros do not move the sum
                for (int q = 0; q < n4; ++q) {
                    const float4 w = s4[q];
                    const float r1 = run + w.x, r2 = r1 + w.y, r3 = r2 + w.z, r4 = r3 + w.w;
                    if (pick < 0 && (u <= r1 || u <= r2 || u <= r3 || u <= r4)) {
                        const int k = u <= r1 ? 0 : u <= r2 ? 1 : u <= r3 ? 2 : 3;
                        if (4 * q + k < n) pick = base + 4 * q + k;
                    }
                    run = r4;
                }
            }
            sm.fval = run;
            sm.ival = pick;
        }
        __syncthreads();
        run = sm.fval;
        pick = sm.ival;
        __syncthreads();
    }
    if (pick_q) *pick_q = pick;
    return run;
}

__global__ void __launch_bounds__(kThreads) sample_kernel(const float* __restrict__ logits, int V, long long ld,
                                                          SampleCfg cfg, const float* __restrict__ u,
                                                          float* __restrict__ work, int* __restrict__ lists,
                                                          uint32_t* __restrict__ out) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    SampleSmem& sm = *reinterpret_cast<SampleSmem*>(smem_raw);
    const int t = blockIdx.x;
    const float* x = logits + (size_t)t * ld;
    float* v = work + (size_t)t * V;
    int* list = lists + (size_t)t * V;
    if (cfg.greedy) {
        const int i = fold_argmax(x, V, sm);
        if (threadIdx.x == 0) out[t] = (uint32_t)i;
        return;
    }
    // temperature, softmax max, exp
    for (int i = threadIdx.x; i < V; i += kThreads) v[i] = cfg.temperature != 1.0f ? __fdiv_rn(x[i], cfg.temperature) : x[i];
    __syncthreads();
    const int im = fold_argmax(v, V, sm);
    const float m = v[im];
    __syncthreads();
    for (int i = threadIdx.x; i < V; i += kThreads) v[i] = exp_f32(v[i] - m);
    __syncthreads();
    const float sum = seq_fold(V, [&](int i) { return v[i]; }, sm);
    for (int i = threadIdx.x; i < V; i += kThreads) v[i] = __fdiv_rn(v[i], sum);
    __syncthreads();
    // kept set so far: all (cut = 0 keeps every key)
    unsigned long long cut = 0ull;
    if (cfg.has_top_k && cfg.top_k < V) {
        cut = cfg.top_k > 0 ? kth_key(v, V, cfg.top_k, sm) : ~0ull;
        __syncthreads();
        const int nk = compact(V, list, sm, [&](int i) { return key_of(v[i], i) >= cut; });
        const float s2 = seq_fold(nk, [&](int q) { return v[list[q]]; }, sm);
        for (int i = threadIdx.x; i < V; i += kThreads) {
            const bool keep = key_of(v[i], i) >= cut;
            v[i] = keep ? (s2 > 0.0f ? __fdiv_rn(v[i], s2) : v[i]) : 0.0f;
        }
        __syncthreads();
    } else if (cfg.has_top_k) {  // k >= V keeps everything; the renormalisation still runs
        const int nk = compact(V, list, sm, [&](int i) { return true; });
        const float s2 = seq_fold(nk, [&](int q) { return v[list[q]]; }, sm);
        if (s2 > 0.0f)
            for (int i = threadIdx.x; i < V; i += kThreads) v[i] = __fdiv_rn(v[i], s2);
        __syncthreads();
    }
    if (cfg.has_top_p) {
        // running sum in key order until it reaches p; the cut key is that element's
        unsigned long long below = ~0ull, pcut = 0ull;
        int taken = 0;
        bool found = false;
        while (!found && taken < V) {
            const int c = next_chunk(v, V, below, V - taken, sm);
            if (threadIdx.x == 0) {
                float run = sm.fval;
                if (taken == 0) run = 0.0f;
                int hit = -1;
                for (int q = 0; q < c; ++q) {
                    run += __uint_as_float((unsigned)(sm.cand[q] >> 32));
                    if (run >= cfg.top_p) {
                        hit = q;
                        break;
                    }
                }
                sm.fval = run;
                sm.ival = hit;
                // the rest are zeros when this chunk ended in a zero: the sum cannot grow
                sm.prefix = (hit < 0 && (c == 0 || (unsigned)(sm.cand[c - 1] >> 32) == 0u)) ? 1u : 0u;
            }
            __syncthreads();
            const int hit = sm.ival;
            if (hit >= 0) {
                pcut = sm.cand[hit];
                found = true;
            } else if (sm.prefix) {
                break;  // never reaches p: keep all
            }
            taken += c;
            below = c ? sm.cand[c - 1] : 0ull;
            __syncthreads();
        }
        if (found) {
            const int nk = compact(V, list, sm, [&](int i) { return key_of(v[i], i) >= pcut; });
            const float s3 = seq_fold(nk, [&](int q) { return v[list[q]]; }, sm);
            for (int i = threadIdx.x; i < V; i += kThreads) {
                const bool keep = key_of(v[i], i) >= pcut;
                v[i] = keep ? (s3 > 0.0f ? __fdiv_rn(v[i], s3) : v[i]) : 0.0f;
            }
        } else {  // all kept: renormalise by the full sum (index order)
            const int nk = compact(V, list, sm, [&](int i) { return true; });
            const float s3 = seq_fold(nk, [&](int q) { return v[list[q]]; }, sm);
            if (s3 > 0.0f)
                for (int i = threadIdx.x; i < V; i += kThreads) v[i] = __fdiv_rn(v[i], s3);
        }
        __syncthreads();
    }
    // draw: one running sum in index order over the non-zero values
    const int nz = compact(V, list, sm, [&](int i) { return v[i] != 0.0f; });
    const float r = u[t];
    int pick_q = -1;
    const float total = seq_fold(nz, [&](int q) { return v[list[q]]; }, sm, true, r, &pick_q);
    // zeros never move the running sum, so they can only be picked before the
    // first non-zero value, and only by r <= 0
    int pick = (r <= 0.0f && v[0] == 0.0f) ? 0 : (pick_q >= 0 ? list[pick_q] : -1);
    if (total <= 0.0f) {
        pick = fold_argmax(v, V, sm);  // degenerate distribution
    } else if (pick < 0) {
        pick = V - 1;  // never reached u (or a NaN sum)
    }
    if (threadIdx.x == 0) out[t] = (uint32_t)pick;
}

}  // namespace

size_t sample_smem_bytes() { return sizeof(SampleSmem); }

cudaError_t launch_sample(const float* logits, int T, int V, long long ld, const SampleCfg& cfg, const float* u,
                          float* work, int* lists, uint32_t* out, cudaStream_t s) {
    if (T <= 0) return cudaSuccess;
    cudaError_t e = cudaFuncSetAttribute(sample_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)sizeof(SampleSmem));
    if (e != cudaSuccess) return e;
    sample_kernel<<<T, kThreads, sizeof(SampleSmem), s>>>(logits, V, ld, cfg, u, work, lists, out);
    return cudaGetLastError();
}

}  // namespace aos

using namespace aos;

extern "C" int aos_sample_dev(const float* logits, uint32_t T, uint32_t V, uint64_t ld, const aos_sample_params* p,
                              const float* u, uint32_t* tokens, void* stream) {
    if (!p || (T && (!logits || !tokens)) || V == 0 || V > 0x7FFFFFFFu || ld < V) {
        set_global_error("aos_sample_dev: bad arguments (V >= 1, ld >= V, pointers)");
        return AOS_ERR_INVALID;
    }
    const bool greedy = (p->flags & AOS_SAMPLE_GREEDY) != 0;
    if (!greedy && (!u || !(p->temperature > 0.0f) || !std::isfinite(p->temperature))) {
        set_global_error("aos_sample_dev: sampling needs u[T] and a finite temperature > 0");
        return AOS_ERR_INVALID;
    }
    if (T == 0) return AOS_OK;
    int rc = require_device();
    if (rc) return rc;
    SampleCfg cfg;
    cfg.temperature = p->temperature;
    cfg.top_k = (int)std::min<uint32_t>(p->top_k, 0x7FFFFFFFu);
    cfg.top_p = p->top_p;
    cfg.greedy = greedy ? 1 : 0;
    cfg.has_top_k = (p->flags & AOS_SAMPLE_TOP_K) ? 1 : 0;
    cfg.has_top_p = (p->flags & AOS_SAMPLE_TOP_P) ? 1 : 0;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    float* work = nullptr;
    int* lists = nullptr;
    if (!greedy) {
        AOS_RETURN_IF_CUDA(cudaMallocAsync((void**)&work, (size_t)T * V * sizeof(float), s), set_global_error);
        AOS_RETURN_IF_CUDA(cudaMallocAsync((void**)&lists, (size_t)T * V * sizeof(int), s), set_global_error);
    }
    const cudaError_t e = launch_sample(logits, (int)T, (int)V, (long long)ld, cfg, u, work, lists, tokens, s);
    if (work) cudaFreeAsync(work, s);
    if (lists) cudaFreeAsync(lists, s);
    AOS_RETURN_IF_CUDA(e, set_global_error);
    return AOS_OK;
}
