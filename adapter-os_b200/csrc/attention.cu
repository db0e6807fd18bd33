// attention.cu — GQA decode attention over the paged bf16 KV cache.
//
// Semantics: softmax(q k^T / sqrt(hd)) v over positions 0..pos (the token's
// own K/V included), query head h reading KV head h / (n_heads / n_kv_heads)
// (mlx_cpp_wrapper_real.cpp:3284-3324; kv_cache.metal:101-183 for the decode
// form).
//
// Split-KV: one CTA per (token, kv head, chunk of 64 pages = 1024 positions);
// its 4 warps take pages round-robin.  Pages (16 positions x 128 dims) arrive
// by TMA (SWIZZLE_128B, two 64-dim boxes each for K and V) into per-warp
// double buffers; QK^T and PV run on mma.sync m16n8k16 with the query heads
// of the group as the 16 rows (FA2 register layout, so P never leaves
// registers).  Each CTA writes (m, l, O) for its chunk and counts itself in;
// the CTA that writes the last chunk of a (token, kv head) merges the chunks
// of its query heads in chunk order (no separate combine launch).  Every
// order is fixed, so results are bit-identical run to run.

#include <cuda.h>

#include "common.cuh"

namespace aos {
namespace {

constexpr int kPages = 64;          // pages per chunk
constexpr int kWarps = 4;
constexpr int kPageBytes = 16 * 128 * 2;  // one of K or V
constexpr int kBufBytes = 2 * kPageBytes;  // K + V

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait; false on timeout or when another role already failed.  The
// fast path only polls the barrier; the error word and the clock are checked
// every 1024 polls so a completed phase is seen without an extra L2 round trip.
__device__ __noinline__ bool mbar_wait_slow(uint32_t bar, uint32_t parity, int* err) {
    const long long t0 = clock64();
    uint32_t n = 0;
    while (!mbar_try(bar, parity)) {
        if ((++n & 1023u) == 0) {
            if (*(volatile int*)err != 0) return false;
            if (clock64() - t0 > kSpinLimitCycles) {
                atomicCAS(err, 0, AOS_ERR_TIMEOUT);
                return false;
            }
        }
    }
    return true;
}
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, int* err) {
#pragma unroll 1
    for (int i = 0; i < 64; ++i)
        if (mbar_try(bar, parity)) return true;
    return mbar_wait_slow(bar, parity, err);
}
// Time-bounded wait that ignores the error word: used only to drain this
// CTA's own copies / MMAs before it exits on an error path.
__device__ __noinline__ bool mbar_wait_drain(uint32_t bar, uint32_t parity) {
    const long long t0 = clock64();
    while (!mbar_try(bar, parity))
        if (clock64() - t0 > kSpinLimitCycles) return false;
    return true;
}

__device__ __forceinline__ void tma_page(const CUtensorMap* m, uint32_t dst, uint32_t bar, int row) {
#pragma unroll
    for (int h = 0; h < 2; ++h)
        asm volatile(
            "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
                dst + h * 2048),
            "l"(reinterpret_cast<uint64_t>(m)), "r"(bar), "r"(h * 64), "r"(row)
            : "memory");
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}
__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
    return (uint32_t)f2bf(lo) | ((uint32_t)f2bf(hi) << 16);
}
// Address of 16-byte chunk `chunk` (0..15 over the 128 dims) of page row p in
// the SWIZZLE_128B layout written by two 64-dim TMA boxes.
__device__ __forceinline__ uint32_t sw_addr(uint32_t base, int p, int chunk) {
    return base + (uint32_t)((chunk >> 3) * 2048 + p * 128 + (((chunk & 7) ^ (p & 7)) << 4));
}

struct AttnParams {
    CUtensorMap tm_k, tm_v;  // [rows = L*NB*nkv*16, 128] bf16
    const uint16_t* q;       // [T][nq*128]
    const int* block_tables;  // [T][max_blocks]
    const int* ctx_lens;      // [T] tokens cached before this step (new token at that position)
    float* part;              // [T][nkv][max_chunks][G][128] O, then m, l
    float* part_ml;           // [T][nkv][max_chunks][G][2]
    int* chunk_cnt;           // [T][nkv] chunks written so far (zero between launches)
    uint16_t* out;            // [T][nq*128] bf16
    int T, nq, nkv, G, layer, num_blocks, max_blocks, max_chunks;
    float scale_log2;         // log2(e) / sqrt(hd)
    int* err;
};

// Merges the chunk partials of query head row r of (token t, kv head) in
// chunk order, one warp: lane i owns dims 4i .. 4i+3; lane c holds chunk c's
// (m, l), and the running sums of l and of O are taken in chunk order, so the
// result is the same on every run whichever chunk finished last.  The
// partials were written by other CTAs of this launch: plain (coherent) loads.
__device__ __forceinline__ void combine_row(const float* __restrict__ part, const float* __restrict__ part_ml,
                                            size_t base, int G, int r, int n_chunks, int lane, uint16_t* dst) {
    float m = -INFINITY;
    for (int c = lane; c < n_chunks; c += 32) m = fmaxf(m, __ldcg(part_ml + ((base + c) * G + r) * 2));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    float l = 0.f;
    for (int c0 = 0; c0 < n_chunks; c0 += 32) {
        const int c = c0 + lane;
        float sc = 0.f, lc = 0.f;
        if (c < n_chunks) {
            const float2 ml = __ldcg(reinterpret_cast<const float2*>(part_ml) + (base + c) * G + r);
            sc = ml.x == -INFINITY ? 0.f : exp2f(ml.x - m);
            lc = ml.y;
        }
        const int nc = min(32, n_chunks - c0);
#pragma unroll 4
        for (int j = 0; j < nc; ++j) {
            const float scj = __shfl_sync(0xffffffffu, sc, j);
            l += __shfl_sync(0xffffffffu, lc, j) * scj;
            const float4 v = __ldcg(reinterpret_cast<const float4*>(part + ((base + c0 + j) * G + r) * 128) + lane);
            acc.x += v.x * scj;
            acc.y += v.y * scj;
            acc.z += v.z * scj;
            acc.w += v.w * scj;
        }
    }
    uint2 w;
    w.x = (uint32_t)f2bf(acc.x / l) | ((uint32_t)f2bf(acc.y / l) << 16);
    w.y = (uint32_t)f2bf(acc.z / l) | ((uint32_t)f2bf(acc.w / l) << 16);
    *reinterpret_cast<uint2*>(dst + lane * 4) = w;
}

__global__ void __launch_bounds__(128) attn_decode_kernel(const __grid_constant__ AttnParams p) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kWarps * 2 * kBufBytes);  // [warps][2]
    float* red = reinterpret_cast<float*>(smem);  // combine scratch, reuses the page buffers

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    int idx = blockIdx.x;
    const int chunk = idx % p.max_chunks;
    idx /= p.max_chunks;
    const int kvh = idx % p.nkv;
    const int t = idx / p.nkv;
    if (t >= p.T) return;
    const int L = __ldg(p.ctx_lens + t) + 1;
    const int n_pages = (L + 15) >> 4;
    const int pg0 = chunk * kPages;
    if (pg0 >= n_pages) return;
    const int pg1 = min(n_pages, pg0 + kPages);

    if (threadIdx.x < kWarps * 2) {
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_u32(&bars[threadIdx.x])) : "memory");
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    __syncthreads();

    const int* bt = p.block_tables + (size_t)t * p.max_blocks;
    const uint32_t buf0 = smem_u32(smem + warp * 2 * kBufBytes);
    const uint32_t bar0 = smem_u32(&bars[warp * 2]);
    auto page_row = [&](int pg) { return ((p.layer * p.num_blocks + __ldg(bt + pg)) * p.nkv + kvh) * 16; };
    auto issue = [&](int pg, int b) {
        const uint32_t bar = bar0 + b * 8, dst = buf0 + b * kBufBytes;
        asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(kBufBytes) : "memory");
        const int row = page_row(pg);
        tma_page(&p.tm_k, dst, bar, row);
        tma_page(&p.tm_v, dst + kPageBytes, bar, row);
    };

    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
    float o[16][4];
#pragma unroll
    for (int i = 0; i < 16; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;

    // Pages before the sequence's last one were written by earlier steps, so
    // the first of them may be fetched before the previous launch (the QKV
    // GEMM that appends this step's K/V) has finished.
    int my_first = pg0 + warp;
    bool first_issued = false;
    if (lane == 0 && my_first < pg1 && my_first < n_pages - 1) {
        issue(my_first, 0);
        first_issued = true;
    }
    pdl_wait();
    pdl_trigger();
    if (lane == 0 && my_first < pg1 && !first_issued) issue(my_first, 0);

    // Q fragments (rows = heads of the group, zero beyond G), all 8 k-chunks.
    const int g = lane >> 2, c2 = (lane & 3) * 2;
    uint32_t qa[8][4];
    {
        const int h0 = kvh * p.G + g, h1 = kvh * p.G + g + 8;
        const uint16_t* q0 = p.q + (size_t)t * p.nq * 128 + (size_t)h0 * 128;
        const uint16_t* q1 = p.q + (size_t)t * p.nq * 128 + (size_t)h1 * 128;
        const bool v0 = g < p.G, v1 = g + 8 < p.G;
#pragma unroll
        for (int kc = 0; kc < 8; ++kc) {
            const int c = kc * 16 + c2;
            qa[kc][0] = v0 ? *reinterpret_cast<const uint32_t*>(q0 + c) : 0u;
            qa[kc][1] = v1 ? *reinterpret_cast<const uint32_t*>(q1 + c) : 0u;
            qa[kc][2] = v0 ? *reinterpret_cast<const uint32_t*>(q0 + c + 8) : 0u;
            qa[kc][3] = v1 ? *reinterpret_cast<const uint32_t*>(q1 + c + 8) : 0u;
        }
    }

    int it = 0;
    bool ok = true;
    for (int pg = my_first; pg < pg1; pg += kWarps, ++it) {
        const int b = it & 1;
        if (lane == 0 && pg + kWarps < pg1) issue(pg + kWarps, b ^ 1);
        const bool got = mbar_wait(bar0 + b * 8, (uint32_t)((it >> 1) & 1), p.err);
        if (!__all_sync(0xffffffffu, got)) { ok = false; break; }
        const uint32_t kb = buf0 + b * kBufBytes, vb = kb + kPageBytes;
        // S = Q K^T for 16 positions (two n-blocks of 8)
        float s[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
        const int mat = lane >> 3, r8 = lane & 7;
#pragma unroll
        for (int kc = 0; kc < 8; ++kc) {
            uint32_t b00, b01, b10, b11;
            ldsm_x4(sw_addr(kb, (mat >> 1) * 8 + r8, kc * 2 + (mat & 1)), b00, b01, b10, b11);
            mma16816(s[0], qa[kc][0], qa[kc][1], qa[kc][2], qa[kc][3], b00, b01);
            mma16816(s[1], qa[kc][0], qa[kc][1], qa[kc][2], qa[kc][3], b10, b11);
        }
        // scale (log2 domain) + mask positions >= L
        const int base_pos = pg * 16;
        float x[2][4];
#pragma unroll
        for (int nb = 0; nb < 2; ++nb)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int pos = base_pos + nb * 8 + c2 + (e & 1);
                x[nb][e] = pos < L ? s[nb][e] * p.scale_log2 : -INFINITY;
            }
        float mx0 = fmaxf(fmaxf(x[0][0], x[0][1]), fmaxf(x[1][0], x[1][1]));
        float mx1 = fmaxf(fmaxf(x[0][2], x[0][3]), fmaxf(x[1][2], x[1][3]));
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
        const float nm0 = fmaxf(m0, mx0), nm1 = fmaxf(m1, mx1);
        const float a0 = exp2f(m0 - nm0), a1 = exp2f(m1 - nm1);  // m = -inf initially -> 0
        m0 = nm0;
        m1 = nm1;
        float pr[2][4];
#pragma unroll
        for (int nb = 0; nb < 2; ++nb) {
            pr[nb][0] = exp2f(x[nb][0] - nm0);
            pr[nb][1] = exp2f(x[nb][1] - nm0);
            pr[nb][2] = exp2f(x[nb][2] - nm1);
            pr[nb][3] = exp2f(x[nb][3] - nm1);
        }
        l0 = l0 * a0 + (pr[0][0] + pr[0][1]) + (pr[1][0] + pr[1][1]);
        l1 = l1 * a1 + (pr[0][2] + pr[0][3]) + (pr[1][2] + pr[1][3]);
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            o[i][0] *= a0;
            o[i][1] *= a0;
            o[i][2] *= a1;
            o[i][3] *= a1;
        }
        // P as the A operand (rows = heads, k = the 16 positions)
        const uint32_t pa0 = pack_bf16(pr[0][0], pr[0][1]), pa1 = pack_bf16(pr[0][2], pr[0][3]);
        const uint32_t pa2 = pack_bf16(pr[1][0], pr[1][1]), pa3 = pack_bf16(pr[1][2], pr[1][3]);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            uint32_t v0, v1, v2, v3;
            ldsm_x4_t(sw_addr(vb, (mat & 1) * 8 + r8, 2 * j + (mat >> 1)), v0, v1, v2, v3);
            mma16816(o[2 * j], pa0, pa1, pa2, pa3, v0, v1);
            mma16816(o[2 * j + 1], pa0, pa1, pa2, pa3, v2, v3);
        }
        __syncwarp();  // all lanes done reading buffer b before it is refilled
    }
    // Error path: drain the copies this warp still has in flight (the page of
    // iteration it and, if issued, the one after) before the buffers are reused.
    if (!ok && lane == 0) {
        mbar_wait_drain(bar0 + (it & 1) * 8, (uint32_t)((it >> 1) & 1));
        const int nxt = it + 1;
        if (my_first + nxt * kWarps - kWarps < pg1 && my_first + nxt * kWarps < pg1)
            mbar_wait_drain(bar0 + (nxt & 1) * 8, (uint32_t)((nxt >> 1) & 1));
    }
    // row sums across the 4 lanes of a row
    l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
    l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 2);

    // ---- combine the 4 warps in warp order through shared memory
    // red layout: [warp][16 rows][128] O, then [warp][16][2] (m, l)
    float* ro = red;
    float* rml = red + kWarps * 16 * 128;
    __syncthreads();
#pragma unroll
    for (int i = 0; i < 16; ++i) {
        const int col = i * 8 + c2;
        ro[(warp * 16 + g) * 128 + col] = o[i][0];
        ro[(warp * 16 + g) * 128 + col + 1] = o[i][1];
        ro[(warp * 16 + g + 8) * 128 + col] = o[i][2];
        ro[(warp * 16 + g + 8) * 128 + col + 1] = o[i][3];
    }
    if ((lane & 3) == 0) {
        rml[(warp * 16 + g) * 2] = m0;
        rml[(warp * 16 + g) * 2 + 1] = l0;
        rml[(warp * 16 + g + 8) * 2] = m1;
        rml[(warp * 16 + g + 8) * 2 + 1] = l1;
    }
    __syncthreads();
    const size_t slot = ((size_t)t * p.nkv + kvh) * p.max_chunks + chunk;
    for (int e = threadIdx.x; e < p.G * 128; e += 128) {
        const int r = e >> 7, d = e & 127;
        float m = -INFINITY;
        for (int w = 0; w < kWarps; ++w) m = fmaxf(m, rml[(w * 16 + r) * 2]);
        float acc = 0.f, l = 0.f;
        for (int w = 0; w < kWarps; ++w) {
            const float mw = rml[(w * 16 + r) * 2];
            const float sc = mw == -INFINITY ? 0.f : exp2f(mw - m);
            acc += ro[(w * 16 + r) * 128 + d] * sc;
            l += rml[(w * 16 + r) * 2 + 1] * sc;
        }
        p.part[(slot * p.G + r) * 128 + d] = acc;
        if (d == 0) {
            p.part_ml[(slot * p.G + r) * 2] = m;
            p.part_ml[(slot * p.G + r) * 2 + 1] = l;
        }
    }
    // ---- the CTA that writes the last chunk of (t, kv head) merges all of them
    const int n_chunks = (n_pages + kPages - 1) / kPages;
    __threadfence();  // this CTA's partial is visible before it is counted
    __syncthreads();
    int* last = reinterpret_cast<int*>(rml);  // scratch no longer read
    if (threadIdx.x == 0) {
        int* cnt = p.chunk_cnt + (size_t)t * p.nkv + kvh;
        const bool is_last = atomicAdd(cnt, 1) == n_chunks - 1;
        if (is_last) *cnt = 0;  // every chunk has counted: clear for the next launch
        *last = is_last ? 1 : 0;
    }
    __syncthreads();
    if (!*last) return;
    __threadfence();  // the other chunks' partials, counted before this one
    const size_t base = ((size_t)t * p.nkv + kvh) * p.max_chunks;
    for (int r = warp; r < p.G; r += kWarps)
        combine_row(p.part, p.part_ml, base, p.G, r, n_chunks, lane,
                    p.out + (size_t)t * p.nq * 128 + (size_t)(kvh * p.G + r) * 128);
}

// ---------------------------------------------------------------- prefill
// Causal attention of a prompt over the paged cache: the prompt's own K/V rows
// were appended by the q/k/v GEMM of this layer, so query token t (position
// pos_t) attends to positions 0..pos_t of its sequence.  One CTA per (block of
// up to 16 consecutive query tokens of one sequence, kv head); warp w takes
// query head kvh * G + w with the block's tokens as its 16 MMA rows, and all
// warps share each K/V page (TMA into a 4-deep ring).  Output bf16
// attn[t][head * 128 + d]; every reduction runs in a fixed order.
constexpr int kPfRing = 4;

struct PrefillAttnParams {
    CUtensorMap tm_k, tm_v;
    const uint16_t* q;         // [T][nq*128]
    const int* block_tables;   // [T][max_blocks] (the token's sequence)
    const int* pos;            // [T] position of each token
    const int2* qblk;          // [n_qblk] (first token, tokens <= 16)
    uint16_t* out;             // [T][nq*128]
    int n_qblk, nq, nkv, G, layer, num_blocks, max_blocks;
    float scale_log2;
    int* err;
};

__global__ void __launch_bounds__(512) attn_prefill_kernel(const __grid_constant__ PrefillAttnParams p) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + kPfRing * kBufBytes);
    uint64_t* empty = full + kPfRing;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // longest blocks (latest in each prompt) first
    const int qb = p.n_qblk - 1 - (int)(blockIdx.x / p.nkv);
    const int kvh = (int)(blockIdx.x % p.nkv);
    const int2 d = __ldg(p.qblk + qb);
    const int t0 = d.x, nt = d.y;
    const int p0 = __ldg(p.pos + t0);
    const int n_pages = (p0 + nt - 1) / 16 + 1;  // through the block's last position
    if (threadIdx.x < kPfRing) {
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_u32(&full[threadIdx.x])) : "memory");
        asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(&empty[threadIdx.x])), "r"(p.G) : "memory");
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    __syncthreads();
    pdl_wait();
    pdl_trigger();
    const int* bt = p.block_tables + (size_t)t0 * p.max_blocks;
    auto issue = [&](int pg) {
        const int b = pg % kPfRing;
        const uint32_t bar = smem_u32(&full[b]), dst = smem_u32(smem + b * kBufBytes);
        asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(kBufBytes) : "memory");
        const int row = ((p.layer * p.num_blocks + __ldg(bt + pg)) * p.nkv + kvh) * 16;
        tma_page(&p.tm_k, dst, bar, row);
        tma_page(&p.tm_v, dst + kPageBytes, bar, row);
    };
    int n_issued = 0;  // thread 0: pages issued so far
    if (threadIdx.x == 0)
        for (; n_issued < min(kPfRing, n_pages); ++n_issued) issue(n_issued);

    const int g = lane >> 2, c2 = (lane & 3) * 2;
    const int h = kvh * p.G + warp;
    uint32_t qa[8][4];
    {
        const bool v0 = g < nt, v1 = g + 8 < nt;
        const uint16_t* q0 = p.q + (size_t)(t0 + (v0 ? g : 0)) * p.nq * 128 + (size_t)h * 128;
        const uint16_t* q1 = p.q + (size_t)(t0 + (v1 ? g + 8 : 0)) * p.nq * 128 + (size_t)h * 128;
#pragma unroll
        for (int kc = 0; kc < 8; ++kc) {
            const int c = kc * 16 + c2;
            qa[kc][0] = v0 ? *reinterpret_cast<const uint32_t*>(q0 + c) : 0u;
            qa[kc][1] = v1 ? *reinterpret_cast<const uint32_t*>(q1 + c) : 0u;
            qa[kc][2] = v0 ? *reinterpret_cast<const uint32_t*>(q0 + c + 8) : 0u;
            qa[kc][3] = v1 ? *reinterpret_cast<const uint32_t*>(q1 + c + 8) : 0u;
        }
    }
    const int qpos0 = p0 + g, qpos1 = p0 + g + 8;  // causal limits of the thread's two rows
    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
    float o[16][4];
#pragma unroll
    for (int i = 0; i < 16; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
    bool ok = true;
    const int mat = lane >> 3, r8 = lane & 7;
    for (int pg = 0; pg < n_pages; ++pg) {
        const int b = pg % kPfRing;
        const bool got = mbar_wait(smem_u32(&full[b]), (uint32_t)((pg / kPfRing) & 1), p.err);
        if (!__all_sync(0xffffffffu, got)) { ok = false; break; }
        const uint32_t kb = smem_u32(smem + b * kBufBytes), vb = kb + kPageBytes;
        float s[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
        for (int kc = 0; kc < 8; ++kc) {
            uint32_t b00, b01, b10, b11;
            ldsm_x4(sw_addr(kb, (mat >> 1) * 8 + r8, kc * 2 + (mat & 1)), b00, b01, b10, b11);
            mma16816(s[0], qa[kc][0], qa[kc][1], qa[kc][2], qa[kc][3], b00, b01);
            mma16816(s[1], qa[kc][0], qa[kc][1], qa[kc][2], qa[kc][3], b10, b11);
        }
        const int base_pos = pg * 16;
        float x[2][4];
        if (base_pos + 15 <= p0) {  // every key of the page precedes every query of the block
#pragma unroll
            for (int nb = 0; nb < 2; ++nb)
#pragma unroll
                for (int e = 0; e < 4; ++e) x[nb][e] = s[nb][e] * p.scale_log2;
        } else {  // the diagonal page(s): causal mask
#pragma unroll
            for (int nb = 0; nb < 2; ++nb)
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const int kp = base_pos + nb * 8 + c2 + (e & 1);
                    x[nb][e] = kp <= (e < 2 ? qpos0 : qpos1) ? s[nb][e] * p.scale_log2 : -INFINITY;
                }
        }
        float mx0 = fmaxf(fmaxf(x[0][0], x[0][1]), fmaxf(x[1][0], x[1][1]));
        float mx1 = fmaxf(fmaxf(x[0][2], x[0][3]), fmaxf(x[1][2], x[1][3]));
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
        const float nm0 = fmaxf(m0, mx0), nm1 = fmaxf(m1, mx1);
        // a row whose every key so far is masked keeps m = -inf: scale factors 0 / 1 without NaN
        const float a0 = nm0 == -INFINITY ? 1.f : exp2f(m0 - nm0), a1 = nm1 == -INFINITY ? 1.f : exp2f(m1 - nm1);
        m0 = nm0;
        m1 = nm1;
        float pr[2][4];
#pragma unroll
        for (int nb = 0; nb < 2; ++nb) {
            pr[nb][0] = nm0 == -INFINITY ? 0.f : exp2f(x[nb][0] - nm0);
            pr[nb][1] = nm0 == -INFINITY ? 0.f : exp2f(x[nb][1] - nm0);
            pr[nb][2] = nm1 == -INFINITY ? 0.f : exp2f(x[nb][2] - nm1);
            pr[nb][3] = nm1 == -INFINITY ? 0.f : exp2f(x[nb][3] - nm1);
        }
        l0 = l0 * a0 + (pr[0][0] + pr[0][1]) + (pr[1][0] + pr[1][1]);
        l1 = l1 * a1 + (pr[0][2] + pr[0][3]) + (pr[1][2] + pr[1][3]);
        // rescale only when some row's running max moved (rare after the first pages)
        if (__any_sync(0xffffffffu, a0 != 1.f || a1 != 1.f)) {
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                o[i][0] *= a0;
                o[i][1] *= a0;
                o[i][2] *= a1;
                o[i][3] *= a1;
            }
        }
        const uint32_t pa0 = pack_bf16(pr[0][0], pr[0][1]), pa1 = pack_bf16(pr[0][2], pr[0][3]);
        const uint32_t pa2 = pack_bf16(pr[1][0], pr[1][1]), pa3 = pack_bf16(pr[1][2], pr[1][3]);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            uint32_t v0, v1, v2, v3;
            ldsm_x4_t(sw_addr(vb, (mat & 1) * 8 + r8, 2 * j + (mat >> 1)), v0, v1, v2, v3);
            mma16816(o[2 * j], pa0, pa1, pa2, pa3, v0, v1);
            mma16816(o[2 * j + 1], pa0, pa1, pa2, pa3, v2, v3);
        }
        __syncwarp();
        if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(&empty[b])) : "memory");
        // Thread 0 refills buffer b with page pg + kPfRing once every warp
        // released it.  If that wait fails it has set the error word, and the
        // next wait of every warp on an unfilled page fails with it, so all
        // lanes leave the loop together.
        if (threadIdx.x == 0 && pg + kPfRing < n_pages &&
            mbar_wait(smem_u32(&empty[b]), (uint32_t)((pg / kPfRing) & 1), p.err)) {
            issue(pg + kPfRing);
            ++n_issued;
        }
    }
    // Error path: thread 0 waits (bounded) for the pages it still has in flight
    // (the last kPfRing issued; earlier ones were consumed before their refill).
    if (!ok && threadIdx.x == 0)
        for (int pg = max(0, n_issued - kPfRing); pg < n_issued; ++pg)
            mbar_wait_drain(smem_u32(&full[pg % kPfRing]), (uint32_t)((pg / kPfRing) & 1));
    l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
    l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
    if (!ok) return;
    const float i0 = l0 > 0.f ? 1.f / l0 : 0.f, i1 = l1 > 0.f ? 1.f / l1 : 0.f;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
        const int col = h * 128 + i * 8 + c2;
        if (g < nt)
            *reinterpret_cast<uint32_t*>(p.out + (size_t)(t0 + g) * p.nq * 128 + col) = pack_bf16(o[i][0] * i0, o[i][1] * i0);
        if (g + 8 < nt)
            *reinterpret_cast<uint32_t*>(p.out + (size_t)(t0 + g + 8) * p.nq * 128 + col) =
                pack_bf16(o[i][2] * i1, o[i][3] * i1);
    }
}

}  // namespace

size_t attn_prefill_smem_bytes() { return 1024 + kPfRing * kBufBytes + 2 * kPfRing * 8; }

cudaError_t launch_attention_prefill(const CUtensorMap& tm_k, const CUtensorMap& tm_v, const uint16_t* q,
                                     const int* block_tables, const int* pos, const int2* qblk, int n_qblk, int nq,
                                     int nkv, int layer, int num_blocks, int max_blocks, int* err, uint16_t* out,
                                     cudaStream_t s) {
    if (n_qblk <= 0) return cudaSuccess;
    if (nq % nkv || nq / nkv > 16) return cudaErrorInvalidValue;
    PrefillAttnParams p;
    p.tm_k = tm_k;
    p.tm_v = tm_v;
    p.q = q;
    p.block_tables = block_tables;
    p.pos = pos;
    p.qblk = qblk;
    p.out = out;
    p.n_qblk = n_qblk;
    p.nq = nq;
    p.nkv = nkv;
    p.G = nq / nkv;
    p.layer = layer;
    p.num_blocks = num_blocks;
    p.max_blocks = max_blocks;
    p.scale_log2 = 1.4426950408889634f / sqrtf(128.0f);
    p.err = err;
    return launch_k(attn_prefill_kernel, dim3(n_qblk * nkv), dim3(32 * p.G), attn_prefill_smem_bytes(), s, p);
}

size_t attn_smem_bytes() { return 1024 + kWarps * 2 * kBufBytes + 64; }
static_assert(kWarps * 16 * 128 * 4 + kWarps * 16 * 2 * 4 <= kWarps * 2 * kBufBytes, "combine scratch fits the page buffers");

cudaError_t attn_configure() {
    cudaError_t e = cudaFuncSetAttribute(attn_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)attn_smem_bytes());
    if (e != cudaSuccess) return e;
    return cudaFuncSetAttribute(attn_prefill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                (int)attn_prefill_smem_bytes());
}

int attn_max_chunks(int max_seq_len) { return ((max_seq_len + 15) / 16 + kPages - 1) / kPages; }

cudaError_t launch_attention(const CUtensorMap& tm_k, const CUtensorMap& tm_v, const uint16_t* q, const int* block_tables,
                             const int* ctx_lens, float* part, float* part_ml, int* chunk_cnt, int T, int nq, int nkv,
                             int layer, int num_blocks, int max_blocks, int max_chunks, int* err, uint16_t* out,
                             cudaStream_t s) {
    if (T <= 0) return cudaSuccess;
    AttnParams p;
    p.tm_k = tm_k;
    p.tm_v = tm_v;
    p.q = q;
    p.block_tables = block_tables;
    p.ctx_lens = ctx_lens;
    p.part = part;
    p.part_ml = part_ml;
    p.chunk_cnt = chunk_cnt;
    p.out = out;
    p.T = T;
    p.nq = nq;
    p.nkv = nkv;
    p.G = nq / nkv;
    p.layer = layer;
    p.num_blocks = num_blocks;
    p.max_blocks = max_blocks;
    p.max_chunks = max_chunks;
    p.scale_log2 = 1.4426950408889634f / sqrtf(128.0f);
    p.err = err;
    const size_t smem = attn_smem_bytes();
    return launch_k(attn_decode_kernel, dim3(T * nkv * max_chunks), dim3(128), smem, s, p);
}

}  // namespace aos
