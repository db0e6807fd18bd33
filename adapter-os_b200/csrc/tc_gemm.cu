// tc_gemm.cu — tcgen05/TMEM/TMA weight-streaming GEMM with the LoRA shrink
// and expand fused into the same launch, and the decoder's epilogues.
//
// One launch computes, for one input X (normed hidden, attention output or
// SwiGLU activation):
//   shrink tiles : hm[t, group cols] = gate(t, owner) * (x_t . A_cat[group rows])
//                  for four touched 64-column rank groups per tile, of every
//                  LoRA module that reads X (TC_SHRINK_HM epilogue);
//   base tiles   : X . W[256 rows]^T  +  sum over touched groups of
//                  hm[group cols] . B_cat[256 rows, group cols]^T
// so a base tile's accumulator ends as  x W^T + sum_a (g_a * scale_a * x A_a^T) B_a^T
// (mlx_cpp_wrapper_real.cpp:3372-3419) without materialising the LoRA delta.
// MMA M = 128 token lanes, N = 256 weight rows (a kind::f16 MMA takes the same
// time for any N up to 256, so the wide side carries the weights).
//   K step      : bulk copy of two packed 16 KB weight blocks (or four 8 KB
//                 lora_A group blocks) + TMA box X[T x 64]
//   expand step : two packed lora_B blocks [128 rows x one group] + TMA box
//                 hm[T x the same group]
// all SWIZZLE_128B shared-memory images, four K=16 MMAs per step.
//
// Roles (192 threads, one CTA per SM, grid = SM count):
//   warp 0      : TMA / bulk-copy producer (one elected lane)
//   warp 1      : TMEM allocator + MMA issuer (one elected lane)
//   warps 2..5  : drain (TMEM lane quarter = warp % 4, one token per lane)
//                 and the parallel reduction of split tiles
// Work is split stream-K style (see "schedule"): every CTA streams the same
// number of steps.  Split tiles are summed in piece order after bounded grid
// barriers (fixed order: bit-identical run to run; no float atomics).
//
// Every wait is bounded (kSpinLimitCycles): on timeout the kernel records
// AOS_ERR_TIMEOUT in p.err, drains its own copies and MMAs, frees TMEM and
// returns.

#include <algorithm>
#include <cstring>

#include "tc_gemm.cuh"

namespace aos {
namespace {

// ---------------------------------------------------------------- PTX helpers
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
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
__device__ __forceinline__ void tma_2d(const CUtensorMap* m, uint32_t dst, uint32_t bar, int x, int y,
                                       uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1, {%3, %4}], [%2], %5;" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(m)), "r"(bar), "r"(x), "r"(y), "l"(policy)
        : "memory");
}
// Contiguous global -> shared bulk copy (no tensor map), completing on `bar`.
// Both addresses 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(dst),
        "l"(src), "r"(bytes), "r"(bar), "l"(policy)
        : "memory");
}
__device__ __forceinline__ uint64_t policy_evict_first() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}
__device__ __forceinline__ uint64_t policy_evict_last() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
    return p;
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void umma_bf16(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d),
        "l"(a), "l"(b), "r"(idesc), "r"(acc));
}
__device__ __forceinline__ void umma_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
          "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]),
          "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]),
          "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void epi_bar() { asm volatile("bar.sync 1, 128;" ::: "memory"); }
// Shared-memory matrix descriptors (tcgen05 "version 1"), K-major operands.
__device__ __forceinline__ uint64_t desc_sw128(uint32_t addr) {
    return (uint64_t)((addr >> 4) & 0x3FFFu) | ((uint64_t)1u << 16) | ((uint64_t)(1024u >> 4) << 32) |
           ((uint64_t)1u << 46) | ((uint64_t)2u << 61);
}
// kind::f16 instruction descriptor: D f32, A/B bf16, both K-major, M=128.
__device__ __forceinline__ uint32_t idesc_bf16(int n) {
    return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
}

__device__ __forceinline__ int cdiv(int a, int b) { return (a + b - 1) / b; }
__device__ __forceinline__ unsigned long long gtimer() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}


// Fixed-point scale of the split-tile accumulators (value * 2^32 in int64).
constexpr float kFix = 4294967296.0f;
constexpr float kFixInv = 2.3283064365386963e-10f;
// Fixed-point scale of the folded norms' sums of squares (value * 2^16):
// finer than fp32 for any row, and room for hidden values in the thousands
// across the whole row before int64 overflows.
constexpr float kNormFix = 65536.0f;
constexpr uint32_t kTcTailBytes = 512;  // mbarriers and flags after the stages

// ---------------------------------------------------------------- epilogue
// The accumulator of a tile holds, per token (TMEM lane), 256 columns.  The
// epilogue walks them as 4 chunks of 32 column PAIRS (cA + i, cB + i): the
// pairs a mode needs together -- RoPE rotates d with d + 64 of the same head
// (mlx_cpp_wrapper_real.cpp:3270-3280), SwiGLU combines gate feature f with up
// feature f (:3522) -- so one thread finishes its token without exchanging
// data with other threads.
__device__ __forceinline__ void chunk_cols(int mode, int k, int& cA, int& cB) {
    if (mode == TC_SWIGLU) {  // gate columns [0,128), up columns [128,256)
        cA = 32 * k;
        cB = 128 + 32 * k;
    } else if (mode == TC_QKV_ROPE) {  // head k/2 of the tile, dims [32j, 32j+32) and +64
        cA = 128 * (k >> 1) + 32 * (k & 1);
        cB = cA + 64;
    } else {
        cA = 64 * k;
        cB = 64 * k + 32;
    }
}

template <int N>
__device__ __forceinline__ void store_bf16_run(uint16_t* o, const float* v) {
    if constexpr (N % 8 == 0) {
#pragma unroll
        for (int i = 0; i < N; i += 8) {
            uint4 w;
            w.x = (uint32_t)f2bf(v[i]) | ((uint32_t)f2bf(v[i + 1]) << 16);
            w.y = (uint32_t)f2bf(v[i + 2]) | ((uint32_t)f2bf(v[i + 3]) << 16);
            w.z = (uint32_t)f2bf(v[i + 4]) | ((uint32_t)f2bf(v[i + 5]) << 16);
            w.w = (uint32_t)f2bf(v[i + 6]) | ((uint32_t)f2bf(v[i + 7]) << 16);
            *reinterpret_cast<uint4*>(o + i) = w;
        }
    } else {
#pragma unroll
        for (int i = 0; i < N; i += 4) {
            uint2 w;
            w.x = (uint32_t)f2bf(v[i]) | ((uint32_t)f2bf(v[i + 1]) << 16);
            w.y = (uint32_t)f2bf(v[i + 2]) | ((uint32_t)f2bf(v[i + 3]) << 16);
            *reinterpret_cast<uint2*>(o + i) = w;
        }
    }
}

// out/resid run of N columns starting at segment row `r0` for token t.
template <int N>
__device__ __forceinline__ void store_run(const TcParams& p, int mode, int seg, int t, int r0, const float* v) {
    const int lim = p.seg_rows[seg];
    if (r0 >= lim) return;
    const size_t off = (size_t)t * p.ld_out + p.seg_out0[seg] + r0;
    const bool full = r0 + N <= lim;
    if (mode == TC_STORE_F32) {
        float* o = reinterpret_cast<float*>(p.out[seg]) + off;
        if (full) {
#pragma unroll
            for (int i = 0; i < N; i += 4) *reinterpret_cast<float4*>(o + i) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
        } else {
#pragma unroll
            for (int i = 0; i < N; ++i)
                if (r0 + i < lim) o[i] = v[i];
        }
    } else if (mode == TC_RESID_BF16) {
        // h += v, eight columns at a time; with a folded norm also the next
        // norm's input hw = h * w and this run's share of sum(h^2), from the
        // same registers
        uint16_t* h = p.resid + off;
        float sq = 0.f;
        if (full) {
#pragma unroll
            for (int i0 = 0; i0 < N; i0 += 8) {
                const uint4 hv = *reinterpret_cast<const uint4*>(h + i0);
                const uint32_t hu[4] = {hv.x, hv.y, hv.z, hv.w};
                uint32_t nu[4];
#pragma unroll
                for (int j = 0; j < 4; ++j)
                    nu[j] = (uint32_t)f2bf(bf2f((uint16_t)(hu[j] & 0xFFFFu)) + v[i0 + 2 * j]) |
                            ((uint32_t)f2bf(bf2f((uint16_t)(hu[j] >> 16)) + v[i0 + 2 * j + 1]) << 16);
                *reinterpret_cast<uint4*>(h + i0) = make_uint4(nu[0], nu[1], nu[2], nu[3]);
                if (p.ss_out) {
                    const uint4 wv = __ldg(reinterpret_cast<const uint4*>(p.norm_w + r0 + i0));
                    const uint32_t wu[4] = {wv.x, wv.y, wv.z, wv.w};
                    uint32_t ou[4];
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const float a = bf2f((uint16_t)(nu[j] & 0xFFFFu)), b = bf2f((uint16_t)(nu[j] >> 16));
                        sq = fmaf(a, a, sq);
                        sq = fmaf(b, b, sq);
                        ou[j] = (uint32_t)f2bf(a * bf2f((uint16_t)(wu[j] & 0xFFFFu))) |
                                ((uint32_t)f2bf(b * bf2f((uint16_t)(wu[j] >> 16))) << 16);
                    }
                    *reinterpret_cast<uint4*>(p.hw_out + off + i0) = make_uint4(ou[0], ou[1], ou[2], ou[3]);
                }
            }
        } else {
#pragma unroll
            for (int i = 0; i < N; ++i)
                if (r0 + i < lim) {
                    const uint16_t nb = f2bf(bf2f(h[i]) + v[i]);
                    h[i] = nb;
                    if (p.ss_out) {
                        const float a = bf2f(nb);
                        sq = fmaf(a, a, sq);
                        p.hw_out[off + i] = f2bf(a * bf2f(__ldg(p.norm_w + r0 + i)));
                    }
                }
        }
        if (p.ss_out) atomicAdd(p.ss_out + t, (unsigned long long)__float2ll_rn(sq * kNormFix));
    } else {  // TC_STORE_BF16
        uint16_t* o = reinterpret_cast<uint16_t*>(p.out[seg]) + off;
        if (full) {
            store_bf16_run<N>(o, v);
        } else {
#pragma unroll
            for (int i = 0; i < N; ++i)
                if (r0 + i < lim) o[i] = f2bf(v[i]);
        }
    }
}

// hm[t][c0 + cc + i] = bf16(v[i]): the values arrive already multiplied by
// the gate * alpha/rank of each column's adapter for token t (applied when
// the accumulator is drained, see gate_coefs).
template <int N>
__device__ __forceinline__ void shrink_run(const TcParams& p, int seg, int t, int c0, int cc, const float* v) {
    store_bf16_run<N>(reinterpret_cast<uint16_t*>(p.sh_out[seg]) + (size_t)t * p.R + c0 + cc, v);
}

// v[i] += sum over owners o (in order) of delta[o][t][col + i], i < n.
template <int N>
__device__ __forceinline__ void add_delta_run(const TcParams& p, int t, int col, int n, float (&v)[N]) {
    const uint16_t* d = p.delta + (size_t)t * p.ld_delta + col;
    if (n >= N) {
        for (int o = 0; o < p.n_delta; ++o, d += p.delta_stride) {
#pragma unroll
            for (int i = 0; i < N; i += 8) {
                const uint4 w = __ldg(reinterpret_cast<const uint4*>(d + i));
                const uint32_t u[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    v[i + 2 * j] += bf2f((uint16_t)(u[j] & 0xFFFFu));
                    v[i + 2 * j + 1] += bf2f((uint16_t)(u[j] >> 16));
                }
            }
        }
    } else {
        for (int o = 0; o < p.n_delta; ++o, d += p.delta_stride) {
#pragma unroll
            for (int i = 0; i < N; ++i)
                if (i < n) v[i] += bf2f(__ldg(d + i));
        }
    }
}

// s[i] = gate[i] * sigmoid(gate[i]) * up[i] with the hardware exp2 and a
// fast reciprocal: a few ulp of fp32 (the output is bf16); a very negative
// gate gives exp -> inf and sigmoid -> 0 exactly.
template <int N>
__device__ __forceinline__ void swiglu_run(const float (&gate)[N], const float (&up)[N], float (&s)[N]) {
#pragma unroll
    for (int i = 0; i < N; ++i) {
        const float sg = __fdividef(1.0f, 1.0f + __expf(-gate[i]));
        s[i] = (gate[i] * sg) * up[i];
    }
}

// Half-split RoPE of N dimension pairs (x_d, x_{d+64}) -> (x_d c - x_{d+64} s,
// x_d s + x_{d+64} c), cs = the position's (cos, sin) from dimension d on.
template <int N>
__device__ __forceinline__ void rope_run(const float (&x0)[N], const float (&x1)[N], const float2* cs, float (&a)[N],
                                         float (&b)[N]) {
#pragma unroll
    for (int i = 0; i < N; ++i) {
        const float2 c = __ldg(cs + i);
        a[i] = x0[i] * c.x - x1[i] * c.y;
        b[i] = x1[i] * c.x + x0[i] * c.y;
    }
}

// Per-token scale of a launch that reads a folded norm's hw: 1 / rms of the
// token's hidden row, from the fixed-point sum of squares the previous
// launch accumulated; 1 without one.
__device__ __noinline__ float token_scale_of(const unsigned long long* ss_in, int t, float ss_scale, float eps) {
    const double ss = (double)(long long)__ldcg(ss_in + t);
    return 1.0f / sqrtf((float)(ss * (double)ss_scale) + eps);
}
__device__ __forceinline__ float token_scale(const TcParams& p, int t) {
    return p.ss_in ? token_scale_of(p.ss_in, t, p.ss_scale, p.norm_eps) : 1.f;
}

// Applies the epilogue of `mode` to pairs [pr0, pr0 + N) of chunk k of tile
// `tile` (segment `seg`) for token t (t < T).  vA/vB: accumulator values of
// the pairs' first and second columns (the owners' deltas, if any, are added
// in place).
template <int N>
__device__ __forceinline__ void apply_pairs(const TcParams& p, int mode, int seg, int tile, int k, int t, int pr0,
                                            float (&vA)[N], float (&vB)[N], int ng, float st = 1.f) {
    int cA, cB;
    chunk_cols(mode, k, cA, cB);
    cA += pr0;
    cB += pr0;
    if (p.delta && mode != TC_SHRINK_HM) {  // owners' LoRA deltas join the accumulator
        if (mode == TC_SWIGLU) {
            const int f0 = tile * (kTcBN / 2) + cA, n = p.seg_rows[seg] - f0;
            if (n > 0) {
                add_delta_run<N>(p, t, p.dseg0[0] + f0, n, vA);
                add_delta_run<N>(p, t, p.dseg0[1] + f0, n, vB);
            }
        } else {
            const int rA = tile * kTcBN + cA, rB = tile * kTcBN + cB, lim = p.seg_rows[seg];
            if (rA < lim) add_delta_run<N>(p, t, p.dseg0[seg] + rA, lim - rA, vA);
            if (rB < lim) add_delta_run<N>(p, t, p.dseg0[seg] + rB, lim - rB, vB);
        }
    }
    // a folded norm's 1 / rms scales the whole sum (base, expand and owners'
    // deltas all read the unscaled hw); the shrink output stays unscaled
    if (st != 1.f && mode != TC_SHRINK_HM) {
#pragma unroll
        for (int i = 0; i < N; ++i) {
            vA[i] *= st;
            vB[i] *= st;
        }
    }
    switch (mode) {
        case TC_STORE_BF16:
        case TC_STORE_F32:
        case TC_RESID_BF16:
            store_run<N>(p, mode, seg, t, tile * kTcBN + cA, vA);
            store_run<N>(p, mode, seg, t, tile * kTcBN + cB, vB);
            break;
        case TC_SWIGLU: {
            const int f0 = tile * (kTcBN / 2) + cA;
            if (f0 >= p.seg_rows[seg]) break;
            float s[N];
            swiglu_run<N>(vA, vB, s);
            uint16_t* o = reinterpret_cast<uint16_t*>(p.out[seg]) + (size_t)t * p.ld_out + f0;
            if (f0 + N <= p.seg_rows[seg]) {
                store_bf16_run<N>(o, s);
            } else {
#pragma unroll
                for (int i = 0; i < N; ++i)
                    if (f0 + i < p.seg_rows[seg]) o[i] = f2bf(s[i]);
            }
            break;
        }
        case TC_QKV_ROPE: {
            const int module = p.seg_module[seg];
            const int head = tile * 2 + (cA >> 7);  // one head = 128 columns
            if (head * 128 >= p.seg_rows[seg]) break;
            const int d = cA & 127;  // < 64; its partner is d + 64
            const int pos = __ldg(p.ctx_lens + t);
            float a[N], b[N];
            if (module != AOS_MOD_V) {
                // half-split RoPE: (x_d, x_{d+64}) -> (x_d c - x_{d+64} s, x_d s + x_{d+64} c)
                rope_run<N>(vA, vB, reinterpret_cast<const float2*>(p.rope) + (size_t)pos * 64 + d, a, b);
            } else {
#pragma unroll
                for (int i = 0; i < N; ++i) {
                    a[i] = vA[i];
                    b[i] = vB[i];
                }
            }
            uint16_t* dst;
            if (module == AOS_MOD_Q) {
                dst = reinterpret_cast<uint16_t*>(p.out[seg]) + (size_t)t * p.ld_out + head * 128 + d;
            } else {
                uint16_t* pool = module == AOS_MOD_K ? p.k_pool : p.v_pool;
                const int blk = __ldg(p.block_tables + (size_t)t * p.max_blocks + (pos >> 4));
                dst = pool + ((((size_t)p.layer * p.num_blocks + blk) * p.nkv + head) * 16 + (pos & 15)) * 128 + d;
            }
            store_bf16_run<N>(dst, a);
            store_bf16_run<N>(dst + 64, b);
            break;
        }
        case TC_SHRINK_HM: {
            const int slot = tile * kShrinkGroupsPerTile + k;
            if (slot >= ng) break;
            const int c0 = __ldg(p.groups + slot) * kGroup;  // rank column of the group's first column
            shrink_run<N>(p, seg, t, c0, cA - 64 * k, vA);
            shrink_run<N>(p, seg, t, c0, cB - 64 * k, vB);
            break;
        }
        default:
            break;
    }
}

// ---------------------------------------------------------------- schedule
// Stream-K over two pools, taken by every CTA in this order:
//   A: the K steps of the shrink tiles (four touched lora_A groups each);
//   B: the "positions" of the base tiles.  A base tile has kbe K steps and
//      nge expand steps (one per touched rank group); position q of the tile
//      is a K step or an expand step in proportion (bpos), so any range of
//      positions holds both kinds in the tile's ratio.
// CTA c takes the contiguous slice [c*P/G, (c+1)*P/G) of each pool.  A piece
// (one tile's share of one slice) accumulates its K steps and then its expand
// steps in one TMEM accumulator.  A CTA with at most two base pieces runs
// both pieces' K steps before either's expand steps, so it has its whole
// base share to stream while the shrink output is being finished.  A tile
// cut into several pieces is summed in fixed point (see the drain).
struct Sched {
    int ng;            // touched rank groups
    int kb;            // K steps per tile
    int sh_per_seg;    // shrink tiles per shrink segment
    int n_sh, n_base;  // shrink tiles, base tiles
    int kbe, nge;      // K steps and expand steps per base tile in this launch
    int P[2];          // pool lengths: shrink K steps, base positions (< 2^31 / SMs)
    int G[2];          // CTAs that take part in each pool
    int len[2];        // steps (positions) per tile
};

struct Piece {
    int tile;  // global tile id: shrink tiles first, then base tiles
    int n;     // pieces of the tile in total
    bool shrink;
    int seg, t;  // segment, and tile index within the segment
};

__device__ __forceinline__ Sched make_sched(const TcParams& p) {
    Sched s;
    s.ng = (p.lora || p.sh_nseg) ? __ldg(p.n_groups) : 0;
    s.kb = p.kb;
    s.sh_per_seg = p.sh_nseg ? cdiv(s.ng, kShrinkGroupsPerTile) : 0;
    s.n_sh = p.sh_nseg * s.sh_per_seg;
    s.n_base = 0;
    for (int g = 0; g < p.n_seg; ++g) s.n_base += p.seg_tiles[g];
    s.kbe = (p.pools & 2) ? s.kb : 0;
    s.nge = (p.lora && (p.pools & 4)) ? s.ng : 0;
    s.len[0] = s.kb;
    s.len[1] = s.kbe + s.nge;
    s.P[0] = s.n_sh * s.kb;
    s.P[1] = s.n_base * s.len[1];
    // Every slice is at least len/kMaxPiecesPerPool steps long, so no tile is
    // cut into more than kMaxPiecesPerPool + 1 pieces.
    for (int q = 0; q < 2; ++q) {
        const int l = max(1, cdiv(max(s.len[q], 1), kMaxPiecesPerPool));
        s.G[q] = s.P[q] > 0 ? max(1, min((int)gridDim.x, s.P[q] / l)) : 0;
    }
    return s;
}
// Pool lengths times the grid stay below 2^31 (the host checks the plan).
__device__ __forceinline__ int pstart(int c, int P, int G) { return c * P / G; }
// CTA whose slice of a pool (length P, G CTAs) contains step s.
__device__ __forceinline__ int cta_of(int s, int P, int G) { return ((s + 1) * G - 1) / P; }
// K steps among the first `pos` positions of a base tile.
__device__ __forceinline__ int bpos(const Sched& sc, int pos) {
    return sc.len[1] ? pos * sc.kbe / sc.len[1] : 0;
}

__device__ __forceinline__ void tile_info(const TcParams& p, const Sched& sc, int tile, Piece& pc) {
    pc.tile = tile;
    if (tile < sc.n_sh) {
        pc.shrink = true;
        pc.seg = tile / sc.sh_per_seg;
        pc.t = tile % sc.sh_per_seg;
    } else {
        pc.shrink = false;
        int b = tile - sc.n_sh, g = 0;
        while (g < p.n_seg - 1 && b >= p.seg_tiles[g]) {
            b -= p.seg_tiles[g];
            ++g;
        }
        pc.seg = g;
        pc.t = b;
    }
}
// Pieces of `tile` (CTAs whose slice touches it).
__device__ __forceinline__ int tile_npieces(const Sched& sc, int tile) {
    const int q = tile < sc.n_sh ? 0 : 1;
    const int local = q ? tile - sc.n_sh : tile;
    if (sc.P[q] <= 0) return 0;
    const int a = local * sc.len[q];
    return cta_of(a + sc.len[q] - 1, sc.P[q], sc.G[q]) - cta_of(a, sc.P[q], sc.G[q]) + 1;
}

// This CTA's work, built once by thread 0 in shared memory and read by every
// role: its pieces (in drain order) and the parts the producer and the MMA
// run (a piece's K steps, or its expand steps), in execution order.
constexpr int kMaxPieces = 24;
constexpr int kMaxParts = 40;
struct PieceRec {
    int tile, n;      // tile, pieces of the tile in total
    int b0, b1;       // K steps [b0, b1) of the tile
    int c0, c1;       // expand steps [c0, c1) (touched-group list indices)
};
struct PartRec {
    uint16_t piece;   // index into pc[]
    uint8_t expand;   // 1: expand steps, 0: K steps
    uint8_t flags;    // 1: first part of its piece (fresh accumulator), 2: last part (commit)
};
struct WorkTable {
    int n_pieces, n_parts;
    PieceRec pc[kMaxPieces];
    PartRec pt[kMaxParts];
};

__device__ bool build_work(const Sched& sc, int acc_stages, WorkTable& w) {
    const int c = blockIdx.x;
    int np = 0;
    for (int q = 0; q < 2; ++q) {
        if (c >= sc.G[q]) continue;
        int s = pstart(c, sc.P[q], sc.G[q]);
        const int e = pstart(c + 1, sc.P[q], sc.G[q]);
        const int L = sc.len[q];
        while (s < e) {
            const int local = s / L;
            const int ts = local * L, te = min(ts + L, e);
            if (np == kMaxPieces) return false;
            PieceRec& r = w.pc[np++];
            const int p0 = (int)(s - ts), p1 = (int)(te - ts);
            if (q == 0) {
                r.tile = local;
                r.b0 = p0;
                r.b1 = p1;
                r.c0 = r.c1 = 0;
            } else {
                r.tile = sc.n_sh + local;
                r.b0 = bpos(sc, p0);
                r.b1 = bpos(sc, p1);
                r.c0 = p0 - r.b0;
                r.c1 = p1 - r.b1;
            }
            r.n = tile_npieces(sc, r.tile);
            s = te;
        }
    }
    w.n_pieces = np;
    int first_base = 0;
    while (first_base < np && w.pc[first_base].tile < sc.n_sh) ++first_base;
    int nt = 0;
    bool ok = true;
    auto add = [&](int i, int ex) {
        const PieceRec& r = w.pc[i];
        if ((ex ? r.c1 - r.c0 : r.b1 - r.b0) <= 0) return;
        if (nt == kMaxParts) {
            ok = false;
            return;
        }
        w.pt[nt].piece = (uint16_t)i;
        w.pt[nt].expand = (uint8_t)ex;
        w.pt[nt].flags = 0;
        ++nt;
    };
    for (int i = 0; i < first_base; ++i) add(i, 0);
    if (acc_stages == 2 && np - first_base <= 2) {  // both base pieces' K steps first
        for (int i = first_base; i < np; ++i) add(i, 0);
        for (int i = first_base; i < np; ++i) add(i, 1);
    } else {
        for (int i = first_base; i < np; ++i) {
            add(i, 0);
            add(i, 1);
        }
    }
    if (!ok) return false;
    for (int k = 0; k < nt; ++k) {
        bool first = true, last = true;
        for (int j = 0; j < k; ++j) first = first && w.pt[j].piece != w.pt[k].piece;
        for (int j = k + 1; j < nt; ++j) last = last && w.pt[j].piece != w.pt[k].piece;
        w.pt[k].flags = (uint8_t)((first ? 1 : 0) | (last ? 2 : 0));
    }
    w.n_parts = nt;
    return true;
}

// Bounded spin until *ptr >= target (acquire); false on timeout or when
// another role already failed.
__device__ __noinline__ bool spin_ge(const int* ptr, int target, int* err) {
    const long long t0 = clock64();
    uint32_t n = 0;
    while (true) {
        int v;
        asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(ptr) : "memory");
        if (v >= target) return true;
        if ((++n & 255u) == 0) {
            if (*(volatile int*)err != 0) return false;
            if (clock64() - t0 > kSpinLimitCycles) {
                atomicCAS(err, 0, AOS_ERR_TIMEOUT);
                return false;
            }
        }
    }
}

// ---------------------------------------------------------------- the kernel
// kPart: split base tiles go through fp32 partials (p.part; the runtime sets
// it for every launch); the instance without it (p.part null) adds base
// pieces in fixed point like the shrink pieces.
template <bool kPart>
__global__ void __launch_bounds__(kTcThreads, 1) tc_gemm_kernel(const __grid_constant__ TcParams p) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    // 1024-align the dynamic region (SWIZZLE_128B atoms).
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int NS = p.n_stages;
    uint8_t* stages = smem;
    uint8_t* tail = smem + (size_t)NS * p.stage_bytes;
    uint64_t* full_bar = reinterpret_cast<uint64_t*>(tail);
    uint64_t* empty_bar = full_bar + NS;
    uint64_t* tfull_bar = empty_bar + NS;   // [2]
    uint64_t* tempty_bar = tfull_bar + 2;   // [2]
    uint64_t* drain_bar = tempty_bar + 2;   // [1]
    uint64_t* a_done_bar = drain_bar + 1;   // drain warps: shrink pieces added (4 arrivals)
    uint64_t* all_done_bar = a_done_bar + 1;  // drain warps: every piece added (4 arrivals)
    uint64_t* sh_conv_bar = all_done_bar + 1;  // drain warps: their share of the shrink conversion done (4)
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sh_conv_bar + 1);
    int* flag = reinterpret_cast<int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const Sched sc = make_sched(p);
    const int cols_per_acc = p.tb * kTcBN;
    const int acc_stages = (2 * cols_per_acc <= 512) ? 2 : 1;
    constexpr int tmem_cols = 512;
    __shared__ WorkTable wt;

    if (threadIdx.x == 0) {
        if (!build_work(sc, acc_stages, wt)) {  // schedule limits exceeded: report, do nothing
            atomicCAS(p.err, 0, AOS_ERR_INVALID);
            wt.n_pieces = 0;
            wt.n_parts = 0;
        }
        for (int s = 0; s < NS; ++s) {
            mbar_init(smem_u32(&full_bar[s]), 1);
            mbar_init(smem_u32(&empty_bar[s]), 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(smem_u32(&tfull_bar[a]), 1);
            mbar_init(smem_u32(&tempty_bar[a]), 4);
        }
        mbar_init(smem_u32(drain_bar), 1);
        mbar_init(smem_u32(a_done_bar), 4);
        mbar_init(smem_u32(all_done_bar), 4);
        mbar_init(smem_u32(sh_conv_bar), 4);
        flag[1] = 0;
        flag[2] = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(tmem_cols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    unsigned long long* tr = p.trace ? p.trace + (size_t)blockIdx.x * kTraceStride : nullptr;
    if (tr && threadIdx.x == 0) {
        tr[210] = tr[211] = tr[212] = tr[213] = 0;
        tr[192] = gtimer();
        uint32_t smid;
        asm volatile("mov.u32 %0, %%smid;" : "=r"(smid));
        tr[220] = smid;
    }
    constexpr uint32_t kBlkW = kBlkRows * kTcBK;  // elements of a 128 x 64 weight block (16 KB)
    constexpr uint32_t kBlkA = kGroup * kTcBK;    // elements of a 64 x 64 lora_A block (8 KB)
    constexpr uint32_t kActBox = kTcTok * 128;    // shared-memory bytes reserved per activation box

    // Conversion of the split tiles in [lo, hi) by `nthr` threads of every CTA
    // (thread index `ti`): an item is (tile, pair chunk k, token, 8-column
    // group g); its thread reads 8 pairs of one token from the fixed-point
    // accumulator, zeroes them for the next launch and applies the epilogue.
    // kConvItems items per thread are loaded before any is used (the pass is
    // bound by L2 round trips, not bandwidth).
    constexpr int kConvItems = 2;
    auto convert = [&](int lo, int hi, int nthr, int ti) {
        // item = (tile, pair chunk k, 8-column group g, token), token fastest.
        // Three phases per batch of items, so that no store waits on a load of
        // the same batch: every load is issued first (the accumulator words
        // and, for shrink tiles, the group id), then the epilogues run, then
        // the words are zeroed for the next launch.
        const int n_items = (hi - lo) * 16 * p.T;
        const int stride = (int)gridDim.x * nthr;
        const bool tt = tr && ti == 128 && lo + hi > sc.n_sh;  // trace the converter's final pass
        if (tt) tr[210] = gtimer();
        bool first_it = true;
        if (kPart && lo >= sc.n_sh) {
            // base tiles from fp32 partials: sum the pieces in CTA order, two
            // pieces' words in flight at a time
            for (int item = (int)blockIdx.x * nthr + ti; item < n_items; item += stride) {
                const int tok = item % p.T;
                const int r = item / p.T;
                const int g = r % 4, k = (r / 4) % 4, tile = lo + r / 16;
                const int local = tile - sc.n_sh;
                const int s0 = local * sc.len[1];
                const int c0 = cta_of(s0, sc.P[1], sc.G[1]), c1 = cta_of(s0 + sc.len[1] - 1, sc.P[1], sc.G[1]);
                if (c1 == c0) continue;  // finished straight from TMEM
                int cA, cB;
                chunk_cols(p.mode, k, cA, cB);
                float a[8], b[8];
#pragma unroll
                for (int j = 0; j < 8; ++j) a[j] = b[j] = 0.f;
                for (int c = c0; c <= c1; c += 2) {
                    float x[2][2][8];
#pragma unroll
                    for (int e = 0; e < 2; ++e) {
                        if (c + e > c1) continue;
                        const float* src = p.part + (size_t)(c + e + local) * kTcBN * p.acc_T + tok;
#pragma unroll
                        for (int j = 0; j < 8; ++j) {
                            x[e][0][j] = __ldcg(src + (size_t)(cA + 8 * g + j) * p.acc_T);
                            x[e][1][j] = __ldcg(src + (size_t)(cB + 8 * g + j) * p.acc_T);
                        }
                    }
#pragma unroll
                    for (int e = 0; e < 2; ++e) {
                        if (c + e > c1) continue;
#pragma unroll
                        for (int j = 0; j < 8; ++j) {
                            a[j] += x[e][0][j];
                            b[j] += x[e][1][j];
                        }
                    }
                }
                Piece pc;
                tile_info(p, sc, tile, pc);
                apply_pairs<8>(p, p.mode, pc.seg, pc.t, k, tok, 8 * g, a, b, sc.ng, token_scale(p, tok));
            }
            return;
        }
        for (int base = (int)blockIdx.x * nthr + ti; base < n_items; base += kConvItems * stride) {
            unsigned long long w[kConvItems][2][8];
            unsigned long long* src[kConvItems][2];
            bool live[kConvItems];
            int tile_[kConvItems], k_[kConvItems], tok_[kConvItems], g_[kConvItems], gid[kConvItems];
#pragma unroll
            for (int e = 0; e < kConvItems; ++e) {
                const int item = base + e * stride;
                live[e] = item < n_items;
                if (!live[e]) continue;
                tok_[e] = item % p.T;
                const int r = item / p.T;
                g_[e] = r % 4;
                k_[e] = (r / 4) % 4;
                tile_[e] = lo + r / 16;
                live[e] = tile_npieces(sc, tile_[e]) > 1;  // else finished straight from TMEM
                if (!live[e]) continue;
                const bool shrink = tile_[e] < sc.n_sh;
                const int mode = shrink ? TC_SHRINK_HM : p.mode;
                int cA, cB;
                chunk_cols(mode, k_[e], cA, cB);
                gid[e] = -1;
                if (shrink) {  // the touched group this chunk belongs to
                    const int slot = (tile_[e] % sc.sh_per_seg) * kShrinkGroupsPerTile + k_[e];
                    if (slot < sc.ng) gid[e] = __ldg(p.groups + slot);
                }
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    src[e][h] = reinterpret_cast<unsigned long long*>(p.acc) +
                                ((size_t)tile_[e] * kTcBN + (h ? cB : cA) + 8 * g_[e]) * p.acc_T + tok_[e];
#pragma unroll
                    for (int j = 0; j < 8; ++j) w[e][h][j] = __ldcg(src[e][h] + (size_t)j * p.acc_T);
                }
            }
            if (tt && first_it) tr[211] = gtimer();
#pragma unroll
            for (int e = 0; e < kConvItems; ++e) {
                if (!live[e]) continue;
                if (tt && first_it && e == 0) {
                    volatile unsigned long long sink = w[e][0][0];
                    (void)sink;
                    tr[212] = gtimer();
                }
                float a[8], b[8];
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    a[j] = __ll2float_rn((long long)w[e][0][j]) * kFixInv;
                    b[j] = __ll2float_rn((long long)w[e][1][j]) * kFixInv;
                }
                if (tile_[e] < sc.n_sh) {  // gated hm of shrink segment tile / per-segment tiles
                    if (gid[e] >= 0) {
                        const int seg = tile_[e] / sc.sh_per_seg;
                        shrink_run<8>(p, seg, tok_[e], gid[e] * kGroup, 8 * g_[e], a);
                        shrink_run<8>(p, seg, tok_[e], gid[e] * kGroup, 32 + 8 * g_[e], b);
                    }
                } else {
                    Piece pc;
                    tile_info(p, sc, tile_[e], pc);
                    apply_pairs<8>(p, p.mode, pc.seg, pc.t, k_[e], tok_[e], 8 * g_[e], a, b, sc.ng,
                                   token_scale(p, tok_[e]));
                }
            }
#pragma unroll
            for (int e = 0; e < kConvItems; ++e) {
                if (!live[e]) continue;
#pragma unroll
                for (int h = 0; h < 2; ++h)
#pragma unroll
                    for (int j = 0; j < 8; ++j) __stcg(src[e][h] + (size_t)j * p.acc_T, 0ull);
            }
            if (tt && first_it) tr[213] = gtimer();
            first_it = false;
        }
    };
    volatile int* go_final = flag + 1;  // converter -> drain: 1 = every CTA's pieces are in, -1 = failed
    volatile int* go_shrink = flag + 2;  // converter -> drain: 1 = every CTA's shrink pieces are in, -1 = failed
    const bool handoff = sc.n_sh > 0 && sc.nge > 0;  // expand steps wait for this launch's shrink

    if (warp == 0) {
        // ============================ TMA producer ============================
        // The weight-side copies (W, lora_A, lora_B) of the first NS stages are
        // issued before pdl_wait(): weights are static and the group list was
        // written two or more launches earlier.  The activation-side boxes (X,
        // hm) follow once the previous launch has completed; hm boxes also wait
        // for the grid barrier after which every shrink tile is gated and stored.
        if (lane == 0) {
            const uint64_t pol_w = policy_evict_first();
            const uint64_t pol_x = policy_evict_last();
            uint32_t last_phase[16];
            uint32_t used_mask = 0;
            int n_issued = 0;
            int stage = 0;
            uint32_t phase = 0;
            bool ok = true, waited = false, shrink_ready = (sc.n_sh == 0);
            int pre_tile[16], pre_ex[16], pre_step[16];
            int n_pre = 0;
            // weight blocks of a step: shrink -> lora_A groups (8 KB each); base / expand -> two 16 KB blocks
            auto weights = [&](const Piece& pc, bool ex, int st, uint32_t sbase, uint32_t fb, bool issue) -> uint32_t {
                uint32_t bytes = 0;
                if (pc.shrink) {
                    const int first = pc.t * kShrinkGroupsPerTile;
                    const int nv = min(kShrinkGroupsPerTile, sc.ng - first);
                    for (int q = 0; q < nv; ++q) {
                        if (issue)
                            bulk_g2s(sbase + q * (kBlkA * 2),
                                     p.a_pk[pc.seg] + ((size_t)__ldg(p.groups + first + q) * sc.kb + st) * kBlkA,
                                     kBlkA * 2, fb, pol_w);
                        bytes += kBlkA * 2;
                    }
                    return bytes;
                }
                const int seg_blocks = (p.seg_rows[pc.seg] + kBlkRows - 1) / kBlkRows;
                const int g = ex ? __ldg(p.groups + st) : 0;
                for (int h = 0; h < 2; ++h) {
                    const uint16_t* src;
                    if (p.n_sub == 2) {  // gate / up: block t of each
                        src = !ex ? p.w_pk[pc.seg * 2 + h] + (((size_t)(p.seg_wrow0[pc.seg] / kBlkRows + pc.t)) * sc.kb + st) * kBlkW
                                           : p.b_pk[pc.seg * 2 + h] + ((size_t)pc.t * p.n_rgroups + g) * kBlkW;
                    } else {  // blocks 2t and 2t+1 of the segment
                        if (2 * pc.t + h >= seg_blocks) continue;
                        src = !ex
                                  ? p.w_pk[pc.seg] + (((size_t)(p.seg_wrow0[pc.seg] / kBlkRows + 2 * pc.t + h)) * sc.kb + st) * kBlkW
                                  : p.b_pk[pc.seg] + ((size_t)(2 * pc.t + h) * p.n_rgroups + g) * kBlkW;
                    }
                    if (issue) bulk_g2s(sbase + h * (kBlkW * 2), src, kBlkW * 2, fb, pol_w);
                    bytes += kBlkW * 2;
                }
                return bytes;
            };
            auto act_bytes = [&](bool ex) -> uint32_t {
                const int nh = (ex && p.n_sub == 2) ? 2 : 1;
                return (uint32_t)(nh * p.tb * p.T_box * 128);
            };
            auto issue_x = [&](const Piece& pc, bool ex, int st, uint32_t sbase, uint32_t fb) -> bool {
                const uint32_t act = sbase + p.act_off;
                if (!ex) {
                    for (int b = 0; b < p.tb; ++b) tma_2d(&p.tm_x, act + b * kActBox, fb, st * kTcBK, b * kTcTok, pol_x);
                    return true;
                }
                if (!shrink_ready) {  // hm is written by this launch's shrink tiles and reduction
                    if (tr) tr[202] = gtimer();
                    if (!spin_ge(p.sync + 1, (int)gridDim.x, p.err)) return false;
                    asm volatile("fence.proxy.async.global;" ::: "memory");
                    if (tr) tr[203] = gtimer();
                    shrink_ready = true;
                }
                const int gcol = __ldg(p.groups + st) * kGroup;
                const int nh = p.n_sub == 2 ? 2 : 1;
                for (int h = 0; h < nh; ++h) {
                    for (int b = 0; b < p.tb; ++b)
                        tma_2d(&p.tm_lh[pc.seg * p.n_sub + h], act + (h * p.tb + b) * kActBox, fb, gcol, b * kTcTok, pol_x);
                }
                return true;
            };
            auto finish_wait = [&]() -> bool {
                pdl_wait();
                pdl_trigger();
                waited = true;
                for (int i = 0; i < n_pre; ++i) {
                    Piece pc;
                    tile_info(p, sc, pre_tile[i], pc);
                    if (!issue_x(pc, pre_ex[i] != 0, pre_step[i], smem_u32(stages + (size_t)i * p.stage_bytes),
                                 smem_u32(&full_bar[i])))
                        return false;
                }
                return true;
            };
            for (int k = 0; ok && k < wt.n_parts; ++k) {
                const PartRec pt = wt.pt[k];
                const PieceRec& r = wt.pc[pt.piece];
                const bool ex = pt.expand != 0;
                Piece pc;
                tile_info(p, sc, r.tile, pc);
                const int s0 = ex ? r.c0 : r.b0, s1 = ex ? r.c1 : r.b1;
                for (int st = s0; st < s1; ++st) {
                    if (!waited && n_pre == NS && !finish_wait()) { ok = false; break; }
                    if (!mbar_wait(smem_u32(&empty_bar[stage]), phase ^ 1u, p.err)) { ok = false; break; }
                    const uint32_t fb = smem_u32(&full_bar[stage]);
                    const uint32_t sbase = smem_u32(stages + (size_t)stage * p.stage_bytes);
                    mbar_expect_tx(fb, weights(pc, ex, st, sbase, fb, false) + act_bytes(ex));
                    weights(pc, ex, st, sbase, fb, true);
                    if (waited) {
                        if (!issue_x(pc, ex, st, sbase, fb)) ok = false;
                    } else {  // first round of stages: stage index == n_pre
                        pre_tile[n_pre] = r.tile;
                        pre_ex[n_pre] = ex ? 1 : 0;
                        pre_step[n_pre] = st;
                        ++n_pre;
                    }
                    last_phase[stage] = phase;
                    used_mask |= 1u << stage;
                    if (tr && n_issued < 64) tr[n_issued] = gtimer();
                    if (tr && pc.shrink) tr[204] = gtimer();
                    ++n_issued;
                    if (++stage == NS) { stage = 0; phase ^= 1u; }
                    if (!ok) break;
                }
            }
            if (!waited) finish_wait();
            // Drain: every issued copy must land before the CTA may exit.
            for (int s = 0; s < NS; ++s)
                if (used_mask & (1u << s)) mbar_wait_drain(smem_u32(&full_bar[s]), last_phase[s]);
        }
    } else if (warp == 1) {
        // ============================ MMA issuer ==============================
        if (lane == 0) {
            const uint32_t idesc256 = idesc_bf16(kTcBN), idesc128 = idesc_bf16(kTcBN / 2);
            int stage = 0;
            uint32_t phase = 0;
            int n_waited = 0;
            bool ok = true, issued_any = false;
            bool fresh[2] = {false, false};  // accumulator slot gets its first MMA next
            for (int k = 0; ok && k < wt.n_parts; ++k) {
                const PartRec pt = wt.pt[k];
                const PieceRec& r = wt.pc[pt.piece];
                const int acc = pt.piece % acc_stages;
                if (pt.flags & 1) {  // a new piece takes the slot once its previous piece is drained
                    const uint32_t tphase = (uint32_t)((pt.piece / acc_stages) & 1);
                    if (!mbar_wait(smem_u32(&tempty_bar[acc]), tphase ^ 1u, p.err)) { ok = false; break; }
                    tc_fence_after();
                    fresh[acc] = true;
                }
                const uint32_t d0 = tmem_base + (uint32_t)(acc * cols_per_acc);
                const bool ex = pt.expand != 0;
                const bool split = ex && p.n_sub == 2;  // gate / up expand: two N=128 halves
                const int s0 = ex ? r.c0 : r.b0, s1 = ex ? r.c1 : r.b1;
                for (int st = s0; st < s1; ++st) {
                    const bool first = fresh[acc];
                    if (!mbar_wait(smem_u32(&full_bar[stage]), phase, p.err)) { ok = false; break; }
                    tc_fence_after();
                    if (tr && n_waited < 64) tr[64 + n_waited] = gtimer();
                    if (tr && r.tile < sc.n_sh) tr[205] = gtimer();
                    ++n_waited;
                    const uint32_t sbase = smem_u32(stages + (size_t)stage * p.stage_bytes);
                    const uint32_t act = sbase + p.act_off;
                    for (int b = 0; b < p.tb; ++b) {
                        if (split) {
                            for (int h = 0; h < 2; ++h) {
                                const uint32_t a0 = act + (h * p.tb + b) * kActBox, b0 = sbase + h * (kBlkW * 2);
#pragma unroll
                                for (int kk = 0; kk < kTcBK / 16; ++kk)
                                    umma_bf16(d0 + b * kTcBN + h * (kTcBN / 2), desc_sw128(a0 + kk * 32),
                                              desc_sw128(b0 + kk * 32), idesc128, (first && kk == 0) ? 0u : 1u);
                            }
                        } else {
                            const uint32_t a0 = act + b * kActBox;
#pragma unroll
                            for (int kk = 0; kk < kTcBK / 16; ++kk)
                                umma_bf16(d0 + b * kTcBN, desc_sw128(a0 + kk * 32), desc_sw128(sbase + kk * 32), idesc256,
                                          (first && kk == 0) ? 0u : 1u);
                        }
                    }
                    issued_any = true;
                    umma_commit(smem_u32(&empty_bar[stage]));  // frees the stage when these MMAs finish
                    fresh[acc] = false;
                    if (++stage == NS) { stage = 0; phase ^= 1u; }
                }
                if (!ok) break;
                if (pt.flags & 2) umma_commit(smem_u32(&tfull_bar[acc]));  // the piece is complete
            }
            if (!ok && issued_any) {
                umma_commit(smem_u32(drain_bar));
                mbar_wait_drain(smem_u32(drain_bar), 0);
            }
        }
    } else if (warp < 6) {
        // ============================ drain (warps 2-5) =========================
        // A warp reads TMEM lanes 32 * (warp % 4) ... + 31, i.e. those tokens.
        // Whole tiles get their epilogue straight from TMEM; pieces of split
        // tiles are added into the fixed-point accumulators.  The drain never
        // waits on other CTAs: it tells the converter warps through shared-
        // memory barriers when its shrink pieces and all its pieces are in.
        const int q = warp & 3;
        const int tok_lane = q * 32 + lane;
        const uint32_t lane_off = (uint32_t)(q * 32) << 16;
        const int tid = threadIdx.x - 64;  // 0..127
        pdl_wait();  // reads and writes activations and accumulators of earlier launches
        // signal a converter barrier once this warp's atomic adds have landed
        auto signal = [&](uint64_t* bar) {
            __threadfence();  // this thread's atomic adds are performed
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_u32(bar));
        };
        // Gate * alpha/rank for token `tok` of the 32 eight-column units of
        // shrink tile `t`: one contiguous 128-byte run of the prep table.
        auto gate_coefs = [&](int t, int tok, float (&cf)[32]) {
            const float4* src = reinterpret_cast<const float4*>(
                p.ucoef + ((size_t)(tok < p.T ? tok : 0) * p.n_rgroups + (size_t)t * kShrinkGroupsPerTile) * 8);
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const float4 w = __ldg(src + j);
                cf[4 * j] = w.x;
                cf[4 * j + 1] = w.y;
                cf[4 * j + 2] = w.z;
                cf[4 * j + 3] = w.w;
            }
        };

        bool sh_joined = false;
        auto join_shrink = [&]() {  // the drain warps' share (threads 0..127 of 192)
            if (*go_shrink == 1) {
                __threadfence();
                if (tr && tid == 0) tr[208] = gtimer();
                convert(0, sc.n_sh, 192, tid);
                if (tr && tid == 0) tr[209] = gtimer();
            }
            signal(sh_conv_bar);
            sh_joined = true;
        };
        bool a_signalled = false;
        for (int it = 0; it < wt.n_pieces; ++it) {
            const PieceRec& r = wt.pc[it];
            Piece pc;
            tile_info(p, sc, r.tile, pc);
            pc.n = r.n;
            if (!a_signalled && !pc.shrink) {  // this CTA's shrink pieces are all in
                signal(a_done_bar);
                a_signalled = true;
            }
            const int acc = it % acc_stages;
            const uint32_t tphase = (uint32_t)((it / acc_stages) & 1);
            float cf[32];
            if (pc.shrink)  // loads overlap the MMAs of this piece
                gate_coefs(pc.t, tok_lane, cf);
            // Wait for this piece's accumulator; meanwhile take a share of the
            // shrink conversion as soon as the converter opens it (the expand
            // steps of every CTA wait for it).
            int ev = 0;
            while (true) {
                if (tid == 0) {
                    const long long t0 = clock64();
                    uint32_t n = 0;
                    ev = 0;
                    while (ev == 0) {
                        if (mbar_try(smem_u32(&tfull_bar[acc]), tphase)) ev = 1;
                        else if (handoff && !sh_joined && *go_shrink != 0) ev = 2;
                        else if ((++n & 1023u) == 0) {
                            if (*(volatile int*)p.err != 0) ev = -1;
                            else if (clock64() - t0 > kSpinLimitCycles) {
                                atomicCAS(p.err, 0, AOS_ERR_TIMEOUT);
                                ev = -1;
                            }
                        }
                    }
                    *flag = ev;
                }
                epi_bar();
                ev = *flag;
                epi_bar();
                if (ev != 2) break;
                join_shrink();
            }
            if (ev < 0) break;
            mbar_wait(smem_u32(&tfull_bar[acc]), tphase, p.err);  // completed: every thread observes it
            if (tr && tid == 0 && it < 32) tr[128 + it] = gtimer();
            tc_fence_after();
            const uint32_t t_acc = tmem_base + lane_off + (uint32_t)(acc * cols_per_acc);
            const int mode = pc.shrink ? TC_SHRINK_HM : p.mode;
            // token held by this thread's TMEM lane in token block b (-1: none)
            auto token_of = [&](int b) -> int { return b * kTcTok + tok_lane; };
            if (pc.n == 1 && pc.shrink) {  // whole shrink tile: gate and store hm from TMEM
                for (int b = 0; b < p.tb; ++b) {
                    const int tok = token_of(b);
                    if (b > 0) gate_coefs(pc.t, tok < 0 ? 0 : tok, cf);
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        float vA[32], vB[32];
                        tmem_ld32(t_acc + b * kTcBN + 64 * k, vA);
                        tmem_ld32(t_acc + b * kTcBN + 64 * k + 32, vB);
#pragma unroll
                        for (int i = 0; i < 32; ++i) {
                            vA[i] *= cf[8 * k + i / 8];
                            vB[i] *= cf[8 * k + 4 + i / 8];
                        }
                        if (tok >= 0 && tok < p.T) apply_pairs<32>(p, mode, pc.seg, pc.t, k, tok, 0, vA, vB, sc.ng);
                    }
                }
            } else if (pc.n == 1) {  // the whole tile is here: epilogue straight from TMEM
                for (int b = 0; b < p.tb; ++b) {
                    const int tok = token_of(b);
                    const float st = (tok >= 0 && tok < p.T) ? token_scale(p, tok) : 1.f;
#pragma unroll 1
                    for (int k = 0; k < 4; ++k) {
                        int cA, cB;
                        chunk_cols(mode, k, cA, cB);
                        float vA[32], vB[32];
                        tmem_ld32(t_acc + b * kTcBN + cA, vA);
                        tmem_ld32(t_acc + b * kTcBN + cB, vB);
                        if (tok >= 0 && tok < p.T) apply_pairs<32>(p, mode, pc.seg, pc.t, k, tok, 0, vA, vB, sc.ng, st);
                    }
                }
            } else {
                // add the piece into the tile's fixed-point accumulator: value * 2^32
                // rounded to int64, summed by atomic adds in L2 (integer addition
                // is order-independent, so the sum is exact and the same on every
                // run); shrink pieces are gated first.  Layout [tile][column][token]:
                // one red instruction adds a column for 32 consecutive tokens.
                const bool to_part = kPart && !pc.shrink;
                for (int b = 0; b < p.tb && to_part; ++b) {  // fp32 partials, plain stores
                    const int tok = token_of(b);
                    const bool valid = tok >= 0 && tok < p.T;
                    float* dst = p.part + (size_t)(blockIdx.x + pc.tile - sc.n_sh) * kTcBN * p.acc_T + (valid ? tok : 0);
#pragma unroll
                    for (int c = 0; c < kTcBN / 32; ++c) {
                        float v[32];
                        tmem_ld32(t_acc + b * kTcBN + c * 32, v);
                        if (!valid) continue;
#pragma unroll
                        for (int i = 0; i < 32; ++i) __stcg(dst + (size_t)(c * 32 + i) * p.acc_T, v[i]);
                    }
                }
                for (int b = 0; b < p.tb && !to_part; ++b) {
                    const int tok = token_of(b);
                    if (b > 0 && pc.shrink) gate_coefs(pc.t, tok < 0 ? 0 : tok, cf);
                    const bool valid = tok >= 0 && tok < p.T;
                    unsigned long long* dst =
                        reinterpret_cast<unsigned long long*>(p.acc) + (size_t)pc.tile * kTcBN * p.acc_T + (valid ? tok : 0);
#pragma unroll
                    for (int c = 0; c < kTcBN / 32; ++c) {
                        float v[32];
                        tmem_ld32(t_acc + b * kTcBN + c * 32, v);
                        if (!valid) continue;
                        if (pc.shrink) {
#pragma unroll
                            for (int i = 0; i < 32; ++i) v[i] *= cf[4 * c + i / 8];
                        }
#pragma unroll
                        for (int i = 0; i < 32; ++i) {
                            // A shrink column whose adapter this token did not
                            // select is gated to exactly zero: adding it would
                            // change nothing, and skipping it keeps the L2
                            // atomic traffic to the token's own adapters.
                            if (pc.shrink && cf[4 * c + i / 8] == 0.f) continue;
                            const long long x = __float2ll_rn(v[i] * kFix);
                            asm volatile("red.global.add.u64 [%0], %1;" ::"l"(dst + (size_t)(c * 32 + i) * p.acc_T),
                                         "l"((unsigned long long)x)
                                         : "memory");
                        }
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_u32(&tempty_bar[acc]));
            if (tr && tid == 0 && it < 32) tr[160 + it] = gtimer();
        }
        // also on the error path: the converter warps wait (bounded) for these
        if (!a_signalled) signal(a_done_bar);
        if (handoff && !sh_joined) {
            const long long t0 = clock64();
            while (*go_shrink == 0)
                if (clock64() - t0 > 2 * kSpinLimitCycles) break;  // the converter's own waits are bounded
            join_shrink();
        }
        signal(all_done_bar);
        // then help with the final conversion once every CTA's pieces are in
        {
            const long long t0 = clock64();
            int go = 0;
            while ((go = *go_final) == 0)
                if (clock64() - t0 > 2 * kSpinLimitCycles) break;  // the converter's own waits are bounded
            if (go == 1) {
                __threadfence();
                if (!handoff) convert(0, sc.n_sh, 192, tid);  // else converted at the hand-off
                convert(sc.n_sh, sc.n_sh + sc.n_base, 192, tid);
            }
        }
    } else {
        // ===================== converter (warps 6-7, 64 threads) =================
        // Grid barriers over all CTAs and the conversion of split tiles: after
        // every CTA's shrink pieces are in, the split shrink tiles' fixed-point
        // sums become gated bf16 hm (then the expand steps may start); after
        // every piece is in, the split base tiles get their epilogue.  Thread
        // cid 0 does the atomics; the other drain and MMA work never waits here.
        const int cid = threadIdx.x - 192;  // 0..63
        pdl_wait();
        auto cv_bar = [] { asm volatile("bar.sync 2, 64;" ::: "memory"); };
        // every converter thread's writes happen before thread 0's release
        auto release = [&](int i) {
            cv_bar();
            if (cid == 0) {
                __threadfence();
                atomicAdd(p.sync + i, 1);
                if (tr) tr[194 + 2 * i] = gtimer();
            }
        };
        // wait (thread 0, bounded) for an smem barrier phase, then for every CTA's arrival at sync[i]
        auto await = [&](uint64_t* bar, int i) -> bool {
            if (cid == 0) {
                bool ok = mbar_wait(smem_u32(bar), 0, p.err);
                if (ok && i >= 0) {
                    __threadfence();
                    atomicAdd(p.sync + i, 1);
                    if (tr) tr[194 + 2 * i] = gtimer();
                    ok = spin_ge(p.sync + i, (int)gridDim.x, p.err);
                    if (ok && tr) tr[195 + 2 * i] = gtimer();
                }
                *flag = ok ? 1 : 0;
            }
            cv_bar();
            const bool ok = *flag != 0;
            cv_bar();
            if (ok) __threadfence();
            return ok;
        };
        bool ok = true;
        // Without expand steps in this launch nothing waits for hm here: the
        // shrink tiles are converted with the base tiles after one barrier.
        if (handoff) {
            ok = await(a_done_bar, 0);
            if (cid == 0) *go_shrink = ok ? 1 : -1;  // the drain warps take two thirds
            if (ok) {
                convert(0, sc.n_sh, 192, 128 + cid);
                if (tr && cid == 0) tr[206] = gtimer();
                if (cid == 0) ok = mbar_wait(smem_u32(sh_conv_bar), 0, p.err);
                if (tr && cid == 0) tr[207] = gtimer();
                cv_bar();
                release(1);
            }
        }
        ok = ok && await(all_done_bar, 2);
        if (cid == 0) *go_final = ok ? 1 : -1;  // the drain warps join the final conversion
        if (ok) {
            if (tr && cid == 0) tr[200] = gtimer();
            if (!handoff) convert(0, sc.n_sh, 192, 128 + cid);  // else converted at the hand-off
            convert(sc.n_sh, sc.n_sh + sc.n_base, 192, 128 + cid);
            if (tr && cid == 0) tr[201] = gtimer();
        }
    }

    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (threadIdx.x == 0) {
        if (tr) tr[193] = gtimer();
        // the last CTA to leave resets the launch's grid-barrier counters
        __threadfence();
        const int old = atomicAdd(p.sync + 3, 1);
        if (old == (int)gridDim.x - 1) {
            p.sync[0] = 0;
            p.sync[1] = 0;
            p.sync[2] = 0;
            p.sync[3] = 0;
            // every CTA has read the folded norm's sums: clear them for the
            // launch that accumulates the next ones
            if (p.ss_in)
                for (int i = 0; i < p.T; ++i) p.ss_in[i] = 0ull;
            __threadfence();
        }
    }
    if (warp == 1)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(tmem_cols));
}

// ---------------------------------------------------------------- prefill GEMM
// Prompt-sized token counts (prefill) have enough output tiles to fill the GPU
// without cutting K: every tile of 256 tokens (two MMA M blocks of 128) x 256
// weight rows (MMA N) is one CTA iteration over the whole K -- the base K
// steps, then the LoRA expand steps of every touched rank group -- so the
// epilogue runs straight from TMEM and nothing is reduced across CTAs.  Two
// token blocks share each weight box: a step is 32 KB of weights plus 32 KB of
// activations for eight MMAs, which halves the L2 bytes per MMA of a
// 128-token tile.  The 256 x 256 fp32 accumulator takes all 512 TMEM columns,
// so the MMA waits while a tile drains (about a tenth of the launch time at
// 8B shapes).  The drain is kept short by eight drain warps (one per lane
// quarter and 128-token block) and by stores staged through a per-warp slab.
// Persistent CTAs walk the tiles in bands of kPfBand token tiles per weight
// tile, so the tiles running at the same time share boxes in L2.
// Gate/up expand steps come in halves (gate rows, then up rows, N = 128 each),
// so every stage has the same size.  A shrink launch (p.n_seg == 0,
// p.sh_nseg > 0) has tiles of 256 tokens x four touched rank groups of one
// LoRA module and writes the gated hm (bf16).
constexpr int kPfBand = 8;
constexpr int kPfTok = 2 * kTcTok;  // tokens per tile

struct PfTile {
    int m;              // token tile (256 tokens)
    int seg, t;         // segment and tile within it (shrink: module and group quad)
    bool shrink;
};

__device__ __forceinline__ void pf_tile(const TcParams& p, int n_m, int n_n, int ng, int it, PfTile& pt) {
    const int band = it / (kPfBand * n_n), in = it % (kPfBand * n_n);
    const int bm = min(kPfBand, n_m - band * kPfBand);
    const int n = in / bm;
    pt.m = band * kPfBand + in % bm;
    if (p.n_seg == 0) {
        const int per = cdiv(ng, kShrinkGroupsPerTile);
        pt.shrink = true;
        pt.seg = n / per;
        pt.t = n % per;
    } else {
        int b = n, g = 0;
        while (g < p.n_seg - 1 && b >= p.seg_tiles[g]) {
            b -= p.seg_tiles[g];
            ++g;
        }
        pt.shrink = false;
        pt.seg = g;
        pt.t = b;
    }
}

// Prefill epilogue rows through a per-warp shared-memory slab of 32 rows x 64
// bytes.  A drain lane holds one token's run of 32 bf16 (64 bytes); stored by
// its own lane, one warp instruction would touch 32 rows.  Transposed through
// the slab, lane (j, c) = (lane / 4, lane % 4) moves 16-byte chunk c of row
// 8 r + j, so one instruction covers 8 rows x 64 contiguous bytes.  Chunk i of
// slab row r sits at chunk i ^ ((r / 2) % 4): both directions are free of bank
// conflicts.  row_of(r) is row r's destination (or source), null to skip it.
constexpr int kPfSlabBytes = 32 * 64;
constexpr int kPfEpiBytes = 8 * kPfSlabBytes;  // one slab per drain warp
__device__ __forceinline__ uint32_t slab_off(int row, int chunk) {
    return (uint32_t)(row * 64 + ((chunk ^ ((row >> 1) & 3)) * 16));
}
template <class RowFn>
__device__ __forceinline__ void warp_store_runs(uint8_t* slab, const uint32_t (&w)[16], int lane, RowFn row_of) {
#pragma unroll
    for (int i = 0; i < 4; ++i)
        *reinterpret_cast<uint4*>(slab + slab_off(lane, i)) = make_uint4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
    __syncwarp();
    const int j = lane >> 2, c = lane & 3;
#pragma unroll
    for (int r = 0; r < 4; ++r) {
        const int row = 8 * r + j;
        const uint4 v = *reinterpret_cast<const uint4*>(slab + slab_off(row, c));
        uint16_t* dst = row_of(row);
        if (dst) *reinterpret_cast<uint4*>(dst + 8 * c) = v;
    }
    __syncwarp();
}
// The inverse: lane L receives row L's run (zeros for a skipped row).
template <class RowFn>
__device__ __forceinline__ void warp_load_runs(uint8_t* slab, uint32_t (&w)[16], int lane, RowFn row_of) {
    const int j = lane >> 2, c = lane & 3;
#pragma unroll
    for (int r = 0; r < 4; ++r) {
        const int row = 8 * r + j;
        const uint16_t* src = row_of(row);
        const uint4 v = src ? *reinterpret_cast<const uint4*>(src + 8 * c) : make_uint4(0u, 0u, 0u, 0u);
        *reinterpret_cast<uint4*>(slab + slab_off(row, c)) = v;
    }
    __syncwarp();
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const uint4 v = *reinterpret_cast<const uint4*>(slab + slab_off(lane, i));
        w[4 * i] = v.x;
        w[4 * i + 1] = v.y;
        w[4 * i + 2] = v.z;
        w[4 * i + 3] = v.w;
    }
    __syncwarp();
}
__device__ __forceinline__ void pack_bf16_run(const float (&v)[32], uint32_t (&w)[16]) {
#pragma unroll
    for (int i = 0; i < 16; ++i) w[i] = (uint32_t)f2bf(v[2 * i]) | ((uint32_t)f2bf(v[2 * i + 1]) << 16);
}

// Warps: 0 producer, 1 MMA issuer, 2-9 drain (two per TMEM lane quarter: warps
// 2-5 take a tile's first 128 tokens, warps 6-9 its second), 10-11 idle.
constexpr int kPfThreads = 384;
__global__ void __launch_bounds__(kPfThreads, 1) pf_gemm_kernel(const __grid_constant__ TcParams p) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int NS = p.n_stages;
    uint8_t* stages = smem;
    uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + (size_t)NS * p.stage_bytes);
    uint64_t* empty_bar = full_bar + NS;
    uint64_t* tfull_bar = empty_bar + NS;  // [1]
    uint64_t* tempty_bar = tfull_bar + 1;  // [1]
    uint64_t* drain_bar = tempty_bar + 1;  // [1]
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain_bar + 1);
    // after the barriers: the drain warps' slabs (kPfSlabBytes each, warps 2-9)
    uint8_t* epi = smem + (size_t)NS * p.stage_bytes + kTcTailBytes;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int ng = (p.lora || p.sh_nseg) ? __ldg(p.n_groups) : 0;
    const int n_m = cdiv(p.T, kPfTok);
    int n_n = 0;
    if (p.n_seg == 0) {
        n_n = p.sh_nseg * cdiv(ng, kShrinkGroupsPerTile);
    } else {
        for (int g = 0; g < p.n_seg; ++g) n_n += p.seg_tiles[g];
    }
    const int n_tiles = n_m * n_n;
    const int ex_per_group = p.n_sub == 2 ? 2 : 1;  // gate/up: gate half, then up half
    const int nge = (p.n_seg > 0 && p.lora) ? ng * ex_per_group : 0;
    const int steps = p.kb + nge;

    if (threadIdx.x == 0) {
        for (int s = 0; s < NS; ++s) {
            mbar_init(smem_u32(&full_bar[s]), 1);
            mbar_init(smem_u32(&empty_bar[s]), 1);
        }
        mbar_init(smem_u32(tfull_bar), 1);
        mbar_init(smem_u32(tempty_bar), 8);
        mbar_init(smem_u32(drain_bar), 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(512));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    constexpr uint32_t kBlkW = kBlkRows * kTcBK;
    constexpr uint32_t kBlkA = kGroup * kTcBK;
    constexpr uint32_t kActBox = kTcTok * 128;

    if (warp == 0) {
        // ---------------- producer
        if (lane == 0) {
            const uint64_t pol_w = policy_evict_last();  // weights are re-read by the other token tiles
            const uint64_t pol_x = policy_evict_last();
            int stage = 0;
            uint32_t phase = 0;
            uint32_t last_phase[16];
            uint32_t used = 0;
            bool ok = true, waited = false;
            // A base launch with LoRA runs right after its own shrink launch,
            // which waited for the launch that wrote X before it let this one
            // start: X can be read at once, and only the expand steps' hm
            // (the shrink's output) waits for the previous grid.  The base
            // K steps then start on the SMs the shrink's last wave leaves.
            const bool x_ready = p.n_seg > 0 && p.lora;
            for (int it = blockIdx.x; ok && it < n_tiles; it += gridDim.x) {
                PfTile pt;
                pf_tile(p, n_m, n_n, ng, it, pt);
                const int nsteps = pt.shrink ? p.kb : steps;
                const int seg_blocks = pt.shrink ? 0 : (p.seg_rows[pt.seg] + kBlkRows - 1) / kBlkRows;
                for (int st = 0; st < nsteps; ++st) {
                    if (!mbar_wait(smem_u32(&empty_bar[stage]), phase ^ 1u, p.err)) { ok = false; break; }
                    const uint32_t fb = smem_u32(&full_bar[stage]);
                    const uint32_t sb = smem_u32(stages + (size_t)stage * p.stage_bytes);
                    const bool ex = !pt.shrink && st >= p.kb;
                    const int e = st - p.kb;
                    const int gi = ex ? e / ex_per_group : 0;  // touched-group list index
                    const int hh = (ex && p.n_sub == 2) ? e % 2 : -1;  // gate/up expand half
                    uint32_t bytes = 2 * kActBox;
                    if (pt.shrink) {
                        const int first = pt.t * kShrinkGroupsPerTile;
                        bytes += (uint32_t)min(kShrinkGroupsPerTile, ng - first) * kBlkA * 2;
                    } else if (hh >= 0) {
                        bytes += kBlkW * 2;
                    } else if (p.n_sub == 2) {
                        bytes += 2 * kBlkW * 2;
                    } else {
                        bytes += (uint32_t)min(2, seg_blocks - 2 * pt.t) * kBlkW * 2;
                    }
                    mbar_expect_tx(fb, bytes);
                    if (pt.shrink) {
                        const int first = pt.t * kShrinkGroupsPerTile;
                        const int nv = min(kShrinkGroupsPerTile, ng - first);
                        for (int q = 0; q < nv; ++q)
                            bulk_g2s(sb + q * (kBlkA * 2),
                                     p.a_pk[pt.seg] + ((size_t)__ldg(p.groups + first + q) * p.kb + st) * kBlkA, kBlkA * 2,
                                     fb, pol_w);
                    } else if (hh >= 0) {  // one 128-row block of lora_B (gate or up)
                        const int g = __ldg(p.groups + gi);
                        bulk_g2s(sb, p.b_pk[pt.seg * 2 + hh] + ((size_t)pt.t * p.n_rgroups + g) * kBlkW, kBlkW * 2, fb,
                                 pol_w);
                    } else {
                        const int g = ex ? __ldg(p.groups + gi) : 0;
                        for (int h = 0; h < 2; ++h) {
                            const uint16_t* src;
                            if (p.n_sub == 2) {
                                src = p.w_pk[pt.seg * 2 + h] +
                                      (((size_t)(p.seg_wrow0[pt.seg] / kBlkRows + pt.t)) * p.kb + st) * kBlkW;
                            } else {
                                if (2 * pt.t + h >= seg_blocks) continue;
                                src = !ex ? p.w_pk[pt.seg] +
                                                (((size_t)(p.seg_wrow0[pt.seg] / kBlkRows + 2 * pt.t + h)) * p.kb + st) * kBlkW
                                          : p.b_pk[pt.seg] + ((size_t)(2 * pt.t + h) * p.n_rgroups + g) * kBlkW;
                            }
                            bulk_g2s(sb + h * (kBlkW * 2), src, kBlkW * 2, fb, pol_w);
                        }
                    }
                    if (!waited && (!x_ready || ex)) {  // this step reads the previous launch's output
                        pdl_wait();
                        pdl_trigger();
                        waited = true;
                    }
                    const uint32_t act = sb + p.act_off;
                    for (int b = 0; b < 2; ++b) {
                        if (!ex) {
                            tma_2d(&p.tm_x, act + b * kActBox, fb, st * kTcBK, pt.m * kPfTok + b * kTcTok, pol_x);
                        } else {
                            const int gcol = __ldg(p.groups + gi) * kGroup;
                            const int map = pt.seg * p.n_sub + (hh >= 0 ? hh : 0);
                            tma_2d(&p.tm_lh[map], act + b * kActBox, fb, gcol, pt.m * kPfTok + b * kTcTok, pol_x);
                        }
                    }
                    last_phase[stage] = phase;
                    used |= 1u << stage;
                    if (++stage == NS) { stage = 0; phase ^= 1u; }
                }
            }
            if (!waited) {
                pdl_wait();
                pdl_trigger();
            }
            for (int s = 0; s < NS; ++s)
                if (used & (1u << s)) mbar_wait_drain(smem_u32(&full_bar[s]), last_phase[s]);
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer
        if (lane == 0) {
            const uint32_t idesc256 = idesc_bf16(kTcBN), idesc128 = idesc_bf16(kTcBN / 2);
            int stage = 0;
            uint32_t phase = 0;
            bool ok = true, issued = false;
            int local = 0;
            for (int it = blockIdx.x; ok && it < n_tiles; it += gridDim.x, ++local) {
                PfTile pt;
                pf_tile(p, n_m, n_n, ng, it, pt);
                if (!mbar_wait(smem_u32(tempty_bar), (uint32_t)((local & 1) ^ 1), p.err)) { ok = false; break; }
                tc_fence_after();
                const int nsteps = pt.shrink ? p.kb : steps;
                for (int st = 0; st < nsteps; ++st) {
                    if (!mbar_wait(smem_u32(&full_bar[stage]), phase, p.err)) { ok = false; break; }
                    tc_fence_after();
                    const uint32_t sb = smem_u32(stages + (size_t)stage * p.stage_bytes);
                    const uint32_t act = sb + p.act_off;
                    const bool ex = !pt.shrink && st >= p.kb;
                    const int hh = (ex && p.n_sub == 2) ? (st - p.kb) % 2 : -1;
                    for (int b = 0; b < 2; ++b) {
                        const uint32_t a0 = act + b * kActBox, d = tmem_base + (uint32_t)(b * kTcBN);
                        if (hh >= 0) {
#pragma unroll
                            for (int kk = 0; kk < kTcBK / 16; ++kk)
                                umma_bf16(d + hh * (kTcBN / 2), desc_sw128(a0 + kk * 32), desc_sw128(sb + kk * 32), idesc128,
                                          1u);
                        } else {
#pragma unroll
                            for (int kk = 0; kk < kTcBK / 16; ++kk)
                                umma_bf16(d, desc_sw128(a0 + kk * 32), desc_sw128(sb + kk * 32), idesc256,
                                          (st == 0 && kk == 0) ? 0u : 1u);
                        }
                    }
                    issued = true;
                    umma_commit(smem_u32(&empty_bar[stage]));
                    if (++stage == NS) { stage = 0; phase ^= 1u; }
                }
                if (!ok) break;
                umma_commit(smem_u32(tfull_bar));
            }
            if (!ok && issued) {
                umma_commit(smem_u32(drain_bar));
                mbar_wait_drain(smem_u32(drain_bar), 0);
            }
        }
    } else if (warp < 10) {
        // ---------------- drain + epilogue from TMEM (warps 2-9): token block b
        const int q = warp & 3, b = (warp - 2) >> 2;
        const uint32_t lane_off = (uint32_t)(q * 32) << 16;
        pdl_wait();
        int local = 0;
        for (int it = blockIdx.x; it < n_tiles; it += gridDim.x, ++local) {
            PfTile pt;
            pf_tile(p, n_m, n_n, ng, it, pt);
            // warp-uniform: the epilogue's slab transposes need all 32 lanes
            const bool got = mbar_wait(smem_u32(tfull_bar), (uint32_t)(local & 1), p.err);
            if (!__all_sync(0xffffffffu, got)) break;
            tc_fence_after();
            {
                const uint32_t t_acc = tmem_base + lane_off + (uint32_t)(b * kTcBN);
                const int tok = pt.m * kPfTok + b * kTcTok + q * 32 + lane;
                const bool valid = tok < p.T;
                // rows [tok0, tok0 + 32) of the tile are this warp's; the staged
                // stores (and the residual's loads) skip rows at or past T
                const int tok0 = tok - lane;
                uint8_t* slab = epi + (warp - 2) * kPfSlabBytes;
                const bool staged = !p.delta && !p.ss_out && !p.ss_in;
                if (pt.shrink) {
                    float cf[32];
                    const float4* src = reinterpret_cast<const float4*>(
                        p.ucoef + ((size_t)(valid ? tok : 0) * p.n_rgroups + (size_t)pt.t * kShrinkGroupsPerTile) * 8);
#pragma unroll
                    for (int j = 0; j < 8; ++j) {
                        const float4 w = __ldg(src + j);
                        cf[4 * j] = w.x;
                        cf[4 * j + 1] = w.y;
                        cf[4 * j + 2] = w.z;
                        cf[4 * j + 3] = w.w;
                    }
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        float vA[32], vB[32];
                        tmem_ld32(t_acc + 64 * k, vA);
                        tmem_ld32(t_acc + 64 * k + 32, vB);
#pragma unroll
                        for (int i = 0; i < 32; ++i) {
                            vA[i] *= cf[8 * k + i / 8];
                            vB[i] *= cf[8 * k + 4 + i / 8];
                        }
                        const int slot = pt.t * kShrinkGroupsPerTile + k;
                        if (slot >= ng) continue;
                        // hm[t][group column + 0..63]: two runs of 32 (see shrink_run)
                        uint16_t* hm = reinterpret_cast<uint16_t*>(p.sh_out[pt.seg]) + __ldg(p.groups + slot) * kGroup;
                        uint32_t w[16];
                        pack_bf16_run(vA, w);
                        warp_store_runs(slab, w, lane, [&](int r) -> uint16_t* {
                            return tok0 + r < p.T ? hm + (size_t)(tok0 + r) * p.R : nullptr;
                        });
                        pack_bf16_run(vB, w);
                        warp_store_runs(slab, w, lane, [&](int r) -> uint16_t* {
                            return tok0 + r < p.T ? hm + (size_t)(tok0 + r) * p.R + 32 : nullptr;
                        });
                    }
                } else {
#pragma unroll 1
                    for (int k = 0; k < 4; ++k) {
                        int cA, cB;
                        chunk_cols(p.mode, k, cA, cB);
                        float vA[32], vB[32];
                        tmem_ld32(t_acc + cA, vA);
                        tmem_ld32(t_acc + cB, vB);
                        const int lim = p.seg_rows[pt.seg];
                        if (staged && p.mode == TC_SWIGLU && pt.t * (kTcBN / 2) + cA + 32 <= lim) {
                            // act[t][f0 + 0..31] = silu(gate) * up
                            uint16_t* o = reinterpret_cast<uint16_t*>(p.out[pt.seg]) + pt.t * (kTcBN / 2) + cA;
                            float sv[32];
                            swiglu_run<32>(vA, vB, sv);
                            uint32_t w[16];
                            pack_bf16_run(sv, w);
                            warp_store_runs(slab, w, lane, [&](int r) -> uint16_t* {
                                return tok0 + r < p.T ? o + (size_t)(tok0 + r) * p.ld_out : nullptr;
                            });
                        } else if (staged && p.mode == TC_RESID_BF16) {
                            // h[t][r0 + 0..31] += v for the two runs, h read and written
                            // through the slab; rows that end past the segment go per lane
#pragma unroll
                            for (int hh = 0; hh < 2; ++hh) {
                                const int r0 = pt.t * kTcBN + (hh ? cB : cA);
                                const float(&v)[32] = hh ? vB : vA;
                                if (r0 + 32 <= lim) {
                                    uint16_t* h = p.resid + p.seg_out0[pt.seg] + r0;
                                    auto row_of = [&](int r) -> uint16_t* {
                                        return tok0 + r < p.T ? h + (size_t)(tok0 + r) * p.ld_out : nullptr;
                                    };
                                    uint32_t w[16];
                                    warp_load_runs(slab, w, lane, row_of);
#pragma unroll
                                    for (int i = 0; i < 16; ++i)
                                        w[i] = (uint32_t)f2bf(bf2f((uint16_t)(w[i] & 0xFFFFu)) + v[2 * i]) |
                                               ((uint32_t)f2bf(bf2f((uint16_t)(w[i] >> 16)) + v[2 * i + 1]) << 16);
                                    warp_store_runs(slab, w, lane, row_of);
                                } else if (valid && r0 < lim) {
                                    store_run<32>(p, TC_RESID_BF16, pt.seg, tok, r0, v);
                                }
                            }
                        } else if (staged && p.mode == TC_QKV_ROPE) {
                            // RoPE of dims d, d + 64 of one head (see apply_pairs); the
                            // two runs go to q, or to the token's paged K/V row
                            const int module = p.seg_module[pt.seg];
                            const int head = pt.t * 2 + (cA >> 7);
                            if (head * 128 >= lim) continue;
                            const int d = cA & 127;
                            float a[32], bv[32];
                            if (module != AOS_MOD_V) {
                                const int pos = valid ? __ldg(p.ctx_lens + tok) : 0;
                                rope_run<32>(vA, vB, reinterpret_cast<const float2*>(p.rope) + (size_t)pos * 64 + d, a, bv);
                            } else {
#pragma unroll
                                for (int i = 0; i < 32; ++i) {
                                    a[i] = vA[i];
                                    bv[i] = vB[i];
                                }
                            }
                            auto row_of = [&](int r) -> uint16_t* {
                                const int tk = tok0 + r;
                                if (tk >= p.T) return nullptr;
                                if (module == AOS_MOD_Q)
                                    return reinterpret_cast<uint16_t*>(p.out[pt.seg]) + (size_t)tk * p.ld_out + head * 128 + d;
                                const int pos = __ldg(p.ctx_lens + tk);
                                const int blk = __ldg(p.block_tables + (size_t)tk * p.max_blocks + (pos >> 4));
                                uint16_t* pool = module == AOS_MOD_K ? p.k_pool : p.v_pool;
                                return pool + ((((size_t)p.layer * p.num_blocks + blk) * p.nkv + head) * 16 + (pos & 15)) * 128 + d;
                            };
                            uint32_t w[16];
                            pack_bf16_run(a, w);
                            warp_store_runs(slab, w, lane, row_of);
                            pack_bf16_run(bv, w);
                            warp_store_runs(slab, w, lane, [&](int r) -> uint16_t* {
                                uint16_t* dst = row_of(r);
                                return dst ? dst + 64 : nullptr;
                            });
                        } else if (valid) {
                            apply_pairs<32>(p, p.mode, pt.seg, pt.t, k, tok, 0, vA, vB, ng);
                        }
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_u32(tempty_bar));
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(512));
}

// Runs one of the GEMM kernel's bounded waits against a condition that never
// comes true, so that its time limit is what ends it: kind 0 spins on a
// global counter that nothing increments (the grid barriers' spin_ge), kind 1
// waits on a shared-memory mbarrier that nothing arrives on (the pipeline's
// mbar_wait).  Either returns after kSpinLimitCycles with AOS_ERR_TIMEOUT in
// *err, as a real stalled wait would.
__global__ void debug_wait_kernel(int kind, const int* never, int* err) {
    __shared__ __align__(8) uint64_t bar;
    if (threadIdx.x != 0) return;
    if (kind == 0) {
        spin_ge(never, 1, err);
    } else {
        mbar_init(smem_u32(&bar), 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        mbar_wait(smem_u32(&bar), 0, err);
    }
}

}  // namespace

cudaError_t tc_debug_wait(int kind, const int* never, int* err, cudaStream_t s) {
    debug_wait_kernel<<<1, 32, 0, s>>>(kind, never, err);
    return cudaGetLastError();
}

// ---------------------------------------------------------------- host side
namespace {
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    if (!fn) {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(f);
    }
    return fn;
}

CUtensorMapSwizzle swz(int bytes) {
    switch (bytes) {
        case 128: return CU_TENSOR_MAP_SWIZZLE_128B;
        case 64: return CU_TENSOR_MAP_SWIZZLE_64B;
        case 32: return CU_TENSOR_MAP_SWIZZLE_32B;
        default: return CU_TENSOR_MAP_SWIZZLE_NONE;
    }
}

}  // namespace

int tc_encode_2d(CUtensorMap* m, const void* base, uint64_t inner, uint64_t outer, uint64_t row_bytes,
                 uint32_t box_inner, uint32_t box_outer, int swizzle_bytes) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return AOS_ERR_CUDA;
    if ((reinterpret_cast<uintptr_t>(base) & 15) || (row_bytes & 15) || ((box_inner * 2) & 15)) return AOS_ERR_INVALID;
    cuuint64_t dims[2] = {inner, outer};
    cuuint64_t strides[1] = {row_bytes};
    cuuint32_t box[2] = {box_inner, box_outer};
    cuuint32_t es[2] = {1, 1};
    CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, es,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, swz(swizzle_bytes), CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? AOS_OK : AOS_ERR_CUDA;
}

int tc_encode_3d(CUtensorMap* m, const void* base, uint64_t d0, uint64_t d1, uint64_t d2, uint64_t stride1_bytes,
                 uint64_t stride2_bytes, uint32_t b0, uint32_t b1, uint32_t b2, int swizzle_bytes) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return AOS_ERR_CUDA;
    if ((reinterpret_cast<uintptr_t>(base) & 15) || (stride1_bytes & 15) || (stride2_bytes & 15)) return AOS_ERR_INVALID;
    cuuint64_t dims[3] = {d0, d1, d2};
    cuuint64_t strides[2] = {stride1_bytes, stride2_bytes};
    cuuint32_t box[3] = {b0, b1, b2};
    cuuint32_t es[3] = {1, 1, 1};
    CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, es,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, swz(swizzle_bytes), CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? AOS_OK : AOS_ERR_CUDA;
}

size_t tc_tail_bytes(const TcParams&) { return kTcTailBytes; }  // mbarriers and flags
int tc_max_dynamic_smem();


size_t tc_smem_bytes(const TcParams& p) {
    return 1024 + (size_t)p.n_stages * p.stage_bytes + tc_tail_bytes(p);
}

int tc_prepare(TcParams& p, int smem_budget) {
    if (p.T <= 0 || p.T > 256 || p.n_sub < 1 || p.n_sub > 2 || p.n_seg < 1 || p.n_seg > kTcMaxSets ||
        p.n_seg * p.n_sub > kTcMaxSets || p.sh_nseg < 0 || p.sh_nseg > kTcMaxSets || p.kb < 1)
        return AOS_ERR_INVALID;
    {  // the device schedule computes pool positions x grid in 32 bits
        long long tiles = p.sh_nseg * ((long long)p.n_rgroups / kShrinkGroupsPerTile + 1);
        for (int g = 0; g < p.n_seg; ++g) tiles += p.seg_tiles[g];
        if (tiles * (p.kb + (long long)p.n_rgroups + 1) * tc_num_sms() >= (1ll << 31)) return AOS_ERR_INVALID;
    }
    p.T_pad = tc_t_pad(p.T);
    p.T_box = tc_t_box(p.T);
    p.tb = (p.T_pad + kTcTok - 1) / kTcTok;
    // stage: 256 weight rows x 128 B, then one 128-row activation box per
    // token block (two for the gate/up expand, whose halves read different hm)
    const int n_act = p.tb * ((p.n_sub == 2 && p.lora) ? 2 : 1);
    p.act_off = (uint32_t)kTcBN * 128;
    p.stage_bytes = p.act_off + (uint32_t)n_act * kTcTok * 128;
    const size_t fixed = 1024 + tc_tail_bytes(p);
    smem_budget = std::min(smem_budget, tc_max_dynamic_smem());
    int ns = (int)((smem_budget - (int)fixed) / (int)p.stage_bytes);
    static const int max_stages = [] {
        const char* e = getenv("AOS_TC_MAX_STAGES");  // tuning knob, default 4
        const int v = e ? atoi(e) : 4;
        return v < 2 ? 2 : (v > 16 ? 16 : v);
    }();
    ns = std::min(ns, max_stages);
    if (ns < 2) return AOS_ERR_INVALID;
    p.n_stages = ns;
    return AOS_OK;
}

int tc_num_sms() {
    static int n = 0;
    if (!n) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        if (n <= 0) n = 148;
    }
    return n;
}

// Opt the kernel in to the full 227 KB of shared memory (once per device,
// outside any stream capture).
// The dynamic budget is the device's opt-in limit minus the kernel's static
// shared memory (its work table).
static int g_tc_max_dyn = 0;
cudaError_t tc_configure() {
    int dev = 0, optin = 0;
    cudaFuncAttributes fa{};
    cudaError_t e = cudaGetDevice(&dev);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    if (e == cudaSuccess) e = cudaFuncGetAttributes(&fa, tc_gemm_kernel<false>);
    if (e != cudaSuccess) return e;
    g_tc_max_dyn = optin - (int)fa.sharedSizeBytes;
    e = cudaFuncSetAttribute(tc_gemm_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, g_tc_max_dyn);
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(tc_gemm_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, g_tc_max_dyn);
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(pf_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, g_tc_max_dyn);
    if (e != cudaSuccess) return e;
    // The decode GEMM's grid (one CTA per SM) waits on itself at its grid
    // barriers: every SM must hold one CTA at the largest shared-memory size.
    for (auto* k : {tc_gemm_kernel<false>, tc_gemm_kernel<true>}) {
        int per_sm = 0;
        e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k, kTcThreads, (size_t)g_tc_max_dyn);
        if (e != cudaSuccess) return e;
        if (per_sm < 1) return cudaErrorCooperativeLaunchTooLarge;
    }
    return cudaSuccess;
}
int tc_max_dynamic_smem() { return g_tc_max_dyn > 0 ? g_tc_max_dyn : 227 * 1024 - 4096; }

size_t tc_acc_bytes(const TcParams& p, int n_tiles) {
    return (size_t)n_tiles * kTcBN * p.acc_T * sizeof(long long);
}

// Prefill GEMM (pf_gemm_kernel): same operand layout as the decode GEMM, any
// T; stages of 256 weight rows x 128 B plus two 128-token activation boxes.
int pf_prepare(TcParams& p) {
    if (p.T <= 0 || p.n_sub < 1 || p.n_sub > 2 || p.n_seg < 0 || p.n_seg > kTcMaxSets ||
        p.n_seg * p.n_sub > kTcMaxSets || p.sh_nseg < 0 || p.sh_nseg > kTcMaxSets || p.kb < 1 ||
        (p.n_seg == 0 && p.sh_nseg == 0))
        return AOS_ERR_INVALID;
    p.T_box = kTcTok;
    p.tb = 2;
    p.act_off = (uint32_t)kTcBN * 128;
    p.stage_bytes = p.act_off + 2u * kTcTok * 128;  // 32 KB weights + two 128-token boxes
    const int budget = tc_max_dynamic_smem() - 1024 - (int)kTcTailBytes - kPfEpiBytes;
    p.n_stages = std::min(4, budget / (int)p.stage_bytes);
    return p.n_stages >= 2 ? AOS_OK : AOS_ERR_INVALID;
}

cudaError_t pf_launch(const TcParams& p, cudaStream_t stream) {
    const size_t smem = tc_smem_bytes(p) + kPfEpiBytes;
    if ((int)smem > tc_max_dynamic_smem()) return cudaErrorInvalidValue;
    return launch_k(pf_gemm_kernel, dim3(tc_num_sms()), dim3(kPfThreads), smem, stream, p);
}

cudaError_t tc_launch(const TcParams& p, int grid, cudaStream_t stream) {
    const size_t smem = tc_smem_bytes(p);
    if ((int)smem > tc_max_dynamic_smem()) return cudaErrorInvalidValue;
    // The grid barriers need every CTA resident (one per SM).  On a device
    // the context has to itself that holds by construction; in shared-device
    // mode (p.cooperative) the launch asks for it, at the cost of the overlap
    // with the neighbouring launches.
    const bool coop = p.cooperative != 0;
    if (p.part) return launch_k_ex(coop, tc_gemm_kernel<true>, dim3(grid), dim3(kTcThreads), smem, stream, p);
    return launch_k_ex(coop, tc_gemm_kernel<false>, dim3(grid), dim3(kTcThreads), smem, stream, p);
}

}  // namespace aos
