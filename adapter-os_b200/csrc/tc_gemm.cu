// tc_gemm.cu — tcgen05/TMEM/TMA weight-streaming GEMM with the LoRA shrink
// and expand fused into the same launch, and the decoder's epilogues.
//
// One launch computes, for one input X (normed hidden, attention output or
// SwiGLU activation):
//   shrink tiles : hm[t, group cols] = gate(t, owner) * (A_cat[group rows] . x_t)
//                  for every touched 64-column rank group of every LoRA module
//                  that reads X (TC_SHRINK_HM epilogue);
//   base tiles   : W[128 rows] . X^T  +  sum over touched groups of
//                  B_cat[128 rows, group cols] . hm[group cols]^T
// so a base tile's accumulator ends as  W x + sum_a B_a (g_a * scale_a * A_a x)
// (mlx_cpp_wrapper_real.cpp:3372-3419) without materialising the LoRA delta.
// MMA M = 128 weight rows, N = decode tokens ("swap-AB").
//   K step      : TMA W[128 x 64] (or two lora_A group boxes [64 x 64]) + X[T x 64]
//   expand step : TMA lora_B[128 rows x one group] + hm[T x the same group]
// all SWIZZLE_128B, four K=16 MMAs per step and sub-tile.
//
// Roles (192 threads, one CTA per SM, grid = SM count):
//   warp 0      : TMA producer (one elected lane)
//   warp 1      : TMEM allocator + MMA issuer (one elected lane)
//   warps 2..5  : epilogue, TMEM lane quarter = warp % 4
// Work is split stream-K style (see "schedule" below): every CTA streams the
// same number of steps, a tile cut between CTAs is finished by the last piece
// to arrive, which sums the pieces' fp32 partials in piece order (fixed order,
// so the result is bit-identical run to run; no float atomics).  Expand steps
// wait until every shrink tile of the launch has been written.
//
// Every wait is bounded (kSpinLimitCycles): on timeout the kernel records
// AOS_ERR_TIMEOUT in p.err, drains its own TMA copies and MMAs, frees TMEM and
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
// Barrier over the 4 epilogue warps that also ORs a predicate, so a failed
// (timed-out) wait in any thread makes every epilogue thread leave together.
__device__ __forceinline__ bool epi_bar_any(bool pred) {
    uint32_t r;
    asm volatile(
        "{\n .reg .pred p, q;\n setp.ne.u32 p, %1, 0;\n bar.red.or.pred q, 1, 128, p;\n selp.u32 %0, 1, 0, q;\n}\n"
        : "=r"(r)
        : "r"((uint32_t)pred)
        : "memory");
    return r != 0;
}

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


// ---------------------------------------------------------------- epilogue
struct EpiSmem {
    float* xbuf;  // [128][33] exchange buffer (RoPE)
};

// Apply the epilogue to tokens [t0, t0+32) of one tile row.  v[sub][j] holds
// the fp32 accumulator for token t0 + j.  Must be called uniformly by all
// 128 epilogue threads (RoPE uses a named barrier).  Every loop is fully
// unrolled with predicates, and all loads of a chunk are issued before its
// stores, so a chunk costs one or two memory latencies, not 32.
__device__ __forceinline__ void epilogue_chunk(const TcParams& p, const EpiSmem& es, int mode, int seg, int tile,
                                               void* out_base, int ng, int row, int t0, float (&v)[2][32]) {
    const int col = p.seg_out0[seg] + tile * kTcBM + row;
    if (mode != TC_SHRINK_HM && mode != TC_QKV_ROPE && tile * kTcBM + row >= p.seg_rows[seg]) return;
    const int nt = min(32, p.T - t0);  // valid tokens in this chunk
    switch (mode) {
        case TC_STORE_BF16: {
            uint16_t* o = reinterpret_cast<uint16_t*>(out_base) + (size_t)t0 * p.ld_out + col;
#pragma unroll
            for (int j = 0; j < 32; ++j)
                if (j < nt) o[(size_t)j * p.ld_out] = f2bf(v[0][j]);
            break;
        }
        case TC_STORE_F32: {
            float* o = reinterpret_cast<float*>(out_base) + (size_t)t0 * p.ld_out + col;
#pragma unroll
            for (int j = 0; j < 32; ++j)
                if (j < nt) o[(size_t)j * p.ld_out] = v[0][j];
            break;
        }
        case TC_RESID_BF16: {
            uint16_t* h = p.resid + (size_t)t0 * p.ld_out + col;
            uint16_t hv[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) hv[j] = j < nt ? h[(size_t)j * p.ld_out] : (uint16_t)0;
#pragma unroll
            for (int j = 0; j < 32; ++j)
                if (j < nt) h[(size_t)j * p.ld_out] = f2bf(bf2f(hv[j]) + v[0][j]);
            break;
        }
        case TC_SWIGLU: {
            uint16_t* o = reinterpret_cast<uint16_t*>(out_base) + (size_t)t0 * p.ld_out + col;
#pragma unroll
            for (int j = 0; j < 32; ++j) {
                const float g = v[0][j], up = v[1][j];
                const float sg = 1.0f / (1.0f + expf(-g));  // gate * sigmoid(gate) * up (:3522)
                if (j < nt) o[(size_t)j * p.ld_out] = f2bf((g * sg) * up);
            }
            break;
        }
        case TC_QKV_ROPE: {
            const int module = p.seg_module[seg];
            int pos[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) pos[j] = j < nt ? __ldg(p.ctx_lens + t0 + j) : 0;
            if (module != AOS_MOD_V) {
                // half-split RoPE (mlx_cpp_wrapper_real.cpp:3270-3280): pair (d, d+64)
                const int half = kTcBM / 2, i = row & (half - 1);
                const int partner = row ^ half;
                float2 cs[32];
#pragma unroll
                for (int j = 0; j < 32; ++j)
                    cs[j] = *reinterpret_cast<const float2*>(p.rope + ((size_t)pos[j] * half + i) * 2);
#pragma unroll
                for (int j = 0; j < 32; ++j) es.xbuf[row * 33 + j] = v[0][j];
                epi_bar();
#pragma unroll
                for (int j = 0; j < 32; ++j) {
                    const float x = v[0][j], y = es.xbuf[partner * 33 + j];
                    v[0][j] = row < half ? (x * cs[j].x - y * cs[j].y) : (y * cs[j].y + x * cs[j].x);
                }
                epi_bar();
            }
            if (module == AOS_MOD_Q) {
                uint16_t* o = reinterpret_cast<uint16_t*>(out_base) + (size_t)t0 * p.ld_out + col;
#pragma unroll
                for (int j = 0; j < 32; ++j)
                    if (j < nt) o[(size_t)j * p.ld_out] = f2bf(v[0][j]);
            } else {
                uint16_t* pool = module == AOS_MOD_K ? p.k_pool : p.v_pool;
                const int kvh = tile;  // one tile per kv head (head_dim == 128)
                int blk[32];
#pragma unroll
                for (int j = 0; j < 32; ++j)
                    blk[j] = j < nt ? __ldg(p.block_tables + (size_t)(t0 + j) * p.max_blocks + (pos[j] >> 4)) : 0;
#pragma unroll
                for (int j = 0; j < 32; ++j)
                    if (j < nt) {
                        const size_t idx =
                            ((((size_t)p.layer * p.num_blocks + blk[j]) * p.nkv + kvh) * 16 + (pos[j] & 15)) * 128 + row;
                        pool[idx] = f2bf(v[0][j]);
                    }
            }
            break;
        }
        case TC_SHRINK_HM: {
            const int slot = tile * kShrinkGroupsPerTile + row / kGroup;
            if (slot >= ng) break;
            const int c = __ldg(p.groups + slot) * kGroup + row % kGroup;
            const int owner = __ldg(p.col_owner + c);
            // per-token gate * alpha/rank of the column's adapter (0 when the
            // token did not select it); built by the routing prep each step
            const float* ct = p.coef + (size_t)t0 * p.max_adapters + (owner >= 0 ? owner : 0);
            float cf[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) cf[j] = (owner >= 0 && j < nt) ? __ldg(ct + (size_t)j * p.max_adapters) : 0.0f;
            uint16_t* o = reinterpret_cast<uint16_t*>(out_base) + (size_t)t0 * p.R + c;
#pragma unroll
            for (int j = 0; j < 32; ++j)
                if (j < nt) o[(size_t)j * p.R] = f2bf(v[0][j] * cf[j]);
            break;
        }
        default:
            break;
    }
}


// ---------------------------------------------------------------- schedule
// Stream-K over two pools.  Pool A holds the K steps of the shrink tiles
// (64-column blocks of the input against two touched lora_A groups); pool B
// holds the steps of the base tiles, each tile's K steps followed by its
// expand steps (one per touched rank group).  CTA c takes the contiguous slice
// [c*P/G, (c+1)*P/G) of pool A and then of pool B, so every SM streams the
// same amount, every SM finishes its shrink share first, and only the expand
// steps (which read the shrink output) wait for the shrink tiles.  A tile cut
// between CTAs is finished by the piece that arrives last: it waits until the
// other pieces have stored their fp32 partials and sums them with its own
// accumulator in piece order.
struct Sched {
    int ng;            // touched rank groups
    int kb;            // K steps per tile
    int lenB;          // steps per base tile (K steps + expand steps)
    int sh_per_seg;    // shrink tiles per shrink segment
    int n_sh, n_base;  // shrink tiles, base tiles
    long long PA, PB;  // pool lengths in steps
    int GA, GB;        // CTAs that take part in each pool (<= pool length)
};

struct Piece {
    int tile;          // global tile id: shrink tiles first, then base tiles
    int s0, s1;        // step range within the tile
    int idx, n;        // piece index within the tile, pieces of the tile in total
    bool shrink;
    int seg, t;        // segment, and tile index within the segment
};

__device__ __forceinline__ Sched make_sched(const TcParams& p) {
    Sched s;
    s.ng = (p.lora || p.sh_nseg) ? __ldg(p.n_groups) : 0;
    s.kb = p.kb;
    s.lenB = p.kb + (p.lora ? s.ng : 0);
    s.sh_per_seg = p.sh_nseg ? cdiv(s.ng, kShrinkGroupsPerTile) : 0;
    s.n_sh = p.sh_nseg * s.sh_per_seg;
    s.n_base = 0;
    for (int g = 0; g < p.n_seg; ++g) s.n_base += p.seg_tiles[g];
    s.PA = (long long)s.n_sh * s.kb;
    s.PB = (long long)s.n_base * s.lenB;
    // Every slice is at least len/kMaxPiecesPerPool steps long, so no tile is
    // cut into more than kMaxPiecesPerPool + 1 pieces.
    const long long la = max(1, cdiv(s.kb, kMaxPiecesPerPool));
    const long long lb = max(1, cdiv(s.lenB, kMaxPiecesPerPool));
    s.GA = s.PA > 0 ? (int)max(1ll, min((long long)gridDim.x, s.PA / la)) : 0;
    s.GB = (int)max(1ll, min((long long)gridDim.x, s.PB / lb));
    return s;
}
__device__ __forceinline__ long long pstart(int c, long long P, int G) { return (long long)c * P / G; }
// CTA whose slice of a pool (length P, G CTAs) contains step s.
__device__ __forceinline__ int cta_of(long long s, long long P, int G) { return (int)(((s + 1) * G - 1) / P); }

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

// Iterates this CTA's pieces in order (pool A, then pool B).  All three roles
// walk the same sequence.
struct PieceIter {
    int pool;
    long long s, e;  // current step, end of this CTA's slice
    __device__ __forceinline__ void init(const Sched& sc) {
        pool = 0;
        const int c = blockIdx.x;
        s = c < sc.GA ? pstart(c, sc.PA, sc.GA) : 0;
        e = c < sc.GA ? pstart(c + 1, sc.PA, sc.GA) : 0;
    }
    __device__ __forceinline__ bool next(const TcParams& p, const Sched& sc, Piece& pc) {
        while (s >= e) {
            if (pool == 1) return false;
            pool = 1;
            const int c = blockIdx.x;
            s = c < sc.GB ? pstart(c, sc.PB, sc.GB) : 0;
            e = c < sc.GB ? pstart(c + 1, sc.PB, sc.GB) : 0;
        }
        const long long P = pool == 0 ? sc.PA : sc.PB;
        const int G = pool == 0 ? sc.GA : sc.GB;
        const int len = pool == 0 ? sc.kb : sc.lenB;
        const int local_tile = (int)(s / len);
        const long long tstart = (long long)local_tile * len;
        const long long tend = min(tstart + len, e);
        tile_info(p, sc, pool == 0 ? local_tile : local_tile + sc.n_sh, pc);
        pc.s0 = (int)(s - tstart);
        pc.s1 = (int)(tend - tstart);
        const int c0 = cta_of(tstart, P, G);
        pc.n = cta_of(tstart + len - 1, P, G) - c0 + 1;
        pc.idx = (int)blockIdx.x - c0;
        s = tend;
        return true;
    }
};

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
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain_bar + 1);
    int* flag = reinterpret_cast<int*>(tmem_slot + 1);
    float* xbuf = reinterpret_cast<float*>(tail + 512);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const Sched sc = make_sched(p);
    const int cols_per_acc = p.n_sub * p.T_pad;
    const int acc_stages = (2 * cols_per_acc <= 512) ? 2 : 1;
    int tmem_cols = 32;
    while (tmem_cols < acc_stages * cols_per_acc) tmem_cols <<= 1;

    if (threadIdx.x == 0) {
        for (int s = 0; s < NS; ++s) {
            mbar_init(smem_u32(&full_bar[s]), 1);
            mbar_init(smem_u32(&empty_bar[s]), 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(smem_u32(&tfull_bar[a]), 1);
            mbar_init(smem_u32(&tempty_bar[a]), 4);
        }
        mbar_init(smem_u32(drain_bar), 1);
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
    const uint32_t idesc = idesc_bf16(p.T_pad);
    unsigned long long* tr = p.trace ? p.trace + (size_t)blockIdx.x * kTraceStride : nullptr;
    if (tr && threadIdx.x == 0) tr[192] = gtimer();

    if (warp == 0) {
        // ============================ TMA producer ============================
        // The weight-side boxes (W, lora_A, lora_B) of the first NS stages are
        // issued before pdl_wait(): weights are static and the group list was
        // written two or more launches earlier.  The activation-side boxes (X,
        // hm) follow once the previous launch has completed; hm boxes also wait
        // until every shrink tile of this launch is finished.
        if (lane == 0) {
            const uint64_t pol_w = policy_evict_first();
            const uint64_t pol_x = policy_evict_last();
            uint32_t last_phase[16];
            uint32_t used_mask = 0;
            int n_issued = 0;
            int stage = 0;
            uint32_t phase = 0;
            bool ok = true, waited = false, shrink_ready = (sc.n_sh == 0);
            int pre_tile[16], pre_step[16];
            int n_pre = 0;
            auto step_bytes = [&](const Piece& pc, int st) -> uint32_t {
                if (pc.shrink) {
                    const int nv = min(kShrinkGroupsPerTile, sc.ng - pc.t * kShrinkGroupsPerTile);
                    return (uint32_t)(nv * kGroup * 128 + p.T_pad * 128);
                }
                if (st >= sc.kb) return (uint32_t)(p.n_sub * (kTcBM * 128 + p.T_pad * 128));
                return (uint32_t)(p.n_sub * kTcBM * 128 + p.T_pad * 128);
            };
            auto issue_w = [&](const Piece& pc, int st, uint32_t sbase, uint32_t fb) {
                if (pc.shrink) {  // lora_A rows of the tile's (up to) two touched groups
                    const int first = pc.t * kShrinkGroupsPerTile;
                    const int nv = min(kShrinkGroupsPerTile, sc.ng - first);
                    for (int q = 0; q < nv; ++q)
                        tma_2d(&p.tm_a[pc.seg], sbase + q * (kGroup * 128), fb, st * kTcBK,
                               __ldg(p.groups + first + q) * kGroup, pol_w);
                } else if (st < sc.kb) {
                    for (int sub = 0; sub < p.n_sub; ++sub)
                        tma_2d(&p.tm_w[pc.seg * p.n_sub + sub], sbase + sub * (kTcBM * 128), fb, st * kTcBK,
                               p.seg_wrow0[pc.seg] + pc.t * kTcBM, pol_w);
                } else {  // LoRA expand: lora_B[tile rows, group cols]
                    const int gcol = __ldg(p.groups + (st - sc.kb)) * kGroup;
                    for (int sub = 0; sub < p.n_sub; ++sub)
                        tma_2d(&p.tm_lb[pc.seg * p.n_sub + sub], sbase + sub * (kTcBM * 128), fb, gcol, pc.t * kTcBM,
                               pol_w);
                }
            };
            auto issue_x = [&](const Piece& pc, int st, uint32_t sbase, uint32_t fb) -> bool {
                const uint32_t act = sbase + p.act_off;
                if (pc.shrink || st < sc.kb) {
                    tma_2d(&p.tm_x, act, fb, st * kTcBK, 0, pol_x);
                    return true;
                }
                if (!shrink_ready) {  // hm is written by this launch's shrink tiles
                    if (tr) tr[198] = gtimer();
                    if (!spin_ge(p.sync, sc.n_sh, p.err)) return false;
                    asm volatile("fence.proxy.async.global;" ::: "memory");
                    if (tr) tr[199] = gtimer();
                    shrink_ready = true;
                }
                const int gcol = __ldg(p.groups + (st - sc.kb)) * kGroup;
                for (int sub = 0; sub < p.n_sub; ++sub)
                    tma_2d(&p.tm_lh[pc.seg * p.n_sub + sub], act + sub * (p.T_pad * 128), fb, gcol, 0, pol_x);
                return true;
            };
            auto finish_wait = [&]() -> bool {
                pdl_wait();
                pdl_trigger();
                waited = true;
                for (int i = 0; i < n_pre; ++i) {
                    Piece pc;
                    tile_info(p, sc, pre_tile[i], pc);
                    if (!issue_x(pc, pre_step[i], smem_u32(stages + (size_t)i * p.stage_bytes), smem_u32(&full_bar[i])))
                        return false;
                }
                return true;
            };
            PieceIter itr;
            itr.init(sc);
            Piece pc;
            while (ok && itr.next(p, sc, pc)) {
                for (int st = pc.s0; st < pc.s1; ++st) {
                    if (!waited && n_pre == NS && !finish_wait()) { ok = false; break; }
                    if (!mbar_wait(smem_u32(&empty_bar[stage]), phase ^ 1u, p.err)) { ok = false; break; }
                    const uint32_t fb = smem_u32(&full_bar[stage]);
                    const uint32_t sbase = smem_u32(stages + (size_t)stage * p.stage_bytes);
                    mbar_expect_tx(fb, step_bytes(pc, st));
                    issue_w(pc, st, sbase, fb);
                    if (waited) {
                        if (!issue_x(pc, st, sbase, fb)) ok = false;
                    } else {  // first round of stages: stage index == n_pre
                        pre_tile[n_pre] = pc.tile;
                        pre_step[n_pre] = st;
                        ++n_pre;
                    }
                    last_phase[stage] = phase;
                    used_mask |= 1u << stage;
                    if (tr && n_issued < 64) tr[n_issued] = gtimer();
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
            int stage = 0;
            uint32_t phase = 0;
            int it = 0, n_waited = 0;
            bool ok = true, issued_any = false;
            PieceIter itr;
            itr.init(sc);
            Piece pc;
            while (ok && itr.next(p, sc, pc)) {
                const int acc = it % acc_stages;
                const uint32_t tphase = (uint32_t)((it / acc_stages) & 1);
                ++it;
                if (!mbar_wait(smem_u32(&tempty_bar[acc]), tphase ^ 1u, p.err)) { ok = false; break; }
                tc_fence_after();
                const uint32_t d0 = tmem_base + (uint32_t)(acc * cols_per_acc);
                const int nsub = pc.shrink ? 1 : p.n_sub;
                bool first = true;
                for (int st = pc.s0; st < pc.s1; ++st) {
                    if (!mbar_wait(smem_u32(&full_bar[stage]), phase, p.err)) { ok = false; break; }
                    tc_fence_after();
                    if (tr && n_waited < 64) tr[64 + n_waited] = gtimer();
                    ++n_waited;
                    const uint32_t sbase = smem_u32(stages + (size_t)stage * p.stage_bytes);
                    const uint32_t act = sbase + p.act_off;
                    const bool expand = !pc.shrink && st >= sc.kb;
                    for (int sub = 0; sub < nsub; ++sub) {
                        const uint32_t a0 = sbase + sub * (kTcBM * 128);
                        const uint32_t b0 = act + (expand ? sub * (p.T_pad * 128) : 0);
#pragma unroll
                        for (int kk = 0; kk < kTcBK / 16; ++kk)
                            umma_bf16(d0 + sub * p.T_pad, desc_sw128(a0 + kk * 32), desc_sw128(b0 + kk * 32), idesc,
                                      (first && kk == 0) ? 0u : 1u);
                    }
                    issued_any = true;
                    umma_commit(smem_u32(&empty_bar[stage]));  // frees the stage when these MMAs finish
                    first = false;
                    if (++stage == NS) { stage = 0; phase ^= 1u; }
                }
                if (!ok) break;
                umma_commit(smem_u32(&tfull_bar[acc]));
            }
            if (!ok && issued_any) {
                umma_commit(smem_u32(drain_bar));
                mbar_wait_drain(smem_u32(drain_bar), 0);
            }
        }
    } else {
        // ============================ epilogue ================================
        const int q = warp & 3;
        const int row = q * 32 + lane;
        const uint32_t lane_off = (uint32_t)(q * 32) << 16;
        EpiSmem es{xbuf};
        pdl_wait();  // the epilogue reads and writes activations of the previous launches
        const size_t slot_floats = (size_t)p.n_sub * p.T_pad * kTcBM;
        int it = 0, n_partial = 0;
        PieceIter itr;
        itr.init(sc);
        Piece pc;
        while (itr.next(p, sc, pc)) {
            const int acc = it % acc_stages;
            const uint32_t tphase = (uint32_t)((it / acc_stages) & 1);
            const bool ok = mbar_wait(smem_u32(&tfull_bar[acc]), tphase, p.err);
            if (epi_bar_any(!ok)) break;
            if (tr && threadIdx.x == 64 && it < 32) tr[128 + it] = gtimer();
            tc_fence_after();
            const uint32_t t_acc = tmem_base + lane_off + (uint32_t)(acc * cols_per_acc);
            const int mode = pc.shrink ? TC_SHRINK_HM : p.mode;
            void* out = pc.shrink ? p.sh_out[pc.seg] : p.out[pc.seg];
            const int nsub = pc.shrink ? 1 : p.n_sub;
            int* arrived = p.counters + 2 * pc.tile;  // [0] pieces arrived, [1] partials stored
            float v[2][32];
            bool finished = false;  // this piece produced the tile's final output
            bool last = pc.n == 1;
            if (!last) {
                if (threadIdx.x == 64) *flag = (atomicAdd(arrived, 1) == pc.n - 1);
                epi_bar();
                last = *flag != 0;
                epi_bar();  // everyone has read the flag before it can be rewritten
            }
            if (pc.n == 1) {
                for (int t0 = 0; t0 < p.T_pad; t0 += 32) {
                    tmem_ld32(t_acc + t0, v[0]);
                    if (nsub == 2) tmem_ld32(t_acc + p.T_pad + t0, v[1]);
                    epilogue_chunk(p, es, mode, pc.seg, pc.t, out, sc.ng, row, t0, v);
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(smem_u32(&tempty_bar[acc]));
                finished = true;
            } else if (!last) {
                // store the partial in this CTA's next workspace slot [sub][t][row]
                const bool room = n_partial < kMaxPartialsPerCta && pc.idx < kMaxPiecesPerTile;
                const int slot = (int)blockIdx.x * kMaxPartialsPerCta + n_partial;
                n_partial += room ? 1 : 0;
                float* wsu = p.ws + (size_t)slot * slot_floats;
                for (int t0 = 0; t0 < p.T_pad; t0 += 32)
#pragma unroll
                    for (int sub = 0; sub < 2; ++sub) {
                        if (sub >= nsub) break;
                        tmem_ld32(t_acc + sub * p.T_pad + t0, v[sub]);
                        if (room) {
#pragma unroll
                            for (int j = 0; j < 32; ++j)
                                __stcg(wsu + ((size_t)sub * p.T_pad + t0 + j) * kTcBM + row, v[sub][j]);
                        }
                    }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(smem_u32(&tempty_bar[acc]));
                if (room) {
                    if (threadIdx.x == 64) p.tile_slots[(size_t)pc.tile * kMaxPiecesPerTile + pc.idx] = slot;
                    __threadfence();
                    epi_bar();
                    if (threadIdx.x == 64) atomicAdd(arrived + 1, 1);  // publish (after the fence)
                } else if (threadIdx.x == 64) {
                    atomicCAS(p.err, 0, AOS_ERR_INVALID);  // schedule limits exceeded
                }
            } else {
                // last piece: wait for the other pieces' partials, then sum in
                // piece order with this piece's own accumulator (from TMEM)
                if (threadIdx.x == 64) *flag = spin_ge(arrived + 1, pc.n - 1, p.err) ? 1 : 0;
                epi_bar();
                const bool ready = *flag != 0;
                epi_bar();
                if (ready) {
                    __threadfence();
                    for (int t0 = 0; t0 < p.T_pad; t0 += 32) {
#pragma unroll
                        for (int sub = 0; sub < 2; ++sub) {
                            if (sub >= nsub) break;
                            float part[2][32];
                            int k = 0;
                            // pieces before this one, two at a time (independent loads in flight)
                            for (; k < pc.idx; k += 2) {
                                const bool two = k + 1 < pc.idx;
#pragma unroll
                                for (int u = 0; u < 2; ++u) {
                                    if (u == 1 && !two) break;
                                    const int sl = __ldcg(p.tile_slots + (size_t)pc.tile * kMaxPiecesPerTile + k + u);
                                    const float* src =
                                        p.ws + (size_t)sl * slot_floats + ((size_t)sub * p.T_pad + t0) * kTcBM + row;
#pragma unroll
                                    for (int j = 0; j < 32; ++j) part[u][j] = __ldcg(src + (size_t)j * kTcBM);
                                }
#pragma unroll
                                for (int j = 0; j < 32; ++j) {
                                    float a = k == 0 ? part[0][j] : v[sub][j] + part[0][j];
                                    if (two) a += part[1][j];
                                    v[sub][j] = a;
                                }
                            }
                            // this piece
                            tmem_ld32(t_acc + sub * p.T_pad + t0, part[0]);
#pragma unroll
                            for (int j = 0; j < 32; ++j) v[sub][j] = pc.idx == 0 ? part[0][j] : v[sub][j] + part[0][j];
                            // pieces after this one
                            for (k = pc.idx + 1; k < pc.n; k += 2) {
                                const bool two = k + 1 < pc.n;
#pragma unroll
                                for (int u = 0; u < 2; ++u) {
                                    if (u == 1 && !two) break;
                                    const int sl = __ldcg(p.tile_slots + (size_t)pc.tile * kMaxPiecesPerTile + k + u);
                                    const float* src =
                                        p.ws + (size_t)sl * slot_floats + ((size_t)sub * p.T_pad + t0) * kTcBM + row;
#pragma unroll
                                    for (int j = 0; j < 32; ++j) part[u][j] = __ldcg(src + (size_t)j * kTcBM);
                                }
#pragma unroll
                                for (int j = 0; j < 32; ++j) {
                                    float a = v[sub][j] + part[0][j];
                                    if (two) a += part[1][j];
                                    v[sub][j] = a;
                                }
                            }
                        }
                        epilogue_chunk(p, es, mode, pc.seg, pc.t, out, sc.ng, row, t0, v);
                    }
                    finished = true;
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(smem_u32(&tempty_bar[acc]));
                if (threadIdx.x == 64) {  // self-reset for the next launch
                    arrived[0] = 0;
                    arrived[1] = 0;
                }
            }
            if (finished && pc.shrink) {
                // this shrink tile's hm columns are written: publish them to the expand steps
                __threadfence();
                epi_bar();
                if (threadIdx.x == 64) atomicAdd(p.sync, 1);
            }
            if (tr && threadIdx.x == 64 && it < 32) tr[160 + it] = gtimer();
            ++it;
        }
    }

    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (threadIdx.x == 0) {
        if (tr) tr[193] = gtimer();
        // the last CTA to leave resets the launch's shrink counter
        __threadfence();
        const int old = atomicAdd(p.sync + 1, 1);
        if (old == (int)gridDim.x - 1) {
            p.sync[0] = 0;
            p.sync[1] = 0;
            __threadfence();
        }
    }
    if (warp == 1)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(tmem_cols));
}

// ---------------------------------------------------------------- host side
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

size_t tc_tail_bytes(const TcParams&) { return 512 + 128 * 33 * 4; }

size_t tc_smem_bytes(const TcParams& p) {
    return 1024 + (size_t)p.n_stages * p.stage_bytes + tc_tail_bytes(p);
}

int tc_prepare(TcParams& p, int smem_budget) {
    if (p.T <= 0 || p.T > 256 || p.n_sub < 1 || p.n_sub > 2 || p.n_seg < 1 || p.n_seg > kTcMaxSets ||
        p.n_seg * p.n_sub > kTcMaxSets || p.sh_nseg < 0 || p.sh_nseg > kTcMaxSets || p.kb < 1)
        return AOS_ERR_INVALID;
    p.T_pad = ((p.T + 15) / 16) * 16;
    if (p.T_pad < 32) p.T_pad = 32;  // epilogue works in 32-token chunks
    const uint32_t w_bytes = (uint32_t)p.n_sub * kTcBM * 128;
    const uint32_t act_base = (uint32_t)p.T_pad * 128;
    const uint32_t act_lora = (uint32_t)p.n_sub * p.T_pad * 128;
    const uint32_t act = std::max(act_base, p.lora ? act_lora : 0u);
    p.act_off = w_bytes;
    p.stage_bytes = (w_bytes + act + 1023) & ~1023u;
    const size_t fixed = 1024 + tc_tail_bytes(p);
    int ns = (int)((smem_budget - (int)fixed) / (int)p.stage_bytes);
    static const int max_stages = [] {
        const char* e = getenv("AOS_TC_MAX_STAGES");  // tuning knob, default 8
        const int v = e ? atoi(e) : 8;
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
cudaError_t tc_configure() {
    return cudaFuncSetAttribute(tc_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
}

size_t tc_ws_bytes(const TcParams& p, int grid) {
    return (size_t)grid * kMaxPartialsPerCta * p.n_sub * p.T_pad * kTcBM * sizeof(float);
}

cudaError_t tc_launch(const TcParams& p, int grid, cudaStream_t stream) {
    const size_t smem = tc_smem_bytes(p);
    if (smem > 227 * 1024) return cudaErrorInvalidValue;
    return launch_k(tc_gemm_kernel, dim3(grid), dim3(kTcThreads), smem, stream, p);
}

}  // namespace aos
