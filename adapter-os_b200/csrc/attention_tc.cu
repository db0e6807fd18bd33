// attention_tc.cu — causal prefill attention over the paged KV cache on the
// fifth-generation tensor cores (tcgen05.mma with TMEM accumulators, TMA).
//
// Semantics as attn_prefill_kernel (attention.cu): query token t at position
// pos_t attends to positions 0..pos_t of its own sequence,
// softmax(q k^T / sqrt(128)) v, query head h reading KV head h / G
// (mlx_cpp_wrapper_real.cpp:3284-3324 with the causal mask;
// flash_attention.metal:23-97 for the tiled online softmax).
//
// A unit of work is (block of TB = 128 / G consecutive prompt tokens of one
// sequence, KV head); persistent CTAs walk the units, longest first.  The
// MMA's 128 rows are the group's G query heads times the block's tokens
// (row r = head r / TB, token r % TB), so each K/V tile is loaded once for the
// whole GQA group.
//   warp 0    : TMA producer -- the Q block once, then K and V tiles of 128
//               keys (8 pages of 16, each page two SWIZZLE_128B boxes of 64
//               dims)
//   warp 1    : TMEM allocation and the MMA-issuing thread
//   warps 2-5 : softmax, one query row (TMEM lane) per thread, then the output
// Key tile j:
//   S_j  = Q K_j^T         A = Q (smem, K-major), B = K_j (smem, K-major), D in TMEM
//   P_j  = 2^(S_j c - m)   softmax threads, written as bf16 pairs over S_j's first 64 columns
//   O   += P_j V_j         A = P_j (TMEM), B = V_j (smem, MN-major: keys are K, dims are N)
// A CTA takes 96 KB of shared memory and 256 TMEM columns, so two CTAs share
// an SM and one CTA's softmax runs while the other's MMAs and copies do.
//
// A row's running maximum m is raised only when a tile's maximum exceeds it by
// more than kLazyMax (log2 units); O and l are rescaled then.  Otherwise the
// tile's probabilities stay below 2^kLazyMax and O and l keep the same m, so
// O / l is the same softmax.  Sums run in a fixed order in each thread and the
// MMAs accumulate in a fixed order: results are bit-identical run to run.
//
// Every wait is bounded (kSpinLimitCycles): on a timeout the kernel records
// AOS_ERR_TIMEOUT in the error word, each role stops, the MMA thread waits for
// its issued MMAs and the producer for its copies, TMEM is freed and the
// kernel returns.

#include <cuda.h>

#include "common.cuh"

namespace aos {
namespace {

constexpr int kAtThreads = 192;
constexpr int kAtKeys = 128;                        // keys per tile
constexpr int kAtPages = kAtKeys / 16;              // pages per tile
constexpr uint32_t kAtTileBytes = kAtKeys * 256;    // K or V tile: 128 keys x 128 dims bf16
constexpr uint32_t kAtHalf = kAtKeys * 128;         // one 64-dim half of a tile (16 KB)
constexpr uint32_t kAtQBytes = 128 * 256;           // Q block: 128 rows x 128 dims
constexpr uint32_t kAtSmem = 1024 + kAtQBytes + 2 * kAtTileBytes + 256;  // Q, K, V, barriers: two CTAs per SM
constexpr uint32_t kAtCols = 256;  // TMEM columns per CTA (two CTAs per SM)
constexpr uint32_t kColS = 0;      // S (fp32), then P_j written over its first 64 columns (bf16 pairs)
constexpr uint32_t kColO = 128;    // O accumulator
constexpr float kLazyMax = 8.0f;

struct PfAttnTcParams {
    CUtensorMap tm_q;          // q [rows][nq*128] bf16, box 64 dims x TB tokens, SW128
    CUtensorMap tm_k, tm_v;    // pools [L*NB*nkv*16 rows][128], box 64 dims x 16 rows, SW128
    const int* block_tables;   // [T][max_blocks]: each token's sequence's pages
    const int* pos;            // [T] position of each token
    const int2* qblk;          // [n_qblk] (first token, tokens <= TB) of one sequence
    uint16_t* out;             // [T][nq*128]
    int n_qblk, nq, nkv, G, TB, layer, num_blocks, max_blocks;
    float scale_log2;          // log2(e) / sqrt(128)
    int* err;
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
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
// Bounded wait for the completion of the phase with this parity; false on
// timeout (recorded in err) or when another role already failed.
__device__ __noinline__ bool mbar_wait(uint32_t bar, uint32_t parity, int* err) {
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
// Time-bounded wait that ignores the error word (draining this CTA's own work).
__device__ __noinline__ void mbar_wait_drain(uint32_t bar, uint32_t parity) {
    const long long t0 = clock64();
    while (!mbar_try(bar, parity))
        if (clock64() - t0 > kSpinLimitCycles) return;
}
__device__ __forceinline__ void tma_2d(const CUtensorMap* m, uint32_t dst, uint32_t bar, int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
            dst),
        "l"(reinterpret_cast<uint64_t>(m)), "r"(bar), "r"(x), "r"(y)
        : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
// D (TMEM) (+)= A (smem descriptor) . B (smem descriptor)
__device__ __forceinline__ void umma_ss(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d),
        "l"(a), "l"(b), "r"(idesc), "r"(acc));
}
// D (TMEM) (+)= A (TMEM, lane = row, bf16 pairs per column) . B (smem descriptor)
__device__ __forceinline__ void umma_ts(uint32_t d, uint32_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}\n" ::"r"(d),
        "r"(a), "l"(b), "r"(idesc), "r"(acc));
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
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float (&v)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
        "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
        "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])), "r"(__float_as_uint(v[3])),
        "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])), "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])),
        "r"(__float_as_uint(v[8])), "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
        "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
        "r"(__float_as_uint(v[15])), "r"(__float_as_uint(v[16])), "r"(__float_as_uint(v[17])),
        "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])), "r"(__float_as_uint(v[20])),
        "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])), "r"(__float_as_uint(v[23])),
        "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])), "r"(__float_as_uint(v[26])),
        "r"(__float_as_uint(v[27])), "r"(__float_as_uint(v[28])), "r"(__float_as_uint(v[29])),
        "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
        : "memory");
}
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&u)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
            taddr),
        "r"(u[0]), "r"(u[1]), "r"(u[2]), "r"(u[3]), "r"(u[4]), "r"(u[5]), "r"(u[6]), "r"(u[7]), "r"(u[8]), "r"(u[9]),
        "r"(u[10]), "r"(u[11]), "r"(u[12]), "r"(u[13]), "r"(u[14]), "r"(u[15])
        : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
// 64 consecutive columns of this thread's lane, one TMEM round trip.
__device__ __forceinline__ void tmem_ld64(uint32_t taddr, float* v) {
    uint32_t r[64];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x64.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32,%33,%34,%35,%36,%37,%38,%39,"
        "%40,%41,%42,%43,%44,%45,%46,%47,%48,%49,%50,%51,%52,%53,%54,%55,%56,%57,%58,%59,%60,%61,%62,%63}, [%64];\n"
        "tcgen05.wait::ld.sync.aligned;"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31]),
          "=r"(r[32]), "=r"(r[33]), "=r"(r[34]), "=r"(r[35]), "=r"(r[36]), "=r"(r[37]), "=r"(r[38]), "=r"(r[39]),
          "=r"(r[40]), "=r"(r[41]), "=r"(r[42]), "=r"(r[43]), "=r"(r[44]), "=r"(r[45]), "=r"(r[46]), "=r"(r[47]),
          "=r"(r[48]), "=r"(r[49]), "=r"(r[50]), "=r"(r[51]), "=r"(r[52]), "=r"(r[53]), "=r"(r[54]), "=r"(r[55]),
          "=r"(r[56]), "=r"(r[57]), "=r"(r[58]), "=r"(r[59]), "=r"(r[60]), "=r"(r[61]), "=r"(r[62]), "=r"(r[63])
        : "r"(taddr)
        : "memory");
#pragma unroll
    for (int i = 0; i < 64; ++i) v[i] = __uint_as_float(r[i]);
}
// 2^x on the special-function unit (PTX ex2.approx.ftz.f32: 2^-inf = +0).
__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
__device__ __forceinline__ uint32_t bf16x2(float lo, float hi) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&h);
}

// Shared-memory matrix descriptors (tcgen05 "version 1"), SWIZZLE_128B.
// K-major: 8-row groups 1024 B apart (SBO); the K offset inside the 128-byte
// swizzle span goes into the start address.
__device__ __forceinline__ uint64_t desc_k(uint32_t addr) {
    return (uint64_t)((addr >> 4) & 0x3FFFu) | ((uint64_t)1u << 16) | ((uint64_t)(1024u >> 4) << 32) |
           ((uint64_t)1u << 46) | ((uint64_t)2u << 61);
}
// MN-major (V as the B operand: N = dims contiguous within 64-dim halves,
// K = keys): 64-dim halves kAtHalf bytes apart (LBO), 8-key groups 1024 B
// apart (SBO).
__device__ __forceinline__ uint64_t desc_mn(uint32_t addr) {
    return (uint64_t)((addr >> 4) & 0x3FFFu) | ((uint64_t)(kAtHalf >> 4) << 16) | ((uint64_t)(1024u >> 4) << 32) |
           ((uint64_t)1u << 46) | ((uint64_t)2u << 61);
}
// kind::f16 instruction descriptor: D f32, A/B bf16, M = 128, N = 128; B
// transposed (MN-major) when b_mn.
__device__ __forceinline__ uint32_t idesc_128(bool b_mn) {
    return (1u << 4) | (1u << 7) | (1u << 10) | (b_mn ? (1u << 16) : 0u) | ((uint32_t)(128 >> 3) << 17) |
           ((uint32_t)(128 >> 4) << 24);
}

// One attention unit: a query block of one sequence and a KV head.
struct AtUnit {
    int t0, nt, kvh, p_first, last_page, n_tiles;
    const int* bt;
};
__device__ __forceinline__ AtUnit at_unit(const PfAttnTcParams& p, int u) {
    AtUnit a;
    const int qb = p.n_qblk - 1 - u / p.nkv;  // longest blocks (latest in each prompt) first
    a.kvh = u % p.nkv;
    const int2 blk = __ldg(p.qblk + qb);
    a.t0 = blk.x;
    a.nt = blk.y;
    a.p_first = __ldg(p.pos + a.t0);
    const int p_last = a.p_first + a.nt - 1;
    a.last_page = p_last >> 4;
    a.n_tiles = p_last / kAtKeys + 1;
    a.bt = p.block_tables + (size_t)a.t0 * p.max_blocks;
    return a;
}

// Persistent: CTA c takes units c, c + grid, c + 2 grid, ... (longest first).
// Barriers complete once per key tile across all units (parity = the CTA's
// running tile count J), q_full and o_free once per unit (parity = the CTA's
// unit count U).  The producer loads a unit's Q as soon as the previous unit's
// last S has read its Q, so the next unit's first copies overlap the previous
// unit's last softmax, PV and output.
__global__ void __launch_bounds__(kAtThreads, 2) attn_prefill_tc_kernel(const __grid_constant__ PfAttnTcParams p) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const uint32_t q_s = smem_u32(smem);
    const uint32_t k_s = q_s + kAtQBytes;
    const uint32_t v_s = k_s + kAtTileBytes;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kAtQBytes + 2 * kAtTileBytes);
    uint64_t* q_full = bars;       // a unit's Q block landed
    uint64_t* k_full = bars + 1;   // K_J landed
    uint64_t* v_full = bars + 2;   // V_J landed
    uint64_t* k_empty = bars + 3;  // MMA: S_J done (K stage free; after a unit's last S, its Q too)
    uint64_t* s_full = bars + 4;   // MMA: S_J in TMEM
    uint64_t* p_full = bars + 5;   // softmax: P_J written over S_J, O rescaled (4 warps)
    uint64_t* pv_done = bars + 6;  // MMA: PV_J done (V stage, S/P columns and O free)
    uint64_t* o_free = bars + 7;   // softmax: a unit's O read out (4 warps)
    uint64_t* drain = bars + 8;    // MMA error path
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 9);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n_units = p.n_qblk * p.nkv;

    if (threadIdx.x == 0) {
        mbar_init(smem_u32(q_full), 1);
        mbar_init(smem_u32(k_full), 1);
        mbar_init(smem_u32(v_full), 1);
        mbar_init(smem_u32(k_empty), 1);
        mbar_init(smem_u32(s_full), 1);
        mbar_init(smem_u32(p_full), 4);
        mbar_init(smem_u32(pv_done), 1);
        mbar_init(smem_u32(o_free), 4);
        mbar_init(smem_u32(drain), 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(kAtCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        // ============================ TMA producer ============================
        if (lane == 0) {
            pdl_wait();  // q and the prompt's own K/V rows come from the previous launches
            pdl_trigger();
            int J = 0, q_issued = 0, k_issued = 0, v_issued = 0;
            bool ok = true;
            auto load = [&](const CUtensorMap* m, uint32_t base, uint64_t* full, const AtUnit& a, int j) {
                mbar_expect_tx(smem_u32(full), kAtTileBytes);
                for (int pg = 0; pg < kAtPages; ++pg) {
                    // pages past the block's last position repeat that page (masked; finite values)
                    const int page = min(j * kAtPages + pg, a.last_page);
                    const int row = ((p.layer * p.num_blocks + __ldg(a.bt + page)) * p.nkv + a.kvh) * 16;
                    for (int h = 0; h < 2; ++h) tma_2d(m, base + h * kAtHalf + pg * 2048, smem_u32(full), 64 * h, row);
                }
            };
            for (int u = blockIdx.x; ok && u < n_units; u += gridDim.x) {
                const AtUnit a = at_unit(p, u);
                for (int j = 0; j < a.n_tiles; ++j, ++J) {
                    const uint32_t prev = ((uint32_t)J & 1u) ^ 1u;  // completion J - 1 (a fresh barrier passes)
                    if (!mbar_wait(smem_u32(k_empty), prev, p.err)) { ok = false; break; }
                    if (j == 0) {  // the previous unit's last S has read its Q
                        ++q_issued;
                        mbar_expect_tx(smem_u32(q_full), (uint32_t)(p.G * p.TB) * 256u);
                        for (int g = 0; g < p.G; ++g)
                            for (int c = 0; c < 2; ++c)
                                tma_2d(&p.tm_q, q_s + c * kAtHalf + g * p.TB * 128, smem_u32(q_full),
                                       (a.kvh * p.G + g) * 128 + 64 * c, a.t0);
                    }
                    load(&p.tm_k, k_s, k_full, a, j);
                    ++k_issued;
                    if (!mbar_wait(smem_u32(pv_done), prev, p.err)) { ok = false; break; }
                    load(&p.tm_v, v_s, v_full, a, j);
                    ++v_issued;
                }
            }
            // every issued copy lands before the CTA may exit (the older ones
            // were consumed before their buffer was refilled)
            if (q_issued) mbar_wait_drain(smem_u32(q_full), (uint32_t)(q_issued - 1) & 1u);
            if (k_issued) mbar_wait_drain(smem_u32(k_full), (uint32_t)(k_issued - 1) & 1u);
            if (v_issued) mbar_wait_drain(smem_u32(v_full), (uint32_t)(v_issued - 1) & 1u);
        }
    } else if (warp == 1) {
        // ============================ MMA issuer ==============================
        if (lane == 0) {
            const uint32_t id_s = idesc_128(false), id_pv = idesc_128(true);
            bool ok = true, any = false;
            int J = 0, U = 0;
            for (int u = blockIdx.x; ok && u < n_units; u += gridDim.x, ++U) {
                const AtUnit a = at_unit(p, u);
                if (!mbar_wait(smem_u32(q_full), (uint32_t)U & 1u, p.err)) { ok = false; break; }
                for (int j = 0; j < a.n_tiles; ++j, ++J) {
                    const uint32_t par = (uint32_t)J & 1u;
                    // S_J overwrites the S/P columns that PV_{J-1} reads as its A
                    // operand; MMAs issued by one thread run in issue order, so
                    // S_J's accumulator writes come after PV_{J-1}'s operand reads
                    if (!mbar_wait(smem_u32(k_full), par, p.err)) { ok = false; break; }
                    tc_fence_after();
#pragma unroll
                    for (int kk = 0; kk < 8; ++kk) {
                        const uint32_t off = (uint32_t)(kk >> 2) * kAtHalf + (uint32_t)(kk & 3) * 32;
                        umma_ss(tmem + kColS, desc_k(q_s + off), desc_k(k_s + off), id_s, kk > 0 ? 1u : 0u);
                    }
                    any = true;
                    umma_commit(smem_u32(k_empty));
                    umma_commit(smem_u32(s_full));
                    if (!mbar_wait(smem_u32(p_full), par, p.err) || !mbar_wait(smem_u32(v_full), par, p.err) ||
                        (j == 0 && U > 0 && !mbar_wait(smem_u32(o_free), (uint32_t)(U - 1) & 1u, p.err))) {
                        ok = false;  // (a unit's first PV overwrites O: the previous unit's O is read out)
                        break;
                    }
                    tc_fence_after();
#pragma unroll
                    for (int kk = 0; kk < 8; ++kk)  // 16 keys per step: 8 TMEM columns of P, 2048 bytes of V
                        umma_ts(tmem + kColO, tmem + kColS + 8 * kk, desc_mn(v_s + kk * 2048), id_pv,
                                (j > 0 || kk > 0) ? 1u : 0u);
                    umma_commit(smem_u32(pv_done));
                }
            }
            if (!ok && any) {  // the MMAs already issued finish before TMEM is freed
                umma_commit(smem_u32(drain));
                mbar_wait_drain(smem_u32(drain), 0);
            }
        }
    } else {
        // ======================= softmax + output (warps 2-5) ==================
        const int q = warp & 3;  // TMEM lane quarter this warp may access
        const int r = q * 32 + lane;
        const uint32_t lane_off = (uint32_t)(q * 32) << 16;
        const uint32_t sb = tmem + lane_off + kColS, ob = tmem + lane_off + kColO;
        const int g = r / p.TB, i = r % p.TB;
        bool ok = true;
        int J = 0;
        for (int u = blockIdx.x; ok && u < n_units; u += gridDim.x) {
            const AtUnit a = at_unit(p, u);
            const bool valid = g < p.G && i < a.nt;
            const int qpos = valid ? a.p_first + i : -1;  // a row that is no query masks every key
            float m_used = -INFINITY, l = 0.f;
            for (int j = 0; j < a.n_tiles; ++j, ++J) {
                const uint32_t par = (uint32_t)J & 1u;
                const bool got = mbar_wait(smem_u32(s_full), par, p.err);
                if (!__all_sync(0xffffffffu, got)) { ok = false; break; }
                tc_fence_after();
                const int k0 = j * kAtKeys;
                // the row's 128 scores in registers (two TMEM round trips); a tile
                // whose keys all precede the block's first query needs no mask
                float v[kAtKeys];
                tmem_ld64(sb, v);
                tmem_ld64(sb + 64, v + 64);
                if (k0 + kAtKeys - 1 > a.p_first) {
#pragma unroll
                    for (int e = 0; e < kAtKeys; ++e)
                        if (k0 + e > qpos) v[e] = -INFINITY;
                }
                // tile maximum from eight partial maxima (the scale is positive, so
                // max(v) * scale = max(v * scale))
                float mx[8];
#pragma unroll
                for (int e = 0; e < 8; ++e) mx[e] = v[e];
#pragma unroll
                for (int e = 8; e < kAtKeys; ++e) mx[e & 7] = fmaxf(mx[e & 7], v[e]);
                const float tmax = fmaxf(fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])),
                                         fmaxf(fmaxf(mx[4], mx[5]), fmaxf(mx[6], mx[7]))) *
                                   p.scale_log2;
                const bool raise = tmax > -INFINITY && (m_used == -INFINITY || tmax > m_used + kLazyMax);
                const float m_new = raise ? tmax : m_used;
                const float m_sub = m_new > -INFINITY ? m_new : 0.f;  // a row with no key yet: every score is -inf
                // a raised maximum rescales O once PV_{J-1} is done, and l
                const float alpha = (raise && m_used > -INFINITY) ? ex2(m_used - m_new) : 1.f;
                if (__any_sync(0xffffffffu, alpha != 1.f)) {
                    const bool got_o = mbar_wait(smem_u32(pv_done), par ^ 1u, p.err);
                    if (!__all_sync(0xffffffffu, got_o)) { ok = false; break; }
                    tc_fence_after();
#pragma unroll
                    for (int c = 0; c < 4; ++c) {
                        float o[32];
                        tmem_ld32(ob + 32 * c, o);
#pragma unroll
                        for (int e = 0; e < 32; ++e) o[e] *= alpha;
                        tmem_st32(ob + 32 * c, o);
                    }
                }
                // probabilities as bf16 pairs over the S columns (every score of the
                // row is already in registers); their sum from eight partial sums
                // in a fixed order
                float sp[8];
#pragma unroll
                for (int e = 0; e < 8; ++e) sp[e] = 0.f;
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    uint32_t w[16];
#pragma unroll
                    for (int e = 0; e < 32; e += 2) {
                        const float p0 = ex2(fmaf(v[32 * c + e], p.scale_log2, -m_sub));
                        const float p1 = ex2(fmaf(v[32 * c + e + 1], p.scale_log2, -m_sub));
                        sp[(e >> 1) & 7] += p0 + p1;
                        w[e >> 1] = bf16x2(p0, p1);
                    }
                    tmem_st16(sb + 16 * c, w);
                }
                l = l * alpha + (((sp[0] + sp[1]) + (sp[2] + sp[3])) + ((sp[4] + sp[5]) + (sp[6] + sp[7])));
                m_used = m_new;
                tmem_wait_st();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(smem_u32(p_full));  // P_J written, O rescaled: PV_J may run
            }
            if (!ok) break;
            // O / l once the unit's last PV is done; then O is free for the next unit
            const bool got = mbar_wait(smem_u32(pv_done), (uint32_t)(J - 1) & 1u, p.err);
            if (!__all_sync(0xffffffffu, got)) { ok = false; break; }
            tc_fence_after();
            const float inv = l > 0.f ? 1.f / l : 0.f;
            uint16_t* dst = p.out + (size_t)(a.t0 + i) * p.nq * 128 + (size_t)(a.kvh * p.G + g) * 128;
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                float o[32];
                tmem_ld32(ob + 32 * c, o);
                if (!valid) continue;
#pragma unroll
                for (int e = 0; e < 32; e += 8) {
                    uint4 w;
                    w.x = bf16x2(o[e] * inv, o[e + 1] * inv);
                    w.y = bf16x2(o[e + 2] * inv, o[e + 3] * inv);
                    w.z = bf16x2(o[e + 4] * inv, o[e + 5] * inv);
                    w.w = bf16x2(o[e + 6] * inv, o[e + 7] * inv);
                    *reinterpret_cast<uint4*>(dst + 32 * c + e) = w;
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_u32(o_free));
        }
        tmem_wait_st();
    }

    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kAtCols));
}

}  // namespace

// The tensor-core kernel takes GQA groups whose size divides the 128 MMA rows.
bool attn_prefill_tc_supported(int nq, int nkv) {
    if (nkv <= 0 || nq % nkv) return false;
    const int G = nq / nkv;
    return G >= 1 && G <= 16 && (G & (G - 1)) == 0;
}
int attn_prefill_tc_block(int nq, int nkv) { return 128 / (nq / nkv); }
size_t attn_prefill_tc_smem_bytes() { return kAtSmem; }

cudaError_t attn_tc_configure() {
    return cudaFuncSetAttribute(attn_prefill_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kAtSmem);
}

cudaError_t launch_attention_prefill_tc(const CUtensorMap& tm_q, const CUtensorMap& tm_k, const CUtensorMap& tm_v,
                                        const int* block_tables, const int* pos, const int2* qblk, int n_qblk, int nq,
                                        int nkv, int layer, int num_blocks, int max_blocks, int* err, uint16_t* out,
                                        cudaStream_t s) {
    if (n_qblk <= 0) return cudaSuccess;
    if (!attn_prefill_tc_supported(nq, nkv)) return cudaErrorInvalidValue;
    PfAttnTcParams p;
    p.tm_q = tm_q;
    p.tm_k = tm_k;
    p.tm_v = tm_v;
    p.block_tables = block_tables;
    p.pos = pos;
    p.qblk = qblk;
    p.out = out;
    p.n_qblk = n_qblk;
    p.nq = nq;
    p.nkv = nkv;
    p.G = nq / nkv;
    p.TB = 128 / p.G;
    p.layer = layer;
    p.num_blocks = num_blocks;
    p.max_blocks = max_blocks;
    p.scale_log2 = 1.4426950408889634f / sqrtf(128.0f);
    p.err = err;
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int units = n_qblk * nkv, grid = units < 2 * sms ? units : 2 * sms;  // two CTAs per SM, persistent
    return launch_k(attn_prefill_tc_kernel, dim3(grid), dim3(kAtThreads), kAtSmem, s, p);
}

}  // namespace aos
