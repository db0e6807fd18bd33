// decode_kernels.cu — the small per-step kernels around the GEMMs:
// embedding gather, RMSNorm, the LoRA routing prep (touched rank groups), and
// synthetic KV fill.  All reductions use a fixed order.

#include <algorithm>

#include "common.cuh"
#include "loader.cuh"

namespace aos {
namespace {

// Embedding lookup (mlx_cpp_wrapper_real.cpp:3424-3430 mx::take); ids outside
// the vocabulary give a zero row (metal/src/kernels/adapteros_kernels.metal:195-234).
__global__ void embed_kernel(const uint16_t* __restrict__ table, const uint32_t* __restrict__ ids, int T, int H,
                             int V, uint16_t* __restrict__ out) {
    pdl_wait();
    pdl_trigger();
    const int t = blockIdx.x;
    if (t >= T) return;
    const uint32_t id = ids[t];
    const uint4* src = reinterpret_cast<const uint4*>(table + (size_t)id * H);
    uint4* dst = reinterpret_cast<uint4*>(out + (size_t)t * H);
    for (int i = threadIdx.x; i < H / 8; i += blockDim.x) dst[i] = id < (uint32_t)V ? src[i] : make_uint4(0, 0, 0, 0);
}

// RMSNorm (mlx_cpp_wrapper_real.cpp:3384-3390): y = x * (w / sqrt(mean(x^2) + eps)),
// computed as x * (w * r) with r = 1 / sqrt(mean(x^2) + eps) taken once per
// row (one fp32 rounding more than w / denom; the output is bf16).
// One CTA (256 threads) per token; thread i owns columns [8 (i + 256 c), +8)
// for chunks c and keeps the first kCached chunks in registers between the
// sum of squares and the scaling; fixed-order reduction; bf16 in/out.
template <int kCached>
__global__ void __launch_bounds__(256) rmsnorm_kernel(const uint16_t* __restrict__ x, const uint16_t* __restrict__ w,
                                                      int T, int H, float eps, uint16_t* __restrict__ y) {
    pdl_wait();
    pdl_trigger();
    const int t = blockIdx.x;
    if (t >= T) return;
    const uint16_t* xt = x + (size_t)t * H;
    uint4 xc[kCached];
    float ss = 0.0f;
    for (int c = 0, i = threadIdx.x * 8; i < H; ++c, i += 256 * 8) {
        uint4 v;
        if (c < kCached) {
#pragma unroll
            for (int k = 0; k < kCached; ++k)
                if (k == c) xc[k] = *reinterpret_cast<const uint4*>(xt + i);
#pragma unroll
            for (int k = 0; k < kCached; ++k)
                if (k == c) v = xc[k];
        } else {
            v = *reinterpret_cast<const uint4*>(xt + i);
        }
        const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float a = __uint_as_float(u[j] << 16), b = __uint_as_float(u[j] & 0xffff0000u);
            ss = fmaf(a, a, ss);
            ss = fmaf(b, b, ss);
        }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
    __shared__ float part[8];
    if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = ss;
    __syncthreads();
    float tot = 0.0f;
    for (int i = 0; i < 8; ++i) tot += part[i];
    const float r = 1.0f / sqrtf(tot / (float)H + eps);
    for (int c = 0, i = threadIdx.x * 8; i < H; ++c, i += 256 * 8) {
        uint4 v;
        if (c < kCached) {
#pragma unroll
            for (int k = 0; k < kCached; ++k)
                if (k == c) v = xc[k];
        } else {
            v = *reinterpret_cast<const uint4*>(xt + i);
        }
        const uint4 ww = __ldg(reinterpret_cast<const uint4*>(w + i));
        const uint32_t u[4] = {v.x, v.y, v.z, v.w};
        const uint32_t g[4] = {ww.x, ww.y, ww.z, ww.w};
        uint32_t o[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float a = __uint_as_float(u[j] << 16), b = __uint_as_float(u[j] & 0xffff0000u);
            const float wa = __uint_as_float(g[j] << 16), wb = __uint_as_float(g[j] & 0xffff0000u);
            o[j] = (uint32_t)f2bf(a * (wa * r)) | ((uint32_t)f2bf(b * (wb * r)) << 16);
        }
        *reinterpret_cast<uint4*>(y + (size_t)t * H + i) = make_uint4(o[0], o[1], o[2], o[3]);
    }
}

// First half of a folded RMSNorm (the decode GEMMs apply the second): per
// token, hw = bf16(x * w) and the sum of x^2 in fixed point (each thread's
// fp32 partial * 2^16 rounded, then an integer sum: order-independent, so
// the result is the same on every run).  One CTA of 256 threads per token.
__global__ void __launch_bounds__(256) norm_prep_kernel(const uint16_t* __restrict__ x, const uint16_t* __restrict__ w,
                                                        int T, int H, uint16_t* __restrict__ hw,
                                                        unsigned long long* __restrict__ ss) {
    pdl_wait();
    pdl_trigger();
    const int t = blockIdx.x;
    if (t >= T) return;
    const uint16_t* xt = x + (size_t)t * H;
    float sq = 0.0f;
    for (int i = threadIdx.x * 8; i < H; i += 256 * 8) {
        const uint4 v = *reinterpret_cast<const uint4*>(xt + i);
        const uint4 ww = *reinterpret_cast<const uint4*>(w + i);
        const uint32_t u[4] = {v.x, v.y, v.z, v.w};
        const uint32_t g[4] = {ww.x, ww.y, ww.z, ww.w};
        uint32_t o[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float a = __uint_as_float(u[j] << 16), b = __uint_as_float(u[j] & 0xffff0000u);
            const float wa = __uint_as_float(g[j] << 16), wb = __uint_as_float(g[j] & 0xffff0000u);
            sq = fmaf(a, a, sq);
            sq = fmaf(b, b, sq);
            o[j] = (uint32_t)f2bf(a * wa) | ((uint32_t)f2bf(b * wb) << 16);
        }
        *reinterpret_cast<uint4*>(hw + (size_t)t * H + i) = make_uint4(o[0], o[1], o[2], o[3]);
    }
    unsigned long long q = (unsigned long long)__float2ll_rn(sq * 65536.0f);  // the GEMMs' norm scale, 2^16
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) q += __shfl_xor_sync(0xffffffffu, q, off);
    __shared__ unsigned long long part[8];
    if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = q;
    __syncthreads();
    if (threadIdx.x == 0) {
        unsigned long long tot = 0;
        for (int i = 0; i < 8; ++i) tot += part[i];
        ss[t] = tot;
    }
}

// Routing prep for the LoRA GEMMs: mark every 64-column rank group of the
// arena that holds a column of an adapter selected (q15 > 0) by any token,
// then compact the marks in ascending group order.  One CTA of 1024 threads.
// (Names below say "slab" for a group of kPrepGroupCols arena columns.)
constexpr int kPrepGroupCols = 64;
__global__ void __launch_bounds__(1024) lora_prep_kernel(const aos_router_ring* __restrict__ rings, int T,
                                                         const int* __restrict__ col_off, const int* __restrict__ rank,
                                                         int max_adapters, int n_slab_total, int* __restrict__ slabs,
                                                         int* __restrict__ n_slabs) {
    extern __shared__ int marks[];  // [n_slab_total]
    __shared__ int warp_sums[32];
    pdl_wait();
    pdl_trigger();
    for (int i = threadIdx.x; i < n_slab_total; i += blockDim.x) marks[i] = 0;
    __syncthreads();
    for (int i = threadIdx.x; i < T * AOS_MAX_K; i += blockDim.x) {
        const aos_router_ring& r = rings[i / AOS_MAX_K];
        const int s = i % AOS_MAX_K;
        if (s >= (int)r.top_k || r.gates_q15[s] <= 0) continue;
        const int a = r.indices[s];
        if (a >= max_adapters) continue;
        const int c0 = col_off[a], rk = rank[a];
        if (c0 < 0 || rk <= 0) continue;
        for (int sl = c0 / kPrepGroupCols; sl <= (c0 + rk - 1) / kPrepGroupCols; ++sl)
            marks[sl] = 1;  // benign same-value race
    }
    __syncthreads();
    // ordered compaction: chunked exclusive scan over marks
    int running = 0;
    for (int base = 0; base < n_slab_total; base += blockDim.x) {
        const int i = base + threadIdx.x;
        const int m = i < n_slab_total ? marks[i] : 0;
        const unsigned bal = __ballot_sync(0xffffffffu, m);
        const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
        if (lane == 0) warp_sums[w] = __popc(bal);
        __syncthreads();
        int before = running;
        for (int j = 0; j < w; ++j) before += warp_sums[j];
        before += __popc(bal & ((1u << lane) - 1u));
        if (m) slabs[before] = i;
        int tot = 0;
        for (int j = 0; j < (int)(blockDim.x >> 5); ++j) tot += warp_sums[j];
        __syncthreads();
        running += tot;
    }
    if (threadIdx.x == 0) *n_slabs = running;
}

// Per-token LoRA coefficient table coef[t][a] = sum over the ring slots that
// name adapter a with q15 > 0 of (q15 / 32767) * (alpha_a / rank_a), i.e. the
// blend weight of mlx-ffi/src/backend.rs:405-418 times the module scale of
// mlx_cpp_wrapper_real.cpp:3410-3411 (0 for adapters the token did not select
// or that are not loaded).  One CTA per token.
__global__ void __launch_bounds__(256) lora_coef_kernel(const aos_router_ring* __restrict__ rings,
                                                        const int* __restrict__ rank, const float* __restrict__ scale,
                                                        int max_adapters, float* __restrict__ coef,
                                                        const int* __restrict__ groups, const int* __restrict__ n_groups,
                                                        const int* __restrict__ col_owner, int n_group_total,
                                                        float* __restrict__ ucoef) {
    pdl_wait();
    pdl_trigger();
    const int t = blockIdx.x;
    float* row = coef + (size_t)t * max_adapters;
    for (int a = threadIdx.x; a < max_adapters; a += blockDim.x) row[a] = 0.0f;
    __syncthreads();
    if (threadIdx.x == 0) {
        const aos_router_ring r = rings[t];
        const int k = min((int)r.top_k, AOS_MAX_K);
        for (int s = 0; s < k; ++s) {
            const int a = r.indices[s];
            if (r.gates_q15[s] <= 0 || a >= max_adapters || rank[a] <= 0) continue;
            row[a] += __fdiv_rn((float)r.gates_q15[s], AOS_Q15_DENOM) * scale[a];
        }
    }
    __syncthreads();
    // Per 8-column unit of every touched group (list order): the coefficient
    // of the unit's adapter for this token, so the GEMM gates a shrink tile
    // with one contiguous load per token.  Adapter columns come in units of 8.
    const int ng = *n_groups;
    float* urow = ucoef + (size_t)t * n_group_total * 8;
    for (int i = threadIdx.x; i < n_group_total * 8; i += blockDim.x) {
        float v = 0.0f;
        if (i / 8 < ng) {
            const int owner = col_owner[groups[i / 8] * 64 + (i % 8) * 8];
            if (owner >= 0 && owner < max_adapters) v = row[owner];
        }
        urow[i] = v;
    }
}

// SplitMix64-based synthetic bf16 fill ~N(0, std) (Box-Muller), seeded and
// position-independent so any page can be regenerated.
__device__ __forceinline__ uint64_t splitmix64(uint64_t x) {
    x += 0x9E3779B97F4A7C15ull;
    x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
    x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
    return x ^ (x >> 31);
}

__global__ void fill_normal_bf16(uint16_t* __restrict__ p, size_t n, uint64_t seed, float std) {
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < (n + 1) / 2; i += (size_t)gridDim.x * blockDim.x) {
        const uint64_t r = splitmix64(seed ^ (i * 0xD1B54A32D192ED03ull));
        const float u1 = ((float)(r >> 40) + 0.5f) * (1.0f / 16777216.0f);
        const float u2 = (float)((r >> 16) & 0xFFFFFF) * (1.0f / 16777216.0f);
        const float rad = sqrtf(-2.0f * logf(u1)) * std;
        float s, c;
        sincospif(2.0f * u2, &s, &c);
        p[2 * i] = f2bf(rad * c);
        if (2 * i + 1 < n) p[2 * i + 1] = f2bf(rad * s);
    }
}


// Packs rows x cols of a row-major bf16 matrix (src == nullptr: zeros) into
// the blocked layout the GEMM streams: the destination matrix (dst_cols
// columns) is cut into blocks of `br` rows x 64 columns, stored block after
// block in (row block, column block) order; inside a block row r's 16-byte
// chunk q sits at byte r*128 + (q ^ (r % 8)) * 16, which is the SWIZZLE_128B
// shared-memory image of that block.  One thread moves one 16-byte chunk.
__global__ void pack_blocks_kernel(const uint16_t* __restrict__ src, int rows, int cols, long long src_ld,
                                   uint16_t* __restrict__ dst, int row0, int col0, int dst_cols, int br) {
    const int c8n = cols / 8;
    const long long n = (long long)rows * c8n;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
        const int r = (int)(i / c8n), c8 = (int)(i % c8n);
        uint4 v = make_uint4(0u, 0u, 0u, 0u);
        if (src) v = *reinterpret_cast<const uint4*>(src + r * src_ld + c8 * 8);
        const int dr = row0 + r, dc = col0 + c8 * 8;
        const long long blk = (long long)(dr / br) * (dst_cols / 64) + dc / 64;
        const int rr = dr % br, q = (dc % 64) / 8;
        uint8_t* d = reinterpret_cast<uint8_t*>(dst) + blk * br * 128 + rr * 128 + ((q ^ (rr & 7)) * 16);
        *reinterpret_cast<uint4*>(d) = v;
    }
}

// Reads elements of the canonical (row-major, unpacked) view of packed
// matrices: element e of window w is starts[w] + k; the segment holding it is
// found by binary search over segs[].e0 (ascending), and its packed address
// is the one pack_blocks_kernel writes for (row0 + i, col0 + j).
__global__ void unpack_samples_kernel(const UnpackSeg* __restrict__ segs, int n_segs,
                                      const long long* __restrict__ starts, int n_per, uint16_t* __restrict__ out) {
    const int idx = blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= 3 * n_per) return;
    const long long e = starts[idx / n_per] + idx % n_per;
    int lo = 0, hi = n_segs - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) / 2;
        if (segs[mid].e0 <= e) lo = mid;
        else hi = mid - 1;
    }
    const UnpackSeg sg = segs[lo];
    const long long local = e - sg.e0;
    const int dr = sg.row0 + (int)(local / sg.cols), dc = sg.col0 + (int)(local % sg.cols);
    const long long blk = (long long)(dr / sg.br) * (sg.dst_cols / 64) + dc / 64;
    const int rr = dr % sg.br, q = (dc % 64) / 8;
    const uint8_t* p = reinterpret_cast<const uint8_t*>(sg.base) + blk * sg.br * 128 + rr * 128 +
                       ((q ^ (rr & 7)) * 16) + (dc % 8) * 2;
    out[idx] = *reinterpret_cast<const uint16_t*>(p);
}

// Zeroes the K and V pages of blocks[0..n) in every layer: CTA (i, layer)
// clears nkv pages of 16 x 128 bf16 in each pool (one contiguous run).
__global__ void zero_kv_blocks_kernel(uint16_t* __restrict__ k_pool, uint16_t* __restrict__ v_pool,
                                      const int* __restrict__ blocks, int num_blocks, int nkv) {
    const int b = blocks[blockIdx.x], layer = blockIdx.y;
    const size_t off = ((size_t)layer * num_blocks + b) * nkv * 16 * 128;
    const int n16 = nkv * 16 * 128 / 8;  // uint4 per pool run
    uint4* k = reinterpret_cast<uint4*>(k_pool + off);
    uint4* v = reinterpret_cast<uint4*>(v_pool + off);
    for (int i = threadIdx.x; i < n16; i += blockDim.x) {
        k[i] = make_uint4(0, 0, 0, 0);
        v[i] = make_uint4(0, 0, 0, 0);
    }
}

// Sliding-window rotate, the part inside pages: position i of the sequence
// takes the row of position i + r (0 < r < 16) for i < new_len, over the
// sequence's pages blocks[0..n) in order.  CTA (layer, kv head, pool) walks
// the pages in order, one thread per head dimension: it reads page b's rows
// r..15 and page b+1's rows 0..r-1 (rows needed only below new_len), waits
// for every thread, then writes page b.  Page b+1 is overwritten only in the
// next iteration, after its first rows were read, so the in-place shift
// never reads a row it has already moved.
__global__ void kv_shift_rows_kernel(uint16_t* __restrict__ k_pool, uint16_t* __restrict__ v_pool,
                                     const int* __restrict__ blocks, int n, int r, int new_len, int num_blocks, int nkv) {
    const int layer = blockIdx.x, h = blockIdx.y, d = threadIdx.x;
    uint16_t* pool = blockIdx.z ? v_pool : k_pool;
    auto row = [&](int blk, int j) -> uint16_t* {
        return pool + ((((size_t)layer * num_blocks + blk) * nkv + h) * 16 + j) * 128 + d;
    };
    const int n_dst = (new_len + 15) / 16;
    for (int b = 0; b < n_dst && b < n; ++b) {
        uint16_t val[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            const int src = j + r;  // row of page b (< 16) or of page b + 1
            val[j] = 0;
            if (b * 16 + j < new_len) val[j] = src < 16 ? *row(blocks[b], src) : *row(blocks[b + 1], src - 16);
        }
        __syncthreads();
#pragma unroll
        for (int j = 0; j < 16; ++j)
            if (b * 16 + j < new_len) *row(blocks[b], j) = val[j];
        __syncthreads();
    }
}

}  // namespace

cudaError_t launch_kv_shift_rows(uint16_t* k_pool, uint16_t* v_pool, const int* blocks, int n, int r, int new_len,
                                 int n_layers, int num_blocks, int nkv, cudaStream_t s) {
    if (n <= 0 || n_layers <= 0 || new_len <= 0 || r <= 0 || r >= 16) return cudaSuccess;
    kv_shift_rows_kernel<<<dim3(n_layers, nkv, 2), 128, 0, s>>>(k_pool, v_pool, blocks, n, r, new_len, num_blocks, nkv);
    return cudaGetLastError();
}

cudaError_t launch_zero_kv_blocks(uint16_t* k_pool, uint16_t* v_pool, const int* blocks, int n, int n_layers,
                                  int num_blocks, int nkv, cudaStream_t s) {
    if (n <= 0 || n_layers <= 0) return cudaSuccess;
    zero_kv_blocks_kernel<<<dim3(n, n_layers), 256, 0, s>>>(k_pool, v_pool, blocks, num_blocks, nkv);
    return cudaGetLastError();
}

cudaError_t launch_unpack_samples(const UnpackSeg* segs, int n_segs, const long long* starts, int n_per,
                                  uint16_t* out, cudaStream_t s) {
    const int n = 3 * n_per;
    if (n <= 0) return cudaSuccess;
    unpack_samples_kernel<<<(n + 255) / 256, 256, 0, s>>>(segs, n_segs, starts, n_per, out);
    return cudaGetLastError();
}

cudaError_t launch_embed(const uint16_t* table, const uint32_t* ids, int T, int H, int V, uint16_t* out,
                         cudaStream_t s) {
    if (T <= 0) return cudaSuccess;
    return launch_k(embed_kernel, dim3(T), dim3(128), 0, s, table, ids, T, H, V, out);
}

cudaError_t launch_rmsnorm(const uint16_t* x, const uint16_t* w, int T, int H, float eps, uint16_t* y,
                           cudaStream_t s) {
    if (T <= 0) return cudaSuccess;
    // rows of up to 2048 / 4096 / 8192 columns stay in registers; longer rows
    // re-read the columns past 8192
    if (H <= 2048) return launch_k(rmsnorm_kernel<1>, dim3(T), dim3(256), 0, s, x, w, T, H, eps, y);
    if (H <= 4096) return launch_k(rmsnorm_kernel<2>, dim3(T), dim3(256), 0, s, x, w, T, H, eps, y);
    return launch_k(rmsnorm_kernel<4>, dim3(T), dim3(256), 0, s, x, w, T, H, eps, y);
}

cudaError_t launch_norm_prep(const uint16_t* x, const uint16_t* w, int T, int H, uint16_t* hw,
                             unsigned long long* ss, cudaStream_t s) {
    if (T <= 0) return cudaSuccess;
    return launch_k(norm_prep_kernel, dim3(T), dim3(256), 0, s, x, w, T, H, hw, ss);
}

cudaError_t launch_lora_prep(const aos_router_ring* rings, int T, const int* col_off, const int* rank,
                             const float* scale, int max_adapters, int n_slab_total, int* slabs, int* n_slabs,
                             float* coef, const int* col_owner, float* ucoef, cudaStream_t s) {
    cudaError_t e = launch_k(lora_prep_kernel, dim3(1), dim3(1024), (size_t)n_slab_total * sizeof(int), s, rings, T,
                             col_off, rank, max_adapters, n_slab_total, slabs, n_slabs);
    if (e != cudaSuccess || T <= 0) return e;
    return launch_k(lora_coef_kernel, dim3(T), dim3(256), 0, s, rings, rank, scale, max_adapters, coef,
                    (const int*)slabs, (const int*)n_slabs, col_owner, n_slab_total, ucoef);
}

cudaError_t launch_pack_blocks(const uint16_t* src, int rows, int cols, long long src_ld, uint16_t* dst, int row0,
                               int col0, int dst_cols, int br, cudaStream_t s) {
    if (rows <= 0 || cols <= 0) return cudaSuccess;
    if (cols % 8 || col0 % 8 || dst_cols % 64 || (br != 64 && br != 128) || src_ld % 8 ||
        (reinterpret_cast<uintptr_t>(src) & 15))
        return cudaErrorInvalidValue;
    const long long n = (long long)rows * (cols / 8);
    const int blocks = (int)std::min<long long>((n + 255) / 256, 148 * 16);
    pack_blocks_kernel<<<blocks, 256, 0, s>>>(src, rows, cols, src_ld, dst, row0, col0, dst_cols, br);
    return cudaGetLastError();
}

// p[0, n) = 0 when the step touched no rank group (*n_groups == 0).
__global__ void zero_if_no_groups_kernel(const int* __restrict__ n_groups, uint16_t* __restrict__ p, size_t n) {
    pdl_wait();
    pdl_trigger();
    if (*n_groups != 0) return;
    uint4* q = reinterpret_cast<uint4*>(p);
    const size_t n16 = n / 8;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n16; i += (size_t)gridDim.x * blockDim.x)
        q[i] = make_uint4(0, 0, 0, 0);
    for (size_t i = n16 * 8 + (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        p[i] = 0;
}

cudaError_t launch_zero_if_no_groups(const int* n_groups, uint16_t* p, size_t n, cudaStream_t s) {
    if (!n) return cudaSuccess;
    if (reinterpret_cast<uintptr_t>(p) & 15) return cudaErrorInvalidValue;
    return launch_k(zero_if_no_groups_kernel, dim3(148 * 4), dim3(256), 0, s, n_groups, p, n);
}

cudaError_t launch_fill_normal(uint16_t* p, size_t n, uint64_t seed, float std, cudaStream_t s) {
    if (!n) return cudaSuccess;
    fill_normal_bf16<<<148 * 8, 256, 0, s>>>(p, n, seed, std);
    return cudaGetLastError();
}

}  // namespace aos
