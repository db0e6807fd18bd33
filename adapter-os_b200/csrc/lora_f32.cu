// lora_f32.cu — fp32 base + K-sparse LoRA op (config 1).
//
// y[t] = W x[t] + sum_{ring slots, q15 > 0} (q15/32767 * (B_a (A_a x[t]))) * (alpha_a/rank)
// restating cpu_lora_forward (crates/adapteros-testing/src/kernel_testing.rs:220-257)
// and the liquid blend loop (crates/adapteros-lora-kernel-api/src/liquid.rs:222-250),
// with the gate dequantised as in mlx-ffi/src/backend.rs:405-418 (skip q15 <= 0).
//
// Three launches, all with fixed reduction orders (bit-identical run to run):
//   1. shrink: one warp per (token, slot, rank row): h = A_a[r] . x[t]
//   2. base: CTA tiles of 64 outputs x 64 tokens x one eighth of K (enough CTAs
//      to occupy the SMs at config 1's 64 tokens), register tiles of 4 x 8,
//      fp32 partials per eighth;
//   3. expand: the eighths summed in order, then the slots' expand terms in
//      ring order.
// fp32 in, fp32 FMA accumulation; W is read once per token tile.

#include "common.cuh"

namespace aos {
namespace {

constexpr int kMaxRank = 64;

__global__ void __launch_bounds__(256) lora_shrink_f32(const float* __restrict__ x, int T, int in_dim,
                                                       const float* __restrict__ A, int n_adapters,
                                                       int rank, const aos_router_ring* __restrict__ rings,
                                                       float* __restrict__ h /* [T][8][rank] */) {
    const int gw = (int)((blockIdx.x * blockDim.x + threadIdx.x) >> 5);
    const int lane = threadIdx.x & 31;
    const int per_tok = AOS_MAX_K * rank;
    if (gw >= T * per_tok) return;
    const int t = gw / per_tok, rem = gw % per_tok, s = rem / rank, r = rem % rank;
    const aos_router_ring& ring = rings[t];
    float acc = 0.0f;
    if (s < (int)ring.top_k && ring.gates_q15[s] > 0 && ring.indices[s] < n_adapters) {
        const float* a = A + ((size_t)ring.indices[s] * rank + r) * in_dim;
        const float* xt = x + (size_t)t * in_dim;
        for (int c = lane * 4; c < in_dim; c += 128) {
            const float4 av = *reinterpret_cast<const float4*>(a + c);
            const float4 xv = *reinterpret_cast<const float4*>(xt + c);
            acc = fmaf(av.x, xv.x, acc);
            acc = fmaf(av.y, xv.y, acc);
            acc = fmaf(av.z, xv.z, acc);
            acc = fmaf(av.w, xv.w, acc);
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
    }
    if (lane == 0) h[gw] = acc;
}

// Base GEMM: CTA tile of 64 outputs x 64 tokens over one eighth of K
// (blockIdx.z), 128 threads with a 4-output x 8-token register tile each; K
// is staged through shared memory 32 at a time, the next chunk's global loads
// in flight while the current one is multiplied.  The eight K eighths are
// written as fp32 partials and summed in order by the expand kernel.
constexpr int kBO = 64, kBT = 64, kBK = 32, kSplit = 8;

__global__ void __launch_bounds__(128) lora_base_f32(const float* __restrict__ x, int T, int in_dim, int out_dim,
                                                     const float* __restrict__ W, float* __restrict__ part) {
    __shared__ __align__(16) float ws[kBK][kBO + 4];
    __shared__ __align__(16) float xs[kBK][kBT + 4];
    const int o0 = blockIdx.x * kBO, t0 = blockIdx.y * kBT, ks = blockIdx.z;
    const int kq = (in_dim + kSplit - 1) / kSplit;
    const int k_lo = ks * kq, k_hi = min(in_dim, k_lo + kq);
    const int tid = threadIdx.x, tx = tid % 16, ty = tid / 16;  // outputs 4*tx.., tokens 8*ty..
    float acc[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;
    // loader: 64 rows x 32 k of W and of x per chunk; thread -> rows r0, r0+32 ... (4 floats each)
    auto load = [&](int k0, float (&wv)[4][4], float (&xv)[4][4]) {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const int idx = tid + 128 * q;  // 0..511 = 64 rows x 8 float4 columns
            const int r = idx / 8, c = (idx % 8) * 4, k = k0 + c;
            const int o = o0 + r, t = t0 + r;
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                wv[q][e] = (o < out_dim && k + e < k_hi) ? __ldg(W + (size_t)o * in_dim + k + e) : 0.f;
                xv[q][e] = (t < T && k + e < k_hi) ? __ldg(x + (size_t)t * in_dim + k + e) : 0.f;
            }
        }
    };
    auto store = [&](const float (&wv)[4][4], const float (&xv)[4][4]) {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const int idx = tid + 128 * q;
            const int r = idx / 8, c = (idx % 8) * 4;
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                ws[c + e][r] = wv[q][e];
                xs[c + e][r] = xv[q][e];
            }
        }
    };
    float wv[4][4], xv[4][4];
    load(k_lo, wv, xv);
    for (int k0 = k_lo; k0 < k_hi; k0 += kBK) {
        __syncthreads();  // the previous chunk has been consumed
        store(wv, xv);
        __syncthreads();
        if (k0 + kBK < k_hi) load(k0 + kBK, wv, xv);  // in flight during the FMAs below
#pragma unroll 8
        for (int kk = 0; kk < kBK; ++kk) {
            const float4 w4 = *reinterpret_cast<const float4*>(&ws[kk][4 * tx]);
            const float4 xa = *reinterpret_cast<const float4*>(&xs[kk][8 * ty]);
            const float4 xb = *reinterpret_cast<const float4*>(&xs[kk][8 * ty + 4]);
            const float wr[4] = {w4.x, w4.y, w4.z, w4.w};
            const float xr[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
#pragma unroll
            for (int i = 0; i < 8; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(wr[j], xr[i], acc[i][j]);
        }
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int t = t0 + 8 * ty + i;
        if (t >= T) continue;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int o = o0 + 4 * tx + j;
            if (o < out_dim) part[((size_t)ks * T + t) * out_dim + o] = acc[i][j];
        }
    }
}

// y[t][o] = sum of the K-eighth partials (in order) + the ring
// slots' expand terms in ring order: coeff * (B_a[o] . h[t][slot]) * scale.
__global__ void __launch_bounds__(256) lora_expand_f32(int T, int out_dim, const float* __restrict__ part,
                                                       const float* __restrict__ B, int n_adapters, int rank,
                                                       const float* __restrict__ alpha,
                                                       const aos_router_ring* __restrict__ rings,
                                                       const float* __restrict__ h, float* __restrict__ y) {
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (size_t)T * out_dim) return;
    const int t = (int)(i / out_dim), o = (int)(i % out_dim);
    float v = part[i];
#pragma unroll
    for (int ks = 1; ks < kSplit; ++ks) v = __fadd_rn(v, part[(size_t)ks * T * out_dim + i]);
    const aos_router_ring& ring = rings[t];
    for (int s = 0; s < (int)ring.top_k && s < AOS_MAX_K; ++s) {
        const int16_t q = ring.gates_q15[s];
        const int a = ring.indices[s];
        if (q <= 0 || a >= n_adapters) continue;
        const float coeff = __fdiv_rn((float)q, AOS_Q15_DENOM);
        const float scaling = __fdiv_rn(alpha ? alpha[a] : (float)rank, (float)rank);
        const float* b = B + ((size_t)a * out_dim + o) * rank;
        const float* hh = h + ((size_t)t * AOS_MAX_K + s) * rank;
        float d = 0.f;
        for (int r = 0; r < rank; ++r) d = fmaf(b[r], hh[r], d);
        v = __fadd_rn(v, __fmul_rn(__fmul_rn(coeff, d), scaling));
    }
    y[i] = v;
}

// Single-pass base + expand for callers with a small fixed scratch (only the
// shrink outputs): CTA tile of 32 outputs x 32 tokens over the whole K.
constexpr int TO = 32, TT = 32, TK = 32;  // tile outputs x tokens x k

__global__ void __launch_bounds__(256) lora_base_expand_f32(
    const float* __restrict__ x, int T, int in_dim, int out_dim, const float* __restrict__ W,
    const float* __restrict__ B, int n_adapters, int rank, const float* __restrict__ alpha,
    const aos_router_ring* __restrict__ rings, const float* __restrict__ h, float* __restrict__ y) {
    __shared__ float ws[TK][TO + 1];
    __shared__ float xs[TK][TT + 1];
    const int o0 = blockIdx.x * TO, t0 = blockIdx.y * TT;
    const int tid = threadIdx.x;
    const int to = tid % 16, tt = tid / 16;  // each thread: outputs {to, to+16}, tokens {tt, tt+16}
    float acc[2][2] = {{0.f, 0.f}, {0.f, 0.f}};
    for (int k0 = 0; k0 < in_dim; k0 += TK) {
        for (int i = tid; i < TO * TK; i += 256) {
            const int r = i / TK, c = i % TK;
            const int o = o0 + r, kk = k0 + c;
            ws[c][r] = (o < out_dim && kk < in_dim) ? W[(size_t)o * in_dim + kk] : 0.f;
            const int t = t0 + r;
            xs[c][r] = (t < T && kk < in_dim) ? x[(size_t)t * in_dim + kk] : 0.f;
        }
        __syncthreads();
#pragma unroll 8
        for (int c = 0; c < TK; ++c) {
            const float w0 = ws[c][to], w1 = ws[c][to + 16];
            const float x0 = xs[c][tt], x1 = xs[c][tt + 16];
            acc[0][0] = fmaf(w0, x0, acc[0][0]);
            acc[0][1] = fmaf(w0, x1, acc[0][1]);
            acc[1][0] = fmaf(w1, x0, acc[1][0]);
            acc[1][1] = fmaf(w1, x1, acc[1][1]);
        }
        __syncthreads();
    }
    for (int j = 0; j < 2; ++j) {
        const int t = t0 + tt + 16 * j;
        if (t >= T) continue;
        const aos_router_ring& ring = rings[t];
        for (int i = 0; i < 2; ++i) {
            const int o = o0 + to + 16 * i;
            if (o >= out_dim) continue;
            float v = acc[i][j];
            for (int s = 0; s < (int)ring.top_k && s < AOS_MAX_K; ++s) {
                const int16_t q = ring.gates_q15[s];
                const int a = ring.indices[s];
                if (q <= 0 || a >= n_adapters) continue;
                const float coeff = __fdiv_rn((float)q, AOS_Q15_DENOM);
                const float scaling = __fdiv_rn(alpha ? alpha[a] : (float)rank, (float)rank);
                const float* b = B + ((size_t)a * out_dim + o) * rank;
                const float* hh = h + ((size_t)t * AOS_MAX_K + s) * rank;
                float d = 0.f;
                for (int r = 0; r < rank; ++r) d = fmaf(b[r], hh[r], d);
                v = __fadd_rn(v, __fmul_rn(__fmul_rn(coeff, d), scaling));
            }
            y[(size_t)t * out_dim + o] = v;
        }
    }
}

}  // namespace

cudaError_t launch_lora_op_f32(const float* x, int T, int in_dim, int out_dim, const float* W,
                               const float* A, const float* B, int n_adapters, int rank,
                               const float* alpha, const aos_router_ring* rings, float* y,
                               float* h_scratch, cudaStream_t stream) {
    if (T <= 0) return cudaSuccess;
    const int warps = T * AOS_MAX_K * rank;
    lora_shrink_f32<<<(warps * 32 + 255) / 256, 256, 0, stream>>>(x, T, in_dim, A, n_adapters, rank,
                                                                   rings, h_scratch);
    // h_scratch holds [T][8][rank] shrink outputs, then [4][T][out] base partials
    float* part = h_scratch + (size_t)T * AOS_MAX_K * rank;
    dim3 grid((out_dim + kBO - 1) / kBO, (T + kBT - 1) / kBT, kSplit);
    lora_base_f32<<<grid, 128, 0, stream>>>(x, T, in_dim, out_dim, W, part);
    const size_t n = (size_t)T * out_dim;
    lora_expand_f32<<<(unsigned)((n + 255) / 256), 256, 0, stream>>>(T, out_dim, part, B, n_adapters, rank, alpha,
                                                                      rings, h_scratch, y);
    return cudaGetLastError();
}

// Same op with scratch for the shrink outputs only ([T][8][rank] floats):
// the single-pass base + expand kernel.
cudaError_t launch_lora_op_f32_small(const float* x, int T, int in_dim, int out_dim, const float* W,
                                     const float* A, const float* B, int n_adapters, int rank,
                                     const float* alpha, const aos_router_ring* rings, float* y,
                                     float* h_scratch, cudaStream_t stream) {
    if (T <= 0) return cudaSuccess;
    const int warps = T * AOS_MAX_K * rank;
    lora_shrink_f32<<<(warps * 32 + 255) / 256, 256, 0, stream>>>(x, T, in_dim, A, n_adapters, rank,
                                                                   rings, h_scratch);
    dim3 grid((out_dim + TO - 1) / TO, (T + TT - 1) / TT);
    lora_base_expand_f32<<<grid, 256, 0, stream>>>(x, T, in_dim, out_dim, W, B, n_adapters, rank,
                                                   alpha, rings, h_scratch, y);
    return cudaGetLastError();
}

// Scratch floats launch_lora_op_f32 needs: shrink outputs + K-eighth partials.
size_t lora_op_scratch_floats(int T, int out_dim, int rank) {
    return (size_t)T * AOS_MAX_K * rank + (size_t)kSplit * T * out_dim;
}

int lora_op_max_rank() { return kMaxRank; }

}  // namespace aos
