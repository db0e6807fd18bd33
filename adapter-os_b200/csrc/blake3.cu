// blake3.cu — BLAKE3 (hash mode, 32-byte digest) on the GPU, many messages
// per launch.
//
// The reference hashes adapter archive segments, per-tensor payloads and GPU
// buffer samples with BLAKE3 through B3Hash::hash / hash_multi
// (crates/adapteros-infra-common/src/hash.rs:22-36), which calls the
// `blake3` crate 1.8.3.  This file computes the same function from the
// published specification: the compression function (7 rounds of the G
// mixing function over a 4x4 word state, message words permuted between
// rounds), 1024-byte chunks of 64-byte blocks chained with CHUNK_START /
// CHUNK_END, and a left-balanced binary tree of PARENT nodes whose top
// compression carries ROOT.
//
// Work decomposition (the host builds it, blake3_plan below):
//   level 0  one CTA of 256 threads per 256 consecutive chunks of a message;
//            each thread compresses one chunk, reading it with 16-byte loads
//            (no shared-memory staging, so occupancy stays high for this
//            integer-ALU-bound work), and the 256 chaining values are reduced
//            pairwise to one subtree value in shared memory.
//   level k  one CTA per 256 consecutive nodes of the level below, reduced
//            the same way, until a message has one task left: that task's top
//            compression is the root.
// Pairing nodes (2i, 2i+1) and carrying an odd last node up unchanged at
// every level builds exactly the specification's left-balanced tree, and a
// 256-node group is an aligned subtree at every level, so CTAs never need to
// see each other's nodes.  Every message of a batch advances one level per
// launch; a batch of messages up to 256^L chunks long needs L + 1 launches.

#include <algorithm>
#include <cstring>
#include <vector>

#include "common.cuh"

namespace aos {

struct B3Task {
    uint64_t src;     // level 0: byte offset of the task's first chunk; level k: first input node
    uint64_t len;     // level 0: message bytes from src to the message's end; level k: input nodes (<= 64)
    uint64_t chunk0;  // level 0: chunk counter of the first chunk
    uint32_t out;     // output node slot (unused for a root task)
    uint32_t root;    // 0, or 1 + the message's digest slot when this task produces the root
};

namespace {

constexpr int kB3Group = 256;  // chunks / nodes per CTA (one thread each)
constexpr uint32_t kStart = 1, kEnd = 2, kParent = 4, kRoot = 8;

__device__ __forceinline__ uint32_t rotr(uint32_t x, int n) { return __funnelshift_r(x, x, n); }

#define B3_G(a, b, c, d, x, y)            \
    do {                                  \
        s[a] = s[a] + s[b] + (x);         \
        s[d] = rotr(s[d] ^ s[a], 16);     \
        s[c] = s[c] + s[d];               \
        s[b] = rotr(s[b] ^ s[c], 12);     \
        s[a] = s[a] + s[b] + (y);         \
        s[d] = rotr(s[d] ^ s[a], 8);      \
        s[c] = s[c] + s[d];               \
        s[b] = rotr(s[b] ^ s[c], 7);      \
    } while (0)

// h <- first 8 words of compress(h, m, counter, len, flags)
__device__ __forceinline__ void b3_compress(uint32_t h[8], uint32_t m[16], uint64_t counter, uint32_t len,
                                            uint32_t flags) {
    uint32_t s[16] = {h[0], h[1], h[2], h[3], h[4], h[5], h[6], h[7],
                      0x6A09E667u, 0xBB67AE85u, 0x3C6EF372u, 0xA54FF53Au,
                      (uint32_t)counter, (uint32_t)(counter >> 32), len, flags};
#pragma unroll
    for (int r = 0; r < 7; ++r) {
        B3_G(0, 4, 8, 12, m[0], m[1]);
        B3_G(1, 5, 9, 13, m[2], m[3]);
        B3_G(2, 6, 10, 14, m[4], m[5]);
        B3_G(3, 7, 11, 15, m[6], m[7]);
        B3_G(0, 5, 10, 15, m[8], m[9]);
        B3_G(1, 6, 11, 12, m[10], m[11]);
        B3_G(2, 7, 8, 13, m[12], m[13]);
        B3_G(3, 4, 9, 14, m[14], m[15]);
        if (r < 6) {  // message permutation (2, 6, 3, 10, 7, 0, 4, 13, 1, 11, 12, 5, 9, 14, 15, 8)
            const uint32_t t0 = m[2], t1 = m[6], t2 = m[3], t3 = m[10], t4 = m[7], t5 = m[0], t6 = m[4], t7 = m[13];
            const uint32_t t8 = m[1], t9 = m[11], t10 = m[12], t11 = m[5], t12 = m[9], t13 = m[14], t14 = m[15],
                           t15 = m[8];
            m[0] = t0; m[1] = t1; m[2] = t2; m[3] = t3; m[4] = t4; m[5] = t5; m[6] = t6; m[7] = t7;
            m[8] = t8; m[9] = t9; m[10] = t10; m[11] = t11; m[12] = t12; m[13] = t13; m[14] = t14; m[15] = t15;
        }
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) h[i] = s[i] ^ s[i + 8];
}

__device__ __forceinline__ void b3_iv(uint32_t h[8]) {
    h[0] = 0x6A09E667u; h[1] = 0xBB67AE85u; h[2] = 0x3C6EF372u; h[3] = 0xA54FF53Au;
    h[4] = 0x510E527Fu; h[5] = 0x9B05688Cu; h[6] = 0x1F83D9ABu; h[7] = 0x5BE0CD19u;
}

// Reduces cv[0..m) (shared memory) to cv[0]; the compression that leaves one
// node carries ROOT when `root`.  Every thread of the CTA calls it.
__device__ void b3_reduce(uint32_t (*cv)[8], int m, bool root) {
    const int t = threadIdx.x;
    while (m > 1) {
        const int half = m >> 1;
        uint32_t h[8];
        if (t < half) {
            uint32_t w[16];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                w[i] = cv[2 * t][i];
                w[8 + i] = cv[2 * t + 1][i];
            }
            b3_iv(h);
            b3_compress(h, w, 0, 64, kParent | (root && m == 2 ? kRoot : 0));
        }
        __syncthreads();
        if (t < half)
#pragma unroll
            for (int i = 0; i < 8; ++i) cv[t][i] = h[i];
        if ((m & 1) && t == 0)
#pragma unroll
            for (int i = 0; i < 8; ++i) cv[half][i] = cv[m - 1][i];
        __syncthreads();
        m = half + (m & 1);
    }
}

__device__ __forceinline__ void b3_emit(const uint32_t* h, const B3Task& tk, uint32_t* nodes, uint32_t* digests) {
    uint32_t* dst = tk.root ? digests + 8 * (size_t)(tk.root - 1) : nodes + 8 * (size_t)tk.out;
#pragma unroll
    for (int i = 0; i < 8; ++i) dst[i] = h[i];
}

__global__ void __launch_bounds__(kB3Group) b3_chunks_kernel(const uint8_t* __restrict__ base,
                                                              const B3Task* __restrict__ tasks,
                                                              uint32_t* __restrict__ nodes,
                                                              uint32_t* __restrict__ digests) {
    __shared__ uint32_t cv[kB3Group][8];
    const B3Task tk = tasks[blockIdx.x];
    const int t = threadIdx.x;
    const uint64_t cap = (uint64_t)kB3Group * 1024;
    const uint64_t bytes = tk.len < cap ? tk.len : cap;
    const int nc = tk.len == 0 ? 1 : (int)((bytes + 1023) / 1024);
    const uint8_t* src = base + tk.src;
    const bool single = tk.root && nc == 1;  // a one-chunk message: the chunk is the root
    if (t < nc) {
        // each thread reads its own chunk straight from memory: 16-byte loads
        // (the chunk's 64-byte blocks are consecutive, so the L1 line a load
        // brings in serves the thread's next loads), bytes when unaligned
        const uint64_t left = bytes - (uint64_t)t * 1024;
        const uint32_t clen = left < 1024 ? (uint32_t)left : 1024u;
        const int nb = clen == 0 ? 1 : (int)((clen + 63) / 64);
        const uint8_t* cp = src + (size_t)t * 1024;
        const bool vec = (reinterpret_cast<uintptr_t>(cp) & 15) == 0;
        uint32_t h[8];
        b3_iv(h);
        for (int b = 0; b < nb; ++b) {
            const uint32_t blen = min(64u, clen - 64u * b);
            uint32_t m[16];
            if (vec && blen == 64) {
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const uint4 x = __ldg(reinterpret_cast<const uint4*>(cp + 64 * b) + i);
                    m[4 * i] = x.x;
                    m[4 * i + 1] = x.y;
                    m[4 * i + 2] = x.z;
                    m[4 * i + 3] = x.w;
                }
            } else {  // the message's last, partial block (zero padded), or an unaligned start
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    uint32_t w = 0;
                    for (int k = 0; k < 4; ++k)
                        if (4 * i + k < (int)blen) w |= (uint32_t)__ldg(cp + 64 * b + 4 * i + k) << (8 * k);
                    m[i] = w;
                }
            }
            uint32_t f = (b == 0 ? kStart : 0u) | (b + 1 == nb ? kEnd : 0u);
            if (single && b + 1 == nb) f |= kRoot;
            b3_compress(h, m, tk.chunk0 + t, blen, f);
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) cv[t][i] = h[i];
    }
    __syncthreads();
    b3_reduce(cv, nc, tk.root != 0);
    if (t == 0) b3_emit(cv[0], tk, nodes, digests);
}

__global__ void __launch_bounds__(kB3Group) b3_level_kernel(const uint32_t* __restrict__ in,
                                                             const B3Task* __restrict__ tasks,
                                                             uint32_t* __restrict__ out,
                                                             uint32_t* __restrict__ digests) {
    __shared__ uint32_t cv[kB3Group][8];
    const B3Task tk = tasks[blockIdx.x];
    const int t = threadIdx.x, n = (int)tk.len;
    if (t < n)
#pragma unroll
        for (int i = 0; i < 8; ++i) cv[t][i] = in[8 * (tk.src + t) + i];
    __syncthreads();
    b3_reduce(cv, n, tk.root != 0);
    if (t == 0) b3_emit(cv[0], tk, out, digests);
}

}  // namespace

// Host plan: per level, the task list and the node count it writes.
struct B3Plan {
    std::vector<std::vector<B3Task>> levels;
    std::vector<uint32_t> nodes_out;  // nodes written by each level
};

static void blake3_plan(const uint64_t* offsets, const uint64_t* lens, int n_msg, B3Plan& plan) {
    // level 0
    std::vector<B3Task> l0;
    std::vector<uint64_t> cur_nodes(n_msg), cur_first(n_msg);  // per message: nodes after this level, first slot
    uint32_t slot = 0;
    for (int i = 0; i < n_msg; ++i) {
        const uint64_t nch = lens[i] == 0 ? 1 : (lens[i] + 1023) / 1024;
        const uint64_t ntask = (nch + kB3Group - 1) / kB3Group;
        cur_first[i] = slot;
        for (uint64_t k = 0; k < ntask; ++k) {
            B3Task tk;
            tk.src = offsets[i] + k * kB3Group * 1024ull;
            tk.len = lens[i] - k * kB3Group * 1024ull;
            tk.chunk0 = k * kB3Group;
            tk.out = ntask == 1 ? 0u : slot++;
            tk.root = ntask == 1 ? (uint32_t)i + 1 : 0u;
            l0.push_back(tk);
        }
        cur_nodes[i] = ntask == 1 ? 0 : ntask;
    }
    plan.levels.push_back(std::move(l0));
    plan.nodes_out.push_back(slot);
    while (true) {
        std::vector<B3Task> lv;
        uint32_t oslot = 0;
        std::vector<uint64_t> next_nodes(n_msg, 0), next_first(n_msg, 0);
        for (int i = 0; i < n_msg; ++i) {
            const uint64_t m = cur_nodes[i];
            if (m == 0) continue;
            const uint64_t ntask = (m + kB3Group - 1) / kB3Group;
            next_first[i] = oslot;
            for (uint64_t k = 0; k < ntask; ++k) {
                B3Task tk;
                tk.src = cur_first[i] + k * kB3Group;
                tk.len = std::min<uint64_t>(kB3Group, m - k * kB3Group);
                tk.chunk0 = 0;
                tk.out = ntask == 1 ? 0u : oslot++;
                tk.root = ntask == 1 ? (uint32_t)i + 1 : 0u;
                lv.push_back(tk);
            }
            next_nodes[i] = ntask == 1 ? 0 : ntask;
        }
        if (lv.empty()) break;
        plan.levels.push_back(std::move(lv));
        plan.nodes_out.push_back(oslot);
        cur_nodes.swap(next_nodes);
        cur_first.swap(next_first);
    }
}


// Digests of messages [base + offsets[i], + lens[i]) of device memory, into
// host digests[i][32].  Synchronizes `s`.
int blake3_many(const uint8_t* d_base, const uint64_t* offsets, const uint64_t* lens, int n_msg, uint8_t* digests,
                cudaStream_t s, std::string& err) {
    if (n_msg <= 0) return AOS_OK;
    B3Plan plan;
    blake3_plan(offsets, lens, n_msg, plan);
    size_t n_tasks = 0, n_nodes = 0;
    for (size_t l = 0; l < plan.levels.size(); ++l) {
        n_tasks += plan.levels[l].size();
        n_nodes = std::max<size_t>(n_nodes, plan.nodes_out[l]);
    }
    std::vector<B3Task> all;
    all.reserve(n_tasks);
    for (const auto& lv : plan.levels) all.insert(all.end(), lv.begin(), lv.end());
    B3Task* d_tasks = nullptr;
    uint32_t *d_nodes = nullptr, *d_dig = nullptr;
    const size_t node_words = 8 * std::max<size_t>(1, n_nodes);
    cudaError_t e = cudaMallocAsync((void**)&d_tasks, sizeof(B3Task) * n_tasks, s);
    if (e == cudaSuccess) e = cudaMallocAsync((void**)&d_nodes, 2 * node_words * 4, s);
    if (e == cudaSuccess) e = cudaMallocAsync((void**)&d_dig, (size_t)n_msg * 32, s);
    if (e == cudaSuccess) e = cudaMemcpyAsync(d_tasks, all.data(), sizeof(B3Task) * n_tasks, cudaMemcpyHostToDevice, s);
    size_t t0 = 0;
    for (size_t l = 0; l < plan.levels.size() && e == cudaSuccess; ++l) {
        const unsigned grid = (unsigned)plan.levels[l].size();
        uint32_t* out = d_nodes + (l & 1) * node_words;
        if (l == 0) {
            b3_chunks_kernel<<<grid, kB3Group, 0, s>>>(d_base, d_tasks, out, d_dig);
        } else {
            const uint32_t* in = d_nodes + ((l - 1) & 1) * node_words;
            b3_level_kernel<<<grid, kB3Group, 0, s>>>(in, d_tasks + t0, out, d_dig);
        }
        t0 += grid;
        e = cudaGetLastError();
    }
    if (e == cudaSuccess) e = cudaMemcpyAsync(digests, d_dig, (size_t)n_msg * 32, cudaMemcpyDeviceToHost, s);
    if (d_tasks) cudaFreeAsync(d_tasks, s);
    if (d_nodes) cudaFreeAsync(d_nodes, s);
    if (d_dig) cudaFreeAsync(d_dig, s);
    const cudaError_t e2 = cudaStreamSynchronize(s);
    if (e == cudaSuccess) e = e2;
    if (e != cudaSuccess) {
        err = std::string("BLAKE3 on the device: ") + cudaGetErrorString(e);
        return AOS_ERR_CUDA;
    }
    return AOS_OK;
}

}  // namespace aos
