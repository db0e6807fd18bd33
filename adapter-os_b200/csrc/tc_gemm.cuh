// tc_gemm.cuh — parameters of the tcgen05 weight-streaming GEMM (tc_gemm.cu).
//
// D[rows, tokens] = W[rows, K] . X[tokens, K]^T  (+ sum over touched LoRA rank
// groups of  B_cat[rows, 64 group cols] . Hm[tokens, 64 group cols]^T), i.e. the
// base projection y = x W^T of mlx_cpp_wrapper_real.cpp:3372-3381 fused with
// the LoRA shrink and expand of :3394-3419, computed "swap-AB": weight rows are
// the MMA's M (128 per tile) and the decode tokens are its N (<= 256).  Every
// pipeline step is one 128-row x 128-byte box of weights plus one T x 128-byte
// box of activations (SWIZZLE_128B) and four K=16 MMAs.
#pragma once

#include <cuda.h>

#include "common.cuh"

namespace aos {

enum TcMode : int {
    TC_STORE_BF16 = 0,  // out[t][col] = bf16(acc)
    TC_RESID_BF16 = 1,  // resid[t][col] = bf16(resid + acc)          (o / down + residual)
    TC_STORE_F32 = 2,   // out[t][col] = acc                           (lm_head logits)
    TC_QKV_ROPE = 3,    // q -> out (RoPE), k -> paged K (RoPE), v -> paged V
    TC_SWIGLU = 4,      // out[t][col] = bf16(silu(acc0) * acc1)        (n_sub = 2)
    TC_SHRINK_HM = 5    // hm[t][group col] = bf16(acc * gate(t, owner(col)))
};

constexpr int kTcMaxSets = 3;    // operand sets = segments x sub-tiles
constexpr int kTcThreads = 192;  // warp 0 TMA, warp 1 MMA, warps 2-5 epilogue
constexpr int kTcBM = 128;       // weight rows per tile
constexpr int kTcBK = 64;        // K elements per step (128 B, one SW128 row)
constexpr int kGroup = 64;       // LoRA rank columns per group (= one K step)
constexpr int kShrinkGroupsPerTile = kTcBM / kGroup;  // 2

struct TcParams {
    CUtensorMap tm_w[kTcMaxSets];   // base weights [rows, K], SW128, per segment x sub-tile
    CUtensorMap tm_x;               // activations [T, K], SW128
    CUtensorMap tm_lb[kTcMaxSets];  // lora_B [rows, R], SW128
    CUtensorMap tm_lh[kTcMaxSets];  // gated shrink output hm [T, R], SW128
    CUtensorMap tm_a[kTcMaxSets];   // lora_A [R, K] per shrink segment, box 64 x 64, SW128
    int mode, n_sub, n_seg, T, T_pad, kb, n_stages, lora;
    int sh_nseg;                    // shrink segments (LoRA modules that read X), 0 = none
    int seg_tiles[kTcMaxSets];      // base tiles per segment
    int seg_wrow0[kTcMaxSets];      // first W row of the segment
    int seg_out0[kTcMaxSets];       // first output feature of the segment
    int seg_rows[kTcMaxSets];       // valid output rows of the segment
    int seg_module[kTcMaxSets];
    uint32_t stage_bytes, act_off;  // bytes per pipeline stage; offset of the activation region
    const int* groups;              // touched rank-group list (ascending)
    const int* n_groups;            // its length
    // epilogue
    void* out[kTcMaxSets];
    void* sh_out[kTcMaxSets];       // hm buffer written by each shrink segment
    int ld_out;
    uint16_t* resid;
    const float* rope;  // [max_pos][hd/2][2] cos/sin
    uint16_t* k_pool;
    uint16_t* v_pool;
    const int* block_tables;
    const int* ctx_lens;
    int max_blocks, num_blocks, nkv, layer;
    int R;                          // arena rank capacity (columns of hm)
    const int* col_owner;           // [R] adapter id owning the column, -1 if free
    const float* coef;              // [T][max_adapters] gate * alpha/rank (0 = not selected)
    int max_adapters;
    float* ws;                      // fp32 partials: [grid][kMaxPartialsPerCta][n_sub][T_pad][128]
    int* counters;                  // [tile][2]: pieces arrived, partials stored; self-resetting
    int* tile_slots;                // [tile][kMaxPiecesPerTile] partial slot of each piece
    int* sync;                      // [0] finished shrink tiles, [1] exited CTAs; self-resetting
    int* err;                       // device error word (0 = ok)
    unsigned long long* trace;      // optional per-CTA %globaltimer trace (null = off)
};

constexpr int kMaxPiecesPerPool = 30;                  // a slice is at least 1/30 of a tile
constexpr int kMaxPiecesPerTile = kMaxPiecesPerPool + 2;  // tile_slots row length (>= 31 pieces)
// A CTA's slice of a pool cuts at most its first and its last tile, so it
// stores at most two partial tiles per pool.
constexpr int kMaxPartialsPerCta = 4;

// Trace layout per CTA (kTraceStride slots): [0,64) producer step issues,
// [64,128) MMA full-barrier waits done, [128,160) epilogue unit starts,
// [160,192) epilogue unit ends, 192 kernel start, 193 kernel end, 198/199
// producer wait for the shrink tiles begins/ends.
constexpr int kTraceStride = 256;

// Host helpers (tc_gemm.cu).
int tc_encode_2d(CUtensorMap* m, const void* base, uint64_t inner, uint64_t outer, uint64_t row_bytes,
                 uint32_t box_inner, uint32_t box_outer, int swizzle_bytes);
int tc_encode_3d(CUtensorMap* m, const void* base, uint64_t d0, uint64_t d1, uint64_t d2,
                 uint64_t stride1_bytes, uint64_t stride2_bytes, uint32_t b0, uint32_t b1, uint32_t b2,
                 int swizzle_bytes);
// Fills stage sizes; returns 0 or an aos_status.
int tc_prepare(TcParams& p, int smem_budget);
// Launch on `grid` CTAs; every CTA must be resident at once (grid <= SM count),
// because expand steps wait for shrink tiles computed by other CTAs.
cudaError_t tc_launch(const TcParams& p, int grid, cudaStream_t stream);
// Bytes of p.ws a launch on `grid` CTAs needs.
size_t tc_ws_bytes(const TcParams& p, int grid);
cudaError_t tc_configure();
size_t tc_smem_bytes(const TcParams& p);
int tc_num_sms();

}  // namespace aos
