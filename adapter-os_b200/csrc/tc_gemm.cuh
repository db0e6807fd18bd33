// tc_gemm.cuh — parameters of the tcgen05 weight-streaming GEMM (tc_gemm.cu).
//
// D[tokens, rows] = X[tokens, K] . W[rows, K]^T  (+ sum over touched LoRA rank
// groups of  Hm[tokens, 64 group cols] . B_cat[rows, 64 group cols]^T), i.e.
// the base projection y = x W^T of mlx_cpp_wrapper_real.cpp:3372-3381 fused
// with the LoRA shrink and expand of :3394-3419.  Decode tokens are the MMA's
// M (128 TMEM lanes) and weight rows its N (256 per tile): a kind::f16 MMA
// costs the same for every N up to 256, so 256 weight rows per instruction
// stream twice the bytes of 128.  Every pipeline step is 256 rows x 128 bytes
// of weights (two packed 16 KB blocks) plus a T x 128-byte box of activations
// (SWIZZLE_128B) and four K=16 MMAs.
#pragma once

#include <cuda.h>

#include "common.cuh"

namespace aos {

enum TcMode : int {
    TC_STORE_BF16 = 0,  // out[t][col] = bf16(acc)
    TC_RESID_BF16 = 1,  // resid[t][col] = bf16(resid + acc)          (o / down + residual)
    TC_STORE_F32 = 2,   // out[t][col] = acc                           (lm_head logits)
    TC_QKV_ROPE = 3,    // q -> out (RoPE), k -> paged K (RoPE), v -> paged V
    TC_SWIGLU = 4,      // out[t][f] = bf16(silu(gate) * up)            (n_sub = 2)
    TC_SHRINK_HM = 5    // hm[t][group col] = bf16(acc * gate(t, owner(col)))
};

constexpr int kTcMaxSets = 3;    // operand sets = segments x sub-tiles
constexpr int kTcThreads = 256;  // warp 0 TMA, warp 1 MMA, warps 2-5 drain, warps 6-7 convert
constexpr int kTcBN = 256;       // weight rows per tile = MMA N (gate/up: 128 + 128)
constexpr int kTcBK = 64;        // K elements per step (128 B, one SW128 row)
constexpr int kTcTok = 128;      // tokens per MMA = MMA M
constexpr int kBlkRows = 128;    // rows of one packed weight block (16 KB)
constexpr int kGroup = 64;       // LoRA rank columns per group (= one K step)
constexpr int kShrinkGroupsPerTile = kTcBN / kGroup;  // 4

struct TcParams {
    // Weights are read in the packed layout (pack_blocks_kernel): blocks of
    // 128 (lora_A: 64) rows x 64 columns, each the SWIZZLE_128B shared-memory
    // image of one box, so every weight box is one contiguous bulk copy.
    const uint16_t* w_pk[kTcMaxSets];  // base weights per segment x sub-tile: [row block][K step] blocks
    const uint16_t* a_pk[kTcMaxSets];  // lora_A [R, K] per shrink segment: [rank group][K step] blocks
    const uint16_t* b_pk[kTcMaxSets];  // lora_B [rows, R] per segment x sub-tile: [row block][rank group] blocks
    CUtensorMap tm_x;                  // activations [T, K], SW128 box 64 x T_box
    CUtensorMap tm_lh[kTcMaxSets];     // gated shrink output hm [T, R], SW128 box 64 x T_box
    int mode, n_sub, n_seg, T, T_pad, T_box, tb, kb, n_stages, lora;
    int pools;                      // work pools: 1 shrink K steps, 2 base K steps, 4 expand steps
    int sh_nseg;                    // shrink segments (LoRA modules that read X), 0 = none
    int n_rgroups;                  // rank groups of the arena (R / 64)
    int seg_tiles[kTcMaxSets];      // tiles per segment (256 rows; gate/up: 128 features)
    int seg_wrow0[kTcMaxSets];      // first W row of the segment (multiple of 128)
    int seg_out0[kTcMaxSets];       // first output feature of the segment
    int seg_rows[kTcMaxSets];       // valid output rows (features) of the segment
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
    // LoRA deltas computed by the adapter owners (adapter-sharded decode):
    // n_delta blocks of [T][ld_delta] bf16, delta_stride elements apart, one
    // per owner rank.  The epilogue adds their sum, taken in owner order, to
    // the accumulator before the mode's own math.  Segment s's columns start
    // at dseg0[s]; TC_SWIGLU reads the gate deltas at dseg0[0] and the up
    // deltas at dseg0[1].  Null = none.
    const uint16_t* delta;
    long long delta_stride;
    int n_delta, ld_delta;
    int dseg0[kTcMaxSets];
    int R;                          // arena rank capacity (columns of hm)
    // [T][n_rgroups slots][8]: gate * alpha/rank of the adapter owning each
    // 8-column unit of the slot-th touched group for each token (0 when the
    // token did not select it or the unit is free)
    const float* ucoef;
    // Fixed-point (x 2^32) int64 accumulators of tiles cut between CTAs,
    // [tile][256 columns][acc_T tokens]; all zero between launches (the
    // conversion re-zeroes what it reads).
    long long* acc;
    int acc_T;                      // token stride of the accumulator (T_cap)
    // Split base tiles write fp32 partial sums here with plain stores,
    // [slot][256 columns][acc_T tokens] with slot = CTA + base tile index
    // (unique per piece), and the final conversion sums a tile's pieces in
    // CTA order (fixed order: bit-identical run to run).  Shrink tiles keep
    // the fixed-point adds into acc, which touch only a token's own adapters'
    // columns.  Null selects fixed-point adds for base tiles too.
    float* part;
    // Token t sits in TMEM lane t % 128 of MMA token block t / 128.
    // RMSNorm folded into the neighbouring launches (decode).  A launch that
    // adds into the residual (o, down) also writes hw = bf16(h * w) with the
    // next norm's weight w and adds each token's sum of squares of h, in
    // fixed point (value * 2^16), into ss_out.  A launch that reads hw (q/k/v,
    // gate/up, lm_head) scales its outputs by 1 / sqrt(ss * ss_scale + eps)
    // per token (ss_scale = 2^-16 / H) and clears ss_in when it ends.
    unsigned long long* ss_out;
    uint16_t* hw_out;               // [T][ld_out] bf16
    const uint16_t* norm_w;         // [ld_out] bf16
    unsigned long long* ss_in;      // [T]
    float ss_scale, norm_eps;
    int* sync;                      // [4] grid barriers (shrink drained, shrink reduced, all drained, exit)
    int cooperative;                // host side: launch as a cooperative grid (shared-device mode)
    int* err;                       // device error word (0 = ok)
    unsigned long long* trace;      // optional per-CTA %globaltimer trace (null = off)
};

constexpr int kMaxPiecesPerPool = 30;  // a slice is at least 1/30 of a tile

// Trace layout per CTA (kTraceStride slots): [0,64) producer step issues,
// [64,128) MMA full-barrier waits done, [128,160) drain piece starts,
// [160,192) drain piece ends, 192 kernel start, 193 kernel end, 194-199 grid
// barrier events (arrive/complete of the three barriers), 200/201 final
// reduction start/end, 202/203 producer wait for the shrink output, 204
// producer's last shrink step issued, 205 MMA's last shrink step consumed,
// 206/207 converter's shrink share done / drain share done, 208/209 drain's
// shrink share start / end.
constexpr int kTraceStride = 256;

// Host helpers (tc_gemm.cu).
int tc_encode_2d(CUtensorMap* m, const void* base, uint64_t inner, uint64_t outer, uint64_t row_bytes,
                 uint32_t box_inner, uint32_t box_outer, int swizzle_bytes);
int tc_encode_3d(CUtensorMap* m, const void* base, uint64_t d0, uint64_t d1, uint64_t d2,
                 uint64_t stride1_bytes, uint64_t stride2_bytes, uint32_t b0, uint32_t b1, uint32_t b2,
                 int swizzle_bytes);
// Token padding of a batch of T (T_pad: multiple of 16) and the activation box
// height: T_pad rows, at most 128 (one MMA token block).
inline int tc_t_pad(int T) { return ((T + 15) / 16) * 16; }
inline int tc_t_box(int T) { return tc_t_pad(T) < kTcTok ? tc_t_pad(T) : kTcTok; }
// Fills T_pad, tb, T_box, stage sizes; returns 0 or an aos_status.
int tc_prepare(TcParams& p, int smem_budget);
// Launch on `grid` CTAs; every CTA must be resident at once (grid <= SM
// count): the launch synchronises its CTAs through bounded grid barriers.
// Failure-path check of the GEMM kernel's bounded waits (see tc_gemm.cu).
cudaError_t tc_debug_wait(int kind, const int* never, int* err, cudaStream_t s);
cudaError_t tc_launch(const TcParams& p, int grid, cudaStream_t stream);
// Prefill GEMM: data-parallel tiles of 128 tokens over the whole K (no split),
// for any T.  n_seg == 0 with sh_nseg > 0 is a shrink launch (gated hm out).
int pf_prepare(TcParams& p);
cudaError_t pf_launch(const TcParams& p, cudaStream_t stream);
// Bytes of the accumulator for n_tiles tiles (p.acc_T set).
size_t tc_acc_bytes(const TcParams& p, int n_tiles);
cudaError_t tc_configure();
size_t tc_smem_bytes(const TcParams& p);
int tc_num_sms();

}  // namespace aos
