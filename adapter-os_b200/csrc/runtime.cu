// runtime.cu — the backend context behind the C ABI: base weights, the LoRA
// adapter arena, the paged KV cache, per-batch-size step plans (prebuilt TMA
// descriptors + a captured CUDA graph) and the decode step itself.
//
// This is the B200 counterpart of a FusedKernels backend
// (crates/adapteros-lora-kernel-api/src/lib.rs:308-716): load() -> aos_init +
// aos_load_weight; load_adapter_with_metadata()/unload_adapter() ->
// aos_adapter_*; run_step() -> aos_run_step_batch; KV-cache methods ->
// aos_kv_*; get_metrics()/health_check()/attest_determinism().
//
// Arena layout (per layer and LoRA module, allocated once at init):
//   A_cat  [R][in]   bf16  lora_A rows of every adapter, adapter a at rows [off_a, off_a + r_a)
//   B_cat  [out][R]  bf16  lora_B columns of every adapter at columns [off_a, off_a + r_a)
// where R is the arena's rank capacity (a multiple of 64).  Column ranges are
// handed out in 8-column units aligned to the rank's power-of-two factor, and
// a decode step streams only the 64-column rank groups its tokens selected
// (one TMA box of 128 rows x 128 B per group and weight tile).

#include <algorithm>
#include <cfloat>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <memory>
#include <string>
#include <unordered_map>
#include <vector>

#include <nccl.h>

#include "loader.cuh"
#include "tc_gemm.cuh"

namespace aos {
cudaError_t launch_kv_shift_rows(uint16_t* k_pool, uint16_t* v_pool, const int* blocks, int n, int r, int new_len,
                                 int n_layers, int num_blocks, int nkv, cudaStream_t s);
cudaError_t launch_zero_kv_blocks(uint16_t* k_pool, uint16_t* v_pool, const int* blocks, int n, int n_layers,
                                  int num_blocks, int nkv, cudaStream_t s);
cudaError_t launch_embed(const uint16_t*, const uint32_t*, int, int, int, uint16_t*, cudaStream_t);
cudaError_t launch_rmsnorm(const uint16_t*, const uint16_t*, int, int, float, uint16_t*, cudaStream_t);
cudaError_t launch_norm_prep(const uint16_t*, const uint16_t*, int, int, uint16_t*, unsigned long long*, cudaStream_t);
cudaError_t launch_lora_prep(const aos_router_ring* rings, int T, const int* col_off, const int* rank,
                             const float* scale, int max_adapters, int n_slab_total, int* slabs, int* n_slabs,
                             float* coef, const int* col_owner, float* ucoef, cudaStream_t s);
cudaError_t launch_fill_normal(uint16_t*, size_t, uint64_t, float, cudaStream_t);
cudaError_t launch_zero_if_no_groups(const int* n_groups, uint16_t* p, size_t n, cudaStream_t s);
cudaError_t launch_pack_blocks(const uint16_t* src, int rows, int cols, long long src_ld, uint16_t* dst, int row0,
                               int col0, int dst_cols, int br, cudaStream_t s);
cudaError_t launch_attention(const CUtensorMap&, const CUtensorMap&, const uint16_t*, const int*, const int*, float*,
                             float*, int*, int, int, int, int, int, int, int, int*, uint16_t*, cudaStream_t);
int attn_max_chunks(int max_seq_len);
cudaError_t launch_attention_prefill(const CUtensorMap& tm_k, const CUtensorMap& tm_v, const uint16_t* q,
                                     const int* block_tables, const int* pos, const int2* qblk, int n_qblk, int nq,
                                     int nkv, int layer, int num_blocks, int max_blocks, int* err, uint16_t* out,
                                     cudaStream_t s);
cudaError_t attn_configure();
bool attn_prefill_tc_supported(int nq, int nkv);
int attn_prefill_tc_block(int nq, int nkv);
cudaError_t attn_tc_configure();
cudaError_t launch_attention_prefill_tc(const CUtensorMap& tm_q, const CUtensorMap& tm_k, const CUtensorMap& tm_v,
                                        const int* block_tables, const int* pos, const int2* qblk, int n_qblk, int nq,
                                        int nkv, int layer, int num_blocks, int max_blocks, int* err, uint16_t* out,
                                        cudaStream_t s);
}  // namespace aos

using namespace aos;

namespace {

constexpr int kGroupQKV = 0, kGroupO = 1, kGroupGU = 2, kGroupD = 3;

struct AdapterEntry {
    int off = -1;
    int rank = 0;
    float alpha = 0.f;
};

struct Sequence {
    std::vector<int> blocks;
    uint32_t len = 0;
    uint32_t cap = 0;
};

struct LayerPlan {
    TcParams gemm[4];    // per input group: LoRA shrink + base + LoRA expand in one launch
    TcParams owner[4];   // adapter-sharded step: this rank's LoRA (shrink + expand) for every rank's rows
    int gemm_grid[4];
};

struct StepPlan {
    int T = 0, T_pad = 0;
    bool sharded = false;  // adapter-sharded step: T home tokens, T * world rows at the owner
    bool eager_done = false;  // sharded: the first step runs uncaptured (NCCL connects its peers)
    std::vector<LayerPlan> layers;
    TcParams lm_head;
    int lm_grid = 0;
    void* logits_dst = nullptr;
    cudaGraphExec_t graph = nullptr;
    void* graph_logits = nullptr;
    bool graph_valid = false;
};

}  // namespace

struct aos_ctx {
    aos_model_config cfg{};
    int device = 0;
    cudaStream_t stream = nullptr;
    std::string err;
    std::string dev_name;
    uint32_t QD = 0, KVD = 0, G = 0;
    uint32_t module_mask = 0;

    // base weights
    uint16_t *embed = nullptr, *lm_head = nullptr, *final_norm = nullptr;
    std::vector<uint16_t*> attn_norm, mlp_norm, w_qkv, w_o, w_gate, w_up, w_down;
    std::vector<uint8_t> loaded;  // bookkeeping of loaded tensors
    uint64_t base_bytes = 0;

    // arena
    int R = 0;
    std::vector<uint16_t*> A[AOS_NUM_MODULES], B[AOS_NUM_MODULES];  // [layer]
    int *d_col_owner = nullptr, *d_col_off = nullptr, *d_rank = nullptr;
    float* d_scale = nullptr;
    float* d_coef = nullptr;  // [T_cap][max_adapters] per-step gate * alpha/rank
    float* d_ucoef = nullptr; // [T_cap][R/64 touched-group slots][8 units] per-step unit coefficients
    std::vector<int> col_owner;  // host mirror, 8-column units
    std::unordered_map<uint16_t, AdapterEntry> adapters;
    std::map<uint16_t, std::pair<uint64_t, std::string>> fingerprints;  // id -> (buffer bytes, checkpoint hash hex)
    struct Footprint {  // MemoryFootprintBaseline (kernel-mtl/src/vram.rs:82-196)
        std::vector<uint64_t> samples;
        size_t max_samples = 0;
    };
    std::map<uint16_t, Footprint> footprints;
    uint64_t kv_generation = 0;                  // KvCache::stack_generation
    std::map<uint64_t, uint64_t> kv_guards;      // sequence -> generation it was allocated under
    uint64_t arena_bytes = 0;

    // KV cache
    uint16_t *k_pool = nullptr, *v_pool = nullptr;
    std::vector<int> free_blocks;
    std::unordered_map<uint64_t, Sequence> seqs;
    int max_blocks = 0;
    CUtensorMap tm_k{}, tm_v{};

    // scratch
    int T_cap = 0;
    uint16_t *d_hidden = nullptr, *d_normed = nullptr, *d_q = nullptr, *d_attn = nullptr, *d_act = nullptr;
    uint16_t* d_hm[AOS_NUM_MODULES] = {};
    int *d_groups = nullptr, *d_n_groups = nullptr;
    int *d_block_tables = nullptr, *d_ctx_lens = nullptr;
    int* d_zero_blocks = nullptr;  // [kv_num_blocks]: block list of aos_kv_zeroize
    // Pinned staging of the per-step block tables and lengths.  A ring of
    // kStageSlots buffers, each reused only after the event recorded behind
    // its last copy has completed, so the host may run steps ahead of the GPU
    // without overwriting a table that a queued copy has not read yet.
    static constexpr int kStageSlots = 4;
    int* h_stage[kStageSlots] = {};
    cudaEvent_t stage_ev[kStageSlots] = {};
    int stage_slot = 0;
    int *h_block_tables = nullptr, *h_ctx_lens = nullptr;  // the slot being filled
    aos_router_ring* d_rings = nullptr;
    uint32_t* d_tokens = nullptr;
    float* d_logits = nullptr;
    float *d_rope = nullptr;
    float *d_attn_part = nullptr, *d_attn_ml = nullptr;
    int* d_attn_cnt = nullptr;  // [T_cap][n_kv] decode attention chunks counted, zero between launches
    unsigned long long* d_ss = nullptr;  // [T_cap] folded RMSNorm: sum of squares of each token's hidden row
    int attn_chunks = 0;
    uint16_t* d_stage = nullptr;  // bounded staging for packing host or unaligned weights
    size_t stage_bytes = 0;
    long long* d_acc = nullptr;   // GEMM fixed-point accumulators of split shrink tiles (kept zero)
    size_t acc_bytes = 0;
    float* d_part = nullptr;      // GEMM fp32 partials of split base tiles
    uint16_t* d_fp = nullptr;     // adapter buffer samples [3][2048] for fingerprints
    int* d_sync = nullptr;        // [4] GEMM grid-barrier counters
    int gemm_coop = 0;            // AOS_GEMM_COOPERATIVE=1: cooperative GEMM launches (shared device)
    int* d_err = nullptr;
    unsigned long long* d_trace = nullptr;  // AOS_TC_TRACE diagnostics

    // Adapter-sharded decode (aos_shard_init): this rank owns the adapters
    // with id % world == rank.  Per layer and input site every rank sends its
    // T input rows to every rank (NCCL send/recv), each rank runs the LoRA of
    // its own adapters on all world * T rows, and the bf16 deltas go back to
    // the rows' home ranks, which add them in owner order in the base GEMM's
    // epilogue.
    int shard_rank = 0, shard_world = 1;
    ncclComm_t nccl = nullptr;
    uint16_t* d_xrecv = nullptr;       // [world * T][in]  rows from every rank (rank-major)
    uint16_t* d_dsend = nullptr;       // [world * T][W]   this rank's deltas for every rank's rows
    uint16_t* d_drecv = nullptr;       // [world][T][W]    deltas for the home rows, by owner
    aos_router_ring* d_rings_all = nullptr;  // [world * T] every rank's rings (rank-major)

    // Prefill (aos_prefill_dev): activations of every prompt token, grown on
    // demand to the largest prompt batch seen.
    struct Prefill {
        int cap = 0;  // tokens
        uint16_t *hidden = nullptr, *normed = nullptr, *q = nullptr, *attn = nullptr, *act = nullptr;
        uint16_t* hm[AOS_NUM_MODULES] = {};
        float *coef = nullptr, *ucoef = nullptr;
        aos_router_ring* rings = nullptr;
        uint32_t* tokens = nullptr;
        int *pos = nullptr, *block_tables = nullptr;
        int2* qblk = nullptr;
    } pf;
    std::map<int, std::unique_ptr<StepPlan>> plans;

    // metrics
    aos_metrics m{};
    bool prof_on = false;
    std::vector<cudaEvent_t> prof_ev;
    std::vector<int> prof_cls;
    size_t prof_used = 0;
    aos_profile prof{};
    cudaEvent_t ev0 = nullptr, ev1 = nullptr;

    int fail(int code, const std::string& msg) {
        err = msg;
        return code;
    }
};

namespace {

#define CTX_CUDA(ctx, expr)                                                                  \
    do {                                                                                     \
        cudaError_t _e = (expr);                                                             \
        if (_e != cudaSuccess)                                                               \
            return (ctx)->fail(AOS_ERR_CUDA, std::string(#expr ": ") + cudaGetErrorString(_e)); \
    } while (0)

uint32_t mod_out(const aos_ctx* c, int m) {
    const uint32_t H = c->cfg.hidden, I = c->cfg.intermediate;
    const uint32_t outs[7] = {c->QD, c->KVD, c->KVD, H, I, I, H};
    return outs[m];
}
uint32_t mod_in(const aos_ctx* c, int m) {
    const uint32_t H = c->cfg.hidden, I = c->cfg.intermediate;
    const uint32_t ins[7] = {H, H, H, c->QD, H, H, I};
    return ins[m];
}

template <class T>
cudaError_t dalloc(T** p, size_t n_elems, uint64_t* counter = nullptr) {
    cudaError_t e = cudaMalloc((void**)p, n_elems * sizeof(T) + 256);
    if (e == cudaSuccess) {
        e = cudaMemset(*p, 0, n_elems * sizeof(T));
        if (counter) *counter += n_elems * sizeof(T);
    }
    return e;
}

// Upper bound of the tiles of one GEMM launch (base tiles of the largest
// projection plus shrink tiles of up to three LoRA modules).
size_t max_launch_tiles(const aos_ctx* c) {
    const size_t H = c->cfg.hidden, I = c->cfg.intermediate, V = c->cfg.vocab;
    const size_t base = std::max<size_t>({(c->QD + 2 * (size_t)c->KVD) / kTcBN + 3, (I + 127) / 128, (H + kTcBN - 1) / kTcBN,
                                          (V + kTcBN - 1) / kTcBN});
    return base + 3 * ((size_t)c->R / kGroup / kShrinkGroupsPerTile + 1);
}

// This rank's LoRA for input site g of one layer over the T rows of every
// rank (rank-major in d_xrecv): shrink of each module's touched groups, then
// the expand, stored as bf16 deltas [T][W] (modules side by side) in d_dsend.
// Adapters this rank does not own have no arena columns, so the prep kernel's
// touched-group list and coefficients cover only this rank's adapters.
int build_owner_plan(aos_ctx* c, int layer, int g, int T, TcParams& p) {
    const uint32_t H = c->cfg.hidden, I = c->cfg.intermediate;
    const int T_box = tc_t_box(T);
    const int mods[4][3] = {{AOS_MOD_Q, AOS_MOD_K, AOS_MOD_V}, {AOS_MOD_O, -1, -1}, {AOS_MOD_GATE, AOS_MOD_UP, -1},
                            {AOS_MOD_DOWN, -1, -1}};
    const uint32_t K[4] = {H, c->QD, H, I};
    std::memset(&p, 0, sizeof(p));
    p.T = T;
    p.groups = c->d_groups;
    p.n_groups = c->d_n_groups;
    p.acc = c->d_acc;
    p.acc_T = c->T_cap;
    p.part = c->d_part;
    p.sync = c->d_sync;
    p.cooperative = c->gemm_coop;
    p.err = c->d_err;
    p.R = c->R;
    p.n_rgroups = c->R / kGroup;
    p.ucoef = c->d_ucoef;
    p.layer = layer;
    p.lora = 1;
    p.kb = (int)(K[g] / 64);
    int rc = tc_encode_2d(&p.tm_x, c->d_xrecv, K[g], (uint64_t)c->T_cap, (uint64_t)K[g] * 2, 64, (uint32_t)T_box, 128);
    if (rc) return rc;
    p.mode = TC_STORE_BF16;
    p.n_sub = 1;
    int col = 0;
    for (int j = 0; j < 3; ++j) {
        const int mod = mods[g][j];
        if (mod < 0) continue;
        p.a_pk[p.sh_nseg] = c->A[mod][layer];
        p.sh_out[p.sh_nseg] = c->d_hm[mod];
        ++p.sh_nseg;
        const int s = p.n_seg++;
        const int rows = (int)mod_out(c, mod);
        p.b_pk[s] = c->B[mod][layer];
        if ((rc = tc_encode_2d(&p.tm_lh[s], c->d_hm[mod], (uint64_t)c->R, (uint64_t)c->T_cap, (uint64_t)c->R * 2, kGroup,
                               (uint32_t)T_box, 128)))
            return rc;
        p.seg_tiles[s] = (rows + kTcBN - 1) / kTcBN;
        p.seg_rows[s] = rows;
        p.seg_module[s] = mod;
        p.seg_out0[s] = col;
        p.out[s] = c->d_dsend;
        col += rows;
    }
    p.ld_out = col;
    p.pools = 1 | 4;  // shrink and expand, no base weights
    return tc_prepare(p, 227 * 1024);
}

// Build the TcParams of every GEMM of one layer for a batch of T tokens.
// sharded: the base GEMMs carry no LoRA of their own but add the deltas the
// adapter owners return, and owner[g] is this rank's LoRA launch over the
// world * T rows of every rank.
int build_layer_plan(aos_ctx* c, int layer, int T, LayerPlan& lp, bool sharded = false) {
    const uint32_t H = c->cfg.hidden, I = c->cfg.intermediate;
    const int T_box = tc_t_box(T);  // activation box rows (128 per token block at most)
    const int smem_budget = 227 * 1024;
    int rc;
    auto x_map = [&](CUtensorMap* m, const uint16_t* buf, uint32_t K) {
        return tc_encode_2d(m, buf, K, (uint64_t)c->T_cap, (uint64_t)K * 2, 64, (uint32_t)T_box, 128);
    };
    auto h_map = [&](CUtensorMap* m, int mod) {  // hm [T][R]
        return tc_encode_2d(m, c->d_hm[mod], (uint64_t)c->R, (uint64_t)c->T_cap, (uint64_t)c->R * 2, kGroup,
                            (uint32_t)T_box, 128);
    };
    auto common = [&](TcParams& p) {
        std::memset(&p, 0, sizeof(p));
        p.T = T;
        p.groups = c->d_groups;
        p.n_groups = c->d_n_groups;
        p.acc = c->d_acc;
        p.acc_T = c->T_cap;
        p.part = c->d_part;
        p.sync = c->d_sync;
        p.cooperative = c->gemm_coop;
        p.err = c->d_err;
        p.R = c->R;
        p.n_rgroups = c->R / kGroup;
        p.ucoef = c->d_ucoef;
        p.layer = layer;
    };
    const bool lora[4] = {(c->module_mask & 0x7u) != 0, (c->module_mask & 0x8u) != 0, (c->module_mask & 0x30u) != 0,
                          (c->module_mask & 0x40u) != 0};
    const int groups_mods[4][3] = {{AOS_MOD_Q, AOS_MOD_K, AOS_MOD_V}, {AOS_MOD_O, -1, -1},
                                   {AOS_MOD_GATE, AOS_MOD_UP, -1}, {AOS_MOD_DOWN, -1, -1}};
    const uint16_t* group_x[4] = {c->d_normed, c->d_attn, c->d_normed, c->d_act};
    const uint32_t group_k[4] = {H, c->QD, H, I};

    for (int g = 0; g < 4; ++g) {
        // ---------------- LoRA shrink + base GEMM + fused LoRA expand + epilogue
        TcParams& p = lp.gemm[g];
        common(p);
        p.lora = (lora[g] && !sharded) ? 1 : 0;
        p.kb = (int)(group_k[g] / 64);
        if ((rc = x_map(&p.tm_x, group_x[g], group_k[g]))) return rc;
        if (p.lora) {  // hm = gate * (A_cat x) of every module of the group, in the same launch
            for (int j = 0; j < 3; ++j) {
                const int mod = groups_mods[g][j];
                if (mod < 0) continue;
                p.a_pk[p.sh_nseg] = c->A[mod][layer];
                p.sh_out[p.sh_nseg] = c->d_hm[mod];
                ++p.sh_nseg;
            }
        }
        if (g == kGroupQKV) {
            p.mode = TC_QKV_ROPE;
            p.n_sub = 1;
            p.n_seg = 3;
            const uint32_t rows_total = c->QD + 2 * c->KVD;
            const uint32_t r0[3] = {0, c->QD, c->QD + c->KVD};
            const uint32_t nr[3] = {c->QD, c->KVD, c->KVD};
            for (int j = 0; j < 3; ++j) {
                p.w_pk[j] = c->w_qkv[layer];
                p.seg_wrow0[j] = (int)r0[j];
                p.seg_tiles[j] = (int)((nr[j] + kTcBN - 1) / kTcBN);  // two heads per tile
                p.seg_rows[j] = (int)nr[j];
                p.seg_module[j] = groups_mods[g][j];
                p.seg_out0[j] = 0;
                if (p.lora) {
                    p.b_pk[j] = c->B[groups_mods[g][j]][layer];
                    if ((rc = h_map(&p.tm_lh[j], groups_mods[g][j]))) return rc;
                }
            }
            p.out[0] = p.out[1] = p.out[2] = c->d_q;
            p.ld_out = (int)c->QD;
            p.rope = c->d_rope;
            p.k_pool = c->k_pool;
            p.v_pool = c->v_pool;
            p.block_tables = c->d_block_tables;
            p.ctx_lens = c->d_ctx_lens;
            p.max_blocks = c->max_blocks;
            p.num_blocks = (int)c->cfg.kv_num_blocks;
            p.nkv = (int)c->cfg.n_kv_heads;
        } else if (g == kGroupGU) {
            p.mode = TC_SWIGLU;
            p.n_sub = 2;
            p.n_seg = 1;
            p.w_pk[0] = c->w_gate[layer];
            p.w_pk[1] = c->w_up[layer];
            if (p.lora) {
                p.b_pk[0] = c->B[AOS_MOD_GATE][layer];
                p.b_pk[1] = c->B[AOS_MOD_UP][layer];
                if ((rc = h_map(&p.tm_lh[0], AOS_MOD_GATE))) return rc;
                if ((rc = h_map(&p.tm_lh[1], AOS_MOD_UP))) return rc;
            }
            p.seg_tiles[0] = (int)((I + kTcBN / 2 - 1) / (kTcBN / 2));  // 128 gate + 128 up rows per tile
            p.seg_rows[0] = (int)I;
            p.seg_module[0] = AOS_MOD_GATE;
            p.out[0] = c->d_act;
            p.ld_out = (int)I;
        } else {
            const int mod = g == kGroupO ? AOS_MOD_O : AOS_MOD_DOWN;
            p.mode = TC_RESID_BF16;
            p.n_sub = 1;
            p.n_seg = 1;
            p.w_pk[0] = g == kGroupO ? c->w_o[layer] : c->w_down[layer];
            if (p.lora) {
                p.b_pk[0] = c->B[mod][layer];
                if ((rc = h_map(&p.tm_lh[0], mod))) return rc;
            }
            p.seg_tiles[0] = (int)((H + kTcBN - 1) / kTcBN);
            p.seg_rows[0] = (int)H;
            p.seg_module[0] = mod;
            p.resid = c->d_hidden;
            p.ld_out = (int)H;
        }
        if (sharded && lora[g]) {
            // deltas of every owner rank: [world][T][W], W = the site's output width
            const uint32_t W[4] = {c->QD + 2 * c->KVD, H, 2 * I, H};
            p.delta = c->d_drecv;
            p.n_delta = c->shard_world;
            p.ld_delta = (int)W[g];
            p.delta_stride = (long long)T * W[g];
            if (g == kGroupQKV) {
                p.dseg0[0] = 0;
                p.dseg0[1] = (int)c->QD;
                p.dseg0[2] = (int)(c->QD + c->KVD);
            } else if (g == kGroupGU) {
                p.dseg0[0] = 0;
                p.dseg0[1] = (int)I;
            }
            if ((rc = build_owner_plan(c, layer, g, T * c->shard_world, lp.owner[g]))) return rc;
        }
        // RMSNorm folded into the neighbouring launches: o and down write the
        // next norm's hw = h * w (into d_normed) and each token's sum of h^2;
        // q/k/v and gate/up read hw and scale by 1 / rms in their epilogue
        if (g == kGroupQKV || g == kGroupGU) {
            p.ss_in = c->d_ss;
            p.ss_scale = (float)(1.0 / 65536.0 / (double)H);
            p.norm_eps = c->cfg.rms_eps;
        } else {
            p.ss_out = c->d_ss;
            p.hw_out = c->d_normed;
            p.norm_w = g == kGroupO ? c->mlp_norm[layer]
                                    : (layer + 1 < (int)c->cfg.n_layers ? c->attn_norm[layer + 1] : c->final_norm);
        }
        p.pools = 7;
        if ((rc = tc_prepare(p, smem_budget))) return rc;
        lp.gemm_grid[g] = tc_num_sms();
        // Diagnostics: AOS_TC_TRACE=<0..3> traces layer 0's GEMM g.
        if (const char* tv = getenv("AOS_TC_TRACE"))
            if (layer == 0 && c->d_trace && atoi(tv) == g) p.trace = c->d_trace;
    }
    return AOS_OK;
}

int get_plan(aos_ctx* c, int T, StepPlan** out, bool sharded = false) {
    const int T_pad = std::max(32, ((T + 15) / 16) * 16);
    const int key = sharded ? -T : T;
    auto it = c->plans.find(key);
    if (it != c->plans.end()) {
        *out = it->second.get();
        return AOS_OK;
    }
    auto plan = std::make_unique<StepPlan>();
    plan->T = T;
    plan->T_pad = T_pad;
    plan->sharded = sharded;
    plan->layers.resize(c->cfg.n_layers);
    for (uint32_t l = 0; l < c->cfg.n_layers; ++l) {
        int rc = build_layer_plan(c, (int)l, T, plan->layers[l], sharded);
        if (rc) return c->fail(rc, "building the GEMM plan failed (tensor map encode)");
    }
    // lm_head: logits = normed . lm_head^T (f32 out)
    TcParams& p = plan->lm_head;
    std::memset(&p, 0, sizeof(p));
    p.T = T;
    p.mode = TC_STORE_F32;
    p.pools = 7;
    p.n_sub = 1;
    p.n_seg = 1;
    p.kb = (int)(c->cfg.hidden / 64);
    p.err = c->d_err;
    p.acc = c->d_acc;
    p.acc_T = c->T_cap;
    p.part = c->d_part;
    p.sync = c->d_sync;
    p.cooperative = c->gemm_coop;
    const uint32_t V = c->cfg.vocab;
    p.w_pk[0] = c->lm_head;
    int rc = tc_encode_2d(&p.tm_x, c->d_normed, c->cfg.hidden, (uint64_t)c->T_cap, (uint64_t)c->cfg.hidden * 2, 64,
                       (uint32_t)tc_t_box(T), 128);
    if (rc) return c->fail(AOS_ERR_CUDA, "lm_head tensor map encode failed");
    p.seg_tiles[0] = (int)((V + kTcBN - 1) / kTcBN);
    p.seg_rows[0] = (int)V;
    p.out[0] = c->d_logits;
    p.ld_out = (int)V;
    p.ss_in = c->d_ss;  // the final norm, folded: hw from the last down launch, 1 / rms here
    p.ss_scale = (float)(1.0 / 65536.0 / (double)c->cfg.hidden);
    p.norm_eps = c->cfg.rms_eps;
    if ((rc = tc_prepare(p, 227 * 1024))) return c->fail(rc, "lm_head plan");
    plan->lm_grid = tc_num_sms();
    *out = plan.get();
    c->plans[key] = std::move(plan);
    return AOS_OK;
}

#define LAUNCH(ctx, expr)                                                                       \
    do {                                                                                        \
        cudaError_t _e = (expr);                                                                \
        if (_e != cudaSuccess)                                                                  \
            return (ctx)->fail(AOS_ERR_CUDA, std::string("launch " #expr ": ") + cudaGetErrorString(_e)); \
    } while (0)

// Per-kernel-class device timing (aos_profile_enable): each launch is
// bracketed by two CUDA events taken from a pool; aos_profile_read sums them.
int prof_begin(aos_ctx* c, int cls, cudaStream_t s);
void prof_end(aos_ctx* c, int slot, cudaStream_t s);

#define PLAUNCH(ctx, cls, s, expr)                 \
    do {                                           \
        const int _slot = prof_begin(ctx, cls, s); \
        LAUNCH(ctx, expr);                         \
        prof_end(ctx, _slot, s);                   \
    } while (0)

#define NCCL_CHECK(ctx, expr)                                                                      \
    do {                                                                                           \
        ncclResult_t _r = (expr);                                                                  \
        if (_r != ncclSuccess) return (ctx)->fail(AOS_ERR_CUDA, std::string(#expr ": ") + ncclGetErrorString(_r)); \
    } while (0)

// Adapter-sharded step, input site g of one layer: x [T][in] (the home rows)
// goes to every rank; this rank's LoRA over the world * T rows it received
// writes deltas [world * T][W]; block o of them goes back to rank o, and the
// base GEMM of the site adds the blocks it receives, in owner order, in its
// epilogue (lp.gemm[g].delta).
int shard_site(aos_ctx* c, const StepPlan& plan, const LayerPlan& lp, int g, const uint16_t* x, uint32_t in,
               cudaStream_t s) {
    const int world = c->shard_world;
    const size_t nx = (size_t)plan.T * in, nd = (size_t)plan.T * lp.gemm[g].ld_delta;
    int slot = prof_begin(c, AOS_K_COMM, s);
    NCCL_CHECK(c, ncclGroupStart());
    for (int o = 0; o < world; ++o) {
        NCCL_CHECK(c, ncclSend(x, nx, ncclBfloat16, o, c->nccl, s));
        NCCL_CHECK(c, ncclRecv(c->d_xrecv + (size_t)o * nx, nx, ncclBfloat16, o, c->nccl, s));
    }
    NCCL_CHECK(c, ncclGroupEnd());
    prof_end(c, slot, s);
    PLAUNCH(c, AOS_K_SHRINK, s, tc_launch(lp.owner[g], lp.gemm_grid[g], s));
    slot = prof_begin(c, AOS_K_COMM, s);
    NCCL_CHECK(c, ncclGroupStart());
    for (int o = 0; o < world; ++o) {
        NCCL_CHECK(c, ncclSend(c->d_dsend + (size_t)o * nd, nd, ncclBfloat16, o, c->nccl, s));
        NCCL_CHECK(c, ncclRecv(c->d_drecv + (size_t)o * nd, nd, ncclBfloat16, o, c->nccl, s));
    }
    NCCL_CHECK(c, ncclGroupEnd());
    prof_end(c, slot, s);
    return AOS_OK;
}

// Enqueue one decoder layer on `s` (hidden state in ctx->d_hidden).
int enqueue_layer(aos_ctx* c, const StepPlan& plan, int layer, cudaStream_t s) {
    const LayerPlan& lp = plan.layers[layer];
    const int T = plan.T;
    const uint32_t H = c->cfg.hidden;
    if (plan.sharded) {
        const bool lora[4] = {lp.gemm[kGroupQKV].delta != nullptr, lp.gemm[kGroupO].delta != nullptr,
                              lp.gemm[kGroupGU].delta != nullptr, lp.gemm[kGroupD].delta != nullptr};
        int rc;
        // d_normed holds hw (the norms are folded into the GEMMs)
        if (lora[kGroupQKV] && (rc = shard_site(c, plan, lp, kGroupQKV, c->d_normed, H, s))) return rc;
        PLAUNCH(c, AOS_K_GEMM, s, tc_launch(lp.gemm[kGroupQKV], lp.gemm_grid[kGroupQKV], s));
        PLAUNCH(c, AOS_K_ATTN, s,
                launch_attention(c->tm_k, c->tm_v, c->d_q, c->d_block_tables, c->d_ctx_lens, c->d_attn_part, c->d_attn_ml,
                                 c->d_attn_cnt, T, (int)c->cfg.n_heads, (int)c->cfg.n_kv_heads, layer, (int)c->cfg.kv_num_blocks,
                                 c->max_blocks, c->attn_chunks, c->d_err, c->d_attn, s));
        if (lora[kGroupO] && (rc = shard_site(c, plan, lp, kGroupO, c->d_attn, c->QD, s))) return rc;
        PLAUNCH(c, AOS_K_GEMM, s, tc_launch(lp.gemm[kGroupO], lp.gemm_grid[kGroupO], s));
        if (lora[kGroupGU] && (rc = shard_site(c, plan, lp, kGroupGU, c->d_normed, H, s))) return rc;
        PLAUNCH(c, AOS_K_GEMM, s, tc_launch(lp.gemm[kGroupGU], lp.gemm_grid[kGroupGU], s));
        if (lora[kGroupD] && (rc = shard_site(c, plan, lp, kGroupD, c->d_act, c->cfg.intermediate, s))) return rc;
        PLAUNCH(c, AOS_K_GEMM, s, tc_launch(lp.gemm[kGroupD], lp.gemm_grid[kGroupD], s));
        return AOS_OK;
    }
    // the attention norm arrives folded: hw in d_normed and the sums in d_ss,
    // from the previous layer's down launch (or the step's norm prep)
    PLAUNCH(c, AOS_K_GEMM, s, tc_launch(lp.gemm[kGroupQKV], lp.gemm_grid[kGroupQKV], s));
    PLAUNCH(c, AOS_K_ATTN, s,
            launch_attention(c->tm_k, c->tm_v, c->d_q, c->d_block_tables, c->d_ctx_lens, c->d_attn_part, c->d_attn_ml,
                             c->d_attn_cnt, T,
                             (int)c->cfg.n_heads, (int)c->cfg.n_kv_heads, layer, (int)c->cfg.kv_num_blocks, c->max_blocks,
                             c->attn_chunks, c->d_err, c->d_attn, s));
    PLAUNCH(c, AOS_K_GEMM, s, tc_launch(lp.gemm[kGroupO], lp.gemm_grid[kGroupO], s));  // + the MLP norm's first half
    PLAUNCH(c, AOS_K_GEMM, s, tc_launch(lp.gemm[kGroupGU], lp.gemm_grid[kGroupGU], s));
    PLAUNCH(c, AOS_K_GEMM, s, tc_launch(lp.gemm[kGroupD], lp.gemm_grid[kGroupD], s));
    return AOS_OK;
}

// Device part of a decode step: routing prep, embedding, layers, final norm, lm_head.
int enqueue_step(aos_ctx* c, StepPlan& plan, bool with_logits, cudaStream_t s) {
    const int T = plan.T;
    if (plan.sharded) {
        // every rank's rings (rank-major), then the touched groups and
        // coefficients of this rank's adapters over all world * T rows
        const int slot = prof_begin(c, AOS_K_COMM, s);
        NCCL_CHECK(c, ncclAllGather(c->d_rings, c->d_rings_all, (size_t)T * sizeof(aos_router_ring), ncclUint8, c->nccl, s));
        prof_end(c, slot, s);
        const int TG = T * c->shard_world;
        PLAUNCH(c, AOS_K_PREP, s,
                launch_lora_prep(c->d_rings_all, TG, c->d_col_off, c->d_rank, c->d_scale, (int)c->cfg.lora_max_adapters,
                                 c->R / kGroup, c->d_groups, c->d_n_groups, c->d_coef, c->d_col_owner, c->d_ucoef, s));
        // no touched group: the owner launches have no work and write no
        // deltas, so the delta rows must read as zero
        PLAUNCH(c, AOS_K_PREP, s,
                launch_zero_if_no_groups(c->d_n_groups, c->d_dsend, (size_t)TG * 2 * c->cfg.intermediate, s));
    } else {
        PLAUNCH(c, AOS_K_PREP, s,
                launch_lora_prep(c->d_rings, T, c->d_col_off, c->d_rank, c->d_scale, (int)c->cfg.lora_max_adapters,
                                 c->R / kGroup, c->d_groups, c->d_n_groups, c->d_coef, c->d_col_owner, c->d_ucoef, s));
    }
    PLAUNCH(c, AOS_K_EMBED, s, launch_embed(c->embed, c->d_tokens, T, (int)c->cfg.hidden, (int)c->cfg.vocab, c->d_hidden, s));
    // layer 0's attention norm, first half (every later norm is folded into
    // the launch that writes the residual)
    PLAUNCH(c, AOS_K_NORM, s,
            launch_norm_prep(c->d_hidden, c->attn_norm[0], T, (int)c->cfg.hidden, c->d_normed, c->d_ss, s));
    for (uint32_t l = 0; l < c->cfg.n_layers; ++l) {
        int rc = enqueue_layer(c, plan, (int)l, s);
        if (rc) return rc;
    }
    if (with_logits)  // the final norm: hw and sums from the last down launch
        PLAUNCH(c, AOS_K_LM_HEAD, s, tc_launch(plan.lm_head, plan.lm_grid, s));
    return AOS_OK;
}

int prof_begin(aos_ctx* c, int cls, cudaStream_t s) {
    if (!c->prof_on) return -1;
    if (c->prof_used + 2 > c->prof_ev.size()) {
        for (int i = 0; i < 64; ++i) {
            cudaEvent_t e;
            if (cudaEventCreate(&e) != cudaSuccess) return -1;
            c->prof_ev.push_back(e);
        }
        c->prof_cls.resize(c->prof_ev.size() / 2);
    }
    const int slot = (int)c->prof_used;
    c->prof_used += 2;
    c->prof_cls[slot / 2] = cls;
    cudaEventRecord(c->prof_ev[slot], s);
    return slot;
}

void prof_end(aos_ctx* c, int slot, cudaStream_t s) {
    if (slot >= 0) cudaEventRecord(c->prof_ev[slot + 1], s);
}

int run_step_device(aos_ctx* c, int T, bool with_logits, cudaStream_t s, bool sharded = false) {
    StepPlan* plan = nullptr;
    int rc = get_plan(c, T, &plan, sharded);
    if (rc) return rc;
    if (c->prof_on) {  // instrumented, graph-less step; times are collected after the step
        rc = enqueue_step(c, *plan, with_logits, s);
        if (rc) return rc;
        CTX_CUDA(c, cudaStreamSynchronize(s));
        for (size_t i = 0; i + 1 < c->prof_used; i += 2) {
            float ms = 0.f;
            cudaEventElapsedTime(&ms, c->prof_ev[i], c->prof_ev[i + 1]);
            c->prof.ms[c->prof_cls[i / 2]] += ms;
            c->prof.launches[c->prof_cls[i / 2]] += 1;
        }
        c->prof_used = 0;
        c->prof.steps += 1;
        int ns = 0;
        CTX_CUDA(c, cudaMemcpy(&ns, c->d_n_groups, 4, cudaMemcpyDeviceToHost));
        c->prof.last_touched_groups = (uint32_t)ns;
        return AOS_OK;
    }
    if (plan->sharded && !plan->eager_done) {
        plan->eager_done = true;
        return enqueue_step(c, *plan, with_logits, s);
    }
    if (!plan->graph_valid || (plan->graph_logits != (void*)(with_logits ? c->d_logits : nullptr))) {
        if (plan->graph) cudaGraphExecDestroy(plan->graph);
        plan->graph = nullptr;
        cudaGraph_t g;
        CTX_CUDA(c, cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal));
        rc = enqueue_step(c, *plan, with_logits, s);
        cudaError_t e = cudaStreamEndCapture(s, &g);
        if (rc) return rc;
        if (e != cudaSuccess) return c->fail(AOS_ERR_CUDA, std::string("graph capture: ") + cudaGetErrorString(e));
        e = cudaGraphInstantiate(&plan->graph, g, 0);
        cudaGraphDestroy(g);
        if (e != cudaSuccess) return c->fail(AOS_ERR_CUDA, std::string("graph instantiate: ") + cudaGetErrorString(e));
        plan->graph_valid = true;
        plan->graph_logits = with_logits ? c->d_logits : nullptr;
    }
    CTX_CUDA(c, cudaGraphLaunch(plan->graph, s));
    return AOS_OK;
}

// Resolve sequences to page tables and positions for a step (host side).
int stage_sequences(aos_ctx* c, const uint64_t* seq_ids, uint32_t T) {
    if (T > (uint32_t)c->cfg.max_batch) return c->fail(AOS_ERR_INVALID, "T exceeds max_batch");
    c->stage_slot = (c->stage_slot + 1) % aos_ctx::kStageSlots;
    CTX_CUDA(c, cudaEventSynchronize(c->stage_ev[c->stage_slot]));  // its previous copy has been read
    c->h_block_tables = c->h_stage[c->stage_slot];
    c->h_ctx_lens = c->h_block_tables + (size_t)c->T_cap * c->max_blocks;
    for (uint32_t t = 0; t < T; ++t) {
        auto it = c->seqs.find(seq_ids[t]);
        if (it == c->seqs.end()) return c->fail(AOS_ERR_NOT_FOUND, "unknown sequence id " + std::to_string(seq_ids[t]));
        Sequence& sq = it->second;
        if (sq.len >= sq.cap) return c->fail(AOS_ERR_NOMEM, "sequence " + std::to_string(seq_ids[t]) + " is full");
        for (uint32_t u = 0; u < t; ++u)
            if (seq_ids[u] == seq_ids[t]) return c->fail(AOS_ERR_INVALID, "a sequence appears twice in one step");
        int* row = c->h_block_tables + (size_t)t * c->max_blocks;
        std::fill(row, row + c->max_blocks, 0);
        std::copy(sq.blocks.begin(), sq.blocks.end(), row);
        c->h_ctx_lens[t] = (int)sq.len;
    }
    return AOS_OK;
}

int upload_tables(aos_ctx* c, uint32_t T, cudaStream_t s) {
    CTX_CUDA(c, cudaMemcpyAsync(c->d_block_tables, c->h_block_tables, (size_t)T * c->max_blocks * 4,
                                cudaMemcpyHostToDevice, s));
    CTX_CUDA(c, cudaMemcpyAsync(c->d_ctx_lens, c->h_ctx_lens, (size_t)T * 4, cudaMemcpyHostToDevice, s));
    CTX_CUDA(c, cudaEventRecord(c->stage_ev[c->stage_slot], s));
    return AOS_OK;
}

void advance(aos_ctx* c, const uint64_t* seq_ids, uint32_t T) {
    for (uint32_t t = 0; t < T; ++t) c->seqs[seq_ids[t]].len += 1;
    c->m.steps += 1;
    c->m.tokens += T;
}

// Copies a rows x cols row-major bf16 matrix (leading dimension ld, host or
// device memory; nullptr writes zeros) into the packed block layout of dst
// (dst_cols columns, blocks of br rows x 64 columns, SWIZZLE_128B images) at
// row0/col0, on the context stream.  Host or unaligned sources go through a
// staging buffer of at most kMaxStage bytes, a slab of rows at a time.
int pack_upload(aos_ctx* c, const uint16_t* src, int src_on_device, int rows, int cols, long long ld, uint16_t* dst,
                int row0, int col0, int dst_cols, int br) {
    constexpr size_t kMaxStage = 64u << 20;
    cudaStream_t s = c->stream;
    if (!src || (src_on_device && (reinterpret_cast<uintptr_t>(src) & 15) == 0 && ld % 8 == 0)) {
        LAUNCH(c, launch_pack_blocks(src, rows, cols, ld, dst, row0, col0, dst_cols, br, s));
        return AOS_OK;
    }
    const size_t row_bytes = (size_t)cols * 2;
    const int slab = (int)std::max<size_t>(1, std::min<size_t>((size_t)rows, kMaxStage / row_bytes));
    const size_t need = (size_t)slab * row_bytes;
    if (need > c->stage_bytes) {
        CTX_CUDA(c, cudaStreamSynchronize(s));
        if (c->d_stage) cudaFree(c->d_stage);
        c->d_stage = nullptr;
        c->stage_bytes = 0;
        CTX_CUDA(c, cudaMalloc((void**)&c->d_stage, need));
        c->stage_bytes = need;
    }
    for (int r = 0; r < rows; r += slab) {
        const int nr = std::min(slab, rows - r);
        CTX_CUDA(c, cudaMemcpy2DAsync(c->d_stage, row_bytes, src + (size_t)r * ld, (size_t)ld * 2, row_bytes, nr,
                                      src_on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice, s));
        LAUNCH(c, launch_pack_blocks(c->d_stage, nr, cols, cols, dst, row0 + r, col0, dst_cols, br, s));
    }
    return AOS_OK;
}

int check_device_error(aos_ctx* c) {
    int e = 0;
    CTX_CUDA(c, cudaMemcpy(&e, c->d_err, 4, cudaMemcpyDeviceToHost));
    if (e) {
        // The failed launch may have left tile counters and the shrink
        // counter part-way: clear them so the next step starts clean.
        cudaDeviceSynchronize();  // nothing of this context may still be running
        cudaMemset(c->d_sync, 0, 4 * sizeof(int));
        cudaMemset(c->d_attn_cnt, 0, (size_t)c->T_cap * c->cfg.n_kv_heads * sizeof(int));
        cudaMemset(c->d_ss, 0, (size_t)c->T_cap * sizeof(unsigned long long));
        cudaMemset(c->d_acc, 0, c->acc_bytes);
        cudaMemset(c->d_err, 0, sizeof(int));
        cudaDeviceSynchronize();
        return c->fail(e, "a bounded device-side wait timed out or a launch limit was exceeded (the kernel returned early)");
    }
    return AOS_OK;
}

// ------------------------------------------------------------------ prefill
int prefill_reserve(aos_ctx* c, int T) {
    auto& b = c->pf;
    if (T <= b.cap) return AOS_OK;
    CTX_CUDA(c, cudaDeviceSynchronize());  // earlier prefills on any stream may still read the old buffers
    auto f = [](void* p) {
        if (p) cudaFree(p);
    };
    f(b.hidden); f(b.normed); f(b.q); f(b.attn); f(b.act); f(b.coef); f(b.ucoef);
    f(b.rings); f(b.tokens); f(b.pos); f(b.block_tables); f(b.qblk);
    for (int m = 0; m < AOS_NUM_MODULES; ++m) f(b.hm[m]);
    b = aos_ctx::Prefill{};
    // whole 256-token tiles of the prefill GEMM
    const size_t Tc = (size_t)((T + 255) / 256) * 256, H = c->cfg.hidden, I = c->cfg.intermediate;
    const size_t NA = std::max(1u, c->cfg.lora_max_adapters);
    CTX_CUDA(c, dalloc(&b.hidden, Tc * H));
    CTX_CUDA(c, dalloc(&b.normed, Tc * H));
    CTX_CUDA(c, dalloc(&b.q, Tc * c->QD));
    CTX_CUDA(c, dalloc(&b.attn, Tc * c->QD));
    CTX_CUDA(c, dalloc(&b.act, Tc * I));
    for (int m = 0; m < AOS_NUM_MODULES; ++m)
        if (c->module_mask & (1u << m)) CTX_CUDA(c, dalloc(&b.hm[m], Tc * c->R));
    CTX_CUDA(c, dalloc(&b.coef, Tc * NA));
    CTX_CUDA(c, dalloc(&b.ucoef, Tc * (size_t)(c->R / kGroup) * 8));
    CTX_CUDA(c, dalloc(&b.rings, Tc));
    CTX_CUDA(c, dalloc(&b.tokens, Tc));
    CTX_CUDA(c, dalloc(&b.pos, Tc));
    CTX_CUDA(c, dalloc(&b.block_tables, Tc * c->max_blocks));
    CTX_CUDA(c, dalloc(&b.qblk, Tc + 1));
    b.cap = (int)Tc;
    return AOS_OK;
}

// TcParams of one prefill GEMM launch of group g (shrink: the LoRA modules
// that read the group's input; else the base projection + expand + epilogue).
int prefill_gemm_params(aos_ctx* c, int layer, int g, int T, bool shrink, TcParams& p) {
    const uint32_t H = c->cfg.hidden, I = c->cfg.intermediate;
    auto& b = c->pf;
    const int mods[4][3] = {{AOS_MOD_Q, AOS_MOD_K, AOS_MOD_V}, {AOS_MOD_O, -1, -1}, {AOS_MOD_GATE, AOS_MOD_UP, -1},
                            {AOS_MOD_DOWN, -1, -1}};
    const uint16_t* xs[4] = {b.normed, b.attn, b.normed, b.act};
    const uint32_t K[4] = {H, c->QD, H, I};
    const bool lora = (c->module_mask & (1u << mods[g][0])) != 0;
    std::memset(&p, 0, sizeof(p));
    p.T = T;
    p.groups = c->d_groups;
    p.n_groups = c->d_n_groups;
    p.err = c->d_err;
    p.R = c->R;
    p.n_rgroups = c->R / kGroup;
    p.ucoef = b.ucoef;
    p.layer = layer;
    p.kb = (int)(K[g] / 64);
    p.n_sub = 1;
    int rc = tc_encode_2d(&p.tm_x, xs[g], K[g], (uint64_t)b.cap, (uint64_t)K[g] * 2, 64, kTcTok, 128);
    if (rc) return rc;
    auto h_map = [&](CUtensorMap* m, int mod) {
        return tc_encode_2d(m, b.hm[mod], (uint64_t)c->R, (uint64_t)b.cap, (uint64_t)c->R * 2, kGroup, kTcTok, 128);
    };
    if (shrink) {
        for (int j = 0; j < 3; ++j) {
            const int mod = mods[g][j];
            if (mod < 0) continue;
            p.a_pk[p.sh_nseg] = c->A[mod][layer];
            p.sh_out[p.sh_nseg] = b.hm[mod];
            ++p.sh_nseg;
        }
        p.mode = TC_SHRINK_HM;
        return pf_prepare(p);
    }
    p.lora = lora ? 1 : 0;
    if (g == kGroupQKV) {
        p.mode = TC_QKV_ROPE;
        p.n_seg = 3;
        const uint32_t r0[3] = {0, c->QD, c->QD + c->KVD}, nr[3] = {c->QD, c->KVD, c->KVD};
        for (int j = 0; j < 3; ++j) {
            p.w_pk[j] = c->w_qkv[layer];
            p.seg_wrow0[j] = (int)r0[j];
            p.seg_tiles[j] = (int)((nr[j] + kTcBN - 1) / kTcBN);
            p.seg_rows[j] = (int)nr[j];
            p.seg_module[j] = mods[g][j];
            if (lora) {
                p.b_pk[j] = c->B[mods[g][j]][layer];
                if ((rc = h_map(&p.tm_lh[j], mods[g][j]))) return rc;
            }
        }
        p.out[0] = p.out[1] = p.out[2] = b.q;
        p.ld_out = (int)c->QD;
        p.rope = c->d_rope;
        p.k_pool = c->k_pool;
        p.v_pool = c->v_pool;
        p.block_tables = b.block_tables;
        p.ctx_lens = b.pos;
        p.max_blocks = c->max_blocks;
        p.num_blocks = (int)c->cfg.kv_num_blocks;
        p.nkv = (int)c->cfg.n_kv_heads;
    } else if (g == kGroupGU) {
        p.mode = TC_SWIGLU;
        p.n_sub = 2;
        p.n_seg = 1;
        p.w_pk[0] = c->w_gate[layer];
        p.w_pk[1] = c->w_up[layer];
        if (lora) {
            p.b_pk[0] = c->B[AOS_MOD_GATE][layer];
            p.b_pk[1] = c->B[AOS_MOD_UP][layer];
            if ((rc = h_map(&p.tm_lh[0], AOS_MOD_GATE)) || (rc = h_map(&p.tm_lh[1], AOS_MOD_UP))) return rc;
        }
        p.seg_tiles[0] = (int)((I + kTcBN / 2 - 1) / (kTcBN / 2));
        p.seg_rows[0] = (int)I;
        p.seg_module[0] = AOS_MOD_GATE;
        p.out[0] = b.act;
        p.ld_out = (int)I;
    } else {
        const int mod = mods[g][0];
        p.mode = TC_RESID_BF16;
        p.n_seg = 1;
        p.w_pk[0] = g == kGroupO ? c->w_o[layer] : c->w_down[layer];
        if (lora) {
            p.b_pk[0] = c->B[mod][layer];
            if ((rc = h_map(&p.tm_lh[0], mod))) return rc;
        }
        p.seg_tiles[0] = (int)((H + kTcBN - 1) / kTcBN);
        p.seg_rows[0] = (int)H;
        p.seg_module[0] = mod;
        p.resid = b.hidden;
        p.ld_out = (int)H;
    }
    return pf_prepare(p);
}

// One prefill layer: per input group, the LoRA shrink launch then the base +
// expand launch (data-parallel prefill GEMM), with causal attention between.
int enqueue_prefill_layer(aos_ctx* c, int layer, int T, int n_qblk, const CUtensorMap* tm_q, cudaStream_t s) {
    auto& b = c->pf;
    const uint32_t H = c->cfg.hidden;
    const int gmod[4] = {AOS_MOD_Q, AOS_MOD_O, AOS_MOD_GATE, AOS_MOD_DOWN};
    auto gemm = [&](int g) -> int {
        TcParams p;
        int rc;
        if (c->module_mask & (1u << gmod[g])) {
            if ((rc = prefill_gemm_params(c, layer, g, T, true, p))) return c->fail(rc, "prefill shrink plan");
            PLAUNCH(c, AOS_K_SHRINK, s, pf_launch(p, s));
        }
        if ((rc = prefill_gemm_params(c, layer, g, T, false, p))) return c->fail(rc, "prefill GEMM plan");
        PLAUNCH(c, AOS_K_GEMM, s, pf_launch(p, s));
        return AOS_OK;
    };
    int rc;
    PLAUNCH(c, AOS_K_NORM, s, launch_rmsnorm(b.hidden, c->attn_norm[layer], T, (int)H, c->cfg.rms_eps, b.normed, s));
    if ((rc = gemm(kGroupQKV))) return rc;
    if (tm_q)  // tensor-core kernel: query blocks of 128 / G tokens
        PLAUNCH(c, AOS_K_ATTN, s,
                launch_attention_prefill_tc(*tm_q, c->tm_k, c->tm_v, b.block_tables, b.pos, b.qblk, n_qblk,
                                            (int)c->cfg.n_heads, (int)c->cfg.n_kv_heads, layer,
                                            (int)c->cfg.kv_num_blocks, c->max_blocks, c->d_err, b.attn, s));
    else  // GQA groups that do not divide 128 rows: query blocks of 16 tokens on mma.sync
        PLAUNCH(c, AOS_K_ATTN, s,
                launch_attention_prefill(c->tm_k, c->tm_v, b.q, b.block_tables, b.pos, b.qblk, n_qblk,
                                         (int)c->cfg.n_heads, (int)c->cfg.n_kv_heads, layer,
                                         (int)c->cfg.kv_num_blocks, c->max_blocks, c->d_err, b.attn, s));
    if ((rc = gemm(kGroupO))) return rc;
    PLAUNCH(c, AOS_K_NORM, s, launch_rmsnorm(b.hidden, c->mlp_norm[layer], T, (int)H, c->cfg.rms_eps, b.normed, s));
    if ((rc = gemm(kGroupGU))) return rc;
    return gemm(kGroupD);
}

}  // namespace

// Model dimensions and the context's error channel, for the loaders in
// safetensors.cu.
namespace aos {
int ctx_model_dims(const aos_ctx* c, uint32_t* n_layers, uint32_t* in_dims, uint32_t* out_dims, uint32_t* hidden,
                   uint32_t* vocab) {
    *n_layers = c->cfg.n_layers;
    for (int m = 0; m < AOS_NUM_MODULES; ++m) {
        in_dims[m] = mod_in(c, m);
        out_dims[m] = mod_out(c, m);
    }
    *hidden = c->cfg.hidden;
    *vocab = c->cfg.vocab;
    return AOS_OK;
}
int ctx_fail(aos_ctx* c, int code, const std::string& msg) { return c->fail(code, msg); }
cudaStream_t ctx_stream(aos_ctx* c) { return c->stream; }
int ctx_set_device(aos_ctx* c) {
    CTX_CUDA(c, cudaSetDevice(c->device));
    return AOS_OK;
}
}  // namespace aos

// ============================================================================ C ABI
extern "C" {

const char* aos_last_error(const aos_ctx* ctx) { return ctx ? ctx->err.c_str() : global_error(); }

aos_ctx* aos_init(const aos_model_config* cfg) {
    if (!cfg) {
        set_global_error("aos_init: cfg is NULL");
        return nullptr;
    }
    const aos_model_config& k = *cfg;
    if (k.head_dim != 128 || k.n_heads == 0 || k.n_kv_heads == 0 || k.n_heads % k.n_kv_heads ||
        k.n_heads / k.n_kv_heads > 16 || k.hidden % 128 || k.intermediate % 128 || k.n_layers == 0 ||
        k.kv_block_size != 16 || k.max_batch == 0 || k.max_batch > 256 || k.vocab == 0 || k.kv_num_blocks == 0 ||
        k.max_seq_len == 0 || k.lora_max_adapters > 65535) {
        set_global_error("aos_init: unsupported config (head_dim 128, hidden/intermediate % 128, KV block 16, "
                         "max_batch <= 256, rank capacity % 16, GQA group <= 16)");
        return nullptr;
    }
    if (require_device(k.device)) return nullptr;
    if (cudaSetDevice(k.device) != cudaSuccess) {
        set_global_error("aos_init: cudaSetDevice failed");
        return nullptr;
    }
    auto c = std::make_unique<aos_ctx>();
    c->cfg = k;
    c->device = k.device;
    c->QD = k.n_heads * k.head_dim;
    c->KVD = k.n_kv_heads * k.head_dim;
    c->G = k.n_heads / k.n_kv_heads;
    uint32_t mask = k.lora_module_mask ? k.lora_module_mask : 0x7Fu;
    // a fused GEMM group shares one LoRA flag
    if (mask & 0x7u) mask |= 0x7u;
    if (mask & 0x30u) mask |= 0x30u;
    if (k.lora_rank_capacity == 0 || k.lora_max_adapters == 0) mask = 0;
    c->module_mask = mask;
    c->R = mask ? (int)((k.lora_rank_capacity + kGroup - 1) / kGroup) * kGroup : kGroup;
    c->T_cap = std::max(32, (int)((k.max_batch + 15) / 16) * 16);
    c->max_blocks = (int)((k.max_seq_len + 15) / 16);
    cudaDeviceProp prop;
    cudaGetDeviceProperties(&prop, k.device);
    c->dev_name = prop.name;
    auto fail_init = [&](const char* what, cudaError_t e) -> aos_ctx* {
        set_global_error(std::string("aos_init: ") + what + ": " + cudaGetErrorString(e));
        return nullptr;
    };
    cudaError_t e;
#define INIT_CHECK(expr, what)                 \
    if ((e = (expr)) != cudaSuccess) return fail_init(what, e);
    INIT_CHECK(cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking), "stream");
    const uint32_t L = k.n_layers, H = k.hidden, I = k.intermediate, V = k.vocab;
    // base weights
    INIT_CHECK(dalloc(&c->embed, (size_t)V * H, &c->base_bytes), "embed");
    // packed in 128-row blocks: rows padded to a multiple of 128 (zeros)
    INIT_CHECK(dalloc(&c->lm_head, (size_t)((V + 127) / 128 * 128) * H, &c->base_bytes), "lm_head");
    INIT_CHECK(dalloc(&c->final_norm, (size_t)H, &c->base_bytes), "final_norm");
    c->attn_norm.resize(L);
    c->mlp_norm.resize(L);
    c->w_qkv.resize(L);
    c->w_o.resize(L);
    c->w_gate.resize(L);
    c->w_up.resize(L);
    c->w_down.resize(L);
    for (uint32_t l = 0; l < L; ++l) {
        INIT_CHECK(dalloc(&c->attn_norm[l], H, &c->base_bytes), "norm");
        INIT_CHECK(dalloc(&c->mlp_norm[l], H, &c->base_bytes), "norm");
        INIT_CHECK(dalloc(&c->w_qkv[l], (size_t)(c->QD + 2 * c->KVD) * H, &c->base_bytes), "w_qkv");
        INIT_CHECK(dalloc(&c->w_o[l], (size_t)H * c->QD, &c->base_bytes), "w_o");
        INIT_CHECK(dalloc(&c->w_gate[l], (size_t)I * H, &c->base_bytes), "w_gate");
        INIT_CHECK(dalloc(&c->w_up[l], (size_t)I * H, &c->base_bytes), "w_up");
        INIT_CHECK(dalloc(&c->w_down[l], (size_t)H * I, &c->base_bytes), "w_down");
    }
    // arena
    for (int m = 0; m < AOS_NUM_MODULES; ++m) {
        c->A[m].assign(L, nullptr);
        c->B[m].assign(L, nullptr);
        if (!(mask & (1u << m))) continue;
        for (uint32_t l = 0; l < L; ++l) {
            INIT_CHECK(dalloc(&c->A[m][l], (size_t)c->R * mod_in(c.get(), m), &c->arena_bytes), "arena A");
            INIT_CHECK(dalloc(&c->B[m][l], (size_t)c->R * mod_out(c.get(), m), &c->arena_bytes), "arena B");
        }
    }
    INIT_CHECK(dalloc(&c->d_col_owner, (size_t)c->R), "col_owner");
    INIT_CHECK(cudaMemset(c->d_col_owner, 0xFF, (size_t)c->R * 4), "col_owner");
    const uint32_t NA = std::max(1u, k.lora_max_adapters);
    INIT_CHECK(dalloc(&c->d_col_off, NA), "col_off");
    INIT_CHECK(cudaMemset(c->d_col_off, 0xFF, (size_t)NA * 4), "col_off");
    INIT_CHECK(dalloc(&c->d_rank, NA), "rank");
    INIT_CHECK(dalloc(&c->d_scale, NA), "scale");
    c->col_owner.assign(c->R / 8, -1);
    // KV cache
    const size_t kv_elems = (size_t)L * k.kv_num_blocks * k.n_kv_heads * 16 * 128;
    INIT_CHECK(dalloc(&c->k_pool, kv_elems), "k_pool");
    INIT_CHECK(dalloc(&c->v_pool, kv_elems), "v_pool");
    for (int b = (int)k.kv_num_blocks - 1; b >= 0; --b) c->free_blocks.push_back(b);
    const uint64_t kv_rows = (uint64_t)L * k.kv_num_blocks * k.n_kv_heads * 16;
    if (tc_encode_2d(&c->tm_k, c->k_pool, 128, kv_rows, 256, 64, 16, 128) ||
        tc_encode_2d(&c->tm_v, c->v_pool, 128, kv_rows, 256, 64, 16, 128)) {
        set_global_error("aos_init: KV tensor map encode failed");
        return nullptr;
    }
    // scratch
    const size_t TC = (size_t)c->T_cap;
    INIT_CHECK(dalloc(&c->d_hidden, TC * H), "hidden");
    INIT_CHECK(dalloc(&c->d_normed, TC * H), "normed");
    INIT_CHECK(dalloc(&c->d_q, TC * c->QD), "q");
    INIT_CHECK(dalloc(&c->d_attn, TC * c->QD), "attn");
    INIT_CHECK(dalloc(&c->d_act, TC * I), "act");
    for (int m = 0; m < AOS_NUM_MODULES; ++m) INIT_CHECK(dalloc(&c->d_hm[m], TC * c->R), "hm");
    INIT_CHECK(dalloc(&c->d_groups, (size_t)c->R / kGroup + 1), "groups");
    INIT_CHECK(dalloc(&c->d_n_groups, 1), "n_groups");
    INIT_CHECK(dalloc(&c->d_block_tables, TC * c->max_blocks), "block tables");
    INIT_CHECK(dalloc(&c->d_zero_blocks, (size_t)c->cfg.kv_num_blocks), "zeroization block list");
    INIT_CHECK(dalloc(&c->d_ctx_lens, TC), "ctx lens");
    for (int i = 0; i < aos_ctx::kStageSlots; ++i) {
        INIT_CHECK(cudaMallocHost((void**)&c->h_stage[i], (TC * c->max_blocks + TC) * 4), "pinned tables");
        INIT_CHECK(cudaEventCreateWithFlags(&c->stage_ev[i], cudaEventDisableTiming), "staging event");
    }
    c->h_block_tables = c->h_stage[0];
    c->h_ctx_lens = c->h_block_tables + TC * c->max_blocks;
    INIT_CHECK(dalloc(&c->d_rings, TC), "rings");
    INIT_CHECK(dalloc(&c->d_tokens, TC), "tokens");
    INIT_CHECK(dalloc(&c->d_logits, TC * V), "logits");
    INIT_CHECK(dalloc(&c->d_coef, TC * NA), "lora coef");
    INIT_CHECK(dalloc(&c->d_ucoef, TC * (size_t)(c->R / kGroup) * 8), "lora unit coef");
    c->attn_chunks = attn_max_chunks((int)k.max_seq_len);
    INIT_CHECK(dalloc(&c->d_attn_part, TC * k.n_kv_heads * c->attn_chunks * c->G * 128), "attn part");
    INIT_CHECK(dalloc(&c->d_attn_ml, TC * k.n_kv_heads * c->attn_chunks * c->G * 2), "attn ml");
    INIT_CHECK(dalloc(&c->d_attn_cnt, TC * k.n_kv_heads), "attn chunk counts");
    INIT_CHECK(dalloc(&c->d_ss, TC), "norm sums");
    {  // tiles of the largest launch: base tiles plus up to three shrink segments
        const size_t tiles = max_launch_tiles(c.get());
        c->acc_bytes = tiles * kTcBN * (size_t)c->T_cap * sizeof(long long);
        INIT_CHECK(dalloc(&c->d_acc, c->acc_bytes / sizeof(long long)), "GEMM accumulators");
        // one slot per (CTA, base tile) pair that can hold a piece
        INIT_CHECK(dalloc(&c->d_part, (tc_num_sms() + tiles) * kTcBN * (size_t)c->T_cap), "GEMM partials");
        INIT_CHECK(dalloc(&c->d_sync, 4), "sync");
    }
    INIT_CHECK(dalloc(&c->d_err, 1), "err");
    if (getenv("AOS_TC_TRACE")) INIT_CHECK(dalloc(&c->d_trace, (size_t)tc_num_sms() * kTraceStride), "trace");
    if (const char* e = getenv("AOS_GEMM_COOPERATIVE")) c->gemm_coop = atoi(e) != 0 ? 1 : 0;
    // RoPE table, angles as the reference computes them (mlx_cpp_wrapper_real.cpp:3249-3268)
    {
        const uint32_t half = 64, P = k.max_seq_len + 1;
        std::vector<float> inv(half), tab((size_t)P * half * 2);
        for (uint32_t i = 0; i < half; ++i) {
            const float ex = k.rope_mlx_as_written ? (-2.0f * (float)i / 128.0f) : (2.0f * (float)i / 128.0f);
            inv[i] = 1.0f / std::pow(k.rope_theta, ex);
        }
        for (uint32_t p = 0; p < P; ++p)
            for (uint32_t i = 0; i < half; ++i) {
                const float ang = (float)p * inv[i];
                tab[((size_t)p * half + i) * 2] = std::cos(ang);
                tab[((size_t)p * half + i) * 2 + 1] = std::sin(ang);
            }
        INIT_CHECK(cudaMalloc((void**)&c->d_rope, tab.size() * 4), "rope");
        INIT_CHECK(cudaMemcpy(c->d_rope, tab.data(), tab.size() * 4, cudaMemcpyHostToDevice), "rope");
    }
    INIT_CHECK(tc_configure(), "GEMM smem attribute");
    INIT_CHECK(attn_configure(), "attention smem attribute");
    INIT_CHECK(attn_tc_configure(), "tensor-core prefill attention smem attribute");
    INIT_CHECK(cudaEventCreate(&c->ev0), "event");
    INIT_CHECK(cudaEventCreate(&c->ev1), "event");
    INIT_CHECK(cudaDeviceSynchronize(), "init sync");
#undef INIT_CHECK
    c->m.base_weight_bytes = c->base_bytes;
    c->m.arena_bytes = c->arena_bytes;
    c->m.kv_pool_bytes = kv_elems * 4;
    c->m.kv_blocks_total = k.kv_num_blocks;
    return c.release();
}

void aos_destroy(aos_ctx* c) {
    if (!c) return;
    cudaSetDevice(c->device);
    cudaStreamSynchronize(c->stream);
    for (auto& kv : c->plans)
        if (kv.second->graph) cudaGraphExecDestroy(kv.second->graph);
    if (c->nccl) ncclCommDestroy(c->nccl);  // after the graphs that hold its calls
    auto f = [](void* p) {
        if (p) cudaFree(p);
    };
    f(c->d_xrecv); f(c->d_dsend); f(c->d_drecv); f(c->d_rings_all);
    f(c->pf.hidden); f(c->pf.normed); f(c->pf.q); f(c->pf.attn); f(c->pf.act); f(c->pf.coef); f(c->pf.ucoef);
    f(c->pf.rings); f(c->pf.tokens); f(c->pf.pos); f(c->pf.block_tables); f(c->pf.qblk);
    for (int m = 0; m < AOS_NUM_MODULES; ++m) f(c->pf.hm[m]);
    f(c->embed); f(c->lm_head); f(c->final_norm);
    for (auto* p : c->attn_norm) f(p);
    for (auto* p : c->mlp_norm) f(p);
    for (auto* p : c->w_qkv) f(p);
    for (auto* p : c->w_o) f(p);
    for (auto* p : c->w_gate) f(p);
    for (auto* p : c->w_up) f(p);
    for (auto* p : c->w_down) f(p);
    for (int m = 0; m < AOS_NUM_MODULES; ++m) {
        for (auto* p : c->A[m]) f(p);
        for (auto* p : c->B[m]) f(p);
        f(c->d_hm[m]);
    }
    f(c->d_col_owner); f(c->d_col_off); f(c->d_rank); f(c->d_scale); f(c->d_coef); f(c->d_ucoef);
    f(c->k_pool); f(c->v_pool);
    f(c->d_hidden); f(c->d_normed); f(c->d_q); f(c->d_attn); f(c->d_act);
    f(c->d_groups); f(c->d_n_groups); f(c->d_block_tables); f(c->d_ctx_lens); f(c->d_zero_blocks);
    f(c->d_rings); f(c->d_tokens); f(c->d_logits); f(c->d_rope);
    f(c->d_attn_part); f(c->d_attn_ml); f(c->d_attn_cnt); f(c->d_ss); f(c->d_stage); f(c->d_acc); f(c->d_part); f(c->d_fp); f(c->d_sync); f(c->d_err); f(c->d_trace);
    for (int i = 0; i < aos_ctx::kStageSlots; ++i) {
        if (c->h_stage[i]) cudaFreeHost(c->h_stage[i]);
        if (c->stage_ev[i]) cudaEventDestroy(c->stage_ev[i]);
    }
    if (c->ev0) cudaEventDestroy(c->ev0);
    if (c->ev1) cudaEventDestroy(c->ev1);
    for (auto e : c->prof_ev) cudaEventDestroy(e);
    if (c->stream) cudaStreamDestroy(c->stream);
    delete c;
}

const char* aos_device_name(const aos_ctx* c) { return c ? c->dev_name.c_str() : ""; }
void* aos_stream(aos_ctx* c) { return c ? (void*)c->stream : nullptr; }

int aos_load_weight(aos_ctx* c, aos_weight_kind kind, uint32_t layer, aos_module module, const uint16_t* data,
                    uint64_t n, int src_on_device) {
    if (!c || !data) return AOS_ERR_INVALID;
    const uint32_t H = c->cfg.hidden, V = c->cfg.vocab;
    uint16_t* dst = nullptr;
    uint64_t want = 0;
    if (kind != AOS_W_EMBED && kind != AOS_W_LM_HEAD && kind != AOS_W_FINAL_NORM && layer >= c->cfg.n_layers)
        return c->fail(AOS_ERR_INVALID, "layer out of range");
    switch (kind) {
        case AOS_W_EMBED: dst = c->embed; want = (uint64_t)V * H; break;
        case AOS_W_LM_HEAD: dst = c->lm_head; want = (uint64_t)V * H; break;
        case AOS_W_FINAL_NORM: dst = c->final_norm; want = H; break;
        case AOS_W_ATTN_NORM: dst = c->attn_norm[layer]; want = H; break;
        case AOS_W_MLP_NORM: dst = c->mlp_norm[layer]; want = H; break;
        case AOS_W_PROJ: {
            if ((int)module < 0 || (int)module >= AOS_NUM_MODULES) return c->fail(AOS_ERR_INVALID, "bad module");
            want = (uint64_t)mod_out(c, module) * mod_in(c, module);
            switch (module) {
                case AOS_MOD_Q: dst = c->w_qkv[layer]; break;
                case AOS_MOD_K: dst = c->w_qkv[layer] + (size_t)c->QD * H; break;
                case AOS_MOD_V: dst = c->w_qkv[layer] + (size_t)(c->QD + c->KVD) * H; break;
                case AOS_MOD_O: dst = c->w_o[layer]; break;
                case AOS_MOD_GATE: dst = c->w_gate[layer]; break;
                case AOS_MOD_UP: dst = c->w_up[layer]; break;
                case AOS_MOD_DOWN: dst = c->w_down[layer]; break;
            }
            break;
        }
        default: return c->fail(AOS_ERR_INVALID, "bad weight kind");
    }
    if (n != want) return c->fail(AOS_ERR_INVALID, "weight size mismatch: got " + std::to_string(n) + ", want " + std::to_string(want));
    CTX_CUDA(c, cudaSetDevice(c->device));
    if (kind == AOS_W_PROJ || kind == AOS_W_LM_HEAD) {
        // projection matrices are stored packed (128 x 64 SWIZZLE_128B blocks)
        int rows, cols, row0 = 0;
        uint16_t* base = dst;
        if (kind == AOS_W_LM_HEAD) {
            rows = (int)V;
            cols = (int)H;
        } else {
            rows = (int)mod_out(c, module);
            cols = (int)mod_in(c, module);
            if (module == AOS_MOD_Q || module == AOS_MOD_K || module == AOS_MOD_V) {
                base = c->w_qkv[layer];
                row0 = module == AOS_MOD_Q ? 0 : (module == AOS_MOD_K ? (int)c->QD : (int)(c->QD + c->KVD));
            }
        }
        int rc = pack_upload(c, data, src_on_device, rows, cols, cols, base, row0, 0, cols, 128);
        if (rc) return rc;
        CTX_CUDA(c, cudaStreamSynchronize(c->stream));
        return AOS_OK;
    }
    CTX_CUDA(c, cudaStreamSynchronize(c->stream));  // no queued step may still read the tensor
    CTX_CUDA(c, cudaMemcpy(dst, data, n * 2, src_on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice));
    return AOS_OK;
}

// ------------------------------------------------------------------ adapters
int aos_adapter_new(aos_ctx* c, uint16_t id, uint32_t rank, float alpha) {
    if (!c) return AOS_ERR_INVALID;
    return aos::ctx_adapter_new(c, id, rank, alpha, alpha / (float)rank);
}

}  // extern "C"

int aos::ctx_adapter_new(aos_ctx* c, uint16_t id, uint32_t rank, float alpha, float scale) {
    if (!c->module_mask) return c->fail(AOS_ERR_STATE, "this context has no LoRA arena");
    if (id >= c->cfg.lora_max_adapters) return c->fail(AOS_ERR_INVALID, "adapter id >= lora_max_adapters");
    if (rank < 8 || rank > 256 || rank % 8) return c->fail(AOS_ERR_INVALID, "rank must be a multiple of 8 in [8, 256]");
    if (!std::isfinite(alpha)) return c->fail(AOS_ERR_INVALID, "alpha must be finite");
    if (c->adapters.count(id)) return c->fail(AOS_ERR_INVALID, "adapter id already loaded");
    // First fit over 8-column units, aligned to the rank's largest power-of-two
    // factor (capped at one 64-column group) so an adapter spans as few rank
    // groups as its size allows.
    const int pow2 = (int)(rank & (~rank + 1u));
    const int units = (int)rank / 8, align = std::min(pow2, kGroup) / 8, n_units = (int)c->col_owner.size();
    int start = -1;
    for (int u = 0; u + units <= n_units; u += align) {
        bool free_run = true;
        for (int j = 0; j < units; ++j)
            if (c->col_owner[u + j] >= 0) { free_run = false; break; }
        if (free_run) { start = u; break; }
    }
    if (start < 0) return c->fail(AOS_ERR_NOMEM, "adapter arena full");
    const int off = start * 8;
    CTX_CUDA(c, cudaSetDevice(c->device));
    // zero the adapter's lora_A rows and lora_B columns in every layer and module
    for (int m = 0; m < AOS_NUM_MODULES; ++m) {
        if (!(c->module_mask & (1u << m))) continue;
        const int in = (int)mod_in(c, m), out = (int)mod_out(c, m);
        for (uint32_t l = 0; l < c->cfg.n_layers; ++l) {
            int rc = pack_upload(c, nullptr, 1, (int)rank, in, in, c->A[m][l], off, 0, in, kGroup);
            if (!rc) rc = pack_upload(c, nullptr, 1, out, (int)rank, (int)rank, c->B[m][l], 0, off, c->R, 128);
            if (rc) return rc;
        }
    }
    CTX_CUDA(c, cudaStreamSynchronize(c->stream));
    for (int j = 0; j < units; ++j) c->col_owner[start + j] = id;
    std::vector<int> owner((size_t)rank, (int)id);
    CTX_CUDA(c, cudaMemcpy(c->d_col_owner + off, owner.data(), rank * 4, cudaMemcpyHostToDevice));
    const int irank = (int)rank;
    CTX_CUDA(c, cudaMemcpy(c->d_col_off + id, &off, 4, cudaMemcpyHostToDevice));
    CTX_CUDA(c, cudaMemcpy(c->d_rank + id, &irank, 4, cudaMemcpyHostToDevice));
    CTX_CUDA(c, cudaMemcpy(c->d_scale + id, &scale, 4, cudaMemcpyHostToDevice));
    c->adapters[id] = AdapterEntry{off, (int)rank, alpha};
    c->m.adapters_loaded = (uint32_t)c->adapters.size();
    c->m.arena_used_rank_cols += rank;
    return AOS_OK;
}

extern "C" {

int aos_adapter_set_module(aos_ctx* c, uint16_t id, uint32_t layer, aos_module module, const uint16_t* A,
                           const uint16_t* B, int src_on_device) {
    if (!c || !A || !B) return AOS_ERR_INVALID;
    auto it = c->adapters.find(id);
    if (it == c->adapters.end()) return c->fail(AOS_ERR_NOT_FOUND, "adapter not loaded");
    if (layer >= c->cfg.n_layers || (int)module < 0 || (int)module >= AOS_NUM_MODULES)
        return c->fail(AOS_ERR_INVALID, "layer or module out of range");
    if (!(c->module_mask & (1u << module))) return c->fail(AOS_ERR_INVALID, "module not enabled for LoRA in this context");
    const int off = it->second.off, rank = it->second.rank;
    const uint32_t in = mod_in(c, module), out = mod_out(c, module);
    CTX_CUDA(c, cudaSetDevice(c->device));
    // lora_A [rank, in] -> arena rows [off, off + rank) (64-row blocks);
    // lora_B [out, rank] -> arena columns [off, off + rank) (128-row blocks)
    int rc = pack_upload(c, A, src_on_device, rank, (int)in, (long long)in, c->A[module][layer], off, 0, (int)in, kGroup);
    if (!rc) rc = pack_upload(c, B, src_on_device, (int)out, rank, rank, c->B[module][layer], 0, off, c->R, 128);
    if (rc) return rc;
    CTX_CUDA(c, cudaStreamSynchronize(c->stream));
    return AOS_OK;
}

int aos_adapter_unload(aos_ctx* c, uint16_t id) {
    if (!c) return AOS_ERR_INVALID;
    auto it = c->adapters.find(id);
    if (it == c->adapters.end()) return c->fail(AOS_ERR_NOT_FOUND, "adapter not loaded");
    const int off = it->second.off, rank = it->second.rank;
    CTX_CUDA(c, cudaSetDevice(c->device));
    CTX_CUDA(c, cudaStreamSynchronize(c->stream));  // no step may still read the columns
    for (int j = 0; j < rank / 8; ++j) c->col_owner[off / 8 + j] = -1;
    CTX_CUDA(c, cudaMemset(c->d_col_owner + off, 0xFF, (size_t)rank * 4));
    const int neg = -1, zero = 0;
    CTX_CUDA(c, cudaMemcpy(c->d_col_off + id, &neg, 4, cudaMemcpyHostToDevice));
    CTX_CUDA(c, cudaMemcpy(c->d_rank + id, &zero, 4, cudaMemcpyHostToDevice));
    c->m.arena_used_rank_cols -= rank;
    c->adapters.erase(it);
    c->m.adapters_loaded = (uint32_t)c->adapters.size();
    return AOS_OK;
}

int aos_adapter_is_loaded(const aos_ctx* c, uint16_t id) { return c && c->adapters.count(id) ? 1 : 0; }

}  // extern "C"

// The adapter's device buffer in canonical form: for every layer and every
// LoRA-enabled module (aos_module order), its lora_A rows [rank][in] and then
// its lora_B columns [out][rank], bf16 row-major, read out of the packed
// arena.  Windows of 4 KB (or the whole buffer when smaller) at its start,
// its end and its middle (start (size - window) / 2, in elements) are
// gathered on the device into c->d_fp [first | last | mid].
static int adapter_samples(aos_ctx* c, uint16_t id, uint64_t* size_bytes, int* n_per) {
    auto it = c->adapters.find(id);
    if (it == c->adapters.end()) return c->fail(AOS_ERR_NOT_FOUND, "adapter not loaded");
    const int off = it->second.off, rank = it->second.rank;
    std::vector<UnpackSeg> segs;
    long long e = 0;
    for (uint32_t l = 0; l < c->cfg.n_layers; ++l)
        for (int m = 0; m < AOS_NUM_MODULES; ++m) {
            if (!(c->module_mask & (1u << m))) continue;
            const int in = (int)mod_in(c, m), out = (int)mod_out(c, m);
            segs.push_back(UnpackSeg{e, c->A[m][l], rank, in, in, kGroup, off, 0});
            e += (long long)rank * in;
            segs.push_back(UnpackSeg{e, c->B[m][l], out, rank, c->R, 128, 0, off});
            e += (long long)out * rank;
        }
    if (segs.empty()) return c->fail(AOS_ERR_STATE, "this context has no LoRA arena");
    const int w = (int)std::min<long long>(2048, e);
    const long long starts[3] = {0, e - w, (e - w) / 2};
    CTX_CUDA(c, cudaSetDevice(c->device));
    cudaStream_t s = c->stream;
    UnpackSeg* d_segs = nullptr;
    long long* d_starts = nullptr;
    CTX_CUDA(c, cudaMallocAsync((void**)&d_segs, segs.size() * sizeof(UnpackSeg), s));
    CTX_CUDA(c, cudaMallocAsync((void**)&d_starts, sizeof starts, s));
    if (!c->d_fp) CTX_CUDA(c, cudaMalloc((void**)&c->d_fp, 3 * 2048 * sizeof(uint16_t)));
    CTX_CUDA(c, cudaMemcpyAsync(d_segs, segs.data(), segs.size() * sizeof(UnpackSeg), cudaMemcpyHostToDevice, s));
    CTX_CUDA(c, cudaMemcpyAsync(d_starts, starts, sizeof starts, cudaMemcpyHostToDevice, s));
    LAUNCH(c, launch_unpack_samples(d_segs, (int)segs.size(), d_starts, w, c->d_fp, s));
    CTX_CUDA(c, cudaFreeAsync(d_segs, s));
    CTX_CUDA(c, cudaFreeAsync(d_starts, s));
    *size_bytes = (uint64_t)e * 2;
    *n_per = w;
    return AOS_OK;
}

static std::string hex_lower(const uint8_t* h, int n) {
    static const char* d = "0123456789abcdef";
    std::string s;
    for (int i = 0; i < n; ++i) {
        s += d[h[i] >> 4];
        s += d[h[i] & 15];
    }
    return s;
}

extern "C" {

int aos_adapter_verify_buffers(aos_ctx* c, uint16_t id, uint64_t* buffer_bytes, void* first, void* last, void* mid,
                               uint32_t* sample_bytes) {
    if (!c || !buffer_bytes) return AOS_ERR_INVALID;
    int n_per = 0, rc = adapter_samples(c, id, buffer_bytes, &n_per);
    if (rc) return rc;
    void* dst[3] = {first, last, mid};
    for (int k = 0; k < 3; ++k)
        if (dst[k])
            CTX_CUDA(c, cudaMemcpyAsync(dst[k], c->d_fp + (size_t)k * n_per, (size_t)n_per * 2, cudaMemcpyDeviceToHost,
                                        c->stream));
    CTX_CUDA(c, cudaStreamSynchronize(c->stream));
    if (sample_bytes) *sample_bytes = (uint32_t)n_per * 2;
    return AOS_OK;
}

int aos_adapter_fingerprint(aos_ctx* c, uint16_t id, uint64_t* buffer_bytes, uint8_t* hash) {
    if (!c || !buffer_bytes || !hash) return AOS_ERR_INVALID;
    int n_per = 0, rc = adapter_samples(c, id, buffer_bytes, &n_per);
    if (rc) return rc;
    const uint64_t off = 0, len = (uint64_t)n_per * 6;  // first || last || mid, contiguous
    std::string err;
    if ((rc = aos::blake3_many(reinterpret_cast<const uint8_t*>(c->d_fp), &off, &len, 1, hash, c->stream, err)))
        return c->fail(rc, err);
    return AOS_OK;
}

int aos_store_gpu_fingerprint(aos_ctx* c, uint16_t id, uint64_t buffer_bytes, const char* checkpoint_hash_hex) {
    if (!c || !checkpoint_hash_hex) return AOS_ERR_INVALID;
    const std::string h = checkpoint_hash_hex;
    if (h.size() != 64 || h.find_first_not_of("0123456789abcdefABCDEF") != std::string::npos)
        return c->fail(AOS_ERR_INVALID, "Invalid checkpoint hash hex: " + h);
    std::string lower = h;
    for (auto& ch : lower) ch = (char)tolower((unsigned char)ch);
    c->fingerprints[id] = {buffer_bytes, lower};
    // VramTracker::store_fingerprint also feeds the footprint baseline (window 10)
    auto& fp = c->footprints[id];
    if (!fp.max_samples) fp.max_samples = 10;
    if (fp.samples.size() >= fp.max_samples) fp.samples.erase(fp.samples.begin());
    fp.samples.push_back(buffer_bytes);
    return AOS_OK;
}

// FusedKernels::check_memory_footprint (VramTracker, kernel-mtl/src/vram.rs:
// 386-407, MemoryFootprintBaseline 82-196): with a baseline, |bytes - mean| /
// stddev <= 2 (population stddev; an exact match when every sample is equal);
// without one, a baseline of window 100 is started with this sample.
int aos_check_memory_footprint(aos_ctx* c, uint16_t id, uint64_t bytes, int* within, double* z_score, double* mean,
                               double* stddev, uint32_t* n_samples) {
    if (!c || !within || !z_score) return AOS_ERR_INVALID;
    auto it = c->footprints.find(id);
    const bool fresh = it == c->footprints.end();
    if (fresh) {
        auto& fp = c->footprints[id];
        fp.max_samples = 100;
        fp.samples.push_back(bytes);
        it = c->footprints.find(id);
    }
    const auto& v = it->second.samples;
    double m = 0.0, sd = 0.0;
    if (!v.empty()) {
        uint64_t sum = 0;
        for (uint64_t x : v) sum += x;
        m = (double)sum / (double)v.size();
    }
    if (v.size() >= 2) {
        double var = 0.0;
        for (uint64_t x : v) {
            const double d = (double)x - m;
            var += d * d;
        }
        sd = std::sqrt(var / (double)v.size());
    }
    if (fresh || v.size() < 2) {
        *within = 1;
        *z_score = 0.0;
    } else if (sd == 0.0) {
        *within = (double)bytes == m;
        *z_score = *within ? 0.0 : DBL_MAX;
    } else {
        *z_score = std::fabs((double)bytes - m) / sd;
        *within = *z_score <= 2.0;
    }
    if (mean) *mean = m;
    if (stddev) *stddev = sd;
    if (n_samples) *n_samples = (uint32_t)v.size();
    return AOS_OK;
}

// FusedKernels::get_gpu_fingerprints: the stored baselines in id order.
int aos_get_gpu_fingerprints(const aos_ctx* c, uint32_t* ids, uint64_t* buffer_bytes, char* hex65, uint32_t max,
                             uint32_t* n) {
    if (!c || !n) return AOS_ERR_INVALID;
    uint32_t k = 0;
    for (const auto& kv : c->fingerprints) {
        if (k < max) {
            if (ids) ids[k] = kv.first;
            if (buffer_bytes) buffer_bytes[k] = kv.second.first;
            if (hex65) std::snprintf(hex65 + 65 * (size_t)k, 65, "%s", kv.second.second.c_str());
        }
        ++k;
    }
    *n = k;
    return AOS_OK;
}

int aos_verify_gpu_fingerprint(aos_ctx* c, uint16_t id, uint64_t buffer_bytes, const char* checkpoint_hash_hex,
                               int* matches) {
    if (!c || !checkpoint_hash_hex || !matches) return AOS_ERR_INVALID;
    auto it = c->fingerprints.find(id);
    *matches = it != c->fingerprints.end() && it->second.first == buffer_bytes &&
               it->second.second == checkpoint_hash_hex;
    return AOS_OK;
}

// ------------------------------------------------------------------ KV cache
int aos_kv_alloc(aos_ctx* c, uint64_t seq_id, uint32_t max_tokens) {
    if (!c) return AOS_ERR_INVALID;
    if (c->seqs.count(seq_id)) return c->fail(AOS_ERR_INVALID, "sequence already allocated");
    if (max_tokens == 0 || max_tokens > c->cfg.max_seq_len) return c->fail(AOS_ERR_INVALID, "max_tokens out of range");
    const size_t need = (max_tokens + 15) / 16;
    if (need > c->free_blocks.size()) return c->fail(AOS_ERR_NOMEM, "KV pool exhausted");
    Sequence s;
    s.cap = max_tokens;
    for (size_t i = 0; i < need; ++i) {
        s.blocks.push_back(c->free_blocks.back());
        c->free_blocks.pop_back();
    }
    c->seqs[seq_id] = std::move(s);
    c->m.sequences = (uint32_t)c->seqs.size();
    c->m.kv_blocks_used = c->cfg.kv_num_blocks - (uint32_t)c->free_blocks.size();
    return AOS_OK;
}

int aos_kv_free(aos_ctx* c, uint64_t seq_id) {
    if (!c) return AOS_ERR_INVALID;
    auto it = c->seqs.find(seq_id);
    if (it == c->seqs.end()) return c->fail(AOS_ERR_NOT_FOUND, "unknown sequence");
    for (int b : it->second.blocks) c->free_blocks.push_back(b);
    c->seqs.erase(it);
    c->kv_guards.erase(seq_id);
    c->m.sequences = (uint32_t)c->seqs.size();
    c->m.kv_blocks_used = c->cfg.kv_num_blocks - (uint32_t)c->free_blocks.size();
    return AOS_OK;
}

int aos_kv_set_len(aos_ctx* c, uint64_t seq_id, uint32_t len) {
    if (!c) return AOS_ERR_INVALID;
    auto it = c->seqs.find(seq_id);
    if (it == c->seqs.end()) return c->fail(AOS_ERR_NOT_FOUND, "unknown sequence");
    if (len > it->second.cap) return c->fail(AOS_ERR_INVALID, "len beyond the sequence's capacity");
    it->second.len = len;
    return AOS_OK;
}

int aos_kv_get_len(const aos_ctx* c, uint64_t seq_id, uint32_t* len) {
    if (!c || !len) return AOS_ERR_INVALID;
    auto it = c->seqs.find(seq_id);
    if (it == c->seqs.end()) return AOS_ERR_NOT_FOUND;
    *len = it->second.len;
    return AOS_OK;
}

static int kv_copy(aos_ctx* c, uint64_t seq_id, uint32_t layer, uint32_t pos0, uint32_t n, const uint16_t* k_src,
                   const uint16_t* v_src, uint16_t* k_dst, uint16_t* v_dst, int src_on_device) {
    auto it = c->seqs.find(seq_id);
    if (it == c->seqs.end()) return c->fail(AOS_ERR_NOT_FOUND, "unknown sequence");
    if (layer >= c->cfg.n_layers || pos0 + n > it->second.cap) return c->fail(AOS_ERR_INVALID, "KV range out of bounds");
    const uint32_t nkv = c->cfg.n_kv_heads;
    const bool write = k_src != nullptr;
    CTX_CUDA(c, cudaSetDevice(c->device));
    // Runs of positions inside one page: per head the page rows are contiguous
    // (256 B each), the caller's rows are strided by n_kv_heads * 256 B.
    for (uint32_t i = 0; i < n;) {
        const uint32_t pos = pos0 + i;
        const uint32_t run = std::min(n - i, 16 - pos % 16);
        const int blk = it->second.blocks[pos / 16];
        for (uint32_t h = 0; h < nkv; ++h) {
            const size_t idx = ((((size_t)layer * c->cfg.kv_num_blocks + blk) * nkv + h) * 16 + pos % 16) * 128;
            const size_t src = ((size_t)i * nkv + h) * 128;
            const size_t pitch = (size_t)nkv * 256;
            if (write) {
                const cudaMemcpyKind kd = src_on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice;
                CTX_CUDA(c, cudaMemcpy2D(c->k_pool + idx, 256, k_src + src, pitch, 256, run, kd));
                CTX_CUDA(c, cudaMemcpy2D(c->v_pool + idx, 256, v_src + src, pitch, 256, run, kd));
            } else {
                CTX_CUDA(c, cudaMemcpy2D(k_dst + src, pitch, c->k_pool + idx, 256, 256, run, cudaMemcpyDeviceToHost));
                CTX_CUDA(c, cudaMemcpy2D(v_dst + src, pitch, c->v_pool + idx, 256, 256, run, cudaMemcpyDeviceToHost));
            }
        }
        i += run;
    }
    return AOS_OK;
}

int aos_kv_write(aos_ctx* c, uint64_t seq_id, uint32_t layer, uint32_t pos0, uint32_t n, const uint16_t* k,
                 const uint16_t* v, int src_on_device) {
    if (!c || !k || !v) return AOS_ERR_INVALID;
    return kv_copy(c, seq_id, layer, pos0, n, k, v, nullptr, nullptr, src_on_device);
}

int aos_kv_read(aos_ctx* c, uint64_t seq_id, uint32_t layer, uint32_t pos0, uint32_t n, uint16_t* k, uint16_t* v) {
    if (!c || !k || !v) return AOS_ERR_INVALID;
    CTX_CUDA(c, cudaStreamSynchronize(c->stream));
    return kv_copy(c, seq_id, layer, pos0, n, nullptr, nullptr, k, v, 0);
}

// Sliding-window rotate (kv_cache.metal:200-236, kv_cache_rotate): drop the
// sequence's oldest `shift` positions; position i takes the K/V rows of
// position i + shift in every layer and KV head, and the length becomes
// len - shift.  On the paged pool the whole pages of the shift are a
// rotation of the sequence's page list (the dropped pages move to its end
// and keep serving its capacity); only the remainder shift % 16 moves rows,
// in place, page by page.  The reference's Rust code never dispatches that
// shader; this is its semantics on this cache.
int aos_kv_rotate(aos_ctx* c, uint64_t seq_id, uint32_t shift) {
    if (!c) return AOS_ERR_INVALID;
    auto it = c->seqs.find(seq_id);
    if (it == c->seqs.end()) return c->fail(AOS_ERR_NOT_FOUND, "unknown sequence");
    Sequence& sq = it->second;
    if (shift > sq.len) return c->fail(AOS_ERR_INVALID, "rotate shift beyond the sequence length");
    if (shift == 0) return AOS_OK;
    const uint32_t new_len = sq.len - shift, whole = shift / 16, r = shift % 16;
    std::rotate(sq.blocks.begin(), sq.blocks.begin() + whole, sq.blocks.end());
    if (r && new_len) {
        CTX_CUDA(c, cudaSetDevice(c->device));
        CTX_CUDA(c, cudaMemcpyAsync(c->d_zero_blocks, sq.blocks.data(), sq.blocks.size() * sizeof(int),
                                    cudaMemcpyHostToDevice, c->stream));
        LAUNCH(c, launch_kv_shift_rows(c->k_pool, c->v_pool, c->d_zero_blocks, (int)sq.blocks.size(), (int)r,
                                       (int)new_len, (int)c->cfg.n_layers, (int)c->cfg.kv_num_blocks,
                                       (int)c->cfg.n_kv_heads, c->stream));
        CTX_CUDA(c, cudaStreamSynchronize(c->stream));  // the page list buffer is reused by the next call
    }
    sq.len = new_len;
    return AOS_OK;
}

int aos_kv_fill_synthetic(aos_ctx* c, uint64_t seed, float std) {
    if (!c) return AOS_ERR_INVALID;
    const size_t n = (size_t)c->cfg.n_layers * c->cfg.kv_num_blocks * c->cfg.n_kv_heads * 16 * 128;
    CTX_CUDA(c, cudaSetDevice(c->device));
    LAUNCH(c, launch_fill_normal(c->k_pool, n, seed, std, c->stream));
    LAUNCH(c, launch_fill_normal(c->v_pool, n, seed ^ 0x5bd1e995ull, std, c->stream));
    CTX_CUDA(c, cudaStreamSynchronize(c->stream));
    return AOS_OK;
}

int aos_kv_clear_all(aos_ctx* c) {
    if (!c) return AOS_ERR_INVALID;
    std::vector<uint64_t> ids;
    for (auto& kv : c->seqs) ids.push_back(kv.first);
    for (auto id : ids) aos_kv_free(c, id);
    return AOS_OK;
}

// ---- KvCache generation guards and zeroization (crates/adapteros-lora-worker/
// src/kvcache.rs:288-402 and 586-733)
int aos_kv_zeroize(aos_ctx* c, uint64_t seq_id) {
    if (!c) return AOS_ERR_INVALID;
    auto it = c->seqs.find(seq_id);
    if (it == c->seqs.end()) return c->fail(AOS_ERR_NOT_FOUND, "Sequence ID " + std::to_string(seq_id) + " not found");
    const std::vector<int>& bl = it->second.blocks;
    if (bl.empty()) return AOS_OK;
    CTX_CUDA(c, cudaSetDevice(c->device));
    // a sequence holds at most kv_num_blocks blocks: the list goes into the
    // context's preallocated buffer (the synchronize below keeps it from
    // being overwritten by the next call while the kernel still reads it)
    CTX_CUDA(c, cudaMemcpyAsync(c->d_zero_blocks, bl.data(), bl.size() * sizeof(int), cudaMemcpyHostToDevice,
                                c->stream));
    LAUNCH(c, launch_zero_kv_blocks(c->k_pool, c->v_pool, c->d_zero_blocks, (int)bl.size(), (int)c->cfg.n_layers,
                                    (int)c->cfg.kv_num_blocks, (int)c->cfg.n_kv_heads, c->stream));
    CTX_CUDA(c, cudaStreamSynchronize(c->stream));
    return AOS_OK;
}

int aos_kv_zeroize_all(aos_ctx* c) {  // zeroize / reset_all: both pools to zero, every sequence released
    if (!c) return AOS_ERR_INVALID;
    CTX_CUDA(c, cudaSetDevice(c->device));
    CTX_CUDA(c, cudaStreamSynchronize(c->stream));
    const size_t bytes = aos_kv_memory_bytes(c) / 2;
    CTX_CUDA(c, cudaMemsetAsync(c->k_pool, 0, bytes, c->stream));
    CTX_CUDA(c, cudaMemsetAsync(c->v_pool, 0, bytes, c->stream));
    CTX_CUDA(c, cudaStreamSynchronize(c->stream));
    aos_kv_clear_all(c);
    c->kv_guards.clear();
    return AOS_OK;
}

int aos_kv_set_generation(aos_ctx* c, uint64_t generation) {
    if (!c) return AOS_ERR_INVALID;
    c->kv_generation = generation;
    return AOS_OK;
}

uint64_t aos_kv_generation(const aos_ctx* c) { return c ? c->kv_generation : 0; }

int aos_kv_ensure_coherence(aos_ctx* c, uint64_t generation, int* reset) {
    if (!c) return AOS_ERR_INVALID;
    if (reset) *reset = 0;
    if (generation == c->kv_generation) return AOS_OK;
    int rc = aos_kv_zeroize_all(c);  // reset_all: release every sequence, zero the pools
    if (rc) return rc;
    c->kv_generation = generation;
    if (reset) *reset = 1;
    return AOS_OK;
}

int aos_kv_alloc_guarded(aos_ctx* c, uint64_t seq_id, uint32_t max_tokens, uint64_t generation) {
    if (!c) return AOS_ERR_INVALID;
    int rc = aos_kv_ensure_coherence(c, generation, nullptr);
    if (!rc) rc = aos_kv_alloc(c, seq_id, max_tokens);
    if (!rc) c->kv_guards[seq_id] = generation;
    return rc;
}

int aos_kv_has_stale_guards(const aos_ctx* c, uint64_t generation) {
    if (!c) return 0;
    for (const auto& kv : c->kv_guards)
        if (kv.second != generation) return 1;
    return 0;
}

int aos_kv_drain_guarded(aos_ctx* c, uint32_t* n_drained) {
    if (!c) return AOS_ERR_INVALID;
    std::vector<uint64_t> ids;
    for (const auto& kv : c->kv_guards) ids.push_back(kv.first);
    for (uint64_t id : ids) aos_kv_free(c, id);
    c->kv_guards.clear();
    if (n_drained) *n_drained = (uint32_t)ids.size();
    return AOS_OK;
}

uint64_t aos_kv_memory_bytes(const aos_ctx* c) {
    return c ? (uint64_t)c->cfg.n_layers * c->cfg.kv_num_blocks * c->cfg.n_kv_heads * 16 * 128 * 2 * 2 : 0;
}

// ------------------------------------------------------------------ the step
int aos_run_step_batch_dev(aos_ctx* c, const aos_router_ring* rings, const uint32_t* token_ids, const uint64_t* seq_ids,
                           uint32_t T, float* logits, uint16_t* hidden_out, void* stream) {
    if (!c || !rings || !token_ids || !seq_ids || T == 0) return AOS_ERR_INVALID;
    cudaStream_t s = stream ? (cudaStream_t)stream : c->stream;
    CTX_CUDA(c, cudaSetDevice(c->device));
    int rc = stage_sequences(c, seq_ids, T);
    if (rc) return rc;
    if ((rc = upload_tables(c, T, s))) return rc;
    if (rings != c->d_rings)
        CTX_CUDA(c, cudaMemcpyAsync(c->d_rings, rings, (size_t)T * sizeof(aos_router_ring), cudaMemcpyDeviceToDevice, s));
    if (token_ids != c->d_tokens)
        CTX_CUDA(c, cudaMemcpyAsync(c->d_tokens, token_ids, (size_t)T * 4, cudaMemcpyDeviceToDevice, s));
    if ((rc = run_step_device(c, (int)T, true, s))) return rc;
    if (logits && logits != c->d_logits)
        CTX_CUDA(c, cudaMemcpyAsync(logits, c->d_logits, (size_t)T * c->cfg.vocab * 4, cudaMemcpyDeviceToDevice, s));
    if (hidden_out)
        CTX_CUDA(c, cudaMemcpyAsync(hidden_out, c->d_hidden, (size_t)T * c->cfg.hidden * 2, cudaMemcpyDeviceToDevice, s));
    advance(c, seq_ids, T);
    return AOS_OK;
}

int aos_run_step_batch(aos_ctx* c, const aos_router_ring* rings, const uint32_t* token_ids, const uint64_t* seq_ids,
                       uint32_t T, float* logits, uint16_t* hidden_out) {
    if (!c || !rings || !token_ids || !seq_ids || T == 0) return AOS_ERR_INVALID;
    if (T > c->cfg.max_batch) return c->fail(AOS_ERR_INVALID, "T exceeds max_batch");
    cudaStream_t s = c->stream;
    CTX_CUDA(c, cudaSetDevice(c->device));
    CTX_CUDA(c, cudaMemcpyAsync(c->d_rings, rings, (size_t)T * sizeof(aos_router_ring), cudaMemcpyHostToDevice, s));
    CTX_CUDA(c, cudaMemcpyAsync(c->d_tokens, token_ids, (size_t)T * 4, cudaMemcpyHostToDevice, s));
    CTX_CUDA(c, cudaEventRecord(c->ev0, s));
    int rc = aos_run_step_batch_dev(c, c->d_rings, c->d_tokens, seq_ids, T, c->d_logits, nullptr, s);
    if (rc) return rc;
    CTX_CUDA(c, cudaEventRecord(c->ev1, s));
    if (logits) CTX_CUDA(c, cudaMemcpyAsync(logits, c->d_logits, (size_t)T * c->cfg.vocab * 4, cudaMemcpyDeviceToHost, s));
    if (hidden_out)
        CTX_CUDA(c, cudaMemcpyAsync(hidden_out, c->d_hidden, (size_t)T * c->cfg.hidden * 2, cudaMemcpyDeviceToHost, s));
    CTX_CUDA(c, cudaStreamSynchronize(s));
    float ms = 0.f;
    cudaEventElapsedTime(&ms, c->ev0, c->ev1);
    c->m.last_step_ms = ms;
    return check_device_error(c);
}

// ------------------------------------------------------------------ prefill
namespace {
// The prefill step; `in_kind` says where rings and token_ids live
// (cudaMemcpyDeviceToDevice for aos_prefill_dev, HostToDevice for aos_prefill).
int prefill_run(aos_ctx* c, uint32_t n_seq, const uint64_t* seq_ids, const uint32_t* n_tok,
                const aos_router_ring* rings, const uint32_t* token_ids, float* logits, void* stream,
                cudaMemcpyKind in_kind) {
    if (!c || !seq_ids || !n_tok || !rings || !token_ids || n_seq == 0) return AOS_ERR_INVALID;
    if (n_seq > c->cfg.max_batch) return c->fail(AOS_ERR_INVALID, "more sequences than max_batch");
    cudaStream_t s = stream ? (cudaStream_t)stream : c->stream;
    CTX_CUDA(c, cudaSetDevice(c->device));
    // host side: positions, per-token page tables, query blocks of <= 16 tokens of one sequence
    size_t T = 0;
    for (uint32_t i = 0; i < n_seq; ++i) {
        if (n_tok[i] == 0) return c->fail(AOS_ERR_INVALID, "a sequence with no prompt tokens");
        T += n_tok[i];
    }
    if (T > (1u << 24)) return c->fail(AOS_ERR_INVALID, "prompt batch too large");
    std::vector<int> pos(T), bt(T * (size_t)c->max_blocks, 0);
    std::vector<int2> qblk;
    // query blocks of the prompt attention: 128 / G tokens (the tensor-core
    // kernel's 128 MMA rows hold the GQA group's heads for each token), else 16
    const bool attn_tc = attn_prefill_tc_supported((int)c->cfg.n_heads, (int)c->cfg.n_kv_heads);
    const uint32_t qb_size = attn_tc ? (uint32_t)attn_prefill_tc_block((int)c->cfg.n_heads, (int)c->cfg.n_kv_heads) : 16u;
    std::vector<size_t> last(n_seq);
    size_t t = 0;
    for (uint32_t i = 0; i < n_seq; ++i) {
        auto it = c->seqs.find(seq_ids[i]);
        if (it == c->seqs.end()) return c->fail(AOS_ERR_NOT_FOUND, "unknown sequence id " + std::to_string(seq_ids[i]));
        for (uint32_t u = 0; u < i; ++u)
            if (seq_ids[u] == seq_ids[i]) return c->fail(AOS_ERR_INVALID, "a sequence appears twice in one prefill");
        const Sequence& sq = it->second;
        if (sq.len + n_tok[i] > sq.cap) return c->fail(AOS_ERR_NOMEM, "prompt exceeds the sequence's KV capacity");
        for (uint32_t j = 0; j < n_tok[i]; ++j, ++t) {
            pos[t] = (int)(sq.len + j);
            std::copy(sq.blocks.begin(), sq.blocks.end(), bt.begin() + t * c->max_blocks);
            if (j % qb_size == 0) qblk.push_back(make_int2((int)t, (int)std::min<uint32_t>(qb_size, n_tok[i] - j)));
        }
        last[i] = t - 1;
    }
    int rc = prefill_reserve(c, (int)T);
    if (rc) return rc;
    auto& b = c->pf;
    CTX_CUDA(c, cudaMemcpyAsync(b.pos, pos.data(), T * 4, cudaMemcpyHostToDevice, s));
    CTX_CUDA(c, cudaMemcpyAsync(b.block_tables, bt.data(), bt.size() * 4, cudaMemcpyHostToDevice, s));
    CTX_CUDA(c, cudaMemcpyAsync(b.qblk, qblk.data(), qblk.size() * sizeof(int2), cudaMemcpyHostToDevice, s));
    CTX_CUDA(c, cudaMemcpyAsync(b.rings, rings, T * sizeof(aos_router_ring), in_kind, s));
    CTX_CUDA(c, cudaMemcpyAsync(b.tokens, token_ids, T * 4, in_kind, s));
    PLAUNCH(c, AOS_K_PREP, s,
            launch_lora_prep(b.rings, (int)T, c->d_col_off, c->d_rank, c->d_scale, (int)c->cfg.lora_max_adapters,
                             c->R / kGroup, c->d_groups, c->d_n_groups, b.coef, c->d_col_owner, b.ucoef, s));
    PLAUNCH(c, AOS_K_EMBED, s, launch_embed(c->embed, b.tokens, (int)T, (int)c->cfg.hidden, (int)c->cfg.vocab, b.hidden, s));
    CUtensorMap tm_q{};  // the q buffer [cap][n_heads * 128], boxes of 64 dims x qb_size tokens
    if (attn_tc && tc_encode_2d(&tm_q, b.q, (uint64_t)c->QD, (uint64_t)b.cap, (uint64_t)c->QD * 2, 64, qb_size, 128))
        return c->fail(AOS_ERR_CUDA, "prefill q tensor map encode failed");
    for (uint32_t l = 0; l < c->cfg.n_layers; ++l)
        if ((rc = enqueue_prefill_layer(c, (int)l, (int)T, (int)qblk.size(), attn_tc ? &tm_q : nullptr, s))) return rc;
    // every sequence's last token: final norm and lm_head on the decode buffers
    const size_t H = c->cfg.hidden;
    for (uint32_t i = 0; i < n_seq; ++i)
        CTX_CUDA(c, cudaMemcpyAsync(c->d_hidden + i * H, b.hidden + last[i] * H, H * 2, cudaMemcpyDeviceToDevice, s));
    if (logits) {
        StepPlan* plan = nullptr;
        if ((rc = get_plan(c, (int)n_seq, &plan))) return rc;
        // the final norm's first half; the decode lm_head plan applies 1 / rms
        PLAUNCH(c, AOS_K_NORM, s, launch_norm_prep(c->d_hidden, c->final_norm, (int)n_seq, (int)H, c->d_normed, c->d_ss, s));
        PLAUNCH(c, AOS_K_LM_HEAD, s, tc_launch(plan->lm_head, plan->lm_grid, s));
        if (logits != c->d_logits)
            CTX_CUDA(c, cudaMemcpyAsync(logits, c->d_logits, (size_t)n_seq * c->cfg.vocab * 4, cudaMemcpyDeviceToDevice, s));
    }
    for (uint32_t i = 0; i < n_seq; ++i) c->seqs[seq_ids[i]].len += n_tok[i];
    c->m.tokens += T;
    if (c->prof_on) {  // instrumented: collect the launch times now
        CTX_CUDA(c, cudaStreamSynchronize(s));
        for (size_t i = 0; i + 1 < c->prof_used; i += 2) {
            float ms = 0.f;
            cudaEventElapsedTime(&ms, c->prof_ev[i], c->prof_ev[i + 1]);
            c->prof.ms[c->prof_cls[i / 2]] += ms;
            c->prof.launches[c->prof_cls[i / 2]] += 1;
        }
        c->prof_used = 0;
    }
    return AOS_OK;
}
}  // namespace

int aos_prefill_dev(aos_ctx* c, uint32_t n_seq, const uint64_t* seq_ids, const uint32_t* n_tok,
                    const aos_router_ring* rings, const uint32_t* token_ids, float* logits, void* stream) {
    return prefill_run(c, n_seq, seq_ids, n_tok, rings, token_ids, logits, stream, cudaMemcpyDeviceToDevice);
}

int aos_prefill(aos_ctx* c, uint32_t n_seq, const uint64_t* seq_ids, const uint32_t* n_tok,
                const aos_router_ring* rings, const uint32_t* token_ids, float* logits) {
    if (!c) return AOS_ERR_INVALID;
    int rc = prefill_run(c, n_seq, seq_ids, n_tok, rings, token_ids, logits ? c->d_logits : nullptr, nullptr,
                         cudaMemcpyHostToDevice);
    if (rc) return rc;
    if (logits)
        CTX_CUDA(c, cudaMemcpyAsync(logits, c->d_logits, (size_t)n_seq * c->cfg.vocab * 4, cudaMemcpyDeviceToHost,
                                    c->stream));
    CTX_CUDA(c, cudaStreamSynchronize(c->stream));
    return check_device_error(c);
}

// ------------------------------------------------------------------ adapter-sharded step
int aos_shard_get_unique_id(void* id) {
    if (!id) return AOS_ERR_INVALID;
    static_assert(sizeof(ncclUniqueId) == AOS_SHARD_ID_BYTES, "NCCL unique id size");
    ncclUniqueId u;
    const ncclResult_t r = ncclGetUniqueId(&u);
    if (r != ncclSuccess) {
        set_global_error(std::string("ncclGetUniqueId: ") + ncclGetErrorString(r));
        return AOS_ERR_CUDA;
    }
    std::memcpy(id, &u, sizeof(u));
    return AOS_OK;
}

int aos_shard_init(aos_ctx* c, uint32_t rank, uint32_t world, const void* id) {
    if (!c || !id || world == 0 || rank >= world) return AOS_ERR_INVALID;
    if (c->nccl) return c->fail(AOS_ERR_STATE, "the context is already sharded");
    if (c->T_cap < (int)world) return c->fail(AOS_ERR_INVALID, "max_batch must hold one token of every rank");
    CTX_CUDA(c, cudaSetDevice(c->device));
    ncclUniqueId u;
    std::memcpy(&u, id, sizeof(u));
    NCCL_CHECK(c, ncclCommInitRank(&c->nccl, (int)world, u, (int)rank));
    c->shard_rank = (int)rank;
    c->shard_world = (int)world;
    const size_t TC = (size_t)c->T_cap, H = c->cfg.hidden, I = c->cfg.intermediate;
    const size_t in_max = std::max<size_t>({H, (size_t)c->QD, I});
    const size_t w_max = std::max<size_t>({(size_t)c->QD + 2 * c->KVD, H, 2 * I});
    CTX_CUDA(c, dalloc(&c->d_xrecv, TC * in_max));
    CTX_CUDA(c, dalloc(&c->d_dsend, TC * w_max));
    CTX_CUDA(c, dalloc(&c->d_drecv, TC * w_max));
    CTX_CUDA(c, dalloc(&c->d_rings_all, TC));
    for (auto& kv : c->plans)  // plans are built per mode; drop any built before
        if (kv.second->graph) cudaGraphExecDestroy(kv.second->graph);
    c->plans.clear();
    return AOS_OK;
}

int aos_run_step_sharded_dev(aos_ctx* c, const aos_router_ring* rings, const uint32_t* token_ids, const uint64_t* seq_ids,
                             uint32_t T, float* logits, uint16_t* hidden_out, void* stream) {
    if (!c || !rings || !token_ids || !seq_ids || T == 0) return AOS_ERR_INVALID;
    if (!c->nccl) return c->fail(AOS_ERR_STATE, "aos_shard_init has not been called");
    if ((size_t)T * c->shard_world > (size_t)c->T_cap)
        return c->fail(AOS_ERR_INVALID, "T * world exceeds max_batch (the owner side runs every rank's rows)");
    cudaStream_t s = stream ? (cudaStream_t)stream : c->stream;
    CTX_CUDA(c, cudaSetDevice(c->device));
    int rc = stage_sequences(c, seq_ids, T);
    if (rc) return rc;
    if ((rc = upload_tables(c, T, s))) return rc;
    if (rings != c->d_rings)
        CTX_CUDA(c, cudaMemcpyAsync(c->d_rings, rings, (size_t)T * sizeof(aos_router_ring), cudaMemcpyDeviceToDevice, s));
    if (token_ids != c->d_tokens)
        CTX_CUDA(c, cudaMemcpyAsync(c->d_tokens, token_ids, (size_t)T * 4, cudaMemcpyDeviceToDevice, s));
    if ((rc = run_step_device(c, (int)T, true, s, true))) return rc;
    if (logits && logits != c->d_logits)
        CTX_CUDA(c, cudaMemcpyAsync(logits, c->d_logits, (size_t)T * c->cfg.vocab * 4, cudaMemcpyDeviceToDevice, s));
    if (hidden_out)
        CTX_CUDA(c, cudaMemcpyAsync(hidden_out, c->d_hidden, (size_t)T * c->cfg.hidden * 2, cudaMemcpyDeviceToDevice, s));
    advance(c, seq_ids, T);
    return AOS_OK;
}

int aos_layer_step_dev(aos_ctx* c, uint32_t layer, const aos_router_ring* rings, const uint64_t* seq_ids, uint32_t T,
                       uint16_t* hidden, int adv, void* stream) {
    if (!c || !rings || !seq_ids || !hidden || T == 0) return AOS_ERR_INVALID;
    if (layer >= c->cfg.n_layers) return c->fail(AOS_ERR_INVALID, "layer out of range");
    cudaStream_t s = stream ? (cudaStream_t)stream : c->stream;
    CTX_CUDA(c, cudaSetDevice(c->device));
    int rc = stage_sequences(c, seq_ids, T);
    if (rc) return rc;
    if ((rc = upload_tables(c, T, s))) return rc;
    StepPlan* plan = nullptr;
    if ((rc = get_plan(c, (int)T, &plan))) return rc;
    if (rings != c->d_rings)
        CTX_CUDA(c, cudaMemcpyAsync(c->d_rings, rings, (size_t)T * sizeof(aos_router_ring), cudaMemcpyDeviceToDevice, s));
    CTX_CUDA(c, cudaMemcpyAsync(c->d_hidden, hidden, (size_t)T * c->cfg.hidden * 2, cudaMemcpyDeviceToDevice, s));
    LAUNCH(c, launch_lora_prep(c->d_rings, (int)T, c->d_col_off, c->d_rank, c->d_scale, (int)c->cfg.lora_max_adapters,
                               c->R / kGroup, c->d_groups, c->d_n_groups, c->d_coef, c->d_col_owner, c->d_ucoef, s));
    LAUNCH(c, launch_norm_prep(c->d_hidden, c->attn_norm[layer], (int)T, (int)c->cfg.hidden, c->d_normed, c->d_ss, s));
    if ((rc = enqueue_layer(c, *plan, (int)layer, s))) return rc;
    CTX_CUDA(c, cudaMemcpyAsync(hidden, c->d_hidden, (size_t)T * c->cfg.hidden * 2, cudaMemcpyDeviceToDevice, s));
    if (adv) advance(c, seq_ids, T);
    return AOS_OK;
}

// ------------------------------------------------------------------ metrics etc.
// Failure-path check: a kernel whose bounded wait can never be satisfied
// (0: a global-counter spin, 1: an mbarrier wait) runs on the context's
// stream; its time limit ends it, and the status comes back as a step's
// would: AOS_ERR_TIMEOUT, with the context's device state cleared so the next
// step runs normally.
int aos_debug_bounded_wait(aos_ctx* c, int kind) {
    if (!c || kind < 0 || kind > 1) return AOS_ERR_INVALID;
    CTX_CUDA(c, cudaSetDevice(c->device));
    int* never = nullptr;
    CTX_CUDA(c, cudaMallocAsync((void**)&never, sizeof(int), c->stream));
    CTX_CUDA(c, cudaMemsetAsync(never, 0, sizeof(int), c->stream));
    LAUNCH(c, tc_debug_wait(kind, never, c->d_err, c->stream));
    CTX_CUDA(c, cudaFreeAsync(never, c->stream));
    CTX_CUDA(c, cudaStreamSynchronize(c->stream));
    return check_device_error(c);
}

int aos_memory_report(aos_ctx* c, aos_memory_report_data* out, aos_adapter_allocation* allocs, uint32_t max_allocs,
                      uint32_t* n_allocs) {
    if (!c || !out) return AOS_ERR_INVALID;
    std::memset(out, 0, sizeof *out);
    CTX_CUDA(c, cudaSetDevice(c->device));
    size_t free_b = 0, total_b = 0;
    CTX_CUDA(c, cudaMemGetInfo(&free_b, &total_b));
    out->total_gpu_bytes = total_b;
    out->used_gpu_bytes = total_b - free_b;
    // bytes one rank column takes in every layer and LoRA module (lora_A row + lora_B column)
    uint64_t per_col = 0;
    for (int m = 0; m < AOS_NUM_MODULES; ++m)
        if (c->module_mask & (1u << m)) per_col += (uint64_t)(mod_in(c, m) + mod_out(c, m)) * 2;
    per_col *= c->cfg.n_layers;
    std::vector<uint16_t> ids;
    for (const auto& kv : c->adapters) ids.push_back(kv.first);
    std::sort(ids.begin(), ids.end());
    uint32_t k = 0;
    for (uint16_t id : ids) {
        const uint64_t b = per_col * (uint64_t)c->adapters[id].rank;
        out->adapter_vram_total += b;
        if (allocs && k < max_allocs) allocs[k++] = aos_adapter_allocation{id, b};
    }
    if (n_allocs) *n_allocs = (uint32_t)ids.size();
    out->adapter_count = (uint32_t)ids.size();
    out->arena_bytes = per_col * (uint64_t)c->R;
    out->arena_used_bytes = per_col * (uint64_t)c->m.arena_used_rank_cols;
    out->kv_pool_bytes = aos_kv_memory_bytes(c);
    const uint64_t used_blocks = c->cfg.kv_num_blocks - (uint64_t)c->free_blocks.size();
    out->kv_used_bytes = c->cfg.kv_num_blocks ? out->kv_pool_bytes / c->cfg.kv_num_blocks * used_blocks : 0;
    return AOS_OK;
}

int aos_debug_trace_read(aos_ctx* c, uint64_t* out, uint64_t n) {
    if (!c || !out) return AOS_ERR_INVALID;
    if (!c->d_trace) return c->fail(AOS_ERR_STATE, "tracing is off (set AOS_TC_TRACE before aos_init)");
    const uint64_t cap = (uint64_t)tc_num_sms() * kTraceStride;
    CTX_CUDA(c, cudaStreamSynchronize(c->stream));
    CTX_CUDA(c, cudaMemcpy(out, c->d_trace, (n < cap ? n : cap) * 8, cudaMemcpyDeviceToHost));
    return AOS_OK;
}

int aos_profile_enable(aos_ctx* c, int enable) {
    if (!c) return AOS_ERR_INVALID;
    c->prof_on = enable != 0;
    return AOS_OK;
}

int aos_profile_read(aos_ctx* c, aos_profile* out, int reset) {
    if (!c || !out) return AOS_ERR_INVALID;
    *out = c->prof;
    if (reset) c->prof = aos_profile{};
    return AOS_OK;
}

int aos_get_metrics(const aos_ctx* c, aos_metrics* out) {
    if (!c || !out) return AOS_ERR_INVALID;
    *out = c->m;
    return AOS_OK;
}

int aos_health_check(aos_ctx* c) {
    if (!c) return AOS_ERR_INVALID;
    cudaError_t e = cudaStreamQuery(c->stream);
    if (e != cudaSuccess && e != cudaErrorNotReady) return c->fail(AOS_ERR_CUDA, cudaGetErrorString(e));
    return check_device_error(c);
}

int aos_attest_determinism(const aos_ctx* c, aos_determinism_report* out) {
    if (!c || !out) return AOS_ERR_INVALID;
    std::memset(out, 0, sizeof(*out));
    std::snprintf(out->backend, sizeof(out->backend), "cuda-sm100a");
    std::snprintf(out->device_name, sizeof(out->device_name), "%s", c->dev_name.c_str());
    cudaDeviceProp p;
    cudaGetDeviceProperties(&p, c->device);
    out->sm_major = (uint32_t)p.major;
    out->sm_minor = (uint32_t)p.minor;
    out->fast_math = 0;
    out->float_atomics = 0;
    out->fixed_reduction_order = 1;
#ifndef AOS_BUILD_STAMP
#define AOS_BUILD_STAMP "unstamped"
#endif
#ifndef AOS_BUILD_FLAGS
#define AOS_BUILD_FLAGS ""
#endif
    std::snprintf(out->kernel_build_id, sizeof(out->kernel_build_id), "%s", AOS_BUILD_STAMP);
    std::snprintf(out->compiler_flags, sizeof(out->compiler_flags), "%s", AOS_BUILD_FLAGS);
    int rt = 0, drv = 0;
    cudaRuntimeGetVersion(&rt);
    cudaDriverGetVersion(&drv);
    std::snprintf(out->runtime_version, sizeof(out->runtime_version), "cuda runtime %d.%d, driver api %d.%d", rt / 1000,
                  (rt % 1000) / 10, drv / 1000, (drv % 1000) / 10);
    char bus[32] = {0};
    cudaDeviceGetPCIBusId(bus, sizeof bus, c->device);
    std::snprintf(out->device_id, sizeof(out->device_id), "cuda:%d %s", c->device, bus);
    out->rng_seed_method = 0;       // the device path draws no random numbers; routing and sampling take the caller's
    out->floating_point_mode = 0;   // IEEE division and square root, no flush-to-zero, no fast-math
    out->determinism_level = 2;     // bit-identical run to run (fixed-order reductions, no float atomics)
    out->deterministic = 1;
    return AOS_OK;
}

}  // extern "C"
