/*
 * aos_oracle.h — CPU restatement of adapter-os's per-token hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the product library links, loads or
 * calls this code; only tests/, __graft_entry__.smoke() and bench.py's CPU
 * baseline arm use it, and only as the checker / timed CPU reference.
 *
 * Each function cites the reference file:line it restates.  Paths are relative
 * to the rogu3bear/adapter-os source tree.
 *
 * Built with -O3 -fno-fast-math -ffp-contract=off so every float/double
 * operation is a single IEEE-754 rounding, in the order written, matching the
 * reference's "no fast-math" determinism rule (DETERMINISM.md:30-32).
 */
#ifndef AOS_ORACLE_H
#define AOS_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Same 40-byte layout as the device RouterRing
 * (crates/adapteros-lora-kernel-mtl/src/ring_buffer.rs:44-58). */
typedef struct oracle_ring {
    uint32_t top_k;
    uint32_t position;
    uint16_t indices[8];
    int16_t gates_q15[8];
} oracle_ring;

/* Status codes (mirrors AOS_* in include/aos_cuda.h). */
#define ORACLE_OK 0
#define ORACLE_ERR_INVALID (-1)
#define ORACLE_ERR_NONFINITE (-4)

/* ---- router numeric core ------------------------------------------------ */

/* quantize_gate (crates/adapteros-lora-router/src/quantization.rs:172-175). */
int16_t oracle_quantize_gate(float gate);

/* deterministic_softmax (router.rs:1340-1411): writes n f32 probabilities. */
void oracle_deterministic_softmax(const float* scores, int n, float tau, float* out);

/* Route T tokens independently, each with the reference router
 * (router.rs:1567-1952).  priors: [T, N] row-major.  stable_ids: [N].
 * version_weights: [N] or NULL (=1.0).  allowed: [N] or NULL (=allow all).
 * k/tau/eps are sanitised exactly as Router::new_with_weights does
 * (router.rs:397-400 via :127-187).  positions: [T] or NULL (ring.position = 0).
 * Outputs: rings[T], entropy[T] (may be
 * NULL), status[T] (may be NULL; 0 or ORACLE_ERR_NONFINITE).
 * Returns 0, or ORACLE_ERR_NONFINITE if any token's routing errored. */
int oracle_route_batch(const float* priors, const uint64_t* stable_ids,
                       const float* version_weights, const uint8_t* allowed,
                       uint32_t T, uint32_t N, uint32_t k, float tau, float eps,
                       float routing_bias, const uint32_t* positions,
                       oracle_ring* rings, float* entropy, int32_t* status,
                       int n_threads);

/* ---- fp32 LoRA op (config 1) ------------------------------------------- */

/* y[t] = W x[t] + sum_{slots with q15>0} (q15/32767 * acc) * (alpha/rank)
 * restating cpu_lora_forward (crates/adapteros-testing/src/kernel_testing.rs:220-257)
 * for the base product and blend_and_forward_reference
 * (crates/adapteros-lora-kernel-api/src/liquid.rs:222-250) for the adapter loop.
 * W: [out, in]; A: [n_adapters, rank, in]; B: [n_adapters, out, rank];
 * alpha: [n_adapters] (NULL → alpha = rank, i.e. scaling 1). */
int oracle_lora_op_f32(const float* x, uint32_t T, uint32_t in_dim, uint32_t out_dim,
                       const float* W, const float* A, const float* B,
                       uint32_t n_adapters, uint32_t rank, const float* alpha,
                       const oracle_ring* rings, float* y, int n_threads);

/* blend_and_forward_reference (crates/adapteros-lora-kernel-api/src/liquid.rs:163-251)
 * with f32 coefficients: y = sum_i coeff_i * (B_i (A_i x)) * (alpha_i / rank_i),
 * skipping coeff == 0.  A_i: [rank_i, in], B_i: [out_i, rank_i] (out_i <= out).
 * Returns ORACLE_ERR_INVALID on the reference's validation failures (zero
 * adapters, more than 3, or rank mismatch). */
int oracle_liquid_blend_f32(const float* x, uint32_t in_dim, uint32_t out_dim,
                            uint32_t n_adapters, const float* const* A, const float* const* B,
                            const uint32_t* rank, const uint32_t* b_rows, const float* alpha,
                            const float* coeff, float* y);

/* ---- bf16 decoder (configs 2-4) ---------------------------------------- */

/* Module ids, in the order of MLXLoraLayer (mlx_cpp_wrapper_real.cpp:1248-1256). */
enum { ORACLE_MOD_Q = 0, ORACLE_MOD_K, ORACLE_MOD_V, ORACLE_MOD_O,
       ORACLE_MOD_GATE, ORACLE_MOD_UP, ORACLE_MOD_DOWN, ORACLE_NUM_MODS };

typedef struct oracle_model {
    uint32_t hidden, n_heads, n_kv_heads, head_dim, inter, vocab, n_layers;
    float rms_eps, rope_theta;
    uint32_t rope_mlx_as_written; /* 1 = reproduce inv_freq = 1/theta^(-2i/hd) */
    const uint16_t* embed;        /* [vocab, hidden] bf16 (may be NULL for layer-only use) */
    const uint16_t* lm_head;      /* [vocab, hidden] */
    const uint16_t* final_norm;   /* [hidden] */
    const uint16_t* const* attn_norm; /* [n_layers] -> [hidden] */
    const uint16_t* const* mlp_norm;  /* [n_layers] -> [hidden] */
    const uint16_t* const* w[ORACLE_NUM_MODS]; /* [n_layers] -> [out, in] */
} oracle_model;

typedef struct oracle_adapters {
    uint32_t n_adapters;
    const uint32_t* rank;         /* [n_adapters] */
    const float* alpha;           /* [n_adapters] */
    /* [n_adapters * n_layers * 7] -> A [rank, in] / B [out, rank]; NULL = absent */
    const uint16_t* const* A;
    const uint16_t* const* B;
} oracle_adapters;

/* Paged KV cache: pools are [n_layers][num_blocks][n_kv_heads][block_size][head_dim]
 * bf16; block_tables [T][max_blocks]; ctx_lens[T] = tokens already cached for
 * token t's sequence (its position).  The step writes the new K/V at that
 * position. */
typedef struct oracle_kv {
    uint16_t* k_pool;
    uint16_t* v_pool;
    uint32_t num_blocks, block_size, max_blocks;
    const int32_t* block_tables;
    const int32_t* ctx_lens;
} oracle_kv;

/* rounding_mode 0: round to bf16 at the storage points of the fused CUDA path;
 * 1: round after every op as MLX's bf16 graph does (mlx_cpp_wrapper_real.cpp:3437-3531). */
int oracle_layer_step(const oracle_model* m, const oracle_adapters* ad, uint32_t layer,
                      const oracle_ring* rings, uint32_t T, oracle_kv* kv,
                      uint16_t* hidden /* [T, hidden] bf16, in/out */,
                      int rounding_mode, int n_threads);

/* Whole decode step: embedding -> n_layers_run layers -> final norm -> lm_head.
 * logits [T, vocab] f32 (may be NULL); hidden_out [T, hidden] bf16 final hidden
 * after the last run layer (before the final norm; may be NULL). */
int oracle_decode_step(const oracle_model* m, const oracle_adapters* ad,
                       const oracle_ring* rings, const int32_t* token_ids, uint32_t T,
                       oracle_kv* kv, uint32_t n_layers_run, int rounding_mode,
                       float* logits, uint16_t* hidden_out, int n_threads);

/* RoPE cos/sin table [max_pos][head_dim/2] (cos, sin interleaved), computed the
 * way the oracle's RoPE computes its angles. */
void oracle_rope_table(uint32_t head_dim, float theta, uint32_t mlx_as_written,
                       uint32_t max_pos, float* table);

/* Helpers exposed for tests. */
float oracle_bf16_to_f32(uint16_t h);
uint16_t oracle_f32_to_bf16(float f);

#ifdef __cplusplus
}
#endif
#endif
