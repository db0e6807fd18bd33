"""Decoder parity at BASELINE config 3's own shapes (the configuration the
decode tok/s metric is quoted on), against the CPU oracle's restatement of
mlx_cpp_wrapper_real.cpp:3338-3559.

Shapes: hidden 4096, 32 query / 8 KV heads of 128, SwiGLU intermediate 14336,
vocab 128256, RMSNorm eps 1e-5, RoPE theta 1e6; 128 adapters with ranks drawn
from {8, 16, 32, 64} on all seven modules (q/k/v/o/gate/up/down) in one
shared rank-group arena; K=4 routing of 64 decode tokens from N(0,1) priors;
ragged paged contexts drawn from U[512, 4096] (one to four 64-page attention
chunks, partial last pages).  Two layers instead of 32: every layer runs the
same launches, and the second layer checks that the first layer's outputs
feed it correctly.

Checked: the GPU router's rings byte for byte against the oracle's; the
logits over the full vocabulary, the final hidden state and the K/V rows the
step appends in both layers for all 64 tokens, each within relative L2 and
relative max-abs error 2e-2 (bf16 path); and a second step from the same
cache state giving bit-identical logits and hidden state."""
import numpy as np
import pytest

from oracle import oracle as O
from tests.aos_import import aos
from tests.test_decoder_gpu import assert_close

pytestmark = pytest.mark.gpu

H, NH, NKV, HD, INTER, VOCAB = 4096, 32, 8, 128, 14336, 128256
LAYERS, T, N_ADAPTERS, K = 2, 64, 128, 4
CTX_LO, CTX_HI = 512, 4096


def _paged_kv(rng, m, ctx):
    """Oracle KV pools: sequence t owns consecutive blocks, ~N(0,1) bf16 rows."""
    nb = (ctx + 1 + 15) // 16  # room for the appended row
    off = np.concatenate([[0], np.cumsum(nb)[:-1]]).astype(np.int64)
    mb = int(nb.max())
    bt = np.zeros((len(ctx), mb), np.int32)
    for t in range(len(ctx)):
        bt[t, :nb[t]] = off[t] + np.arange(nb[t])
    n_blocks = int(nb.sum())
    kv = O.HostKV(m, n_blocks, 16, bt, ctx)
    for pool in (kv.k_pool, kv.v_pool):
        for l in range(LAYERS):
            pool[l] = O.f32_to_bf16_bits(rng.standard_normal(pool[l].shape, dtype=np.float32))
    return kv, nb, off


def _seq_rows(kv, l, off, nb, n):
    """Rows [0, n) of one sequence in a pool: [n, n_kv, 128]."""
    k = kv.k_pool[l, off:off + nb].transpose(0, 2, 1, 3).reshape(-1, NKV, HD)[:n]
    v = kv.v_pool[l, off:off + nb].transpose(0, 2, 1, 3).reshape(-1, NKV, HD)[:n]
    return k, v


def test_config3_shapes_two_layers():
    rng = np.random.default_rng(303)
    m = O.HostModel.random(rng, H, NH, NKV, HD, INTER, VOCAB, LAYERS)
    ranks = [int(r) for r in rng.choice(np.array([8, 16, 32, 64]), size=N_ADAPTERS)]
    ad = O.HostAdapters.random(rng, m, ranks)
    ctx = rng.integers(CTX_LO, CTX_HI + 1, size=T).astype(np.int32)
    kv, nb, off = _paged_kv(rng, m, ctx)
    priors = rng.standard_normal((T, N_ADAPTERS), dtype=np.float32)
    tokens = rng.integers(0, VOCAB, size=T).astype(np.int32)

    rings, _, _, _ = O.route_batch(priors, None, k=K)
    g_rings, _, _ = aos.route_batch(priors, k=K)
    assert g_rings.tobytes() == rings.tobytes(), "GPU router rings differ from the oracle's at config 3"

    cap = sum(((r + 15) // 16) * 16 for r in ranks) + 64
    seq_cap = ctx + 16  # each sequence's KV reservation: its context plus the appended row
    gpu = aos.CudaKernels(H, NH, NKV, HD, INTER, VOCAB, LAYERS, max_batch=T,
                          kv_num_blocks=int(((seq_cap + 15) // 16).sum()) + 64, max_seq_len=CTX_HI + 32,
                          lora_rank_capacity=cap, lora_max_adapters=N_ADAPTERS)
    try:
        gpu.load_host_model(m)
        for a in range(N_ADAPTERS):
            gpu.load_adapter_with_metadata(a, ranks[a], ad.alphas[a],
                                           {(l, mod): (ad.A[a][l][mod], ad.B[a][l][mod])
                                            for l in range(LAYERS) for mod in range(7)})
        sids = np.arange(1000, 1000 + T, dtype=np.uint64)
        for t in range(T):
            gpu.kv_alloc(int(sids[t]), int(seq_cap[t]))
            for l in range(LAYERS):
                k, v = _seq_rows(kv, l, int(off[t]), int(nb[t]), int(ctx[t]))
                gpu.kv_write(int(sids[t]), l, 0, k, v)
            gpu.kv_set_len(int(sids[t]), int(ctx[t]))

        logits, hidden = gpu.run_step_batch(rings, tokens.astype(np.uint32), sids, want_hidden=True)
        new_rows = [[gpu.kv_read(int(sids[t]), l, int(ctx[t]), 1) for l in range(LAYERS)] for t in range(T)]
        assert [gpu.kv_len(int(x)) for x in sids] == [int(n) + 1 for n in ctx]

        # the same step again from the same cache state: bit-identical
        for t in range(T):
            gpu.kv_set_len(int(sids[t]), int(ctx[t]))
        logits2, hidden2 = gpu.run_step_batch(rings, tokens.astype(np.uint32), sids, want_hidden=True)
        assert logits2.tobytes() == logits.tobytes(), "config-3 logits differ run to run"
        assert hidden2.tobytes() == hidden.tobytes(), "config-3 hidden state differs run to run"
    finally:
        gpu.close()

    ref_logits, ref_hidden = O.decode_step(m, ad, rings, tokens, kv)
    assert_close(O.bf16_bits_to_f32(hidden), O.bf16_bits_to_f32(ref_hidden), "config-3 hidden")
    assert_close(logits, ref_logits, "config-3 logits")
    for t in range(T):
        pos = int(ctx[t])
        blk = kv.block_tables[t, pos // 16]
        for l in range(LAYERS):
            gk, gv = new_rows[t][l]
            assert_close(O.bf16_bits_to_f32(gk[0]), O.bf16_bits_to_f32(kv.k_pool[l, blk, :, pos % 16]),
                         f"config-3 k row t={t} l={l}")
            assert_close(O.bf16_bits_to_f32(gv[0]), O.bf16_bits_to_f32(kv.v_pool[l, blk, :, pos % 16]),
                         f"config-3 v row t={t} l={l}")
