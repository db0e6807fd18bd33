"""Prefill (aos_prefill_dev) on the GPU vs the CPU oracle fed one token at a
time (oracle/aos_oracle.cpp: the decode step of mlx_cpp_wrapper_real.cpp:3338-3559
at consecutive positions is the causal prompt pass).

The prompt attention runs on the tensor-core kernel (attention_tc.cu) when the
GQA group size divides 128, else on the mma.sync kernel; both are checked.

Small case: three prompts (37 tokens from an empty cache, 50 tokens after 20
cached ones, a single token) in one 256-token tile.  Multi-tile case: prompts
of 300 tokens, 2100 tokens after 24 cached ones, and 5 tokens (2405 tokens:
ten 256-token tiles, so the two-accumulator M=256 tiles, the band schedule of
eight token tiles per weight tile and a partial last tile all run; causal
attention over up to 133 pages).  LoRA on all seven modules.  Checked: each
sequence's last-token logits, every K/V row the prompt appends (all layers,
which also checks every prompt token's attention output of the first layer
through the second layer's K/V), the new sequence lengths, and bit-identical
results run to run.
Tolerance (bf16 path): relative L2 <= 2e-2 and max-abs <= 2e-2 * max|ref|."""
import numpy as np
import pytest

from oracle import oracle as O
from tests.aos_import import aos
from tests.test_decoder_gpu import assert_close

pytestmark = pytest.mark.gpu


def _case(seed=7, hidden=256, nh=4, nkv=2, inter=384, vocab=1000, L=2, prompts=((0, 37), (20, 50), (0, 1)),
          ranks=(16, 8, 32, 16, 64, 8), K=4, max_seq=256):
    rng = np.random.default_rng(seed)
    m = O.HostModel.random(rng, hidden, nh, nkv, 128, inter, vocab, L)
    ad = O.HostAdapters.random(rng, m, list(ranks), modules=list(range(7)))
    S = len(prompts)
    mb = (max_seq + 15) // 16
    bt = np.arange(S * mb, dtype=np.int32).reshape(S, mb)
    kv = O.HostKV(m, S * mb, 16, bt, np.array([p[0] for p in prompts], np.int32))
    for i, (n0, _) in enumerate(prompts):  # cached context before the prompt
        for l in range(L):
            for p in range(n0):
                kv.k_pool[l, bt[i, p // 16], :, p % 16] = O.f32_to_bf16_bits(rng.standard_normal((nkv, 128), dtype=np.float32))
                kv.v_pool[l, bt[i, p // 16], :, p % 16] = O.f32_to_bf16_bits(rng.standard_normal((nkv, 128), dtype=np.float32))
    T = sum(p[1] for p in prompts)
    rings, _, _, _ = O.route_batch(rng.standard_normal((T, len(ranks))).astype(np.float32), None, k=K)
    tokens = rng.integers(0, vocab, size=T).astype(np.int32)
    return m, ad, kv, bt, rings, tokens, prompts, max_seq


def _gpu(m, ad, kv, bt, prompts, max_seq, sids):
    S, mb = bt.shape
    gpu = aos.CudaKernels(m.hidden, m.n_heads, m.n_kv_heads, 128, m.inter, m.vocab, m.n_layers, max_batch=8,
                          kv_num_blocks=S * mb + 8, max_seq_len=max_seq, lora_rank_capacity=256,
                          lora_max_adapters=ad.n)
    gpu.load_host_model(m)
    for a in range(ad.n):
        gpu.load_adapter_with_metadata(a, ad.ranks[a], ad.alphas[a],
                                       {(l, mod): (ad.A[a][l][mod], ad.B[a][l][mod])
                                        for l in range(m.n_layers) for mod in range(7)})
    for i, (n0, _) in enumerate(prompts):
        gpu.kv_alloc(int(sids[i]), max_seq)
        for l in range(m.n_layers):
            if n0:
                k = kv.k_pool[l, bt[i]].transpose(0, 2, 1, 3).reshape(-1, m.n_kv_heads, 128)[:n0]
                v = kv.v_pool[l, bt[i]].transpose(0, 2, 1, 3).reshape(-1, m.n_kv_heads, 128)[:n0]
                gpu.kv_write(int(sids[i]), l, 0, k, v)
        gpu.kv_set_len(int(sids[i]), n0)
    return gpu


def _check_prefill(**case):
    import torch
    m, ad, kv, bt, rings, tokens, prompts, max_seq = _case(**case)
    S = len(prompts)
    sids = np.arange(500, 500 + S, dtype=np.uint64)
    n_tok = np.array([p[1] for p in prompts], np.uint32)
    outs = []
    for rep in range(2):
        gpu = _gpu(m, ad, kv, bt, prompts, max_seq, sids)
        rd = torch.from_numpy(rings.view(np.uint8).copy()).cuda()
        td = torch.from_numpy(tokens.copy()).cuda()
        logits = torch.empty((S, m.vocab), dtype=torch.float32, device="cuda")
        gpu.prefill_dev(sids, n_tok, rd, td, logits=logits)
        torch.cuda.synchronize()
        gpu.health_check()
        lens = [gpu.kv_len(int(x)) for x in sids]
        rows = [[gpu.kv_read(int(sids[i]), l, prompts[i][0], prompts[i][1]) for l in range(m.n_layers)]
                for i in range(S)]
        outs.append((logits.cpu().numpy(), rows, lens))
        gpu.close()
    assert outs[0][0].tobytes() == outs[1][0].tobytes(), "prefill logits differ run to run"
    assert outs[0][2] == [p[0] + p[1] for p in prompts]
    # oracle: the same tokens one position at a time
    t = 0
    for i, (n0, n) in enumerate(prompts):
        kvi = O.HostKV(m, kv.num_blocks, 16, bt[i:i + 1], np.array([n0], np.int32), k_pool=kv.k_pool, v_pool=kv.v_pool)
        ref = None
        for j in range(n):
            kvi.ctx_lens[0] = n0 + j
            ref, _ = O.decode_step(m, ad, rings[t:t + 1], tokens[t:t + 1], kvi)
            t += 1
        assert_close(outs[0][0][i], ref[0], f"sequence {i} last-token logits")
        for l in range(m.n_layers):
            gk, gv = outs[0][1][i][l]
            rk = np.stack([kv.k_pool[l, bt[i, p // 16], :, p % 16] for p in range(n0, n0 + n)])
            rv = np.stack([kv.v_pool[l, bt[i, p // 16], :, p % 16] for p in range(n0, n0 + n)])
            assert_close(O.bf16_bits_to_f32(gk), O.bf16_bits_to_f32(rk), f"sequence {i} layer {l} k rows")
            assert_close(O.bf16_bits_to_f32(gv), O.bf16_bits_to_f32(rv), f"sequence {i} layer {l} v rows")


def test_prefill_matches_oracle():
    _check_prefill()


@pytest.mark.parametrize("nh,nkv", [(4, 2), (8, 2)])
def test_prefill_multi_tile_matches_oracle(nh, nkv):
    """GQA groups of 2 and 4 (config 4's group): the tensor-core attention with
    query blocks of 64 and 32 tokens, 128-key tiles up to 2124 positions."""
    _check_prefill(seed=11, nh=nh, nkv=nkv, prompts=((0, 300), (24, 2100), (0, 5)), max_seq=2144)


def test_prefill_gqa3_mma_sync_path():
    """A GQA group of 3 does not divide the tensor-core kernel's 128 rows: the
    prompt attention runs on the mma.sync kernel (16-token query blocks)."""
    _check_prefill(seed=13, nh=6, nkv=2, prompts=((0, 70), (33, 150), (0, 1)), max_seq=256)
