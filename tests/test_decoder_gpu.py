"""Decoder path on the GPU vs the CPU oracle (mlx_cpp_wrapper_real.cpp:3338-3559
restated in oracle/aos_oracle.cpp).

Tolerance (bf16 path): relative L2 error <= 2e-2 and max-abs error <= 2e-2 *
max|ref| for logits, hidden states and the K/V rows the step appends; the same
bound is checked against the oracle's MLX op-by-op bf16 rounding mode."""
import numpy as np
import pytest

from oracle import oracle as O
from tests.aos_import import aos

pytestmark = pytest.mark.gpu

TOL = 2e-2


def rel_err(got, ref):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    l2 = np.linalg.norm(got - ref) / max(np.linalg.norm(ref), 1e-30)
    mx = np.abs(got - ref).max() / max(np.abs(ref).max(), 1e-30)
    return l2, mx


def assert_close(got, ref, what):
    l2, mx = rel_err(got, ref)
    assert l2 <= TOL and mx <= TOL, f"{what}: rel-L2 {l2:.3e}, rel-max {mx:.3e}"


class Setup:
    def __init__(self, seed=0, hidden=256, nh=4, nkv=2, inter=384, vocab=1000, L=2, ctx_lens=(0, 1, 15, 16, 300),
                 ranks=(8, 16, 32, 8, 64, 16), K=4, modules=range(7), max_seq=512, route=True, rank_cap=256):
        rng = np.random.default_rng(seed)
        self.rng = rng
        self.m = O.HostModel.random(rng, hidden, nh, nkv, 128, inter, vocab, L)
        self.ad = O.HostAdapters.random(rng, self.m, list(ranks), modules=list(modules)) if ranks else None
        T = len(ctx_lens)
        self.T = T
        self.ctx_lens = np.array(ctx_lens, np.int32)
        mb = (max_seq + 15) // 16
        self.nb = T * mb
        bt = np.arange(T * mb, dtype=np.int32).reshape(T, mb)
        self.kv = O.HostKV(self.m, self.nb, 16, bt, self.ctx_lens.copy())  # own copy: tests advance it
        # cached K/V ~ N(0, 1)
        for t, n in enumerate(ctx_lens):
            for l in range(L):
                k = O.f32_to_bf16_bits(rng.standard_normal((n, nkv, 128), dtype=np.float32))
                v = O.f32_to_bf16_bits(rng.standard_normal((n, nkv, 128), dtype=np.float32))
                for p in range(n):
                    blk = bt[t, p // 16]
                    self.kv.k_pool[l, blk, :, p % 16, :] = k[p]
                    self.kv.v_pool[l, blk, :, p % 16, :] = v[p]
        n_ad = len(ranks) if ranks else 1
        logits = rng.standard_normal((T, n_ad), dtype=np.float32)
        if ranks and route:
            self.rings, _, _, _ = O.route_batch(logits, None, k=min(K, n_ad))
        else:
            self.rings = np.zeros(T, O.RING_DTYPE)
        self.tokens = rng.integers(0, vocab, size=T).astype(np.int32)
        self.tokens[0] = vocab + 5  # out of vocabulary -> zero embedding
        self.gpu = aos.CudaKernels(hidden, nh, nkv, 128, inter, vocab, L, max_batch=max(T, 8),
                                   kv_num_blocks=self.nb + 8, max_seq_len=max_seq, lora_rank_capacity=rank_cap,
                                   lora_max_adapters=max(n_ad, 1), lora_modules=[aos.MODULES[i] for i in modules])
        self.gpu.load_host_model(self.m)
        if self.ad is not None:
            for a in range(self.ad.n):
                mods = {(l, mod): (self.ad.A[a][l][mod], self.ad.B[a][l][mod])
                        for l in range(L) for mod in modules}
                self.gpu.load_adapter_with_metadata(a, self.ad.ranks[a], self.ad.alphas[a], mods)
        self.seq_ids = np.arange(100, 100 + T, dtype=np.uint64)
        for t, n in enumerate(ctx_lens):
            sid = int(self.seq_ids[t])
            self.gpu.kv_alloc(sid, max_seq)
            for l in range(L):
                if n:
                    k = np.stack([self.kv.k_pool[l, bt[t, p // 16], :, p % 16, :] for p in range(n)])
                    v = np.stack([self.kv.v_pool[l, bt[t, p // 16], :, p % 16, :] for p in range(n)])
                    self.gpu.kv_write(sid, l, 0, k, v)
            self.gpu.kv_set_len(sid, n)

    def oracle_kv_row(self, t, l, pos):
        blk = self.kv.block_tables[t, pos // 16]
        return self.kv.k_pool[l, blk, :, pos % 16, :], self.kv.v_pool[l, blk, :, pos % 16, :]


def _decode_and_compare(s: Setup, mode=0):
    ref_logits, ref_hidden = O.decode_step(s.m, s.ad, s.rings, s.tokens, s.kv, rounding_mode=mode)
    return ref_logits, ref_hidden


@pytest.mark.parametrize("with_lora", [False, True])
def test_decode_step_small(with_lora):
    s = Setup(seed=1, ranks=(8, 16, 32, 8, 64, 16) if with_lora else ())
    logits, hidden = s.gpu.run_step_batch(s.rings, s.tokens.astype(np.uint32), s.seq_ids, want_hidden=True)
    ref_logits, ref_hidden = O.decode_step(s.m, s.ad, s.rings, s.tokens, s.kv)
    # appended K/V rows (RoPE'd k, v) for every layer
    for t in range(s.T):
        pos = int(s.ctx_lens[t])
        for l in range(s.m.n_layers):
            gk, gv = s.gpu.kv_read(int(s.seq_ids[t]), l, pos, 1)
            rk, rv = s.oracle_kv_row(t, l, pos)
            assert_close(O.bf16_bits_to_f32(gk[0]), O.bf16_bits_to_f32(rk), f"k t={t} l={l}")
            assert_close(O.bf16_bits_to_f32(gv[0]), O.bf16_bits_to_f32(rv), f"v t={t} l={l}")
    assert_close(O.bf16_bits_to_f32(hidden), O.bf16_bits_to_f32(ref_hidden), "hidden")
    assert_close(logits, ref_logits, "logits")
    # the MLX op-by-op rounding of the same math stays within the same bound
    s2 = Setup(seed=1, ranks=(8, 16, 32, 8, 64, 16) if with_lora else ())
    mlx_logits, _ = O.decode_step(s2.m, s2.ad, s2.rings, s2.tokens, s2.kv, rounding_mode=1)
    assert_close(logits, mlx_logits, "logits vs MLX rounding")
    # positions advanced (IoBuffers.position += 1)
    assert [s.gpu.kv_len(int(x)) for x in s.seq_ids] == [int(n) + 1 for n in s.ctx_lens]
    s.gpu.close()
    s2.gpu.close()


def test_decode_step_two_token_blocks():
    """T > 128: two MMA token blocks per tile, one TMEM accumulator, split base
    tiles summed from fp32 partials."""
    rng = np.random.default_rng(9)
    ctx = tuple(int(x) for x in rng.integers(0, 90, size=160))
    outs = []
    for _ in range(2):
        s = Setup(seed=4, ctx_lens=ctx, max_seq=128)
        logits, hidden = s.gpu.run_step_batch(s.rings, s.tokens.astype(np.uint32), s.seq_ids, want_hidden=True)
        outs.append((logits.tobytes(), hidden.tobytes()))
        if len(outs) == 1:
            ref_logits, ref_hidden = O.decode_step(s.m, s.ad, s.rings, s.tokens, s.kv)
            assert_close(O.bf16_bits_to_f32(hidden), O.bf16_bits_to_f32(ref_hidden), "hidden (T=160)")
            assert_close(logits, ref_logits, "logits (T=160)")
        s.gpu.close()
    assert outs[0] == outs[1], "T=160 step differs run to run"


@pytest.mark.parametrize("T", [1, 17, 64, 65, 127, 128, 129, 256])
def test_decode_step_batch_sizes(T):
    """Ragged batch sizes across the token-block and tile boundaries (one and
    two MMA token blocks, T = 256 as the adapter owners run it): logits and
    hidden states within tolerance of the oracle, and every appended K/V row
    of the first and last token."""
    rng = np.random.default_rng(100 + T)
    ctx = tuple(int(x) for x in rng.integers(0, 40, size=T))
    s = Setup(seed=T, ctx_lens=ctx, max_seq=64)
    logits, hidden = s.gpu.run_step_batch(s.rings, s.tokens.astype(np.uint32), s.seq_ids, want_hidden=True)
    ref_logits, ref_hidden = O.decode_step(s.m, s.ad, s.rings, s.tokens, s.kv)
    assert_close(O.bf16_bits_to_f32(hidden), O.bf16_bits_to_f32(ref_hidden), f"hidden (T={T})")
    assert_close(logits, ref_logits, f"logits (T={T})")
    for t in {0, T - 1}:
        pos = int(s.ctx_lens[t])
        for l in range(s.m.n_layers):
            gk, gv = s.gpu.kv_read(int(s.seq_ids[t]), l, pos, 1)
            rk, rv = s.oracle_kv_row(t, l, pos)
            assert_close(O.bf16_bits_to_f32(gk[0]), O.bf16_bits_to_f32(rk), f"k t={t} l={l} (T={T})")
            assert_close(O.bf16_bits_to_f32(gv[0]), O.bf16_bits_to_f32(rv), f"v t={t} l={l} (T={T})")
    s.gpu.close()


def test_decode_bit_identical_run_to_run():
    outs = []
    for _ in range(2):
        s = Setup(seed=2)
        logits, hidden = s.gpu.run_step_batch(s.rings, s.tokens.astype(np.uint32), s.seq_ids, want_hidden=True)
        outs.append((logits.tobytes(), hidden.tobytes()))
        s.gpu.close()
    assert outs[0] == outs[1]


def test_decode_step_large_hidden_values():
    """Hidden values in the thousands (embedding rows scaled to |x| ~ 3000):
    the folded RMSNorm's fixed-point sums of squares keep their headroom (a
    row of such values overflows int64 at a 2^32 scale), and the step still
    matches the oracle."""
    s = Setup(seed=11)
    try:
        big = O.f32_to_bf16_bits(O.bf16_bits_to_f32(s.m.embed) * 3000.0)
        s.m.embed = big
        s.gpu.load_weight(aos.W_EMBED, big)
        logits, hidden = s.gpu.run_step_batch(s.rings, s.tokens.astype(np.uint32), s.seq_ids, want_hidden=True)
        ref_logits, ref_hidden = O.decode_step(s.m, s.ad, s.rings, s.tokens, s.kv)
        assert np.abs(O.bf16_bits_to_f32(ref_hidden)).max() > 1000.0
        assert_close(O.bf16_bits_to_f32(hidden), O.bf16_bits_to_f32(ref_hidden), "hidden (large values)")
        assert_close(logits, ref_logits, "logits (large hidden values)")
    finally:
        s.gpu.close()


def test_cooperative_gemm_mode_matches_default(monkeypatch):
    """Shared-device mode (AOS_GEMM_COOPERATIVE=1 at init) launches the same
    GEMMs as cooperative grids: the step's logits and hidden state are
    bit-identical to the default launches."""
    outs = []
    for coop in ("0", "1"):
        monkeypatch.setenv("AOS_GEMM_COOPERATIVE", coop)
        s = Setup(seed=2)
        logits, hidden = s.gpu.run_step_batch(s.rings, s.tokens.astype(np.uint32), s.seq_ids, want_hidden=True)
        outs.append((logits.tobytes(), hidden.tobytes()))
        s.gpu.close()
    assert outs[0] == outs[1]


def test_two_steps_and_unload():
    s = Setup(seed=3, ctx_lens=(5, 40, 64, 200, 17, 33, 1, 250), ranks=(16, 16, 8, 8, 32))
    toks = s.tokens.astype(np.uint32)
    l1, _ = s.gpu.run_step_batch(s.rings, toks, s.seq_ids)
    r1, _ = O.decode_step(s.m, s.ad, s.rings, s.tokens, s.kv)
    assert_close(l1, r1, "step 1")
    # second step: the oracle's cache advanced by its own first step
    s.kv.ctx_lens[:] = s.ctx_lens + 1
    toks2 = s.rng.integers(0, s.m.vocab, size=s.T).astype(np.int32)
    l2, _ = s.gpu.run_step_batch(s.rings, toks2.astype(np.uint32), s.seq_ids)
    r2, _ = O.decode_step(s.m, s.ad, s.rings, toks2, s.kv)
    assert_close(l2, r2, "step 2")
    # unloading an adapter: rings that still name it skip it (backend.rs:405-418)
    s.gpu.unload_adapter(2)
    s.ad.A[2] = [[None] * 7 for _ in range(s.m.n_layers)]
    s.ad.B[2] = [[None] * 7 for _ in range(s.m.n_layers)]
    s.kv.ctx_lens[:] = s.ctx_lens + 2
    l3, _ = s.gpu.run_step_batch(s.rings, toks2.astype(np.uint32), s.seq_ids)
    r3, _ = O.decode_step(s.m, s.ad, s.rings, toks2, s.kv)
    assert_close(l3, r3, "after unload")
    s.gpu.close()


def test_config2_single_layer_full_size():
    """hidden 3584, 28/4 heads, I=18944, 32 rank-16 adapters on
    q/k/v/o, K=4, batch 32, KV length 2048."""
    rng = np.random.default_rng(22)
    H, nh, nkv, I, T, ctx = 3584, 28, 4, 18944, 32, 2048
    m = O.HostModel.random(rng, H, nh, nkv, 128, I, 256, 1, with_embed=False)
    ad = O.HostAdapters.random(rng, m, [16] * 32, modules=[0, 1, 2, 3])
    mb = (ctx + 16 + 15) // 16
    bt = np.arange(T * mb, dtype=np.int32).reshape(T, mb)
    kv = O.HostKV(m, T * mb, 16, bt, np.full(T, ctx, np.int32))
    kv.k_pool[...] = O.f32_to_bf16_bits(rng.standard_normal(kv.k_pool.shape, dtype=np.float32))
    kv.v_pool[...] = O.f32_to_bf16_bits(rng.standard_normal(kv.v_pool.shape, dtype=np.float32))
    pri = rng.standard_normal((T, 32), dtype=np.float32)
    rings, _, _, _ = O.route_batch(pri, None, k=4)
    hidden0 = O.f32_to_bf16_bits(rng.standard_normal((T, H), dtype=np.float32))
    gpu = aos.CudaKernels(H, nh, nkv, 128, I, 256, 1, max_batch=T, kv_num_blocks=T * mb + 8, max_seq_len=mb * 16,
                          lora_rank_capacity=512, lora_max_adapters=32,
                          lora_modules=["q_proj", "k_proj", "v_proj", "o_proj"])
    gpu.load_host_model(m)
    for a in range(32):
        gpu.load_adapter_with_metadata(a, 16, ad.alphas[a], {(0, mod): (ad.A[a][0][mod], ad.B[a][0][mod])
                                                              for mod in range(4)})
    sids = np.arange(T, dtype=np.uint64)
    for t in range(T):
        gpu.kv_alloc(int(sids[t]), mb * 16)
        k = kv.k_pool[0, bt[t]].transpose(0, 2, 1, 3).reshape(-1, nkv, 128)[:ctx]
        v = kv.v_pool[0, bt[t]].transpose(0, 2, 1, 3).reshape(-1, nkv, 128)[:ctx]
        gpu.kv_write(int(sids[t]), 0, 0, k, v)
        gpu.kv_set_len(int(sids[t]), ctx)
    import torch
    h = torch.from_numpy(hidden0.view(np.int16).copy()).cuda()
    rd = torch.from_numpy(rings.view(np.uint8).copy()).cuda()
    gpu.layer_step_dev(0, rd, sids, h)
    torch.cuda.synchronize()
    got = h.cpu().numpy().view(np.uint16)
    ref = hidden0.copy()
    O.layer_step(m, ad, 0, rings, kv, ref)
    assert_close(O.bf16_bits_to_f32(got), O.bf16_bits_to_f32(ref), "config-2 layer hidden")
    for t in (0, 17, 31):
        gk, gv = gpu.kv_read(int(sids[t]), 0, ctx, 1)
        blk = bt[t, ctx // 16]
        assert_close(O.bf16_bits_to_f32(gk[0]), O.bf16_bits_to_f32(kv.k_pool[0, blk, :, ctx % 16]), "config-2 k")
        assert_close(O.bf16_bits_to_f32(gv[0]), O.bf16_bits_to_f32(kv.v_pool[0, blk, :, ctx % 16]), "config-2 v")
    gpu.close()
