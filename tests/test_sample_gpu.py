"""Next-token sampling on the GPU (aos_sample_dev) against the oracle's
restatement of Generator (crates/adapteros-lora-worker/src/generation.rs:
321-490): the chosen token must be identical for the same logits and draw u.

Cases: greedy on the reference's own known answer (generation.rs:497-505),
ties, NaN and -inf logits; full-vocabulary rows (V = 128256) with plain
temperature sampling, top-k (below, inside and above one 2048-key chunk,
k = 0, k >= V), top-p alone on peaked and on flat rows (the flat ones walk
tens of chunks), top-k + top-p, heavily tied (quantised) logits, and draws at
0, near 1 and in between."""
import numpy as np
import pytest

from oracle import oracle as O
from tests.aos_import import aos

pytestmark = pytest.mark.gpu


def gpu_sample(x, u=None, **kw):
    import torch
    xt = torch.tensor(np.ascontiguousarray(x, np.float32), device="cuda")
    ut = torch.tensor(np.asarray(u, np.float32), device="cuda") if u is not None else None
    out = aos.sample_dev(xt, ut, **kw)
    torch.cuda.synchronize()
    return out.cpu().numpy().astype(np.uint32)


def test_greedy_known_answers_and_edges():
    x = np.array([[0.1, 0.5, 0.3, 0.8, 0.2]], np.float32)
    assert gpu_sample(x, greedy=True)[0] == 3  # generation.rs test_greedy_sampling
    cases = np.array([[1.0, 1.0, 0.5, 0.0, 0.0],            # tie: the later index
                      [1.0, np.nan, 0.5, 0.2, 0.7],          # NaN resets the fold
                      [3.0, 2.0, 1.0, 0.0, np.nan],          # NaN last
                      [-np.inf] * 5,                          # all -inf: the last
                      [np.inf, 0.0, np.inf, 1.0, -1.0]], np.float32)
    assert list(gpu_sample(cases, greedy=True)) == list(O.sample(cases, greedy=True))
    rng = np.random.default_rng(0)
    big = rng.standard_normal((16, 128256)).astype(np.float32)
    big[3, 1000] = big[3, 2000] = big[3].max() + 1
    assert list(gpu_sample(big, greedy=True)) == list(O.sample(big, greedy=True))


CONFIGS = [
    dict(),
    dict(temperature=0.7),
    dict(top_k=50),
    dict(top_k=50, top_p=0.9, temperature=0.8),
    dict(top_k=5000),
    dict(top_k=2048),
    dict(top_k=0),
    dict(top_k=200000),
    dict(top_p=0.9),
    dict(top_p=1.0),
    dict(top_p=0.0),
]


@pytest.mark.parametrize("cfg", CONFIGS, ids=[str(c) for c in CONFIGS])
def test_sampling_matches_oracle(cfg):
    rng = np.random.default_rng(hash(str(cfg)) & 0xFFFF)
    T, V = 8, 128256
    x = (rng.standard_normal((T, V)) * 3.0).astype(np.float32)
    u = rng.random(T).astype(np.float32)
    u[0], u[1] = 0.0, np.float32(1.0 - 2.0 ** -24)
    got = gpu_sample(x, u, **cfg)
    want = O.sample(x, u, **cfg)
    assert list(got) == list(want)


def test_wide_logits_reach_subnormal_probabilities():
    rng = np.random.default_rng(10)
    T, V = 8, 128256
    x = (rng.standard_normal((T, V)) * 40.0).astype(np.float32)  # exp(l - max) down to 0 through the subnormals
    u = rng.random(T).astype(np.float32)
    for cfg in (dict(), dict(top_k=3000), dict(top_p=0.999999)):
        assert list(gpu_sample(x, u, **cfg)) == list(O.sample(x, u, **cfg)), cfg


def test_top_p_on_flat_rows_walks_many_chunks():
    rng = np.random.default_rng(7)
    T, V = 4, 128256
    x = (rng.standard_normal((T, V)) * 0.05).astype(np.float32)  # near uniform: ~115K tokens inside p = 0.9
    u = rng.random(T).astype(np.float32)
    assert list(gpu_sample(x, u, top_p=0.9)) == list(O.sample(x, u, top_p=0.9))


def test_ties_and_small_vocabularies():
    rng = np.random.default_rng(8)
    for V in (1, 2, 5, 1000, 4099):
        x = np.round(rng.standard_normal((6, V)) * 2) / 2  # many equal logits
        x = x.astype(np.float32)
        u = rng.random(6).astype(np.float32)
        for cfg in (dict(), dict(top_k=3), dict(top_k=100, top_p=0.8), dict(top_p=0.5, temperature=1.3)):
            assert list(gpu_sample(x, u, **cfg)) == list(O.sample(x, u, **cfg)), (V, cfg)


def test_generator_mirror_is_deterministic():
    import torch
    g1 = aos.Generator.new_deterministic(b"test-deterministic-generation!!!", "inference").with_top_k(20)
    g2 = aos.Generator.new_deterministic(b"test-deterministic-generation!!!", "inference").with_top_k(20)
    logits = torch.tensor([[1.0, 2.0, 3.0, 4.0, 5.0]], device="cuda")
    for step in range(5):
        g1.reseed_for_step(step)
        g2.reseed_for_step(step)
        assert g1.next_token(logits) == g2.next_token(logits)
    uni = torch.ones((1, 5), device="cuda")
    toks = set()
    for step in range(10):
        g1.reseed_for_step(step)
        toks.add(g1.next_token(uni))
    assert len(toks) > 1  # generation.rs test_step_seeding_produces_different_results_per_step


def test_generate_tokens_loop():
    """The batched generation loop equals the same steps written out by hand
    (routing with uniform priors at position len - 1, one decode step, the
    generator's draw), stops a sequence at EOS, and caches the prompt."""
    import torch
    rng = np.random.default_rng(9)
    m = O.HostModel.random(rng, 256, 2, 1, 128, 384, 512, 2)
    ad = O.HostAdapters.random(rng, m, [8, 16, 8, 8], modules=range(7))

    def make():
        g = aos.CudaKernels(m.hidden, m.n_heads, m.n_kv_heads, 128, m.inter, m.vocab, m.n_layers, max_batch=8,
                            kv_num_blocks=64, max_seq_len=128, lora_rank_capacity=128, lora_max_adapters=4)
        g.load_host_model(m)
        for a in range(4):
            g.load_adapter_with_metadata(a, ad.ranks[a], ad.alphas[a],
                                         {(l, mod): (ad.A[a][l][mod], ad.B[a][l][mod])
                                          for l in range(2) for mod in range(7)})
        return g

    prompts = [[5, 17, 33], [7], [100, 2, 3, 4, 5]]
    gens = lambda: [aos.Generator.new_deterministic(bytes([i]) * 32, "inference").with_top_k(40).with_temperature(0.9)
                    for i in range(3)]
    g = make()
    try:
        out = g.generate_tokens(gens(), list(range(4)), prompts, 6, eos_token=10**9, seq_ids=[11, 12, 13], k=2)
    finally:
        g.close()
    # by hand
    g = make()
    try:
        gs = gens()
        toks = [list(p) for p in prompts]
        for s, t in zip([11, 12, 13], toks):
            g.kv_alloc(s, len(t) + 6)
        pos = [p for t in toks for p in range(len(t) - 1)]
        rings, _, _, _ = O.route_batch(np.full((len(pos), 4), np.float32(0.25)), np.arange(4, dtype=np.uint64),
                                       k=2, positions=np.array(pos, np.uint32))
        ids = torch.tensor([x for t in toks for x in t[:-1]], dtype=torch.int32, device="cuda")
        g.prefill_dev([11, 13], [len(toks[0]) - 1, len(toks[2]) - 1],  # the one-token prompt has nothing to cache
                      torch.tensor(rings.view(np.uint8), device="cuda"), ids,
                      stream=torch.cuda.current_stream().cuda_stream)
        torch.cuda.synchronize()
        for step in range(6):
            for q in gs:
                q.reseed_for_step(step)
            pos = np.array([len(t) - 1 for t in toks], np.uint32)
            rings, _, _, _ = O.route_batch(np.full((3, 4), np.float32(0.25)), np.arange(4, dtype=np.uint64), k=2,
                                           positions=pos)
            logits, _ = g.run_step_batch(rings, np.array([t[-1] for t in toks], np.uint32),
                                         np.array([11, 12, 13], np.uint64))
            lt = torch.tensor(logits, device="cuda")
            nxt = gs[0].next_tokens_dev(lt, gs).cpu().numpy()
            for t, x in zip(toks, nxt):
                t.append(int(x))
    finally:
        g.close()
    assert all(len(o) == len(p) + 6 for o, p in zip(out, prompts))
    assert out == toks
    g = make()
    try:
        first = out[1][1]
        stop = g.generate_tokens(gens(), list(range(4)), prompts, 6, eos_token=first, seq_ids=[11, 12, 13], k=2)
        assert stop[1] == prompts[1]  # drew EOS at step 0: nothing appended
        for i in (0, 2):  # step 0 runs the same batch, so the same draws
            n0 = len(prompts[i])
            if out[i][n0] == first:
                assert stop[i] == prompts[i]
            else:
                assert stop[i][:n0 + 1] == out[i][:n0 + 1]
    finally:
        g.close()
