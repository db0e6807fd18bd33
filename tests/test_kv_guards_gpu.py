"""KvCache generation guards and zeroization (crates/adapteros-lora-worker/
src/kvcache.rs:288-402, 586-733) on the paged device cache: a generation
change releases every sequence and zeroes the pools; guarded allocation,
stale-guard detection and draining follow the reference; zeroize_sequence
clears one sequence's K/V pages in every layer and leaves the others."""
import numpy as np
import pytest

from oracle import oracle as O
from tests.aos_import import aos

pytestmark = pytest.mark.gpu


def make():
    return aos.CudaKernels(256, 2, 1, 128, 384, 512, 2, max_batch=8, kv_num_blocks=32, max_seq_len=64,
                           lora_rank_capacity=64, lora_max_adapters=2)


def fill(g, sid, n, rng):
    for l in range(2):
        k = O.f32_to_bf16_bits(rng.standard_normal((n, 1, 128), dtype=np.float32))
        v = O.f32_to_bf16_bits(rng.standard_normal((n, 1, 128), dtype=np.float32))
        g.kv_write(sid, l, 0, k, v)
    g.kv_set_len(sid, n)


def test_generation_guards_and_zeroize():
    rng = np.random.default_rng(0)
    g = make()
    try:
        assert g.generation() == 0
        g.allocate_with_guard(1, 40, 0)
        g.allocate_with_guard(2, 40, 0)
        fill(g, 1, 33, rng)
        fill(g, 2, 20, rng)
        assert not g.has_active_sequences_with_generation(0)
        assert g.has_active_sequences_with_generation(7)
        # zeroize one sequence: its rows are zero in every layer, the other's are not
        g.zeroize_sequence(1)
        for l in range(2):
            k, v = g.kv_read(1, l, 0, 33)
            assert not k.any() and not v.any()
            k2, _ = g.kv_read(2, l, 0, 20)
            assert k2.any()
        assert g.kv_len(1) == 33  # still allocated
        # same generation: nothing happens
        assert not g.ensure_cache_coherence(0)
        assert g.kv_len(2) == 20
        # a new generation releases everything and zeroes the pools
        assert g.ensure_cache_coherence(5)
        assert g.generation() == 5
        with pytest.raises(aos.AosError):
            g.kv_len(2)
        g.allocate_with_guard(3, 40, 5)
        g.kv_set_len(3, 40)
        k, v = g.kv_read(3, 0, 0, 40)
        assert not k.any() and not v.any()
        # allocating under another generation resets first
        g.allocate_with_guard(4, 40, 6)
        with pytest.raises(aos.AosError):
            g.kv_len(3)
        g.kv_alloc(9, 16)  # unguarded: not drained
        assert g.drain_active_sequences() == 1
        assert g.kv_len(9) == 0
        with pytest.raises(aos.AosError, match="not found"):
            g.zeroize_sequence(4)
        g.zeroize_all()
        with pytest.raises(aos.AosError):
            g.kv_len(9)
    finally:
        g.close()


def test_memory_report():
    rng = np.random.default_rng(1)
    g = make()
    try:
        m = O.HostModel.random(rng, 256, 2, 1, 128, 384, 512, 2)
        ad = O.HostAdapters.random(rng, m, [8, 16], modules=range(7))
        for a in range(2):
            g.load_adapter_with_metadata(a, ad.ranks[a], ad.alphas[a],
                                         {(l, mod): (ad.A[a][l][mod], ad.B[a][l][mod]) for l in range(2) for mod in range(7)})
        g.kv_alloc(5, 40)
        rep = g.memory_report()
        per_col = 2 * sum(i + o for o, i in (m.mod_shape(k) for k in range(7))) * 2
        assert rep["adapter_count"] == 2
        assert rep["adapter_allocations"] == [(0, 8 * per_col), (1, 16 * per_col)]
        assert rep["adapter_vram_total"] == 24 * per_col == rep["arena_used_bytes"]
        assert rep["kv_used_bytes"] == rep["kv_pool_bytes"] // 32 * 3  # 40 tokens -> 3 blocks of 16
        assert 0 < rep["used_gpu_bytes"] <= rep["total_gpu_bytes"]
    finally:
        g.close()
