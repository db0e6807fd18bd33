"""Sliding-window KV rotate (aos_kv_rotate) against the oracle's restatement of
kv_cache_rotate (crates/adapteros-lora-kernel-mtl/shaders/kv_cache.metal:
200-236): rows bit-exact after whole-page, in-page and mixed shifts, other
sequences untouched, a decode step on the rotated cache within the bf16
tolerance, and the argument checks."""
import numpy as np
import pytest

from oracle import oracle as O
from tests.aos_import import aos
from tests.test_decoder_gpu import Setup, assert_close

pytestmark = pytest.mark.gpu

H, NH, NKV, HD, INTER, VOCAB, L = 256, 4, 2, 128, 384, 1000, 2


def _rows(rng, n):
    return O.f32_to_bf16_bits(rng.standard_normal((n, NKV, HD), dtype=np.float32))


def test_kv_rotate_rows_bit_exact():
    rng = np.random.default_rng(41)
    m = O.HostModel.random(rng, H, NH, NKV, HD, INTER, VOCAB, L)
    gpu = aos.CudaKernels(H, NH, NKV, HD, INTER, VOCAB, L, max_batch=8, kv_num_blocks=64, max_seq_len=256,
                          lora_rank_capacity=64, lora_max_adapters=1)
    try:
        gpu.load_host_model(m)
        # a neighbour sequence on pages between the rotated one's
        gpu.kv_alloc(7, 40)
        gpu.kv_alloc(8, 200)
        nb_rows = {l: (_rows(rng, 40), _rows(rng, 40)) for l in range(L)}
        for l in range(L):
            gpu.kv_write(7, l, 0, *nb_rows[l])
        gpu.kv_set_len(7, 40)
        n = 177
        ref = {l: [_rows(rng, n), _rows(rng, n)] for l in range(L)}
        for l in range(L):
            gpu.kv_write(8, l, 0, ref[l][0], ref[l][1])
        gpu.kv_set_len(8, n)
        length = n
        for shift in (5, 16, 21, 0, 3, 32, 47):  # in-page, whole page, both, none, ...
            gpu.kv_rotate(8, shift)
            for l in range(L):
                for kv in range(2):
                    ref[l][kv], new_len = O.kv_rotate_rows(ref[l][kv], length, shift)
            length = new_len
            assert gpu.kv_len(8) == length
            for l in range(L):
                k, v = gpu.kv_read(8, l, 0, length)
                assert k.tobytes() == ref[l][0][:length].tobytes(), f"K rows after shift {shift}, layer {l}"
                assert v.tobytes() == ref[l][1][:length].tobytes(), f"V rows after shift {shift}, layer {l}"
        for l in range(L):  # the neighbour is untouched
            k, v = gpu.kv_read(7, l, 0, 40)
            assert k.tobytes() == nb_rows[l][0].tobytes() and v.tobytes() == nb_rows[l][1].tobytes()
        # appending after a rotate writes at the new length, within the kept capacity
        extra = (_rows(rng, 3), _rows(rng, 3))
        gpu.kv_write(8, 0, length, *extra)
        gpu.kv_set_len(8, length + 3)
        k, _ = gpu.kv_read(8, 0, 0, length + 3)
        assert k[:length].tobytes() == ref[0][0][:length].tobytes()
        assert k[length:].tobytes() == extra[0].tobytes()
    finally:
        gpu.close()


def test_kv_rotate_bounds():
    rng = np.random.default_rng(42)
    m = O.HostModel.random(rng, H, NH, NKV, HD, INTER, VOCAB, L)
    gpu = aos.CudaKernels(H, NH, NKV, HD, INTER, VOCAB, L, max_batch=8, kv_num_blocks=16, max_seq_len=128,
                          lora_rank_capacity=64, lora_max_adapters=1)
    try:
        gpu.load_host_model(m)
        gpu.kv_alloc(3, 50)
        gpu.kv_set_len(3, 30)
        with pytest.raises(aos.AosError):
            gpu.kv_rotate(3, 31)
        with pytest.raises(aos.AosError):
            gpu.kv_rotate(99, 1)
        gpu.kv_rotate(3, 30)
        assert gpu.kv_len(3) == 0
    finally:
        gpu.close()


def _rotate_oracle_seq(kv, t, n_layers, shift):
    """Rotate sequence t of an oracle HostKV in place (its own block table)."""
    length = int(kv.ctx_lens[t])
    pos = np.arange(length)
    blk, row = kv.block_tables[t, pos // 16], pos % 16
    for l in range(n_layers):
        for pool in (kv.k_pool, kv.v_pool):
            rows = pool[l, blk, :, row, :]  # [length, n_kv, hd]
            new_rows, new_len = O.kv_rotate_rows(rows, length, shift)
            pool[l, blk[:new_len], :, row[:new_len], :] = new_rows[:new_len]
    kv.ctx_lens[t] = length - shift


def test_decode_after_rotate_matches_oracle():
    s = Setup(seed=43, ctx_lens=(0, 1, 15, 40, 300))
    try:
        for t, shift in ((3, 16), (4, 37)):
            s.gpu.kv_rotate(int(s.seq_ids[t]), shift)
            _rotate_oracle_seq(s.kv, t, s.m.n_layers, shift)
        logits, hidden = s.gpu.run_step_batch(s.rings, s.tokens.astype(np.uint32), s.seq_ids, want_hidden=True)
        ref_logits, ref_hidden = O.decode_step(s.m, s.ad, s.rings, s.tokens, s.kv)
        assert_close(O.bf16_bits_to_f32(hidden), O.bf16_bits_to_f32(ref_hidden), "hidden after rotate")
        assert_close(logits, ref_logits, "logits after rotate")
    finally:
        s.gpu.close()
