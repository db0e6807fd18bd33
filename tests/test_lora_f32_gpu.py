"""fp32 LoRA op (config 1) vs the oracle: within 1e-5 relative (max-norm)."""
import numpy as np
import pytest

from tests.aos_import import aos

pytestmark = pytest.mark.gpu

TOL = 1e-5  # fp32 op tolerance from the hot-path contract


def _config1(seed=0, T=64, H=2048, N=8, r=16, K=2):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((T, H), dtype=np.float32)
    W = (rng.standard_normal((H, H), dtype=np.float32) * 0.02).astype(np.float32)
    A = (rng.standard_normal((N, r, H), dtype=np.float32) * 0.02).astype(np.float32)
    B = (rng.standard_normal((N, H, r), dtype=np.float32) * 0.02).astype(np.float32)
    logits = rng.standard_normal((T, N), dtype=np.float32)
    return x, W, A, B, logits, K


def _check(oracle, x, W, A, B, rings, alpha=None):
    ref = oracle.lora_op_f32(x, W, A, B, rings, alpha=alpha)
    got = aos.lora_op_f32(x, W, A, B, rings, alpha=alpha)
    err = np.abs(got - ref).max() / max(np.abs(ref).max(), 1e-30)
    assert err <= TOL, err
    return got


def test_config1_route_then_lora(oracle):
    x, W, A, B, logits, K = _config1()
    rings, _, _ = aos.route_batch(logits, k=K, tau=1.0, eps=0.02)
    o_rings, _, _, _ = oracle.route_batch(logits, None, k=K, tau=1.0, eps=0.02)
    assert rings.tobytes() == o_rings.tobytes()
    _check(oracle, x, W, A, B, rings)  # config 1 has no alpha/r: alpha = rank


def test_lora_alpha_ragged_and_skips(oracle):
    rng = np.random.default_rng(11)
    T, H, O, N, r = 37, 256, 96, 5, 8
    x = rng.standard_normal((T, H), dtype=np.float32)
    W = rng.standard_normal((O, H), dtype=np.float32) * 0.05
    A = rng.standard_normal((N, r, H), dtype=np.float32) * 0.05
    B = rng.standard_normal((N, O, r), dtype=np.float32) * 0.05
    rings = np.zeros(T, aos.RING_DTYPE)
    for t in range(T):
        k = t % 5
        rings[t]["top_k"] = k
        rings[t]["indices"][:k] = rng.choice(N, size=k, replace=False)
        rings[t]["gates_q15"][:k] = rng.integers(-2000, 32767, size=k)
    rings[0]["gates_q15"][0] = 0
    alpha = np.array([1.0, 8.0, 16.0, 4.0, 2.0], np.float32)
    _check(oracle, x, W, A, B, rings, alpha)


def test_lora_bit_identical_run_to_run():
    x, W, A, B, logits, K = _config1(seed=3)
    rings, _, _ = aos.route_batch(logits, k=K)
    a = aos.lora_op_f32(x, W, A, B, rings)
    b = aos.lora_op_f32(x, W, A, B, rings)
    assert a.tobytes() == b.tobytes()
