"""Batched CUDA router vs the CPU oracle: selections and Q15 gates bit-exact
(router.rs:1567-1952), entropy within 1e-6."""
import numpy as np
import pytest

from tests.aos_import import aos

pytestmark = pytest.mark.gpu


def _cmp(oracle, priors, sids=None, **kw):
    o_r, o_e, o_s, o_rc = oracle.route_batch(priors, sids, **kw)
    g_r, g_e, g_s = aos.route_batch(priors, sids, raise_on_nonfinite=False, **kw)
    assert np.array_equal(o_s, g_s)
    assert o_r.tobytes() == g_r.tobytes(), "ring bytes differ"
    assert np.allclose(o_e, g_e, rtol=0, atol=1e-6)
    return g_r


def test_router_config1_bit_exact(oracle):
    rng = np.random.default_rng(1)
    pri = rng.standard_normal((64, 8)).astype(np.float32)
    _cmp(oracle, pri, np.arange(8), k=2, tau=1.0, eps=0.02)


@pytest.mark.parametrize("N,K,T", [(32, 4, 32), (128, 4, 64), (64, 4, 4096), (1024, 8, 256)])
def test_router_configs_bit_exact(oracle, N, K, T):
    rng = np.random.default_rng(N * 7 + K)
    pri = rng.standard_normal((T, N)).astype(np.float32)
    sids = rng.permutation(N).astype(np.uint64)
    _cmp(oracle, pri, sids, k=K, tau=1.0, eps=0.02)


def test_router_forced_ties_and_signed_zero(oracle):
    rng = np.random.default_rng(3)
    pri = (rng.integers(-2, 3, size=(2048, 16)) * 0.5).astype(np.float32)
    pri[::7, 0] = -0.0
    pri[::5, 1] = 0.0
    sids = rng.integers(0, 4, size=16).astype(np.uint64)  # duplicate stable ids too
    _cmp(oracle, pri, sids, k=8, tau=0.5, eps=0.1)


def test_router_params_sanitised(oracle):
    rng = np.random.default_rng(4)
    pri = rng.standard_normal((64, 20)).astype(np.float32)
    for kw in ({"k": 0}, {"k": 12}, {"tau": 0.0}, {"tau": -1.0}, {"tau": float("nan")},
               {"eps": 2.0}, {"eps": float("inf")}, {"routing_bias": -3.0}, {"routing_bias": 2.5}):
        _cmp(oracle, pri, None, **kw)


def test_router_version_weights_mask_positions(oracle):
    rng = np.random.default_rng(5)
    pri = rng.standard_normal((256, 40)).astype(np.float32)
    vw = rng.uniform(-1, 3, size=40).astype(np.float32)
    vw[3] = np.nan
    vw[4] = -0.0
    allowed = (rng.random(40) > 0.3).astype(np.uint8)
    pos = np.arange(256, dtype=np.uint32) * 3
    _cmp(oracle, pri, None, k=4, version_weights=vw, allowed=allowed, positions=pos)
    _cmp(oracle, pri, None, k=4, allowed=np.zeros(40, np.uint8))  # everything masked -> empty


def test_router_nonfinite_rejected(oracle):
    pri = np.ones((8, 16), np.float32)
    pri[2, 5] = np.nan
    pri[6, 0] = np.inf
    _cmp(oracle, pri, None, k=4)
    with pytest.raises(aos.AosError):
        aos.route_batch(pri, k=4)


def test_router_large_sample_mismatch_rate(oracle):
    """f64 exp differs between libm and CUDA in rare last-ulp cases; measure it
    over a million tokens (the bar is zero mismatches)."""
    rng = np.random.default_rng(6)
    T, N = 1 << 20, 128
    pri = rng.standard_normal((T, N), dtype=np.float32)
    o_r, _, _, _ = oracle.route_batch(pri, None, k=4)
    g_r, _, _ = aos.route_batch(pri, None, k=4)
    mism = np.count_nonzero(o_r.view(np.uint8).reshape(T, 40) != g_r.view(np.uint8).reshape(T, 40), axis=1)
    assert int(np.count_nonzero(mism)) == 0


def test_router_run_to_run_identical():
    rng = np.random.default_rng(8)
    pri = rng.standard_normal((4096, 128)).astype(np.float32)
    a, _, _ = aos.route_batch(pri, k=4)
    b, _, _ = aos.route_batch(pri, k=4)
    assert a.tobytes() == b.tobytes()
