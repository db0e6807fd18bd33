"""The CPU oracle reproduces every known-answer value the reference's own
tests pin for this path (the oracle must be pinned before it is trusted)."""
import json
import os

import numpy as np
import pytest

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def test_quantize_gate_known_answers(oracle):
    # crates/adapteros-lora-router/src/quantization.rs:238-253
    assert oracle.quantize_gate(0.0) == 0
    assert oracle.quantize_gate(0.5) == 16384
    assert oracle.quantize_gate(1.0) == 32767
    assert oracle.quantize_gate(-0.5) == 0
    assert oracle.quantize_gate(1.5) == 32767
    # round half away from zero (Rust f32::round): 0.25*32767 = 8191.75 -> 8192
    assert oracle.quantize_gate(0.25) == 8192
    assert oracle.quantize_gate(float("nan")) == 0  # saturating `as i32`


def test_tie_break_stable_id_ascending(oracle):
    # crates/adapteros-lora-router/tests/determinism.rs:537-574
    rings, _, st, rc = oracle.route_batch([0.9, 0.5, 0.5, 0.5, 0.1], [10, 200, 100, 300, 400],
                                          k=3, tau=1.0, eps=0.01)
    assert rc == 0 and st[0] == 0
    r = rings[0]
    assert r["top_k"] == 3
    assert list(r["indices"][:3]) == [0, 2, 1]


def test_deterministic_top_k_ordering(oracle):
    # crates/adapteros-lora-router/tests/determinism.rs:38-86: ties broken by stable_id.
    rings, _, _, rc = oracle.route_batch([0.5, 0.5, 0.5, 0.3, 0.2], [300, 100, 200, 400, 500],
                                         k=3, tau=1.0, eps=0.01)
    assert rc == 0
    assert list(rings[0]["indices"][:3]) == [1, 2, 0]
    again, _, _, _ = oracle.route_batch([0.5, 0.5, 0.5, 0.3, 0.2], [300, 100, 200, 400, 500],
                                        k=3, tau=1.0, eps=0.01)
    assert again.tobytes() == rings.tobytes()


def test_single_adapter_full_gate(oracle):
    # tests/q15_edge_cases.rs:142-199
    rings, _, _, rc = oracle.route_batch([1.0], k=1, tau=1.0, eps=0.02)
    assert rc == 0
    assert rings[0]["top_k"] == 1 and rings[0]["gates_q15"][0] == 32767
    assert np.float32(rings[0]["gates_q15"][0]) / np.float32(32767.0) == 1.0


def test_q15_sum_near_max(oracle):
    # tests/q15_edge_cases.rs:305-380 (equal priors, K=3)
    rings, _, _, rc = oracle.route_batch([1.0, 1.0, 1.0], k=3, tau=1.0, eps=0.02)
    assert rc == 0
    g = rings[0]["gates_q15"][:3].astype(np.int32)
    assert abs(int(g.sum()) - 32767) <= 3
    assert all(x >= 0 for x in g)


def test_structural_invariants(oracle):
    # tests/router_ring_golden.rs:250-304
    pri = [0.1, 0.9, 0.5, 0.3, 0.7, 0.2, 0.8, 0.4, 0.6, 0.0]
    rings, ent, _, rc = oracle.route_batch(pri, np.zeros(10, np.uint64), k=3, tau=1.0, eps=0.02)
    assert rc == 0
    r = rings[0]
    assert r["top_k"] == 3
    idx = list(r["indices"][:3])
    assert len(set(idx)) == 3 and set(idx) == {1, 6, 4}
    assert all(0 <= g <= 32767 for g in r["gates_q15"][:3])
    assert list(r["indices"][3:]) == [0] * 5 and list(r["gates_q15"][3:]) == [0] * 5
    assert ent[0] >= 0.0


def test_nonfinite_prior_rejected(oracle):
    # validate_router_inputs (router.rs:611-625)
    for bad in (np.nan, np.inf, -np.inf):
        rings, _, st, rc = oracle.route_batch([[0.1, bad, 0.3], [0.1, 0.2, 0.3]], k=2)
        assert rc != 0 and st[0] != 0 and st[1] == 0
        assert rings[0]["top_k"] == 0


def test_k_sanitised(oracle):
    # sanitize_k (router.rs:127-144): 0 -> 1, >8 -> 8
    pri = np.linspace(0, 1, 12, dtype=np.float32)
    r0, _, _, _ = oracle.route_batch(pri, k=0)
    r9, _, _, _ = oracle.route_batch(pri, k=20)
    assert r0[0]["top_k"] == 1 and r9[0]["top_k"] == 8


def test_policy_mask_and_empty(oracle):
    # A disallowed adapter never appears; all disallowed -> empty decision.
    pri = [0.9, 0.8, 0.1]
    r, _, _, _ = oracle.route_batch(pri, k=2, allowed=[0, 1, 1])
    assert 0 not in list(r[0]["indices"][:2])
    r, _, _, rc = oracle.route_batch(pri, k=2, allowed=[0, 0, 0])
    assert rc == 0 and r[0]["top_k"] == 0


def test_softmax_kahan_and_tau_zero(oracle):
    # deterministic_softmax (router.rs:1340-1411)
    p = oracle.deterministic_softmax([2.0, 1.0, 0.5], 1.0)
    e = np.exp(np.array([2.0, 1.0, 0.5]) - 2.0)
    assert np.allclose(p, (e / e.sum()).astype(np.float32), rtol=0, atol=1e-7)
    hard = oracle.deterministic_softmax([0.1, 0.9], 0.0)
    assert list(hard) == [1.0, 0.0]


def test_liquid_blend_known_answer(oracle):
    # crates/adapteros-lora-kernel-api/src/liquid.rs:267-336 -> [2.0, 4.0] within 1e-5
    bf = lambda v: oracle.bf16_bits_to_f32(oracle.f32_to_bf16_bits(np.array(v, np.float32)))
    A1 = np.array([[1, 0], [0, 1]], np.float32)
    B1 = np.array([[1, 2], [3, 4]], np.float32)
    A2 = bf(np.ones((2, 2)))
    B2 = bf(np.full((2, 2), 0.5))
    y, rc = oracle.liquid_blend_f32(np.array([1.0, 1.0]), [A1, A2], [B1, B2], [2.0, 1.0], [0.5, 0.5], 2)
    assert rc == 0
    assert abs(y[0] - 2.0) < 1e-5 and abs(y[1] - 4.0) < 1e-5
    # validation errors (liquid.rs:164-184)
    _, rc = oracle.liquid_blend_f32(np.ones(2), [], [], [], [], 2)
    assert rc != 0


@pytest.mark.parametrize("in_dim,rank,alpha", [(4, 1, 8.0), (8, 2, 16.0), (16, 4, 32.0)])
def test_lora_formula_matches_cpu_lora_forward(oracle, in_dim, rank, alpha):
    # crates/adapteros-lora-kernel-mtl/tests/metal_lora_parity.rs:40-100: CPU formula
    # out = W x + (B (A x)) * alpha/rank, tolerance 1e-6 abs + 1e-6 rel.
    rng = np.random.default_rng(in_dim * 100 + rank)
    out_dim = in_dim
    x = rng.standard_normal((1, in_dim)).astype(np.float32)
    W = rng.standard_normal((out_dim, in_dim)).astype(np.float32)
    A = rng.standard_normal((1, rank, in_dim)).astype(np.float32)
    B = rng.standard_normal((1, out_dim, rank)).astype(np.float32)
    ring = np.zeros(1, dtype=oracle.RING_DTYPE)
    ring[0]["top_k"] = 1
    ring[0]["gates_q15"][0] = 32767  # blend weight exactly 1.0
    y = oracle.lora_op_f32(x, W, A, B, ring, alpha=np.array([alpha], np.float32))
    ref = W.astype(np.float64) @ x[0] + (B[0].astype(np.float64) @ (A[0].astype(np.float64) @ x[0])) * (alpha / rank)
    assert np.all(np.abs(y[0] - ref) <= 1e-6 + 1e-6 * np.abs(ref) + 1e-5 * np.abs(ref).max())


def test_negative_and_zero_gates_are_skipped(oracle):
    # RouterRing may carry negative gates (tests/router_ring_golden.rs:175-198);
    # the backend skips q15 <= 0 (mlx-ffi/src/backend.rs:405-418).
    rng = np.random.default_rng(7)
    x = rng.standard_normal((1, 8)).astype(np.float32)
    W = np.zeros((8, 8), np.float32)
    A = rng.standard_normal((3, 2, 8)).astype(np.float32)
    B = rng.standard_normal((3, 8, 2)).astype(np.float32)
    ring = np.zeros(1, dtype=oracle.RING_DTYPE)
    ring[0]["top_k"] = 3
    ring[0]["indices"][:3] = [0, 1, 2]
    ring[0]["gates_q15"][:3] = [16383, -8191, 0]
    y = oracle.lora_op_f32(x, W, A, B, ring, alpha=np.array([2.0, 2.0, 2.0], np.float32))
    only0 = (np.float32(16383) / np.float32(32767.0)) * (B[0] @ (A[0] @ x[0]))
    assert np.allclose(y[0], only0, rtol=1e-5, atol=1e-6)


def test_golden_router_fixture(oracle):
    """The committed fixture (made by tests/golden/make_golden.py) still matches."""
    path = os.path.join(GOLDEN, "router_cases.json")
    cases = json.load(open(path))
    for case in cases:
        pri = np.array(case["priors"], np.float32).reshape(case["T"], case["N"])
        rings, _, st, rc = oracle.route_batch(pri, np.array(case["stable_ids"], np.uint64), k=case["k"],
                                              tau=case["tau"], eps=case["eps"])
        assert rc == case["rc"], case["name"]
        for t in range(case["T"]):
            exp = case["rings"][t]
            assert int(rings[t]["top_k"]) == exp["k"], case["name"]
            assert [int(v) for v in rings[t]["indices"][: exp["k"]]] == exp["indices"], case["name"]
            assert [int(v) for v in rings[t]["gates_q15"][: exp["k"]]] == exp["gates_q15"], case["name"]
