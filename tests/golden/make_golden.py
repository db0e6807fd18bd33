"""Regenerate tests/golden/router_cases.json from the pinned CPU oracle.

The oracle is pinned by the reference's own known-answer tests
(tests/test_oracle_golden.py); this script freezes its outputs on a set of
small inputs so that later changes to either side show up as a diff.
Run:  python tests/golden/make_golden.py
"""
import json
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)
from oracle import oracle  # noqa: E402


def case(name, priors, stable_ids, k, tau=1.0, eps=0.02):
    pri = np.array(priors, np.float32)
    if pri.ndim == 1:
        pri = pri[None, :]
    T, N = pri.shape
    rings, _, _, rc = oracle.route_batch(pri, np.array(stable_ids, np.uint64), k=k, tau=tau, eps=eps)
    return {
        "name": name, "T": T, "N": N, "k": k, "tau": tau, "eps": eps,
        "priors": [float(v) for v in pri.ravel()],
        "stable_ids": [int(v) for v in stable_ids], "rc": int(rc),
        "rings": [{"k": int(r["top_k"]), "indices": [int(v) for v in r["indices"][: r["top_k"]]],
                   "gates_q15": [int(v) for v in r["gates_q15"][: r["top_k"]]]} for r in rings],
    }


def main():
    cases = [
        case("determinism_rs_537", [0.9, 0.5, 0.5, 0.5, 0.1], [10, 200, 100, 300, 400], 3, eps=0.01),
        case("determinism_rs_38", [0.5, 0.5, 0.5, 0.3, 0.2], [300, 100, 200, 400, 500], 3, eps=0.01),
        case("ring_golden_250", [0.1, 0.9, 0.5, 0.3, 0.7, 0.2, 0.8, 0.4, 0.6, 0.0], [0] * 10, 3),
        case("single", [1.0], [0], 1),
        case("equal3", [1.0, 1.0, 1.0], [0, 1, 2], 3),
        case("neg_zero_vs_zero", [-0.0, 0.0, -1.0], [5, 1, 0], 2),
    ]
    rng = np.random.default_rng(20260101)
    # config-1 shape: 64 tokens x 8 adapters, K=2, logits ~N(0,1)
    cases.append(case("config1_64x8_k2", rng.standard_normal((64, 8)).astype(np.float32),
                      list(range(8)), 2))
    # forced ties: logits drawn from a tiny set
    tied = rng.integers(-2, 3, size=(32, 16)).astype(np.float32) * 0.5
    cases.append(case("forced_ties_32x16_k4", tied, list(rng.permutation(16)), 4))
    # K=8 of 128 with temperature 0.7
    cases.append(case("k8_of_128_tau07", rng.standard_normal((16, 128)).astype(np.float32),
                      list(range(128)), 8, tau=0.7, eps=0.05))
    out = os.path.join(os.path.dirname(os.path.abspath(__file__)), "router_cases.json")
    with open(out, "w") as f:
        json.dump(cases, f, indent=1)
    print(f"wrote {len(cases)} cases to {out}")


if __name__ == "__main__":
    main()
