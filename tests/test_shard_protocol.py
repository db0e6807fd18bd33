"""The adapter-sharded exchange on CPU: two gloo ranks run the protocol of
aos_run_step_sharded_dev (adapter-os_b200/csrc/runtime.cu, shard_site) with
the oracle's fp32 LoRA op (kernel_testing.rs:220-257) as the per-owner math,
and the result must equal the unsharded op on all rows.

Protocol under test (the same layout the CUDA path uses):
  * rank r owns the adapters with id % world == r (aos.shard_owner);
  * every rank sends its T home rows to every rank; received rows are
    rank-major ([world * T][in]);
  * each owner computes the LoRA delta of its own adapters for all rows;
  * block o of the deltas (rows of rank o) goes back to rank o, which adds
    the blocks in owner order to its base output.

Tolerance: 1e-5 relative (the fp32 op bound), since only the order of the
per-adapter additions changes."""
import os
import socket

import numpy as np
import pytest

from tests.aos_import import aos

WORLD = 2
T_HOME = 5
IN, OUT, RANK, N_AD, K = 64, 48, 8, 6, 3


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _case():
    from oracle import oracle as O
    rng = np.random.default_rng(11)
    T = WORLD * T_HOME
    x = rng.standard_normal((T, IN)).astype(np.float32)
    W = (rng.standard_normal((OUT, IN)) * 0.02).astype(np.float32)
    A = (rng.standard_normal((N_AD, RANK, IN)) * 0.02).astype(np.float32)
    B = (rng.standard_normal((N_AD, OUT, RANK)) * 0.02).astype(np.float32)
    alpha = rng.uniform(4, 32, size=N_AD).astype(np.float32)
    rings, _, _, _ = O.route_batch(rng.standard_normal((T, N_AD)).astype(np.float32), None, k=K)
    return x, W, A, B, alpha, rings


def _rank_main(rank, port, out_dir):
    import torch
    import torch.distributed as dist
    from oracle import oracle as O
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=WORLD)
    x, W, A, B, alpha, rings = _case()
    home = slice(rank * T_HOME, (rank + 1) * T_HOME)
    # this rank's adapters only (others have no weights here)
    mine = np.array([aos.shard_owner(a, WORLD) == rank for a in range(N_AD)])
    A_own, B_own = A * mine[:, None, None], B * mine[:, None, None]
    # rows to every rank (rank-major on arrival); the rings travel the same way
    send = torch.from_numpy(np.concatenate([x[home]] * WORLD))
    recv = torch.empty_like(send)
    dist.all_to_all_single(recv, send)
    ring_bytes = np.ascontiguousarray(rings[home]).view(np.uint8).reshape(T_HOME, -1)
    rsend = torch.from_numpy(np.concatenate([ring_bytes] * WORLD).copy())
    rrecv = torch.empty_like(rsend)
    dist.all_to_all_single(rrecv, rsend)
    rows = recv.numpy()
    rrings = rrecv.numpy().reshape(-1).view(O.RING_DTYPE)
    # owner: LoRA of its adapters on every rank's rows (base weight zero)
    delta = O.lora_op_f32(rows, np.zeros_like(W), A_own, B_own, rrings, alpha)
    dsend = torch.from_numpy(delta.copy())
    drecv = torch.empty_like(dsend)
    dist.all_to_all_single(drecv, dsend)  # block o: deltas of this rank's rows from owner o
    base = O.lora_op_f32(x[home], W, np.zeros_like(A), np.zeros_like(B), rings[home], alpha)
    y = base.copy()
    for o in range(WORLD):  # owner order
        y += drecv.numpy()[o * T_HOME:(o + 1) * T_HOME]
    np.save(os.path.join(out_dir, f"y{rank}.npy"), y)
    dist.destroy_process_group()


def test_owner_rule():
    assert [aos.shard_owner(a, 4) for a in range(9)] == [0, 1, 2, 3, 0, 1, 2, 3, 0]
    assert all(aos.shard_owner(a, 1) == 0 for a in range(5))


def test_sharded_lora_two_gloo_ranks(tmp_path):
    import torch.multiprocessing as mp
    from oracle import oracle as O
    mp.spawn(_rank_main, args=(_free_port(), str(tmp_path)), nprocs=WORLD, join=True)
    x, W, A, B, alpha, rings = _case()
    ref = O.lora_op_f32(x, W, A, B, rings, alpha)
    assert np.abs(ref - x @ W.T).max() > 1e-3  # the LoRA term is not negligible
    for r in range(WORLD):
        y = np.load(os.path.join(tmp_path, f"y{r}.npy"))
        want = ref[r * T_HOME:(r + 1) * T_HOME]
        err = np.abs(y - want).max() / np.abs(want).max()
        assert err <= 1e-5, f"rank {r}: rel-max {err:.2e}"
