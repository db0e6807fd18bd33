"""Adapter-sharded decode step (aos_run_step_sharded_dev) on 2 GPUs vs the CPU
oracle's unsharded step (oracle/aos_oracle.cpp, mlx_cpp_wrapper_real.cpp:3338-3559).

Two ranks, one GPU each.  Both build the same seeded model, adapters, KV
cache and routing; rank r keeps the adapters with id % 2 == r and decodes the
home tokens [r*T, (r+1)*T).  Every LoRA term crosses the NCCL exchange: rows
go to the owner, bf16 deltas come back and are added in owner order.  The
oracle decodes all 2*T tokens with every adapter on one host.

Tolerance (bf16 path): relative L2 error <= 2e-2 and max-abs error <= 2e-2 *
max|ref| for logits and the final hidden state.  The sharded step must also
be bit-identical run to run.  Skipped without two GPUs."""
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TOL = 2e-2
WORLD = 2
T_HOME = 6


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def make_case(seed=5, hidden=256, nh=4, nkv=2, inter=384, vocab=1000, L=2, n_ad=10, rank=16, K=4, max_seq=256):
    """Host-side model, adapters, KV and routing of 2*T_HOME tokens (same on every rank)."""
    from oracle import oracle as O
    rng = np.random.default_rng(seed)
    m = O.HostModel.random(rng, hidden, nh, nkv, 128, inter, vocab, L)
    ad = O.HostAdapters.random(rng, m, [rank] * n_ad, modules=list(range(7)))
    T = WORLD * T_HOME
    ctx = rng.integers(1, 120, size=T).astype(np.int32)
    mb = (max_seq + 15) // 16
    bt = np.arange(T * mb, dtype=np.int32).reshape(T, mb)
    kv = O.HostKV(m, T * mb, 16, bt, ctx.copy())
    kv.k_pool[...] = O.f32_to_bf16_bits(rng.standard_normal(kv.k_pool.shape, dtype=np.float32))
    kv.v_pool[...] = O.f32_to_bf16_bits(rng.standard_normal(kv.v_pool.shape, dtype=np.float32))
    pri = rng.standard_normal((T, n_ad), dtype=np.float32)
    rings, _, _, _ = O.route_batch(pri, None, k=K)
    tokens = rng.integers(0, vocab, size=T).astype(np.int32)
    return dict(m=m, ad=ad, kv=kv, ctx=ctx, bt=bt, rings=rings, tokens=tokens, max_seq=max_seq, n_ad=n_ad)


def _rank_main(rank, port, out_dir):
    import torch
    import torch.distributed as dist
    from tests.aos_import import aos
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=WORLD)
    torch.cuda.set_device(rank)
    cs = make_case()
    m, ad, kv = cs["m"], cs["ad"], cs["kv"]
    home = slice(rank * T_HOME, (rank + 1) * T_HOME)
    mb = cs["bt"].shape[1]
    gpu = aos.CudaKernels(m.hidden, m.n_heads, m.n_kv_heads, 128, m.inter, m.vocab, m.n_layers,
                          max_batch=WORLD * T_HOME, kv_num_blocks=T_HOME * mb + 8, max_seq_len=cs["max_seq"],
                          lora_rank_capacity=cs["n_ad"] * 16, lora_max_adapters=cs["n_ad"], device=rank)
    gpu.load_host_model(m)
    for a in range(ad.n):
        if aos.shard_owner(a, WORLD) != rank:
            continue
        gpu.load_adapter_with_metadata(a, ad.ranks[a], ad.alphas[a],
                                       {(l, mod): (ad.A[a][l][mod], ad.B[a][l][mod])
                                        for l in range(m.n_layers) for mod in range(7)})
    sids = np.arange(1000 + home.start, 1000 + home.stop, dtype=np.uint64)
    for i, t in enumerate(range(home.start, home.stop)):
        n = int(cs["ctx"][t])
        gpu.kv_alloc(int(sids[i]), cs["max_seq"])
        for l in range(m.n_layers):
            k = kv.k_pool[l, cs["bt"][t]].transpose(0, 2, 1, 3).reshape(-1, m.n_kv_heads, 128)[:n]
            v = kv.v_pool[l, cs["bt"][t]].transpose(0, 2, 1, 3).reshape(-1, m.n_kv_heads, 128)[:n]
            gpu.kv_write(int(sids[i]), l, 0, k, v)
        gpu.kv_set_len(int(sids[i]), n)
    uid = [aos.shard_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(uid, src=0)
    gpu.shard_init(rank, WORLD, uid[0])
    dev = f"cuda:{rank}"
    rings = torch.from_numpy(cs["rings"][home].view(np.uint8).copy()).to(dev)
    toks = torch.from_numpy(cs["tokens"][home].astype(np.int32)).to(dev)
    outs = []
    for rep in range(2):  # the second run repeats the first from the same cache state
        logits = torch.empty((T_HOME, m.vocab), dtype=torch.float32, device=dev)
        hidden = torch.empty((T_HOME, m.hidden), dtype=torch.int16, device=dev)
        gpu.run_step_sharded_dev(rings, toks, sids, logits=logits, hidden=hidden)
        torch.cuda.synchronize()
        outs.append((logits.cpu().numpy(), hidden.cpu().numpy().view(np.uint16)))
        for i, t in enumerate(range(home.start, home.stop)):
            gpu.kv_set_len(int(sids[i]), int(cs["ctx"][t]))
    gpu.health_check()
    np.savez(os.path.join(out_dir, f"rank{rank}.npz"), logits0=outs[0][0], hidden0=outs[0][1],
             logits1=outs[1][0], hidden1=outs[1][1])
    dist.barrier()
    gpu.close()
    dist.destroy_process_group()


def test_sharded_step_two_gpus(tmp_path):
    import torch
    if torch.cuda.device_count() < WORLD:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    from oracle import oracle as O
    from tests.test_decoder_gpu import assert_close
    mp.spawn(_rank_main, args=(_free_port(), str(tmp_path)), nprocs=WORLD, join=True)
    cs = make_case()
    ref_logits, ref_hidden = O.decode_step(cs["m"], cs["ad"], cs["rings"], cs["tokens"], cs["kv"])
    for r in range(WORLD):
        z = np.load(os.path.join(tmp_path, f"rank{r}.npz"))
        home = slice(r * T_HOME, (r + 1) * T_HOME)
        assert z["logits0"].tobytes() == z["logits1"].tobytes(), f"rank {r}: logits differ run to run"
        assert z["hidden0"].tobytes() == z["hidden1"].tobytes(), f"rank {r}: hidden differs run to run"
        assert_close(O.bf16_bits_to_f32(z["hidden0"]), O.bf16_bits_to_f32(ref_hidden[home]), f"rank {r} hidden")
        assert_close(z["logits0"], ref_logits[home], f"rank {r} logits")
