#!/usr/bin/env python
"""Decode throughput of adapter-os's per-token hot path on B200.

Workload: 32-layer Llama-3-8B-shaped decoder, bf16,
random-init weights; 128 LoRA adapters with ranks uniform in {8,16,32,64} on
q/k/v/o/gate/up/down (alpha = 2r); per-token K=4 routing from N(0,1) gate
logits; decode batch 64 (one token per sequence); paged KV (block 16) with
context lengths uniform in [512, 4096].  One step = route the batch (batched
CUDA router) + one decode step (embedding -> 32 layers -> lm_head logits).

``value``  : tok/s with every input resident in HBM (device entry points),
             CUDA events on the library's stream, max over ranks.
``e2e``    : the same metric through the host-pointer C ABI calls a caller
             makes (aos_route_batch + aos_run_step_batch): priors/tokens/page
             tables go host->device and full-vocab f32 logits come back every step.
``--impl reference`` times the reference's CPU path (the C++ restatement in
oracle/, as the Rust reference cannot be built here) on the host cores.
Multi-GPU: one process per GPU (torchrun), request-batch data parallel
replicas, no collective on the data path ("scaling": "weak").
"""
from __future__ import annotations

import argparse
import importlib
import json
import os
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

CFG = dict(hidden=4096, n_heads=32, n_kv_heads=8, head_dim=128, intermediate=14336, vocab=128256, n_layers=32,
           n_adapters=128, ranks=(8, 16, 32, 64), K=4, batch=64, ctx_lo=512, ctx_hi=4096)
METRIC = "decode tok/s, 8B-shape, K=4 of 128 LoRAs; LoRA+attn % of HBM roofline"
# DRAM bytes (read + write) of one layer's four GEMM launches of this workload
# (q/k/v 199.0 MB, o 100.0 MB, gate/up 519.0 MB, down 261.9 MB), from an ncu
# capture (dram__bytes_read.sum + dram__bytes_write.sum) of the 2-layer case.
GEMM_DRAM_BYTES_PER_LAYER = 1079.93e6
SEED = 20261201


def log(*a):
    print(*a, file=sys.stderr, flush=True)


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


# ------------------------------------------------------------------ clocks
class ClockSampler:
    """SM clock and throttle reasons sampled during the timed region: NVML
    polled every 10 ms by a thread (reads only), or nvidia-smi -lms 50 where
    NVML is missing."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    REASONS = (("hw_slowdown", 0x8), ("hw_thermal_slowdown", 0x40), ("sw_thermal_slowdown", 0x20),
               ("sw_power_cap", 0x4))

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.nvml = None
        self.lines = []
        self.samples = []  # (sm MHz, max MHz, reason bits)
        self.stop_ev = threading.Event()

    def start(self):
        try:
            import pynvml
            pynvml.nvmlInit()
            h = pynvml.nvmlDeviceGetHandleByIndex(self.index)
            get_reasons = getattr(pynvml, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                pynvml.nvmlDeviceGetCurrentClocksThrottleReasons
            mx = pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM)
            self.nvml = pynvml

            def poll():
                while not self.stop_ev.is_set():
                    try:
                        self.samples.append((pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM), mx, get_reasons(h)))
                    except Exception:
                        pass
                    self.stop_ev.wait(0.01)

            self.samples.append((pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM), mx, get_reasons(h)))
            self.t = threading.Thread(target=poll, daemon=True)
            self.t.start()
            return
        except Exception:
            self.nvml = None
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                          "-i", str(self.index), "-lms", "50"], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.nvml is not None:
            self.stop_ev.set()
            self.t.join(timeout=2)
            sm = [float(a) for a, _, _ in self.samples]
            mx = max((float(b) for _, b, _ in self.samples), default=0.0)
            reasons = {n for n, bit in self.REASONS for _, _, r in self.samples if r & bit}
            try:
                self.nvml.nvmlShutdown()
            except Exception:
                pass
            return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": mx or None,
                    "reasons": sorted(reasons), "samples": len(sm), "source": "nvml, 10 ms"}
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        sm, mx, reasons = [], 0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = max(mx, float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": mx or None,
                "reasons": sorted(reasons), "samples": len(sm), "source": "nvidia-smi, 50 ms"}


# ------------------------------------------------------------------ model setup
def ranks_of(rng):
    return rng.choice(np.array(CFG["ranks"]), size=CFG["n_adapters"])


def ctx_lens_of(rng, B):
    return rng.integers(CFG["ctx_lo"], CFG["ctx_hi"] + 1, size=B)


def module_shapes():
    """(out, in) of q, k, v, o, gate, up, down."""
    c = CFG
    H, I = c["hidden"], c["intermediate"]
    QD, KVD = c["n_heads"] * 128, c["n_kv_heads"] * 128
    return [(QD, H), (KVD, H), (KVD, H), (H, QD), (I, H), (I, H), (H, I)]


def load_base(gpu, aos, torch, device, layers):
    """Random-init base weights (seeded); returns the seeded bf16 generator used."""
    c = CFG
    g = torch.Generator(device=f"cuda:{device}")
    g.manual_seed(SEED)
    dev = f"cuda:{device}"
    H, V = c["hidden"], c["vocab"]

    def randn(shape, std):
        return (torch.randn(shape, generator=g, device=dev, dtype=torch.float32) * std).to(torch.bfloat16)

    t0 = time.time()
    gpu.load_weight(aos.W_EMBED, randn((V, H), 1.0), on_device=True)
    gpu.load_weight(aos.W_LM_HEAD, randn((V, H), 0.02), on_device=True)
    gpu.load_weight(aos.W_FINAL_NORM, (1 + randn((H,), 0.1).float()).to(torch.bfloat16), on_device=True)
    for l in range(layers):
        gpu.load_weight(aos.W_ATTN_NORM, (1 + randn((H,), 0.1).float()).to(torch.bfloat16), layer=l, on_device=True)
        gpu.load_weight(aos.W_MLP_NORM, (1 + randn((H,), 0.1).float()).to(torch.bfloat16), layer=l, on_device=True)
        for m, shp in enumerate(module_shapes()):
            gpu.load_weight(aos.W_PROJ, randn(shp, 0.02), layer=l, module=m, on_device=True)
    torch.cuda.synchronize()
    log(f"[bench] base weights loaded in {time.time() - t0:.1f}s")
    return randn


def build_gpu_model(aos, torch, device, steps_total, layers):
    c = CFG
    rng = np.random.default_rng(SEED)
    ranks = ranks_of(rng)
    ctx = ctx_lens_of(rng, c["batch"])
    cap = int(sum(((int(r) + 15) // 16) * 16 for r in ranks)) + 64
    max_seq = c["ctx_hi"] + steps_total + 16
    blocks = int(sum((int(n) + steps_total + 16 + 15) // 16 for n in ctx)) + 16
    gpu = aos.CudaKernels(c["hidden"], c["n_heads"], c["n_kv_heads"], c["head_dim"], c["intermediate"], c["vocab"],
                          layers, max_batch=c["batch"], kv_num_blocks=blocks, max_seq_len=max_seq,
                          lora_rank_capacity=cap, lora_max_adapters=c["n_adapters"], device=device)
    randn = load_base(gpu, aos, torch, device, layers)
    shapes = module_shapes()
    t0 = time.time()
    L = gpu._L
    for a in range(c["n_adapters"]):
        r = int(ranks[a])
        aos.check(L.aos_adapter_new(gpu.ctx, a, r, float(2 * r)), gpu.ctx)
        for m, (out, inn) in enumerate(shapes):
            A = randn((layers, r, inn), 0.02)
            B = randn((layers, out, r), 0.02)
            for l in range(layers):
                aos.check(L.aos_adapter_set_module(gpu.ctx, a, l, m, A[l].data_ptr(), B[l].data_ptr(), 1), gpu.ctx)
    torch.cuda.synchronize()
    log(f"[bench] {c['n_adapters']} adapters loaded in {time.time() - t0:.1f}s (rank capacity {cap})")
    seq_ids = np.arange(c["batch"], dtype=np.uint64)
    for t in range(c["batch"]):
        gpu.kv_alloc(int(seq_ids[t]), int(ctx[t]) + steps_total + 16)
    gpu.kv_fill_synthetic(seed=SEED, std=1.0)
    for t in range(c["batch"]):
        gpu.kv_set_len(int(seq_ids[t]), int(ctx[t]))
    return gpu, ranks, ctx, seq_ids


# ------------------------------------------------------------------ byte accounting
def lora_bytes(ranks, rings_np, layers):
    """Unique selected adapters' A and B bytes for one step (all layers, 7 modules)."""
    c = CFG
    H, I = c["hidden"], c["intermediate"]
    QD, KVD = c["n_heads"] * 128, c["n_kv_heads"] * 128
    per_rank = (H + QD) + (H + KVD) * 2 + (QD + H) + (H + I) * 2 + (I + H)  # sum of in+out over modules
    sel = set()
    for r in rings_np:
        for j in range(int(r["top_k"])):
            if r["gates_q15"][j] > 0:
                sel.add(int(r["indices"][j]))
    return sum(int(ranks[a]) for a in sel) * per_rank * 2 * layers, len(sel)


def base_bytes(layers):
    c = CFG
    H, I = c["hidden"], c["intermediate"]
    QD, KVD = c["n_heads"] * 128, c["n_kv_heads"] * 128
    per_layer = (QD + 2 * KVD) * H + H * QD + 2 * I * H + H * I
    return per_layer * 2 * layers


def act_bytes(layers, T):
    c = CFG
    H, I = c["hidden"], c["intermediate"]
    QD = c["n_heads"] * 128
    # GEMM inputs + outputs per layer (normed/q/k/v, attn/o+resid, normed/act, act/resid)
    per_layer = (H + QD + 2 * c["n_kv_heads"] * 128) + (QD + 2 * H) + (H + I) + (I + 2 * H)
    return per_layer * 2 * T * layers


def attn_bytes(ctx_now, layers):
    c = CFG
    kv = sum(int(n) + 1 for n in ctx_now) * c["n_kv_heads"] * 128 * 2 * 2
    qo = len(ctx_now) * c["n_heads"] * 128 * 2 * 2
    return (kv + qo) * layers


# ------------------------------------------------------------------ CPU side (oracle)
class CpuSample:
    """The CPU restatement of the reference path (oracle/) on a bounded sample
    of the same workload: one decoder layer (128 adapters of that layer, K=4)
    for n_tokens tokens with their own contexts, plus lm_head for lm_tokens
    tokens; extrapolated to a full 32-layer, 64-token step."""

    def __init__(self, n_tokens=16, lm_tokens=2, lm_rows=16032):
        import torch

        from oracle import oracle as O

        self.O = O
        c = CFG
        torch.manual_seed(SEED + 7)
        H, nh, nkv, I, V = c["hidden"], c["n_heads"], c["n_kv_heads"], c["intermediate"], c["vocab"]

        def bf(*shape, std=0.02, mean=0.0):
            t = torch.randn(*shape, dtype=torch.float32) * std + mean
            return t.to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)

        self.n_tokens, self.lm_tokens, self.lm_rows = n_tokens, lm_tokens, lm_rows
        m = O.HostModel(H, nh, nkv, 128, I, V, 1)
        m.attn_norm[0] = bf(H, std=0.1, mean=1.0)
        m.mlp_norm[0] = bf(H, std=0.1, mean=1.0)
        for mod in range(7):
            m.w[mod][0] = bf(*m.mod_shape(mod))
        self.m = m
        ranks = [int(r) for r in ranks_of(np.random.default_rng(SEED))]
        ad = O.HostAdapters(m, ranks, [2.0 * r for r in ranks])
        for a, r in enumerate(ranks):
            for mod in range(7):
                out, inn = m.mod_shape(mod)
                ad.A[a][0][mod] = bf(r, inn)
                ad.B[a][0][mod] = bf(out, r)
        self.ad = ad
        ctx = ctx_lens_of(np.random.default_rng(SEED), c["batch"])[:n_tokens]
        mb = (int(ctx.max()) + 16 + 15) // 16
        bt = np.arange(n_tokens * mb, dtype=np.int32).reshape(n_tokens, mb)
        self.kv = O.HostKV(m, n_tokens * mb, 16, bt, ctx.astype(np.int32),
                           k_pool=bf(1, n_tokens * mb, nkv, 16, 128, std=1.0),
                           v_pool=bf(1, n_tokens * mb, nkv, 16, 128, std=1.0))
        self.pri = torch.randn(n_tokens, c["n_adapters"]).numpy()
        self.hid0 = bf(n_tokens, H, std=1.0)
        # lm_head through the oracle's final norm + projection (a 0-layer model)
        # on lm_rows of the vocabulary, scaled to the full vocabulary
        mm = O.HostModel(H, nh, nkv, 128, I, lm_rows, 0)
        mm.lm_head = bf(lm_rows, H)
        mm.embed = bf(1, H, std=1.0)
        mm.final_norm = bf(H, std=0.0, mean=1.0)
        self.mm = mm
        self.kv0 = O.HostKV(mm, 1, 16, np.zeros((lm_tokens, 1), np.int32), np.zeros(lm_tokens, np.int32))

    def run(self, threads):
        O, c = self.O, CFG
        hid = self.hid0.copy()
        t0 = time.perf_counter()
        rings, _, _, _ = O.route_batch(self.pri, None, k=c["K"], n_threads=threads)
        O.layer_step(self.m, self.ad, 0, rings, self.kv, hid, n_threads=threads)
        t_layer = time.perf_counter() - t0
        t0 = time.perf_counter()
        O.decode_step(self.mm, None, np.zeros(self.lm_tokens, O.RING_DTYPE), np.zeros(self.lm_tokens, np.int32),
                      self.kv0, n_threads=threads)
        t_lm = time.perf_counter() - t0
        t_lm *= c["vocab"] / self.lm_rows
        step_s = t_layer * (c["batch"] / self.n_tokens) * c["n_layers"] + t_lm * (c["batch"] / self.lm_tokens)
        sample = (f"oracle (C++ restatement, {threads} threads): 1 of 32 layers x {self.n_tokens} tokens "
                  f"({t_layer:.2f}s) + lm_head {self.lm_rows} of {c['vocab']} rows x {self.lm_tokens} tokens, "
                  f"extrapolated to 32 layers x 64 tokens per step")
        return c["batch"] / step_s, sample


def run_reference(args, rank, world):
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    cs = CpuSample()
    for _ in range(args.warmup):
        cs.run(threads)
    vals = []
    t0 = time.perf_counter()
    for _ in range(args.steps):
        v, sample = cs.run(threads)
        vals.append(v)
    el = time.perf_counter() - t0
    value = float(np.median(vals))
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000.0 * CFG["batch"] / value,
            "ms_per_step_kind": "extrapolated from each step's bounded sample (1 of 32 layers x 16 tokens + an "
                                "lm_head slice), not a timed full step",
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": "config 3: 32-layer 8B-shape decode, batch 64, K=4 of 128 LoRAs (ranks 8-64), "
                                   "paged KV block 16, ctx U[512,4096]", "parallelism": "cpu",
                       "threads": threads},
            "cpu_baseline": {"value": value, "unit": "tok/s", "cores": threads, "kind": "port", "sample": sample},
            "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "wall_s": el}
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------ configs 1 and 2
def _flush_l2(torch, dev, buf=[]):
    """Write a buffer larger than L2 (126 MB) so the next launch reads from HBM."""
    if not buf:
        buf.append(torch.empty(64 << 20, dtype=torch.float32, device=dev))  # 256 MB
    buf[0].fill_(1.0)


def run_config1(args, rank, world, local):
    """router + fp32 LoRA op.  64 tokens, hidden 2048 fp32
    x ~ N(0,1); W 2048x2048, N=8 adapters of rank 16 (A, B ~ N(0, 0.02));
    gate logits N(0,1), K=2, tau 1, eps 0.02; no alpha/rank scale (alpha = r).
    One step = aos_route_batch_dev + aos_lora_op_f32_dev.  The operands fit in
    L2, so L2 is flushed before every timed step (outside the events)."""
    import torch
    aos = importlib.import_module("adapter-os_b200")
    from oracle import oracle as O
    T, H, N, R, K = 64, 2048, 8, 16, 2
    dev = f"cuda:{local}"
    rng = np.random.default_rng(SEED + 1)
    x = rng.standard_normal((T, H)).astype(np.float32)
    W = (rng.standard_normal((H, H)) * 0.02).astype(np.float32)
    A = (rng.standard_normal((N, R, H)) * 0.02).astype(np.float32)
    B = (rng.standard_normal((N, H, R)) * 0.02).astype(np.float32)
    pri = rng.standard_normal((T, N)).astype(np.float32)
    dx, dW, dA, dB, dp = (torch.from_numpy(a).to(dev) for a in (x, W, A, B, pri))
    sids = torch.arange(N, device=dev, dtype=torch.int64)
    rings = torch.zeros((T, 40), dtype=torch.uint8, device=dev)
    y = torch.empty((T, H), dtype=torch.float32, device=dev)

    def step(stream=None):
        aos.route_batch_dev(dp, sids, rings, k=K, tau=1.0, eps=0.02, stream=stream)
        aos.lora_op_f32_dev(dx, dW, dA, dB, rings, y, stream=stream)

    W_, K_ = max(3, args.warmup), args.steps
    for _ in range(W_):
        step()
    torch.cuda.synchronize()
    # The op is a few tens of microseconds: replay it from a CUDA graph so the
    # timed region holds the device work, not the Python call overhead.
    side = torch.cuda.Stream()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(side):
        step(side.cuda_stream)  # warm the stream-ordered allocator on this stream
        torch.cuda.synchronize()
        with torch.cuda.graph(graph, stream=side):
            step(side.cuda_stream)
    torch.cuda.synchronize()
    # Every step is enqueued before any is waited for: the L2 flush that runs on
    # the GPU ahead of each start event gives the host time to enqueue the
    # replay, so host-side delays (the clock sampler's thread among them) do
    # not open a gap inside a timed interval.
    clocks = ClockSampler(local)
    clocks.start()
    evs = []
    for _ in range(K_):
        _flush_l2(torch, dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        graph.replay()
        e1.record()
        evs.append((e0, e1))
    torch.cuda.synchronize()
    clk = clocks.stop()
    ms = sum(a.elapsed_time(b) for a, b in evs) / K_
    # the same op through the Python/C-ABI calls, host overhead included
    t0 = time.perf_counter()
    for _ in range(K_):
        step()
    torch.cuda.synchronize()
    call_ms = (time.perf_counter() - t0) * 1000.0 / K_
    rn = rings.cpu().numpy().view(aos.RING_DTYPE).reshape(T)
    sel = {int(r["indices"][j]) for r in rn for j in range(int(r["top_k"])) if r["gates_q15"][j] > 0}
    nbytes = W.nbytes + len(sel) * (A[0].nbytes + B[0].nbytes) + x.nbytes + T * H * 4 + pri.nbytes + T * 40
    peak, kind = peaks()
    gbs = nbytes / (ms / 1000.0) / 1e9
    # CPU: the oracle's router + fp32 op on the same inputs, 1 thread and all threads
    cpu = {}
    for th in (1, os.cpu_count() or 1):
        reps, t0 = 0, time.perf_counter()
        while time.perf_counter() - t0 < 3.0:
            rg, _, _, _ = O.route_batch(pri, None, k=K, n_threads=th)
            O.lora_op_f32(x, W, A, B, rg, None, n_threads=th)
            reps += 1
        cpu[th] = (time.perf_counter() - t0) / reps
    if rank == 0:
        line = {"metric": "config 1: router + fp32 LoRA op, 64 tokens x 2048, N=8 r=16, K=2 (tokens/s)",
                "value": T / (ms / 1000.0), "unit": "tok/s", "n_gpus": 1, "steps": K_, "warmup": W_,
                "ms_per_step": ms, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                "dtype": "f32", "data": "synthetic",
                "config": {"workload": "config 1", "l2": "flushed before every timed step",
                           "timing": "CUDA-graph replay of route + op between CUDA events"},
                "host_call_ms_per_step": call_ms, "clocks": clk,
                "roofline": {"bound": "hbm", "kernel": "route + lora_shrink_f32 + lora_base_f32 + lora_expand_f32",
                             "achieved": gbs, "peak": peak, "unit": "GB/s", "frac": gbs / peak, "peak_kind": kind,
                             "bytes_per_step": nbytes},
                "cpu_baseline": {"value": T / cpu[1], "unit": "tok/s", "cores": 1, "kind": "port",
                                 "sample": "the whole op (oracle router + fp32 op)",
                                 "all_cores": {"value": T / cpu[os.cpu_count() or 1], "cores": os.cpu_count()}}}
        print(json.dumps(line), flush=True)


def run_config2(args, rank, world, local):
    """one decoder layer, bf16, hidden 3584, 28/4 heads,
    intermediate 18944; 32 rank-16 adapters on q/k/v/o, K=4; decode batch 32
    with 2048 cached positions each.  One step = router + aos_layer_step_dev
    (RMSNorm, q/k/v + LoRA + RoPE + KV append, attention, o + LoRA, RMSNorm,
    gate/up + SwiGLU, down).  466 MB of layer weights exceed L2."""
    import torch
    aos = importlib.import_module("adapter-os_b200")
    from oracle import oracle as O
    H, nh, nkv, I, T, ctx, NA, R, K = 3584, 28, 4, 18944, 32, 2048, 32, 16, 4
    dev = f"cuda:{local}"
    rng = np.random.default_rng(SEED + 2)
    W_, K_ = max(3, args.warmup), args.steps
    mb = (ctx + W_ + K_ + 32 + 15) // 16
    gpu = aos.CudaKernels(H, nh, nkv, 128, I, 256, 1, max_batch=T, kv_num_blocks=T * mb + 8, max_seq_len=mb * 16,
                          lora_rank_capacity=NA * R, lora_max_adapters=NA,
                          lora_modules=["q_proj", "k_proj", "v_proj", "o_proj"], device=local)
    g = torch.Generator(device=dev)
    g.manual_seed(SEED + 2)

    def randn(shape, std):
        return (torch.randn(shape, generator=g, device=dev, dtype=torch.float32) * std).to(torch.bfloat16)

    QD, KVD = nh * 128, nkv * 128
    shapes = [(QD, H), (KVD, H), (KVD, H), (H, QD), (I, H), (I, H), (H, I)]
    gpu.load_weight(aos.W_ATTN_NORM, (1 + randn((H,), 0.1).float()).to(torch.bfloat16), layer=0, on_device=True)
    gpu.load_weight(aos.W_MLP_NORM, (1 + randn((H,), 0.1).float()).to(torch.bfloat16), layer=0, on_device=True)
    for mod, shp in enumerate(shapes):
        gpu.load_weight(aos.W_PROJ, randn(shp, 0.02), layer=0, module=mod, on_device=True)
    L = gpu._L
    for a in range(NA):
        aos.check(L.aos_adapter_new(gpu.ctx, a, R, float(2 * R)), gpu.ctx)
        for mod in range(4):
            out, inn = shapes[mod]
            Am, Bm = randn((R, inn), 0.02), randn((out, R), 0.02)
            aos.check(L.aos_adapter_set_module(gpu.ctx, a, 0, mod, Am.data_ptr(), Bm.data_ptr(), 1), gpu.ctx)
    torch.cuda.synchronize()
    sids = np.arange(T, dtype=np.uint64)
    for t in range(T):
        gpu.kv_alloc(int(sids[t]), mb * 16)
    gpu.kv_fill_synthetic(seed=SEED, std=1.0)
    for t in range(T):
        gpu.kv_set_len(int(sids[t]), ctx)
    pri = torch.from_numpy(rng.standard_normal((T, NA)).astype(np.float32)).to(dev)
    nsids = torch.arange(NA, device=dev, dtype=torch.int64)
    rings = torch.zeros((T, 40), dtype=torch.uint8, device=dev)
    hidden = randn((T, H), 1.0).view(torch.int16)
    stream_ptr = gpu.stream()
    stream = torch.cuda.ExternalStream(stream_ptr)

    def step():
        aos.route_batch_dev(pri, nsids, rings, k=K, tau=1.0, eps=0.02, stream=stream_ptr)
        gpu.layer_step_dev(0, rings, sids, hidden, advance=False, stream=stream_ptr)

    for _ in range(W_):
        step()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clocks = ClockSampler(local)
    clocks.start()
    ev0.record(stream)
    for _ in range(K_):
        step()
    ev1.record(stream)
    torch.cuda.synchronize()
    clk = clocks.stop()
    ms = ev0.elapsed_time(ev1) / K_
    gpu.health_check()
    rn = rings.cpu().numpy().view(aos.RING_DTYPE).reshape(T)
    sel = {int(r["indices"][j]) for r in rn for j in range(int(r["top_k"])) if r["gates_q15"][j] > 0}
    base = ((QD + 2 * KVD) * H + H * QD + 2 * I * H + H * I) * 2
    kvb = T * (ctx + 1) * KVD * 2 * 2
    lora = len(sel) * R * ((H + QD) + 2 * (H + KVD) + (QD + H)) * 2
    acts = T * (4 * H + QD * 2 + 2 * KVD + I) * 2
    nbytes = base + kvb + lora + acts
    peak, kind = peaks()
    gbs = nbytes / (ms / 1000.0) / 1e9
    # CPU: the oracle layer (its own seeded weights of the same shapes) on the
    # host cores for a sample of the tokens
    th = os.cpu_count() or 1
    n_cpu = 4
    m = O.HostModel.random(rng, H, nh, nkv, 128, I, 256, 1, with_embed=False)
    ad = O.HostAdapters.random(rng, m, [R] * NA, modules=[0, 1, 2, 3])
    bt = np.arange(n_cpu * mb, dtype=np.int32).reshape(n_cpu, mb)
    kv = O.HostKV(m, n_cpu * mb, 16, bt, np.full(n_cpu, ctx, np.int32))
    kv.k_pool[...] = O.f32_to_bf16_bits(rng.standard_normal(kv.k_pool.shape, dtype=np.float32))
    kv.v_pool[...] = O.f32_to_bf16_bits(rng.standard_normal(kv.v_pool.shape, dtype=np.float32))
    rg, _, _, _ = O.route_batch(rng.standard_normal((n_cpu, NA)).astype(np.float32), None, k=K)
    hs = O.f32_to_bf16_bits(rng.standard_normal((n_cpu, H), dtype=np.float32))
    t0 = time.perf_counter()
    O.layer_step(m, ad, 0, rg, kv, hs, n_threads=th)
    cpu_s = time.perf_counter() - t0
    if rank == 0:
        line = {"metric": "config 2: one decoder layer, batch 32, KV 2048, 32 rank-16 LoRAs K=4 (tokens/s)",
                "value": T / (ms / 1000.0), "unit": "tok/s", "n_gpus": 1, "steps": K_, "warmup": W_,
                "ms_per_step": ms, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                "dtype": "bf16", "data": "synthetic",
                "config": {"workload": "config 2: H 3584, 28/4 heads, I 18944, q/k/v/o LoRA",
                           "l2": "inputs larger than L2 (466 MB of layer weights)"},
                "clocks": clk,
                "roofline": {"bound": "hbm", "kernel": "whole layer step", "achieved": gbs, "peak": peak,
                             "unit": "GB/s", "frac": gbs / peak, "peak_kind": kind, "bytes_per_step": nbytes,
                             "unique_adapters": len(sel)},
                "cpu_baseline": {"value": n_cpu / cpu_s, "unit": "tok/s", "cores": th, "kind": "port",
                                 "sample": f"oracle layer for {n_cpu} tokens with 2048 cached positions each"}}
        print(json.dumps(line), flush=True)
    gpu.close()


# ------------------------------------------------------------------ config 4
CFG4 = dict(n_prompts=8, prompt_len=2048, n_adapters=64, rank=16, K=4)
METRIC4 = "prefill tok/s, 8B-shape, 8 x 2048-token prompts, K=4 of 64 rank-16 LoRAs; % of bf16 tensor roofline"


def peak_tflops():
    """Sustained bf16 peak: a prefill step runs its GEMMs back to back for
    hundreds of ms, under the power cap like the sustained cuBLAS loop."""
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["bf16_tflops_sustained"]), "measured (sustained)"
    except Exception:
        return 1400.0, "fallback (sustained)"


def run_config4(args, rank, world, local):
    """BASELINE config 4 (prefill): 8 prompts of 2048 tokens (ids uniform over
    the vocabulary), per-token K=4 routing over 64 rank-16 adapters on all 7
    modules, causal attention.  One step = the prompt pass of all 8 prompts
    (aos_prefill_dev) from empty caches, logits of each prompt's last token.
    Each GPU prefills its own 8 prompts (replicas, weak scaling)."""
    import torch
    aos = importlib.import_module("adapter-os_b200")
    c, c4 = CFG, CFG4
    S, P, NA, R = c4["n_prompts"], c4["prompt_len"], c4["n_adapters"], c4["rank"]
    T = S * P
    layers = args.layers
    dev = f"cuda:{local}"
    W, K = max(3, args.warmup), args.steps
    gpu = aos.CudaKernels(c["hidden"], c["n_heads"], c["n_kv_heads"], c["head_dim"], c["intermediate"], c["vocab"],
                          layers, max_batch=S, kv_num_blocks=S * ((P + 15) // 16) + 16, max_seq_len=P + 16,
                          lora_rank_capacity=NA * R, lora_max_adapters=NA, device=local)
    randn = load_base(gpu, aos, torch, local, layers)
    L = gpu._L
    for a in range(NA):
        aos.check(L.aos_adapter_new(gpu.ctx, a, R, float(2 * R)), gpu.ctx)
        for m, (out, inn) in enumerate(module_shapes()):
            A = randn((layers, R, inn), 0.02)
            Bm = randn((layers, out, R), 0.02)
            for l in range(layers):
                aos.check(L.aos_adapter_set_module(gpu.ctx, a, l, m, A[l].data_ptr(), Bm[l].data_ptr(), 1), gpu.ctx)
    torch.cuda.synchronize()
    sids = np.arange(S, dtype=np.uint64)
    for i in range(S):
        gpu.kv_alloc(int(sids[i]), P + 16)
    n_tok = np.full(S, P, np.uint32)
    stream_ptr = gpu.stream()
    stream = torch.cuda.ExternalStream(stream_ptr)
    gen = torch.Generator(device=dev)
    gen.manual_seed(SEED + 4)
    priors = torch.randn((T, NA), generator=gen, device=dev, dtype=torch.float32)
    tokens = torch.randint(0, c["vocab"], (T,), generator=gen, device=dev, dtype=torch.int32)
    rings = torch.zeros((T, 40), dtype=torch.uint8, device=dev)
    nsids = torch.arange(NA, device=dev, dtype=torch.int64)
    logits = torch.empty((S, c["vocab"]), dtype=torch.float32, device=dev)

    def step():
        for i in range(S):
            gpu.kv_set_len(int(sids[i]), 0)
        aos.route_batch_dev(priors, nsids, rings, k=c4["K"], tau=1.0, eps=0.02, stream=stream_ptr)
        gpu.prefill_dev(sids, n_tok, rings, tokens, logits=logits, stream=stream_ptr)

    for _ in range(W):
        step()
    torch.cuda.synchronize()
    clocks = ClockSampler(local)
    clocks.start()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    for _ in range(K):
        step()
    ev1.record(stream)
    torch.cuda.synchronize()
    clk = clocks.stop()
    ms = ev0.elapsed_time(ev1) / K
    gpu.health_check()
    gpu.profile_enable(True)
    gpu.profile_read(reset=True)
    step()
    torch.cuda.synchronize()
    prof = gpu.profile_read(reset=True)
    gpu.profile_enable(False)
    H, I, V = c["hidden"], c["intermediate"], c["vocab"]
    QD, KVD = c["n_heads"] * 128, c["n_kv_heads"] * 128
    per_layer = (QD + 2 * KVD) * H + H * QD + 2 * I * H + H * I
    gemm_flop = 2.0 * T * per_layer * layers
    io = sum(o + i_ for o, i_ in module_shapes())
    lora_flop = 2.0 * T * io * c4["K"] * R * layers  # the K selected adapters of each token (algorithmic)
    lora_exec_flop = 2.0 * T * io * NA * R * layers  # what the dense-over-touched-groups LoRA launches execute
    attn_flop = 4.0 * S * (P * (P + 1) / 2) * QD * layers  # QK^T and PV over the causal triangle
    lm_flop = 2.0 * S * H * V
    flop = gemm_flop + lora_flop + attn_flop + lm_flop
    peak, kind = peak_tflops()
    gemm_ms = prof["ms"]["gemm"] + prof["ms"]["owner_lora"]
    gemm_tf = (gemm_flop + lora_flop) / (gemm_ms / 1000.0) / 1e12
    attn_tf = attn_flop / (prof["ms"]["attention"] / 1000.0) / 1e12
    if rank == 0:
        tf = flop / (ms / 1000.0) / 1e12
        line = {
            "metric": METRIC4, "value": T * world / (ms / 1000.0), "unit": "tok/s", "n_gpus": world, "steps": K,
            "warmup": W, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "bf16", "data": "synthetic",
            "config": {"workload": "config 4: 32-layer 8B-shape prefill, 8 prompts x 2048 tokens (ids uniform), "
                                   "K=4 of 64 rank-16 LoRAs on 7 modules, causal attention",
                       "layers": layers, "tokens_per_step": T, "parallelism": f"dp{world} (replicas)"},
            "roofline": {"bound": "tensor", "kernel": "whole prefill", "achieved": tf, "peak": peak,
                         "unit": "TFLOP/s", "frac": tf / peak, "peak_kind": kind, "flop_per_step": flop},
            "roofline_gemm": {"bound": "tensor", "kernel": "pf_gemm_kernel (base + LoRA shrink/expand)",
                              "achieved": gemm_tf, "peak": peak, "unit": "TFLOP/s", "frac": gemm_tf / peak,
                              "ms_per_step": gemm_ms},
            "roofline_attention": {"bound": "tensor", "kernel": "attn_prefill_tc_kernel (tcgen05, TMEM)",
                                   "achieved": attn_tf, "peak": peak, "unit": "TFLOP/s", "frac": attn_tf / peak,
                                   "ms_per_step": prof["ms"]["attention"]},
            "lora_flop_executed_per_step": lora_exec_flop,
            "kernel_ms_per_step": prof["ms"],
            "clocks": clk,
        }
        print(json.dumps(line), flush=True)
    gpu.close()


# ------------------------------------------------------------------ config 5
CFG5 = dict(n_adapters=1024, rank=16, K=8, batch=256, ctx_lo=512, ctx_hi=1024, zipf_s=1.1)
METRIC5 = "decode tok/s, 8B-shape, K=8 of 1024 rank-16 LoRAs sharded by adapter id, batch 256"


def run_config5(args, rank, world, local, dist):
    """BASELINE config 5 (large adapter pool): 1024 rank-16 adapters on all 7
    modules, sharded by id (rank r holds ids with id % world == r); popularity
    Zipf(s=1.1) over a seeded permutation of ids; K=8; decode batch 256 split
    evenly over the ranks (strong scaling: the box decodes 256 tokens per
    step at every N).  At N > 1 every LoRA term crosses the NCCL exchange of
    aos_run_step_sharded_dev; at N = 1 the whole pool is local and the step
    is the fused one.  Context lengths U[512, 1024] (not stated by the
    config; chosen so the whole pool, the base and the KV of 256 sequences
    fit one GPU)."""
    import torch
    aos = importlib.import_module("adapter-os_b200")
    c, c5 = CFG, CFG5
    B, NA, R = c5["batch"], c5["n_adapters"], c5["rank"]
    if B % world:
        raise SystemExit("config 5 needs a world size that divides 256")
    T = B // world
    dev = f"cuda:{local}"
    W, K, PS = max(3, args.warmup), args.steps, 2
    total = W + K + PS + 2
    layers = args.layers
    rng = np.random.default_rng(SEED + 5)
    ctx_all = rng.integers(c5["ctx_lo"], c5["ctx_hi"] + 1, size=B)
    perm = rng.permutation(NA)  # popularity rank -> adapter id
    pop = 1.0 / np.arange(1, NA + 1) ** c5["zipf_s"]
    logp = np.empty(NA)
    logp[perm] = np.log(pop / pop.sum())
    owned = [a for a in range(NA) if a % world == rank]
    home = slice(rank * T, (rank + 1) * T)
    ctx = ctx_all[home]
    blocks = int(sum((int(n) + total + 16 + 15) // 16 for n in ctx)) + 16
    gpu = aos.CudaKernels(c["hidden"], c["n_heads"], c["n_kv_heads"], c["head_dim"], c["intermediate"], c["vocab"],
                          layers, max_batch=B, kv_num_blocks=blocks, max_seq_len=c5["ctx_hi"] + total + 16,
                          lora_rank_capacity=len(owned) * R, lora_max_adapters=NA, device=local)
    load_base(gpu, aos, torch, local, layers)
    t0 = time.time()
    L = gpu._L
    shapes = module_shapes()
    g = torch.Generator(device=dev)
    for a in owned:  # adapter a's weights depend on a only, so every N decodes the same model
        g.manual_seed(SEED * 7 + a)
        aos.check(L.aos_adapter_new(gpu.ctx, a, R, float(2 * R)), gpu.ctx)
        for m, (out, inn) in enumerate(shapes):
            A = (torch.randn((layers, R, inn), generator=g, device=dev) * 0.02).to(torch.bfloat16)
            Bm = (torch.randn((layers, out, R), generator=g, device=dev) * 0.02).to(torch.bfloat16)
            for l in range(layers):
                aos.check(L.aos_adapter_set_module(gpu.ctx, a, l, m, A[l].data_ptr(), Bm[l].data_ptr(), 1), gpu.ctx)
    torch.cuda.synchronize()
    log(f"[bench] config 5 rank {rank}: {len(owned)} adapters loaded in {time.time() - t0:.1f}s")
    seq_ids = np.arange(rank * T, (rank + 1) * T, dtype=np.uint64)
    for i in range(T):
        gpu.kv_alloc(int(seq_ids[i]), int(ctx[i]) + total + 16)
    gpu.kv_fill_synthetic(seed=SEED + rank, std=1.0)
    for i in range(T):
        gpu.kv_set_len(int(seq_ids[i]), int(ctx[i]))
    if world > 1:
        uid = [aos.shard_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        gpu.shard_init(rank, world, uid[0])
    stream_ptr = gpu.stream()
    stream = torch.cuda.ExternalStream(stream_ptr)
    # priors: log popularity + Gumbel noise, so top-K is a popularity-weighted
    # draw without replacement; generated for all 256 tokens, home rows kept
    gen = torch.Generator(device=dev)
    gen.manual_seed(SEED + 50)
    lp = torch.tensor(logp, dtype=torch.float32, device=dev)
    priors, tokens = [], []
    for i in range(total):
        u = torch.rand((B, NA), generator=gen, device=dev).clamp_(1e-12, 1 - 1e-7)
        priors.append((lp - torch.log(-torch.log(u)))[home].contiguous())
        tokens.append(torch.randint(0, c["vocab"], (B,), generator=gen, device=dev, dtype=torch.int32)[home].contiguous())
    sids = torch.arange(NA, device=dev, dtype=torch.int64)
    rings = torch.zeros((T, 40), dtype=torch.uint8, device=dev)
    logits = torch.empty((T, c["vocab"]), dtype=torch.float32, device=dev)

    def step(i):
        aos.route_batch_dev(priors[i], sids, rings, k=c5["K"], tau=1.0, eps=0.02, stream=stream_ptr)
        if world > 1:
            gpu.run_step_sharded_dev(rings, tokens[i], seq_ids, logits=logits, stream=stream_ptr)
        else:
            gpu.run_step_batch_dev(rings, tokens[i], seq_ids, logits=logits, stream=stream_ptr)

    def barrier():
        torch.cuda.synchronize()
        if dist:
            dist.barrier()

    def max_over_ranks(x):
        if not dist:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    for i in range(W):
        step(i)
    barrier()
    clocks = ClockSampler(local)
    clocks.start()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    ev0.record(stream)
    for i in range(W, W + K):
        step(i)
    ev1.record(stream)
    barrier()
    clk = clocks.stop()
    ms = max_over_ranks(ev0.elapsed_time(ev1))
    value = B * K / (ms / 1000.0)
    gpu.health_check()

    # instrumented steps: per-class device time and this rank's bytes
    gpu.profile_enable(True)
    gpu.profile_read(reset=True)
    H, I, V = c["hidden"], c["intermediate"], c["vocab"]
    QD, KVD = c["n_heads"] * 128, c["n_kv_heads"] * 128
    per_col = sum(o + i_ for o, i_ in shapes)  # bytes / 2 of one rank column over the 7 modules
    slot = {a: j for j, a in enumerate(owned)}  # arena order: adapter j at columns [16j, 16j + 16)
    lora_b, kv_b, groups_n = 0, 0, 0
    for i in range(W + K, W + K + PS):
        ctx_now = [gpu.kv_len(int(s_)) for s_ in seq_ids]
        step(i)
        torch.cuda.synchronize()
        rg = rings
        if dist:
            allr = torch.empty((B, 40), dtype=torch.uint8, device=dev)
            dist.all_gather_into_tensor(allr, rings)
            rg = allr
        rn = rg.cpu().numpy().view(aos.RING_DTYPE).reshape(-1)
        groups = set()
        for r_ in rn:
            for j in range(int(r_["top_k"])):
                a = int(r_["indices"][j])
                if r_["gates_q15"][j] > 0 and a in slot:
                    groups.add(slot[a] * R // 64)
        groups_n += len(groups)
        lora_b += len(groups) * 64 * per_col * 2 * layers
        kv_b += attn_bytes(ctx_now, layers)
    prof = gpu.profile_read(reset=True)
    gpu.profile_enable(False)
    peak, peak_kind = peaks()
    act = act_bytes(layers, T)
    step_bytes = (base_bytes(layers) + V * H * 2 + act) + (lora_b + kv_b) / PS
    achieved = step_bytes / (ms / K / 1000.0) / 1e9
    ins, wid = (H, QD, H, I), (QD + 2 * KVD, H, 2 * I, H)
    x_b = sum(T * n * 2 for n in ins) * layers          # rows sent to each peer
    d_b = sum(T * w_ * 2 for w_ in wid) * layers        # deltas sent back to each peer
    nvlink = (world - 1) * (x_b + d_b) if world > 1 else 0
    if rank == 0:
        line = {
            "metric": METRIC5, "value": value, "unit": "tok/s", "n_gpus": world, "steps": K, "warmup": W,
            "ms_per_step": ms / K, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "bf16", "data": "synthetic",
            "config": {"workload": "config 5: 32-layer 8B-shape decode, 1024 rank-16 adapters on 7 modules sharded "
                                   "by id mod N, Zipf(1.1) popularity, K=8, global batch 256, ctx U[512,1024]",
                       "layers": layers, "global_batch": B, "tokens_per_gpu": T,
                       "parallelism": f"adapter-sharded x{world} (NCCL send/recv per layer and input site)"
                       if world > 1 else "single GPU, whole pool local (fused step)"},
            "roofline": {"bound": "hbm", "kernel": "whole step (rank 0)", "achieved": achieved, "peak": peak,
                         "unit": "GB/s", "frac": achieved / peak, "peak_kind": peak_kind,
                         "bytes_per_step": step_bytes, "lora_bytes_per_step": lora_b / PS,
                         "touched_groups_per_step": groups_n / PS, "kv_bytes_per_step": kv_b / PS},
            "nvlink_bytes_per_step_per_gpu": nvlink,
            "kernel_ms_per_step": {k: v / PS for k, v in prof["ms"].items()},
            "clocks": clk,
        }
        print(json.dumps(line), flush=True)
    barrier()
    gpu.close()


# ------------------------------------------------------------------ GPU arm
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--layers", type=int, default=CFG["n_layers"], help="debug only: fewer layers is not a valid number")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--config", type=int, default=3, choices=[1, 2, 3, 4, 5],
                    help="1: router + fp32 LoRA op; 2: one layer; 3: the headline decode workload; "
                         "4: prefill; 5: the adapter-sharded large pool")
    args = ap.parse_args()

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        run_reference(args, rank, world)
        return

    import torch

    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist_mod

        dist_mod.init_process_group("nccl", timeout=datetime.timedelta(seconds=600))
        dist = dist_mod
    if args.config != 3:
        runner = {1: run_config1, 2: run_config2, 4: run_config4}.get(args.config)
        if runner:
            runner(args, rank, world, local)
        else:
            run_config5(args, rank, world, local, dist)
        if dist:
            dist.barrier()
            dist.destroy_process_group()
        return
    aos = importlib.import_module("adapter-os_b200")
    c = CFG
    W, K = max(3, args.warmup), args.steps
    total = W + K + 3 + K  # warmup + timed + profile + e2e steps
    gpu, ranks, ctx, seq_ids = build_gpu_model(aos, torch, local, total + 4, args.layers)
    B, N = c["batch"], c["n_adapters"]
    stream_ptr = gpu.stream()
    stream = torch.cuda.ExternalStream(stream_ptr)
    gen = torch.Generator(device=f"cuda:{local}")
    gen.manual_seed(SEED + 1)
    priors = torch.randn((total + 4, B, N), generator=gen, device=f"cuda:{local}", dtype=torch.float32)
    tokens = torch.randint(0, c["vocab"], (total + 4, B), generator=gen, device=f"cuda:{local}", dtype=torch.int32)
    sids = torch.arange(N, device=f"cuda:{local}", dtype=torch.int64)
    rings = torch.zeros((B, 40), dtype=torch.uint8, device=f"cuda:{local}")
    logits = torch.empty((B, c["vocab"]), dtype=torch.float32, device=f"cuda:{local}")
    torch.cuda.synchronize()

    def step(i):
        aos.route_batch_dev(priors[i], sids, rings, k=c["K"], tau=1.0, eps=0.02, stream=stream_ptr)
        gpu.run_step_batch_dev(rings, tokens[i], seq_ids, logits=logits, stream=stream_ptr)

    def barrier():
        torch.cuda.synchronize()
        if dist:
            dist.barrier()

    def max_over_ranks(x):
        if not dist:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=f"cuda:{local}")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # ---------------- warmup + timed region (device-resident inputs)
    for i in range(W):
        step(i)
    barrier()
    clocks = ClockSampler(local)
    clocks.start()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    ev0.record(stream)
    for i in range(W, W + K):
        step(i)
    ev1.record(stream)
    barrier()
    clk = clocks.stop()
    ms = ev0.elapsed_time(ev1)
    ms = max_over_ranks(ms)
    value = world * B * K / (ms / 1000.0)
    gpu.health_check()

    # ---------------- instrumented steps: per-kernel-class device time
    ctx_now = [gpu.kv_len(int(s)) for s in seq_ids]
    gpu.profile_enable(True)
    gpu.profile_read(reset=True)
    lbytes, n_sel, abytes = 0, 0, 0
    PS = 3
    for i in range(W + K, W + K + PS):
        ctx_now = [gpu.kv_len(int(s)) for s in seq_ids]
        step(i)
        torch.cuda.synchronize()
        rn = rings.cpu().numpy().view(aos.RING_DTYPE).reshape(B)
        lb, ns = lora_bytes(ranks, rn, args.layers)
        lbytes += lb
        n_sel += ns
        abytes += attn_bytes(ctx_now, args.layers)
    prof = gpu.profile_read(reset=True)
    gpu.profile_enable(False)
    peak, peak_kind = peaks()
    proj_bytes = (base_bytes(args.layers) + act_bytes(args.layers, B)) * PS + lbytes
    proj_ms = prof["ms"]["gemm"] + prof["ms"]["owner_lora"]
    proj_gbs = proj_bytes / (proj_ms / 1000.0) / 1e9
    attn_gbs = abytes / (prof["ms"]["attention"] / 1000.0) / 1e9
    n_gemm_launches = prof["launches"]["gemm"] + prof["launches"]["owner_lora"]
    step_ms_prof = sum(prof["ms"].values()) / PS

    # ---------------- e2e through the host-pointer C ABI
    pin = lambda shape, dt: torch.empty(shape, dtype=dt, pin_memory=True).numpy()
    h_pri = pin((B, N), torch.float32)
    h_sid = np.arange(N, dtype=np.uint64)
    h_tok = pin((B,), torch.int32).view(np.uint32)
    h_logits = pin((B, c["vocab"]), torch.float32)
    h_rings = np.zeros(B, aos.RING_DTYPE)
    L = aos.lib()
    params = aos.RouterParams(c["K"], 1.0, 0.02, 1.0)
    import ctypes as C
    pri_all = priors.cpu().numpy()
    tok_all = tokens.cpu().numpy()
    ent = np.zeros(B, np.float32)
    st = np.zeros(B, np.int32)

    def e2e_step(i):
        h_pri[...] = pri_all[i]
        h_tok[...] = tok_all[i].astype(np.uint32)
        rc = L.aos_route_batch(h_pri.ctypes.data, h_sid.ctypes.data, None, None, None, B, N, C.byref(params),
                               h_rings.ctypes.data, ent.ctypes.data, st.ctypes.data)
        aos.check(rc)
        rc = L.aos_run_step_batch(gpu.ctx, h_rings.ctypes.data, h_tok.ctypes.data, seq_ids.ctypes.data, B,
                                  h_logits.ctypes.data, None)
        aos.check(rc, gpu.ctx)

    base_i = W + K + PS
    e2e_step(base_i)
    barrier()
    t0 = time.perf_counter()
    for i in range(base_i + 1, base_i + 1 + K):
        e2e_step(i)
    barrier()
    e2e_s = max_over_ranks(time.perf_counter() - t0)
    e2e_value = world * B * K / e2e_s
    h2d = B * N * 4 + N * 8 + B * 40 + B * 4 + B * (4 * ((c["ctx_hi"] + total + 16 + 15) // 16) + 4)
    d2h = B * 40 + B * 8 + B * c["vocab"] * 4

    # ---------------- CPU baseline (rank 0, N=1 only)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        threads = os.cpu_count() or 1
        v, sample = CpuSample().run(threads)
        cpu = {"value": v, "unit": "tok/s", "cores": threads, "kind": "port", "sample": sample}

    if rank == 0:
        # kernels per step, from the instrumented pass: one route kernel, plus every
        # launch the step enqueues (the LoRA prep enqueues two kernels: prep +
        # coefficient table)
        lc = prof["launches"]
        # whole step: projections (base + selected LoRA + activations), attention
        # (KV + q/out) and the lm_head weights, per step of the instrumented pass
        step_bytes = proj_bytes / PS + abytes / PS + c["vocab"] * c["hidden"] * 2
        launches_per_step = 1 + (sum(lc.values()) + lc["prep"]) / PS
        line = {
            "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world, "steps": K, "warmup": W,
            "ms_per_step": ms / K, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "bf16", "data": "synthetic",
            "config": {"workload": "config 3: 32-layer 8B-shape decode (H 4096, 32/8 heads, I 14336, V 128256), "
                                   "batch 64 per GPU, K=4 of 128 LoRAs (ranks U{8,16,32,64}, 7 modules), "
                                   "paged KV block 16, ctx U[512,4096]",
                       "layers": args.layers, "global_batch": B * world, "parallelism": f"dp{world} (replicas)",
                       "l2": "inputs larger than L2 (~56 GB weights+adapters+KV per GPU)"},
            "roofline": {"bound": "hbm", "kernel": "tc_gemm_kernel (base + fused LoRA shrink/expand)",
                         "achieved": proj_gbs, "peak": peak, "unit": "GB/s", "frac": proj_gbs / peak,
                         "traffic": GEMM_DRAM_BYTES_PER_LAYER * args.layers, "traffic_unit": "bytes per step",
                         "traffic_source": "a separate ncu capture, not this run: dram__bytes_read.sum + "
                                           "dram__bytes_write.sum of one layer's four GEMM launches on the 2-layer "
                                           "case (its own routing draw), times the layers",
                         "peak_kind": peak_kind,
                         "bytes_per_step": proj_bytes / PS, "ms_per_step": proj_ms / PS,
                         "launches_per_step": n_gemm_launches / PS, "unique_adapters_per_step": n_sel / PS},
            "roofline_attention": {"bound": "hbm", "kernel": "attn_decode_kernel (split-KV; the last chunk's CTA merges the chunks)",
                                   "achieved": attn_gbs, "peak": peak, "unit": "GB/s", "frac": attn_gbs / peak,
                                   "bytes_per_step": abytes / PS, "ms_per_step": prof["ms"]["attention"] / PS},
            "roofline_step": {"bound": "hbm", "what": "whole decode step: projections + attention + lm_head "
                                                      "algorithmic bytes over the timed (graphed) step",
                              "bytes_per_step": step_bytes, "ms_per_step": ms / K,
                              "achieved": step_bytes / (ms / K / 1000.0) / 1e9, "peak": peak, "unit": "GB/s",
                              "frac": step_bytes / (ms / K / 1000.0) / 1e9 / peak},
            "kernel_ms_per_step": {k: v / PS for k, v in prof["ms"].items()},
            "instrumented_step_ms": step_ms_prof,
            "cpu_baseline": cpu,
            "e2e": {"value": e2e_value, "unit": "tok/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
            "gpu_launches": launches_per_step * K,
            "clocks": clk,
        }
        print(json.dumps(line), flush=True)
    gpu.close()
    if dist:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
