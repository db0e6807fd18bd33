"""aos_lora_op_f32_noalloc_dev: the fp32 LoRA op for callers that cannot
allocate device memory -- a host that fixes its device-memory budget at
start-up, code that shares the device with an open CUDA graph capture
(cudaMalloc and cudaFree are not allowed while one is open), or a
latency-critical loop that must not stall on an allocator.  Its scratch is a
fixed device array inside the library instead of a per-call allocation.

Checked through the C ABI, on two calls in a row with different shapes (the
second reuses more of the scratch than the first left in it):
  - against the CPU oracle (kernel_testing.rs:220-257, liquid.rs:222-250
    restated in oracle/) with the 1e-5 relative bound of the other fp32 LoRA
    tests;
  - against aos_lora_op_f32_dev, the entry point that allocates its scratch,
    within the same bound (the two use different base kernels, so they are
    not bit-identical);
  - that the calls allocate nothing: the device's default memory pool (where
    the allocating entry point's cudaMallocAsync draws from) reaches no new
    high-water mark, and the device's free memory is unchanged.
Sizes beyond the scratch are refused.  This file is named so that pytest
collects it last."""
import ctypes as C

import numpy as np
import pytest

from oracle import oracle as O
from tests.aos_import import aos

pytestmark = pytest.mark.gpu

TOL = 1e-5  # fp32 op tolerance, as in tests/test_lora_f32_gpu.py
SCRATCH_FLOATS = 131072  # fixed scratch of the no-allocation entry point
CU_MEMPOOL_ATTR_USED_MEM_CURRENT = 7
CU_MEMPOOL_ATTR_USED_MEM_HIGH = 8


def _bind():
    lib = aos.lib()
    vp, u32 = C.c_void_p, C.c_uint32
    f = lib.aos_lora_op_f32_noalloc_dev
    f.restype = C.c_int
    f.argtypes = [vp, u32, u32, u32, vp, vp, vp, u32, u32, vp, vp, vp, vp]
    return lib, f


class _DefaultPool:
    """The current device's default memory pool, read through the driver API."""

    def __init__(self, device):
        self.cu = C.CDLL("libcuda.so.1")
        dev = C.c_int()
        assert self.cu.cuDeviceGet(C.byref(dev), device) == 0
        self.pool = C.c_void_p()
        assert self.cu.cuDeviceGetDefaultMemPool(C.byref(self.pool), dev) == 0

    def get(self, attr):
        v = C.c_uint64()
        assert self.cu.cuMemPoolGetAttribute(self.pool, attr, C.byref(v)) == 0
        return v.value

    def reset_high(self):
        zero = C.c_uint64(0)  # resets the high-water mark to the current use
        assert self.cu.cuMemPoolSetAttribute(self.pool, CU_MEMPOOL_ATTR_USED_MEM_HIGH, C.byref(zero)) == 0


def _inputs(seed, T, H, Od, N, r):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((T, H), dtype=np.float32)
    W = rng.standard_normal((Od, H), dtype=np.float32) * 0.02
    A = rng.standard_normal((N, r, H), dtype=np.float32) * 0.02
    B = rng.standard_normal((N, Od, r), dtype=np.float32) * 0.02
    alpha = np.linspace(1.0, 2.0 * r, N).astype(np.float32)
    rings, _, _, _ = O.route_batch(rng.standard_normal((T, N), dtype=np.float32), None, k=min(4, N))
    return x, W, A, B, alpha, rings


def _call(fn, torch, dev, x, W, A, B, alpha, rings, y):
    T, H = x.shape
    Od = W.shape[0]
    N, r, _ = A.shape
    rc = fn(dev["x"].data_ptr(), T, H, Od, dev["W"].data_ptr(), dev["A"].data_ptr(), dev["B"].data_ptr(), N, r,
            dev["alpha"].data_ptr(), dev["rings"].data_ptr(), y.data_ptr(), None)
    assert rc == 0, aos.last_error()


def _rel(got, ref):
    return float(np.abs(got - ref).max() / max(np.abs(ref).max(), 1e-30))


def test_no_alloc_matches_oracle_twice_and_allocates_nothing():
    torch = pytest.importorskip("torch")
    lib, noalloc = _bind()
    shapes = ((1, (64, 2048, 2048, 8, 16)), (2, (200, 512, 384, 5, 64)))
    cases = []
    for seed, (T, H, Od, N, r) in shapes:
        assert T * 8 * r <= SCRATCH_FLOATS
        x, W, A, B, alpha, rings = _inputs(seed, T, H, Od, N, r)
        dev = {k: torch.from_numpy(v).cuda() for k, v in (("x", x), ("W", W), ("A", A), ("B", B), ("alpha", alpha))}
        dev["rings"] = torch.from_numpy(rings.view(np.uint8).copy()).cuda()
        ref = O.lora_op_f32(x, W, A, B, rings, alpha)
        y = torch.full((T, Od), float("nan"), device="cuda")
        cases.append((x, W, A, B, alpha, rings, dev, ref, y))
    # warm-up: the first call in the context looks up the scratch array's
    # address and loads the kernels (lazy module loading takes device memory)
    for x, W, A, B, alpha, rings, dev, ref, y in cases:
        _call(noalloc, torch, dev, x, W, A, B, alpha, rings, y)
        y.fill_(float("nan"))
    torch.cuda.synchronize()
    pool = _DefaultPool(torch.cuda.current_device())
    pool.reset_high()
    free0, _ = torch.cuda.mem_get_info()
    for x, W, A, B, alpha, rings, dev, ref, y in cases:  # two calls in a row
        _call(noalloc, torch, dev, x, W, A, B, alpha, rings, y)
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert pool.get(CU_MEMPOOL_ATTR_USED_MEM_HIGH) == pool.get(CU_MEMPOOL_ATTR_USED_MEM_CURRENT), \
        "the no-allocation entry point drew memory from the device pool"
    assert free1 == free0, "device free memory changed across the no-allocation calls"
    for i, (x, W, A, B, alpha, rings, dev, ref, y) in enumerate(cases):
        got = y.cpu().numpy()
        err = _rel(got, ref)
        assert err <= TOL, f"call {i + 1} vs the oracle: rel max error {err:.3e}"
        y2 = torch.full_like(y, float("nan"))
        _call(lib.aos_lora_op_f32_dev, torch, dev, x, W, A, B, alpha, rings, y2)
        torch.cuda.synchronize()
        err2 = _rel(got, y2.cpu().numpy())
        assert err2 <= TOL, f"call {i + 1} vs aos_lora_op_f32_dev: rel max error {err2:.3e}"


def test_no_alloc_rejects_sizes_beyond_its_scratch():
    torch = pytest.importorskip("torch")
    _, noalloc = _bind()
    T, H, Od, N, r = 300, 64, 64, 4, 64  # 300 * 8 * 64 = 153600 > 131072
    x, W, A, B, alpha, rings = _inputs(3, T, H, Od, N, r)
    dev = {k: torch.from_numpy(v).cuda() for k, v in (("x", x), ("W", W), ("A", A), ("B", B), ("alpha", alpha))}
    dev["rings"] = torch.from_numpy(rings.view(np.uint8).copy()).cuda()
    y = torch.zeros((T, Od), device="cuda")
    rc = noalloc(dev["x"].data_ptr(), T, H, Od, dev["W"].data_ptr(), dev["A"].data_ptr(), dev["B"].data_ptr(), N, r,
                 dev["alpha"].data_ptr(), dev["rings"].data_ptr(), y.data_ptr(), None)
    assert rc == -1  # AOS_ERR_INVALID
    assert "exceeds the fixed scratch" in aos.last_error()
