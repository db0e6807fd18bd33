"""aos_lora_op_f32_noalloc_dev: the fp32 LoRA op for callers that cannot
allocate device memory (a fixed device-memory budget, an open CUDA graph
capture on the same device, or a latency-critical loop).  Its scratch is a
fixed device array inside the library instead of a per-call allocation.

Checked through the C ABI against aos_lora_op_f32_dev, the entry point that
allocates its scratch, on two calls in a row, with the same 1e-5 relative
tolerance as the other fp32 LoRA tests.  This file is named so that pytest
collects it last."""
import ctypes as C

import numpy as np
import pytest

from tests.aos_import import aos

pytestmark = pytest.mark.gpu

TOL = 1e-5  # fp32 op tolerance, as in tests/test_lora_f32_gpu.py
SCRATCH_FLOATS = 131072  # fixed scratch of the no-allocation entry point


def _bind():
    lib = aos.lib()
    vp, u32 = C.c_void_p, C.c_uint32
    f = lib.aos_lora_op_f32_noalloc_dev
    f.restype = C.c_int
    f.argtypes = [vp, u32, u32, u32, vp, vp, vp, u32, u32, vp, vp, vp, vp]
    return lib, f


def _inputs(torch, seed, T, H, O, N, r):
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    x = torch.randn(T, H, generator=g, device="cuda")
    W = torch.randn(O, H, generator=g, device="cuda") * 0.02
    A = torch.randn(N, r, H, generator=g, device="cuda") * 0.02
    B = torch.randn(N, O, r, generator=g, device="cuda") * 0.02
    alpha = torch.linspace(1.0, 2.0 * r, N, device="cuda")
    logits = np.random.default_rng(seed).standard_normal((T, N)).astype(np.float32)
    rings, _, _ = aos.route_batch(logits, k=min(4, N))
    rings_d = torch.from_numpy(rings.view(np.uint8).copy()).cuda()
    return x, W, A, B, alpha, rings_d


def _run(fn, torch, x, W, A, B, alpha, rings_d):
    T, H = x.shape
    O = W.shape[0]
    N, r, _ = A.shape
    y = torch.full((T, O), float("nan"), device="cuda")
    rc = fn(x.data_ptr(), T, H, O, W.data_ptr(), A.data_ptr(), B.data_ptr(), N, r, alpha.data_ptr(),
            rings_d.data_ptr(), y.data_ptr(), None)
    assert rc == 0, aos.last_error()
    torch.cuda.synchronize()
    return y


def test_no_alloc_matches_allocating_entry_point_twice():
    torch = pytest.importorskip("torch")
    lib, noalloc = _bind()
    # two calls in a row, the second with a different shape that reuses more of the scratch
    for seed, (T, H, O, N, r) in ((1, (64, 2048, 2048, 8, 16)), (2, (200, 512, 384, 5, 64))):
        assert T * 8 * r <= SCRATCH_FLOATS
        x, W, A, B, alpha, rings_d = _inputs(torch, seed, T, H, O, N, r)
        ref = _run(lib.aos_lora_op_f32_dev, torch, x, W, A, B, alpha, rings_d)
        got = _run(noalloc, torch, x, W, A, B, alpha, rings_d)
        err = (got - ref).abs().max().item() / max(ref.abs().max().item(), 1e-30)
        assert err <= TOL, f"call with seed {seed}: rel max error {err:.3e}"


def test_no_alloc_rejects_sizes_beyond_its_scratch():
    torch = pytest.importorskip("torch")
    _, noalloc = _bind()
    T, H, O, N, r = 300, 64, 64, 4, 64  # 300 * 8 * 64 = 153600 > 131072
    x, W, A, B, alpha, rings_d = _inputs(torch, 3, T, H, O, N, r)
    y = torch.zeros((T, O), device="cuda")
    rc = noalloc(x.data_ptr(), T, H, O, W.data_ptr(), A.data_ptr(), B.data_ptr(), N, r, alpha.data_ptr(),
                 rings_d.data_ptr(), y.data_ptr(), None)
    assert rc == -1  # AOS_ERR_INVALID
    assert "exceeds the fixed scratch" in aos.last_error()
