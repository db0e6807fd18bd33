"""The C-ABI library loads without a GPU and exports every function that
include/aos_cuda.h declares; with no device, compute entry points fail with
AOS_ERR_NO_DEVICE instead of falling back to the CPU."""
import ctypes
import os
import re

import numpy as np
import pytest

from tests.aos_import import aos

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include", "aos_cuda.h")


def declared_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(aos_[a-z0-9_]+)\s*\(", src)))


def test_header_declares_entry_points():
    names = declared_functions()
    assert "aos_route_batch" in names and "aos_run_step_batch" in names and len(names) >= 30


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(aos.LIB_PATH)
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, missing


def test_no_cpu_fallback_without_device():
    if aos.device_count() > 0:
        pytest.skip("a device is present")
    pri = np.zeros((2, 4), np.float32)
    with pytest.raises(aos.AosError) as e:
        aos.route_batch(pri)
    assert e.value.code == -7  # AOS_ERR_NO_DEVICE
    with pytest.raises(aos.AosError):
        aos.CudaKernels(256, 2, 1, 128, 256, 100, 1)


def test_ring_layout_is_40_bytes():
    assert ctypes.sizeof(aos.RouterRingC) == 40 and aos.RING_DTYPE.itemsize == 40


@pytest.mark.parametrize("name", ["aos_lora_op_f32_dev", "aos_lora_op_f32_noalloc_dev"])
def test_fp32_op_rejects_misaligned_vector_operands(name):
    """The fp32 LoRA op reads x and A with 16-byte loads: a pointer off a
    16-byte boundary is refused with AOS_ERR_INVALID before any device work
    (the addresses are only checked, never dereferenced, so no GPU is needed)."""
    lib = aos.lib()
    f = getattr(lib, name)
    vp, u32 = ctypes.c_void_p, ctypes.c_uint32
    f.restype = ctypes.c_int
    f.argtypes = [vp, u32, u32, u32, vp, vp, vp, u32, u32, vp, vp, vp, vp]
    good, bad = 0x10000, 0x10004
    for x, a in ((bad, good), (good, bad)):
        rc = f(x, 4, 64, 64, good, a, good, 2, 16, None, good, good, None)
        assert rc == -1  # AOS_ERR_INVALID
        assert "16-byte aligned" in aos.last_error()
