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
