"""The C++ mirror of the FusedKernels surface (include/aos_fused_kernels.hpp,
crates/adapteros-lora-kernel-api/src/lib.rs:308-716) compiles against the
C ABI it wraps, links against the in-tree libaoscuda.so and reports errors
the reference way: construction throws with aos_last_error's message
(FusedKernels constructors return Result::Err), and without a device the
library refuses instead of falling back to the CPU."""
import os
import shutil
import subprocess

import pytest

from tests.aos_import import aos

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

PROG = r"""
#include <cstdio>
#include "aos_fused_kernels.hpp"

static int try_init(const aos_model_config& cfg) {
    try {
        adapteros::CudaKernels k(cfg);
        std::printf("created %s\n", k.device_name().c_str());
        return 0;
    } catch (const std::runtime_error& e) {
        std::printf("error: %s\n", e.what());
        return 1;
    }
}

int main() {
    aos_model_config bad{};  // head_dim 0: rejected before any device work
    aos_model_config cfg{};
    cfg.hidden = 256; cfg.n_heads = 2; cfg.n_kv_heads = 1; cfg.head_dim = 128;
    cfg.intermediate = 384; cfg.vocab = 1000; cfg.n_layers = 1;
    cfg.rms_eps = 1e-5f; cfg.rope_theta = 1e6f; cfg.max_batch = 8;
    cfg.kv_block_size = 16; cfg.kv_num_blocks = 64; cfg.max_seq_len = 256;
    cfg.lora_rank_capacity = 64; cfg.lora_max_adapters = 4; cfg.device = 0;
    const int a = try_init(bad);
    const int b = try_init(cfg);
    std::printf("codes %d %d\n", a, b);
    return 0;
}
"""


def test_mirror_compiles_links_and_reports_errors(tmp_path):
    gxx = shutil.which("g++")
    if gxx is None:
        pytest.skip("g++ not installed")
    src = tmp_path / "mirror.cpp"
    src.write_text(PROG)
    exe = tmp_path / "mirror"
    libdir = os.path.dirname(aos.LIB_PATH)
    cmd = [gxx, "-std=c++17", "-Wall", "-Werror", "-I", os.path.join(ROOT, "include"), str(src),
           "-L", libdir, "-l:" + os.path.basename(aos.LIB_PATH), "-Wl,-rpath," + libdir,
           "-Wl,--allow-shlib-undefined", "-o", str(exe)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    out = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert out.returncode == 0, out.stderr
    lines = out.stdout.splitlines()
    assert lines[0].startswith("error: aos_init") and "unsupported config" in lines[0]
    if aos.device_count() == 0:
        assert lines[1].startswith("error: aos_init") and lines[-1] == "codes 1 1", out.stdout
    else:
        assert lines[1].startswith("created") and lines[-1] == "codes 1 0", out.stdout
