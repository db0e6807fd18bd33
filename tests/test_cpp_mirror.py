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


PLAN_PROG = r"""
#include <cstdio>
#include <fstream>
#include <iterator>
#include "aos_fused_kernels.hpp"

int main(int argc, char** argv) {
    std::ifstream f(argv[1], std::ios::binary);
    std::vector<uint8_t> plan((std::istreambuf_iterator<char>(f)), std::istreambuf_iterator<char>());
    const std::string json = argv[2];
    aos_plan_config pc{};
    if (aos_plan_config_parse(json.c_str(), json.size(), &pc) != AOS_OK || aos_plan_config_validate(&pc) != AOS_OK) {
        std::printf("config error: %s\n", aos_last_error(nullptr));
        return 1;
    }
    aos_model_config rt{};
    rt.max_batch = 8; rt.kv_block_size = 16; rt.kv_num_blocks = 64; rt.max_seq_len = 128;
    rt.lora_rank_capacity = 64; rt.lora_max_adapters = 2; rt.device = 0;
    aos_model_config dims = rt;
    if (aos_model_config_from_plan(plan.data(), plan.size(), &pc, &dims) != AOS_OK) {
        std::printf("dims error: %s\n", aos_last_error(nullptr));
        return 1;
    }
    std::printf("dims %u %u %u %u %u %u %u\n", dims.hidden, dims.n_heads, dims.n_kv_heads, dims.head_dim,
                dims.intermediate, dims.vocab, dims.n_layers);
    try {
        auto k = adapteros::CudaKernels::from_plan(plan, &pc, rt);
        adapteros::IoBuffers io(dims.vocab);
        io.session_id = "s";
        adapteros::RouterRing ring;  // no adapters: k = 0
        io.input_ids = {5, 17, 301};
        adapteros::AosError e = k->run_step(ring, io);  // prompt pass
        if (!e.ok()) { std::printf("step error: %s\n", e.message.c_str()); return 1; }
        std::vector<float> first = io.output_logits;
        io.input_ids = {42};
        e = k->run_step(ring, io);  // one decode token
        if (!e.ok()) { std::printf("step error: %s\n", e.message.c_str()); return 1; }
        std::ofstream o(argv[3], std::ios::binary);
        o.write((const char*)first.data(), first.size() * 4);
        o.write((const char*)io.output_logits.data(), io.output_logits.size() * 4);
        std::printf("position %zu\n", io.position);
    } catch (const std::runtime_error& ex) {
        std::printf("error: %s\n", ex.what());
    }
    return 0;
}
"""

PLAN_CFG = ('{"name": "t", "architecture": "LlamaForCausalLM", "hidden_size": 256, "intermediate_size": 384, '
            '"num_hidden_layers": 2, "num_attention_heads": 2, "num_key_value_heads": 1, '
            '"max_position_embeddings": 4096, "rope_theta": 1000000.0, "vocab_size": 512}')


def test_mirror_load_plan_prompt_then_decode(tmp_path):
    """The FusedKernels sequence of the Rust backend crate through the C++
    mirror: load(plan_bytes) (dimensions from the plan's shapes and the model
    config, aos_init_from_plan), run_step with a 3-token prompt (aos_prefill),
    run_step with one token (aos_run_step_batch).  Without a device the load
    is refused after the dimensions are inferred; on a GPU both steps' logits
    equal the Python mirror's prefill + decode of the same plan bit for bit."""
    import numpy as np
    from oracle import oracle as O
    from tests.test_safetensors import st_bytes
    gxx = shutil.which("g++")
    if gxx is None:
        pytest.skip("g++ not installed")
    rng = np.random.default_rng(12)
    m = O.HostModel.random(rng, 256, 2, 1, 128, 384, 512, 2)
    names = ["q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj"]
    t = {"model.embed_tokens.weight": ("BF16", m.embed), "lm_head.weight": ("BF16", m.lm_head),
         "model.norm.weight": ("BF16", m.final_norm)}
    for l in range(2):
        t[f"model.layers.{l}.input_layernorm.weight"] = ("BF16", m.attn_norm[l])
        t[f"model.layers.{l}.post_attention_layernorm.weight"] = ("BF16", m.mlp_norm[l])
        for mod in range(7):
            t[f"model.layers.{l}.{'self_attn' if mod < 4 else 'mlp'}.{names[mod]}.weight"] = ("BF16", m.w[mod][l])
    plan = st_bytes(t)
    (tmp_path / "plan.st").write_bytes(plan)
    src = tmp_path / "plan.cpp"
    src.write_text(PLAN_PROG)
    exe = tmp_path / "plan"
    libdir = os.path.dirname(aos.LIB_PATH)
    r = subprocess.run([gxx, "-std=c++17", "-Wall", "-Werror", "-I", os.path.join(ROOT, "include"), str(src),
                        "-L", libdir, "-l:" + os.path.basename(aos.LIB_PATH), "-Wl,-rpath," + libdir,
                        "-Wl,--allow-shlib-undefined", "-o", str(exe)], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    out = subprocess.run([str(exe), str(tmp_path / "plan.st"), PLAN_CFG, str(tmp_path / "logits.bin")],
                         capture_output=True, text=True, timeout=300)
    assert out.returncode == 0, out.stdout + out.stderr
    lines = out.stdout.splitlines()
    assert lines[0] == "dims 256 2 1 128 384 512 2", out.stdout
    if aos.device_count() == 0:
        assert lines[1].startswith("error: load:") and "no CUDA device" in lines[1], out.stdout
        return
    assert lines[1] == "position 4", out.stdout
    got = np.fromfile(tmp_path / "logits.bin", dtype=np.float32).reshape(2, 512)
    import torch
    gpu = aos.CudaKernels.from_plan(plan, PLAN_CFG, max_batch=8, kv_num_blocks=64, max_seq_len=128,
                                    lora_rank_capacity=64, lora_max_adapters=2)
    gpu.kv_alloc(9, 128)
    rings = np.zeros(3, O.RING_DTYPE)
    lg = torch.empty((1, 512), dtype=torch.float32, device="cuda")
    gpu.prefill_dev(np.array([9], np.uint64), np.array([3], np.uint32),
                    torch.from_numpy(rings.view(np.uint8).copy()).cuda(),
                    torch.tensor([5, 17, 301], dtype=torch.int32, device="cuda"), logits=lg)
    torch.cuda.synchronize()
    first = lg.cpu().numpy()[0]
    second, _ = gpu.run_step_batch(rings[:1], np.array([42], np.uint32), np.array([9], np.uint64))
    gpu.close()
    assert got[0].tobytes() == first.tobytes()
    assert got[1].tobytes() == second[0].tobytes()


@pytest.mark.gpu
def test_mirror_load_plan_prompt_then_decode_gpu(tmp_path):
    """The same sequence on a GPU (collected by the -m gpu run)."""
    assert aos.device_count() > 0
    test_mirror_load_plan_prompt_then_decode(tmp_path)
