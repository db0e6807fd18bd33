"""Determinism attestation (FusedKernels::attest_determinism,
crates/adapteros-lora-kernel-api/src/attestation.rs:130-330).

CPU: DeterminismReport::validate's rules (forbidden fast-math flags, level /
flag consistency, RNG and floating-point modes) and the byte layout that
to_attestation_hash hashes (u32-LE length-prefixed components, flags
sorted).  GPU: the CUDA backend's report validates clean, claims bit-exact
determinism, carries the kernel hash of the sources it was built from, and
its attestation hash (BLAKE3 on the GPU) equals the oracle's BLAKE3 of the
same bytes."""
import pytest

from oracle import oracle as O
from tests.aos_import import aos


def report(**kw):
    r = {"backend_type": "Cuda", "rng_seed_method": "HkdfSeeded", "floating_point_mode": "Deterministic",
         "determinism_level": "bit_exact", "deterministic": True, "kernel_hash": "ab" * 32, "kernel_verified": True,
         "runtime_version": "cuda runtime 12.9", "device_id": "cuda:0 0000:1b:00.0",
         "compiler_flags": ["-O3", "-fno-fast-math", "-lineinfo"]}
    r.update(kw)
    return r


def test_validate_rules():
    assert aos.validate_report(report()) == []  # -fno-fast-math is not a forbidden flag
    assert any("Forbidden compiler flag" in e for e in aos.validate_report(report(compiler_flags=["-ffast-math"])))
    assert any("Forbidden" in e for e in
               aos.validate_report(report(compiler_flags=["-Xcompiler=-funsafe-math-optimizations"])))
    assert aos.validate_report(report(deterministic=False, determinism_level="none")) == [
        "Overall deterministic flag is false"]
    assert len(aos.validate_report(report(deterministic=False))) == 2
    assert aos.validate_report(report(floating_point_mode="FastMath"))
    assert aos.validate_report(report(rng_seed_method="SystemEntropy"))
    assert aos.validate_report(report(kernel_hash=""))


def test_attestation_hash_layout():
    b = aos.attestation_hash_input(report(compiler_flags=["-b", "-a"]))
    comps, i = [], 0
    while i < len(b):
        n = int.from_bytes(b[i:i + 4], "little")
        comps.append(b[i + 4:i + 4 + n])
        i += 4 + n
    assert comps == [b"Cuda", b"HkdfSeeded", b"Deterministic", b"bit_exact", bytes.fromhex("ab" * 32), b"\x01",
                     b"cuda runtime 12.9", b"cuda:0 0000:1b:00.0", b"-a", b"-b"]
    # different configurations give different hashes
    h1 = O.blake3(aos.attestation_hash_input(report()))
    h2 = O.blake3(aos.attestation_hash_input(report(device_id="cuda:1 x")))
    assert h1 != h2


@pytest.mark.gpu
def test_cuda_report():
    g = aos.CudaKernels(256, 2, 1, 128, 384, 512, 1, max_batch=8, kv_num_blocks=16, max_seq_len=64,
                        lora_rank_capacity=64, lora_max_adapters=2)
    try:
        rep = g.attest_determinism()
    finally:
        g.close()
    assert rep["violations"] == []
    assert rep["determinism_level"] == "bit_exact" and rep["deterministic"] and not rep["fast_math"]
    assert rep["kernel_verified"] and len(rep["kernel_hash"]) == 64
    assert "-fno-fast-math" in " ".join(rep["compiler_flags"])
    assert rep["attestation_hash"] == O.blake3(aos.attestation_hash_input(rep)).hex()
