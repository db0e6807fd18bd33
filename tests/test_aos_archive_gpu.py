""".aos archives, BLAKE3 and adapter buffer fingerprints on the GPU.

- GPU BLAKE3 (blake3.cu, many messages per launch) equals the pinned CPU
  oracle at sizes from 0 bytes to 96 MB, on host bytes and on device buffers
  at unaligned offsets, and reproduces the reference archives' payload hashes.
- aos_archive_verify accepts the reference archives and names the segment
  whose payload was changed.
- aos_adapter_load_aos (LifecycleLoader::load_from_aos_static + the MLX
  adapter rules) decodes bit-identically to the same weights loaded through
  the array entry point: rank 8 as is, rank 4 padded to 8 columns with the
  scale alpha / 4 kept, backend segment selection, and every refusal the
  loader makes (tampered payload, per-layer and whole-payload hashes, missing
  scope_path, no canonical segment).
- aos_adapter_fingerprint = BLAKE3(first || last || mid 4 KB) of the
  adapter's canonical buffer (GpuBufferFingerprint, kernel-mtl/src/vram.rs),
  with the samples equal to the host-side canonical bytes, and the
  store / verify baseline semantics of kernel-mtl/src/lib.rs:1737-1793.
"""
import json
import os

import numpy as np
import pytest

from oracle import oracle as O
from tests.aos_import import aos
from tests.aos_writer import write_aos

pytestmark = pytest.mark.gpu

GOLD = os.path.join(os.path.dirname(__file__), "golden")
CASES = json.load(open(os.path.join(GOLD, "aos_golden.json")))["cases"]
MODS = list(aos.MODULES)


@pytest.fixture(scope="module")
def model():
    rng = np.random.default_rng(11)
    return O.HostModel.random(rng, 256, 2, 1, 128, 384, 512, 2)


def make_gpu(m, n_ad=4):
    g = aos.CudaKernels(m.hidden, m.n_heads, m.n_kv_heads, 128, m.inter, m.vocab, m.n_layers, max_batch=8,
                        kv_num_blocks=64, max_seq_len=128, lora_rank_capacity=128, lora_max_adapters=n_ad)
    g.load_host_model(m)
    return g


def st_bytes(tensors):
    """safetensors container of F32 tensors (values exact in bf16)."""
    header, blobs, off = {}, [], 0
    for name, arr in tensors.items():
        raw = np.ascontiguousarray(arr, np.float32).tobytes()
        header[name] = {"dtype": "F32", "shape": list(arr.shape), "data_offsets": [off, off + len(raw)]}
        blobs.append(raw)
        off += len(raw)
    h = json.dumps(header).encode()
    h += b" " * (-len(h) % 8)
    return np.array([len(h)], "<u8").tobytes() + h + b"".join(blobs)


def lora_weights(rng, m, rank, mods):
    out = {}
    for name in mods:
        mi = MODS.index(name)
        o, i = m.mod_shape(mi)
        A = O.bf16_bits_to_f32(O.f32_to_bf16_bits(rng.standard_normal((rank, i), dtype=np.float32) * 0.05))
        B = O.bf16_bits_to_f32(O.f32_to_bf16_bits(rng.standard_normal((o, rank), dtype=np.float32) * 0.05))
        out[name] = (A, B)
    return out


def payload(w, suffix_form=False):
    t = {}
    for name, (A, B) in w.items():
        if suffix_form:
            t[f"{name}.lora_A"], t[f"{name}.lora_B"] = A, B
        else:
            t[f"lora_a.{name}"], t[f"lora_b.{name}"] = A, B
    return st_bytes(t)


def manifest(rank, alpha, mods, scope="unspecified/project/project/unspecified", **extra):
    m = {"adapter_id": "t", "rank": rank, "alpha": alpha, "target_modules": mods,
         "metadata": {"scope_path": scope}}
    m.update(extra)
    return m


def decode(g, m, rings, toks):
    T = len(toks)
    sids = np.arange(T, dtype=np.uint64)
    for s in sids:
        g.kv_alloc(int(s), 64)
    logits, _ = g.run_step_batch(rings, toks, sids)
    for s in sids:
        g.kv_free(int(s))
    return logits


def array_load(g, m, slot, w, rank, alpha, store):
    mods = {}
    for name, (A, B) in w.items():
        o, i = m.mod_shape(MODS.index(name))
        Ap = np.zeros((store, i), np.float32)
        Ap[:rank] = A
        Bp = np.zeros((o, store), np.float32)
        Bp[:, :rank] = B
        for l in range(m.n_layers):
            mods[(l, name)] = (O.f32_to_bf16_bits(Ap), O.f32_to_bf16_bits(Bp))
    g.load_adapter_with_metadata(slot, store, alpha, mods)


def step_inputs(rng, slot, T=4):
    rings = np.zeros(T, aos.RING_DTYPE)
    for t in range(T):
        rings[t]["top_k"] = 1
        rings[t]["indices"][0] = slot
        rings[t]["gates_q15"][0] = 32767
    toks = rng.integers(0, 512, size=T).astype(np.uint32)
    return rings, toks


# ---------------------------------------------------------------- BLAKE3
def test_gpu_blake3_matches_oracle_and_golden(model):
    import torch
    g = make_gpu(model)
    try:
        rng = np.random.default_rng(1)
        data = rng.integers(0, 256, (96 << 20) + 13, dtype=np.uint8)
        for n in [0, 1, 64, 1023, 1024, 1025, 4096, 65535, 65536, 65537, 64 * 1024 * 64 + 1, 5_000_003]:
            assert g.blake3(data[:n].tobytes()) == O.blake3(data[:n].tobytes()).hex(), n
        dev = torch.from_numpy(data).cuda()
        for start, n in [(0, len(data)), (3, 1 << 20), (16, 777777), (5, 0)]:
            assert g.blake3(dev[start:start + n]) == O.blake3(data[start:start + n].tobytes()).hex(), (start, n)
        for c in CASES:
            if c["status"] != "ok":
                continue
            b = open(os.path.join(GOLD, "aos", c["file"]), "rb").read()
            if "file_blake3" in c:
                assert g.blake3(b) == c["file_blake3"]
            for s in c["segments"]:
                assert g.blake3(b[s["offset"]: s["offset"] + s["len"]]) == s["weights_hash"]
            g.archive_verify(b)
            bad = bytearray(b)
            bad[c["segments"][0]["offset"] + 9] ^= 0x40
            with pytest.raises(aos.AosError, match="segment 0 hash mismatch"):
                g.archive_verify(bytes(bad))
    finally:
        g.close()


# ---------------------------------------------------------------- loading
def test_load_aos_matches_array_load(model):
    rng = np.random.default_rng(2)
    w8 = lora_weights(rng, model, 8, ["q_proj", "v_proj", "down_proj"])
    w4 = lora_weights(rng, model, 4, ["k_proj", "o_proj", "up_proj"])
    arch8 = write_aos([("canonical", payload(w8))], manifest(8, 16.0, ["q_proj", "v_proj", "down_proj"]))
    arch4 = write_aos([("canonical", payload(w4, suffix_form=True))], manifest(4, 8.0, ["k_proj", "o_proj", "up_proj"]))
    rings, toks = step_inputs(rng, 0)
    outs = {}
    for how in ("aos", "array"):
        g = make_gpu(model)
        try:
            if how == "aos":
                i8 = g.load_adapter_aos(0, arch8)
                i4 = g.load_adapter_aos(1, arch4, backend="auto")
                assert (i8["rank"], i8["tensor_rank"], i8["storage_rank"], i8["alpha"]) == (8, 8, 8, 16.0)
                assert (i4["rank"], i4["tensor_rank"], i4["storage_rank"], i4["alpha"]) == (4, 4, 8, 8.0)
                assert i8["modules"] == ["q_proj", "v_proj", "down_proj"] and i4["backend"] == "canonical"
            else:
                array_load(g, model, 0, w8, 8, 16.0, 8)
                array_load(g, model, 1, w4, 4, 16.0, 8)  # alpha 16 / 8 columns == 8 / 4
            r2 = rings.copy()
            r2["top_k"] = 2
            r2["indices"][:, 1] = 1
            r2["gates_q15"][:, 0] = 20000
            r2["gates_q15"][:, 1] = 12767
            outs[how] = decode(g, model, r2, toks)
        finally:
            g.close()
    assert outs["aos"].tobytes() == outs["array"].tobytes()


def test_load_aos_backend_selection(model):
    rng = np.random.default_rng(3)
    # v_proj: with one cached position per sequence, q and k do not reach the logits
    wc = lora_weights(rng, model, 8, ["v_proj"])
    wm = lora_weights(rng, model, 8, ["v_proj"])
    arch = write_aos([("canonical", payload(wc)), ("mlx", payload(wm))], manifest(8, 16.0, ["v_proj"]))
    rings, toks = step_inputs(rng, 0)
    got = {}
    for backend, want in (("mlx", wm), ("metal", wc), ("canonical", wc)):
        g = make_gpu(model)
        try:
            info = g.load_adapter_aos(0, arch, backend=backend)
            assert info["backend"] == ("mlx" if backend == "mlx" else "canonical")
            a = decode(g, model, rings, toks)
            g.unload_adapter(0)
            array_load(g, model, 0, want, 8, 16.0, 8)
            assert decode(g, model, rings, toks).tobytes() == a.tobytes(), backend
            got[backend] = a
        finally:
            g.close()
    assert got["mlx"].tobytes() != got["canonical"].tobytes()


def test_load_aos_refusals(model):
    rng = np.random.default_rng(4)
    w = lora_weights(rng, model, 8, ["q_proj"])
    p = payload(w)
    good_man = manifest(8, 16.0, ["q_proj"])
    g = make_gpu(model)
    try:
        # per-layer hashes (BLAKE3 of each tensor's bytes by canonical layer id) and the payload hash
        A, B = w["q_proj"]
        plh = {"transformer.lora_A.q_proj": {"hash": O.blake3(A.astype(np.float32).tobytes()).hex()},
               "transformer.lora_B.q_proj": {"hash": O.blake3(B.astype(np.float32).tobytes()).hex()}}
        ok = write_aos([("canonical", p)], manifest(8, 16.0, ["q_proj"], per_layer_hashes=plh,
                                                    weights_hash=O.blake3(p).hex()))
        g.load_adapter_aos(0, ok)
        g.unload_adapter(0)
        bad_plh = dict(plh)
        bad_plh["transformer.lora_B.q_proj"] = {"hash": "00" * 32}
        with pytest.raises(aos.AosError, match="layer hash mismatch"):
            g.load_adapter_aos(0, write_aos([("canonical", p)], manifest(8, 16.0, ["q_proj"], per_layer_hashes=bad_plh)))
        with pytest.raises(aos.AosError, match="missing tensor 'transformer.lora_A.k_proj'"):
            g.load_adapter_aos(0, write_aos([("canonical", p)], manifest(
                8, 16.0, ["q_proj"], per_layer_hashes={"lora_a.k_proj": {"hash": "00" * 32}})))
        with pytest.raises(aos.AosError, match="adapter hash mismatch"):
            g.load_adapter_aos(0, write_aos([("canonical", p)], manifest(8, 16.0, ["q_proj"],
                                                                          weights_hash="11" * 32)))
        tampered = bytearray(write_aos([("canonical", p)], good_man))
        tampered[64 + 80 + 200] ^= 1
        with pytest.raises(aos.AosError, match="segment 0 hash mismatch"):
            g.load_adapter_aos(0, bytes(tampered))
        no_scope = dict(good_man, metadata={})
        with pytest.raises(aos.AosError, match="missing scope_path"):
            g.load_adapter_aos(0, write_aos_raw_no_scope(p, no_scope))
        with pytest.raises(aos.AosError, match="no canonical segment"):
            g.load_adapter_aos(0, write_aos([("mlx", p)], good_man))
        with pytest.raises(aos.AosError, match="no lora_a/lora_b pair"):
            g.load_adapter_aos(0, write_aos([("canonical", p)], manifest(8, 16.0, ["gate_proj"])))
        assert not g.is_loaded(0)
    finally:
        g.close()


def write_aos_raw_no_scope(p, man):
    """An archive whose manifest has no metadata.scope_path (scope hashes zero)."""
    import struct
    body = json.dumps(man, indent=2).encode()
    idx = struct.pack("<IHHQQ", 0, 0, 0, 144, len(p)) + bytes(16) + O.blake3(p) + bytes(8)
    hdr = b"AOS\x00" + struct.pack("<IQQQQ", 1, 64, 80, 144 + len(p), len(body)) + bytes(24)
    return hdr + idx + p + body


# ---------------------------------------------------------------- fingerprints
def test_adapter_fingerprint(model):
    rng = np.random.default_rng(5)
    w = lora_weights(rng, model, 8, ["q_proj", "down_proj"])
    g = make_gpu(model)
    try:
        g.load_adapter_aos(2, write_aos([("canonical", payload(w))], manifest(8, 16.0, ["q_proj", "down_proj"])))
        size, first, last, mid = g.verify_adapter_buffers(2)
        n_el = 0
        for mi in range(7):
            o, i = model.mod_shape(mi)
            n_el += 8 * i + o * 8
        assert size == model.n_layers * n_el * 2
        assert len(first) == len(last) == len(mid) == 4096
        # layer 0 q_proj lora_A is the first 2048 elements; the last layer's down_proj lora_B the last 2048
        assert first == O.f32_to_bf16_bits(w["q_proj"][0]).tobytes()
        assert last == O.f32_to_bf16_bits(w["down_proj"][1]).tobytes()
        fsize, fhash = g.adapter_fingerprint(2)
        assert fsize == size and fhash == O.blake3(first + last + mid).hex()
        assert not g.verify_gpu_fingerprint(2, size, fhash)  # no baseline yet
        g.store_gpu_fingerprint(2, size, fhash.upper())
        assert g.verify_gpu_fingerprint(2, size, fhash)
        assert not g.verify_gpu_fingerprint(2, size + 2, fhash)
        with pytest.raises(aos.AosError, match="Invalid checkpoint hash hex"):
            g.store_gpu_fingerprint(2, size, "xyz")
        # a different adapter in the same slot no longer matches the baseline
        g.unload_adapter(2)
        w2 = lora_weights(rng, model, 8, ["q_proj", "down_proj"])
        g.load_adapter_aos(2, write_aos([("canonical", payload(w2))], manifest(8, 16.0, ["q_proj", "down_proj"])))
        s2, h2 = g.adapter_fingerprint(2)
        assert s2 == size and h2 != fhash and not g.verify_gpu_fingerprint(2, s2, h2)
        assert g.get_gpu_fingerprints() == {2: (size, fhash)}
        # footprint baseline: the stored fingerprint gave one sample; fewer than two -> within
        assert g.check_memory_footprint(2, size) == (True, 0.0, (float(size), 0.0, 1))
        g.store_gpu_fingerprint(2, size, fhash)
        within, z, (mean, sd, n) = g.check_memory_footprint(2, size)
        assert within and z == 0.0 and n == 2 and sd == 0.0  # identical samples: exact match required
        assert not g.check_memory_footprint(2, size + 1)[0]
        g.store_gpu_fingerprint(2, size + 1000, fhash)
        within, z, (mean, sd, n) = g.check_memory_footprint(2, size)
        assert n == 3 and sd > 0 and within and abs(z - abs(size - mean) / sd) < 1e-12
        assert not g.check_memory_footprint(2, size + 10 ** 6)[0]
        # first check of an adapter without a baseline starts one
        assert g.check_memory_footprint(7, 123) == (True, 0.0, (123.0, 0.0, 1))
    finally:
        g.close()
