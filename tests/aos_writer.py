"""Test helper: writes `.aos` archives the way the reference's AosWriter does
(crates/adapteros-aos/src/writer.rs:216-390): 64-byte header, one 80-byte
index entry per segment, the payloads back to back, then the manifest bytes.
Every entry carries the manifest's scope hash (first 16 bytes of BLAKE3 of
metadata.scope_path) and its payload's BLAKE3.  tests/test_aos_archive.py
pins this writer by rebuilding the reference's own archives byte for byte.
Hashes come from the CPU oracle (test infrastructure)."""
import json
import struct

from oracle import oracle as O

TAGS = {"canonical": 0, "mlx": 1, "metal": 2, "coreml": 3}


def blake3(data: bytes) -> bytes:
    return O.blake3(data)


def write_aos(segments, manifest, magic=b"AOS\x00"):
    """segments: [(backend, payload bytes)]; manifest: dict (serialised with
    indent=2, as serde_json::to_vec_pretty) or raw bytes."""
    man = manifest if isinstance(manifest, (bytes, bytearray)) else json.dumps(manifest, indent=2).encode()
    scope = json.loads(man)["metadata"]["scope_path"]
    scope_hash = blake3(scope.encode())[:16]
    off = 64 + 80 * len(segments)
    index = b""
    for i, (backend, payload) in enumerate(segments):
        index += struct.pack("<IHHQQ", i, TAGS[backend], 0, off, len(payload)) + scope_hash + blake3(payload) + bytes(8)
        off += len(payload)
    header = magic + struct.pack("<IQQQQ", 1, 64, len(index), off, len(man)) + bytes(24)
    return header + index + b"".join(p for _, p in segments) + man
