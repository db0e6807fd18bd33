"""`.aos` adapter archives and BLAKE3, CPU side.

- The oracle's BLAKE3 (a restatement of the `blake3` crate 1.8.3 that the
  reference calls through B3Hash, adapteros-infra-common/src/hash.rs:22-36) is
  pinned by the empty-input digest of adapteros-model-hub/src/integrity.rs:
  465-470 and by the reference's own archives (tests/golden/aos/): every
  index entry's payload hash, the scope hash of metadata.scope_path, and the
  content-addressed file names (name = BLAKE3 of the file).
- Its two tree constructions (level by level, and the specification's
  incremental chaining-value stack) agree at sizes past the fixtures'.
- The product's context-free layout parse (aos_archive_parse) follows
  AosWriter::parse_header_bytes / parse_segments (writer.rs:407-558) rule for
  rule and message for message, checked against the oracle's rule codes on
  the fixtures and on planted corruptions.
- The test writer (tests/aos_writer.py) rebuilds the reference archives byte
  for byte, so archives the GPU tests write have the reference's layout.
"""
import json
import os
import struct

import numpy as np
import pytest

from oracle import oracle as O
from tests.aos_import import aos
from tests.aos_writer import write_aos

GOLD = os.path.join(os.path.dirname(__file__), "golden")
CASES = json.load(open(os.path.join(GOLD, "aos_golden.json")))["cases"]


def load(name):
    return open(os.path.join(GOLD, "aos", name), "rb").read()


def ok_cases():
    return [c for c in CASES if c["status"] == "ok"]


def test_blake3_known_answers():
    assert O.blake3(b"").hex() == "af1349b9f5f9a1a6a0404dea36dcc9499bcb25c9adc112b7cc9a93cae41f3262"
    n_payload = n_file = 0
    for c in ok_cases():
        b = load(c["file"])
        if "file_blake3" in c:
            assert O.blake3(b).hex() == c["file_blake3"], c["file"]
            n_file += 1
        for s in c["segments"]:
            payload = b[s["offset"]: s["offset"] + s["len"]]
            assert O.blake3(payload).hex() == s["weights_hash"], c["file"]
            assert O.blake3(c["scope_path"].encode())[:16].hex() == s["scope_hash"], c["file"]
            n_payload += 1
    assert n_file >= 5 and n_payload >= 7


def test_blake3_tree_forms_agree():
    rng = np.random.default_rng(0)
    data = rng.integers(0, 256, (5 << 20) + 333, dtype=np.uint8).tobytes()
    for n in [0, 1, 63, 64, 65, 1023, 1024, 1025, 2047, 2048, 2049, 3 * 1024, 64 * 1024 - 1, 64 * 1024,
              64 * 1024 + 1, 65 * 1024, 129 * 1024 + 5, 4096 * 1024, 4096 * 1024 + 1, len(data)]:
        assert O.blake3(data[:n]) == O.blake3(data[:n], incremental=True), n


def test_oracle_validation_of_fixtures():
    for c in CASES:
        rc, n = O.aos_validate(load(c["file"]))
        if c["status"] == "ok":
            assert rc == 0 and n == len(c["segments"]), c["file"]
        elif "reserved" in c["status"]:
            assert rc == 4
        elif "missing segment index" in c["status"]:
            assert rc == 5


def test_archive_parse_matches_golden():
    for c in CASES:
        b = load(c["file"])
        if c["status"] != "ok":
            with pytest.raises(aos.AosError, match=c["status"]):
                aos.archive_parse(b)
            continue
        info, segs = aos.archive_parse(b)
        assert info["n_segments"] == len(c["segments"])
        for got, want in zip(segs, c["segments"]):
            assert got["segment_id"] == want["segment_id"]
            assert aos.BACKEND_TAGS.index(got["backend"]) == want["backend_tag"]
            assert (got["offset"], got["len"]) == (want["offset"], want["len"])
            assert got["scope_hash"] == want["scope_hash"] and got["weights_hash"] == want["weights_hash"]


def _corrupt(b, what):
    b = bytearray(b)
    flags, io, isz, mo, ms = struct.unpack_from("<IQQQQ", b, 4)
    if what == "small":
        return bytes(b[:63])
    if what == "magic":
        b[0:4] = b"ZIP!"
    elif what == "index_offset":
        struct.pack_into("<Q", b, 8, 72)
    elif what == "reserved":
        b[60] = 1
    elif what == "flags":
        struct.pack_into("<I", b, 4, 0)
    elif what == "index_beyond":
        struct.pack_into("<Q", b, 16, len(b))
    elif what == "index_align":
        struct.pack_into("<Q", b, 16, 81)
    elif what == "manifest_beyond":
        struct.pack_into("<Q", b, 32, len(b))
    elif what == "manifest_overlap":
        struct.pack_into("<Q", b, 24, 100)
    elif what == "tag":
        struct.pack_into("<H", b, io + 4, 9)
    elif what == "seg_index":
        struct.pack_into("<Q", b, io + 8, 100)
    elif what == "seg_manifest":
        struct.pack_into("<Q", b, io + 16, mo)
    elif what == "seg_hash":
        off = struct.unpack_from("<Q", b, io + 8)[0]
        b[off + 40] ^= 1
    return bytes(b)


CORRUPTIONS = [
    ("small", 1, "file too small for AOS header"),
    ("magic", 2, "invalid AOS magic"),
    ("index_offset", 3, "invalid header layout"),
    ("reserved", 4, "reserved header bytes non-zero"),
    ("flags", 5, "missing segment index"),
    ("index_beyond", 6, "index beyond file"),
    ("index_align", 7, "index size not 80-byte aligned"),
    ("manifest_beyond", 8, "manifest beyond file"),
    ("manifest_overlap", 9, "manifest overlaps index/segments"),
    ("tag", 10, "Unknown backend tag: 9"),
    ("seg_index", 11, "segment overlaps index"),
    ("seg_manifest", 12, "segment overlaps manifest"),
]


@pytest.mark.parametrize("what,code,msg", CORRUPTIONS)
def test_planted_corruptions(what, code, msg):
    good = load(ok_cases()[0]["file"])
    bad = _corrupt(good, what)
    assert O.aos_validate(bad)[0] == code
    with pytest.raises(aos.AosError, match=msg):
        aos.archive_parse(bad)


def test_payload_corruption_is_a_hash_failure_not_a_layout_failure():
    good = load(ok_cases()[0]["file"])
    bad = _corrupt(good, "seg_hash")
    assert O.aos_validate(bad)[0] == 14
    aos.archive_parse(bad)  # layout still fine: the hash check needs the device


def test_writer_rebuilds_reference_archives():
    for c in ok_cases():
        b = load(c["file"])
        info, segs = aos.archive_parse(b)
        man = b[info["manifest_offset"]: info["manifest_offset"] + info["manifest_size"]]
        parts = [(aos.BACKEND_TAGS[s["backend_tag"]], b[s["offset"]: s["offset"] + s["len"]]) for s in c["segments"]]
        assert write_aos(parts, man, magic=b[:4]) == b, c["file"]
