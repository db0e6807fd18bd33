"""Copies a few of the reference's own `.aos` test archives into
tests/golden/aos/ and writes tests/golden/aos_golden.json.

Runs only where the reference tree is present (it is not on GPU boxes); the
copied archives and the JSON are committed.  Sources: the reference's
test_data/adapters directory (archives written by its AosWriter; the ones
under objects/ are content-addressed: the file name is the BLAKE3 of the
file), plus its corrupted_adapter.aos (three header bytes changed,
crates/adapteros-lora-worker/tests/create_test_adapters.rs:118-129) and a
pre-index archive (flags bit 0 clear).

Recorded per archive, all taken from the reference's own bytes (none is
computed here): the expected layout outcome (the writer.rs:407-558 message),
the file's BLAKE3 (from its content-addressed name, when it has one), and
each index entry's payload offset, length, scope hash and payload hash, with
the manifest's metadata.scope_path.

usage: python tests/golden/make_aos_golden.py [reference_root]
"""
import glob
import json
import os
import shutil
import struct
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
REF = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("AOS_REFERENCE_ROOT", "")


def entries(b):
    flags, io, isz, mo, ms = struct.unpack_from("<IQQQQ", b, 4)
    out = []
    for i in range(isz // 80):
        e = b[io + 80 * i: io + 80 * (i + 1)]
        sid, tag = struct.unpack_from("<IH", e, 0)
        off, ln = struct.unpack_from("<QQ", e, 8)
        out.append({"segment_id": sid, "backend_tag": tag, "offset": off, "len": ln,
                    "scope_hash": e[24:40].hex(), "weights_hash": e[40:72].hex()})
    return out, json.loads(b[mo:mo + ms])


def main():
    td = os.path.join(REF, "test_data", "adapters")
    objs = sorted(glob.glob(os.path.join(td, "objects", "**", "*.aos"), recursive=True))
    by_size = {}
    for f in objs:
        by_size.setdefault(os.path.getsize(f), f)
    picks = [by_size[k] for k in sorted(by_size)][:6]
    out_dir = os.path.join(HERE, "aos")
    os.makedirs(out_dir, exist_ok=True)
    cases = []
    for f in picks:
        b = open(f, "rb").read()
        segs, man = entries(b)
        name = os.path.basename(f)
        shutil.copyfile(f, os.path.join(out_dir, name))
        cases.append({"file": name, "status": "ok", "file_blake3": name[:-4], "segments": segs,
                      "scope_path": man["metadata"]["scope_path"]})
    extra = [("default/test_adapter/test_adapter.aos", "v2_test_adapter.aos", "ok"),
             ("corrupted_adapter.aos", "corrupted_adapter.aos", "Corrupted / needs retrain: reserved header bytes non-zero"),
             ("adapter_1.aos", "pre_index_adapter_1.aos", "Corrupted / needs retrain: missing segment index")]
    for src, dst, status in extra:
        b = open(os.path.join(td, src), "rb").read()
        shutil.copyfile(os.path.join(td, src), os.path.join(out_dir, dst))
        case = {"file": dst, "status": status}
        if status == "ok":
            segs, man = entries(b)
            case.update({"segments": segs, "scope_path": man["metadata"]["scope_path"]})
        cases.append(case)
    json.dump({"source": "reference test_data/adapters", "cases": cases},
              open(os.path.join(HERE, "aos_golden.json"), "w"), indent=1)
    print(len(cases), "archives")


if __name__ == "__main__":
    main()
