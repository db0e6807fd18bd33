"""Build libaoscuda.so in-tree with nvcc for sm_100a.

Usage: python adapter-os_b200/build.py   (or __graft_entry__.build())
Every .cu under csrc/ is compiled with
``-gencode arch=compute_100a,code=sm_100a -O3 -lineinfo`` (no fast-math) and
linked into one shared library with the CUDA runtime linked statically, so the
.so travels with the source tree.
"""
from __future__ import annotations

import glob
import hashlib
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libaoscuda.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")



def _nccl_dir():
    """NCCL of the PyTorch install (the same libnccl.so.2 torch.distributed loads)."""
    try:
        import nvidia.nccl as n  # noqa: PLC0415
        d = list(n.__path__)[0]
        if os.path.exists(os.path.join(d, "include", "nccl.h")):
            return d
    except Exception:
        pass
    return None


NCCL_DIR = _nccl_dir()
NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC,-O3,-fno-fast-math",
    "--expt-relaxed-constexpr",
    "-ccbin", "/usr/bin/g++",
] + (["-I" + os.path.join(NCCL_DIR, "include")] if NCCL_DIR else [])
# the adapter-sharded step calls NCCL (send/recv over NVLink)
LINK_NCCL = (["-L" + os.path.join(NCCL_DIR, "lib"), "-l:libnccl.so.2", "-Xlinker", "-rpath," + os.path.join(NCCL_DIR, "lib")]
             if NCCL_DIR else ["-lnccl"])


def _sources():
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def _headers():
    return sorted(glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(HERE, "..", "include", "*.h")))


def _stamp(paths):
    h = hashlib.sha256()
    for p in paths:
        with open(p, "rb") as f:
            h.update(f.read())
    h.update(" ".join(NVCC_FLAGS).encode())
    return h.hexdigest()


def current_stamp() -> str:
    """Stamp of the kernel sources and flags as they are now (the value a fresh
    build bakes into the library)."""
    return _stamp(_sources() + _headers())


def build(verbose: bool = False, force: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    srcs = _sources()
    hdrs = _headers()
    stamp = _stamp(srcs + hdrs)
    stamp_file = os.path.join(BUILD, "stamp")
    if not force and os.path.exists(LIB) and os.path.exists(stamp_file):
        if open(stamp_file).read() == stamp:
            return LIB
    objs = []
    procs = []
    for s in srcs:
        o = os.path.join(BUILD, os.path.basename(s) + ".o")
        # the build stamp (sources + flags) and the flags themselves go into
        # the library for aos_attest_determinism
        flags_str = " ".join(NVCC_FLAGS).replace('"', "")
        cmd = [NVCC, *NVCC_FLAGS, f'-DAOS_BUILD_STAMP="{stamp}"', f'-DAOS_BUILD_FLAGS="{flags_str}"', "-c", s, "-o", o]
        if verbose:
            print(" ".join(cmd))
        procs.append((s, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT)))
        objs.append(o)
    failed = False
    for s, p in procs:
        out, _ = p.communicate()
        if p.returncode != 0:
            failed = True
            sys.stderr.write(f"nvcc failed on {s}:\n{out.decode()}\n")
        elif verbose and out:
            sys.stderr.write(out.decode())
    if failed:
        raise RuntimeError("CUDA build failed")
    cmd = [NVCC, "-gencode", "arch=compute_100a,code=sm_100a", "-shared", "-o", LIB, *objs,
           "-cudart", "static", "-ccbin", "/usr/bin/g++", "-Xcompiler", "-fPIC", *LINK_NCCL]
    subprocess.run(cmd, check=True)
    with open(stamp_file, "w") as f:
        f.write(stamp)
    return LIB


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv, force="-f" in sys.argv))
