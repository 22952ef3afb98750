"""Build recipe for oracle/_ref/: the reference's own CUDA factor kernel behind a C-ABI
launcher (oracle/ref_factors.cu).  TEST INFRASTRUCTURE ONLY: tests/ load the result to
check and time the product's factor stage beside the reference kernel.

    python -m oracle.build_ref [--force]

The kernel source stays where it lies in the reference checkout (its
src/models/ops/csrc/vdn_delta_factors.cuh); nothing of it is copied here.  The flags
are the reference builder's (src/models/linear_attention/paper_factor.py:85-93):
-O3 -std=c++17 and compute_100/sm_100.  When the checkout is absent (a GPU box gets
only the prebuilt oracle/_ref/libref_factors.so) the build is skipped and tests that
need the library skip.
"""
from __future__ import annotations

import argparse
import hashlib
import os
import subprocess
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "_ref"
LIB = OUT / "libref_factors.so"
SRC = HERE / "ref_factors.cu"
FLAGS = ["-O3", "-std=c++17", "-gencode", "arch=compute_100,code=sm_100", "-Xcompiler", "-fPIC",
         "-shared", "-cudart", "static"]


def reference_csrc() -> Path:
    root = Path(os.environ.get("VDN_REFERENCE_ROOT", "/root/reference"))
    return root / "src" / "models" / "ops" / "csrc"


def build(force: bool = False) -> Path | None:
    csrc = reference_csrc()
    header = csrc / "vdn_delta_factors.cuh"
    if not header.is_file():
        return LIB if LIB.exists() else None
    h = hashlib.sha256()
    for p in (SRC, header):
        h.update(p.read_bytes())
    h.update(" ".join(FLAGS).encode())
    stamp = OUT / "libref_factors.stamp"
    if not force and LIB.exists() and stamp.exists() and stamp.read_text() == h.hexdigest():
        return LIB
    OUT.mkdir(exist_ok=True)
    nvcc = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda")) / "bin" / "nvcc"
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [str(nvcc), *FLAGS, f"-I{csrc}", str(SRC), "-o", str(tmp)]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode:
        raise RuntimeError(f"reference factor kernel build failed:\n{res.stderr}")
    os.replace(tmp, LIB)
    stamp.write_text(h.hexdigest())
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    print(build(force=ap.parse_args().force))
