"""Build libhx_gemm.so (the C-ABI library with every sm_100a kernel) in-tree.

    python hexagon-mlir_b200/build.py

nvcc cross-compiles for sm_100a on a machine without a GPU; the .so lands
in qcom_hexagon_backend/lib/ and travels with the source tree.
"""

from __future__ import annotations

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
OUT = os.path.join(HERE, "qcom_hexagon_backend", "lib", "libhx_gemm.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def sources():
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cu", ".cuh")))


def up_to_date() -> bool:
    if not os.path.exists(OUT):
        return False
    t = os.path.getmtime(OUT)
    deps = sources() + [os.path.join(ROOT, "include", "hx_gemm.h"), __file__]
    return all(os.path.getmtime(s) <= t for s in deps)


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and up_to_date():
        return OUT
    os.makedirs(os.path.dirname(OUT), exist_ok=True)
    cmd = [NVCC, *ARCH, "-lineinfo", "-O3", "-std=c++17", "-Xcompiler", "-fPIC", "-shared",
           "-I" + os.path.join(ROOT, "include"), "-I" + CSRC,
           os.path.join(CSRC, "hx_gemm.cu"), "-o", OUT + ".tmp", "-ldl"]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    subprocess.run(cmd, check=True)
    os.replace(OUT + ".tmp", OUT)
    return OUT


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
