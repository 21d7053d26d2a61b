"""Build libhx_gemm.so (the C-ABI library with every sm_100a kernel) in-tree.

    python hexagon-mlir_b200/build.py [--force] [-v]

nvcc cross-compiles for sm_100a on a machine without a GPU; the .so lands
in qcom_hexagon_backend/lib/ and travels with the source tree.  Each .cu in
csrc/ is one translation unit (the tile-GEMM kernels are split by input kind),
compiled in parallel into _build/ and linked into the shared library.
"""

from __future__ import annotations

import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
OUT = os.path.join(HERE, "qcom_hexagon_backend", "lib", "libhx_gemm.so")
OBJ = os.path.join(HERE, "_build")
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
    os.makedirs(OBJ, exist_ok=True)
    units = sorted(f for f in os.listdir(CSRC) if f.endswith(".cu"))
    flags = [*ARCH, "-lineinfo", "-O3", "-std=c++17", "-Xcompiler", "-fPIC",
             "-I" + os.path.join(ROOT, "include"), "-I" + CSRC]
    if verbose:
        flags.append("-Xptxas=-v")

    def compile_unit(name: str) -> str:
        obj = os.path.join(OBJ, name[:-3] + ".o")
        subprocess.run([NVCC, *flags, "-c", os.path.join(CSRC, name), "-o", obj], check=True)
        return obj

    with ThreadPoolExecutor(max_workers=max(1, min(len(units), os.cpu_count() or 1))) as ex:
        objs = list(ex.map(compile_unit, units))
    subprocess.run([NVCC, *ARCH, "-shared", *objs, "-o", OUT + ".tmp", "-ldl"], check=True)
    os.replace(OUT + ".tmp", OUT)
    return OUT


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
