"""Build recipe for liblssm_cuda.so (the sm_100a kernels, the C ABI and the C++ engine).

Every .cu / .cpp file under csrc/ is compiled by nvcc for sm_100a only
(-gencode arch=compute_100a,code=sm_100a) and linked into one shared library
next to this file, so the built .so travels with the source tree. Objects go
to _build/ and are rebuilt only when a source or header is newer.
"""

from __future__ import annotations

import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent
CSRC = HERE / "csrc"
OBJ = HERE / "_build"
LIB = HERE / "liblssm_cuda.so"
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-fvisibility=hidden", "--expt-relaxed-constexpr",
          f"-I{ROOT / 'include'}", f"-I{CSRC}"]


def _sources():
    return sorted(list(CSRC.glob("*.cu")) + list(CSRC.glob("*.cpp")))


def _headers_mtime() -> float:
    hs = list(CSRC.glob("*.h")) + list(CSRC.glob("*.cuh")) + list((ROOT / "include").glob("*.h"))
    return max((h.stat().st_mtime for h in hs), default=0.0)


def _compile(src: Path, hdr_mtime: float, extra) -> Path:
    obj = OBJ / (src.name + ".o")
    if obj.exists() and obj.stat().st_mtime >= max(src.stat().st_mtime, hdr_mtime):
        return obj
    cmd = [NVCC, *ARCH, *COMMON, *extra, "-c", str(src), "-o", str(obj)]
    if src.suffix == ".cpp":
        cmd = [NVCC, *COMMON, *extra, "-x", "c++", "-c", str(src), "-o", str(obj)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{r.stdout}\n{r.stderr}")
    return obj


def build(verbose: bool = False, extra=()) -> Path:
    OBJ.mkdir(exist_ok=True)
    hm = _headers_mtime()
    srcs = _sources()
    with ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as ex:
        objs = list(ex.map(lambda s: _compile(s, hm, list(extra)), srcs))
    newest = max(o.stat().st_mtime for o in objs)
    if not LIB.exists() or LIB.stat().st_mtime < newest:
        cmd = [NVCC, *ARCH, "-shared", "-o", str(LIB), *map(str, objs), "-lcudart", "-ldl", "-lpthread"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    build_cpp_shim(verbose)
    if verbose:
        print(LIB)
    return LIB


SHIM_SRC = HERE / "cpp" / "metal_ops.cpp"
SHIM_LIB = HERE / "liblite_ssm_ops.so"


def build_cpp_shim(verbose: bool = False) -> Path:
    """liblite_ssm_ops.so: the C++ `lite_ssm::MetalOps` class (include/lite_ssm_b200/ops.hpp)
    over the C ABI, linked against liblssm_cuda.so next to it (rpath $ORIGIN)."""
    hdr = ROOT / "include" / "lite_ssm_b200" / "ops.hpp"
    newest = max(SHIM_SRC.stat().st_mtime, hdr.stat().st_mtime, LIB.stat().st_mtime)
    if SHIM_LIB.exists() and SHIM_LIB.stat().st_mtime >= newest:
        return SHIM_LIB
    cmd = [os.environ.get("CXX", "g++"), "-O2", "-std=c++17", "-fPIC", "-shared", f"-I{ROOT / 'include'}",
           "-o", str(SHIM_LIB), str(SHIM_SRC), f"-L{HERE}", "-llssm_cuda", "-Wl,-rpath,$ORIGIN", "-ldl"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"C++ shim build failed:\n{r.stdout}\n{r.stderr}")
    if verbose:
        print(SHIM_LIB)
    return SHIM_LIB


if __name__ == "__main__":
    build(verbose=True, extra=sys.argv[1:])
