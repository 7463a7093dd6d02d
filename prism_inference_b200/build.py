"""Build libprism_moe.so (the CUDA kernels + the C ABI of include/prism_moe.h) in-tree.

    python -m prism_inference_b200.build [--force]

Every .cu file under csrc/ is compiled for sm_100a only
(-gencode arch=compute_100a,code=sm_100a) and linked with the static CUDA runtime;
the driver API (cuTensorMapEncodeTiled) is resolved at run time through
cudaGetDriverEntryPoint, so nothing links against libcuda.  csrc/prism_bench.cpp, a C++
caller that uses only include/prism_moe.h, is linked against the library as
prism_inference_b200/prism_bench.
"""
from __future__ import annotations

import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
OUT = PKG / "libprism_moe.so"
BENCH = PKG / "prism_bench"
BUILD = PKG / "_build"
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-lineinfo", "-std=c++17",
         "-Xcompiler", "-fPIC,-O3", "-I", str(PKG.parent / "include"), "--expt-relaxed-constexpr",
         "-diag-suppress", "128,550"]


def _compile(src: Path) -> Path:
    obj = BUILD / (src.stem + ".o")
    deps = [src] + list(CSRC.glob("*.cuh")) + [PKG.parent / "include" / "prism_moe.h"]
    if obj.exists() and obj.stat().st_mtime >= max(d.stat().st_mtime for d in deps):
        return obj
    cmd = [NVCC, *FLAGS, "-c", str(src), "-o", str(obj)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src.name}:\n{r.stdout}\n{r.stderr}")
    return obj


def build(force: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    srcs = sorted(CSRC.glob("*.cu"))
    if force:
        for o in BUILD.glob("*.o"):
            o.unlink()
    with ThreadPoolExecutor(max_workers=min(8, len(srcs))) as ex:
        objs = list(ex.map(_compile, srcs))
    if force or not OUT.exists() or OUT.stat().st_mtime < max(o.stat().st_mtime for o in objs):
        cmd = [NVCC, "-gencode", "arch=compute_100a,code=sm_100a", "-shared", "-Xcompiler", "-fPIC",
               "-cudart", "static", *map(str, objs), "-o", str(OUT)]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    src = CSRC / "prism_bench.cpp"
    deps = [src, OUT, PKG.parent / "include" / "prism_moe.h"]
    if force or not BENCH.exists() or BENCH.stat().st_mtime < max(d.stat().st_mtime for d in deps):
        cmd = [NVCC, "-O2", "-std=c++17", "-I", str(PKG.parent / "include"), str(src), "-L", str(PKG),
               "-lprism_moe", "-Xlinker", "-rpath,$ORIGIN", "-o", str(BENCH)]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"prism_bench build failed:\n{r.stdout}\n{r.stderr}")
    return OUT


if __name__ == "__main__":
    print(build(force="--force" in sys.argv))
