"""Build liblcpp_b200.so in-tree for sm_100a.

Every .cu under csrc/ is compiled with nvcc for sm_100a
(-gencode arch=compute_100a,code=sm_100a) into _build/, then linked into
lcpp_b200/liblcpp_b200.so next to the Python binding.  The CUDA runtime is
linked statically, so the library depends only on the driver.

Usage: python luisacompute-parallelprimitive_b200/build.py [--verbose-ptxas] [-j N]
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
LIB = PKG / "lcpp_b200" / "liblcpp_b200.so"
# NVIDIA CUB behind a small C ABI: the comparison arm of bench.py --impl cub
# only, kept out of liblcpp_b200
CUB_SRC = PKG / "cub_arm" / "cub_arm.cu"
CUB_LIB = PKG / "lcpp_b200" / "libcub_arm.so"
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo", "-O3", "-std=c++17",
    "-Xcompiler", "-fPIC,-O3",
    "--expt-relaxed-constexpr",
]


def _needs_rebuild(obj: Path, src: Path) -> bool:
    if not obj.exists():
        return True
    deps = [src, *CSRC.glob("*.cuh"), *(PKG.parent / "include").glob("*.h"), *(PKG.parent / "include").glob("*.cuh"),
            Path(__file__)]
    return any(d.stat().st_mtime > obj.stat().st_mtime for d in deps)


def _compile(src: Path, verbose_ptxas: bool) -> tuple[Path, str]:
    obj = BUILD / (src.stem + ".o")
    if not _needs_rebuild(obj, src):
        return obj, ""
    cmd = [NVCC, *NVCC_FLAGS, "-c", str(src), "-o", str(obj)]
    if verbose_ptxas:
        cmd += ["-Xptxas", "-v"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{r.stdout}\n{r.stderr}")
    return obj, r.stderr


def build(verbose_ptxas: bool = False, jobs: int | None = None) -> Path:
    BUILD.mkdir(exist_ok=True)
    sources = sorted(CSRC.glob("*.cu"))
    jobs = jobs or min(len(sources), os.cpu_count() or 1)
    with cf.ThreadPoolExecutor(max_workers=jobs) as ex:
        results = list(ex.map(lambda s: _compile(s, verbose_ptxas), sources))
    if verbose_ptxas:
        for _, log in results:
            if log:
                sys.stderr.write(log)
    objs = [o for o, _ in results]
    if not LIB.exists() or any(o.stat().st_mtime > LIB.stat().st_mtime for o in objs):
        cmd = [NVCC, "-shared", "-gencode", "arch=compute_100a,code=sm_100a", "-o", str(LIB),
               *map(str, objs)]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    if CUB_SRC.exists() and (not CUB_LIB.exists() or CUB_SRC.stat().st_mtime > CUB_LIB.stat().st_mtime):
        cmd = [NVCC, *NVCC_FLAGS, "-shared", str(CUB_SRC), "-o", str(CUB_LIB)]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed for {CUB_SRC.name}:\n{r.stdout}\n{r.stderr}")
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--verbose-ptxas", action="store_true")
    ap.add_argument("-j", type=int, default=None)
    a = ap.parse_args()
    print(build(a.verbose_ptxas, a.j))
