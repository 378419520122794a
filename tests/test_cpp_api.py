"""The C++ surface (include/lcpp_b200.hpp): compiled on the CPU; on a GPU the
C++ test program (tests/cpp/device_api_test.cpp, written like the
reference's own tests) is built against the library and run."""
from __future__ import annotations

import shutil
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
SRC = ROOT / "tests" / "cpp" / "device_api_test.cpp"
CU_SRC = ROOT / "tests" / "cpp" / "device_compare_test.cu"
CUDA = Path("/usr/local/cuda")
LIBDIR = ROOT / "luisacompute-parallelprimitive_b200" / "lcpp_b200"


def _gxx():
    gxx = shutil.which("g++")
    if gxx is None or not (CUDA / "include" / "cuda_runtime.h").exists():
        pytest.skip("g++ or the CUDA headers are missing")
    return gxx


def test_header_compiles_cleanly():
    gxx = _gxx()
    r = subprocess.run([gxx, "-std=c++17", "-fsyntax-only", "-Wall", "-Wextra", "-Werror", f"-I{ROOT / 'include'}",
                        f"-I{CUDA / 'include'}", str(SRC)], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr


@pytest.mark.gpu
def test_cpp_program_runs(tmp_path):
    gxx = _gxx()
    exe = tmp_path / "device_api_test"
    r = subprocess.run([gxx, "-std=c++17", "-O2", f"-I{ROOT / 'include'}", f"-I{CUDA / 'include'}", str(SRC),
                        "-o", str(exe), f"-L{LIBDIR}", "-llcpp_b200", f"-L{CUDA / 'lib64'}", "-lcudart",
                        f"-Wl,-rpath,{LIBDIR}", f"-Wl,-rpath,{CUDA / 'lib64'}"], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    run = subprocess.run([str(exe)], capture_output=True, text=True, timeout=300)
    assert run.returncode == 0, run.stdout + run.stderr
    assert run.stdout.startswith("OK "), run.stdout


def _nvcc_cmd(out: Path, compile_only: bool):
    nvcc = CUDA / "bin" / "nvcc"
    if not nvcc.exists():
        pytest.skip("nvcc is missing")
    cmd = [str(nvcc), "-std=c++17", "-O2", "-gencode", "arch=compute_100a,code=sm_100a", "--extended-lambda",
           f"-I{ROOT / 'include'}", str(CU_SRC), "-o", str(out)]
    if compile_only:
        return cmd[:-3] + ["-c", str(CU_SRC), "-o", str(out)]
    return cmd + [f"-L{LIBDIR}", "-llcpp_b200", f"-Xlinker=-rpath,{LIBDIR}"]


def test_comparator_header_compiles(tmp_path):
    """The comparator overloads (lcpp_b200_device.cuh through lcpp_b200.hpp) build with nvcc."""
    r = subprocess.run(_nvcc_cmd(tmp_path / "cmp.o", True), capture_output=True, text=True)
    assert r.returncode == 0, r.stderr


@pytest.mark.gpu
def test_comparator_program_runs(tmp_path):
    exe = tmp_path / "device_compare_test"
    r = subprocess.run(_nvcc_cmd(exe, False), capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    run = subprocess.run([str(exe)], capture_output=True, text=True, timeout=300)
    assert run.returncode == 0, run.stdout + run.stderr
    assert run.stdout.startswith("OK "), run.stdout


def test_predicate_encoding_runs_on_cpu(tmp_path, lcpp):
    """Predicate<T> (the C ABI's predicate encoding) is host code: built and run here
    (linked against the library for its status strings; no device call)."""
    gxx = _gxx()
    exe = tmp_path / "predicate_host_test"
    src = ROOT / "tests" / "cpp" / "predicate_host_test.cpp"
    r = subprocess.run([gxx, "-std=c++17", "-O1", "-Wall", "-Wextra", "-Werror", f"-I{ROOT / 'include'}",
                        f"-I{CUDA / 'include'}", str(src), "-o", str(exe), f"-L{LIBDIR}", "-llcpp_b200",
                        f"-Wl,-rpath,{LIBDIR}"], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    run = subprocess.run([str(exe)], capture_output=True, text=True, timeout=60)
    assert run.returncode == 0, run.stdout + run.stderr
    assert run.stdout.startswith("OK "), run.stdout


DIST_SRC = ROOT / "tests" / "cpp" / "dist_api_test.cpp"


def _dist_cmd(gxx, out: Path):
    return [gxx, "-std=c++17", "-O2", "-Wall", "-Wextra", "-Werror", f"-I{ROOT / 'include'}",
            f"-I{CUDA / 'include'}", str(DIST_SRC), "-o", str(out), f"-L{LIBDIR}", "-llcpp_b200",
            f"-L{CUDA / 'lib64'}", "-lcudart", f"-Wl,-rpath,{LIBDIR}", f"-Wl,-rpath,{CUDA / 'lib64'}"]


def test_dist_program_compiles():
    """The multi-process C++ caller of the distributed C ABI builds (-Wall -Werror)."""
    gxx = _gxx()
    r = subprocess.run([gxx, "-std=c++17", "-fsyntax-only", "-Wall", "-Wextra", "-Werror", f"-I{ROOT / 'include'}",
                        f"-I{CUDA / 'include'}", str(DIST_SRC)], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr


@pytest.mark.gpu
def test_dist_program_runs(tmp_path):
    """A C++ program sorts, scans and reduces across one process per GPU
    (up to 8) through the distributed C ABI, with no Python involved."""
    import torch
    gxx = _gxx()
    exe = tmp_path / "dist_api_test"
    r = subprocess.run(_dist_cmd(gxx, exe), capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    ranks = max(1, min(8, torch.cuda.device_count()))
    run = subprocess.run([str(exe), str(ranks)], capture_output=True, text=True, timeout=600)
    assert run.returncode == 0, run.stdout + run.stderr
    assert run.stdout.startswith(f"OK {ranks}"), run.stdout
