"""C-ABI checks that need no GPU: the library loads, exports every function
declared in include/*.h, answers temp-storage queries and rejects misuse
before touching the device."""
from __future__ import annotations

import ctypes
import re
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
HEADERS = sorted((ROOT / "include").glob("*.h"))
DECL = re.compile(r"^(?:const\s+char\s*\*|lcpp_status|int|void)\s+(lcpp_\w+)\s*\(", re.M)


def declared_functions():
    names = []
    for h in HEADERS:
        names += DECL.findall(h.read_text())
    return sorted(set(names))


def test_headers_declare_functions():
    names = declared_functions()
    assert "lcpp_radix_sort_keys" in names and "lcpp_scan_inclusive_sum" in names
    assert len(names) >= 20


def test_library_exports_every_declared_symbol(lcpp):
    so = lcpp.LIB_PATH
    out = subprocess.run(["nm", "-D", "--defined-only", str(so)], capture_output=True, text=True,
                         check=True).stdout
    exported = set(re.findall(r"\sT\s(lcpp_\w+)$", out, re.M))
    missing = [n for n in declared_functions() if n not in exported]
    assert not missing, missing
    lib = lcpp.lib()
    for n in declared_functions():
        assert hasattr(lib, n)


def test_headers_compile_as_c_and_cpp(tmp_path):
    src = tmp_path / "t.c"
    src.write_text('#include "lcpp_b200.h"\n#include "lcpp_b200_testgen.h"\nint main(void){return 0;}\n')
    subprocess.run(["gcc", "-std=c99", "-Wall", "-Werror", "-I", str(ROOT / "include"), "-c", str(src),
                    "-o", str(tmp_path / "t.o")], check=True)
    subprocess.run(["g++", "-std=c++17", "-Wall", "-Werror", "-x", "c++", "-I", str(ROOT / "include"),
                    "-c", str(src), "-o", str(tmp_path / "t2.o")], check=True)


def test_status_strings(lcpp):
    lib = lcpp.lib()
    assert lib.lcpp_status_string(0) == b"LCPP_OK"
    assert lib.lcpp_status_string(5) == b"LCPP_ERR_LOOKBACK_TIMEOUT"
    assert lib.lcpp_version() >= 100


def test_temp_queries(lcpp):
    R, S, D = lcpp.DeviceRadixSort, lcpp.DeviceScan, lcpp.DeviceReduce
    # empty input needs no temp (tests/device_radix_sort_interface_test.cpp:197-203)
    assert R.GetSortKeysTempStorageBytes(lcpp.I32, 0) == 0
    assert R.GetSortPairsTempStorageBytes(lcpp.U32, lcpp.U32, 0) == 0
    prev = 0
    for n in (1, 1000, 1 << 20, 1 << 28):
        b = R.GetSortKeysTempStorageBytes(lcpp.U32, n)
        assert b >= n * 4 and b > prev and b % 256 == 0
        prev = b
        assert R.GetSortPairsTempStorageBytes(lcpp.U32, lcpp.U32, n) >= b + n * 4
    # 64-bit counts beyond the reference's uint num_items
    assert R.GetSortKeysTempStorageBytes(lcpp.U32, (1 << 32) + 5) > (1 << 34)
    assert S.GetTempStorageBytes(lcpp.I32, 1 << 30) > 0
    assert D.GetTempStorageBytes(lcpp.F32, 1 << 30) > 0
    with pytest.raises(lcpp.LcppError):
        R.GetSortKeysTempStorageBytes(77, 10)


def test_misuse_rejected_without_device(lcpp):
    lib = lcpp.lib()
    vp = ctypes.c_void_p
    fake = vp(0x100000)  # never dereferenced: validation fails first
    # begin_bit > end_bit
    assert lib.lcpp_radix_sort_keys(fake, 1 << 20, fake, fake, 10, 9, 8, 0, lcpp.U32, None) == lcpp.ERR_INVALID_ARG
    # end_bit beyond the key width
    assert lib.lcpp_radix_sort_keys(fake, 1 << 20, fake, fake, 10, 0, 33, 0, lcpp.U32, None) == lcpp.ERR_INVALID_ARG
    # unknown dtype
    assert lib.lcpp_radix_sort_keys(fake, 1 << 20, fake, fake, 10, 0, 8, 0, 99, None) == lcpp.ERR_UNSUPPORTED_DTYPE
    # empty input is a no-op
    assert lib.lcpp_radix_sort_keys(None, 0, None, None, 0, 0, 32, 0, lcpp.U32, None) == lcpp.OK
    # temp too small
    assert lib.lcpp_radix_sort_keys(fake, 16, fake, fake, 10, 0, 32, 0, lcpp.U32, None) == lcpp.ERR_TEMP_TOO_SMALL
    # misaligned temp
    assert lib.lcpp_radix_sort_keys(vp(0x100004), 1 << 20, fake, fake, 10, 0, 32, 0, lcpp.U32, None) == lcpp.ERR_INVALID_ARG
    # DoubleBuffer selector must be 0 or 1
    bufs = (ctypes.c_void_p * 2)(0x100000, 0x200000)
    sel = ctypes.c_int(2)
    assert lib.lcpp_radix_sort_keys_double_buffer(fake, 1 << 20, bufs, ctypes.byref(sel), 10, 0, 32, 0,
                                                  lcpp.U32, None) == lcpp.ERR_INVALID_ARG
    # scans need an init for the exclusive form
    assert lib.lcpp_scan_exclusive(fake, 1 << 20, fake, fake, 10, lcpp.OP_SUM, None, lcpp.I32, None) == lcpp.ERR_INVALID_ARG
    assert lib.lcpp_scan_inclusive(fake, 1 << 20, fake, fake, 10, 7, lcpp.I32, None) == lcpp.ERR_UNSUPPORTED_DTYPE
    assert lib.lcpp_scan_inclusive_sum(None, 0, None, None, 0, lcpp.I32, None) == lcpp.OK
    assert lib.lcpp_reduce(fake, 1 << 20, fake, fake, 10, lcpp.OP_SUM, None, lcpp.F32, None) == lcpp.ERR_INVALID_ARG
    assert lib.lcpp_reduce_sum(fake, 16, fake, fake, 10, lcpp.F32, None) == lcpp.ERR_TEMP_TOO_SMALL


def test_missing_library_fails_loudly(tmp_path, monkeypatch):
    import lcpp_b200
    monkeypatch.setattr(lcpp_b200, "_lib", None)
    monkeypatch.setattr(lcpp_b200, "LIB_PATH", tmp_path / "nope.so")
    with pytest.raises(ImportError):
        lcpp_b200.lib()
