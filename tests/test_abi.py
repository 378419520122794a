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


def test_misuse_new_families_without_device(lcpp):
    """ArgMin/ArgMax, the by-key scans, ReduceByKey, DeviceSelect and
    DevicePartition reject bad arguments before any device work."""
    lib = lcpp.lib()
    vp = ctypes.c_void_p
    a, b, c = vp(0x100000), vp(0x200000), vp(0x300000)  # never dereferenced
    big = 1 << 20

    def clauses(*cl):
        return (lcpp.Clause * max(1, len(cl)))(*[lcpp.Clause(*x) for x in cl]), len(cl)

    # ArgMin / ArgMax: uint32 indices, 4- and 8-byte types only
    assert lib.lcpp_reduce_argmin(a, big, b, c, c, 1 << 32, lcpp.I32, None) == lcpp.ERR_INVALID_ARG
    assert lib.lcpp_reduce_argmax(a, big, b, c, c, 10, lcpp.U8, None) == lcpp.ERR_UNSUPPORTED_DTYPE
    assert lib.lcpp_reduce_argmin(a, big, b, None, c, 10, lcpp.I32, None) == lcpp.ERR_INVALID_ARG
    # by-key scans: init required for the exclusive form; temp size; dtypes; operator
    assert lib.lcpp_scan_exclusive_by_key(a, big, b, c, c, 10, lcpp.OP_SUM, None, lcpp.I32, lcpp.I32,
                                          None) == lcpp.ERR_INVALID_ARG
    assert lib.lcpp_scan_inclusive_by_key(a, 16, b, c, c, 10, lcpp.OP_SUM, lcpp.I32, lcpp.I32,
                                          None) == lcpp.ERR_TEMP_TOO_SMALL
    assert lib.lcpp_scan_inclusive_by_key(a, big, b, c, c, 10, lcpp.OP_SUM, lcpp.U8, lcpp.I32,
                                          None) == lcpp.ERR_UNSUPPORTED_DTYPE
    assert lib.lcpp_scan_inclusive_by_key(a, big, b, c, c, 10, 7, lcpp.I32, lcpp.I32, None) == lcpp.ERR_INVALID_ARG
    assert lib.lcpp_scan_inclusive_sum_by_key(None, 0, None, None, None, 0, lcpp.I32, lcpp.F64, None) == lcpp.OK
    # ReduceByKey: run count pointer, uint32 counts, no aliasing of unique_out and keys_in
    assert lib.lcpp_reduce_by_key(a, big, b, c, vp(0x400000), vp(0x500000), None, 10, lcpp.OP_SUM, lcpp.I32,
                                  lcpp.I32, None) == lcpp.ERR_INVALID_ARG
    assert lib.lcpp_reduce_by_key(a, big, b, c, vp(0x400000), vp(0x500000), vp(0x600000), 1 << 32, lcpp.OP_SUM,
                                  lcpp.I32, lcpp.I32, None) == lcpp.ERR_INVALID_ARG
    assert lib.lcpp_reduce_by_key(a, big, b, c, b, vp(0x500000), vp(0x600000), 10, lcpp.OP_SUM, lcpp.I32,
                                  lcpp.I32, None) == lcpp.ERR_INVALID_ARG
    # DeviceSelect: clause checks (no remainder or bit test on floats, m != 0,
    # at most LCPP_MAX_CLAUSES, known kinds), item and flag dtypes, count pointer
    n_sel = vp(0x600000)
    arr, k = clauses((6, 0, 2, 0))
    f32_two = 0x40000000
    assert lib.lcpp_select_if(a, big, b, c, n_sel, 10, lcpp.F32, arr, k, None) == lcpp.ERR_INVALID_ARG
    arr, k = clauses((7, 0, f32_two, 0))
    assert lib.lcpp_select_if(a, big, b, c, n_sel, 10, lcpp.F32, arr, k, None) == lcpp.ERR_INVALID_ARG
    arr, k = clauses((6, 0, 0, 0))
    assert lib.lcpp_select_if(a, big, b, c, n_sel, 10, lcpp.I32, arr, k, None) == lcpp.ERR_INVALID_ARG
    arr, k = clauses(*[(0, 0, 1, 0)] * 5)
    assert lib.lcpp_select_if(a, big, b, c, n_sel, 10, lcpp.I32, arr, k, None) == lcpp.ERR_INVALID_ARG
    arr, k = clauses((9, 0, 1, 0))
    assert lib.lcpp_select_if(a, big, b, c, n_sel, 10, lcpp.I32, arr, k, None) == lcpp.ERR_INVALID_ARG
    assert lib.lcpp_select_if(a, big, b, c, n_sel, 10, lcpp.U8, arr, k, None) == lcpp.ERR_UNSUPPORTED_DTYPE
    assert lib.lcpp_select_if(a, big, b, c, None, 10, lcpp.I32, arr, k, None) == lcpp.ERR_INVALID_ARG
    assert lib.lcpp_select_if(a, big, b, c, n_sel, 1 << 32, lcpp.I32, arr, k, None) == lcpp.ERR_INVALID_ARG
    assert lib.lcpp_select_flagged(a, big, b, c, vp(0x700000), n_sel, 10, lcpp.I32, 99,
                                   None) == lcpp.ERR_UNSUPPORTED_DTYPE
    assert lib.lcpp_select_unique(a, 16, b, c, n_sel, 10, lcpp.I64, None) == lcpp.ERR_TEMP_TOO_SMALL
    # DevicePartition: never in place; three-way outputs must not overlap the
    # input; the three-way form needs its larger temp storage
    arr, k = clauses((0, 0, 5, 0))
    assert lib.lcpp_partition_if(a, big, b, b, n_sel, 10, lcpp.I32, arr, k, None) == lcpp.ERR_INVALID_ARG
    assert lib.lcpp_partition_flagged(a, big, b, c, b, n_sel, 10, lcpp.I32, lcpp.U8, None) == lcpp.ERR_INVALID_ARG
    # a partly overlapping output (a few items past the input's start) is
    # rejected too: the rejected items are written backwards from its end
    assert lib.lcpp_partition_if(a, big, b, vp(0x200008), n_sel, 10, lcpp.I32, arr, k, None) == lcpp.ERR_INVALID_ARG
    assert lib.lcpp_partition_flagged(a, big, b, c, vp(0x1FFFF8), n_sel, 10, lcpp.I32, lcpp.U8,
                                      None) == lcpp.ERR_INVALID_ARG
    assert lib.lcpp_partition_if_three_way(a, big, b, vp(0x200004), vp(0x800000), vp(0x900000), n_sel, 10,
                                           lcpp.I32, arr, k, arr, k, None) == lcpp.ERR_INVALID_ARG
    two, three = ctypes.c_size_t(), ctypes.c_size_t()
    assert lib.lcpp_partition_temp_bytes(1 << 20, ctypes.byref(two)) == lcpp.OK
    assert lib.lcpp_partition_three_way_temp_bytes(1 << 20, ctypes.byref(three)) == lcpp.OK
    assert three.value > two.value > 0
    assert lib.lcpp_partition_if_three_way(a, two.value, b, vp(0x800000), vp(0x900000), vp(0xA00000), n_sel,
                                           1 << 20, lcpp.I32, arr, k, arr, k, None) == lcpp.ERR_TEMP_TOO_SMALL
    zero = ctypes.c_size_t(7)
    assert lib.lcpp_select_temp_bytes(0, ctypes.byref(zero)) == lcpp.OK and zero.value == 0
