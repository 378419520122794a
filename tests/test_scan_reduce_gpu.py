"""GPU parity tests for DeviceScan and DeviceReduce (C ABI), mirroring the
reference's tests/device_scan_test.cpp, tests/scan_optimization_regression_test.cpp,
tests/device_reduce_test.cpp and tests/pr6_review_regression_test.cpp."""
from __future__ import annotations

import math

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
from gpu_helpers import NP_TO_CODE, dev, empty_like_np, host  # noqa: E402

TILE_SIZES = [0, 1, 31, 32, 33, 255, 256, 257, 3839, 3840, 3841, 4095, 4096, 4097, 7999, 8000, 8001,
              8191, 8192, 8193, 16003, 262147]


def _scan(lcpp, x: np.ndarray, mode: str, op=None, init=None, inplace=False):
    op = lcpp.OP_SUM if op is None else op
    n = x.size
    sc = lcpp.DeviceScan()
    code = NP_TO_CODE[x.dtype]
    temp = lcpp.alloc_temp(sc.GetTempStorageBytes(code, n))
    d_in = dev(x) if n else torch.empty(0, dtype=torch.from_numpy(x[:0]).dtype, device="cuda")
    d_out = d_in if inplace else (empty_like_np(x) if n else d_in)
    if mode == "exclusive":
        sc.ExclusiveScan(temp, d_in, d_out, n, op, init)
    elif mode == "inclusive":
        sc.InclusiveScan(temp, d_in, d_out, n, op)
    else:
        sc.InclusiveScanInit(temp, d_in, d_out, n, op, init)
    assert lcpp.device_status(temp) == lcpp.OK
    return host(d_out)


# ---------------------------------------------------------------- scan golden
def test_scan_all_ones(lcpp):
    """device_scan_test.cpp:80-127: ones, 2^0..2^23, ExclusiveSum and InclusiveSum."""
    sc = lcpp.DeviceScan()
    for k in range(0, 24):
        n = 1 << k
        x = torch.ones(n, dtype=torch.uint32, device="cuda")
        temp = lcpp.alloc_temp(sc.GetTempStorageBytes(lcpp.U32, n))
        ex, inc = torch.empty_like(x), torch.empty_like(x)
        sc.ExclusiveSum(temp, x, ex, n)
        sc.InclusiveSum(temp, x, inc, n)
        np.testing.assert_array_equal(host(ex), np.arange(n, dtype=np.uint32))
        np.testing.assert_array_equal(host(inc), np.arange(1, n + 1, dtype=np.uint32))


@pytest.mark.parametrize("n", [384 * 22 * 3 + 17, 320 * 25 * 3 + 17])
def test_scan_mod7_golden(lcpp, golden, n):
    """device_scan_test.cpp:189-265."""
    assert golden.matches(f"scan_mod7_inclusive_{n}", _scan(lcpp, golden[f"scan_mod7_in_{n}"], "inclusive"))


@pytest.mark.parametrize("n", TILE_SIZES)
def test_scan_tile_boundaries_golden(lcpp, golden, oracle, n):
    """scan_optimization_regression_test.cpp:124-190: value(i) = i%7+1."""
    x = (np.arange(n) % 7 + 1).astype(np.int32)
    ex = _scan(lcpp, x, "exclusive", init=0)
    inc = _scan(lcpp, x, "inclusive")
    if f"scan_tiles_exclusive_{n}" in golden.manifest:
        assert golden.matches(f"scan_tiles_exclusive_{n}", ex)
        assert golden.matches(f"scan_tiles_inclusive_{n}", inc)
    np.testing.assert_array_equal(ex, oracle.scan(x, "exclusive", init=0))
    np.testing.assert_array_equal(inc, oracle.scan(x, "inclusive"))
    if n == 16003:
        for inplace in (False, True):
            assert golden.matches("scan_tiles_exclusive_init3_16003",
                                  _scan(lcpp, x, "exclusive", init=3, inplace=inplace))
            assert golden.matches("scan_tiles_inclusive_init3_16003",
                                  _scan(lcpp, x, "inclusive_init", init=3, inplace=inplace))


def test_scan_init_inplace_golden(lcpp, golden):
    """device_scan_test.cpp:288-322: InclusiveScanInit in place, and on empty input."""
    out = _scan(lcpp, golden["scan_init_in"], "inclusive_init", init=10, inplace=True)
    np.testing.assert_array_equal(out, golden["scan_init_out"])
    _scan(lcpp, np.zeros(0, np.int32), "inclusive_init", init=10)


@pytest.mark.parametrize("dtype", [np.int32, np.uint32, np.int64, np.uint64])
@pytest.mark.parametrize("n", [1, 1000, 8193, 1_000_003])
@pytest.mark.parametrize("opname", ["SUM", "MIN", "MAX"])
def test_scan_int_vs_oracle(lcpp, oracle, dtype, n, opname):
    rng = np.random.default_rng(n)
    x = rng.integers(np.iinfo(dtype).min, np.iinfo(dtype).max, size=n, dtype=dtype, endpoint=True)
    op = getattr(lcpp, f"OP_{opname}")
    init = dtype(12345)
    np.testing.assert_array_equal(_scan(lcpp, x, "exclusive", op, init), oracle.scan(x, "exclusive", op, init))
    np.testing.assert_array_equal(_scan(lcpp, x, "inclusive", op), oracle.scan(x, "inclusive", op))
    np.testing.assert_array_equal(_scan(lcpp, x, "inclusive_init", op, init),
                                  oracle.scan(x, "inclusive_init", op, init))


@pytest.mark.parametrize("dtype", [np.float32, np.float64])
def test_scan_float(lcpp, dtype):
    """Floating-point scans: exact on exactly representable partial sums
    (value(i) = (i%7+1)*0.25, scan_optimization_regression_test.cpp:50-56),
    and within a relative 1e-5 (f32) / 1e-12 (f64) of an fp64 running sum
    otherwise."""
    n = 262147
    x = ((np.arange(n) % 7 + 1) * 0.25).astype(dtype)
    ref = np.cumsum(x.astype(np.float64))
    np.testing.assert_array_equal(_scan(lcpp, x, "inclusive"), ref.astype(dtype))
    rng = np.random.default_rng(3)
    y = rng.random(n).astype(dtype)
    got = _scan(lcpp, y, "inclusive").astype(np.float64)
    ref = np.cumsum(y.astype(np.float64))
    tol = 1e-5 if dtype == np.float32 else 1e-12
    assert np.max(np.abs(got - ref) / np.maximum(ref, 1)) < tol
    mx = _scan(lcpp, y, "inclusive", lcpp.OP_MAX)
    np.testing.assert_array_equal(mx, np.maximum.accumulate(y))


def test_scan_2p30_properties(lcpp):
    """InclusiveSum / ExclusiveSum on 2^30 i32 in [-1000,1000].
    Checks (size independent): out_incl - out_excl == in; out_incl[i] -
    out_incl[i-1] == in[i]; last inclusive == reduce(in) (wrapping)."""
    n = 1 << 30
    x = torch.empty(n, dtype=torch.int32, device="cuda")
    lcpp.testgen_fill(x, lcpp.GEN_I32_SCAN, seed=1)
    sc = lcpp.DeviceScan()
    temp = lcpp.alloc_temp(sc.GetTempStorageBytes(lcpp.I32, n))
    inc = torch.empty_like(x)
    sc.InclusiveSum(temp, x, inc, n)
    assert lcpp.device_status(temp) == lcpp.OK
    assert torch.equal(inc[1:] - inc[:-1], x[1:])
    assert int(inc[0]) == int(x[0])
    total = int(x.to(torch.int64).sum())
    assert int(inc[-1]) == total  # |total| < 2^31 for this distribution
    ex = torch.empty_like(x)
    sc.ExclusiveSum(temp, x, ex, n)
    assert lcpp.device_status(temp) == lcpp.OK
    assert torch.equal(inc - ex, x)


# -------------------------------------------------------------------- reduce
def _reduce(lcpp, x: np.ndarray, which: str):
    n = x.size
    rd = lcpp.DeviceReduce()
    code = NP_TO_CODE[x.dtype]
    temp = lcpp.alloc_temp(rd.GetTempStorageBytes(code, n))
    d_in = dev(x) if n else torch.empty(0, dtype=torch.from_numpy(x[:0]).dtype, device="cuda")
    out = torch.empty(1, dtype=d_in.dtype, device="cuda")
    getattr(rd, which)(temp, d_in, out, n)
    return host(out)[0]


def test_reduce_ones(lcpp):
    """device_reduce_test.cpp:95-118: ones at 2^k + 1, k = 0..23."""
    for k in range(0, 24):
        n = (1 << k) + 1
        assert _reduce(lcpp, np.ones(n, np.uint32), "Sum") == n


def test_reduce_shuffled_golden(lcpp, golden):
    """device_reduce_test.cpp:160-217."""
    x = golden["reduce_shuffled_in"]
    mn, mx = golden["reduce_shuffled_minmax"]
    assert _reduce(lcpp, x, "Min") == mn
    assert _reduce(lcpp, x, "Max") == mx


def test_reduce_float_max_identity(lcpp):
    """device_reduce_test.cpp:220-236."""
    assert _reduce(lcpp, np.array([-8.0, -2.5, -9.0, -4.0], np.float32), "Max") == np.float32(-2.5)


def test_reduce_empty_writes_init(lcpp):
    """device_reduce.h:238-242: n == 0 writes the initial value."""
    assert _reduce(lcpp, np.zeros(0, np.int32), "Sum") == 0
    assert _reduce(lcpp, np.zeros(0, np.int32), "Min") == np.iinfo(np.int32).max
    assert _reduce(lcpp, np.zeros(0, np.float32), "Max") == np.finfo(np.float32).min


def test_reduce_large_tail(lcpp):
    """pr6_review_regression_test.cpp:427-457: 2^24+1 zeros with a tail value."""
    n = (1 << 24) + 1
    x = np.zeros(n, np.uint32)
    x[-1] = 123456789
    assert _reduce(lcpp, x, "Sum") == 123456789
    assert _reduce(lcpp, x, "Max") == 123456789


@pytest.mark.parametrize("dtype", [np.int32, np.uint32, np.int64, np.uint64])
@pytest.mark.parametrize("n", [1, 3, 4097, 1_000_003, 20_971_521])
def test_reduce_int_vs_oracle(lcpp, oracle, dtype, n):
    rng = np.random.default_rng(n)
    x = rng.integers(np.iinfo(dtype).min, np.iinfo(dtype).max, size=n, dtype=dtype, endpoint=True)
    assert _reduce(lcpp, x, "Sum") == oracle.reduce(x, oracle.OP_SUM, 0)
    assert _reduce(lcpp, x, "Min") == oracle.reduce(x, oracle.OP_MIN, np.iinfo(dtype).max)
    assert _reduce(lcpp, x, "Max") == oracle.reduce(x, oracle.OP_MAX, np.iinfo(dtype).min)


def test_reduce_misaligned_input(lcpp, oracle):
    x = np.arange(100_001, dtype=np.int32)
    d = dev(x)
    rd = lcpp.DeviceReduce()
    temp = lcpp.alloc_temp(rd.GetTempStorageBytes(lcpp.I32, 100_000))
    out = torch.empty(1, dtype=torch.int32, device="cuda")
    rd.Sum(temp, d[1:], out, 100_000)
    assert int(out) == int(x[1:].astype(np.int64).sum() & 0xFFFFFFFF) - (1 << 32) * bool(
        x[1:].astype(np.int64).sum() & 0x80000000)  # int32 wrap-around


def test_reduce_f32_2p30(lcpp, oracle):
    """Sum of 2^30 f32 U[0,1) within 1e-6*log2(n) of the fp64 sum,
    and deterministic from run to run."""
    n = 1 << 30
    x = torch.empty(n, dtype=torch.float32, device="cuda")
    lcpp.testgen_fill(x, lcpp.GEN_F32_UNIT, seed=1)
    rd = lcpp.DeviceReduce()
    temp = lcpp.alloc_temp(rd.GetTempStorageBytes(lcpp.F32, n))
    out = torch.empty(1, dtype=torch.float32, device="cuda")
    rd.Sum(temp, x, out, n)
    got = float(out)
    ref = float(x.to(torch.float64).sum())
    assert abs(got - ref) / ref <= 1e-6 * math.log2(n)
    for _ in range(2):
        rd.Sum(temp, x, out, n)
        assert float(out) == got


def test_reduce_i64_max_2p30(lcpp):
    """Max of 2^30 uniform int64 (exact)."""
    n = 1 << 30
    x = torch.empty(n, dtype=torch.int64, device="cuda")
    lcpp.testgen_fill(x, lcpp.GEN_I64_UNIFORM, seed=1)
    rd = lcpp.DeviceReduce()
    temp = lcpp.alloc_temp(rd.GetTempStorageBytes(lcpp.I64, n))
    out = torch.empty(1, dtype=torch.int64, device="cuda")
    rd.Max(temp, x, out, n)
    assert int(out) == int(x.max())
    rd.Min(temp, x, out, n)
    assert int(out) == int(x.min())


def test_reduce_f32_small_vs_fp64(lcpp, oracle):
    for n in (1, 17, 100_000, 3_000_017):
        x = oracle.generate(oracle.GEN_F32_UNIT, n, seed=n)
        got = float(_reduce(lcpp, x, "Sum"))
        ref = oracle.sum_f64(x)
        assert abs(got - ref) <= 1e-6 * max(1.0, math.log2(n)) * max(ref, 1e-30)
