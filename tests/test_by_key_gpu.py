"""GPU parity tests for the by-key scans (DeviceScan::ExclusiveScanByKey /
InclusiveScanByKey / ...SumByKey) and DeviceReduce::ReduceByKey (C ABI),
mirroring the reference's tests/device_scan_test.cpp:324-446 and
tests/device_reduce_test.cpp:422-513 and checking against the CPU
restatement (oracle_scan_by_key / oracle_reduce_by_key)."""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
from gpu_helpers import NP_TO_CODE, dev, empty_like_np, host  # noqa: E402

TILE = 4096
SIZES = [1, 2, 3, 1023, 4095, TILE, TILE + 1, 3 * TILE + 5, 65_537, 1_000_003]


def _keys(kind: str, n: int, dtype, seed: int):
    rng = np.random.default_rng(seed)
    if kind == "runs":  # runs of 1..40 items
        lens = rng.integers(1, 41, size=n // 2 + 2)
        ids = np.repeat(np.arange(lens.size), lens)[:n]
        return (ids % 7).astype(dtype)  # neighbouring runs differ (consecutive ids mod 7 differ)
    if kind == "one":
        return np.full(n, 3, dtype)
    if kind == "distinct":
        return (np.arange(n) % 1000).astype(dtype)
    lens = rng.integers(1, 20_000, size=n // 1000 + 2)  # "long": runs spanning tiles
    ids = np.repeat(np.arange(lens.size), lens)[:n]
    return (ids % 5).astype(dtype)


def _values(n: int, dtype, seed: int):
    rng = np.random.default_rng(seed + 100)
    return rng.integers(-8, 9, size=n).astype(dtype)  # small integers: float sums stay exact


def _scan(lcpp, keys, vals, mode, op=None, init=None, inplace=False, d_keys=None, d_vals=None):
    op = lcpp.OP_SUM if op is None else op
    n = vals.size
    sc = lcpp.DeviceScan()
    temp = lcpp.alloc_temp(sc.GetScanByKeyTempStorageBytes(NP_TO_CODE[keys.dtype], NP_TO_CODE[vals.dtype], n))
    dk = dev(keys) if d_keys is None else d_keys
    dv = dev(vals) if d_vals is None else d_vals
    out = dv if inplace else empty_like_np(vals)
    if mode == "exclusive":
        sc.ExclusiveScanByKey(temp, dk, dv, out, op, n, init)
    elif mode == "inclusive":
        sc.InclusiveScanByKey(temp, dk, dv, out, op, n)
    else:
        sc.InclusiveScanByKey(temp, dk, dv, out, op, n, init)
    assert lcpp.device_status(temp) == lcpp.OK
    return host(out)


def _reduce_by_key(lcpp, keys, vals, op=None):
    op = lcpp.OP_SUM if op is None else op
    n = vals.size
    rd = lcpp.DeviceReduce()
    temp = lcpp.alloc_temp(rd.GetReduceByKeyTempStorageBytes(NP_TO_CODE[keys.dtype], NP_TO_CODE[vals.dtype], n))
    uniq, agg = empty_like_np(keys), empty_like_np(vals)
    runs = torch.full((1,), 17, dtype=torch.int32, device="cuda")
    rd.ReduceByKey(temp, dev(keys), dev(vals), uniq, agg, runs, op, n)
    assert lcpp.device_status(temp) == lcpp.OK
    r = int(runs.cpu().numpy().view(np.uint32)[0])
    return host(uniq)[:r], host(agg)[:r]


# ------------------------------------------------------------ reference tests
def test_exclusive_sum_by_key_segments_of_100(lcpp, golden):
    """device_scan_test.cpp:324-380: ones, keys i / 100, sizes 2^5 .. 2^23."""
    sc = lcpp.DeviceScan()
    for k in range(5, 24):
        n = 1 << k
        keys = torch.arange(n, dtype=torch.int32, device="cuda") // 100
        ones = torch.ones(n, dtype=torch.int32, device="cuda")
        out = torch.empty_like(ones)
        temp = lcpp.alloc_temp(sc.GetScanByKeyTempStorageBytes(lcpp.I32, lcpp.I32, n))
        sc.ExclusiveSumByKey(temp, keys, ones, out, n)
        want = torch.arange(n, dtype=torch.int32, device="cuda") % 100
        assert torch.equal(out, want), k
        if n == golden["sbk_exclusive_sum_out"].size:
            np.testing.assert_array_equal(host(out), golden["sbk_exclusive_sum_out"])


def test_inclusive_sum_by_key_three_tiles(lcpp, golden):
    """device_scan_test.cpp:382-417: int keys, int64 values, segments cut one past each tile."""
    keys = golden["sbk_three_tiles_keys"]
    vals = np.ones(keys.size, np.int64)
    sc = lcpp.DeviceScan()
    temp = lcpp.alloc_temp(sc.GetScanByKeyTempStorageBytes(lcpp.I32, lcpp.I64, keys.size))
    out = empty_like_np(vals)
    sc.InclusiveSumByKey(temp, dev(keys), dev(vals), out, keys.size)
    np.testing.assert_array_equal(host(out), golden["sbk_three_tiles_inclusive_out"])


def test_reduce_by_key_reference(lcpp, golden):
    """device_reduce_test.cpp:422-483: Sum of the shuffled 0..4095 by key i / 100 (41 runs)."""
    uniq, agg = _reduce_by_key(lcpp, golden["sbk_segment_keys"], golden["reduce_shuffled_in"])
    np.testing.assert_array_equal(uniq, golden["rbk_unique_out"])
    np.testing.assert_array_equal(agg, golden["rbk_aggregates_out"])


def test_reduce_by_key_empty_writes_zero_runs(lcpp):
    """device_reduce_test.cpp:485-513: num_runs preset to 17 becomes 0."""
    rd = lcpp.DeviceReduce()
    runs = torch.full((1,), 17, dtype=torch.int32, device="cuda")
    k = torch.zeros(1, dtype=torch.int32, device="cuda")
    rd.ReduceByKey(None, k, k, k.clone(), k.clone(), runs, lcpp.OP_SUM, 0)
    torch.cuda.synchronize()
    assert int(runs) == 0


# ------------------------------------------------------------------ vs oracle
@pytest.mark.parametrize("kdt,vdt", [(np.int32, np.int32), (np.uint32, np.float32), (np.int64, np.int64),
                                     (np.float32, np.uint64), (np.float64, np.float64), (np.int32, np.int64)])
@pytest.mark.parametrize("kind", ["runs", "one", "distinct", "long"])
def test_scans_vs_oracle(lcpp, oracle, kdt, vdt, kind):
    for n in SIZES:
        keys, vals = _keys(kind, n, kdt, n), _values(n, vdt, n)
        for op in (lcpp.OP_SUM, lcpp.OP_MIN, lcpp.OP_MAX):
            for mode, init in (("exclusive", 5), ("inclusive", None), ("inclusive_init", -3)):
                if np.dtype(vdt).kind == "u" and init is not None:
                    init = abs(init)
                got = _scan(lcpp, keys, vals, mode, op, init)
                want = oracle.scan_by_key(keys, vals, mode, op, init)
                np.testing.assert_array_equal(got, want, err_msg=f"n={n} op={op} mode={mode}")


@pytest.mark.parametrize("kdt,vdt", [(np.int32, np.int32), (np.uint64, np.float32), (np.float32, np.int64),
                                     (np.float64, np.uint32)])
@pytest.mark.parametrize("kind", ["runs", "one", "distinct", "long"])
def test_reduce_by_key_vs_oracle(lcpp, oracle, kdt, vdt, kind):
    for n in SIZES + [(1 << 22) + 7]:
        keys, vals = _keys(kind, n, kdt, n + 1), _values(n, vdt, n + 1)
        for op in (lcpp.OP_SUM, lcpp.OP_MIN, lcpp.OP_MAX):
            gu, ga = _reduce_by_key(lcpp, keys, vals, op)
            wu, wa = oracle.reduce_by_key(keys, vals, op)
            np.testing.assert_array_equal(gu, wu, err_msg=f"n={n} op={op}")
            np.testing.assert_array_equal(ga, wa, err_msg=f"n={n} op={op}")


def test_float_key_equality(lcpp, oracle):
    """-0.0 == +0.0 (one run), every NaN starts a run (the reference's a != b)."""
    keys = np.array([0.0, -0.0, 0.0, np.nan, np.nan, 1.0, 1.0, -0.0], np.float32)
    vals = np.arange(1, 9, dtype=np.int32)
    np.testing.assert_array_equal(_scan(lcpp, keys, vals, "inclusive"), oracle.scan_by_key(keys, vals, "inclusive"))
    gu, ga = _reduce_by_key(lcpp, keys, vals)
    wu, wa = oracle.reduce_by_key(keys, vals)
    assert ga.tolist() == wa.tolist() == [6, 4, 5, 13, 8]
    assert gu.tobytes() == wu.tobytes()  # the first key of each run, bit for bit


def test_in_place_and_misaligned(lcpp, oracle):
    n = 300_001
    keys, vals = _keys("runs", n, np.int32, 9), _values(n, np.int32, 9)
    np.testing.assert_array_equal(_scan(lcpp, keys, vals, "inclusive", inplace=True),
                                  oracle.scan_by_key(keys, vals, "inclusive"))
    dk, dv = dev(keys), dev(vals)  # views one item in: not 16-byte aligned
    got = _scan(lcpp, keys[1:], vals[1:], "exclusive", lcpp.OP_SUM, 0, d_keys=dk[1:], d_vals=dv[1:])
    np.testing.assert_array_equal(got, oracle.scan_by_key(keys[1:], vals[1:], "exclusive", lcpp.OP_SUM, 0))


def test_one_segment_2p30(lcpp):
    """One segment of 2^30 items (every tile's look-back walks to an inclusive
    predecessor) and 2^30 items in runs of 1000: InclusiveSumByKey of ones is
    the position within the run."""
    n = 1 << 30
    sc = lcpp.DeviceScan()
    temp = lcpp.alloc_temp(sc.GetScanByKeyTempStorageBytes(lcpp.I32, lcpp.I32, n))
    ones = torch.ones(n, dtype=torch.int32, device="cuda")
    out = torch.empty_like(ones)
    keys = torch.zeros(n, dtype=torch.int32, device="cuda")
    sc.InclusiveSumByKey(temp, keys, ones, out, n)
    assert lcpp.device_status(temp) == lcpp.OK
    pos = torch.arange(n, dtype=torch.int32, device="cuda")
    assert torch.equal(out, pos + 1)
    keys = pos // 1000
    sc.InclusiveSumByKey(temp, keys, ones, out, n)
    assert torch.equal(out, pos % 1000 + 1)
    rd = lcpp.DeviceReduce()
    rtemp = lcpp.alloc_temp(rd.GetReduceByKeyTempStorageBytes(lcpp.I32, lcpp.I32, n))
    uniq = torch.empty_like(keys)
    runs = torch.zeros(1, dtype=torch.int32, device="cuda")
    rd.ReduceByKey(rtemp, keys, ones, uniq, out, runs, lcpp.OP_SUM, n)
    r = int(runs)
    assert r == (n + 999) // 1000
    assert torch.equal(uniq[:r], torch.arange(r, dtype=torch.int32, device="cuda"))
    want = torch.full((r,), 1000, dtype=torch.int32, device="cuda")
    want[-1] = n - 1000 * (r - 1)
    assert torch.equal(out[:r], want)


def test_argument_errors(lcpp):
    rd = lcpp.DeviceReduce()
    k = torch.zeros(1024, dtype=torch.int32, device="cuda")
    runs = torch.zeros(1, dtype=torch.int32, device="cuda")
    temp = lcpp.alloc_temp(rd.GetReduceByKeyTempStorageBytes(lcpp.I32, lcpp.I32, 1024))
    with pytest.raises(lcpp.LcppError) as e:
        rd.ReduceByKey(temp, k, k, k, k.clone(), runs, lcpp.OP_SUM, 1024)  # unique_out aliases keys_in
    assert e.value.status == lcpp.ERR_INVALID_ARG
    with pytest.raises(lcpp.LcppError) as e:
        rd.ReduceByKey(lcpp.alloc_temp(16), k, k, k.clone(), k.clone(), runs, lcpp.OP_SUM, 1024)
    assert e.value.status == lcpp.ERR_TEMP_TOO_SMALL
    with pytest.raises(lcpp.LcppError) as e:
        rd.ReduceByKey(temp, k, k, k.clone(), k.clone(), runs, lcpp.OP_SUM, 1 << 32)
    assert e.value.status == lcpp.ERR_INVALID_ARG
