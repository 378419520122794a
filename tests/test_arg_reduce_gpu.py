"""GPU parity tests for DeviceReduce::ArgMin / ArgMax (C ABI), mirroring the
reference's tests/device_reduce_test.cpp:238-345 and checking against the
CPU restatement of its ArgMinOp / ArgMaxOp fold (oracle_arg_extremum)."""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
from gpu_helpers import NP_TO_CODE, dev  # noqa: E402

DTYPES = [np.int32, np.uint32, np.float32, np.int64, np.uint64, np.float64]
SIZES = [1, 2, 3, 31, 32, 33, 511, 2047, 2048, 2049, 8195, 65_537, 1_000_003, 20_971_521]


def _arg(lcpp, x, is_min: bool, d_in=None, n=None):
    """(value, index) from the library; d_in may be a device view (misaligned)."""
    n = x.size if n is None else n
    code = NP_TO_CODE[np.dtype(x.dtype)]
    rd = lcpp.DeviceReduce()
    temp = lcpp.alloc_temp(rd.GetArgTempStorageBytes(code, n)) if n else None
    if d_in is None:
        d_in = dev(x) if n else None
    out = torch.empty(1, dtype=torch.from_numpy(np.zeros(1, x.dtype)).dtype, device="cuda")
    idx = torch.full((1,), 0x7EADBEEF, dtype=torch.int32, device="cuda")
    (rd.ArgMin if is_min else rd.ArgMax)(temp, d_in, out, idx, n)
    torch.cuda.synchronize()
    return out.cpu().numpy()[0], int(idx.cpu().numpy().view(np.uint32)[0])


def _same(got, want):
    gv, gi = got
    wv, wi = want
    assert gi == wi, (got, want)
    assert np.asarray(gv).tobytes() == np.asarray(wv).tobytes(), (got, want)


# ------------------------------------------------------------ reference tests
def test_argmax_first_equal_extremum(lcpp, golden):
    """device_reduce_test.cpp:238-262: {1, 9, 4, 9, 3} -> (9, 1)."""
    x = golden["arg_ties_in"]
    v, i = golden["arg_ties_max"]
    assert _arg(lcpp, x, False) == (v, i)


def test_float_argmax_negative_values(lcpp, golden):
    """device_reduce_test.cpp:264-288: {-7, -3, -5} -> (-3, 1)."""
    x = golden["arg_negative_in"]
    v, i = golden["arg_negative_max"]
    got = _arg(lcpp, x, False)
    assert got[0] == v and got[1] == int(i)


@pytest.mark.parametrize("dtype", DTYPES)
def test_empty_input_sentinels(lcpp, dtype):
    """device_reduce.h:318-323 / :382-387: 0 items -> max() / lowest() and index 1."""
    x = np.zeros(0, dtype)
    info = np.finfo(dtype) if np.dtype(dtype).kind == "f" else np.iinfo(dtype)
    assert _arg(lcpp, x, True) == (dtype(info.max), 1)
    assert _arg(lcpp, x, False) == (dtype(info.min), 1)


# ------------------------------------------------------------------ vs oracle
@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("n", SIZES)
def test_vs_oracle(lcpp, oracle, dtype, n):
    rng = np.random.default_rng(n * 7 + np.dtype(dtype).num)
    if np.dtype(dtype).kind == "f":
        x = rng.standard_normal(n).astype(dtype)
    else:
        x = rng.integers(np.iinfo(dtype).min, np.iinfo(dtype).max, size=n, dtype=dtype, endpoint=True)
    for is_min in (True, False):
        _same(_arg(lcpp, x, is_min), oracle.arg_extremum(x, is_min))


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("n", [33, 4099, 1_000_003])
def test_many_ties_first_index_wins(lcpp, oracle, dtype, n):
    """Few distinct values, so every block holds the extreme: the first index must win."""
    rng = np.random.default_rng(n)
    x = rng.integers(0, 5, size=n).astype(dtype)
    for is_min in (True, False):
        got = _arg(lcpp, x, is_min)
        _same(got, oracle.arg_extremum(x, is_min))
        assert got[1] == int(np.argmin(x) if is_min else np.argmax(x))


@pytest.mark.parametrize("dtype", [np.int32, np.float64])
def test_all_equal_and_identity_valued(lcpp, dtype):
    """All items equal (including equal to the identity value): index 0."""
    info = np.finfo(dtype) if np.dtype(dtype).kind == "f" else np.iinfo(dtype)
    for fill in (dtype(3), dtype(info.max), dtype(info.min)):
        x = np.full(100_000, fill, dtype)
        assert _arg(lcpp, x, True) == (fill, 0)
        assert _arg(lcpp, x, False) == (fill, 0)


@pytest.mark.parametrize("where", [0, 1, 4095, 4096, 99_998, 99_999])
def test_extreme_position(lcpp, where):
    x = np.ones(100_000, np.float32)
    x[where] = -2.0
    x[(where + 17) % x.size] = 5.0
    assert _arg(lcpp, x, True) == (np.float32(-2.0), where)
    assert _arg(lcpp, x, False) == (np.float32(5.0), (where + 17) % x.size)


def test_nan_never_wins(lcpp, oracle):
    x = np.random.default_rng(3).standard_normal(50_001).astype(np.float32)
    x[::7] = np.nan
    for is_min in (True, False):
        got = _arg(lcpp, x, is_min)
        _same(got, oracle.arg_extremum(x, is_min))
        assert got[1] == int(np.nanargmin(x) if is_min else np.nanargmax(x))
    allnan = np.full(1000, np.nan, np.float32)
    assert _arg(lcpp, allnan, True) == (np.finfo(np.float32).max, 0xFFFFFFFF)
    _same(_arg(lcpp, allnan, False), oracle.arg_extremum(allnan, False))


@pytest.mark.parametrize("dtype,offset", [(np.int32, 1), (np.int32, 3), (np.float32, 2), (np.uint64, 1),
                                          (np.float64, 1)])
def test_misaligned_input(lcpp, oracle, dtype, offset):
    """Input not 16-byte aligned: the scalar-load form."""
    x = np.random.default_rng(offset).integers(0, 1000, size=200_003).astype(dtype)
    d = dev(x)
    sub = x[offset:]
    for is_min in (True, False):
        _same(_arg(lcpp, sub, is_min, d_in=d[offset:]), oracle.arg_extremum(sub, is_min))


def test_indices_above_2p31(lcpp):
    """uint32 indices past 2^31 (the reference's index type)."""
    n = (1 << 31) + 9
    x = torch.ones(n, dtype=torch.float32, device="cuda")
    lo, hi = (1 << 31) + 3, (1 << 31) + 8
    x[lo] = -1.0
    x[lo + 1] = -1.0
    x[hi] = 2.0
    rd = lcpp.DeviceReduce()
    temp = lcpp.alloc_temp(rd.GetArgTempStorageBytes(lcpp.F32, n))
    out = torch.empty(1, dtype=torch.float32, device="cuda")
    idx = torch.empty(1, dtype=torch.int32, device="cuda")
    rd.ArgMin(temp, x, out, idx, n)
    assert float(out) == -1.0 and int(idx.cpu().numpy().view(np.uint32)[0]) == lo
    rd.ArgMax(temp, x, out, idx, n)
    assert float(out) == 2.0 and int(idx.cpu().numpy().view(np.uint32)[0]) == hi


def test_argument_errors(lcpp):
    rd = lcpp.DeviceReduce()
    x = torch.zeros(1024, dtype=torch.int32, device="cuda")
    out = torch.empty(1, dtype=torch.int32, device="cuda")
    idx = torch.empty(1, dtype=torch.int32, device="cuda")
    with pytest.raises(lcpp.LcppError) as e:
        rd.ArgMin(lcpp.alloc_temp(64), x, out, idx, 1024)
    assert e.value.status == lcpp.ERR_TEMP_TOO_SMALL
    temp = lcpp.alloc_temp(rd.GetArgTempStorageBytes(lcpp.I32, 1024))
    with pytest.raises(lcpp.LcppError) as e:
        rd.ArgMax(temp, x, out, idx, 1 << 32)  # indices are uint32
    assert e.value.status == lcpp.ERR_INVALID_ARG
