"""GPU tests of DeviceSegmentedRadixSort (lcpp_segmented_radix_sort_*):
the reference test's own case (golden fixture), then seeded cases against
the oracle for every dtype, direction, bit range and segment layout, bit for
bit, including the DoubleBuffer selector rule and untouched positions."""
from __future__ import annotations

import zlib

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

SENT = {np.dtype(np.uint32): 0xA5A5A5A5, np.dtype(np.int32): -777, np.dtype(np.float32): -12345.5,
        np.dtype(np.uint64): 0xA5A5A5A5A5A5A5A5, np.dtype(np.int64): -777, np.dtype(np.float64): -12345.5}


def _dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _bits(a):
    return a.view(np.uint32 if a.dtype.itemsize == 4 else np.uint64)


def _run(lcpp, keys, vals, b, e, begin_bit, end_bit, desc, form):
    """Runs one entry point; returns (out_keys, out_vals, selector or None)."""
    L = lcpp
    n, nseg = keys.size, b.size
    ss = L.DeviceSegmentedRadixSort()
    kd = L.dtype_code(_dev(keys[:1]) if n else torch.empty(0, dtype=torch.from_numpy(keys).dtype))
    if vals is None:
        tb = L.DeviceSegmentedRadixSort.GetSortKeysTempStorageBytes(kd, n)
    else:
        vd = L.dtype_code(torch.from_numpy(vals[:1].copy()))
        tb = L.DeviceSegmentedRadixSort.GetSortPairsTempStorageBytes(kd, vd, n)
    temp = L.alloc_temp(max(tb, 1))
    db, de = _dev(b), _dev(e)
    kin = _dev(keys)
    sent_k = np.full_like(keys, SENT[keys.dtype])
    kout = _dev(sent_k)
    fn = ss.SortKeysDescending if desc else ss.SortKeys
    pfn = ss.SortPairsDescending if desc else ss.SortPairs
    if form == "copy":
        if vals is None:
            fn(temp, kin, kout, n, nseg, db, de, begin_bit, end_bit)
            return kout.cpu().numpy(), None, None
        vin, vout = _dev(vals), _dev(np.full_like(vals, 0xEE))
        pfn(temp, kin, kout, vin, vout, n, nseg, db, de, begin_bit, end_bit)
        return kout.cpu().numpy(), vout.cpu().numpy(), None
    # DoubleBuffer: the input in slot 1, sentinels in slot 0
    kdb = L.DoubleBuffer(kout, kin, 1)
    if vals is None:
        fn(temp, kdb, n, nseg, db, de, begin_bit, end_bit)
        return kdb.current().cpu().numpy(), None, kdb.selector
    vdb = L.DoubleBuffer(_dev(np.full_like(vals, 0xEE)), _dev(vals), 1)
    pfn(temp, kdb, vdb, n, nseg, db, de, begin_bit, end_bit)
    assert vdb.selector == kdb.selector
    return kdb.current().cpu().numpy(), vdb.current().cpu().numpy(), kdb.selector


def test_reference_case_all_entry_points(golden, lcpp):
    keys, vals = golden["segmented_keys"], golden["segmented_vals"]
    b, e = golden["segmented_begin"], golden["segmented_end"]
    n = keys.size
    for desc, name in ((False, "segmented_asc_order"), (True, "segmented_desc_order")):
        order = golden[name]
        inside = order != 0xFFFFFFFF
        for form in ("copy", "double_buffer"):
            ok, _, sel = _run(lcpp, keys, None, b, e, 0, 32, desc, form)
            np.testing.assert_array_equal(ok[inside], keys[order[inside]])
            if form == "copy":
                assert (ok[~inside] == -777).all()
            else:
                assert sel == 1 ^ (int(n - 1).bit_length() & 1)  # ceil(log2 19) = 5 flips
            ok, ov, sel = _run(lcpp, keys, vals, b, e, 0, 32, desc, form)
            np.testing.assert_array_equal(ok[inside], keys[order[inside]])
            np.testing.assert_array_equal(ov[inside], vals[order[inside]])


def _keys_for(rng, dt, n, case):
    dt = np.dtype(dt)
    if dt.kind == "f":
        k = rng.standard_normal(n).astype(dt)
        k[::11] = 0.0
        k[5::11] = -0.0
        return k
    if case == "ties":
        return rng.integers(0, 5, n).astype(dt)
    info = np.iinfo(dt)
    return rng.integers(info.min, info.max, n, dtype=dt, endpoint=True)


def _segments(rng, n, layout):
    if layout == "one":
        return np.array([0], np.uint32), np.array([n], np.uint32)
    if layout == "gaps":  # sorted segments with gaps, empty and invalid ones
        cuts = np.sort(rng.choice(n, 40, replace=False)).astype(np.uint32)
        b, e = cuts[0::2].copy(), cuts[1::2].copy()
        e[3] = b[3]          # empty
        e[5] = b[5] - 1 if b[5] > 0 else b[5]  # begin > end: inactive
        return b, e
    if layout == "many":  # contiguous small segments covering everything
        sizes = rng.integers(0, 300, n)
        cum = np.concatenate([[0], np.cumsum(sizes)])
        cum = cum[cum < n]
        b = cum.astype(np.uint32)
        e = np.concatenate([cum[1:], [n]]).astype(np.uint32)
        return b, e
    raise ValueError(layout)


@pytest.mark.parametrize("dt", [np.uint32, np.int32, np.float32, np.uint64, np.int64, np.float64])
@pytest.mark.parametrize("desc", [False, True])
@pytest.mark.parametrize("layout", ["one", "gaps", "many"])
def test_keys_vs_oracle(lcpp, oracle, dt, desc, layout):
    rng = np.random.default_rng(zlib.crc32(repr((np.dtype(dt).str, desc, layout)).encode()))
    n = 20_011
    keys = _keys_for(rng, dt, n, "uniform")
    b, e = _segments(rng, n, layout)
    bits = np.dtype(dt).itemsize * 8
    for begin_bit, end_bit in ((0, bits), (3, 17), (0, 0)):
        ok, _, _ = _run(lcpp, keys, None, b, e, begin_bit, end_bit, desc, "copy")
        exp, _ = oracle.segmented_radix_sort(keys, None, b, e, begin_bit, end_bit, desc,
                                             out_keys=np.full_like(keys, SENT[keys.dtype]))
        np.testing.assert_array_equal(_bits(ok), _bits(exp))


@pytest.mark.parametrize("kdt,vdt", [(np.uint32, np.uint32), (np.float32, np.uint32), (np.int64, np.int32),
                                     (np.uint64, np.uint64), (np.int32, np.float64)])
@pytest.mark.parametrize("form", ["copy", "double_buffer"])
def test_pairs_vs_oracle(lcpp, oracle, kdt, vdt, form):
    rng = np.random.default_rng(7)
    n = 50_003
    keys = _keys_for(rng, kdt, n, "ties")  # many equal keys: stability shows in the values
    vals = np.arange(n).astype(vdt)
    b, e = _segments(rng, n, "gaps")
    for desc in (False, True):
        ok, ov, sel = _run(lcpp, keys, vals, b, e, 0, np.dtype(kdt).itemsize * 8, desc, form)
        exp_k, exp_v = oracle.segmented_radix_sort(keys, vals, b, e, 0, None, desc)
        inside = np.zeros(n, bool)
        for lo, hi in zip(b, e):
            inside[lo:hi] |= lo <= hi
        np.testing.assert_array_equal(_bits(ok)[inside], _bits(exp_k)[inside])
        np.testing.assert_array_equal(ov[inside].view(np.uint8).reshape(-1), exp_v[inside].view(np.uint8).reshape(-1))
        if form == "double_buffer":
            assert sel == 1 ^ (int(n - 1).bit_length() & 1)


def test_in_place_double_buffer(lcpp, oracle):
    """An even number of flips puts the result back into the input slot."""
    rng = np.random.default_rng(9)
    n = 1000  # ceil(log2 1000) = 10 flips
    keys = rng.integers(0, 100, n).astype(np.uint32)
    vals = np.arange(n, dtype=np.uint32)
    b, e = _segments(rng, n, "many")
    ok, ov, sel = _run(lcpp, keys, vals, b, e, 0, 32, False, "double_buffer")
    assert sel == 1
    exp_k, exp_v = oracle.segmented_radix_sort(keys, vals, b, e)
    np.testing.assert_array_equal(ok, exp_k)
    np.testing.assert_array_equal(ov, exp_v)


def test_two_sort_path_and_narrow_composite(lcpp, oracle):
    """64-bit keys over the full width with many segments (composite wider
    than 64 bits: key sort, then segment sort) and an 8-bit field with few
    segments (composite within 32 bits)."""
    rng = np.random.default_rng(11)
    n = 100_000
    keys = rng.integers(0, 2**64 - 1, n, dtype=np.uint64)
    keys[::3] = keys[5]
    # long segments (composite sort) mixed with short ones (one block each)
    b = np.array([0, 5000, 5100, 70000, 70001], np.uint32)
    e = np.array([5000, 5100, 70000, 70001, n], np.uint32)
    for desc in (False, True):
        ok, _, _ = _run(lcpp, keys, None, b, e, 0, 64, desc, "copy")
        exp, _ = oracle.segmented_radix_sort(keys, None, b, e, 0, 64, desc)
        np.testing.assert_array_equal(ok, exp)
    k32 = rng.integers(0, 2**32, n, dtype=np.uint64).astype(np.uint32)
    b, e = np.array([0, 10, 60_000], np.uint32), np.array([10, 60_000, n], np.uint32)
    ok, _, _ = _run(lcpp, k32, None, b, e, 8, 16, True, "copy")
    exp, _ = oracle.segmented_radix_sort(k32, None, b, e, 8, 16, True)
    np.testing.assert_array_equal(ok, exp)


@pytest.mark.parametrize("kdt,vdt", [(np.uint32, None), (np.int32, np.uint32), (np.float64, np.uint64),
                                     (np.uint64, np.uint32)])
def test_short_segment_kernel_boundaries(lcpp, oracle, kdt, vdt):
    """Segment lengths around the one-block limit (2048): 0, 1, 2, 2047, 2048
    (one block) and 2049 (composite sort), in one call."""
    rng = np.random.default_rng(17)
    sizes = [0, 1, 2, 31, 33, 2047, 2048, 2049, 5, 4096, 2048]
    cum = np.concatenate([[0], np.cumsum(sizes)]).astype(np.uint32)
    n = int(cum[-1]) + 10  # trailing items outside every segment
    keys = _keys_for(rng, kdt, n, "ties")
    vals = None if vdt is None else np.arange(n).astype(vdt)
    for desc in (False, True):
        ok, ov, _ = _run(lcpp, keys, vals, cum[:-1], cum[1:], 0, np.dtype(kdt).itemsize * 8, desc, "copy")
        exp_k, exp_v = oracle.segmented_radix_sort(keys, vals, cum[:-1], cum[1:], 0, None, desc)
        m = int(cum[-1])
        np.testing.assert_array_equal(_bits(ok)[:m], _bits(exp_k)[:m])
        assert (_bits(ok)[m:] == _bits(np.full(10, SENT[keys.dtype], keys.dtype))).all()
        if vals is not None:
            np.testing.assert_array_equal(ov[:m], exp_v[:m])


def test_large(lcpp, oracle):
    rng = np.random.default_rng(13)
    n = (1 << 24) + 3
    keys = rng.integers(0, 2**32, n, dtype=np.uint64).astype(np.uint32)
    sizes = rng.integers(1, 8192, n // 1000)
    cum = np.concatenate([[0], np.cumsum(sizes)])
    cum = cum[cum < n]
    b = cum.astype(np.uint32)
    e = np.concatenate([cum[1:], [n]]).astype(np.uint32)
    ok, _, _ = _run(lcpp, keys, None, b, e, 0, 32, False, "copy")
    exp, _ = oracle.segmented_radix_sort(keys, None, b, e)
    np.testing.assert_array_equal(ok, exp)


def test_empty_and_misuse(lcpp):
    import ctypes
    L = lcpp.lib()
    t = ctypes.c_size_t(0)
    assert L.lcpp_segmented_radix_sort_keys_temp_bytes(lcpp.U32, 0, ctypes.byref(t)) == lcpp.OK and t.value == 0
    k = torch.zeros(16, dtype=torch.int32, device="cuda")
    o = torch.zeros(16, dtype=torch.int32, device="cuda")
    b = torch.zeros(1, dtype=torch.int32, device="cuda")
    e = torch.full((1,), 16, dtype=torch.int32, device="cuda")
    assert L.lcpp_segmented_radix_sort_keys_temp_bytes(lcpp.I32, 16, ctypes.byref(t)) == lcpp.OK
    temp = lcpp.alloc_temp(t.value)
    p = lambda x: ctypes.c_void_p(x.data_ptr())  # noqa: E731
    args = (p(k), p(o), 16, 1, p(b), p(e))
    assert L.lcpp_segmented_radix_sort_keys(p(temp), t.value, *args, 0, 33, 0, lcpp.I32, None) == lcpp.ERR_INVALID_ARG
    assert L.lcpp_segmented_radix_sort_keys(p(temp), t.value - 1, *args, 0, 32, 0, lcpp.I32,
                                            None) == lcpp.ERR_TEMP_TOO_SMALL
    assert L.lcpp_segmented_radix_sort_keys(p(temp), t.value, p(k), p(o), 16, 0, p(b), p(e), 0, 32, 0, lcpp.I32,
                                            None) == lcpp.OK  # no segments: nothing to do
    assert L.lcpp_segmented_radix_sort_keys(p(temp), t.value, p(k), p(o), 16, 1, None, None, 0, 32, 0, lcpp.I32,
                                            None) == lcpp.ERR_INVALID_ARG
