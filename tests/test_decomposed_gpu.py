"""GPU tests of DeviceRadixSort over decomposed (struct) keys: the reference
test's own case (golden fixture) for all eight entry points and selector
outcomes, then seeded multi-member cases against the oracle."""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def _struct(cols, dtypes):
    """Packs member columns into an (n, key_bytes) uint8 array (natural alignment)."""
    rec = np.dtype({"names": [f"m{i}" for i in range(len(cols))], "formats": dtypes, "align": True})
    a = np.zeros(cols[0].size, dtype=rec)
    for i, c in enumerate(cols):
        a[f"m{i}"] = c
    return a, rec


def _dev_bytes(a):
    return torch.from_numpy(a.view(np.uint8).reshape(-1).copy()).cuda()


def test_reference_case(golden, lcpp):
    p, s = golden["decomposed_primary"], golden["decomposed_secondary"]
    keys, rec = _struct([p, s], [np.uint32, np.int32])
    n = keys.size
    vals = np.arange(n, dtype=np.uint32)
    dec = lcpp.Decomposer(rec.itemsize, [(rec.fields["m0"][1], lcpp.U32), (rec.fields["m1"][1], lcpp.I32)])
    rs = lcpp.DeviceRadixSort()
    temp = lcpp.alloc_temp(lcpp.DeviceRadixSort.GetDecomposedTempStorageBytes(n))
    kin = _dev_bytes(keys)
    vin = torch.from_numpy(vals).cuda()

    def got(t):
        return np.frombuffer(t.cpu().numpy().tobytes(), dtype=rec)

    def check(out_keys, order, out_vals=None):
        np.testing.assert_array_equal(got(out_keys), keys[order])
        if out_vals is not None:
            np.testing.assert_array_equal(out_vals.cpu().numpy(), vals[order])

    full_asc, full_desc = golden["decomposed_full_asc_order"], golden["decomposed_full_desc_order"]
    win_asc, win_desc = golden["decomposed_window_asc_order"], golden["decomposed_window_desc_order"]
    # copy forms (the reference test's combinations)
    ko = torch.empty_like(kin)
    rs.SortKeys(temp, kin, ko, n, dec)
    check(ko, full_asc)
    rs.SortKeysDescending(temp, kin, ko, n, dec, 28, 36)
    check(ko, win_desc)
    vo = torch.empty_like(vin)
    rs.SortPairs(temp, kin, ko, vin, vo, n, dec, 28, 36)
    check(ko, win_asc, vo)
    rs.SortPairsDescending(temp, kin, ko, vin, vo, n, dec)
    check(ko, full_desc, vo)
    # DoubleBuffer forms: one flip each
    db = lcpp.DoubleBuffer(kin.clone(), torch.empty_like(kin))
    rs.SortKeys(temp, db, n, dec, 28, 36)
    assert db.selector == 1
    check(db.current(), win_asc)
    db = lcpp.DoubleBuffer(torch.empty_like(kin), kin.clone(), 1)
    rs.SortKeysDescending(temp, db, n, dec)
    assert db.selector == 0
    check(db.current(), full_desc)
    kdb = lcpp.DoubleBuffer(kin.clone(), torch.empty_like(kin))
    vdb = lcpp.DoubleBuffer(vin.clone(), torch.empty_like(vin))
    rs.SortPairs(temp, kdb, vdb, n, dec)
    assert kdb.selector == 1 and vdb.selector == 1
    check(kdb.current(), full_asc, vdb.current())
    kdb = lcpp.DoubleBuffer(torch.empty_like(kin), kin.clone(), 1)
    vdb = lcpp.DoubleBuffer(torch.empty_like(vin), vin.clone(), 1)
    rs.SortPairsDescending(temp, kdb, vdb, n, dec, 28, 36)
    assert kdb.selector == 0 and vdb.selector == 0
    check(kdb.current(), win_desc, vdb.current())
    # empty window: the copy form copies, the DoubleBuffer form does nothing
    rs.SortKeys(temp, kin, ko, n, dec, 5, 5)
    check(ko, np.arange(n))
    db = lcpp.DoubleBuffer(kin.clone(), torch.empty_like(kin))
    rs.SortKeys(temp, db, n, dec, 5, 5)
    assert db.selector == 0


@pytest.mark.parametrize("desc", [False, True])
@pytest.mark.parametrize("window", [None, (30, 100), (96, 160), (0, 1)])
def test_three_members_vs_oracle(lcpp, oracle, desc, window):
    """{i64, f32, u64} keys (160 bits: three 64-bit chunks), ties and +-0.0."""
    rng = np.random.default_rng(21)
    n = 100_003
    a = rng.integers(-3, 3, n).astype(np.int64)
    b = rng.standard_normal(n).astype(np.float32)
    b[::9] = 0.0
    b[4::9] = -0.0
    c = rng.integers(0, 5, n).astype(np.uint64)
    keys, rec = _struct([a, b, c], [np.int64, np.float32, np.uint64])
    dec = lcpp.Decomposer(rec.itemsize, [(rec.fields["m0"][1], lcpp.I64), (rec.fields["m1"][1], lcpp.F32),
                                         (rec.fields["m2"][1], lcpp.U64)])
    lo, hi = window if window else (0, 160)
    vals = np.arange(n, dtype=np.int32)
    rs = lcpp.DeviceRadixSort()
    temp = lcpp.alloc_temp(lcpp.DeviceRadixSort.GetDecomposedTempStorageBytes(n))
    kin, ko = _dev_bytes(keys), torch.empty(n * rec.itemsize, dtype=torch.uint8, device="cuda")
    vin, vo = torch.from_numpy(vals).cuda(), torch.empty(n, dtype=torch.int32, device="cuda")
    (rs.SortPairsDescending if desc else rs.SortPairs)(temp, kin, ko, vin, vo, n, dec, lo, hi)
    order = oracle.decomposed_sort_order([a, b, c], lo, hi, desc)
    np.testing.assert_array_equal(vo.cpu().numpy(), vals[order])
    got = np.frombuffer(ko.cpu().numpy().tobytes(), dtype=rec)
    np.testing.assert_array_equal(got.view(np.uint8), keys[order].view(np.uint8))


def test_misuse(lcpp):
    import ctypes
    L = lcpp.lib()
    m = (lcpp.KeyMember * 2)(lcpp.KeyMember(0, lcpp.U32), lcpp.KeyMember(4, lcpp.I32))
    k = torch.zeros(64, dtype=torch.uint8, device="cuda")
    o = torch.zeros(64, dtype=torch.uint8, device="cuda")
    temp = lcpp.alloc_temp(lcpp.DeviceRadixSort.GetDecomposedTempStorageBytes(8))
    p = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    assert L.lcpp_radix_sort_decomposed_keys(p(temp), temp.numel(), p(k), p(o), 8, 8, m, 2, 0, 65, 0,
                                             None) == lcpp.ERR_INVALID_ARG  # window past the members
    assert L.lcpp_radix_sort_decomposed_keys(p(temp), temp.numel(), p(k), p(k), 8, 8, m, 2, 0, 64, 0,
                                             None) == lcpp.ERR_INVALID_ARG  # in place
    bad = (lcpp.KeyMember * 1)(lcpp.KeyMember(6, lcpp.U32))  # member past the struct
    assert L.lcpp_radix_sort_decomposed_keys(p(temp), temp.numel(), p(k), p(o), 8, 8, bad, 1, 0, 32, 0,
                                             None) == lcpp.ERR_INVALID_ARG
    assert L.lcpp_radix_sort_decomposed_keys(p(temp), 16, p(k), p(o), 8, 8, m, 2, 0, 64, 0,
                                             None) == lcpp.ERR_TEMP_TOO_SMALL
