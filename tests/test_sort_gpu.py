"""GPU parity tests for DeviceRadixSort (C ABI), mirroring the reference's
tests/device_radix_sort_one_sweep.cpp and tests/device_radix_sort_interface_test.cpp,
plus oracle comparisons across dtypes / bit ranges / edge sizes and
size-independent properties at the BASELINE sizes (2^27, 2^28)."""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
from gpu_helpers import dev, empty_like_np, gpu_sort, host, transformed_key_u64  # noqa: E402


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"


# ------------------------------------------------------------ golden vectors
@pytest.mark.parametrize("n", [1 << k for k in range(5, 15)])
def test_float_keys_golden(golden, n):
    """device_radix_sort_one_sweep.cpp:79-136: float keys, SortKeys + SortKeysDescending."""
    assert golden.matches(f"float_keys_asc_out_{n}", gpu_sort(golden[f"float_keys_asc_in_{n}"]))
    assert golden.matches(f"float_keys_desc_out_{n}",
                          gpu_sort(golden[f"float_keys_desc_in_{n}"], descending=True))


def test_reversed_u32_all_sizes():
    """device_radix_sort_one_sweep.cpp:138-173: keys n-i-1, n = 2^0 .. 2^23."""
    for k in range(0, 24):
        n = 1 << k
        keys = (n - 1 - np.arange(n)).astype(np.uint32)
        np.testing.assert_array_equal(gpu_sort(keys), np.arange(n, dtype=np.uint32), err_msg=f"n={n}")


def test_u64_keys_golden(golden):
    """device_radix_sort_one_sweep.cpp:175-205."""
    assert golden.matches("u64_keys_out", gpu_sort(golden["u64_keys_in"]))


@pytest.mark.parametrize("desc", [False, True])
def test_pairs_golden(golden, desc):
    """device_radix_sort_one_sweep.cpp:207-333 (uint keys, float values)."""
    tag = "desc" if desc else "asc"
    k, v = gpu_sort(golden[f"pairs_{tag}_keys_in"], golden[f"pairs_{tag}_vals_in"], descending=desc)
    assert golden.matches(f"pairs_{tag}_keys_out", k)
    assert golden.matches(f"pairs_{tag}_vals_out", v)


@pytest.mark.parametrize("desc", [False, True])
def test_partial_bits_golden(golden, desc):
    """device_radix_sort_interface_test.cpp:68-158: 257 keys, bits [1,6), stable."""
    keys, vals = golden["partial_bits_keys"], golden["partial_bits_vals"]
    order = golden[f"partial_bits_{'desc' if desc else 'asc'}_order"]
    np.testing.assert_array_equal(gpu_sort(keys, begin_bit=1, end_bit=6, descending=desc), keys[order])
    k, v = gpu_sort(keys, vals, begin_bit=1, end_bit=6, descending=desc)
    np.testing.assert_array_equal(k, keys[order])
    np.testing.assert_array_equal(v, vals[order])


def test_double_buffer_selectors_golden(golden, lcpp):
    """device_radix_sort_interface_test.cpp:205-283."""
    keys, vals = golden["double_buffer_keys"], golden["double_buffer_vals"]
    n = keys.size
    rs = lcpp.DeviceRadixSort()
    temp = lcpp.alloc_temp(rs.GetSortPairsTempStorageBytes(lcpp.U32, lcpp.U32, n))
    kb = lcpp.DoubleBuffer(empty_like_np(keys), dev(keys), selector=1)
    rs.SortKeys(temp, kb, n, 0, 5)
    assert kb.selector == 0
    pk = lcpp.DoubleBuffer(dev(keys), empty_like_np(keys))
    pv = lcpp.DoubleBuffer(dev(vals), empty_like_np(vals))
    rs.SortPairsDescending(temp, pk, pv, n, 0, 5)
    assert pk.selector == 1 and pv.selector == pk.selector
    asc, desc = golden["double_buffer_asc_order"], golden["double_buffer_desc_order"]
    np.testing.assert_array_equal(host(kb.current()), keys[asc])
    np.testing.assert_array_equal(host(pk.current()), keys[desc])
    np.testing.assert_array_equal(host(pv.current()), vals[desc])


def test_double_buffer_zero_width_keeps_current(lcpp):
    """device_radix_sort_interface_test.cpp:285-300: begin == end leaves the selector."""
    data = np.array([7, 2, 5], np.int32)
    db = lcpp.DoubleBuffer(torch.zeros(3, dtype=torch.int32, device="cuda"), dev(data), selector=1)
    lcpp.DeviceRadixSort().SortKeys(None, db, 3, 4, 4)
    assert db.selector == 1
    np.testing.assert_array_equal(host(db.current()), data)


def test_zero_width_copy(lcpp):
    """device_radix_sort_interface_test.cpp:161-195."""
    keys = (np.arange(17) * 7 - 31).astype(np.int32)
    vals = (17 - np.arange(17)).astype(np.uint32)
    kin, vin = dev(keys), dev(vals)
    kout, vout = empty_like_np(keys), empty_like_np(vals)
    lcpp.DeviceRadixSort().SortPairs(None, kin, kout, vin, vout, 17, 9, 9)
    np.testing.assert_array_equal(host(kout), keys)
    np.testing.assert_array_equal(host(vout), vals)


def test_empty_input(lcpp):
    """device_radix_sort_interface_test.cpp:197-203."""
    e = torch.empty(0, dtype=torch.int32, device="cuda")
    lcpp.DeviceRadixSort().SortKeys(None, e, e, 0)
    assert lcpp.DeviceRadixSort.GetSortKeysTempStorageBytes(lcpp.I32, 0) == 0


# ------------------------------------------------- oracle, dtypes x edge sizes
# around the tiles of every key / value class (4-byte keys 448 x 28 = 12544,
# or 448 x 24 = 10752 in the persistent bulk-copy pass, 4-byte pairs 512 x 16
# = 8192, 8-byte keys 384 x 16 = 6144, pairs with an 8-byte key or value
# 256 x 20 = 5120) and multiples of them; 3,500,017 keys give every
# persistent block of a pass several tiles and a partial last tile
EDGE_SIZES = [1, 2, 31, 33, 255, 5119, 5120, 5121, 6143, 6144, 6145, 8191, 8192, 8193, 10751, 10752, 10753,
              12543, 12544, 12545, 21505, 25089, 65537, 1_000_003, 3_500_017]


def _random_keys(dtype, n, seed):
    rng = np.random.default_rng(seed)
    w = np.dtype(dtype).itemsize * 8
    raw = rng.integers(0, 2**63, size=n, dtype=np.uint64) * np.uint64(2) + rng.integers(0, 2, size=n, dtype=np.uint64)
    if w == 32:
        raw = (raw & np.uint64(0xFFFFFFFF)).astype(np.uint32)
    keys = raw.view(dtype).copy()
    if np.dtype(dtype).kind == "f":
        keys[np.isnan(keys)] = 1.5
        keys[::53] = 0.0
        keys[7::61] = -0.0
    keys[3::17] = keys[0]  # duplicates exercise stability
    return keys


@pytest.mark.parametrize("dtype", [np.uint32, np.int32, np.float32, np.uint64, np.int64, np.float64])
@pytest.mark.parametrize("n", EDGE_SIZES)
def test_keys_vs_oracle(oracle, dtype, n):
    keys = _random_keys(dtype, n, n)
    for desc in (False, True):
        got = gpu_sort(keys, descending=desc)
        exp = oracle.radix_sort(keys, descending=desc, threads=4)
        np.testing.assert_array_equal(got.view(np.uint8), exp.view(np.uint8), err_msg=f"desc={desc}")


@pytest.mark.parametrize("dtype", [np.uint32, np.int32, np.float32])
@pytest.mark.parametrize("n", [10753, 3_500_017])
@pytest.mark.parametrize("begin,end", [(0, 32), (4, 27)])
def test_keys_bulk_and_register_paths_agree(oracle, dtype, n, begin, end):
    """Keys-only 4-byte sorts take the persistent bulk-copy pass when every
    pass reads a 16-byte aligned buffer and the register-load pass
    otherwise; buffers 4 bytes past a 16-byte boundary force the latter.
    Both must equal the oracle bit for bit."""
    import lcpp_b200 as L
    from gpu_helpers import NP_TO_CODE

    keys = _random_keys(dtype, n, n + begin)
    kd = NP_TO_CODE[np.dtype(dtype)]
    exp = oracle.radix_sort(keys, begin_bit=begin, end_bit=end, threads=4)
    rs = L.DeviceRadixSort()
    for off in (0, 1):
        src = torch.empty(n + 4, dtype=torch.from_numpy(keys[:0]).dtype, device="cuda")
        dst = torch.empty_like(src)
        src[off:off + n].copy_(torch.from_numpy(keys).to("cuda"))
        temp = L.alloc_temp(rs.GetSortKeysTempStorageBytes(kd, n))
        rs.SortKeys(temp, src[off:off + n], dst[off:off + n], n, begin, end)
        assert L.device_status(temp) == L.OK
        got = dst[off:off + n].cpu().numpy()
        np.testing.assert_array_equal(got.view(np.uint8), exp.view(np.uint8), err_msg=f"buffer offset {off}")


@pytest.mark.parametrize("kdtype,vdtype", [(np.uint32, np.uint32), (np.float32, np.uint32),
                                           (np.uint64, np.int32), (np.int32, np.float64),
                                           (np.float64, np.uint64), (np.int64, np.float32)])
@pytest.mark.parametrize("n", [1, 33, 5119, 5121, 8191, 8193, 16385, 262147, 1_000_003])
def test_pairs_vs_oracle(oracle, kdtype, vdtype, n):
    keys = _random_keys(kdtype, n, n + 1)
    vals = np.arange(n, dtype=np.uint64).astype(vdtype)
    for desc in (False, True):
        k, v = gpu_sort(keys, vals, descending=desc)
        ek, ev = oracle.radix_sort(keys, vals, descending=desc, threads=4)
        np.testing.assert_array_equal(k.view(np.uint8), ek.view(np.uint8))
        np.testing.assert_array_equal(v.view(np.uint8), ev.view(np.uint8))


@pytest.mark.parametrize("dtype", [np.uint32, np.float32, np.int64])
@pytest.mark.parametrize("begin,end", [(0, 1), (1, 6), (3, 11), (8, 24), (5, 29), (16, 32), (7, 8)])
def test_bit_ranges_vs_oracle(oracle, dtype, begin, end):
    n = 300_007
    keys = _random_keys(dtype, n, begin * 100 + end)
    vals = np.arange(n, dtype=np.uint32)
    for desc in (False, True):
        k, v = gpu_sort(keys, vals, begin_bit=begin, end_bit=end, descending=desc)
        ek, ev = oracle.radix_sort(keys, vals, begin_bit=begin, end_bit=end, descending=desc, threads=4)
        np.testing.assert_array_equal(k.view(np.uint8), ek.view(np.uint8))
        np.testing.assert_array_equal(v, ev)


@pytest.mark.parametrize("dist", ["U32_UNIFORM", "U32_AND3", "U32_CONST", "U32_ZIPF", "F32_NORMAL",
                                  "U64_UNIFORM"])
def test_distributions_vs_oracle(oracle, lcpp, dist):
    """BASELINE key distributions at 2^22 (device-generated), bit-exact vs the oracle."""
    n = 1 << 22
    code = getattr(lcpp, f"GEN_{dist}")
    tdt = {"U64": torch.uint64, "F32": torch.float32}.get(dist[:3], torch.uint32)
    keys_t = torch.empty(n, dtype=tdt, device="cuda")
    lcpp.testgen_fill(keys_t, code, seed=1)
    keys = host(keys_t)
    vals = np.arange(n, dtype=np.uint32)
    k, v = gpu_sort(keys, vals)
    ek, ev = oracle.radix_sort(keys, vals, threads=8)
    np.testing.assert_array_equal(k.view(np.uint8), ek.view(np.uint8))
    np.testing.assert_array_equal(v, ev)


def test_input_untouched_and_repeatable():
    keys = _random_keys(np.uint32, 100_003, 11)
    kin = dev(keys)
    import lcpp_b200 as L
    rs = L.DeviceRadixSort()
    temp = L.alloc_temp(rs.GetSortKeysTempStorageBytes(L.U32, keys.size))
    outs = []
    for _ in range(3):
        kout = torch.empty_like(kin)
        rs.SortKeys(temp, kin, kout, keys.size)
        outs.append(host(kout))
    np.testing.assert_array_equal(host(kin), keys)
    for o in outs[1:]:
        np.testing.assert_array_equal(o, outs[0])


def test_guarded_temp_canaries(lcpp):
    """The sort writes nothing past the queried temp size (the reference's
    GuardedTemp fixture, tests/pr6_review_regression_test.cpp:69-98)."""
    for n in (1, 7681, 300_000):
        keys = _random_keys(np.uint32, n, 5)
        vals = np.arange(n, dtype=np.uint32)
        rs = lcpp.DeviceRadixSort()
        tb = rs.GetSortPairsTempStorageBytes(lcpp.U32, lcpp.U32, n)
        backing = torch.full((tb + 16384,), 0xA5, dtype=torch.uint8, device="cuda")
        temp = backing[:tb]
        kout, vout = empty_like_np(keys), empty_like_np(vals)
        rs.SortPairs(temp, dev(keys), kout, dev(vals), vout, n)
        torch.cuda.synchronize()
        assert bool((backing[tb:] == 0xA5).all())


# --------------------------------------- size-independent properties, full size
def _check_sorted_stable_permutation(keys_in, keys_out, vals_out, kind, bits, desc=False):
    """keys_out[i] == keys_in[vals_out[i]] (bit-exact), vals_out a permutation,
    keys ordered by the transformed key, ties in increasing index order."""
    n = keys_in.numel()
    idx = vals_out.view(torch.int32).to(torch.int64) & 0xFFFFFFFF
    seen = torch.zeros(n, dtype=torch.bool, device="cuda")
    seen[idx] = True
    assert bool(seen.all()), "values are not a permutation of the indices"
    del seen
    if bits == 32:
        assert torch.equal(keys_out.view(torch.int32), keys_in.view(torch.int32)[idx])
    else:
        assert torch.equal(keys_out.view(torch.int64), keys_in.view(torch.int64)[idx])
    t = transformed_key_u64(keys_out, kind, bits)
    if desc:
        t = -t if bits == 32 else ~t
    d = t[1:] - t[:-1] if bits == 32 else None
    if bits == 32:
        assert bool((d >= 0).all()), "keys out of order"
        ties = d == 0
    else:
        assert bool((t[1:] >= t[:-1]).all()), "keys out of order"
        ties = t[1:] == t[:-1]
    assert bool((idx[1:][ties] > idx[:-1][ties]).all()), "equal keys lost their input order"


@pytest.mark.parametrize("dist", ["U32_UNIFORM", "U32_AND3", "U32_CONST"])
def test_pairs_2p28_properties(lcpp, dist):
    """SortPairs u32 -> u32 index, n = 2^28, seed 1."""
    n = 1 << 28
    keys = torch.empty(n, dtype=torch.uint32, device="cuda")
    lcpp.testgen_fill(keys, getattr(lcpp, f"GEN_{dist}"), seed=1)
    vals = torch.empty(n, dtype=torch.uint32, device="cuda")
    lcpp.testgen_fill(vals, lcpp.GEN_U32_INDEX, seed=1)
    rs = lcpp.DeviceRadixSort()
    temp = lcpp.alloc_temp(rs.GetSortPairsTempStorageBytes(lcpp.U32, lcpp.U32, n))
    kout, vout = torch.empty_like(keys), torch.empty_like(vals)
    rs.SortPairs(temp, keys, kout, vals, vout, n)
    assert lcpp.device_status(temp) == lcpp.OK
    del temp
    _check_sorted_stable_permutation(keys, kout, vout, "u", 32)


def test_keys_2p28_uniform_exact(lcpp):
    """Headline config (the bench's workload): SortKeys u32, n = 2^28 uniform
    keys, seed 0, bits [0, 32), compared element for element with torch.sort
    of the same keys widened to int64 (the reference test's std::sort check,
    tests/device_radix_sort_one_sweep.cpp:160-171, at the full size)."""
    n = 1 << 28
    keys = torch.empty(n, dtype=torch.uint32, device="cuda")
    lcpp.testgen_fill(keys, lcpp.GEN_U32_UNIFORM, seed=0)
    rs = lcpp.DeviceRadixSort()
    temp = lcpp.alloc_temp(rs.GetSortKeysTempStorageBytes(lcpp.U32, n))
    kout = torch.empty_like(keys)
    rs.SortKeys(temp, keys, kout, n)
    assert lcpp.device_status(temp) == lcpp.OK
    del temp
    expect = torch.sort(keys.view(torch.int32).to(torch.int64) & 0xFFFFFFFF).values
    got = kout.view(torch.int32).to(torch.int64) & 0xFFFFFFFF
    assert torch.equal(got, expect)
    # the input is untouched (copy API)
    again = torch.empty_like(keys)
    lcpp.testgen_fill(again, lcpp.GEN_U32_UNIFORM, seed=0)
    assert torch.equal(again, keys)


@pytest.mark.parametrize("desc", [False, True])
def test_f32_normal_2p27_properties(lcpp, desc):
    """SortPairs f32 N(0,1) with +-0.0 -> u32 index, n = 2^27."""
    n = 1 << 27
    keys = torch.empty(n, dtype=torch.float32, device="cuda")
    lcpp.testgen_fill(keys, lcpp.GEN_F32_NORMAL, seed=1)
    vals = torch.empty(n, dtype=torch.uint32, device="cuda")
    lcpp.testgen_fill(vals, lcpp.GEN_U32_INDEX, seed=1)
    rs = lcpp.DeviceRadixSort()
    temp = lcpp.alloc_temp(rs.GetSortPairsTempStorageBytes(lcpp.F32, lcpp.U32, n))
    kout, vout = torch.empty_like(keys), torch.empty_like(vals)
    (rs.SortPairsDescending if desc else rs.SortPairs)(temp, keys, kout, vals, vout, n)
    assert lcpp.device_status(temp) == lcpp.OK
    del temp
    _check_sorted_stable_permutation(keys, kout, vout, "f", 32, desc)
    # both zeros present, kept in input order within the merged zero run
    z = kout == 0
    assert int(z.sum()) == 2 * (n // 65536)
    assert bool(torch.signbit(kout[z]).any()) and bool((~torch.signbit(kout[z])).any())


def test_u64_2p27_properties(lcpp):
    """SortPairs u64 uniform -> i32 index, n = 2^27."""
    n = 1 << 27
    keys = torch.empty(n, dtype=torch.uint64, device="cuda")
    lcpp.testgen_fill(keys, lcpp.GEN_U64_UNIFORM, seed=1)
    vals = torch.empty(n, dtype=torch.int32, device="cuda")
    lcpp.testgen_fill(vals, lcpp.GEN_U32_INDEX, seed=1)
    rs = lcpp.DeviceRadixSort()
    temp = lcpp.alloc_temp(rs.GetSortPairsTempStorageBytes(lcpp.U64, lcpp.I32, n))
    kout, vout = torch.empty_like(keys), torch.empty_like(vals)
    rs.SortPairs(temp, keys, kout, vals, vout, n)
    assert lcpp.device_status(temp) == lcpp.OK
    del temp
    _check_sorted_stable_permutation(keys, kout, vout, "u", 64)


def test_partial_bits_2p27(lcpp, oracle):
    """SortKeys u32 bits [8,24), n = 2^27; checked against
    the oracle on a 2^22 prefix and by properties at full size."""
    n = 1 << 27
    keys = torch.empty(n, dtype=torch.uint32, device="cuda")
    lcpp.testgen_fill(keys, lcpp.GEN_U32_UNIFORM, seed=1)
    rs = lcpp.DeviceRadixSort()
    temp = lcpp.alloc_temp(rs.GetSortPairsTempStorageBytes(lcpp.U32, lcpp.U32, n))
    vals = torch.empty(n, dtype=torch.uint32, device="cuda")
    lcpp.testgen_fill(vals, lcpp.GEN_U32_INDEX, seed=1)
    kout, vout = torch.empty_like(keys), torch.empty_like(vals)
    rs.SortPairs(temp, keys, kout, vals, vout, n, 8, 24)
    assert lcpp.device_status(temp) == lcpp.OK
    idx = vout.view(torch.int32).to(torch.int64) & 0xFFFFFFFF
    assert torch.equal(kout.view(torch.int32), keys.view(torch.int32)[idx])
    sel = (transformed_key_u64(kout, "u", 32) >> 8) & 0xFFFF
    d = sel[1:] - sel[:-1]
    assert bool((d >= 0).all())
    assert bool((idx[1:][d == 0] > idx[:-1][d == 0]).all())
    kout2 = torch.empty_like(keys)
    rs.SortKeys(temp, keys, kout2, n, 8, 24)
    assert torch.equal(kout2.view(torch.int32), kout.view(torch.int32))
    # small-prefix bit-exact oracle check
    m = 1 << 22
    ks = host(keys[:m])
    got = gpu_sort(ks, begin_bit=8, end_bit=24)
    np.testing.assert_array_equal(got, oracle.radix_sort(ks, begin_bit=8, end_bit=24, threads=8))


def test_wide_layout_above_2p30(lcpp):
    """n >= 2^30 switches the sort to 64-bit look-back status words and
    offsets: SortKeys of 2^30 + 12345 u32 keys against torch.sort (exact),
    plus SortPairs stability on the same size (values = index)."""
    n = (1 << 30) + 12345
    keys = torch.empty(n, dtype=torch.uint32, device="cuda")
    lcpp.testgen_fill(keys, lcpp.GEN_U32_AND3, seed=5)  # low entropy: many ties
    out = torch.empty_like(keys)
    rs = lcpp.DeviceRadixSort()
    temp = lcpp.alloc_temp(lcpp.DeviceRadixSort.GetSortPairsTempStorageBytes(lcpp.U32, lcpp.U32, n))
    rs.SortKeys(temp, keys, out, n)
    assert lcpp.device_status(temp) == lcpp.OK
    k64 = keys.view(torch.int32).to(torch.int64) & 0xFFFFFFFF
    o64 = out.view(torch.int32).to(torch.int64) & 0xFFFFFFFF
    assert torch.equal(o64, torch.sort(k64).values)
    del o64
    vals = torch.arange(n, dtype=torch.int32, device="cuda")
    vout = torch.empty_like(vals)
    rs.SortPairs(temp, keys, out, vals, vout, n)
    assert lcpp.device_status(temp) == lcpp.OK
    o64 = out.view(torch.int32).to(torch.int64) & 0xFFFFFFFF
    assert torch.equal(o64, torch.sort(k64).values)
    # stable: the keys gathered by the value permutation are the output, and
    # equal keys keep ascending indices
    assert torch.equal(k64[vout.to(torch.int64)], o64)
    same = o64[1:] == o64[:-1]
    assert bool((vout[1:][same] > vout[:-1][same]).all())
