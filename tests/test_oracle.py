"""Pin the CPU oracle against the golden fixtures (reference tests' own host
oracles on the reference tests' own inputs) and against independent numpy
restatements.  CPU only."""
from __future__ import annotations

import numpy as np
import pytest


# ------------------------------------------------------------------ sorting
@pytest.mark.parametrize("n", [1 << k for k in range(5, 15)])
def test_float_keys_golden(oracle, golden, n):
    """tests/device_radix_sort_one_sweep.cpp:79-136 (std::sort, std::greater)."""
    asc_in = golden[f"float_keys_asc_in_{n}"]
    desc_in = golden[f"float_keys_desc_in_{n}"]
    assert golden.matches(f"float_keys_asc_out_{n}", oracle.radix_sort(asc_in))
    assert golden.matches(f"float_keys_desc_out_{n}", oracle.radix_sort(desc_in, descending=True))


def test_u64_keys_golden(oracle, golden):
    """tests/device_radix_sort_one_sweep.cpp:175-205."""
    assert golden.matches("u64_keys_out", oracle.radix_sort(golden["u64_keys_in"]))


@pytest.mark.parametrize("desc", [False, True])
def test_pairs_golden(oracle, golden, desc):
    """tests/device_radix_sort_one_sweep.cpp:207-333 (uint keys, float values)."""
    tag = "desc" if desc else "asc"
    k, v = oracle.radix_sort(golden[f"pairs_{tag}_keys_in"], golden[f"pairs_{tag}_vals_in"],
                             descending=desc)
    assert golden.matches(f"pairs_{tag}_keys_out", k)
    assert golden.matches(f"pairs_{tag}_vals_out", v)


@pytest.mark.parametrize("case,begin,end", [("partial_bits", 1, 6), ("double_buffer", 0, 5)])
@pytest.mark.parametrize("desc", [False, True])
def test_partial_bits_golden(oracle, golden, case, begin, end, desc):
    """tests/device_radix_sort_interface_test.cpp:68-158 and :205-283
    (std::stable_sort with a selected-bits comparator)."""
    keys, vals = golden[f"{case}_keys"], golden[f"{case}_vals"]
    order = golden[f"{case}_{'desc' if desc else 'asc'}_order"]
    k = oracle.radix_sort(keys, begin_bit=begin, end_bit=end, descending=desc)
    np.testing.assert_array_equal(k, keys[order])
    k, v = oracle.radix_sort(keys, vals, begin_bit=begin, end_bit=end, descending=desc)
    np.testing.assert_array_equal(k, keys[order])
    np.testing.assert_array_equal(v, vals[order])


def test_zero_width_copy(oracle):
    """tests/device_radix_sort_interface_test.cpp:161-195."""
    keys = (np.arange(17, dtype=np.int64) * 7 - 31).astype(np.int32)
    vals = (17 - np.arange(17)).astype(np.uint32)
    k, v = oracle.radix_sort(keys, vals, begin_bit=9, end_bit=9)
    np.testing.assert_array_equal(k, keys)
    np.testing.assert_array_equal(v, vals)


def test_reversed_u32(oracle):
    """tests/device_radix_sort_one_sweep.cpp:138-173: keys n-i-1 sort to 0..n-1."""
    for k in range(0, 17):
        n = 1 << k
        keys = (n - 1 - np.arange(n)).astype(np.uint32)
        np.testing.assert_array_equal(oracle.radix_sort(keys), np.arange(n, dtype=np.uint32))


def _np_sort_key(keys: np.ndarray, desc: bool, begin: int, end: int):
    """Independent numpy restatement of the comparison key (order-preserving
    bits with +-0 merged), used with a stable argsort."""
    bits = keys.dtype.itemsize * 8
    u = keys.view(np.uint32 if bits == 32 else np.uint64).astype(np.uint64)
    high = np.uint64(1 << (bits - 1))
    mask = np.uint64((1 << bits) - 1)
    if keys.dtype.kind == "i":
        t = u ^ high
    elif keys.dtype.kind == "f":
        neg = (u & high) != 0
        t = np.where(neg, (~u) & mask, u ^ high)
    else:
        t = u
    if desc:
        t = (~t) & mask
    if keys.dtype.kind == "f":
        # the fold runs after the descending inversion and sends both zeros to HIGH
        t = np.where((u & ~high & mask) == 0, high, t)
    sel = (t >> np.uint64(begin)) & np.uint64((1 << (end - begin)) - 1)
    return sel


@pytest.mark.parametrize("dtype", [np.uint32, np.int32, np.float32, np.uint64, np.int64, np.float64])
@pytest.mark.parametrize("desc", [False, True])
@pytest.mark.parametrize("bits", ["full", "partial"])
def test_random_vs_numpy_stable(oracle, dtype, desc, bits):
    rng = np.random.default_rng(7)
    n = 5003
    w = np.dtype(dtype).itemsize * 8
    raw = rng.integers(0, 2**63, size=n, dtype=np.uint64)
    if w == 32:
        raw = (raw & np.uint64(0xFFFFFFFF)).astype(np.uint32)
    keys = raw.view(dtype).copy()
    if np.dtype(dtype).kind == "f":
        keys[np.isnan(keys)] = 0
        keys[::97] = 0.0
        keys[5::89] = -0.0
        keys[7::50] = keys[3]  # duplicates
    begin, end = (0, w) if bits == "full" else (3, w - 5)
    vals = np.arange(n, dtype=np.uint32)
    k, v = oracle.radix_sort(keys, vals, begin_bit=begin, end_bit=end, descending=desc)
    order = np.argsort(_np_sort_key(keys, desc, begin, end), kind="stable")
    np.testing.assert_array_equal(k.view(np.uint8), keys[order].view(np.uint8))
    np.testing.assert_array_equal(v, vals[order])


def test_threads_identical(oracle):
    keys = oracle.generate(oracle.GEN_U32_AND3, 200_003, seed=3)
    vals = np.arange(keys.size, dtype=np.uint32)
    k1, v1 = oracle.radix_sort(keys, vals, threads=1)
    k8, v8 = oracle.radix_sort(keys, vals, threads=8)
    np.testing.assert_array_equal(k1, k8)
    np.testing.assert_array_equal(v1, v8)


def test_float_zero_digits(oracle):
    """+0.0 and -0.0 give identical digits in both directions
    (radix_rank_sort_operations.h:31-43)."""
    pz, nz = 0x00000000, 0x80000000
    for desc in (False, True):
        for shift in (0, 8, 16, 24):
            assert oracle.digit(pz, np.float32, desc, shift, 8) == oracle.digit(nz, np.float32, desc, shift, 8)
    # ascending: both map to the transformed +0.0 = 0x80000000
    assert oracle.digit(nz, np.float32, False, 24, 8) == 0x80


# -------------------------------------------------------------------- scan
@pytest.mark.parametrize("n", [384 * 22 * 3 + 17, 320 * 25 * 3 + 17])
def test_scan_mod7_golden(oracle, golden, n):
    """tests/device_scan_test.cpp:189-265."""
    x = golden[f"scan_mod7_in_{n}"]
    assert golden.matches(f"scan_mod7_inclusive_{n}", oracle.scan(x, "inclusive"))


@pytest.mark.parametrize("n", [0, 1, 31, 32, 33, 255, 256, 257, 3839, 3840, 3841, 4095, 4096, 4097,
                               7999, 8000, 8001, 16003, 262147])
def test_scan_tiles_golden(oracle, golden, n):
    """tests/scan_optimization_regression_test.cpp:124-190 (value(i) = i%7+1)."""
    x = (np.arange(n) % 7 + 1).astype(np.int32)
    assert golden.matches(f"scan_tiles_exclusive_{n}", oracle.scan(x, "exclusive", init=0))
    assert golden.matches(f"scan_tiles_inclusive_{n}", oracle.scan(x, "inclusive"))
    if n == 16003:
        assert golden.matches("scan_tiles_exclusive_init3_16003", oracle.scan(x, "exclusive", init=3))
        assert golden.matches("scan_tiles_inclusive_init3_16003", oracle.scan(x, "inclusive_init", init=3))


def test_scan_init_golden(oracle, golden):
    """tests/device_scan_test.cpp:288-322: InclusiveScanInit {1,2,3,4}, 10 -> {11,13,16,20}."""
    out = oracle.scan(golden["scan_init_in"], "inclusive_init", init=10)
    np.testing.assert_array_equal(out, golden["scan_init_out"])


def test_scan_wraps(oracle):
    x = np.full(10, 2**31 - 1, dtype=np.int32)
    out = oracle.scan(x, "inclusive")
    ref = np.cumsum(x.astype(np.int64)).astype(np.uint64).astype(np.uint32).view(np.int32)
    np.testing.assert_array_equal(out, ref)


def test_scan_minmax(oracle):
    rng = np.random.default_rng(1)
    x = rng.integers(-1000, 1000, 777).astype(np.int32)
    np.testing.assert_array_equal(oracle.scan(x, "inclusive", oracle.OP_MAX), np.maximum.accumulate(x))
    np.testing.assert_array_equal(oracle.scan(x, "inclusive", oracle.OP_MIN), np.minimum.accumulate(x))


# ------------------------------------------------------------------ reduce
def test_reduce_shuffled_golden(oracle, golden):
    """tests/device_reduce_test.cpp:160-217."""
    x = golden["reduce_shuffled_in"]
    mn, mx = golden["reduce_shuffled_minmax"]
    assert oracle.reduce(x, oracle.OP_MIN, np.iinfo(np.int32).max) == mn
    assert oracle.reduce(x, oracle.OP_MAX, np.iinfo(np.int32).min) == mx


def test_arg_extremum_golden(oracle, golden):
    """device_reduce_test.cpp:238-288: first of equal maxima; negative floats."""
    v, i = oracle.arg_extremum(golden["arg_ties_in"], False)
    assert (v, i) == tuple(golden["arg_ties_max"])
    v, i = oracle.arg_extremum(golden["arg_negative_in"], False)
    assert v == golden["arg_negative_max"][0] and i == int(golden["arg_negative_max"][1])


def test_arg_extremum_comparator_golden(oracle, golden):
    """device_reduce_test.cpp:290-330: last-digit comparator, first ties."""
    x = golden["arg_digit_in"]
    mn, mni, mx, mxi = golden["arg_digit_minmax"]
    def less(a, b):
        return a % 10 < b % 10
    assert oracle.arg_extremum_compare(x, True, less) == (mn, mni)
    assert oracle.arg_extremum_compare(x, False, less) == (mx, mxi)


@pytest.mark.parametrize("dtype", [np.int32, np.uint32, np.float32, np.int64, np.uint64, np.float64])
def test_arg_extremum_vs_numpy(oracle, dtype):
    """First index of the extreme (numpy argmin / argmax keep the first), the
    empty-input sentinels (device_reduce.h:318-323), NaN never wins."""
    rng = np.random.default_rng(5)
    x = rng.integers(0, 50, size=10_007).astype(dtype)
    assert oracle.arg_extremum(x, True) == (x.min(), int(np.argmin(x)))
    assert oracle.arg_extremum(x, False) == (x.max(), int(np.argmax(x)))
    info = np.finfo(dtype) if np.dtype(dtype).kind == "f" else np.iinfo(dtype)
    assert oracle.arg_extremum(np.zeros(0, dtype), True) == (info.max, 1)
    assert oracle.arg_extremum(np.zeros(0, dtype), False) == (info.min, 1)
    if np.dtype(dtype).kind == "f":
        x[::3] = np.nan
        assert oracle.arg_extremum(x, True)[1] == int(np.nanargmin(x))
        assert oracle.arg_extremum(x, False)[1] == int(np.nanargmax(x))
    # the comparator walk with "<" is the same fold for NaN-free input
    y = rng.integers(0, 9, size=2000).astype(dtype)
    assert oracle.arg_extremum_compare(y, True, lambda a, b: a < b) == oracle.arg_extremum(y, True)
    assert oracle.arg_extremum_compare(y, False, lambda a, b: a < b) == oracle.arg_extremum(y, False)


def test_arg_extremum_compare_nan_is_sequential(oracle):
    """The comparator ArgMin of the reference is a sequential fold from item 0
    (device_reduce.h:571-600): with `<`, a NaN item never replaces the best
    and, once best, is never replaced.  These are the answers for input with
    NaN; the device comparator path is held to them only for strict weak
    orders (NaN input with `<` is outside that domain)."""
    less = lambda a, b: a < b  # noqa: E731
    x = np.array([5.0, np.nan, 3.0], np.float32)
    best, idx = oracle.arg_extremum_compare(x, True, less)
    assert (float(best), idx) == (3.0, 2)
    best, idx = oracle.arg_extremum_compare(x, False, less)
    assert (float(best), idx) == (5.0, 0)
    y = np.array([np.nan, 1.0, -2.0], np.float32)
    best, idx = oracle.arg_extremum_compare(y, True, less)
    assert np.isnan(best) and idx == 0


def test_scan_by_key_golden(oracle, golden):
    """device_scan_test.cpp:324-446: ExclusiveSumByKey over ones, keys i/100;
    InclusiveSumByKey of int64 ones across three tiles; parity key equality."""
    keys = golden["sbk_segment_keys"]
    ones = np.ones(keys.size, np.int32)
    np.testing.assert_array_equal(oracle.scan_by_key(keys, ones, "exclusive", oracle.OP_SUM, 0),
                                  golden["sbk_exclusive_sum_out"])
    k3 = golden["sbk_three_tiles_keys"]
    np.testing.assert_array_equal(oracle.scan_by_key(k3, np.ones(k3.size, np.int64), "inclusive"),
                                  golden["sbk_three_tiles_inclusive_out"])
    pk = golden["sbk_parity_keys"].tolist()
    assert oracle.scan_by_key_equal(pk, [1] * len(pk), "inclusive",
                                    lambda a, b: (a & 1) == (b & 1)) == golden["sbk_parity_inclusive_out"].tolist()


def test_reduce_by_key_golden(oracle, golden):
    """device_reduce_test.cpp:422-513: Sum by key i/100 of the shuffled 0..4095; empty input."""
    keys, vals = golden["sbk_segment_keys"], golden["reduce_shuffled_in"]
    uniq, agg = oracle.reduce_by_key(keys, vals, oracle.OP_SUM)
    np.testing.assert_array_equal(uniq, golden["rbk_unique_out"])
    np.testing.assert_array_equal(agg, golden["rbk_aggregates_out"])
    u, a = oracle.reduce_by_key(np.zeros(0, np.int32), np.zeros(0, np.int32))
    assert u.size == 0 and a.size == 0


@pytest.mark.parametrize("kdt,vdt", [(np.int32, np.int64), (np.float32, np.float64), (np.uint64, np.int32)])
def test_by_key_vs_numpy(oracle, kdt, vdt):
    """The C restatement against a numpy one (split at key changes)."""
    rng = np.random.default_rng(3)
    keys = rng.integers(0, 4, size=5000).astype(kdt)
    vals = rng.integers(-100, 100, size=5000).astype(vdt)
    cuts = np.flatnonzero(keys[1:] != keys[:-1]) + 1
    segs = np.split(vals, cuts)
    np.testing.assert_array_equal(oracle.scan_by_key(keys, vals, "inclusive"),
                                  np.concatenate([np.cumsum(x, dtype=vdt) for x in segs]))
    np.testing.assert_array_equal(oracle.scan_by_key(keys, vals, "inclusive", oracle.OP_MAX),
                                  np.concatenate([np.maximum.accumulate(x) for x in segs]))
    ex = oracle.scan_by_key(keys, vals, "exclusive", oracle.OP_SUM, 7)
    np.testing.assert_array_equal(ex, np.concatenate([7 + np.concatenate([[0], np.cumsum(x)[:-1]]).astype(vdt)
                                                      for x in segs]))
    ii = oracle.scan_by_key(keys, vals, "inclusive_init", oracle.OP_MIN, 5)
    np.testing.assert_array_equal(ii, np.concatenate([np.minimum(5, np.minimum.accumulate(x)) for x in segs]))
    uniq, agg = oracle.reduce_by_key(keys, vals, oracle.OP_SUM)
    np.testing.assert_array_equal(uniq, keys[np.concatenate([[0], cuts])])
    np.testing.assert_array_equal(agg, np.array([x.sum() for x in segs], dtype=vdt))


def test_select_golden(oracle, golden):
    """device_select_test.cpp:114-500: Flagged, If, FlaggedIf, Unique, UniqueByKey, in-place cases."""
    g = golden
    np.testing.assert_array_equal(oracle.select(g["sel_stable_in"], g["sel_stable_flags"] != 0),
                                  g["sel_stable_flagged_out"])
    x = g["sel_stable_in"]
    np.testing.assert_array_equal(oracle.select(x, oracle.clause_mask(x, [(6, 0, 2, 0)])), g["sel_stable_if_even_out"])
    k, v = g["sel_unique_keys"], g["sel_unique_values"]
    m = oracle.unique_mask(k)
    np.testing.assert_array_equal(k[m], g["sel_unique_keys_out"])
    np.testing.assert_array_equal(v[m], g["sel_unique_values_out"])
    f = g["sel_flaggedif_flags"]
    pos_odd = oracle.clause_mask(f, [(2, 0, 0, 0), (6, 1, 2, 0)])  # flag > 0 and not (flag % 2 == 0)
    np.testing.assert_array_equal(oracle.select(g["sel_flaggedif_in"], pos_odd), g["sel_flaggedif_out"])
    a = g["sel_inplace_aliased"]
    np.testing.assert_array_equal(oracle.select(a, a != 0), g["sel_inplace_aliased_out"])
    p = g["sel_inplace_pred"]
    np.testing.assert_array_equal(oracle.select(p, oracle.clause_mask(p, [(2, 0, 0, 0)])), g["sel_inplace_pred_out"])
    u = g["sel_inplace_unique"]
    np.testing.assert_array_equal(u[oracle.unique_mask(u)], g["sel_inplace_unique_out"])
    w = g["sel_wide_in"]
    np.testing.assert_array_equal(oracle.select(w, g["sel_wide_flags"] != 0), g["sel_wide_flagged_out"])
    np.testing.assert_array_equal(oracle.select(w, oracle.clause_mask(w, [(6, 0, 2, 0)])), g["sel_wide_if_even_out"])
    np.testing.assert_array_equal(w[oracle.unique_mask(w)], g["sel_wide_unique_out"])


def test_partition_golden(oracle, golden):
    """device_partition_test.cpp:122-353: reversed rejects; three-way category order."""
    x = golden["part_in"]
    np.testing.assert_array_equal(oracle.partition(x, golden["part_flags"] != 0), golden["part_flagged_out"])
    np.testing.assert_array_equal(oracle.partition(x, oracle.clause_mask(x, [(0, 0, 7, 0)])),
                                  golden["part_if_lt7_out"])
    f, s2, r = oracle.partition_three_way(x, oracle.clause_mask(x, [(6, 0, 3, 0)]),
                                          oracle.clause_mask(x, [(0, 0, 8, 0)]))
    np.testing.assert_array_equal(f, golden["part3_first_out"])
    np.testing.assert_array_equal(s2, golden["part3_second_out"])
    np.testing.assert_array_equal(r, golden["part3_unselected_out"])


def test_clause_mask_c_remainder(oracle):
    """MOD_EQ follows C: -3 % 2 == -1, so -3 is neither even nor "% 2 == 1"."""
    x = np.array([-4, -3, -1, 0, 1, 2, 3], np.int32)
    np.testing.assert_array_equal(oracle.clause_mask(x, [(6, 0, 2, 0)]), [1, 0, 0, 1, 0, 1, 0])
    np.testing.assert_array_equal(oracle.clause_mask(x, [(6, 0, 2, 1)]), [0, 0, 0, 0, 1, 0, 1])


def test_reduce_identities(oracle):
    """device_reduce_test.cpp:95-118 (ones, 2^k+1) and :220-236 (float max identity)."""
    for k in range(0, 16):
        n = (1 << k) + 1
        assert oracle.reduce(np.ones(n, np.uint32), oracle.OP_SUM, 0) == n
    x = np.array([-8.0, -2.5, -9.0, -4.0], np.float32)
    assert oracle.reduce(x, oracle.OP_MAX, np.finfo(np.float32).min) == np.float32(-2.5)
    assert oracle.reduce(np.zeros(0, np.float32), oracle.OP_SUM, 0) == 0


def test_sum_f64(oracle):
    x = oracle.generate(oracle.GEN_F32_UNIT, 100_000, seed=5)
    assert abs(oracle.sum_f64(x) - float(np.sum(x.astype(np.float64)))) < 1e-6


# -------------------------------------------------------------- generators
def test_generators_match_numpy(oracle):
    """Counter-based generator restated in numpy (splitmix64)."""
    def splitmix(x):
        with np.errstate(over="ignore"):
            z = x + np.uint64(0x9E3779B97F4A7C15)
            z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
            z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
            return z ^ (z >> np.uint64(31))
    i = np.arange(1000, 2000, dtype=np.uint64)
    seed = np.uint64(1)
    r = [splitmix((seed << np.uint64(40)) + (np.uint64(s) << np.uint64(36)) + i) for s in range(3)]
    np.testing.assert_array_equal(oracle.generate(oracle.GEN_U32_UNIFORM, 1000, 1, 1000),
                                  (r[0] & np.uint64(0xFFFFFFFF)).astype(np.uint32))
    np.testing.assert_array_equal(oracle.generate(oracle.GEN_U32_AND3, 1000, 1, 1000),
                                  ((r[0] & r[1] & r[2]) & np.uint64(0xFFFFFFFF)).astype(np.uint32))
    np.testing.assert_array_equal(oracle.generate(oracle.GEN_I32_SCAN, 1000, 1, 1000),
                                  ((r[0] % np.uint64(2001)).astype(np.int64) - 1000).astype(np.int32))


def test_segmented_oracle_matches_golden(golden):
    from oracle import oracle as O
    keys, vals = golden["segmented_keys"], golden["segmented_vals"]
    b, e = golden["segmented_begin"], golden["segmented_end"]
    for desc, name in ((False, "segmented_asc_order"), (True, "segmented_desc_order")):
        order = golden[name]
        sentinel_k = np.full_like(keys, -777)
        sentinel_v = np.full_like(vals, 0xFFFFFFFF)
        ok, ov = O.segmented_radix_sort(keys, vals, b, e, descending=desc, out_keys=sentinel_k,
                                        out_values=sentinel_v)
        inside = order != 0xFFFFFFFF
        np.testing.assert_array_equal(ok[inside], keys[order[inside]])
        np.testing.assert_array_equal(ov[inside], vals[order[inside]])
        assert (ok[~inside] == -777).all() and (ov[~inside] == 0xFFFFFFFF).all()


def _segmented_by_python(keys, b, e, begin_bit, end_bit, desc):
    """Independent pure-Python restatement for small cases."""
    bits = keys.dtype.itemsize * 8
    ubits = keys.view(np.uint32 if bits == 32 else np.uint64)

    def field(i):
        u = int(ubits[i])
        if keys.dtype.kind == "i":
            u ^= 1 << (bits - 1)
        elif keys.dtype.kind == "f":
            u = (~u & ((1 << bits) - 1)) if u >> (bits - 1) else u ^ (1 << (bits - 1))
        return (u >> begin_bit) & ((1 << (end_bit - begin_bit)) - 1)

    out = keys.copy()
    n = keys.size
    for i_s in range(len(b)):
        nb = int(b[i_s + 1]) if i_s + 1 < len(b) else None
        lo, hi = int(b[i_s]), int(e[i_s])
        if not (lo <= hi <= n):
            continue
        members = [i for i in range(lo, hi) if nb is None or i < nb]
        order = sorted(members, key=field, reverse=False)
        if desc:
            order = sorted(members, key=lambda i: -field(i))
        for p, q in zip(members, order):
            out[p] = keys[q]
    return out


@pytest.mark.parametrize("dt", [np.uint32, np.int32, np.float32, np.uint64, np.int64, np.float64])
@pytest.mark.parametrize("desc", [False, True])
def test_segmented_oracle_vs_python(dt, desc):
    from oracle import oracle as O
    rng = np.random.default_rng(3)
    n = 300
    if np.dtype(dt).kind == "f":
        keys = rng.standard_normal(n).astype(dt)
        keys[::7] = 0.0
        keys[3::7] = -0.0
    else:
        keys = rng.integers(0, 50, n).astype(dt) if np.dtype(dt).kind == "u" else rng.integers(-25, 25, n).astype(dt)
    b = np.array([0, 10, 10, 57, 120, 250], dtype=np.uint32)
    e = np.array([7, 10, 50, 120, 240, 300], dtype=np.uint32)
    bits = np.dtype(dt).itemsize * 8
    for begin_bit, end_bit in ((0, bits), (1, 6), (3, 3)):
        ok, _ = O.segmented_radix_sort(keys, None, b, e, begin_bit, end_bit, desc)
        exp = _segmented_by_python(keys, b, e, begin_bit, end_bit, desc)
        np.testing.assert_array_equal(ok.view(np.uint8), exp.view(np.uint8))


def test_decomposed_oracle_matches_golden(golden):
    from oracle import oracle as O
    p, s = golden["decomposed_primary"], golden["decomposed_secondary"]
    cases = [("decomposed_full_asc_order", 0, 64, False), ("decomposed_full_desc_order", 0, 64, True),
             ("decomposed_window_asc_order", 28, 36, False), ("decomposed_window_desc_order", 28, 36, True)]
    for name, b, e, desc in cases:
        np.testing.assert_array_equal(O.decomposed_sort_order([p, s], b, e, desc), golden[name])


def test_decomposed_oracle_vs_python():
    """Members of every dtype, 3 members (160 bits, three chunks), windows
    across member boundaries, against a pure-Python sorted() on the bits."""
    from oracle import oracle as O
    rng = np.random.default_rng(4)
    n = 400
    a = rng.integers(-3, 3, n).astype(np.int64)
    b = rng.standard_normal(n).astype(np.float32)
    b[::9] = 0.0
    b[4::9] = -0.0
    c = rng.integers(0, 4, n).astype(np.uint64)
    cols = [a, b, c]

    def ob(x, kind, bits):
        x = int(x)
        if kind == "i":
            return (x & ((1 << bits) - 1)) ^ (1 << (bits - 1))
        if kind == "f":
            u = x
            t = (~u & ((1 << bits) - 1)) if u >> (bits - 1) else u ^ (1 << (bits - 1))
            return (1 << (bits - 1)) if t == (1 << (bits - 1)) - 1 else t
        return x

    ubits = [a.view(np.uint64), b.view(np.uint32), c]
    kinds = ["i", "f", "u"]
    widths = [64, 32, 64]

    def concat(i):
        v = 0
        for col, kind, w in zip(ubits, kinds, widths):
            v = (v << w) | ob(col[i], kind, w)
        return v

    full = [concat(i) for i in range(n)]
    for lo, hi in ((0, 160), (30, 100), (60, 70), (5, 5)):
        for desc in (False, True):
            key = [(v >> lo) & ((1 << (hi - lo)) - 1) for v in full]
            exp = sorted(range(n), key=(lambda i: -key[i]) if desc else (lambda i: key[i]))
            np.testing.assert_array_equal(O.decomposed_sort_order(cols, lo, hi, desc), exp)
