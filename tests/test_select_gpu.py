"""GPU parity tests for DeviceSelect (Flagged / If / FlaggedIf / Unique /
UniqueByKey) and DevicePartition (Flagged / If / three-way If) through the C
ABI, mirroring the reference's tests/device_select_test.cpp and
tests/device_partition_test.cpp and checking against the numpy restatement
(oracle.select / partition / partition_three_way / unique_mask)."""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
from gpu_helpers import dev, empty_like_np, host  # noqa: E402

SIZES = [1, 2, 4095, 4096, 4097, 5759, 5760, 5761, 230_413, 1_000_003]
EVEN = [(6, 0, 2, 0)]  # x % 2 == 0


def _pred(lcpp, clauses):
    return lcpp.Pred(list(clauses))


def _count(t):
    return int(t.cpu().numpy().view(np.uint32)[0])


def _run_select(lcpp, kind, x, flags=None, clauses=(), inplace=False, d_in=None, out_offset=0):
    n = x.size
    sel = lcpp.DeviceSelect()
    temp = lcpp.alloc_temp(sel.GetTempStorageBytes(n)) if n else None
    din = dev(x) if d_in is None else d_in
    if inplace:
        dout_full, dout = din, din
    else:
        dout_full = torch.empty(n + out_offset + 1, dtype=din.dtype, device="cuda")
        dout = dout_full[out_offset:out_offset + n]
    cnt = torch.full((2,), 99, dtype=torch.int32, device="cuda")
    c = cnt[1:]
    if kind == "flagged":
        df = flags if isinstance(flags, torch.Tensor) else dev(flags)
        sel.Flagged(temp, din, df, dout, c, n)
    elif kind == "flagged_if":
        sel.FlaggedIf(temp, din, dev(flags), dout, c, n, _pred(lcpp, clauses))
    elif kind == "if":
        sel.If(temp, din, dout, c, n, _pred(lcpp, clauses))
    else:
        sel.Unique(temp, din, dout, c, n)
    if temp is not None:
        assert lcpp.device_status(temp) == lcpp.OK
    k = _count(c)
    return host(dout)[:k], k


def _flags(pattern: int, n: int):
    i = np.arange(n)
    return [np.zeros(n, np.uint32), np.ones(n, np.uint32), (i % 3).astype(np.uint32),
            ((i < 11) | (i > 200_000)).astype(np.uint32)][pattern]


# ------------------------------------------------------------ reference tests
def test_flagged_and_if_are_stable(lcpp, golden):
    """device_select_test.cpp:254-320."""
    x, f = golden["sel_stable_in"], golden["sel_stable_flags"]
    got, k = _run_select(lcpp, "flagged", x, f)
    np.testing.assert_array_equal(got, golden["sel_stable_flagged_out"])
    got, k = _run_select(lcpp, "if", x, clauses=EVEN)
    np.testing.assert_array_equal(got, golden["sel_stable_if_even_out"])


def test_unique_and_unique_by_key(lcpp, golden):
    """device_select_test.cpp:322-372: first item of each run, values ride along."""
    k, v = golden["sel_unique_keys"], golden["sel_unique_values"]
    got, _ = _run_select(lcpp, "unique", k)
    np.testing.assert_array_equal(got, golden["sel_unique_keys_out"])
    sel = lcpp.DeviceSelect()
    temp = lcpp.alloc_temp(sel.GetTempStorageBytes(k.size))
    ko, vo = empty_like_np(k), empty_like_np(v)
    cnt = torch.zeros(1, dtype=torch.int32, device="cuda")
    sel.UniqueByKey(temp, dev(k), dev(v), ko, vo, cnt, k.size)
    m = _count(cnt)
    np.testing.assert_array_equal(host(ko)[:m], golden["sel_unique_keys_out"])
    np.testing.assert_array_equal(host(vo)[:m], golden["sel_unique_values_out"])


def test_flagged_if_copy_and_in_place(lcpp, golden):
    """device_select_test.cpp:374-430: flag > 0 and odd; flags and input unchanged by the copy form."""
    x, f = golden["sel_flaggedif_in"], golden["sel_flaggedif_flags"]
    pos_odd = [(2, 0, 0, 0), (6, 1, 2, 0)]
    got, _ = _run_select(lcpp, "flagged_if", x, f, pos_odd)
    np.testing.assert_array_equal(got, golden["sel_flaggedif_out"])
    d = dev(x)
    sel = lcpp.DeviceSelect()
    temp = lcpp.alloc_temp(sel.GetTempStorageBytes(x.size))
    cnt = torch.zeros(1, dtype=torch.int32, device="cuda")
    sel.FlaggedIf(temp, d, dev(f), d, cnt, x.size, lcpp.Pred(pos_odd))
    np.testing.assert_array_equal(host(d)[:_count(cnt)], golden["sel_flaggedif_out"])


def test_in_place_forms(lcpp, golden):
    """device_select_test.cpp:432-500: data as its own flags, If(> 0), Unique; empty If writes 0."""
    a = dev(golden["sel_inplace_aliased"])
    sel = lcpp.DeviceSelect()
    temp = lcpp.alloc_temp(sel.GetTempStorageBytes(8))
    cnt = torch.zeros(1, dtype=torch.int32, device="cuda")
    sel.Flagged(temp, a, a, a, cnt, 8)
    np.testing.assert_array_equal(host(a)[:_count(cnt)], golden["sel_inplace_aliased_out"])
    got, _ = _run_select(lcpp, "if", golden["sel_inplace_pred"], clauses=[(2, 0, 0, 0)], inplace=True)
    np.testing.assert_array_equal(got, golden["sel_inplace_pred_out"])
    got, _ = _run_select(lcpp, "unique", golden["sel_inplace_unique"], inplace=True)
    np.testing.assert_array_equal(got, golden["sel_inplace_unique_out"])
    zero = torch.ones(1, dtype=torch.int32, device="cuda")
    sel.If(None, torch.empty(0, dtype=torch.int32, device="cuda"), torch.empty(0, dtype=torch.int32, device="cuda"),
           zero, 0, lcpp.Pred.gt(0))
    assert _count(zero) == 0


def test_wide_values_and_bool_flags(lcpp, golden):
    """device_select_test.cpp:114-172: uint64 values, bool flags, If(even), Unique."""
    w = golden["sel_wide_in"]
    got, _ = _run_select(lcpp, "flagged", w, torch.from_numpy(golden["sel_wide_flags"].astype(bool)).cuda())
    np.testing.assert_array_equal(got, golden["sel_wide_flagged_out"])
    got, _ = _run_select(lcpp, "if", w, clauses=EVEN)
    np.testing.assert_array_equal(got, golden["sel_wide_if_even_out"])
    got, _ = _run_select(lcpp, "unique", w)
    np.testing.assert_array_equal(got, golden["sel_wide_unique_out"])


@pytest.mark.parametrize("n", [1, 5759, 5760, 5761, 230_413])
def test_multitile_tails_and_empty_tiles(lcpp, oracle, n):
    """device_select_test.cpp:174-252: input and output at odd offsets (3 and 2
    items in), four flag patterns; Unique over runs of 1, 17, 18001 and n."""
    base = np.zeros(n + 3, np.int32)
    base[3:] = np.arange(n, dtype=np.int32)
    dbase = dev(base)
    for pattern in range(4):
        f = _flags(pattern, n)
        got, k = _run_select(lcpp, "flagged", base[3:], f, d_in=dbase[3:], out_offset=2)
        np.testing.assert_array_equal(got, oracle.select(base[3:], f != 0))
    for run in (1, 17, 18001, n):
        x = (np.arange(n) // run).astype(np.int32)
        base[3:] = x
        got, _ = _run_select(lcpp, "unique", x, d_in=dev(base)[3:], out_offset=2)
        np.testing.assert_array_equal(got, x[oracle.unique_mask(x)])


def test_partition_ordering(lcpp, golden):
    """device_partition_test.cpp:122-204: selected in order, rejected reversed."""
    x, f = golden["part_in"], golden["part_flags"]
    part = lcpp.DevicePartition()
    temp = lcpp.alloc_temp(part.GetTempStorageBytes(x.size))
    out = empty_like_np(x)
    cnt = torch.zeros(1, dtype=torch.int32, device="cuda")
    part.Flagged(temp, dev(x), dev(f), out, cnt, x.size)
    assert _count(cnt) == 4
    np.testing.assert_array_equal(host(out), golden["part_flagged_out"])
    part.If(temp, dev(x), out, cnt, x.size, lcpp.Pred.lt(7))
    assert _count(cnt) == 7
    np.testing.assert_array_equal(host(out), golden["part_if_lt7_out"])


def test_partition_multitile_reverse_rejects(lcpp, oracle):
    """device_partition_test.cpp:242-291: 230413 items, four flag patterns."""
    n = 230_413
    x = np.arange(n, dtype=np.int32)
    part = lcpp.DevicePartition()
    temp = lcpp.alloc_temp(part.GetTempStorageBytes(n))
    out = empty_like_np(x)
    cnt = torch.zeros(1, dtype=torch.int32, device="cuda")
    for pattern in range(4):
        f = _flags(pattern, n)
        part.Flagged(temp, dev(x), dev(f), out, cnt, n)
        assert _count(cnt) == int((f != 0).sum())
        np.testing.assert_array_equal(host(out), oracle.partition(x, f != 0))


def test_three_way_category_order(lcpp, golden):
    """device_partition_test.cpp:293-353 and :355-380 (zero items write both counts)."""
    x = golden["part_in"]
    part = lcpp.DevicePartition()
    temp = lcpp.alloc_temp(part.GetThreeWayTempStorageBytes(x.size))
    outs = [empty_like_np(x) for _ in range(3)]
    cnt = torch.zeros(2, dtype=torch.int32, device="cuda")
    part.IfThreeWay(temp, dev(x), *outs, cnt, x.size, lcpp.Pred.mod_eq(3, 0), lcpp.Pred.lt(8))
    c = cnt.cpu().numpy()
    assert c.tolist() == [4, 5]
    np.testing.assert_array_equal(host(outs[0])[:4], golden["part3_first_out"])
    np.testing.assert_array_equal(host(outs[1])[:5], golden["part3_second_out"])
    np.testing.assert_array_equal(host(outs[2])[:3], golden["part3_unselected_out"])
    cnt = torch.tensor([7, 9], dtype=torch.int32, device="cuda")
    e = torch.empty(0, dtype=torch.int32, device="cuda")
    part.IfThreeWay(None, e, e, e, e, cnt, 0, lcpp.Pred.lt(0), lcpp.Pred.gt(0))
    assert cnt.cpu().tolist() == [0, 0]


# ------------------------------------------------------------------ vs oracle
@pytest.mark.parametrize("dtype", [np.int32, np.uint32, np.float32, np.int64, np.uint64, np.float64])
def test_select_and_partition_vs_oracle(lcpp, oracle, dtype):
    for n in SIZES:
        rng = np.random.default_rng(n)
        x = rng.integers(-50, 50, size=n).astype(dtype)
        clauses = [(2, 0, 5, 0)] if np.dtype(dtype).kind == "f" else [(6, 0, 3, 0), (1, 1, 40, 0)]  # x%3==0 and not <= 40
        mask = oracle.clause_mask(x, clauses)
        got, _ = _run_select(lcpp, "if", x, clauses=clauses)
        np.testing.assert_array_equal(got, oracle.select(x, mask))
        for fdt in (np.uint8, np.int32, np.int64, np.float32):
            f = (rng.integers(0, 4, size=n) == 0).astype(fdt) * (-1 if fdt in (np.int32, np.int64) else 1)
            got, _ = _run_select(lcpp, "flagged", x, f)
            np.testing.assert_array_equal(got, oracle.select(x, f != 0))
        fi = rng.integers(-5, 6, size=n).astype(np.int32)
        got, _ = _run_select(lcpp, "flagged_if", x, fi, [(3, 0, 2, 0)])
        np.testing.assert_array_equal(got, oracle.select(x, fi >= 2))
        runs = np.repeat(x, rng.integers(1, 5, size=n))[:n]
        got, _ = _run_select(lcpp, "unique", runs)
        np.testing.assert_array_equal(got, runs[oracle.unique_mask(runs)])
        part = lcpp.DevicePartition()
        temp = lcpp.alloc_temp(part.GetThreeWayTempStorageBytes(n))
        out = empty_like_np(x)
        cnt = torch.zeros(2, dtype=torch.int32, device="cuda")
        part.If(temp, dev(x), out, cnt[:1], n, lcpp.Pred(clauses))
        np.testing.assert_array_equal(host(out), oracle.partition(x, mask))
        outs = [empty_like_np(x) for _ in range(3)]
        second = [(0, 0, 0, 0)]  # x < 0
        part.IfThreeWay(temp, dev(x), *outs, cnt, n, lcpp.Pred(clauses), lcpp.Pred(second))
        want = oracle.partition_three_way(x, mask, oracle.clause_mask(x, second))
        c = cnt.cpu().numpy().view(np.uint32)
        assert (int(c[0]), int(c[1])) == (want[0].size, want[1].size)
        for o, w in zip(outs, want):
            np.testing.assert_array_equal(host(o)[:w.size], w)


@pytest.mark.parametrize("dtype", [np.int32, np.uint32, np.int64, np.uint64])
def test_mod_eq_divisors_vs_oracle(lcpp, oracle, dtype):
    """x % d == r with the C remainder for power-of-two |d| (a masked form
    inside the kernel), other divisors and the most negative divisor, over
    items spanning the type's full range including its extremes."""
    info = np.iinfo(dtype)
    n = 70_001
    rng = np.random.default_rng(7)
    x = rng.integers(info.min, info.max, size=n, dtype=dtype, endpoint=True)
    x[:8] = [info.min, info.max, 0, 1, info.min + 1, info.max - 1, 2, 3]
    if info.min < 0:
        x[8::5] = rng.integers(-40, 40, size=x[8::5].size)
        cases = [(1, 0), (2, 0), (2, 1), (2, -1), (-2, -1), (8, -3), (-16, 5), (1 << 20, -(1 << 19)),
                 (int(info.max) // 2 + 1, 0), (3, -2), (-5, 4), (int(info.min), 0), (int(info.min), -1)]
    else:
        x[8::5] = rng.integers(0, 80, size=x[8::5].size)
        cases = [(1, 0), (2, 0), (2, 1), (8, 3), (1 << 20, 77), (int(info.max) // 2 + 1, 5), (3, 2), (12, 4)]
    for d, r in cases:
        clauses = [(6, 0, d, r)]
        got, _ = _run_select(lcpp, "if", x, clauses=clauses)
        np.testing.assert_array_equal(got, oracle.select(x, oracle.clause_mask(x, clauses)), err_msg=f"{d} {r}")
        clauses = [(6, 1, d, r)]
        got, _ = _run_select(lcpp, "if", x, clauses=clauses)
        np.testing.assert_array_equal(got, oracle.select(x, oracle.clause_mask(x, clauses)), err_msg=f"not {d} {r}")


def test_unique_by_key_vs_oracle(lcpp, oracle):
    rng = np.random.default_rng(4)
    for n in (4097, 1_000_003):
        k = np.repeat(rng.integers(0, 3, size=n), rng.integers(1, 9, size=n))[:n].astype(np.float64)
        k[::97] = -0.0  # -0.0 == +0.0: same run
        v = np.arange(n, dtype=np.int64)
        sel = lcpp.DeviceSelect()
        temp = lcpp.alloc_temp(sel.GetTempStorageBytes(n))
        ko, vo = empty_like_np(k), empty_like_np(v)
        cnt = torch.zeros(1, dtype=torch.int32, device="cuda")
        sel.UniqueByKey(temp, dev(k), dev(v), ko, vo, cnt, n)
        m = oracle.unique_mask(k)
        c = _count(cnt)
        assert c == int(m.sum())
        assert host(ko)[:c].tobytes() == k[m].tobytes()
        np.testing.assert_array_equal(host(vo)[:c], v[m])


def test_select_if_2p30(lcpp):
    """2^30 items, half selected: the output is the selected part of 0..n-1."""
    n = 1 << 30
    x = torch.arange(n, dtype=torch.int32, device="cuda")
    sel = lcpp.DeviceSelect()
    temp = lcpp.alloc_temp(sel.GetTempStorageBytes(n))
    out = torch.empty_like(x)
    cnt = torch.zeros(1, dtype=torch.int32, device="cuda")
    sel.If(temp, x, out, cnt, n, lcpp.Pred.bits_any(2))  # bit 1 set
    assert lcpp.device_status(temp) == lcpp.OK
    c = _count(cnt)
    assert c == n // 2
    want = torch.arange(n // 4, dtype=torch.int64, device="cuda")
    assert torch.equal(out[0:c:2].to(torch.int64), want * 4 + 2)
    assert torch.equal(out[1:c:2].to(torch.int64), want * 4 + 3)


def test_argument_errors(lcpp):
    sel, part = lcpp.DeviceSelect(), lcpp.DevicePartition()
    x = torch.zeros(1024, dtype=torch.float32, device="cuda")
    cnt = torch.zeros(2, dtype=torch.int32, device="cuda")
    temp = lcpp.alloc_temp(part.GetThreeWayTempStorageBytes(1024))
    with pytest.raises(lcpp.LcppError) as e:
        sel.If(temp, x, x.clone(), cnt, 1024, lcpp.Pred.mod_eq(2, 0))  # no remainder on floats
    assert e.value.status == lcpp.ERR_INVALID_ARG
    with pytest.raises(lcpp.LcppError) as e:
        part.If(temp, x, x, cnt, 1024, lcpp.Pred.gt(0))  # partition cannot run in place
    assert e.value.status == lcpp.ERR_INVALID_ARG
    with pytest.raises(lcpp.LcppError) as e:
        part.IfThreeWay(temp, x, x[512:].clone(), x[:10], x.clone(), cnt, 1024, lcpp.Pred.gt(0), lcpp.Pred.lt(0))
    assert e.value.status == lcpp.ERR_INVALID_ARG  # an output overlaps the input
    with pytest.raises(lcpp.LcppError) as e:
        sel.If(lcpp.alloc_temp(8), x, x.clone(), cnt, 1024, lcpp.Pred.gt(0))
    assert e.value.status == lcpp.ERR_TEMP_TOO_SMALL
    with pytest.raises(lcpp.LcppError) as e:
        sel.If(temp, x, x.clone(), cnt, 1 << 32, lcpp.Pred.gt(0))
    assert e.value.status == lcpp.ERR_INVALID_ARG


@pytest.mark.parametrize("dtype", [np.int32, np.float32, np.uint64])
def test_exclusive_sum_transform_and_adjacent(lcpp, oracle, dtype):
    """DeviceScan::ExclusiveSumTransform / ExclusiveSumAdjacent (device_scan.h:387-406):
    exclusive counts of the selected items and of the run heads."""
    sc = lcpp.DeviceScan()
    for n in (1, 4095, 4097, 230_413):
        rng = np.random.default_rng(n)
        x = np.repeat(rng.integers(0, 9, size=n), rng.integers(1, 4, size=n))[:n].astype(dtype)
        temp = lcpp.alloc_temp(sc.GetTransformTempStorageBytes(n))
        out = torch.empty(n, dtype=torch.int32, device="cuda")
        sc.ExclusiveSumTransform(temp, dev(x), out, n, lcpp.Pred.gt(4))
        m = oracle.clause_mask(x, [(2, 0, 4, 0)])
        np.testing.assert_array_equal(host(out).view(np.uint32), np.concatenate([[0], np.cumsum(m)[:-1]]))
        sc.ExclusiveSumAdjacent(temp, dev(x), out, n)
        h = oracle.unique_mask(x)
        np.testing.assert_array_equal(host(out).view(np.uint32), np.concatenate([[0], np.cumsum(h)[:-1]]))
