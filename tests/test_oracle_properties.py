"""Property checks that tie the oracle's restatements to one another (CPU):
the last inclusive by-key value of each segment is that segment's ReduceByKey
aggregate; exclusive (+) own value = inclusive within a segment; partitions
are permutations with the selected items first; the three-way partition's
parts cover the input; selections and unique masks agree with the counting
scans' final counts."""
from __future__ import annotations

import numpy as np
import pytest

hypothesis = pytest.importorskip("hypothesis")
from hypothesis import given, settings  # noqa: E402
from hypothesis import strategies as st  # noqa: E402
from hypothesis.extra import numpy as hnp  # noqa: E402

SMALL = st.integers(min_value=0, max_value=300)


@settings(max_examples=60, deadline=None)
@given(n=SMALL, seed=st.integers(0, 2**31 - 1), nkeys=st.integers(1, 6))
def test_scan_by_key_matches_reduce_by_key(oracle, n, seed, nkeys):
    rng = np.random.default_rng(seed)
    keys = rng.integers(0, nkeys, size=n).astype(np.int32)
    vals = rng.integers(-1000, 1000, size=n).astype(np.int64)
    inc = oracle.scan_by_key(keys, vals, "inclusive")
    exc = oracle.scan_by_key(keys, vals, "exclusive", oracle.OP_SUM, 0)
    np.testing.assert_array_equal(exc + vals, inc)
    uniq, agg = oracle.reduce_by_key(keys, vals)
    if n == 0:
        assert uniq.size == 0
        return
    last = np.flatnonzero(np.append(keys[1:] != keys[:-1], True))
    np.testing.assert_array_equal(agg, inc[last])
    np.testing.assert_array_equal(uniq, keys[last])
    mx = oracle.scan_by_key(keys, vals, "inclusive", oracle.OP_MAX)
    _, amax = oracle.reduce_by_key(keys, vals, oracle.OP_MAX)
    np.testing.assert_array_equal(amax, mx[last])


@settings(max_examples=60, deadline=None)
@given(x=hnp.arrays(np.int32, st.integers(0, 300), elements=st.integers(-50, 50)),
       m=st.integers(1, 7), r=st.integers(-3, 3))
def test_partitions_are_permutations(oracle, x, m, r):
    mask = oracle.clause_mask(x, [(6, 0, m, r)])
    p = oracle.partition(x, mask)
    k = int(mask.sum())
    assert sorted(p.tolist()) == sorted(x.tolist())
    np.testing.assert_array_equal(p[:k], oracle.select(x, mask))
    np.testing.assert_array_equal(p[k:][::-1], x[~mask])
    second = oracle.clause_mask(x, [(0, 0, 0, 0)])
    f, s2, rest = oracle.partition_three_way(x, mask, second)
    assert f.size + s2.size + rest.size == x.size
    assert sorted(np.concatenate([f, s2, rest]).tolist()) == sorted(x.tolist())


@settings(max_examples=60, deadline=None)
@given(x=hnp.arrays(np.int64, st.integers(1, 300), elements=st.integers(-3, 3)))
def test_unique_mask_counts(oracle, x):
    h = oracle.unique_mask(x)
    # the number of runs equals ReduceByKey's run count over the same keys
    uniq, _ = oracle.reduce_by_key(x, np.zeros(x.size, np.int32))
    assert int(h.sum()) == uniq.size
    np.testing.assert_array_equal(x[h], uniq)


@settings(max_examples=40, deadline=None)
@given(x=hnp.arrays(np.float32, st.integers(1, 200),
                    elements=st.one_of(st.floats(-4, 4, width=32), st.just(float("nan")))))
def test_arg_extremum_is_first_extreme(oracle, x):
    finite = x[~np.isnan(x)]
    for is_min in (True, False):
        v, i = oracle.arg_extremum(x, is_min)
        if finite.size == 0:
            assert i == 0xFFFFFFFF
            continue
        want = finite.min() if is_min else finite.max()
        assert v == want
        assert i == int(np.flatnonzero(x == want)[0])
