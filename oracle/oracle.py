"""ctypes front end of the CPU oracle (TEST INFRASTRUCTURE ONLY).

The oracle is the checker for the CUDA library and the timed CPU baseline.
Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
leg import this module; the product path never does.

Every function takes and returns numpy arrays.  The C source
(``oracle/lcpp_oracle.c``) cites the reference file:line each routine
restates.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

_HERE = Path(__file__).resolve().parent
_LIB_PATH = _HERE / "_build" / "liblcpp_oracle.so"

# lcpp_dtype codes (include/lcpp_b200.h)
U32, I32, F32, U64, I64, F64 = 0, 1, 2, 3, 4, 5
OP_SUM, OP_MIN, OP_MAX = 0, 1, 2

NP_TO_DTYPE = {
    np.dtype(np.uint32): U32,
    np.dtype(np.int32): I32,
    np.dtype(np.float32): F32,
    np.dtype(np.uint64): U64,
    np.dtype(np.int64): I64,
    np.dtype(np.float64): F64,
}

# generator codes (oracle_generate)
GEN_U32_UNIFORM, GEN_U32_AND3, GEN_U32_CONST, GEN_U64_UNIFORM = 0, 1, 2, 3
GEN_I32_SCAN, GEN_F32_UNIT, GEN_I64_UNIFORM, GEN_U32_INDEX = 4, 5, 6, 7
GEN_NP_DTYPE = {
    GEN_U32_UNIFORM: np.uint32, GEN_U32_AND3: np.uint32, GEN_U32_CONST: np.uint32,
    GEN_U64_UNIFORM: np.uint64, GEN_I32_SCAN: np.int32, GEN_F32_UNIT: np.float32,
    GEN_I64_UNIFORM: np.int64, GEN_U32_INDEX: np.uint32,
}

_lib = None


def build() -> Path:
    """Compile the oracle with its Makefile (idempotent)."""
    subprocess.run(["make", "-s", "-C", str(_HERE)], check=True)
    return _LIB_PATH


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not _LIB_PATH.exists():
            build()
        l = ctypes.CDLL(str(_LIB_PATH))
        vp, u64, i = ctypes.c_void_p, ctypes.c_uint64, ctypes.c_int
        l.oracle_radix_sort.argtypes = [vp, vp, vp, vp, u64, i, i, i, i, i, i]
        l.oracle_radix_sort.restype = i
        l.oracle_digit.argtypes = [u64, i, i, i, i]
        l.oracle_digit.restype = ctypes.c_uint32
        l.oracle_scan.argtypes = [vp, vp, u64, i, i, i, vp]
        l.oracle_scan.restype = i
        l.oracle_reduce.argtypes = [vp, vp, u64, i, i, vp]
        l.oracle_reduce.restype = i
        l.oracle_arg_extremum.argtypes = [vp, vp, vp, u64, i, i]
        l.oracle_arg_extremum.restype = i
        l.oracle_scan_by_key.argtypes = [vp, vp, vp, u64, i, i, i, i, vp]
        l.oracle_scan_by_key.restype = i
        l.oracle_reduce_by_key.argtypes = [vp, vp, vp, vp, vp, u64, i, i, i]
        l.oracle_reduce_by_key.restype = i
        l.oracle_sum_f64.argtypes = [vp, u64, i]
        l.oracle_sum_f64.restype = ctypes.c_double
        l.oracle_generate.argtypes = [vp, u64, u64, u64, i]
        l.oracle_generate.restype = i
        _lib = l
    return _lib


def _ptr(a: np.ndarray | None):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def radix_sort(keys: np.ndarray, values: np.ndarray | None = None, begin_bit: int = 0,
               end_bit: int | None = None, descending: bool = False, threads: int = 1):
    """Stable LSD radix sort with the reference's semantics.

    Returns ``keys_out`` or ``(keys_out, values_out)``.
    """
    keys = np.ascontiguousarray(keys)
    kd = NP_TO_DTYPE[keys.dtype]
    if end_bit is None:
        end_bit = keys.dtype.itemsize * 8
    kout = np.empty_like(keys)
    vout = None
    vbytes = 0
    if values is not None:
        values = np.ascontiguousarray(values)
        assert values.shape == keys.shape
        vbytes = values.dtype.itemsize
        vout = np.empty_like(values)
    rc = lib().oracle_radix_sort(_ptr(keys), _ptr(kout), _ptr(values), _ptr(vout), keys.size,
                                 begin_bit, end_bit, int(descending), kd, vbytes, threads)
    if rc != 0:
        raise ValueError(f"oracle_radix_sort failed with {rc}")
    return kout if values is None else (kout, vout)


def digit(key: int, dtype, descending: bool, bit_start: int, num_bits: int) -> int:
    return int(lib().oracle_digit(int(key), NP_TO_DTYPE[np.dtype(dtype)], int(descending),
                                  bit_start, num_bits))


def scan(x: np.ndarray, mode: str, op: int = OP_SUM, init=None) -> np.ndarray:
    """mode: 'exclusive' (needs init), 'inclusive', 'inclusive_init' (needs init)."""
    x = np.ascontiguousarray(x)
    out = np.empty_like(x)
    m = {"exclusive": 0, "inclusive": 1, "inclusive_init": 2}[mode]
    init_arr = None if init is None else np.array([init], dtype=x.dtype)
    rc = lib().oracle_scan(_ptr(x), _ptr(out), x.size, NP_TO_DTYPE[x.dtype], op, m, _ptr(init_arr))
    if rc != 0:
        raise ValueError(f"oracle_scan failed with {rc}")
    return out


def reduce(x: np.ndarray, op: int, init):
    x = np.ascontiguousarray(x)
    out = np.empty(1, dtype=x.dtype)
    init_arr = np.array([init], dtype=x.dtype)
    rc = lib().oracle_reduce(_ptr(x), _ptr(out), x.size, NP_TO_DTYPE[x.dtype], op, _ptr(init_arr))
    if rc != 0:
        raise ValueError(f"oracle_reduce failed with {rc}")
    return out[0]


def arg_extremum(x: np.ndarray, is_min: bool):
    """(value, index) of DeviceReduce::ArgMin / ArgMax (lcpp_oracle.c:
    oracle_arg_extremum, after src/lcpp/device/device_reduce.h:310-436)."""
    x = np.ascontiguousarray(x)
    out = np.empty(1, dtype=x.dtype)
    idx = np.empty(1, dtype=np.uint32)
    rc = lib().oracle_arg_extremum(_ptr(x), _ptr(out), _ptr(idx), x.size, NP_TO_DTYPE[x.dtype], int(is_min))
    if rc != 0:
        raise ValueError(f"oracle_arg_extremum failed with {rc}")
    return out[0], int(idx[0])


def arg_extremum_compare(x, is_min: bool, compare):
    """The comparator overloads (src/lcpp/device/device_reduce.h:539-605): one
    walk from item 0 where item i replaces the best when compare(item, best)
    (ArgMin) or compare(best, item) (ArgMax); 0 items give max() / lowest()
    and index 1.  Pure Python: small inputs only."""
    x = np.asarray(x)
    if x.size == 0:
        info = np.finfo(x.dtype) if x.dtype.kind == "f" else np.iinfo(x.dtype)
        return (x.dtype.type(info.max) if is_min else x.dtype.type(info.min)), 1
    best, bi = x[0], 0
    for i in range(1, x.size):
        c = x[i]
        if (compare(c, best) if is_min else compare(best, c)):
            best, bi = c, i
    return best, bi


def scan_by_key(keys: np.ndarray, values: np.ndarray, mode: str, op: int = OP_SUM, init=None) -> np.ndarray:
    """ExclusiveScanByKey / InclusiveScanByKey (lcpp_oracle.c: oracle_scan_by_key,
    after src/lcpp/device/device_scan.h:425-597).  mode: 'exclusive' (needs
    init), 'inclusive', 'inclusive_init' (needs init)."""
    keys, values = np.ascontiguousarray(keys), np.ascontiguousarray(values)
    out = np.empty_like(values)
    m = {"exclusive": 0, "inclusive": 1, "inclusive_init": 2}[mode]
    init_arr = None if init is None else np.array([init], dtype=values.dtype)
    rc = lib().oracle_scan_by_key(_ptr(keys), _ptr(values), _ptr(out), keys.size, NP_TO_DTYPE[keys.dtype],
                                  NP_TO_DTYPE[values.dtype], op, m, _ptr(init_arr))
    if rc != 0:
        raise ValueError(f"oracle_scan_by_key failed with {rc}")
    return out


def reduce_by_key(keys: np.ndarray, values: np.ndarray, op: int = OP_SUM):
    """ReduceByKey (lcpp_oracle.c: oracle_reduce_by_key, after
    src/lcpp/device/device_reduce.h:437-491) -> (unique keys, aggregates)."""
    keys, values = np.ascontiguousarray(keys), np.ascontiguousarray(values)
    uniq = np.empty_like(keys)
    agg = np.empty_like(values)
    runs = np.zeros(1, np.uint32)
    rc = lib().oracle_reduce_by_key(_ptr(keys), _ptr(values), _ptr(uniq), _ptr(agg), _ptr(runs), keys.size,
                                    NP_TO_DTYPE[keys.dtype], NP_TO_DTYPE[values.dtype], op)
    if rc != 0:
        raise ValueError(f"oracle_reduce_by_key failed with {rc}")
    r = int(runs[0])
    return uniq[:r], agg[:r]


def scan_by_key_equal(keys, values, mode: str, equal, op=lambda a, b: a + b, init=None):
    """The by-key scans with a user key-equality (the reference's EqualityOp
    overloads, device_scan.h:441-519); pure Python, small inputs only."""
    out, run = [], None
    for i, (k, v) in enumerate(zip(keys, values)):
        head = i == 0 or not equal(keys[i - 1], k)
        if mode == "exclusive":
            out.append(init if head else op(init, run))
            run = v if head else op(run, v)
        else:
            run = v if head else op(run, v)
            out.append(op(init, run) if mode == "inclusive_init" else run)
    return out


# ------------------------------------------------------------ select / partition
def clause_mask(x: np.ndarray, clauses) -> np.ndarray:
    """The C ABI's predicate (lcpp_clause, include/lcpp_b200.h): the AND of
    clauses (kind, negate, a, b), a and b given as values of x's type; MOD_EQ
    uses the C remainder (sign of the dividend), as the reference's `%`."""
    m = np.ones(x.shape, bool)
    for kind, negate, a, b in clauses:
        a, b = x.dtype.type(a), x.dtype.type(b)
        r = [lambda: x < a, lambda: x <= a, lambda: x > a, lambda: x >= a, lambda: x == a, lambda: x != a,
             lambda: np.fmod(x, a) == b, lambda: (x & a) != 0][kind]()
        m &= ~r if negate else r
    return m


def select(items: np.ndarray, mask: np.ndarray) -> np.ndarray:
    """DeviceSelect::Flagged / If / FlaggedIf (src/lcpp/device/device_select.h:
    65-212): the selected items in input order."""
    return items[mask]


def unique_mask(keys: np.ndarray) -> np.ndarray:
    """DeviceSelect::Unique / UniqueByKey (device_select.h:214-333): item 0 and
    every item that differs (!=, IEEE for floats) from its predecessor."""
    m = np.ones(keys.shape, bool)
    if keys.size > 1:
        m[1:] = keys[1:] != keys[:-1]
    return m


def partition(items: np.ndarray, mask: np.ndarray) -> np.ndarray:
    """DevicePartition::Flagged / If (src/lcpp/device/device_partition.h:
    531-575): selected items in order, then the rejected ones in reverse order."""
    return np.concatenate([items[mask], items[~mask][::-1]])


def partition_three_way(items: np.ndarray, first: np.ndarray, second: np.ndarray):
    """The three-way DevicePartition::If (device_partition.h:582-660): first
    in order, second (and not first) in order, the rest in reverse order."""
    second = second & ~first
    rest = ~(first | second)
    return items[first], items[second], items[rest][::-1]


def sum_f64(x: np.ndarray) -> float:
    x = np.ascontiguousarray(x)
    return float(lib().oracle_sum_f64(_ptr(x), x.size, NP_TO_DTYPE[x.dtype]))


def generate(dist: int, n: int, seed: int, offset: int = 0) -> np.ndarray:
    out = np.empty(n, dtype=GEN_NP_DTYPE[dist])
    rc = lib().oracle_generate(_ptr(out), n, offset, seed, dist)
    if rc != 0:
        raise ValueError(f"oracle_generate failed with {rc}")
    return out


def cpu_threads() -> int:
    return len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)


def segmented_radix_sort(keys: np.ndarray, values: np.ndarray | None, begin_offsets: np.ndarray,
                         end_offsets: np.ndarray, begin_bit: int = 0, end_bit: int | None = None,
                         descending: bool = False, out_keys: np.ndarray | None = None,
                         out_values: np.ndarray | None = None):
    """DeviceSegmentedRadixSort restated (numpy).

    Order: the key bits [begin_bit, end_bit) after the radix bijection --
    Traits<T>::TwiddleIn, no +-0.0 fold -- compared with < (ascending) or >
    (descending) in a stable sort (src/lcpp/device/device_segmented_radix_sort.h:216-243,
    src/lcpp/common/util_type.h:97-175).  Segment rule: item i belongs to the
    last segment s with begin[s] <= i, when i < end[s] and
    begin[s] <= end[s] <= n (src/lcpp/device/device_segmented_sort.h:753-775);
    other positions of the outputs keep their contents.  Returns
    (out_keys, out_values); outputs default to copies of the inputs.
    """
    n = keys.size
    bits = keys.dtype.itemsize * 8
    end_bit = bits if end_bit is None else end_bit
    ok = out_keys if out_keys is not None else keys.copy()
    ov = None
    if values is not None:
        ov = out_values if out_values is not None else values.copy()
    if n == 0 or begin_offsets.size == 0:
        return ok, ov
    u = keys.view(np.uint32 if bits == 32 else np.uint64).astype(np.uint64)
    full = np.uint64((1 << bits) - 1)
    high = np.uint64(1 << (bits - 1))
    if keys.dtype.kind == "i":
        t = u ^ high
    elif keys.dtype.kind == "f":
        t = np.where((u & high) != 0, (~u) & full, u ^ high)
    else:
        t = u
    width = end_bit - begin_bit
    fmask = np.uint64((1 << width) - 1) if width < 64 else np.uint64(0xFFFFFFFFFFFFFFFF)
    field = (t >> np.uint64(begin_bit)) & fmask if width else np.zeros(n, dtype=np.uint64)
    if descending:
        field = fmask - field
    pos = np.arange(n, dtype=np.int64)
    b = begin_offsets.astype(np.int64)
    e = end_offsets.astype(np.int64)
    seg = np.searchsorted(b, pos, side="right") - 1
    sc = np.clip(seg, 0, None)
    valid = (seg >= 0) & (pos >= b[sc]) & (pos < e[sc]) & (b[sc] <= e[sc]) & (e[sc] <= n)
    members = pos[valid]
    order = members[np.lexsort((field[valid], seg[valid]))]  # stable: by segment, then field
    ok[members] = keys[order]
    if ov is not None:
        ov[members] = values[order]
    return ok, ov


def _ordered_bits(col: np.ndarray) -> np.ndarray:
    """Order-preserving bits of one member column (uint64): unsigned as is,
    signed with the high bit flipped, floats sign-dependent with -0.0 as +0.0
    (src/lcpp/block/block_radix_sort.h:264-272)."""
    bits = col.dtype.itemsize * 8
    u = col.view(np.uint32 if bits == 32 else np.uint64).astype(np.uint64)
    high = np.uint64(1 << (bits - 1))
    full = np.uint64((1 << bits) - 1)
    if col.dtype.kind == "i":
        return u ^ high
    if col.dtype.kind == "f":
        t = np.where((u & high) != 0, (~u) & full, u ^ high)
        return np.where(t == high - np.uint64(1), high, t)
    return u


def decomposed_sort_order(members: list[np.ndarray], begin_bit: int = 0, end_bit: int | None = None,
                          descending: bool = False) -> np.ndarray:
    """Stable order of keys decomposed into member columns (most significant
    first), compared on the bit window [begin_bit, end_bit) of the
    concatenation of the members' ordered bits
    (src/lcpp/block/block_radix_sort.h:251-318,
    src/lcpp/device/device_radix_sort.h:788-823).  Returns the permutation."""
    n = members[0].size
    widths = [m.dtype.itemsize * 8 for m in members]
    total = sum(widths)
    end_bit = total if end_bit is None else end_bit
    lows, acc = [0] * len(members), 0
    for k in range(len(members) - 1, -1, -1):
        lows[k] = acc
        acc += widths[k]
    obits = [_ordered_bits(m) for m in members]
    chunks = []  # least significant first
    for lo in range(begin_bit, end_bit, 64):
        w = min(64, end_bit - lo)
        c = np.zeros(n, dtype=np.uint64)
        for k, b in enumerate(obits):
            olo, ohi = max(lows[k], lo), min(lows[k] + widths[k], lo + w)
            if olo >= ohi:
                continue
            ow = ohi - olo
            part = (b >> np.uint64(olo - lows[k])) & np.uint64((1 << ow) - 1 if ow < 64 else 0xFFFFFFFFFFFFFFFF)
            c |= part << np.uint64(olo - lo)
        if descending:
            c = np.uint64((1 << w) - 1 if w < 64 else 0xFFFFFFFFFFFFFFFF) - c
        chunks.append(c)
    if not chunks:
        return np.arange(n)
    return np.lexsort(chunks)  # the last key (most significant chunk) is primary; stable
