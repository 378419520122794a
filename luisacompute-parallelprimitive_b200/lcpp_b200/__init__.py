"""Python front end of liblcpp_b200 (sm_100a sort / scan / reduce).

A thin ctypes layer over the C ABI in ``include/lcpp_b200.h`` plus class
wrappers that mirror the reference's Device-level modules
(``DeviceRadixSort``, ``DeviceScan``, ``DeviceReduce`` in
``src/lcpp/device/``): same method names, same argument order, CUB-style
temp-storage queries.  Device buffers are torch CUDA tensors (torch is only
the allocator and stream provider here); every call enqueues on the current
torch CUDA stream unless a stream is given.

There is no CPU fallback: if ``liblcpp_b200.so`` has not been built, importing
the library raises.
"""
from __future__ import annotations

import ctypes
from pathlib import Path

_HERE = Path(__file__).resolve().parent
LIB_PATH = _HERE / "liblcpp_b200.so"

# lcpp_status
OK, ERR_INVALID_ARG, ERR_TEMP_TOO_SMALL, ERR_UNSUPPORTED_DTYPE = 0, 1, 2, 3
ERR_CUDA, ERR_LOOKBACK_TIMEOUT, ERR_COMM, ERR_INTERNAL = 4, 5, 6, 7
# lcpp_dtype
U32, I32, F32, U64, I64, F64, NONE = 0, 1, 2, 3, 4, 5, 255
U8 = 6  # 1-byte (bool) selection flags only
# lcpp_op
OP_SUM, OP_MIN, OP_MAX = 0, 1, 2
# lcpp_testgen_dist
GEN_U32_UNIFORM, GEN_U32_AND3, GEN_U32_CONST, GEN_U64_UNIFORM = 0, 1, 2, 3
GEN_I32_SCAN, GEN_F32_UNIT, GEN_I64_UNIFORM, GEN_U32_INDEX = 4, 5, 6, 7
GEN_F32_NORMAL, GEN_U32_ZIPF = 8, 9

# lcpp_kernel_kind
KERNEL_SORT_HISTOGRAM, KERNEL_SORT_ONESWEEP, KERNEL_SCAN, KERNEL_REDUCE, KERNEL_SEGMENT_BLOCK = 0, 1, 2, 3, 4
KERNEL_MERGE = 5
KERNEL_ARG_REDUCE = 6
KERNEL_BY_KEY = 7
KERNEL_SELECT = 8

_lib = None


class KernelTime(ctypes.Structure):
    _fields_ = [("kind", ctypes.c_int), ("ms", ctypes.c_float), ("items", ctypes.c_uint64)]


class DistSortTimes(ctypes.Structure):
    """lcpp_dist_sort_times (include/lcpp_b200_dist.h)."""
    _fields_ = [("local_sort_ms", ctypes.c_float), ("splitters_ms", ctypes.c_float),
                ("host_wait_ms", ctypes.c_float), ("exchange_merge_ms", ctypes.c_float),
                ("local_merge_ms", ctypes.c_float), ("total_ms", ctypes.c_float), ("host_ms", ctypes.c_float),
                ("peer_exchange", ctypes.c_int)]


class LcppError(RuntimeError):
    def __init__(self, status: int, what: str):
        self.status = status
        name = lib().lcpp_status_string(status).decode() if _lib is not None else str(status)
        super().__init__(f"{what}: {name}")


def lib() -> ctypes.CDLL:
    """Load liblcpp_b200.so (raises when it has not been built)."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise ImportError(
            f"{LIB_PATH} is missing: build it with "
            "`python luisacompute-parallelprimitive_b200/build.py` (no CPU fallback exists)")
    l = ctypes.CDLL(str(LIB_PATH))
    vp, sz, u64, i = ctypes.c_void_p, ctypes.c_size_t, ctypes.c_uint64, ctypes.c_int
    szp = ctypes.POINTER(ctypes.c_size_t)
    ip = ctypes.POINTER(ctypes.c_int)
    vpa = ctypes.c_void_p * 2
    sigs = {
        "lcpp_status_string": ([i], ctypes.c_char_p),
        "lcpp_version": ([], i),
        "lcpp_radix_sort_keys_temp_bytes": ([i, u64, szp], i),
        "lcpp_radix_sort_pairs_temp_bytes": ([i, i, u64, szp], i),
        "lcpp_radix_sort_keys": ([vp, sz, vp, vp, u64, i, i, i, i, vp], i),
        "lcpp_radix_sort_pairs": ([vp, sz, vp, vp, vp, vp, u64, i, i, i, i, i, vp], i),
        "lcpp_radix_sort_keys_double_buffer": ([vp, sz, vpa, ip, u64, i, i, i, i, vp], i),
        "lcpp_radix_sort_pairs_double_buffer": ([vp, sz, vpa, vpa, ip, u64, i, i, i, i, i, vp], i),
        "lcpp_radix_sort_decomposed_temp_bytes": ([u64, szp], i),
        "lcpp_radix_sort_decomposed_keys": ([vp, sz, vp, vp, u64, ctypes.c_uint32, vp, i, i, i, i, vp], i),
        "lcpp_radix_sort_decomposed_pairs": ([vp, sz, vp, vp, vp, vp, u64, ctypes.c_uint32, vp, i, i, i, i, i, vp],
                                             i),
        "lcpp_radix_sort_decomposed_keys_double_buffer": ([vp, sz, vpa, ip, u64, ctypes.c_uint32, vp, i, i, i, i, vp],
                                                          i),
        "lcpp_radix_sort_decomposed_pairs_double_buffer": ([vp, sz, vpa, vpa, ip, u64, ctypes.c_uint32, vp, i, i, i,
                                                            i, i, vp], i),
        "lcpp_segmented_radix_sort_keys_temp_bytes": ([i, u64, szp], i),
        "lcpp_segmented_radix_sort_pairs_temp_bytes": ([i, i, u64, szp], i),
        "lcpp_segmented_radix_sort_keys": ([vp, sz, vp, vp, u64, u64, vp, vp, i, i, i, i, vp], i),
        "lcpp_segmented_radix_sort_pairs": ([vp, sz, vp, vp, vp, vp, u64, u64, vp, vp, i, i, i, i, i, vp], i),
        "lcpp_segmented_radix_sort_keys_double_buffer": ([vp, sz, vpa, ip, u64, u64, vp, vp, i, i, i, i, vp], i),
        "lcpp_segmented_radix_sort_pairs_double_buffer": ([vp, sz, vpa, vpa, ip, u64, u64, vp, vp, i, i, i, i, i,
                                                           vp], i),
        "lcpp_scan_temp_bytes": ([i, u64, szp], i),
        "lcpp_scan_exclusive": ([vp, sz, vp, vp, u64, i, vp, i, vp], i),
        "lcpp_scan_inclusive": ([vp, sz, vp, vp, u64, i, i, vp], i),
        "lcpp_scan_inclusive_init": ([vp, sz, vp, vp, u64, i, vp, i, vp], i),
        "lcpp_scan_exclusive_sum": ([vp, sz, vp, vp, u64, i, vp], i),
        "lcpp_scan_inclusive_sum": ([vp, sz, vp, vp, u64, i, vp], i),
        "lcpp_scan_inclusive_sum_noalloc": ([vp, vp, u64, i, vp], i),
        "lcpp_reduce_temp_bytes": ([i, u64, szp], i),
        "lcpp_reduce_arg_temp_bytes": ([i, u64, szp], i),
        "lcpp_scan_by_key_temp_bytes": ([i, i, u64, szp], i),
        "lcpp_scan_exclusive_by_key": ([vp, sz, vp, vp, vp, u64, i, vp, i, i, vp], i),
        "lcpp_scan_inclusive_by_key": ([vp, sz, vp, vp, vp, u64, i, i, i, vp], i),
        "lcpp_scan_inclusive_by_key_init": ([vp, sz, vp, vp, vp, u64, i, vp, i, i, vp], i),
        "lcpp_scan_exclusive_sum_by_key": ([vp, sz, vp, vp, vp, u64, i, i, vp], i),
        "lcpp_scan_inclusive_sum_by_key": ([vp, sz, vp, vp, vp, u64, i, i, vp], i),
        "lcpp_reduce_by_key_temp_bytes": ([i, i, u64, szp], i),
        "lcpp_reduce_by_key": ([vp, sz, vp, vp, vp, vp, vp, u64, i, i, i, vp], i),
        "lcpp_scan_transform_temp_bytes": ([u64, szp], i),
        "lcpp_scan_exclusive_sum_transform": ([vp, sz, vp, vp, u64, i, vp, i, vp], i),
        "lcpp_scan_exclusive_sum_adjacent": ([vp, sz, vp, vp, u64, i, vp], i),
        "lcpp_select_temp_bytes": ([u64, szp], i),
        "lcpp_partition_temp_bytes": ([u64, szp], i),
        "lcpp_partition_three_way_temp_bytes": ([u64, szp], i),
        "lcpp_select_flagged": ([vp, sz, vp, vp, vp, vp, u64, i, i, vp], i),
        "lcpp_select_flagged_if": ([vp, sz, vp, vp, vp, vp, u64, i, i, vp, i, vp], i),
        "lcpp_select_if": ([vp, sz, vp, vp, vp, u64, i, vp, i, vp], i),
        "lcpp_select_unique": ([vp, sz, vp, vp, vp, u64, i, vp], i),
        "lcpp_select_unique_by_key": ([vp, sz, vp, vp, vp, vp, vp, u64, i, i, vp], i),
        "lcpp_partition_flagged": ([vp, sz, vp, vp, vp, vp, u64, i, i, vp], i),
        "lcpp_partition_if": ([vp, sz, vp, vp, vp, u64, i, vp, i, vp], i),
        "lcpp_partition_if_three_way": ([vp, sz, vp, vp, vp, vp, vp, u64, i, vp, i, vp, i, vp], i),
        "lcpp_reduce_argmin": ([vp, sz, vp, vp, vp, u64, i, vp], i),
        "lcpp_reduce_argmax": ([vp, sz, vp, vp, vp, u64, i, vp], i),
        "lcpp_reduce": ([vp, sz, vp, vp, u64, i, vp, i, vp], i),
        "lcpp_reduce_sum": ([vp, sz, vp, vp, u64, i, vp], i),
        "lcpp_reduce_min": ([vp, sz, vp, vp, u64, i, vp], i),
        "lcpp_reduce_max": ([vp, sz, vp, vp, u64, i, vp], i),
        "lcpp_device_status": ([vp, vp], i),
        "lcpp_testgen_fill": ([vp, u64, u64, u64, i, vp], i),
        "lcpp_dist_search_sorted": ([vp, u64, vp, u64, i, vp, i, vp], i),
        "lcpp_dist_merge_temp_bytes": ([u64, szp], i),
        "lcpp_dist_merge_sorted": ([vp, sz, vp, u64, vp, u64, vp, i, vp], i),
        "lcpp_dist_merge_batch_temp_bytes": ([i, ctypes.POINTER(u64), ctypes.POINTER(u64), szp], i),
        "lcpp_dist_merge_sorted_batch": ([vp, sz, i, ctypes.POINTER(vp), ctypes.POINTER(u64), ctypes.POINTER(vp),
                                          ctypes.POINTER(u64), ctypes.POINTER(vp), i, vp], i),
        "lcpp_dist_ipc_alloc": ([sz, ctypes.POINTER(ctypes.c_void_p), vp], i),
        "lcpp_dist_ipc_open": ([vp, ctypes.POINTER(ctypes.c_void_p)], i),
        "lcpp_dist_ipc_close": ([vp], i),
        "lcpp_dist_ipc_free": ([vp], i),
        "lcpp_comm_unique_id": ([vp], i),
        "lcpp_comm_init": ([vp, i, i, ctypes.POINTER(ctypes.c_void_p)], i),
        "lcpp_comm_from_nccl": ([vp, ctypes.POINTER(ctypes.c_void_p)], i),
        "lcpp_comm_destroy": ([vp], i),
        "lcpp_comm_rank": ([vp, ip, ip], i),
        "lcpp_dist_sort_keys_temp_bytes": ([vp, i, u64, szp], i),
        "lcpp_dist_sort_keys": ([vp, vp, sz, vp, vp, u64, i, i, ctypes.POINTER(DistSortTimes), vp], i),
        "lcpp_dist_scan_temp_bytes": ([vp, i, u64, szp], i),
        "lcpp_dist_inclusive_sum": ([vp, vp, sz, vp, vp, u64, i, vp], i),
        "lcpp_dist_exclusive_sum": ([vp, vp, sz, vp, vp, u64, i, vp], i),
        "lcpp_dist_reduce_temp_bytes": ([vp, i, u64, szp], i),
        "lcpp_dist_reduce": ([vp, vp, sz, vp, vp, u64, i, vp, i, vp], i),
        "lcpp_diag_timing_enable": ([i], i),
        "lcpp_diag_wait_timeout_probe": ([vp, sz, u64, vp], i),
        "lcpp_diag_timing_read": ([ctypes.POINTER(KernelTime), i, ip], i),
    }
    for name, (args, res) in sigs.items():
        f = getattr(l, name)
        f.argtypes = args
        f.restype = res
    _lib = l
    return l


def check(status: int, what: str) -> None:
    if status != OK:
        raise LcppError(status, what)


# ---------------------------------------------------------------------------
# torch helpers (plumbing only)
# ---------------------------------------------------------------------------
def _torch():
    import torch
    return torch


def dtype_code(t) -> int:
    torch = _torch()
    m = {torch.uint32: U32, torch.int32: I32, torch.float32: F32, torch.uint64: U64,
         torch.int64: I64, torch.float64: F64}
    if t.dtype not in m:
        raise TypeError(f"unsupported dtype {t.dtype}")
    return m[t.dtype]


def _ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream(stream):
    torch = _torch()
    if stream is None:
        stream = torch.cuda.current_stream()
    return ctypes.c_void_p(stream.cuda_stream)


def _host_scalar(value, code):
    import numpy as np
    np_t = {U32: np.uint32, I32: np.int32, F32: np.float32, U64: np.uint64, I64: np.int64,
            F64: np.float64}[code]
    arr = np.array([value], dtype=np_t)
    return arr, ctypes.c_void_p(arr.ctypes.data)


def alloc_temp(nbytes: int, device=None):
    """A 256-byte aligned uint8 CUDA tensor of at least nbytes (>= 1)."""
    torch = _torch()
    return torch.empty(max(int(nbytes), 1), dtype=torch.uint8, device=device or "cuda")


# ---------------------------------------------------------------------------
# Reference-shaped module wrappers
# ---------------------------------------------------------------------------
class DoubleBuffer:
    """Mirror of the reference's DoubleBuffer<T> (src/lcpp/common/util_type.h:57-74)."""

    def __init__(self, current, alternate, selector: int = 0):
        self.d_buffers = [current, alternate]
        self.selector = selector

    def current(self):
        return self.d_buffers[self.selector]

    def alternate(self):
        return self.d_buffers[self.selector ^ 1]


def _bit_range(rest):
    """(begin_bit, end_bit) from trailing positional arguments; end None = key width."""
    if len(rest) > 2:
        raise TypeError("too many arguments")
    begin = rest[0] if len(rest) >= 1 else 0
    end = rest[1] if len(rest) == 2 else None
    return begin, end


class Clause(ctypes.Structure):
    """One clause of a C-ABI predicate (lcpp_clause in include/lcpp_b200.h)."""
    _fields_ = [("kind", ctypes.c_int32), ("negate", ctypes.c_int32), ("a", ctypes.c_uint64),
                ("b", ctypes.c_uint64)]


CLAUSE_LT, CLAUSE_LE, CLAUSE_GT, CLAUSE_GE, CLAUSE_EQ, CLAUSE_NE, CLAUSE_MOD_EQ, CLAUSE_BITS_ANY = range(8)


def _bits(value, code: int) -> int:
    import struct
    if code == F32:
        return struct.unpack("<I", struct.pack("<f", float(value)))[0]
    if code == F64:
        return struct.unpack("<Q", struct.pack("<d", float(value)))[0]
    width = {U8: 8, U32: 32, I32: 32, U64: 64, I64: 64}[code]
    return int(value) & ((1 << width) - 1)


class Pred:
    """A predicate for DeviceSelect / DevicePartition through the C ABI: the
    AND (`&`) of up to 4 clauses, each negatable (`~`).  Examples: the
    reference tests' `value % 2 == 0` is Pred.mod_eq(2, 0), `value < 7` is
    Pred.lt(7), `flag > 0 & flag % 2 != 0` is Pred.gt(0) & ~Pred.mod_eq(2, 0)."""

    def __init__(self, clauses=()):
        self.clauses = list(clauses)  # (kind, negate, a, b)

    def __and__(self, other: "Pred") -> "Pred":
        return Pred(self.clauses + other.clauses)

    def __invert__(self) -> "Pred":
        if len(self.clauses) != 1:
            raise ValueError("~ applies to a single clause")
        k, n, a, b = self.clauses[0]
        return Pred([(k, 1 - n, a, b)])

    @staticmethod
    def lt(a): return Pred([(CLAUSE_LT, 0, a, 0)])
    @staticmethod
    def le(a): return Pred([(CLAUSE_LE, 0, a, 0)])
    @staticmethod
    def gt(a): return Pred([(CLAUSE_GT, 0, a, 0)])
    @staticmethod
    def ge(a): return Pred([(CLAUSE_GE, 0, a, 0)])
    @staticmethod
    def eq(a): return Pred([(CLAUSE_EQ, 0, a, 0)])
    @staticmethod
    def ne(a): return Pred([(CLAUSE_NE, 0, a, 0)])
    @staticmethod
    def mod_eq(m, r): return Pred([(CLAUSE_MOD_EQ, 0, m, r)])
    @staticmethod
    def bits_any(mask): return Pred([(CLAUSE_BITS_ANY, 0, mask, 0)])

    def encode(self, code: int):
        """(ctypes array, count) for values of dtype `code`."""
        arr = (Clause * max(1, len(self.clauses)))()
        for j, (k, n, a, b) in enumerate(self.clauses):
            arr[j] = Clause(k, n, _bits(a, code), _bits(b, code))
        return arr, len(self.clauses)


def flag_code(t) -> int:
    """dtype code of a selection-flag tensor (bool and uint8 are LCPP_U8)."""
    torch = _torch()
    if t.dtype in (torch.bool, torch.uint8):
        return U8
    return dtype_code(t)


class KeyMember(ctypes.Structure):
    _fields_ = [("offset", ctypes.c_uint32), ("dtype", ctypes.c_int)]


class Decomposer:
    """The reference's decomposer for struct keys (device_radix_sort.h:556-940):
    the key struct's size in bytes and its members, most significant first, as
    (byte offset, dtype code) pairs."""

    def __init__(self, key_bytes: int, members):
        self.key_bytes = int(key_bytes)
        self.members = [(int(o), int(d)) for o, d in members]
        self.bits = sum(8 * (4 if d in (U32, I32, F32) else 8) for _, d in self.members)
        arr = (KeyMember * len(self.members))(*[KeyMember(o, d) for o, d in self.members])
        self._arr = arr


class DeviceRadixSort:
    """Mirror of lcpp::DeviceRadixSort (src/lcpp/device/device_radix_sort.h:50-1489)."""

    @staticmethod
    def GetDecomposedTempStorageBytes(num_items: int) -> int:
        out = ctypes.c_size_t()
        check(lib().lcpp_radix_sort_decomposed_temp_bytes(num_items, ctypes.byref(out)),
              "GetDecomposedTempStorageBytes")
        return out.value

    @staticmethod
    def GetSortKeysTempStorageBytes(key_dtype: int, num_items: int) -> int:
        out = ctypes.c_size_t()
        check(lib().lcpp_radix_sort_keys_temp_bytes(key_dtype, num_items, ctypes.byref(out)),
              "GetSortKeysTempStorageBytes")
        return out.value

    @staticmethod
    def GetSortPairsTempStorageBytes(key_dtype: int, value_dtype: int, num_items: int) -> int:
        out = ctypes.c_size_t()
        check(lib().lcpp_radix_sort_pairs_temp_bytes(key_dtype, value_dtype, num_items,
                                                     ctypes.byref(out)),
              "GetSortPairsTempStorageBytes")
        return out.value

    def _keys(self, temp, kin, kout, n, begin, end, desc, stream):
        kd = dtype_code(kin)
        end = kin.element_size() * 8 if end is None else end
        check(lib().lcpp_radix_sort_keys(_ptr(temp), temp.numel() if temp is not None else 0,
                                         _ptr(kin), _ptr(kout), n, begin, end, int(desc), kd,
                                         _stream(stream)), "SortKeys")

    def _pairs(self, temp, kin, kout, vin, vout, n, begin, end, desc, stream):
        kd, vd = dtype_code(kin), dtype_code(vin)
        end = kin.element_size() * 8 if end is None else end
        check(lib().lcpp_radix_sort_pairs(_ptr(temp), temp.numel() if temp is not None else 0,
                                          _ptr(kin), _ptr(kout), _ptr(vin), _ptr(vout), n, begin,
                                          end, int(desc), kd, vd, _stream(stream)), "SortPairs")

    # Overloads as in the reference: copy form (temp, keys_in, keys_out, n, begin, end) and
    # DoubleBuffer form (temp, keys_db, n, begin, end) (device_radix_sort.h:369-555).
    def SortKeys(self, temp, *args, stream=None):
        self._dispatch_keys(temp, args, False, stream)

    def SortKeysDescending(self, temp, *args, stream=None):
        self._dispatch_keys(temp, args, True, stream)

    # Copy form (temp, keys_in, keys_out, values_in, values_out, n, begin, end) and
    # DoubleBuffer form (temp, keys_db, values_db, n, begin, end).
    def SortPairs(self, temp, *args, stream=None):
        self._dispatch_pairs(temp, args, False, stream)

    def SortPairsDescending(self, temp, *args, stream=None):
        self._dispatch_pairs(temp, args, True, stream)

    def _decomposed(self, temp, args, desc, stream, pairs):
        tb = temp.numel() if temp is not None else 0
        st = _stream(stream)
        if isinstance(args[0], DoubleBuffer):
            if pairs:
                kdb, vdb, n, dec, *rest = args
                if kdb.selector != vdb.selector:
                    raise LcppError(ERR_INVALID_ARG, "key and value DoubleBuffer selectors must match")
            else:
                kdb, n, dec, *rest = args
            begin, end = _bit_range(rest)
            end = dec.bits if end is None else end
            kb = (ctypes.c_void_p * 2)(kdb.d_buffers[0].data_ptr(), kdb.d_buffers[1].data_ptr())
            sel = ctypes.c_int(kdb.selector)
            if pairs:
                vb = (ctypes.c_void_p * 2)(vdb.d_buffers[0].data_ptr(), vdb.d_buffers[1].data_ptr())
                check(lib().lcpp_radix_sort_decomposed_pairs_double_buffer(
                    _ptr(temp), tb, kb, vb, ctypes.byref(sel), n, dec.key_bytes, dec._arr, len(dec.members), begin,
                    end, int(desc), dtype_code(vdb.d_buffers[0]), st), "SortPairs(decomposed, DoubleBuffer)")
                vdb.selector = sel.value
            else:
                check(lib().lcpp_radix_sort_decomposed_keys_double_buffer(
                    _ptr(temp), tb, kb, ctypes.byref(sel), n, dec.key_bytes, dec._arr, len(dec.members), begin, end,
                    int(desc), st), "SortKeys(decomposed, DoubleBuffer)")
            kdb.selector = sel.value
            return
        if pairs:
            kin, kout, vin, vout, n, dec, *rest = args
        else:
            kin, kout, n, dec, *rest = args
        begin, end = _bit_range(rest)
        end = dec.bits if end is None else end
        if pairs:
            check(lib().lcpp_radix_sort_decomposed_pairs(
                _ptr(temp), tb, _ptr(kin), _ptr(kout), _ptr(vin), _ptr(vout), n, dec.key_bytes, dec._arr,
                len(dec.members), begin, end, int(desc), dtype_code(vin), st), "SortPairs(decomposed)")
        else:
            check(lib().lcpp_radix_sort_decomposed_keys(
                _ptr(temp), tb, _ptr(kin), _ptr(kout), n, dec.key_bytes, dec._arr, len(dec.members), begin, end,
                int(desc), st), "SortKeys(decomposed)")

    def _dispatch_keys(self, temp, args, desc, stream):
        if any(isinstance(a, Decomposer) for a in args):
            return self._decomposed(temp, args, desc, stream, False)
        if isinstance(args[0], DoubleBuffer):
            db, n, *rest = args
            begin, end = _bit_range(rest)
            return self._keys_db(temp, db, n, begin, end, desc, stream)
        kin, kout, n, *rest = args
        begin, end = _bit_range(rest)
        self._keys(temp, kin, kout, n, begin, end, desc, stream)

    def _dispatch_pairs(self, temp, args, desc, stream):
        if any(isinstance(a, Decomposer) for a in args):
            return self._decomposed(temp, args, desc, stream, True)
        if isinstance(args[0], DoubleBuffer):
            kdb, vdb, n, *rest = args
            begin, end = _bit_range(rest)
            return self._pairs_db(temp, kdb, vdb, n, begin, end, desc, stream)
        kin, kout, vin, vout, n, *rest = args
        begin, end = _bit_range(rest)
        self._pairs(temp, kin, kout, vin, vout, n, begin, end, desc, stream)

    # DoubleBuffer forms: SortKeys(temp, db, n, begin, end)
    def _keys_db(self, temp, db, n, begin, end, desc, stream):
        kd = dtype_code(db.d_buffers[0])
        end = db.d_buffers[0].element_size() * 8 if end is None else end
        bufs = (ctypes.c_void_p * 2)(db.d_buffers[0].data_ptr(), db.d_buffers[1].data_ptr())
        sel = ctypes.c_int(db.selector)
        check(lib().lcpp_radix_sort_keys_double_buffer(
            _ptr(temp), temp.numel() if temp is not None else 0, bufs, ctypes.byref(sel), n,
            begin, end, int(desc), kd, _stream(stream)), "SortKeys(DoubleBuffer)")
        db.selector = sel.value

    def _pairs_db(self, temp, kdb, vdb, n, begin, end, desc, stream):
        if kdb.selector != vdb.selector:
            raise LcppError(ERR_INVALID_ARG, "key and value DoubleBuffer selectors must match")
        kd, vd = dtype_code(kdb.d_buffers[0]), dtype_code(vdb.d_buffers[0])
        end = kdb.d_buffers[0].element_size() * 8 if end is None else end
        kb = (ctypes.c_void_p * 2)(kdb.d_buffers[0].data_ptr(), kdb.d_buffers[1].data_ptr())
        vb = (ctypes.c_void_p * 2)(vdb.d_buffers[0].data_ptr(), vdb.d_buffers[1].data_ptr())
        sel = ctypes.c_int(kdb.selector)
        check(lib().lcpp_radix_sort_pairs_double_buffer(
            _ptr(temp), temp.numel() if temp is not None else 0, kb, vb, ctypes.byref(sel), n,
            begin, end, int(desc), kd, vd, _stream(stream)), "SortPairs(DoubleBuffer)")
        kdb.selector = vdb.selector = sel.value


class DeviceSegmentedRadixSort:
    """Mirror of lcpp::DeviceSegmentedRadixSort
    (src/lcpp/device/device_segmented_radix_sort.h:16-246): copy form
    (temp, keys_in, keys_out, n, num_segments, begin_offsets, end_offsets,
    begin_bit, end_bit) and DoubleBuffer form (temp, keys_db, n, num_segments,
    begin_offsets, end_offsets, begin_bit, end_bit); offsets are uint32 device
    tensors."""

    @staticmethod
    def GetSortKeysTempStorageBytes(key_dtype: int, num_items: int) -> int:
        out = ctypes.c_size_t()
        check(lib().lcpp_segmented_radix_sort_keys_temp_bytes(key_dtype, num_items, ctypes.byref(out)),
              "GetSortKeysTempStorageBytes")
        return out.value

    @staticmethod
    def GetSortPairsTempStorageBytes(key_dtype: int, value_dtype: int, num_items: int) -> int:
        out = ctypes.c_size_t()
        check(lib().lcpp_segmented_radix_sort_pairs_temp_bytes(key_dtype, value_dtype, num_items,
                                                               ctypes.byref(out)), "GetSortPairsTempStorageBytes")
        return out.value

    def SortKeys(self, temp, *args, stream=None):
        self._keys(temp, args, False, stream)

    def SortKeysDescending(self, temp, *args, stream=None):
        self._keys(temp, args, True, stream)

    def SortPairs(self, temp, *args, stream=None):
        self._pairs(temp, args, False, stream)

    def SortPairsDescending(self, temp, *args, stream=None):
        self._pairs(temp, args, True, stream)

    def _keys(self, temp, args, desc, stream):
        tb = temp.numel() if temp is not None else 0
        if isinstance(args[0], DoubleBuffer):
            db, n, nseg, bo, eo, *rest = args
            begin, end = _bit_range(rest)
            k0 = db.d_buffers[0]
            end = k0.element_size() * 8 if end is None else end
            bufs = (ctypes.c_void_p * 2)(db.d_buffers[0].data_ptr(), db.d_buffers[1].data_ptr())
            sel = ctypes.c_int(db.selector)
            check(lib().lcpp_segmented_radix_sort_keys_double_buffer(
                _ptr(temp), tb, bufs, ctypes.byref(sel), n, nseg, _ptr(bo), _ptr(eo), begin, end, int(desc),
                dtype_code(k0), _stream(stream)), "SortKeys(DoubleBuffer)")
            db.selector = sel.value
            return
        kin, kout, n, nseg, bo, eo, *rest = args
        begin, end = _bit_range(rest)
        end = kin.element_size() * 8 if end is None else end
        check(lib().lcpp_segmented_radix_sort_keys(_ptr(temp), tb, _ptr(kin), _ptr(kout), n, nseg, _ptr(bo),
                                                   _ptr(eo), begin, end, int(desc), dtype_code(kin),
                                                   _stream(stream)), "SortKeys")

    def _pairs(self, temp, args, desc, stream):
        tb = temp.numel() if temp is not None else 0
        if isinstance(args[0], DoubleBuffer):
            kdb, vdb, n, nseg, bo, eo, *rest = args
            if kdb.selector != vdb.selector:
                raise LcppError(ERR_INVALID_ARG, "key and value DoubleBuffer selectors must match")
            begin, end = _bit_range(rest)
            k0, v0 = kdb.d_buffers[0], vdb.d_buffers[0]
            end = k0.element_size() * 8 if end is None else end
            kb = (ctypes.c_void_p * 2)(kdb.d_buffers[0].data_ptr(), kdb.d_buffers[1].data_ptr())
            vb = (ctypes.c_void_p * 2)(vdb.d_buffers[0].data_ptr(), vdb.d_buffers[1].data_ptr())
            sel = ctypes.c_int(kdb.selector)
            check(lib().lcpp_segmented_radix_sort_pairs_double_buffer(
                _ptr(temp), tb, kb, vb, ctypes.byref(sel), n, nseg, _ptr(bo), _ptr(eo), begin, end, int(desc),
                dtype_code(k0), dtype_code(v0), _stream(stream)), "SortPairs(DoubleBuffer)")
            kdb.selector = vdb.selector = sel.value
            return
        kin, kout, vin, vout, n, nseg, bo, eo, *rest = args
        begin, end = _bit_range(rest)
        end = kin.element_size() * 8 if end is None else end
        check(lib().lcpp_segmented_radix_sort_pairs(_ptr(temp), tb, _ptr(kin), _ptr(kout), _ptr(vin), _ptr(vout),
                                                    n, nseg, _ptr(bo), _ptr(eo), begin, end, int(desc),
                                                    dtype_code(kin), dtype_code(vin), _stream(stream)), "SortPairs")


class DeviceScan:
    """Mirror of lcpp::DeviceScan (src/lcpp/device/device_scan.h:40-1560)."""

    @staticmethod
    def GetTempStorageBytes(dtype: int, num_items: int) -> int:
        out = ctypes.c_size_t()
        check(lib().lcpp_scan_temp_bytes(dtype, num_items, ctypes.byref(out)), "GetTempStorageBytes")
        return out.value

    def ExclusiveSum(self, temp, d_in, d_out, num_items, stream=None):
        check(lib().lcpp_scan_exclusive_sum(_ptr(temp), temp.numel() if temp is not None else 0,
                                            _ptr(d_in), _ptr(d_out), num_items, dtype_code(d_in),
                                            _stream(stream)), "ExclusiveSum")

    def InclusiveSum(self, temp, d_in, d_out, num_items, stream=None):
        check(lib().lcpp_scan_inclusive_sum(_ptr(temp), temp.numel() if temp is not None else 0,
                                            _ptr(d_in), _ptr(d_out), num_items, dtype_code(d_in),
                                            _stream(stream)), "InclusiveSum")

    def ExclusiveScan(self, temp, d_in, d_out, num_items, op, initial_value, stream=None):
        code = dtype_code(d_in)
        keep, init = _host_scalar(initial_value, code)
        check(lib().lcpp_scan_exclusive(_ptr(temp), temp.numel() if temp is not None else 0,
                                        _ptr(d_in), _ptr(d_out), num_items, op, init, code,
                                        _stream(stream)), "ExclusiveScan")
        del keep

    def InclusiveScan(self, temp, d_in, d_out, num_items, op, initial_value=None, stream=None):
        code = dtype_code(d_in)
        if initial_value is None:
            check(lib().lcpp_scan_inclusive(_ptr(temp), temp.numel() if temp is not None else 0,
                                            _ptr(d_in), _ptr(d_out), num_items, op, code,
                                            _stream(stream)), "InclusiveScan")
        else:
            self.InclusiveScanInit(temp, d_in, d_out, num_items, op, initial_value, stream)

    def InclusiveScanInit(self, temp, d_in, d_out, num_items, op, initial_value, stream=None):
        code = dtype_code(d_in)
        keep, init = _host_scalar(initial_value, code)
        check(lib().lcpp_scan_inclusive_init(_ptr(temp), temp.numel() if temp is not None else 0,
                                             _ptr(d_in), _ptr(d_out), num_items, op, init, code,
                                             _stream(stream)), "InclusiveScanInit")
        del keep

    # ---- counting scans (device_scan.h:387-406)
    @staticmethod
    def GetTransformTempStorageBytes(num_items: int) -> int:
        out = ctypes.c_size_t()
        check(lib().lcpp_scan_transform_temp_bytes(num_items, ctypes.byref(out)), "GetTransformTempStorageBytes")
        return out.value

    def ExclusiveSumTransform(self, temp, d_in, d_out, num_items, pred, stream=None):
        """d_out[i] (4-byte tensor) = how many of d_in[0..i) satisfy pred (a Pred)."""
        code = dtype_code(d_in)
        arr, n = pred.encode(code)
        check(lib().lcpp_scan_exclusive_sum_transform(_ptr(temp), temp.numel() if temp is not None else 0,
                                                      _ptr(d_in), _ptr(d_out), num_items, code, arr, n,
                                                      _stream(stream)), "ExclusiveSumTransform")

    def ExclusiveSumAdjacent(self, temp, d_in, d_out, num_items, stream=None):
        """d_out[i] = how many runs of equal items start before i."""
        check(lib().lcpp_scan_exclusive_sum_adjacent(_ptr(temp), temp.numel() if temp is not None else 0,
                                                     _ptr(d_in), _ptr(d_out), num_items, dtype_code(d_in),
                                                     _stream(stream)), "ExclusiveSumAdjacent")

    # ---- by key (device_scan.h:310-597): argument order as the reference's
    @staticmethod
    def GetScanByKeyTempStorageBytes(key_dtype: int, value_dtype: int, num_items: int) -> int:
        out = ctypes.c_size_t()
        check(lib().lcpp_scan_by_key_temp_bytes(key_dtype, value_dtype, num_items, ctypes.byref(out)),
              "GetScanByKeyTempStorageBytes")
        return out.value

    def ExclusiveScanByKey(self, temp, d_keys_in, d_values_in, d_values_out, scan_op, num_items, initial_value,
                           stream=None):
        vc = dtype_code(d_values_in)
        keep, init = _host_scalar(initial_value, vc)
        check(lib().lcpp_scan_exclusive_by_key(_ptr(temp), temp.numel() if temp is not None else 0,
                                               _ptr(d_keys_in), _ptr(d_values_in), _ptr(d_values_out), num_items,
                                               scan_op, init, dtype_code(d_keys_in), vc, _stream(stream)),
              "ExclusiveScanByKey")
        del keep

    def InclusiveScanByKey(self, temp, d_keys_in, d_values_in, d_values_out, scan_op, num_items,
                           initial_value=None, stream=None):
        vc = dtype_code(d_values_in)
        t = (_ptr(temp), temp.numel() if temp is not None else 0, _ptr(d_keys_in), _ptr(d_values_in),
             _ptr(d_values_out), num_items, scan_op)
        if initial_value is None:
            check(lib().lcpp_scan_inclusive_by_key(*t, dtype_code(d_keys_in), vc, _stream(stream)),
                  "InclusiveScanByKey")
        else:
            keep, init = _host_scalar(initial_value, vc)
            check(lib().lcpp_scan_inclusive_by_key_init(*t, init, dtype_code(d_keys_in), vc, _stream(stream)),
                  "InclusiveScanByKey")
            del keep

    def ExclusiveSumByKey(self, temp, d_keys_in, d_values_in, d_values_out, num_items, stream=None):
        check(lib().lcpp_scan_exclusive_sum_by_key(_ptr(temp), temp.numel() if temp is not None else 0,
                                                   _ptr(d_keys_in), _ptr(d_values_in), _ptr(d_values_out),
                                                   num_items, dtype_code(d_keys_in), dtype_code(d_values_in),
                                                   _stream(stream)), "ExclusiveSumByKey")

    def InclusiveSumByKey(self, temp, d_keys_in, d_values_in, d_values_out, num_items, stream=None):
        check(lib().lcpp_scan_inclusive_sum_by_key(_ptr(temp), temp.numel() if temp is not None else 0,
                                                   _ptr(d_keys_in), _ptr(d_values_in), _ptr(d_values_out),
                                                   num_items, dtype_code(d_keys_in), dtype_code(d_values_in),
                                                   _stream(stream)), "InclusiveSumByKey")


class DeviceReduce:
    """Mirror of lcpp::DeviceReduce (src/lcpp/device/device_reduce.h:102-1187)."""

    @staticmethod
    def GetTempStorageBytes(dtype: int, num_items: int) -> int:
        out = ctypes.c_size_t()
        check(lib().lcpp_reduce_temp_bytes(dtype, num_items, ctypes.byref(out)), "GetTempStorageBytes")
        return out.value

    def Reduce(self, temp, d_in, d_out, num_items, op, initial_value, stream=None):
        code = dtype_code(d_in)
        keep, init = _host_scalar(initial_value, code)
        check(lib().lcpp_reduce(_ptr(temp), temp.numel() if temp is not None else 0, _ptr(d_in),
                                _ptr(d_out), num_items, op, init, code, _stream(stream)), "Reduce")
        del keep

    def _named(self, fn, temp, d_in, d_out, num_items, stream, what):
        check(fn(_ptr(temp), temp.numel() if temp is not None else 0, _ptr(d_in), _ptr(d_out),
                 num_items, dtype_code(d_out), _stream(stream)), what)

    @staticmethod
    def GetReduceByKeyTempStorageBytes(key_dtype: int, value_dtype: int, num_items: int) -> int:
        out = ctypes.c_size_t()
        check(lib().lcpp_reduce_by_key_temp_bytes(key_dtype, value_dtype, num_items, ctypes.byref(out)),
              "GetReduceByKeyTempStorageBytes")
        return out.value

    def ReduceByKey(self, temp, d_keys_in, d_values_in, d_unique_out, d_aggregates_out, d_num_runs_out,
                    reduce_op, num_elements, stream=None):
        """device_reduce.h:437-491 (argument order as the reference's);
        d_num_runs_out: a one-element 4-byte tensor (uint32 run count)."""
        check(lib().lcpp_reduce_by_key(_ptr(temp), temp.numel() if temp is not None else 0, _ptr(d_keys_in),
                                       _ptr(d_values_in), _ptr(d_unique_out), _ptr(d_aggregates_out),
                                       _ptr(d_num_runs_out), num_elements, reduce_op, dtype_code(d_keys_in),
                                       dtype_code(d_values_in), _stream(stream)), "ReduceByKey")

    @staticmethod
    def GetArgTempStorageBytes(dtype: int, num_items: int) -> int:
        out = ctypes.c_size_t()
        check(lib().lcpp_reduce_arg_temp_bytes(dtype, num_items, ctypes.byref(out)), "GetArgTempStorageBytes")
        return out.value

    def ArgMin(self, temp, d_in, d_out, d_index_out, num_items, stream=None):
        """d_out[0] = min value, d_index_out[0] = its first index (uint32 / int32 tensor)."""
        check(lib().lcpp_reduce_argmin(_ptr(temp), temp.numel() if temp is not None else 0, _ptr(d_in), _ptr(d_out),
                                       _ptr(d_index_out), num_items, dtype_code(d_out), _stream(stream)), "ArgMin")

    def ArgMax(self, temp, d_in, d_out, d_index_out, num_items, stream=None):
        check(lib().lcpp_reduce_argmax(_ptr(temp), temp.numel() if temp is not None else 0, _ptr(d_in), _ptr(d_out),
                                       _ptr(d_index_out), num_items, dtype_code(d_out), _stream(stream)), "ArgMax")

    def Sum(self, temp, d_in, d_out, num_items, stream=None):
        self._named(lib().lcpp_reduce_sum, temp, d_in, d_out, num_items, stream, "Sum")

    def Min(self, temp, d_in, d_out, num_items, stream=None):
        self._named(lib().lcpp_reduce_min, temp, d_in, d_out, num_items, stream, "Min")

    def Max(self, temp, d_in, d_out, num_items, stream=None):
        self._named(lib().lcpp_reduce_max, temp, d_in, d_out, num_items, stream, "Max")


def device_status(temp, stream=None) -> int:
    """Synchronise and read the device error word of the call that used `temp`."""
    return lib().lcpp_device_status(_ptr(temp), _stream(stream))


def testgen_fill(dst, dist: int, seed: int, offset: int = 0, stream=None) -> None:
    check(lib().lcpp_testgen_fill(_ptr(dst), dst.numel(), offset, seed, dist, _stream(stream)),
          "testgen_fill")


def diag_timing_enable(enable: bool) -> None:
    """Record CUDA events around every library kernel launch (lcpp_b200_diag.h)."""
    check(lib().lcpp_diag_timing_enable(int(enable)), "diag_timing_enable")


def diag_timing_read() -> list[tuple[int, float, int]]:
    """(kind, ms, items) of every launch recorded since timing was enabled."""
    count = ctypes.c_int()
    check(lib().lcpp_diag_timing_read(None, 0, ctypes.byref(count)), "diag_timing_read")
    buf = (KernelTime * max(count.value, 1))()
    check(lib().lcpp_diag_timing_read(buf, count.value, ctypes.byref(count)), "diag_timing_read")
    return [(buf[i].kind, buf[i].ms, buf[i].items) for i in range(count.value)]


def _tb(temp):
    return temp.numel() if temp is not None else 0


class DeviceSelect:
    """Mirror of lcpp::DeviceSelect (src/lcpp/device/device_select.h); the
    predicate arguments are Pred objects.  Passing d_out = d_in (or omitting
    it in the in-place helpers) compacts in place."""

    @staticmethod
    def GetTempStorageBytes(num_items: int) -> int:
        out = ctypes.c_size_t()
        check(lib().lcpp_select_temp_bytes(num_items, ctypes.byref(out)), "GetTempStorageBytes")
        return out.value

    def Flagged(self, temp, d_in, d_flags, d_out, d_num_selected_out, num_items, stream=None):
        check(lib().lcpp_select_flagged(_ptr(temp), _tb(temp), _ptr(d_in), _ptr(d_flags), _ptr(d_out),
                                        _ptr(d_num_selected_out), num_items, dtype_code(d_in), flag_code(d_flags),
                                        _stream(stream)), "Flagged")

    def FlaggedIf(self, temp, d_in, d_flags, d_out, d_num_selected_out, num_items, pred: Pred, stream=None):
        fc = flag_code(d_flags)
        arr, n = pred.encode(fc)
        check(lib().lcpp_select_flagged_if(_ptr(temp), _tb(temp), _ptr(d_in), _ptr(d_flags), _ptr(d_out),
                                           _ptr(d_num_selected_out), num_items, dtype_code(d_in), fc, arr, n,
                                           _stream(stream)), "FlaggedIf")

    def If(self, temp, d_in, d_out, d_num_selected_out, num_items, pred: Pred, stream=None):
        code = dtype_code(d_in)
        arr, n = pred.encode(code)
        check(lib().lcpp_select_if(_ptr(temp), _tb(temp), _ptr(d_in), _ptr(d_out), _ptr(d_num_selected_out),
                                   num_items, code, arr, n, _stream(stream)), "If")

    def Unique(self, temp, d_in, d_out, d_num_selected_out, num_items, stream=None):
        check(lib().lcpp_select_unique(_ptr(temp), _tb(temp), _ptr(d_in), _ptr(d_out), _ptr(d_num_selected_out),
                                       num_items, dtype_code(d_in), _stream(stream)), "Unique")

    def UniqueByKey(self, temp, d_keys_in, d_values_in, d_keys_out, d_values_out, d_num_selected_out, num_items,
                    stream=None):
        check(lib().lcpp_select_unique_by_key(_ptr(temp), _tb(temp), _ptr(d_keys_in), _ptr(d_values_in),
                                              _ptr(d_keys_out), _ptr(d_values_out), _ptr(d_num_selected_out),
                                              num_items, dtype_code(d_keys_in), dtype_code(d_values_in),
                                              _stream(stream)), "UniqueByKey")


class DevicePartition:
    """Mirror of lcpp::DevicePartition (src/lcpp/device/device_partition.h):
    selected items in order from the front, rejected ones in reverse order
    from the back."""

    @staticmethod
    def GetTempStorageBytes(num_items: int) -> int:
        out = ctypes.c_size_t()
        check(lib().lcpp_partition_temp_bytes(num_items, ctypes.byref(out)), "GetTempStorageBytes")
        return out.value

    @staticmethod
    def GetThreeWayTempStorageBytes(num_items: int) -> int:
        out = ctypes.c_size_t()
        check(lib().lcpp_partition_three_way_temp_bytes(num_items, ctypes.byref(out)),
              "GetThreeWayTempStorageBytes")
        return out.value

    def Flagged(self, temp, d_in, d_flags, d_out, d_num_selected_out, num_items, stream=None):
        check(lib().lcpp_partition_flagged(_ptr(temp), _tb(temp), _ptr(d_in), _ptr(d_flags), _ptr(d_out),
                                           _ptr(d_num_selected_out), num_items, dtype_code(d_in),
                                           flag_code(d_flags), _stream(stream)), "Flagged")

    def If(self, temp, d_in, d_out, d_num_selected_out, num_items, pred: Pred, stream=None):
        code = dtype_code(d_in)
        arr, n = pred.encode(code)
        check(lib().lcpp_partition_if(_ptr(temp), _tb(temp), _ptr(d_in), _ptr(d_out), _ptr(d_num_selected_out),
                                      num_items, code, arr, n, _stream(stream)), "If")

    def IfThreeWay(self, temp, d_in, d_first_out, d_second_out, d_unselected_out, d_num_selected_out, num_items,
                   select_first: Pred, select_second: Pred, stream=None):
        """The reference's three-way If overload (device_partition.h:157-227);
        d_num_selected_out holds two counts."""
        code = dtype_code(d_in)
        a1, n1 = select_first.encode(code)
        a2, n2 = select_second.encode(code)
        check(lib().lcpp_partition_if_three_way(_ptr(temp), _tb(temp), _ptr(d_in), _ptr(d_first_out),
                                                _ptr(d_second_out), _ptr(d_unselected_out),
                                                _ptr(d_num_selected_out), num_items, code, a1, n1, a2, n2,
                                                _stream(stream)), "IfThreeWay")
