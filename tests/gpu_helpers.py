"""Helpers shared by the GPU parity tests (device buffers via torch; the
library is always called through its C ABI)."""
from __future__ import annotations

import numpy as np
import torch

import lcpp_b200 as L

NP_TO_CODE = {np.dtype(np.uint32): L.U32, np.dtype(np.int32): L.I32, np.dtype(np.float32): L.F32,
              np.dtype(np.uint64): L.U64, np.dtype(np.int64): L.I64, np.dtype(np.float64): L.F64}


def dev(a: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def host(t: torch.Tensor) -> np.ndarray:
    return t.cpu().numpy()


def empty_like_np(a: np.ndarray) -> torch.Tensor:
    return torch.empty(a.shape, dtype=torch.from_numpy(a[:0]).dtype, device="cuda")


def gpu_sort(keys: np.ndarray, values: np.ndarray | None = None, begin_bit=0, end_bit=None,
             descending=False):
    """Copy-API sort through the C ABI; returns numpy outputs."""
    n = keys.size
    rs = L.DeviceRadixSort()
    kin, kout = dev(keys), empty_like_np(keys)
    kd = NP_TO_CODE[keys.dtype]
    if values is None:
        temp = L.alloc_temp(rs.GetSortKeysTempStorageBytes(kd, n))
        (rs.SortKeysDescending if descending else rs.SortKeys)(temp, kin, kout, n, begin_bit, end_bit)
        assert L.device_status(temp) == L.OK
        return host(kout)
    vin, vout = dev(values), empty_like_np(values)
    temp = L.alloc_temp(rs.GetSortPairsTempStorageBytes(kd, NP_TO_CODE[values.dtype], n))
    (rs.SortPairsDescending if descending else rs.SortPairs)(temp, kin, kout, vin, vout, n, begin_bit,
                                                             end_bit)
    assert L.device_status(temp) == L.OK
    return host(kout), host(vout)


def transformed_key_u64(keys: torch.Tensor, kind: str, bits: int) -> torch.Tensor:
    """Order-preserving key bits as int64 (for sortedness checks on the device).
    For 64-bit keys the result is the transformed key XOR the high bit, so
    that signed int64 comparison orders it like the unsigned value."""
    if bits == 32:
        u = keys.view(torch.int32).to(torch.int64) & 0xFFFFFFFF
        high = 1 << 31
        if kind == "i":
            t = u ^ high
        elif kind == "f":
            neg = (u & high) != 0
            t = torch.where(neg, (~u) & 0xFFFFFFFF, u ^ high)
            t = torch.where((u & 0x7FFFFFFF) == 0, torch.full_like(t, high), t)
        else:
            t = u
        return t
    s = keys.view(torch.int64)
    sign = torch.iinfo(torch.int64).min
    if kind == "i":
        return s
    if kind == "f":
        neg = s < 0
        t = torch.where(neg, ~s, s ^ sign)  # unsigned order of the transformed key
        t = t ^ sign  # map unsigned order onto signed int64
        zero = (s & 0x7FFFFFFFFFFFFFFF) == 0
        return torch.where(zero, torch.zeros_like(t), t)
    return s ^ sign
