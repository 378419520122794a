"""Failure detection on the GPU without a fault: a bounded device wait that
nothing satisfies runs out, is reported through the error word, and the
context stays usable."""
from __future__ import annotations

import ctypes
import time

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def test_wait_timeout_is_reported_and_context_survives(lcpp, oracle):
    temp = lcpp.alloc_temp(256)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    t0 = time.perf_counter()
    assert lcpp.lib().lcpp_diag_wait_timeout_probe(ctypes.c_void_p(temp.data_ptr()), 256, 50_000_000,
                                                   stream) == lcpp.OK
    assert lcpp.device_status(temp) == lcpp.ERR_LOOKBACK_TIMEOUT
    assert time.perf_counter() - t0 >= 0.05  # the wait ran to its limit
    # the context is still usable: a sort right after is correct and clean
    n = 1 << 20
    keys = torch.empty(n, dtype=torch.uint32, device="cuda")
    lcpp.testgen_fill(keys, lcpp.GEN_U32_UNIFORM, seed=2)
    out = torch.empty_like(keys)
    st = lcpp.alloc_temp(lcpp.DeviceRadixSort.GetSortKeysTempStorageBytes(lcpp.U32, n))
    lcpp.DeviceRadixSort().SortKeys(st, keys, out, n)
    assert lcpp.device_status(st) == lcpp.OK
    np.testing.assert_array_equal(out.cpu().numpy(), np.sort(keys.cpu().numpy()))


def test_wait_timeout_probe_rejects_misuse(lcpp):
    L = lcpp.lib()
    temp = lcpp.alloc_temp(256)
    p = ctypes.c_void_p(temp.data_ptr())
    assert L.lcpp_diag_wait_timeout_probe(p, 255, 1000, None) == lcpp.ERR_INVALID_ARG
    assert L.lcpp_diag_wait_timeout_probe(p, 256, 5_000_000_000, None) == lcpp.ERR_INVALID_ARG  # above 4 s
    assert L.lcpp_diag_wait_timeout_probe(None, 256, 1000, None) == lcpp.ERR_INVALID_ARG
