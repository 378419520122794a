"""GPU test of lcpp_scan_inclusive_sum_noalloc, the InclusiveSum entry point
for callers that cannot allocate device memory (it keeps its scratch in a
fixed array inside the library).  It must give what the regular
lcpp_scan_inclusive_sum gives, call after call, since every call reuses the
same array, and what an independent prefix sum gives (numpy's cumsum, or
torch's on the device at the largest size).  Kept in its own file, named to
be collected last."""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def _regular(lcpp, x):
    out = torch.empty_like(x)
    temp = lcpp.alloc_temp(lcpp.DeviceScan.GetTempStorageBytes(lcpp.dtype_code(x), x.numel()))
    lcpp.check(lcpp.lib().lcpp_scan_inclusive_sum(ctypes.c_void_p(temp.data_ptr()), temp.numel(),
                                                  ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(out.data_ptr()),
                                                  x.numel(), lcpp.dtype_code(x),
                                                  ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)),
               "lcpp_scan_inclusive_sum")
    return out


def _noalloc(lcpp, x, n=None):
    out = torch.empty_like(x)
    status = lcpp.lib().lcpp_scan_inclusive_sum_noalloc(
        ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(out.data_ptr()), x.numel() if n is None else n,
        lcpp.dtype_code(x), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    return status, out


@pytest.mark.parametrize("dtype,n", [(torch.int32, 1), (torch.int32, 1_000_003), (torch.int32, 1 << 26),
                                     (torch.float32, 262_147), (torch.int64, 3_000_001),
                                     (torch.float64, 65_537)])
def test_noalloc_matches_regular_twice(lcpp, dtype, n):
    assert torch.cuda.is_available()
    g = torch.Generator(device="cuda").manual_seed(n)
    if dtype.is_floating_point:
        x = torch.rand(n, dtype=dtype, device="cuda", generator=g)
    else:
        x = torch.randint(-1000, 1001, (n,), dtype=dtype, device="cuda", generator=g)
    ref = _regular(lcpp, x)
    xh = x.cpu().numpy()
    if dtype.is_floating_point:
        indep = np.cumsum(xh.astype(np.float64))
    else:  # two's-complement wrap in the item type, as the reference's integer scan
        indep = np.cumsum(xh.astype(np.int64)).astype(xh.dtype)
    for _ in range(2):  # the second call starts from the first call's scratch contents
        status, out = _noalloc(lcpp, x)
        assert status == lcpp.OK
        torch.cuda.synchronize()
        oh = out.cpu().numpy()
        if dtype.is_floating_point:
            # the calls may associate floating-point partial sums differently
            tol = 1e-5 if dtype == torch.float32 else 1e-12
            rel = ((out.double() - ref.double()).abs() / ref.double().abs().clamp_min(1.0)).max().item()
            assert rel < tol
            rel = np.max(np.abs(oh.astype(np.float64) - indep) / np.maximum(np.abs(indep), 1.0))
            assert rel < tol
        else:
            assert torch.equal(out, ref)
            np.testing.assert_array_equal(oh, indep)


def test_noalloc_at_the_four_byte_limit(lcpp):
    """1,075,707,904 int32 items, the most the fixed array holds, twice in a
    row, against torch.cumsum on the device (exact)."""
    n = 1_075_707_904
    x = torch.randint(-1000, 1001, (n,), dtype=torch.int32, device="cuda",
                      generator=torch.Generator(device="cuda").manual_seed(5))
    expect = torch.cumsum(x, 0, dtype=torch.int64).to(torch.int32)
    for _ in range(2):
        status, out = _noalloc(lcpp, x)
        assert status == lcpp.OK
        assert torch.equal(out, expect)
        del out


def test_noalloc_rejects_too_many_items(lcpp):
    x = torch.zeros(4, dtype=torch.int32, device="cuda")
    status, _ = _noalloc(lcpp, x, n=1_075_707_904 + 1)
    assert status == lcpp.ERR_TEMP_TOO_SMALL
    status, _ = _noalloc(lcpp, torch.zeros(4, dtype=torch.int64, device="cuda"), n=215_089_152 + 1)
    assert status == lcpp.ERR_TEMP_TOO_SMALL
    status, _ = _noalloc(lcpp, x, n=0)
    assert status == lcpp.OK
