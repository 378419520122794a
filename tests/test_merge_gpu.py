"""GPU parity tests of the merge-path building blocks of the distributed sort
(lcpp_dist_merge_sorted / lcpp_dist_merge_sorted_batch, include/lcpp_b200_dist.h)
against a stable host merge: the keys of `a` come first among equal images,
+-0.0 share one image.  Runs start at every alignment (views at element
offsets 0..3 of a larger buffer, so the kernel's 16-byte-boundary bulk copies
and the plain loads of the ragged ends both run), at the output-tile
boundaries (3840 keys), empty on either side, and with heavy ties."""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
import dist_model  # noqa: E402
from gpu_helpers import NP_TO_CODE, dev, host  # noqa: E402

TILE = 3840
SIZES = [(0, 0), (0, 5), (7, 0), (1, 1), (TILE - 1, 1), (TILE, TILE), (TILE + 1, 3), (3, 2 * TILE + 5),
         (1_000_003, 999_983)]
DTYPES = [np.uint32, np.int32, np.float32, np.uint64, np.int64, np.float64]


def _sorted_run(rng, dtype, n, ties):
    if np.dtype(dtype).kind == "f":
        x = (rng.integers(-3, 4, size=n) if ties else rng.standard_normal(n)).astype(dtype)
        x[::5] = -0.0
        x[1::7] = 0.0
    elif ties:
        x = rng.integers(0, 3, size=n).astype(dtype)
    else:
        info = np.iinfo(dtype)
        x = rng.integers(info.min, info.max, size=n, dtype=dtype, endpoint=True)
    return x[np.argsort(dist_model.images(x), kind="stable")]


def _expected(a, b):
    both = np.concatenate([a, b])
    return both[np.argsort(dist_model.images(both), kind="stable")]


def _placed(x, offset):
    """x on the device at element `offset` of a larger buffer (a view)."""
    buf = torch.empty(x.size + offset + 4, dtype=dev(x[:0]).dtype, device="cuda")
    view = buf[offset:offset + x.size]
    if x.size:
        view.copy_(dev(x))
    return view


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr()) if t.numel() else ctypes.c_void_p(0)


def _merge_batch(lcpp, runs_a, runs_b, outs, code):
    lib = lcpp.lib()
    count = len(runs_a)
    u64 = ctypes.c_uint64
    na = (u64 * count)(*[t.numel() for t in runs_a])
    nb = (u64 * count)(*[t.numel() for t in runs_b])
    need = ctypes.c_size_t()
    lcpp.check(lib.lcpp_dist_merge_batch_temp_bytes(count, na, nb, ctypes.byref(need)), "temp bytes")
    temp = lcpp.alloc_temp(max(need.value, 256))
    pa = (ctypes.c_void_p * count)(*[_ptr(t).value for t in runs_a])
    pb = (ctypes.c_void_p * count)(*[_ptr(t).value for t in runs_b])
    po = (ctypes.c_void_p * count)(*[_ptr(t).value for t in outs])
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    lcpp.check(lib.lcpp_dist_merge_sorted_batch(_ptr(temp), temp.numel(), count, pa, na, pb, nb, po, code, stream),
               "lcpp_dist_merge_sorted_batch")
    assert lcpp.device_status(temp) == lcpp.OK
    return temp


@pytest.mark.parametrize("dtype", DTYPES)
def test_merge_sizes_alignments_ties(lcpp, dtype):
    from lcpp_b200.distributed import merge_sorted
    rng = np.random.default_rng(17)
    for k, (na, nb) in enumerate(SIZES):
        for ties in (False, True):
            a, b = _sorted_run(rng, dtype, na, ties), _sorted_run(rng, dtype, nb, ties)
            off_a, off_b = k % 4, (k * 3 + int(ties)) % 4
            da, db = _placed(a, off_a), _placed(b, off_b)
            out = torch.empty(na + nb, dtype=da.dtype, device="cuda")
            if na + nb:
                merge_sorted(da, db, out)
            got = host(out)
            want = _expected(a, b)
            assert got.tobytes() == want.tobytes(), (dtype, na, nb, ties, off_a, off_b)


@pytest.mark.parametrize("dtype", [np.uint32, np.float32, np.int64])
def test_merge_batch(lcpp, dtype):
    """One launch merging independent pairs of runs of different sizes and
    alignments (one level of the distributed sort's merge tree)."""
    rng = np.random.default_rng(5)
    shapes = [(0, 9), (TILE, TILE - 1), (12_345, 0), (250_001, 70_000), (1, 1), (3 * TILE, 17)]
    runs_a, runs_b, outs, want = [], [], [], []
    for k, (na, nb) in enumerate(shapes):
        a, b = _sorted_run(rng, dtype, na, k % 2 == 1), _sorted_run(rng, dtype, nb, k % 2 == 1)
        runs_a.append(_placed(a, k % 4))
        runs_b.append(_placed(b, (k + 1) % 4))
        outs.append(torch.empty(na + nb, dtype=runs_a[-1].dtype, device="cuda"))
        want.append(_expected(a, b))
    _merge_batch(lcpp, runs_a, runs_b, outs, NP_TO_CODE[np.dtype(dtype)])
    for k, (o, w) in enumerate(zip(outs, want)):
        assert host(o).tobytes() == w.tobytes(), k


def test_merge_2p28_properties(lcpp):
    """Two runs of 2^27 u32 keys: the merge is sorted, and is the sort of the
    concatenation (compared on the device)."""
    from lcpp_b200.distributed import local_sort, merge_sorted
    import lcpp_b200 as L
    n = 1 << 27
    a = torch.empty(n, dtype=torch.uint32, device="cuda")
    b = torch.empty(n, dtype=torch.uint32, device="cuda")
    L.testgen_fill(a, L.GEN_U32_UNIFORM, seed=3)
    L.testgen_fill(b, L.GEN_U32_ZIPF, seed=4)
    sa, sb = local_sort(a), local_sort(b)
    out = torch.empty(2 * n, dtype=torch.uint32, device="cuda")
    merge_sorted(sa, sb, out)
    want = local_sort(torch.cat([a, b]))
    assert torch.equal(out, want)
