"""GPU tests of the distributed sort / scan / reduce (lcpp_b200.distributed)
over NCCL: one rank in-process on any box, and two ranks (one per GPU) when
the box has two or more GPUs."""
from __future__ import annotations

import os
import socket
import zlib

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
import torch.distributed as dist  # noqa: E402
import torch.multiprocessing as mp  # noqa: E402


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.fixture(scope="module")
def pg1():
    assert torch.cuda.is_available()
    from datetime import timedelta
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{_free_port()}", rank=0, world_size=1,
                            timeout=timedelta(seconds=60))
    yield dist
    dist.destroy_process_group()


def test_single_rank_sort_equals_local(pg1, lcpp, oracle):
    from lcpp_b200.distributed import distributed_sort_keys
    n = (1 << 22) + 17
    keys = torch.empty(n, dtype=torch.uint32, device="cuda")
    lcpp.testgen_fill(keys, lcpp.GEN_U32_ZIPF, seed=7)
    out = distributed_sort_keys(keys, pg1)
    np.testing.assert_array_equal(out.cpu().numpy(), np.sort(keys.cpu().numpy()))


def test_single_rank_scan_reduce(pg1, lcpp, oracle):
    from lcpp_b200.distributed import distributed_inclusive_sum, distributed_reduce
    n = 1_000_003
    x = torch.empty(n, dtype=torch.int32, device="cuda")
    lcpp.testgen_fill(x, lcpp.GEN_I32_SCAN, seed=3)
    xh = x.cpu().numpy()
    np.testing.assert_array_equal(distributed_inclusive_sum(x, pg1).cpu().numpy(), oracle.scan(xh, "inclusive"))
    assert distributed_reduce(x, pg1, lcpp.OP_SUM) == int(oracle.reduce(xh, oracle.OP_SUM, 0))
    assert distributed_reduce(x, pg1, lcpp.OP_MAX) == int(xh.max())


def _worker(rank, world, port, n, q):
    import sys
    from pathlib import Path
    root = Path(__file__).resolve().parent.parent
    sys.path[:0] = [str(root), str(root / "luisacompute-parallelprimitive_b200")]
    import lcpp_b200 as L
    from lcpp_b200.distributed import GpuOps, distributed_inclusive_sum, distributed_reduce, distributed_sort_keys
    torch.cuda.set_device(rank)
    from datetime import timedelta
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=timedelta(seconds=60), device_id=torch.device("cuda", rank))
    try:
        keys = torch.empty(n, dtype=torch.uint32, device="cuda")
        L.testgen_fill(keys, L.GEN_U32_ZIPF, seed=7, offset=rank * n)
        out = distributed_sort_keys(keys, dist)
        out_nccl = distributed_sort_keys(keys, dist, exchange="nccl")
        # one GpuOps over several steps: the exchange buffers alternate and
        # are reused; every step's keys differ (and the sizes differ by rank)
        ops = GpuOps()
        steps = []
        for s in range(3):
            m = n // 2 + 1000 * rank + 7 * s
            k = torch.empty(m, dtype=torch.uint32, device="cuda")
            L.testgen_fill(k, L.GEN_U32_UNIFORM if s != 1 else L.GEN_U32_AND3, seed=100 + s, offset=rank * n)
            steps.append((k.cpu().numpy(), distributed_sort_keys(k, dist, ops).cpu().numpy()))
        ops.close(dist)
        x = torch.empty(n, dtype=torch.int32, device="cuda")
        L.testgen_fill(x, L.GEN_I32_SCAN, seed=3, offset=rank * n)
        scan = distributed_inclusive_sum(x, dist)
        red = distributed_reduce(x, dist, L.OP_SUM)
        torch.cuda.synchronize()
        q.put((rank, out.cpu().numpy(), keys.cpu().numpy(), scan.cpu().numpy(), x.cpu().numpy(), red,
               out_nccl.cpu().numpy(), steps))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3, 4, 8])
def test_multi_rank(world):
    """One process per GPU over NCCL: the distributed sort (peer exchange and
    NCCL all-to-all), repeated calls on one set of exchange buffers, scan and
    reduce, against host references."""
    if not torch.cuda.is_available() or torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    n = 1 << 21
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, n, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = dict((t[0], t[1:]) for t in (q.get(timeout=300) for _ in range(world)))
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    allk = np.concatenate([got[r][1] for r in range(world)])
    expect = np.sort(allk)
    # peer exchange (default on one node) and NCCL all-to-all give the same slices
    np.testing.assert_array_equal(np.concatenate([got[r][0] for r in range(world)]), expect)
    np.testing.assert_array_equal(np.concatenate([got[r][5] for r in range(world)]), expect)
    for s in range(3):
        allk = np.concatenate([got[r][6][s][0] for r in range(world)])
        N = allk.size
        for r in range(world):
            np.testing.assert_array_equal(got[r][6][s][1], np.sort(allk)[r * N // world:(r + 1) * N // world])
    allx = np.concatenate([got[r][3] for r in range(world)]).astype(np.int64)
    np.testing.assert_array_equal(np.concatenate([got[r][2] for r in range(world)]).astype(np.int64),
                                  np.cumsum(allx))
    assert all(got[r][4] == int(allx.sum()) for r in range(world))


def _stable_merge_np(a, b):
    from lcpp_b200.distributed import key_images_np
    ab = np.concatenate([a, b])
    return ab[np.argsort(key_images_np(ab), kind="stable")]


def _sorted_run(rng, n, np_dt, case):
    from lcpp_b200.distributed import key_images_np
    if np_dt == np.float32 or np_dt == np.float64:
        x = rng.standard_normal(n).astype(np_dt)
        x[::9] = 0.0
        x[4::9] = -0.0
    elif case == "ties":
        x = rng.integers(0, 4, n).astype(np_dt)
    else:
        info = np.iinfo(np_dt)
        x = rng.integers(info.min, info.max, n, dtype=np_dt, endpoint=True)
    return x[np.argsort(key_images_np(x), kind="stable")]


@pytest.mark.parametrize("np_dt", [np.uint32, np.int32, np.float32, np.uint64, np.int64, np.float64])
@pytest.mark.parametrize("sizes", [(0, 0), (0, 5), (7, 0), (1, 1), (3840, 3840), (3839, 3841),
                                   (100_003, 17), (1 << 20, (1 << 20) + 3), (1 << 22, 999_999)])
@pytest.mark.parametrize("case", ["uniform", "ties"])
def test_merge_sorted_parity(np_dt, sizes, case):
    """lcpp_dist_merge_sorted against a stable host merge, bit for bit (ties:
    keys of the first run first; +-0.0 compare equal and keep their bits)."""
    from lcpp_b200.distributed import GpuOps
    rng = np.random.default_rng(zlib.crc32(repr((np.dtype(np_dt).str, sizes, case)).encode()))
    a = _sorted_run(rng, sizes[0], np_dt, case)
    b = _sorted_run(rng, sizes[1], np_dt, case)
    ops = GpuOps()
    ta, tb = torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda()
    out = torch.full((a.size + b.size,), 0x5A, dtype=ta.dtype, device="cuda") if a.size + b.size else \
        torch.empty(0, dtype=ta.dtype, device="cuda")
    ops.merge(ta, tb, out)
    ub = np.uint32 if np.dtype(np_dt).itemsize == 4 else np.uint64
    np.testing.assert_array_equal(out.cpu().numpy().view(ub), _stable_merge_np(a, b).view(ub))


def test_merge_sorted_rejects_misuse(lcpp):
    import ctypes
    L = lcpp.lib()
    need = ctypes.c_size_t(0)
    assert L.lcpp_dist_merge_temp_bytes(10_000, ctypes.byref(need)) == lcpp.OK and need.value > 0
    a = torch.zeros(5000, dtype=torch.int32, device="cuda")
    b = torch.zeros(5000, dtype=torch.int32, device="cuda")
    out = torch.empty(10_000, dtype=torch.int32, device="cuda")
    temp = lcpp.alloc_temp(need.value)
    p = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    assert L.lcpp_dist_merge_sorted(p(temp), need.value - 1, p(a), 5000, p(b), 5000, p(out), lcpp.I32,
                                    None) == lcpp.ERR_TEMP_TOO_SMALL
    assert L.lcpp_dist_merge_sorted(p(temp), need.value, p(a), 5000, p(b), 5000, p(out), 99,
                                    None) == lcpp.ERR_UNSUPPORTED_DTYPE
    assert L.lcpp_dist_merge_sorted(p(temp), need.value, None, 5000, p(b), 5000, p(out), lcpp.I32,
                                    None) == lcpp.ERR_INVALID_ARG


@pytest.mark.parametrize("counts", [[5], [3, 0, 4], [1 << 20, 77, (1 << 19) + 1, 0, 4096, 12345, 1 << 18],
                                    [1000] * 8])
def test_merge_runs_tree(counts):
    """The pairwise merge tree over G received runs equals the stable sort of
    their concatenation (equal keys in run order)."""
    from lcpp_b200.distributed import GpuOps, key_images_np, merge_runs
    rng = np.random.default_rng(len(counts))
    runs = [_sorted_run(rng, c, np.uint32, "ties" if i % 2 else "uniform") for i, c in enumerate(counts)]
    allk = np.concatenate(runs)
    res = merge_runs(torch.from_numpy(allk).cuda(), counts, GpuOps())
    np.testing.assert_array_equal(res.cpu().numpy(), allk[np.argsort(key_images_np(allk), kind="stable")])


def test_merge_batch_parity():
    """One batched merge level (lcpp_dist_merge_sorted_batch): independent
    pairs of different sizes, empty ones and a copy (empty b) included."""
    from lcpp_b200.distributed import GpuOps
    rng = np.random.default_rng(5)
    sizes = [(1000, 3), (0, 0), (4096, 0), (0, 77), (300_000, 123_457), (3840, 3840), (5, 100_000)]
    ops = GpuOps()
    pairs, expect = [], []
    for na, nb in sizes:
        a = _sorted_run(rng, na, np.uint32, "ties")
        b = _sorted_run(rng, nb, np.uint32, "uniform")
        ta, tb = torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda()
        out = torch.full((na + nb,), 0xAB, dtype=torch.uint32, device="cuda")
        pairs.append((ta, tb if nb else None, out))
        expect.append(_stable_merge_np(a, b))
    ops.merge_level(pairs)
    for (_, _, out), e in zip(pairs, expect):
        np.testing.assert_array_equal(out.cpu().numpy(), e)
