"""GPU tests of the distributed sort / scan / reduce C entry points
(include/lcpp_b200_dist.h, through lcpp_b200.distributed): one rank on any
box, and 2, 3, 4 or 8 ranks (one process per GPU) when the box has that
many GPUs, against stable host sorts and numpy prefix sums / folds."""
from __future__ import annotations

import ctypes
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
import torch.distributed as dist  # noqa: E402
import torch.multiprocessing as mp  # noqa: E402

import dist_model  # noqa: E402


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.fixture(scope="module")
def comm1():
    assert torch.cuda.is_available()
    from datetime import timedelta

    from lcpp_b200.distributed import Comm
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{_free_port()}", rank=0, world_size=1,
                            timeout=timedelta(seconds=60), device_id=torch.device("cuda", 0))
    c = Comm(dist)
    yield c
    c.close(dist)
    dist.destroy_process_group()


def _stable(keys: np.ndarray) -> np.ndarray:
    return keys[np.argsort(dist_model.images(keys), kind="stable")]


@pytest.mark.parametrize("dtype", [torch.uint32, torch.int32, torch.float32, torch.uint64, torch.int64,
                                   torch.float64])
def test_single_rank_sort(comm1, lcpp, dtype):
    from lcpp_b200.distributed import distributed_sort_keys
    n = (1 << 20) + 17
    g = torch.Generator(device="cuda").manual_seed(3)
    if dtype.is_floating_point:
        keys = torch.randn(n, dtype=dtype, device="cuda", generator=g)
        keys[::101] = 0.0
        keys[7::103] = -0.0
    else:
        wide = dtype in (torch.uint64, torch.int64)
        signed = torch.randint(-(1 << 62) if wide else -(1 << 31), (1 << 62) if wide else (1 << 31), (n,),
                               dtype=torch.int64 if wide else torch.int32, device="cuda", generator=g)
        signed[::5] = signed[1]  # ties
        keys = signed.view(dtype)
    out, t = distributed_sort_keys(keys, comm1, times=True)
    kh = keys.cpu().numpy()
    ubits = np.uint32 if kh.itemsize == 4 else np.uint64
    np.testing.assert_array_equal(out.cpu().numpy().view(ubits), _stable(kh).view(ubits))
    assert t["total_ms"] > 0 and t["local_sort_ms"] > 0


def test_single_rank_scan_reduce(comm1, lcpp):
    from lcpp_b200.distributed import distributed_exclusive_sum, distributed_inclusive_sum, distributed_reduce
    n = 1_000_003
    x = torch.empty(n, dtype=torch.int32, device="cuda")
    lcpp.testgen_fill(x, lcpp.GEN_I32_SCAN, seed=3)
    xh = x.cpu().numpy()
    inc = np.cumsum(xh.astype(np.int64)).astype(np.int32)
    np.testing.assert_array_equal(distributed_inclusive_sum(x, comm1).cpu().numpy(), inc)
    np.testing.assert_array_equal(distributed_exclusive_sum(x, comm1).cpu().numpy(),
                                  np.concatenate([np.zeros(1, np.int32), inc[:-1]]))
    assert int(distributed_reduce(x, comm1, lcpp.OP_SUM, 5).item()) == int(inc[-1]) + 5
    assert int(distributed_reduce(x, comm1, lcpp.OP_MAX).item()) == int(xh.max())
    assert int(distributed_reduce(x, comm1, lcpp.OP_MIN, -5000).item()) == -5000
    f = torch.rand(n, dtype=torch.float32, device="cuda")
    s = float(distributed_reduce(f, comm1, lcpp.OP_SUM).item())
    ref = float(f.double().sum())
    assert abs(s - ref) <= 1e-6 * np.log2(n) * ref


def test_single_rank_argument_errors(comm1, lcpp):
    lib = lcpp.lib()
    n = 1000
    need = ctypes.c_size_t()
    assert lib.lcpp_dist_sort_keys_temp_bytes(comm1.handle, lcpp.U32, n, ctypes.byref(need)) == lcpp.OK
    temp = lcpp.alloc_temp(need.value)
    keys = torch.zeros(n, dtype=torch.uint32, device="cuda")
    vp = ctypes.c_void_p
    assert lib.lcpp_dist_sort_keys(comm1.handle, vp(temp.data_ptr()), need.value - 256, vp(keys.data_ptr()),
                                   vp(keys.data_ptr()), n, lcpp.U32, 0, None, None) == lcpp.ERR_TEMP_TOO_SMALL
    assert lib.lcpp_dist_sort_keys(comm1.handle, vp(temp.data_ptr()), need.value, vp(keys.data_ptr()),
                                   vp(keys.data_ptr()), n, lcpp.U32, 7, None, None) == lcpp.ERR_INVALID_ARG
    # the output may not overlap temp storage
    assert lib.lcpp_dist_sort_keys(comm1.handle, vp(temp.data_ptr()), need.value, vp(keys.data_ptr()),
                                   vp(temp.data_ptr() + 256), n, lcpp.U32, 0, None, None) == lcpp.ERR_INVALID_ARG


# --------------------------------------------------------------- many ranks
def _cases(rank, base):
    """(name, generator, dtype, n) per case; sizes differ by rank."""
    return [("zipf_u32", "GEN_U32_ZIPF", torch.uint32, base + 1000 * rank),
            ("and3_u32", "GEN_U32_AND3", torch.uint32, base // 2 + 77 * rank),
            ("normal_f32", "GEN_F32_NORMAL", torch.float32, base + 13 * rank),
            ("uniform_u64", "GEN_U64_UNIFORM", torch.uint64, base // 4 + 5 * rank)]


def _worker(rank, world, port, base, q):
    import sys
    from datetime import timedelta
    from pathlib import Path
    root = Path(__file__).resolve().parent.parent
    sys.path[:0] = [str(root), str(root / "luisacompute-parallelprimitive_b200")]
    import lcpp_b200 as L
    from lcpp_b200.distributed import (Comm, distributed_exclusive_sum, distributed_inclusive_sum,
                                       distributed_reduce, distributed_sort_keys)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=timedelta(seconds=90), device_id=torch.device("cuda", rank))
    comm = Comm(dist)
    try:
        res = {}
        for name, gen, dt, n in _cases(rank, base):
            keys = torch.empty(n, dtype=dt, device="cuda")
            L.testgen_fill(keys, getattr(L, gen), seed=7, offset=rank * base)
            peer = distributed_sort_keys(keys, comm, exchange="peer")
            nccl = distributed_sort_keys(keys, comm, exchange="nccl")
            pushed = distributed_sort_keys(keys, comm, exchange="copy")
            inplace = keys.clone()
            distributed_sort_keys(inplace, comm, out=inplace)
            pushed_inplace = keys.clone()
            distributed_sort_keys(pushed_inplace, comm, out=pushed_inplace, exchange="copy")
            res[name] = (keys.cpu().numpy(), peer.cpu().numpy(), nccl.cpu().numpy(), inplace.cpu().numpy(),
                         pushed.cpu().numpy(), pushed_inplace.cpu().numpy())
        # consecutive calls with a new temp allocation each time (the peers'
        # mappings are opened again)
        steps = []
        for s in range(3):
            comm._temps.clear()
            k = torch.empty(base // 3 + 11 * rank + s, dtype=torch.uint32, device="cuda")
            L.testgen_fill(k, L.GEN_U32_UNIFORM, seed=100 + s, offset=rank * base)
            steps.append((k.cpu().numpy(), distributed_sort_keys(k, comm).cpu().numpy()))
        x = torch.empty(base + 3 * rank, dtype=torch.int32, device="cuda")
        L.testgen_fill(x, L.GEN_I32_SCAN, seed=3, offset=rank * base)
        scan = (distributed_inclusive_sum(x, comm).cpu().numpy(), distributed_exclusive_sum(x, comm).cpu().numpy(),
                int(distributed_reduce(x, comm, L.OP_SUM, 11).item()),
                int(distributed_reduce(x, comm, L.OP_MIN).item()), int(distributed_reduce(x, comm, L.OP_MAX).item()),
                x.cpu().numpy())
        _, t = distributed_sort_keys(keys, comm, times=True)
        torch.cuda.synchronize()
        q.put((rank, res, steps, scan, t["peer_exchange"]))
        dist.barrier()
    finally:
        comm.close(dist)
        dist.destroy_process_group()


def _collect(q, procs, world, limit_s):
    """Results of all workers; fails as soon as one exits without its
    result (instead of waiting out the whole limit)."""
    import queue
    import time
    got, t0 = {}, time.monotonic()
    while len(got) < world:
        try:
            t = q.get(timeout=5)
            got[t[0]] = t[1:]
        except queue.Empty:
            dead = [p.exitcode for p in procs if p.exitcode not in (None, 0)]
            if dead or time.monotonic() - t0 > limit_s:
                for p in procs:
                    p.kill()
                pytest.fail(f"workers failed (exit codes {dead}) or timed out")
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    return got


@pytest.mark.parametrize("world", [2, 3, 4, 8])
def test_multi_rank(world):
    """One process per GPU: the distributed sort in its three exchange modes
    (peer loads, NCCL send / receive, copy-engine pushes) and in place, 4 key types with rank-dependent sizes, consecutive calls on new
    temp allocations, scan and reduce -- all bit-exact against host
    references."""
    if not torch.cuda.is_available() or torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    base = 1 << 20
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, base, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = _collect(q, procs, world, 600)
    # one host: peer loads with 2-3 ranks, copy-engine pushes from 4 ranks on
    assert all(got[r][3] == (2 if world >= 4 else 1) for r in range(world))
    for name, *_ in _cases(0, base):
        allk = np.concatenate([got[r][0][name][0] for r in range(world)])
        expect = _stable(allk)
        ubits = np.uint32 if allk.itemsize == 4 else np.uint64
        pos = 0
        for r in range(world):
            keys, peer, nccl, inplace, pushed, pushed_inplace = got[r][0][name]
            want = expect[pos:pos + keys.size].view(ubits)
            for arr in (peer, nccl, inplace, pushed, pushed_inplace):
                np.testing.assert_array_equal(arr.view(ubits), want, err_msg=f"{name} rank {r}")
            pos += keys.size
    for s in range(3):
        allk = np.concatenate([got[r][1][s][0] for r in range(world)])
        expect = np.sort(allk)
        pos = 0
        for r in range(world):
            n = got[r][1][s][0].size
            np.testing.assert_array_equal(got[r][1][s][1], expect[pos:pos + n])
            pos += n
    allx = np.concatenate([got[r][2][5] for r in range(world)])
    inc = np.cumsum(allx.astype(np.int64)).astype(np.int32)
    exc = np.concatenate([np.zeros(1, np.int32), inc[:-1]])
    pos = 0
    for r in range(world):
        a, e, ssum, mn, mx, x = got[r][2]
        np.testing.assert_array_equal(a, inc[pos:pos + x.size])
        np.testing.assert_array_equal(e, exc[pos:pos + x.size])
        assert ssum == int(inc[-1]) + 11 and mn == int(allx.min()) and mx == int(allx.max())
        pos += x.size
