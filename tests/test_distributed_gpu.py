"""GPU tests of the distributed sort / scan / reduce (lcpp_b200.distributed)
over NCCL: one rank in-process on any box, and two ranks (one per GPU) when
the box has two or more GPUs."""
from __future__ import annotations

import os
import socket

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
    from lcpp_b200.distributed import distributed_inclusive_sum, distributed_reduce, distributed_sort_keys
    torch.cuda.set_device(rank)
    from datetime import timedelta
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=timedelta(seconds=60), device_id=torch.device("cuda", rank))
    try:
        keys = torch.empty(n, dtype=torch.uint32, device="cuda")
        L.testgen_fill(keys, L.GEN_U32_ZIPF, seed=7, offset=rank * n)
        out = distributed_sort_keys(keys, dist)
        x = torch.empty(n, dtype=torch.int32, device="cuda")
        L.testgen_fill(x, L.GEN_I32_SCAN, seed=3, offset=rank * n)
        scan = distributed_inclusive_sum(x, dist)
        red = distributed_reduce(x, dist, L.OP_SUM)
        torch.cuda.synchronize()
        q.put((rank, out.cpu().numpy(), keys.cpu().numpy(), scan.cpu().numpy(), x.cpu().numpy(), red))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_two_ranks_nccl():
    world, n = 2, 1 << 21
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
    np.testing.assert_array_equal(np.concatenate([got[r][0] for r in range(world)]), np.sort(allk))
    allx = np.concatenate([got[r][3] for r in range(world)]).astype(np.int64)
    np.testing.assert_array_equal(np.concatenate([got[r][2] for r in range(world)]).astype(np.int64),
                                  np.cumsum(allx))
    assert got[0][4] == got[1][4] == int(allx.sum())
