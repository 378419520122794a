"""Failure detection of the distributed sort on the host (gloo ranks on the
CPU): a rank that dies before its collectives, or never joins them, makes
the other ranks end with an error within the process-group timeout instead
of hanging."""
from __future__ import annotations

import os
import socket
import time
from datetime import timedelta

import numpy as np
import pytest

torch = pytest.importorskip("torch")
import torch.distributed as dist  # noqa: E402
import torch.multiprocessing as mp  # noqa: E402

import dist_model  # noqa: E402


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, port, mode, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=2, timeout=timedelta(seconds=4))
    if rank == 1:
        if mode == "dies":
            os._exit(3)  # gone before any collective of the sort
        time.sleep(12)   # alive, but never joins the sort's collectives
        os._exit(0)
    t0 = time.perf_counter()
    try:
        dist_model.sort_keys(np.arange(1000, dtype=np.uint32), dist)
        q.put(("finished", time.perf_counter() - t0))
    except Exception as e:  # noqa: BLE001 - any error is the expected outcome
        q.put(("error", time.perf_counter() - t0, type(e).__name__))
    # flush the queue's feeder thread before leaving without the process
    # group's teardown (which would wait for the missing peer)
    q.close()
    q.join_thread()
    os._exit(0)


@pytest.mark.parametrize("mode", ["dies", "never_joins"])
def test_peer_failure_ends_with_an_error(mode):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, port, mode, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = q.get(timeout=90)
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    assert res[0] == "error", res
    assert res[1] < 60
