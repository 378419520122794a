"""The distributed sort, scan and reduce algorithms on the CPU: gloo process
groups of 2 and 3 ranks run the host model of lcpp_dist_sort_keys /
lcpp_dist_inclusive_sum / lcpp_dist_exclusive_sum / lcpp_dist_reduce
(tests/dist_model.py: the library's steps and collectives, numpy for the
device work), against a stable host sort of all ranks' keys and numpy
prefix sums / folds.  The device path is covered by
tests/test_distributed_gpu.py."""
from __future__ import annotations

import os
import queue
import socket
import time

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import dist_model


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _shards(case, world):
    rng = np.random.default_rng(11)
    sizes = [1000 + 37 * r for r in range(world)]
    if case == "empty_rank":
        sizes[0] = 0
    total = sum(sizes)
    if case in ("uniform", "empty_rank"):
        keys = rng.integers(0, 2**32, total, dtype=np.uint64).astype(np.uint32)
    elif case == "heavy":
        keys = rng.integers(0, 2**32, total, dtype=np.uint64).astype(np.uint32)
        keys[rng.random(total) < 0.6] = 0x9E3779B9  # one value fills more than one rank
    elif case == "equal":
        keys = np.full(total, 7, dtype=np.uint32)
    elif case == "u64":
        keys = rng.integers(0, 2**63, total, dtype=np.uint64) * np.uint64(2) + np.uint64(1)
        keys[::5] = keys[3]
    elif case == "i32":
        keys = rng.integers(-2**31, 2**31, total, dtype=np.int64).astype(np.int32)
        keys[::7] = -5
    elif case == "f32":
        keys = rng.standard_normal(total).astype(np.float32)
        keys[::11] = 0.0
        keys[5::13] = -0.0
    elif case == "top":  # keys at the very top of the range (last sub-bucket edges)
        keys = (np.uint32(0xFFFFFFFF) - rng.integers(0, 3, total, dtype=np.uint64).astype(np.uint32))
    out, pos = [], 0
    for s in sizes:
        out.append(keys[pos:pos + s].copy())
        pos += s
    return out


def _scan_shards(dtype, world):
    rng = np.random.default_rng(5)
    sizes = [2000 + 101 * r for r in range(world)]
    sizes[-1] = 0 if world > 2 else sizes[-1]  # an empty rank
    if np.dtype(dtype).kind == "f":
        x = rng.random(sum(sizes)).astype(dtype)
    else:
        x = rng.integers(-1000, 1001, sum(sizes)).astype(dtype)
        x[::97] = np.iinfo(dtype).max  # sums wrap
    out, pos = [], 0
    for s in sizes:
        out.append(x[pos:pos + s].copy())
        pos += s
    return out


def _worker(rank, world, port, kind, case, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        if kind == "sort":
            res = dist_model.sort_keys(_shards(case, world)[rank], dist)
        else:
            x = _scan_shards(np.dtype(case), world)[rank]
            res = (dist_model.scan(x, dist, False), dist_model.scan(x, dist, True),
                   dist_model.reduce(x, dist, "sum", 0), dist_model.reduce(x, dist, "min", 7),
                   dist_model.reduce(x, dist, "max", 0 if x.dtype.kind == "u" else -3))
        q.put((rank, res))
    finally:
        dist.destroy_process_group()


def _run(world, kind, case):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, kind, case, q)) for r in range(world)]
    for p in procs:
        p.start()
    got, t0 = {}, time.monotonic()
    while len(got) < world:  # fail as soon as a worker exits without its result
        try:
            r, res = q.get(timeout=2)
            got[r] = res
        except queue.Empty:
            dead = [p.exitcode for p in procs if p.exitcode not in (None, 0)]
            if dead or time.monotonic() - t0 > 120:
                for p in procs:
                    p.kill()
                pytest.fail(f"workers failed (exit codes {dead}) or timed out")
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    return got


@pytest.mark.parametrize("world", [2, 3])
@pytest.mark.parametrize("case", ["uniform", "heavy", "equal", "u64", "i32", "f32", "empty_rank", "top"])
def test_distributed_sort_gloo(world, case):
    got = _run(world, "sort", case)
    shards = _shards(case, world)
    allk = np.concatenate(shards)
    expect = allk[np.argsort(dist_model.images(allk), kind="stable")]
    pos = 0
    ubits = np.uint32 if allk.itemsize == 4 else np.uint64
    for r in range(world):
        n = shards[r].size
        assert got[r].size == n  # every rank gets as many keys as it passed
        # the stable global sort, bit for bit (+-0.0 in input order)
        np.testing.assert_array_equal(got[r].view(ubits), expect[pos:pos + n].view(ubits))
        pos += n
    assert pos == allk.size


@pytest.mark.parametrize("world", [2, 3])
@pytest.mark.parametrize("dtype", ["int32", "uint64", "float32"])
def test_distributed_scan_reduce_gloo(world, dtype):
    got = _run(world, "scan", dtype)
    shards = _scan_shards(np.dtype(dtype), world)
    allx = np.concatenate(shards)
    if allx.dtype.kind == "f":
        inc = np.cumsum(allx.astype(np.float64))
        tol = 1e-6 * np.log2(max(allx.size, 2))
    else:
        inc = np.cumsum(allx.astype(np.uint64), dtype=np.uint64).astype(allx.dtype)  # wraps
    exc = np.concatenate([np.zeros(1, inc.dtype), inc[:-1]])
    pos = 0
    for r in range(world):
        n = shards[r].size
        a, e, s, mn, mx = got[r]
        if allx.dtype.kind == "f":
            np.testing.assert_allclose(a.astype(np.float64), inc[pos:pos + n], rtol=tol, atol=tol)
            np.testing.assert_allclose(e.astype(np.float64), exc[pos:pos + n], rtol=tol, atol=tol)
            assert abs(float(s) - allx.astype(np.float64).sum()) <= tol * max(1.0, abs(float(s)))
        else:
            np.testing.assert_array_equal(a, inc[pos:pos + n])
            np.testing.assert_array_equal(e, exc[pos:pos + n])
            assert s == inc[-1]
        assert mn == min(allx.min(), allx.dtype.type(7))
        assert mx == max(allx.max(), allx.dtype.type(0 if allx.dtype.kind == "u" else -3))
        pos += n
    # every rank gets the same reductions
    assert len({(float(got[r][2]), float(got[r][3]), float(got[r][4])) for r in range(world)}) == 1
