"""Host logic of the distributed sort on CPU: gloo process groups of 2 and 3
ranks run lcpp_b200.distributed's splitter selection and exchange with
numpy stand-ins for the two device operations (local sort, sorted search).
The GPU path is covered by tests/test_distributed_gpu.py."""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from lcpp_b200.distributed import distributed_sort_keys, key_images_np


class NumpyOps:
    """Test-only host versions of the device operations."""

    device = torch.device("cpu")

    def local_sort(self, keys):
        a = keys.numpy()
        return torch.from_numpy(a[np.argsort(key_images_np(a), kind="stable")].copy())

    def search(self, sorted_keys, queries, upper):
        img = key_images_np(sorted_keys.numpy())
        q = queries.astype(np.uint64)
        return torch.from_numpy(np.searchsorted(img, q, side="right" if upper else "left").astype(np.int64))

    def search_bits(self, sorted_keys, queries, upper):
        q = queries.numpy().view(np.uint32 if queries.element_size() == 4 else np.uint64)
        return self.search(sorted_keys, q, upper)

    def merge(self, a, b, out):
        ab = np.concatenate([a.numpy(), b.numpy()])
        out.copy_(torch.from_numpy(ab[np.argsort(key_images_np(ab), kind="stable")].copy()))

    def merge_level(self, pairs):
        for a, b, out in pairs:
            if b is None:
                out.copy_(a)
            else:
                self.merge(a, b, out)

    def empty_like(self, t):
        return torch.empty_like(t)


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
    out, pos = [], 0
    for s in sizes:
        out.append(keys[pos:pos + s].copy())
        pos += s
    return out


def _worker(rank, world, port, case, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        shard = torch.from_numpy(_shards(case, world)[rank])
        res = distributed_sort_keys(shard, dist, NumpyOps())
        q.put((rank, res.numpy().copy()))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
@pytest.mark.parametrize("case", ["uniform", "heavy", "equal", "u64", "i32", "f32", "empty_rank"])
def test_distributed_sort_gloo(world, case):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, case, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    shards = _shards(case, world)
    allk = np.concatenate(shards)
    expect = allk[np.argsort(key_images_np(allk), kind="stable")]
    N = allk.size
    pos = 0
    for r in range(world):
        lo, hi = r * N // world, (r + 1) * N // world
        assert got[r].size == hi - lo  # exact balance, duplicates included
        # same multiset of bit patterns in the same key order; equal keys are
        # interchangeable for a keys-only sort except for +-0.0, compared by image
        # the merge of the received runs keeps equal keys in (source rank,
        # local position) order, so the result is the stable global sort bit
        # for bit (+-0.0 included)
        ubits = np.uint32 if got[r].itemsize == 4 else np.uint64
        np.testing.assert_array_equal(got[r].view(ubits), expect[lo:hi].view(ubits))
        pos = hi
    assert pos == N
