"""Host model of the distributed sort, scan and reduce of the library
(lcpp_dist_sort_keys / lcpp_dist_inclusive_sum / lcpp_dist_exclusive_sum /
lcpp_dist_reduce, luisacompute-parallelprimitive_b200/csrc/dist_sort.cu),
step for step, for gloo ranks on the CPU: numpy stands in for the device
kernels and torch.distributed (gloo) carries the collectives the library
issues over NCCL, in the same order.  Test infrastructure only: the tests
run it on 2 and 3 ranks and compare with a stable host sort / numpy scans,
which pins the algorithm (exact splitters, rank-order tie split, merge
order, carry-in) independently of a GPU."""
from __future__ import annotations

import numpy as np
import torch

SUB_BITS = 16
SUB_EDGES = (1 << SUB_BITS) + 1


def images(keys: np.ndarray) -> np.ndarray:
    """Order-preserving unsigned images (the sort's ascending bijection,
    +-0.0 folded) as uint64."""
    bits = keys.dtype.itemsize * 8
    u = keys.view(np.uint32 if bits == 32 else np.uint64).astype(np.uint64)
    high = np.uint64(1 << (bits - 1))
    mask = np.uint64((1 << bits) - 1)
    if keys.dtype.kind == "i":
        return u ^ high
    if keys.dtype.kind == "f":
        t = np.where((u & high) != 0, (~u) & mask, u ^ high)
        return np.where(t == high - np.uint64(1), high, t)
    return u


def _all_gather(dist, arr: np.ndarray):
    """all_gather of a numpy array (unsigned types travel as the signed type
    of the same width: gloo has no unsigned tensors)."""
    arr = np.ascontiguousarray(arr)
    signed = {np.dtype(np.uint32): np.int32, np.dtype(np.uint64): np.int64}.get(arr.dtype)
    t = torch.from_numpy(arr.view(signed) if signed else arr)
    parts = [torch.empty_like(t) for _ in range(dist.get_world_size())]
    dist.all_gather(parts, t)
    return [p.numpy().view(arr.dtype) for p in parts]


def sort_keys(keys: np.ndarray, dist) -> np.ndarray:
    """This rank's part of the distributed stable sort: the keys at global
    sorted positions [n_0 + ... + n_{r-1}, n_0 + ... + n_r)."""
    G, r = dist.get_world_size(), dist.get_rank()
    # 1. local stable sort
    local = keys[np.argsort(images(keys), kind="stable")]
    img = images(local)
    n = local.size
    if G == 1:
        return local
    bits = keys.dtype.itemsize * 8
    # descriptors: every rank's key count
    sizes = [int(v[0]) for v in _all_gather(dist, np.array([n], np.int64))]
    P = [sum(sizes[:j + 1]) for j in range(G - 1)]
    # 2. splitters, 16 bits per round: counts below every sub-bucket edge,
    # all-reduced, then the last edge whose global count is <= P_j
    prefix = [0] * (G - 1)
    below = [0] * (G - 1)
    for rnd in range(bits // SUB_BITS):
        pbits = SUB_BITS * rnd
        sh = bits - SUB_BITS * (rnd + 1)
        L = np.zeros((G - 1, SUB_EDGES), np.int64)
        for j in range(G - 1):
            p = prefix[j]
            q = [((p << SUB_BITS) + e) << sh for e in range(SUB_EDGES)]
            at_end = p == ((1 << pbits) - 1 if pbits else 0)
            if at_end:
                q[-1] = 0
            L[j] = np.searchsorted(img, np.array(q, dtype=np.uint64), side="left")
            if at_end:
                L[j, -1] = n
        t = torch.from_numpy(L)
        dist.all_reduce(t)
        Lg = t.numpy()
        for j in range(G - 1):
            lo = int(np.searchsorted(Lg[j, :SUB_EDGES - 1], P[j], side="right")) - 1
            below[j] = int(Lg[j, lo])
            prefix[j] = (prefix[j] << SUB_BITS) | lo
    # 3. ties with the boundary keys, split in rank order
    k = np.array(prefix, dtype=np.uint64)
    less = np.searchsorted(img, k, side="left").astype(np.int64)
    le = np.searchsorted(img, k, side="right").astype(np.int64)
    ties = np.stack([less, le - less], axis=1)
    tie_all = _all_gather(dist, ties)
    pos = [[0] * (G + 1) for _ in range(G)]
    for s in range(G):
        pos[s][G] = sizes[s]
    for j in range(G - 1):
        need = P[j] - below[j]
        assert sum(int(tie_all[s][j, 0]) for s in range(G)) == below[j]
        for s in range(G):
            lt, eq = int(tie_all[s][j, 0]), int(tie_all[s][j, 1])
            take = min(eq, need)
            need -= take
            pos[s][j + 1] = lt + take
        assert need == 0
    # 4./5. exchange: every rank's sorted keys (padded to the largest), then
    # this rank's segment of each
    width = max(sizes)
    pad = np.zeros(width, local.dtype)
    pad[:n] = local
    gathered = _all_gather(dist, pad.view(np.uint32 if local.itemsize == 4 else np.uint64))
    runs = [gathered[s][pos[s][r]:pos[s][r + 1]].view(local.dtype) for s in range(G)]
    # 6. merge, ties from the lower rank's run first
    cat = np.concatenate(runs)
    return cat[np.argsort(images(cat), kind="stable")]


def _wrap_sum(x: np.ndarray):
    if x.dtype.kind in "iu":
        return x.astype(np.uint64).sum(dtype=np.uint64).astype(x.dtype) if x.size else x.dtype.type(0)
    return x.sum(dtype=x.dtype)


def _cumsum(x: np.ndarray, init):
    if x.dtype.kind in "iu":
        u = np.cumsum(x.astype(np.uint64), dtype=np.uint64) + np.uint64(int(init) % (1 << 64))
        return u.astype(x.dtype)
    return np.cumsum(np.concatenate([[x.dtype.type(init)], x]), dtype=x.dtype)[1:]


def scan(x: np.ndarray, dist, exclusive: bool) -> np.ndarray:
    """This rank's part of the inclusive / exclusive sum over all ranks'
    items: local total, all-gather, carry = totals of lower ranks in rank
    order, local scan from the carry."""
    r = dist.get_rank()
    totals = _all_gather(dist, np.array([_wrap_sum(x)], x.dtype))
    carry = x.dtype.type(0)
    for s in range(r):
        carry = _wrap_sum(np.array([carry, totals[s][0]], x.dtype))
    inc = _cumsum(x, carry)
    if not exclusive:
        return inc
    out = np.empty_like(x)
    if x.size:
        out[0] = carry
        out[1:] = inc[:-1]
    return out


def reduce(x: np.ndarray, dist, op: str, init):
    """The value every rank gets: init (op) the per-rank results in rank
    order (each computed from the operator's identity)."""
    if op == "sum":
        part = _wrap_sum(x)
    elif op == "min":
        part = x.min() if x.size else (np.finfo(x.dtype).max if x.dtype.kind == "f" else np.iinfo(x.dtype).max)
    else:
        part = x.max() if x.size else (np.finfo(x.dtype).min if x.dtype.kind == "f" else np.iinfo(x.dtype).min)
    parts = _all_gather(dist, np.array([part], x.dtype))
    acc = x.dtype.type(init)
    for p in parts:
        v = p[0]
        if op == "sum":
            acc = _wrap_sum(np.array([acc, v], x.dtype))
        elif op == "min":
            acc = v if v < acc else acc
        else:
            acc = v if acc < v else acc
    return acc
