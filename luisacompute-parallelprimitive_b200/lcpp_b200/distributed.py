"""Distributed sort / scan / reduce across GPUs (one process per GPU).

No counterpart in the reference, which is single-GPU.  torch.distributed is
the plumbing (NCCL over NVLink on GPUs); the device work is the library's
own kernels.

Sort (keys only), per rank:
  1. local onesweep sort of the rank's keys;
  2. exact global splitters: the global rank positions P_j = floor(j N / G)
     are located by refining a key-image prefix 16 bits per round: every
     rank counts its sorted keys per 16-bit sub-bucket of each boundary's
     current prefix (device binary searches), the counts are all-reduced,
     and the sub-bucket holding P_j extends the prefix; after key_bits/16
     rounds the prefix is the exact boundary key k_j;
  3. keys equal to k_j are split between the ranks below and above the
     boundary in rank order, so every rank receives exactly its share even
     when one key value fills several ranks (heavy hitters);
  4. one all-to-all exchange of the sorted runs (NCCL send / recv);
  5. the G received runs (each sorted) are merged pairwise, ceil(log2 G)
     merge-path levels (lcpp_dist_merge_sorted), instead of a second sort.
Rank r ends with global sorted positions [P_r, P_{r+1}).

Scan and reduce: local pass, one all-gather of per-rank totals, then the
carry-in (exclusive prefix of the totals in rank order) is applied locally;
reduce folds the totals in rank order, so every rank gets the same result.
"""
from __future__ import annotations

import ctypes

import numpy as np

from . import (F32, F64, I32, I64, OP_MAX, OP_MIN, OP_SUM, U32, U64, DeviceRadixSort, DeviceReduce,
               DeviceScan, LcppError, alloc_temp, check, dtype_code, lib)

KEY_BITS = {U32: 32, I32: 32, F32: 32, U64: 64, I64: 64, F64: 64}
SUB_BITS = 16  # prefix bits resolved per splitter round


def key_images_np(keys: np.ndarray) -> np.ndarray:
    """Order-preserving unsigned images of keys (the sort's ascending
    bijection, +-0.0 folded), as uint64 -- host restatement used to build
    search queries from key values."""
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


class GpuOps:
    """Device work of the distributed algorithms, on the current CUDA device."""

    def __init__(self):
        import torch
        self.torch = torch
        self.device = torch.device("cuda", torch.cuda.current_device())
        self._temps = {}
        self.rs = DeviceRadixSort()
        self.launches = 0  # search and merge kernels launched (the sorts are counted by diag timing)

    def _temp(self, key, nbytes):
        t = self._temps.get(key)
        if t is None or t.numel() < nbytes:
            t = alloc_temp(nbytes, self.device)
            self._temps[key] = t
        return t

    def local_sort(self, keys):
        n = keys.numel()
        out = self.torch.empty_like(keys)
        if n:
            temp = self._temp("sort", DeviceRadixSort.GetSortKeysTempStorageBytes(dtype_code(keys), n))
            self.rs.SortKeys(temp, keys, out, n)
        return out

    def search(self, sorted_keys, queries_np: np.ndarray, upper: bool):
        """counts[i] = number of keys with image < (<= when upper) queries[i]."""
        torch = self.torch
        kbits = sorted_keys.element_size() * 8
        q = torch.from_numpy(queries_np.astype(np.uint32 if kbits == 32 else np.uint64)).to(self.device)
        out = torch.empty(q.numel(), dtype=torch.int64, device=self.device)
        if q.numel():
            self.launches += 1
            check(lib().lcpp_dist_search_sorted(
                ctypes.c_void_p(sorted_keys.data_ptr()), sorted_keys.numel(), ctypes.c_void_p(q.data_ptr()),
                q.numel(), int(upper), ctypes.c_void_p(out.data_ptr()), dtype_code(sorted_keys),
                ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)), "lcpp_dist_search_sorted")
        return out

    def merge(self, a, b, out):
        """out[:a.numel() + b.numel()] = stable merge of sorted runs a, b."""
        torch = self.torch
        total = a.numel() + b.numel()
        if total == 0:
            return
        nbytes = ctypes.c_size_t(0)
        check(lib().lcpp_dist_merge_temp_bytes(total, ctypes.byref(nbytes)), "lcpp_dist_merge_temp_bytes")
        temp = self._temp("merge", nbytes.value)
        self.launches += 2
        check(lib().lcpp_dist_merge_sorted(
            ctypes.c_void_p(temp.data_ptr()), temp.numel(), ctypes.c_void_p(a.data_ptr()), a.numel(),
            ctypes.c_void_p(b.data_ptr()), b.numel(), ctypes.c_void_p(out.data_ptr()), dtype_code(a),
            ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)), "lcpp_dist_merge_sorted")

    def empty_like(self, t):
        return self.torch.empty_like(t)


def _all_gather_int64(dist, values, device):
    import torch
    t = torch.tensor(values, dtype=torch.int64, device=device)
    out = [torch.empty_like(t) for _ in range(dist.get_world_size())]
    dist.all_gather(out, t)
    return [o.tolist() for o in out]


def exact_splits(sorted_keys, dist, ops):
    """Split indices of this rank's sorted keys so that rank j receives global
    sorted positions [P_j, P_{j+1}).  Returns (send_counts, recv_counts, idx)
    where idx[r][j] is the split index of rank r before destination j."""
    import torch
    G, r = dist.get_world_size(), dist.get_rank()
    device = ops.device
    n_local = sorted_keys.numel()
    sizes = [v[0] for v in _all_gather_int64(dist, [n_local], device)]
    N = sum(sizes)
    kbits = sorted_keys.element_size() * 8
    P = [j * N // G for j in range(1, G)]
    # Per boundary: image prefix (top `bits` bits) and the global count of
    # keys whose image is below prefix << (kbits - bits).
    prefix = [0] * (G - 1)
    below = [0] * (G - 1)
    bits = 0
    sub = 1 << SUB_BITS
    while bits < kbits:
        shift = kbits - bits - SUB_BITS
        uniq = sorted(set(prefix))
        # query q(p, l) = ((p << 16) | l) << shift for l in [0, 2^16]; the last
        # one (end of the prefix range) is the key count when it would overflow
        base = (np.array(uniq, dtype=np.uint64)[:, None] << np.uint64(SUB_BITS)) + np.arange(sub + 1, dtype=np.uint64)[None, :]
        ends_overflow = np.array([((p + 1) << (SUB_BITS + shift)) >= (1 << kbits) for p in uniq])
        q = base.copy()
        q[:, -1] = np.where(ends_overflow, 0, q[:, -1])
        q = (q << np.uint64(shift)) if shift else q
        counts = ops.search(sorted_keys, q.reshape(-1), upper=False).view(len(uniq), sub + 1)
        if ends_overflow.any():
            counts[torch.from_numpy(np.nonzero(ends_overflow)[0]).to(counts.device), -1] = n_local
        hist = (counts[:, 1:] - counts[:, :-1]).contiguous()
        dist.all_reduce(hist)
        cum = torch.cumsum(hist, dim=1)
        row_of = {p: i for i, p in enumerate(uniq)}
        rows = torch.tensor([row_of[p] for p in prefix], dtype=torch.int64, device=cum.device)
        need = torch.tensor([P[j] - below[j] for j in range(G - 1)], dtype=torch.int64, device=cum.device)
        c = cum[rows]
        # first sub-bucket whose cumulative count exceeds the residual rank
        l = torch.searchsorted(c, need.unsqueeze(1), right=True).squeeze(1)
        below_add = torch.where(l > 0, c.gather(1, (l - 1).clamp_min(0).unsqueeze(1)).squeeze(1), torch.zeros_like(l))
        l_list, add_list = l.tolist(), below_add.tolist()
        for j in range(G - 1):
            prefix[j] = (prefix[j] << SUB_BITS) | int(l_list[j])
            below[j] += int(add_list[j])
        bits += SUB_BITS
    # prefix[j] is now the image k_j of the P_j-th key; below[j] keys are smaller.
    kq = np.array(prefix, dtype=np.uint64)
    lo = ops.search(sorted_keys, kq, upper=False).tolist()
    hi = ops.search(sorted_keys, kq, upper=True).tolist()
    gathered = _all_gather_int64(dist, lo + hi, device)
    idx = [[0] * (G + 1) for _ in range(G)]
    for rr in range(G):
        idx[rr][G] = sizes[rr]
    for j in range(G - 1):
        remaining = P[j] - below[j]  # keys equal to k_j that go below boundary j, in rank order
        for rr in range(G):
            lo_r, hi_r = gathered[rr][j], gathered[rr][G - 1 + j]
            take = min(hi_r - lo_r, remaining)
            idx[rr][j + 1] = lo_r + take
            remaining -= take
        if remaining != 0:
            raise LcppError(7, "distributed splitter selection is inconsistent")
    send = [idx[r][j + 1] - idx[r][j] for j in range(G)]
    recv = [idx[i][r + 1] - idx[i][r] for i in range(G)]
    return send, recv, idx


def _bitcast_for_comm(t):
    """View unsigned tensors as same-width signed ones for collectives."""
    import torch
    if t.dtype == torch.uint32:
        return t.view(torch.int32)
    if t.dtype == torch.uint64:
        return t.view(torch.int64)
    return t


def distributed_sort_keys(keys_local, dist, ops=None):
    """Globally sort the keys held by all ranks; returns this rank's slice of
    the result (global positions [floor(r N / G), floor((r+1) N / G)))."""
    import torch
    ops = ops or GpuOps()
    local = ops.local_sort(keys_local)
    send, recv, _ = exact_splits(local, dist, ops)
    out = torch.empty(sum(recv), dtype=local.dtype, device=local.device)
    dist.all_to_all_single(_bitcast_for_comm(out), _bitcast_for_comm(local), recv, send)
    return merge_runs(out, recv, ops)


def merge_runs(buf, counts, ops):
    """Merge the consecutive sorted runs of `buf` (lengths `counts`, in rank
    order) into one sorted run: pairwise merge-path levels ping-ponging
    between `buf` and one scratch buffer.  Merging adjacent runs with ties
    taken from the left run keeps equal keys in rank order."""
    bounds = [0]
    for c in counts:
        bounds.append(bounds[-1] + int(c))
    runs = [(bounds[i], bounds[i + 1]) for i in range(len(counts))]
    src, dst = buf, None
    while len(runs) > 1:
        if dst is None:
            dst = ops.empty_like(buf)
        nxt = []
        for i in range(0, len(runs), 2):
            if i + 1 == len(runs):
                s0, s1 = runs[i]
                dst[s0:s1].copy_(src[s0:s1])
                nxt.append(runs[i])
                continue
            (a0, a1), (b0, b1) = runs[i], runs[i + 1]
            ops.merge(src[a0:a1], src[b0:b1], dst[a0:b1])
            nxt.append((a0, b1))
        runs = nxt
        src, dst = dst, src
    return src


# ---------------------------------------------------------------------------
# Scan and reduce
# ---------------------------------------------------------------------------
def _fold(op, a, b):
    if op == OP_SUM:
        return a + b
    if op == OP_MIN:
        return min(a, b)
    return max(a, b)


def _np_of(t):
    import torch
    return {torch.int32: np.int32, torch.uint32: np.uint32, torch.float32: np.float32, torch.int64: np.int64,
            torch.uint64: np.uint64, torch.float64: np.float64}[t.dtype]


def _wrap(value, t):
    """A python number as a value of the tensor's dtype: integers wrap
    (two's complement), floats round to the nearest value."""
    npt = np.dtype(_np_of(t))
    if npt.kind in "iu":
        bits = npt.itemsize * 8
        v = int(value) & ((1 << bits) - 1)
        if npt.kind == "i" and v >= (1 << (bits - 1)):
            v -= 1 << bits
        return v
    return float(npt.type(value))


def _local_reduce(x_local, op):
    import torch
    n = x_local.numel()
    out = torch.empty(1, dtype=x_local.dtype, device=x_local.device)
    rd = DeviceReduce()
    temp = alloc_temp(DeviceReduce.GetTempStorageBytes(dtype_code(x_local), n), x_local.device)
    {OP_SUM: rd.Sum, OP_MIN: rd.Min, OP_MAX: rd.Max}[op](temp, x_local, out, n)
    return out


def _gather_scalars(t, dist):
    import torch
    parts = [torch.empty_like(t) for _ in range(dist.get_world_size())]
    dist.all_gather([_bitcast_for_comm(p) for p in parts], _bitcast_for_comm(t))
    return [p.item() for p in parts]


def distributed_reduce(x_local, dist, op=OP_SUM):
    """Reduce over all ranks' items; every rank gets the same value.  Each
    rank reduces locally (DeviceReduce), the per-rank results are
    all-gathered and folded in rank order (deterministic for floats)."""
    vals = _gather_scalars(_local_reduce(x_local, op), dist)
    acc = vals[0]
    for v in vals[1:]:
        acc = _fold(op, acc, v)
    return _wrap(acc, x_local)


def distributed_inclusive_sum(x_local, dist):
    """Inclusive sum over the concatenation of all ranks' items (rank order);
    returns this rank's part.  Local reduce -> all-gather of totals -> local
    InclusiveScanInit with the carry-in (exclusive prefix of earlier ranks'
    totals) as initial value."""
    import torch
    r = dist.get_rank()
    n = x_local.numel()
    code = dtype_code(x_local)
    total = distributed_reduce_totals(x_local, dist)
    carry = 0
    for v in total[:r]:
        carry += v
    out = torch.empty_like(x_local)
    if n:
        sc = DeviceScan()
        temp = alloc_temp(DeviceScan.GetTempStorageBytes(code, n), x_local.device)
        sc.InclusiveScanInit(temp, x_local, out, n, OP_SUM, _wrap(carry, x_local))
    return out


def distributed_reduce_totals(x_local, dist):
    """All ranks' local sums, in rank order."""
    return _gather_scalars(_local_reduce(x_local, OP_SUM), dist)


# ---------------------------------------------------------------------------
# Benchmark (bench.py, N > 1)
# ---------------------------------------------------------------------------
def bench_distributed_sort(n_local, steps, warmup, dist, clock_sampler_cls, peak):
    """Weak-scaling benchmark of distributed_sort_keys: 2^k uniform u32 keys
    per rank (rank r holds elements [r n, (r+1) n) of the seed-0 stream).
    Device time per step is the max over ranks."""
    import torch

    from . import GEN_U32_UNIFORM, KERNEL_SORT_ONESWEEP, diag_timing_enable, diag_timing_read, testgen_fill
    G, r = dist.get_world_size(), dist.get_rank()
    dev = torch.device("cuda", torch.cuda.current_device())
    keys = torch.empty(n_local, dtype=torch.uint32, device=dev)
    testgen_fill(keys, GEN_U32_UNIFORM, seed=0, offset=r * n_local)
    ops = GpuOps()
    for _ in range(warmup):
        out = distributed_sort_keys(keys, dist, ops)
    torch.cuda.synchronize()
    dist.barrier()
    # correctness of the last warm-up result: locally sorted, ordered across ranks
    o = out.view(torch.int32).to(torch.int64) & 0xFFFFFFFF
    ok = bool((o[1:] >= o[:-1]).all()) and out.numel() == n_local
    edges = torch.tensor([o[0].item(), o[-1].item(), int(ok)], dtype=torch.int64, device=dev)
    all_edges = [torch.empty_like(edges) for _ in range(G)]
    dist.all_gather(all_edges, edges)
    e = [t.tolist() for t in all_edges]
    ordered = all(x[2] for x in e) and all(e[i][1] <= e[i + 1][0] for i in range(G - 1))

    props = torch.cuda.get_device_properties(dev)
    bus = getattr(props, "pci_bus_id", None)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    stream = torch.cuda.current_stream()
    with clock_sampler_cls(f"{bus:02x}:00.0" if isinstance(bus, int) else None) as clocks:
        diag_timing_enable(True)
        dist.barrier()
        torch.cuda.synchronize()
        ops.launches = 0
        e0.record(stream)
        for _ in range(steps):
            distributed_sort_keys(keys, dist, ops)
        e1.record(stream)
        torch.cuda.synchronize()
        recs = diag_timing_read()
        diag_timing_enable(False)
        other_launches = ops.launches
    ms = torch.tensor([e0.elapsed_time(e1) / steps], dtype=torch.float64, device=dev)
    dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    ms = ms.item()
    value = G * n_local / (ms * 1e-3) / 1e9

    # e2e: pinned host keys -> device, distributed sort, sorted slice -> host
    host_in = torch.empty(n_local, dtype=torch.uint32, pin_memory=True).copy_(keys)
    host_out = torch.empty(n_local, dtype=torch.uint32, pin_memory=True)
    d_in = torch.empty_like(keys)
    k_e2e = max(3, min(steps, 10))

    def e2e_step():
        d_in.copy_(host_in, non_blocking=True)
        res = distributed_sort_keys(d_in, dist, ops)
        host_out[: res.numel()].copy_(res, non_blocking=True)

    e2e_step()
    torch.cuda.synchronize()
    dist.barrier()
    e0.record(stream)
    for _ in range(k_e2e):
        e2e_step()
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = torch.tensor([e0.elapsed_time(e1) / k_e2e], dtype=torch.float64, device=dev)
    dist.all_reduce(e2e_ms, op=dist.ReduceOp.MAX)
    e2e_ms = e2e_ms.item()

    onesweep = [x[1] for x in recs if x[0] == KERNEL_SORT_ONESWEEP]
    avg_pass = sum(onesweep) / max(1, len(onesweep))
    achieved = 8 * n_local / (avg_pass * 1e-3) / 1e9
    peak_gbs, peak_src = peak
    # per GPU in HBM: the local sort (4 passes x 8 B/key + 4 B/key histogram read), the
    # exchange (read + write 8 B/key) and ceil(log2 G) merge levels (8 B/key each);
    # (G-1)/G of the keys cross NVLink in each direction.
    levels = (G - 1).bit_length()
    hbm_bytes = (36 + 8 + 8 * levels) * n_local
    nvlink_bytes = (G - 1) / G * 4 * n_local
    return {
        "metric": "Gkeys/s uint32 SortKeys @2^28", "value": value, "unit": "Gkeys/s", "n_gpus": G,
        "steps": steps, "warmup": warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "u32",
        "data": "synthetic (splitmix64 counter streams; see include/lcpp_b200_testgen.h)",
        "config": {"workload": f"distributed SortKeys u32 uniform, 2^{n_local.bit_length() - 1} keys per GPU "
                               f"(global 2^{(G * n_local).bit_length() - 1})",
                   "items_per_gpu": n_local, "parallelism": f"sort-partitioned over {G} GPUs (NCCL all-to-all)",
                   "algorithm": "local onesweep -> exact 16-bit-refined splitters (2 all-reduce rounds) -> "
                                "all-to-all -> pairwise merge-path merge of the G received runs",
                   "l2": "inputs larger than L2; no flush", "globally_sorted_check": ordered},
        "roofline": {"bound": "hbm", "kernel": "onesweep_kernel (one 8-bit pass)", "achieved": achieved,
                     "peak": peak_gbs, "peak_source": peak_src, "unit": "GB/s", "frac": achieved / peak_gbs,
                     "algorithmic_bytes_per_launch": 8 * n_local, "avg_launch_ms": avg_pass, "traffic": None},
        "op_roofline": {"hbm_bytes_per_gpu": hbm_bytes, "nvlink_bytes_per_gpu": nvlink_bytes,
                        "target_ms": max(hbm_bytes / (peak_gbs * 1e9), nvlink_bytes / 770e9) * 1e3,
                        "frac": max(hbm_bytes / (peak_gbs * 1e9), nvlink_bytes / 770e9) * 1e3 / ms},
        "e2e": {"value": G * n_local / (e2e_ms * 1e-3) / 1e9, "unit": "Gkeys/s",
                "h2d_bytes_per_step": 4 * n_local * G, "d2h_bytes_per_step": 4 * n_local * G, "steps": k_e2e,
                "ms_per_step": e2e_ms},
        "gpu_launches": len(recs) + other_launches, "clocks": clocks.summary(), "cpu_baseline": None,
    }
