"""Distributed sort / scan / reduce across GPUs, one process per GPU.

No counterpart in the reference, which is single-GPU.  This module is the
Python front end of the library's distributed C entry points
(include/lcpp_b200_dist.h): `Comm` wraps an lcpp_comm (an NCCL communicator
of the library's own), whose ID torch.distributed (any backend) hands from
rank 0 to the other ranks; every exchange, collective and kernel of the
calls below is the library's.

  distributed_sort_keys      lcpp_dist_sort_keys: rank r receives the keys at
                             global sorted positions [n_0 + ... + n_{r-1},
                             n_0 + ... + n_r) of the stable sort of all ranks'
                             keys in rank order (as many keys as it passed)
  distributed_inclusive_sum  lcpp_dist_inclusive_sum
  distributed_exclusive_sum  lcpp_dist_exclusive_sum
  distributed_reduce         lcpp_dist_reduce
"""
from __future__ import annotations

import ctypes
import os

from . import DeviceRadixSort, DistSortTimes, OP_MIN, OP_SUM, _host_scalar, alloc_temp, check, dtype_code, lib

EXCHANGE = {"auto": 0, "peer": 1, "nccl": 2, "copy": 3}


def _stream_ptr():
    import torch
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr() if t is not None and t.numel() else 0)


class Comm:
    """An lcpp_comm over the ranks of a torch.distributed process group (one
    process per GPU; the current CUDA device is this rank's GPU).  Creating
    and closing it are collective.  Temp storage of the calls is cached per
    operation, so repeated calls reuse it (and, for the sort, the peers'
    mappings of it)."""

    def __init__(self, dist):
        import torch
        self.rank, self.size = dist.get_rank(), dist.get_world_size()
        self.device = torch.device("cuda", torch.cuda.current_device())
        idb = (ctypes.c_ubyte * 128)()
        if self.rank == 0:
            check(lib().lcpp_comm_unique_id(idb), "lcpp_comm_unique_id")
        obj = [bytes(idb)]
        dist.broadcast_object_list(obj, src=0)
        idb = (ctypes.c_ubyte * 128).from_buffer_copy(obj[0])
        h = ctypes.c_void_p()
        check(lib().lcpp_comm_init(idb, self.size, self.rank, ctypes.byref(h)), "lcpp_comm_init")
        self.handle = h
        self._temps = {}

    def temp(self, key, nbytes):
        t = self._temps.get(key)
        if t is None or t.numel() < nbytes:
            self._temps.pop(key, None)
            t = alloc_temp(nbytes, self.device)
            self._temps[key] = t
        return t

    def close(self, dist=None):
        """Collective: releases the communicator once every rank's calls are
        done (a barrier first when `dist` is given)."""
        import torch
        if self.handle is None:
            return
        torch.cuda.synchronize()
        if dist is not None:
            dist.barrier()
        check(lib().lcpp_comm_destroy(self.handle), "lcpp_comm_destroy")
        self.handle = None
        self._temps.clear()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()
        return False


def distributed_sort_keys(keys, comm: Comm, out=None, exchange: str = "auto", times: bool = False):
    """Stable sort of all ranks' keys (concatenated in rank order); returns
    this rank's part, as many keys as `keys` holds (global positions
    [n_0 + ... + n_{r-1}, n_0 + ... + n_r)).  `out` may be `keys`.  With
    times=True also returns the call's per-phase times (dict)."""
    import torch
    n = keys.numel()
    code = dtype_code(keys)
    if out is None:
        out = torch.empty_like(keys)
    need = ctypes.c_size_t()
    check(lib().lcpp_dist_sort_keys_temp_bytes(comm.handle, code, n, ctypes.byref(need)),
          "lcpp_dist_sort_keys_temp_bytes")
    temp = comm.temp(("sort", code), need.value)
    tm = DistSortTimes() if times else None
    check(lib().lcpp_dist_sort_keys(comm.handle, _ptr(temp), temp.numel(), _ptr(keys), _ptr(out), n, code,
                                    EXCHANGE[exchange], ctypes.byref(tm) if tm is not None else None,
                                    _stream_ptr()), "lcpp_dist_sort_keys")
    if times:
        return out, {f: getattr(tm, f) for f, _ in DistSortTimes._fields_}
    return out


def _scan(x, comm: Comm, out, exclusive: bool):
    import torch
    n = x.numel()
    code = dtype_code(x)
    if out is None:
        out = torch.empty_like(x)
    need = ctypes.c_size_t()
    check(lib().lcpp_dist_scan_temp_bytes(comm.handle, code, n, ctypes.byref(need)), "lcpp_dist_scan_temp_bytes")
    temp = comm.temp(("scan", code), need.value)
    fn = lib().lcpp_dist_exclusive_sum if exclusive else lib().lcpp_dist_inclusive_sum
    check(fn(comm.handle, _ptr(temp), temp.numel(), _ptr(x), _ptr(out), n, code, _stream_ptr()),
          "lcpp_dist_exclusive_sum" if exclusive else "lcpp_dist_inclusive_sum")
    return out


def distributed_inclusive_sum(x, comm: Comm, out=None):
    """Inclusive sum over all ranks' items in rank order; returns this rank's
    part (integer sums wrap)."""
    return _scan(x, comm, out, False)


def distributed_exclusive_sum(x, comm: Comm, out=None):
    """Exclusive sum over all ranks' items in rank order; returns this rank's
    part (the first item of rank 0 gets 0)."""
    return _scan(x, comm, out, True)


def distributed_reduce(x, comm: Comm, op: int = OP_SUM, init=None):
    """Reduce over all ranks' items; every rank gets the same one-element
    tensor: init (op) rank 0's items (op) ... in rank order.  init defaults
    to the operator's identity (0, the type's max for MIN, lowest for MAX)."""
    import torch
    n = x.numel()
    code = dtype_code(x)
    if init is None:
        info = torch.finfo(x.dtype) if x.is_floating_point() else torch.iinfo(x.dtype)
        init = 0 if op == OP_SUM else (info.max if op == OP_MIN else info.min)
    out = torch.empty(1, dtype=x.dtype, device=x.device)
    need = ctypes.c_size_t()
    check(lib().lcpp_dist_reduce_temp_bytes(comm.handle, code, n, ctypes.byref(need)), "lcpp_dist_reduce_temp_bytes")
    temp = comm.temp(("reduce", code), need.value)
    keep, iv = _host_scalar(init, code)
    check(lib().lcpp_dist_reduce(comm.handle, _ptr(temp), temp.numel(), _ptr(x), _ptr(out), n, op, iv, code,
                                 _stream_ptr()), "lcpp_dist_reduce")
    del keep
    return out


# ---------------------------------------------------------------------------
# Single-GPU helpers of the bench's merge op.
# ---------------------------------------------------------------------------
def local_sort(keys):
    import torch
    n = keys.numel()
    out = torch.empty_like(keys)
    if n:
        temp = alloc_temp(DeviceRadixSort.GetSortKeysTempStorageBytes(dtype_code(keys), n), keys.device)
        DeviceRadixSort().SortKeys(temp, keys, out, n)
    return out


def merge_sorted(a, b, out):
    """out[:a.numel() + b.numel()] = stable merge of the sorted runs a, b
    (lcpp_dist_merge_sorted)."""
    total = a.numel() + b.numel()
    need = ctypes.c_size_t()
    check(lib().lcpp_dist_merge_temp_bytes(total, ctypes.byref(need)), "lcpp_dist_merge_temp_bytes")
    temp = alloc_temp(need.value, a.device)
    check(lib().lcpp_dist_merge_sorted(_ptr(temp), temp.numel(), _ptr(a), a.numel(), _ptr(b), b.numel(), _ptr(out),
                                       dtype_code(a), _stream_ptr()), "lcpp_dist_merge_sorted")


# ---------------------------------------------------------------------------
# Benchmark (bench.py, N > 1, and the distributed ops at any N)
# ---------------------------------------------------------------------------
class _NoSampler:
    def __enter__(self):
        return self

    def __exit__(self, *exc):
        return False

    def summary(self):
        return None


def bind_to_gpu_numa_node(device_index: int):
    """Restrict this process's CPUs to the NUMA node of its GPU (pinned host
    buffers allocated afterwards are then first touched there).  Returns the
    node, or None when the topology is not visible."""
    import torch
    try:
        props = torch.cuda.get_device_properties(device_index)
        bus = f"{props.pci_domain_id:04x}:{props.pci_bus_id:02x}:{props.pci_device_id:02x}.0"
        with open(f"/sys/bus/pci/devices/{bus}/numa_node") as f:
            node = int(f.read().strip())
        if node < 0:
            return None
        with open(f"/sys/devices/system/node/node{node}/cpulist") as f:
            spec = f.read().strip()
        cpus = set()
        for part in spec.split(","):
            a, _, b = part.partition("-")
            cpus.update(range(int(a), int(b or a) + 1))
        os.sched_setaffinity(0, (cpus & os.sched_getaffinity(0)) or cpus)
        return node
    except (OSError, ValueError, AttributeError):
        return None


def image_i64(t):
    """Order-preserving images of u32 / f32 keys (the sort's ascending
    bijection, +-0.0 folded) as int64, for checks."""
    import torch
    b = t.view(torch.int32).to(torch.int64) & 0xFFFFFFFF
    if t.dtype == torch.float32:
        neg = (b >> 31) == 1
        img = torch.where(neg, b ^ 0xFFFFFFFF, b ^ 0x80000000)
        return torch.where(img == 0x7FFFFFFF, torch.full_like(img, 0x80000000), img)
    return b


def parity_check(comm: Comm, dist, n_per_rank: int = 1 << 22):
    """Bit-exact check of the distributed sort on three inputs of n_per_rank
    keys per rank -- uniform u32, Zipf(1.1) u32 (the heavy hitter spans
    ranks), and N(0,1) f32 with both signed zeros (equal keys with different
    bits: their order shows stability) -- against a stable sort of all
    ranks' inputs gathered in rank order.  Returns {case: bool}."""
    import torch

    from . import GEN_F32_NORMAL, GEN_U32_UNIFORM, GEN_U32_ZIPF, testgen_fill
    G, r = dist.get_world_size(), dist.get_rank()
    dev = comm.device
    res = {}
    for name, gen, dt, seed in (("uniform_u32", GEN_U32_UNIFORM, torch.uint32, 11),
                                ("zipf_u32", GEN_U32_ZIPF, torch.uint32, 12),
                                ("normal_f32_signed_zeros", GEN_F32_NORMAL, torch.float32, 13)):
        keys = torch.empty(n_per_rank, dtype=dt, device=dev)
        testgen_fill(keys, gen, seed=seed, offset=r * n_per_rank)
        out = distributed_sort_keys(keys, comm)
        ins = [torch.empty(n_per_rank, dtype=torch.int32, device=dev) for _ in range(G)]
        outs = [torch.empty(n_per_rank, dtype=torch.int32, device=dev) for _ in range(G)]
        dist.all_gather(ins, keys.view(torch.int32))
        dist.all_gather(outs, out.view(torch.int32))
        allin = torch.cat(ins)
        allout = torch.cat(outs)
        order = torch.sort(image_i64(allin.view(dt)), stable=True).indices
        ok = torch.tensor([int(torch.equal(allout, allin[order]))], device=dev)
        dist.all_reduce(ok, op=dist.ReduceOp.MIN)
        res[name] = bool(ok.item())
        del ins, outs, allin, allout, order
    return res


def _timed_steps(fn, steps, dist, stream):
    """Device time per step of fn() (CUDA events on the launching stream),
    max over ranks."""
    import torch
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    dist.barrier()
    torch.cuda.synchronize()
    e0.record(stream)
    for _ in range(steps):
        fn()
    e1.record(stream)
    torch.cuda.synchronize()
    ms = torch.tensor([e0.elapsed_time(e1) / steps], dtype=torch.float64, device="cuda")
    dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    return ms.item()


def _phase_times(comm, keys, out, dist, exchange="auto"):
    """Per-phase times of one call, max over ranks per phase.  The ranks
    start together: a rank that arrives late would otherwise show up as the
    others' wait in their first collective (the splitter rounds)."""
    import torch
    dist.barrier()
    torch.cuda.synchronize()
    distributed_sort_keys(keys, comm, out=out, exchange=exchange)  # warm for this exchange
    dist.barrier()
    torch.cuda.synchronize()
    _, t = distributed_sort_keys(keys, comm, out=out, exchange=exchange, times=True)
    names = ["local_sort_ms", "splitters_ms", "host_wait_ms", "exchange_merge_ms", "local_merge_ms", "total_ms",
             "host_ms"]
    v = torch.tensor([t[k] for k in names], dtype=torch.float64, device="cuda")
    dist.all_reduce(v, op=dist.ReduceOp.MAX)
    d = dict(zip(names, v.tolist()))
    d["exchange"] = {1: "peer memory (CUDA IPC, plain loads over NVLink)",
                     2: "copy-engine pushes over CUDA IPC, local merges"}.get(t["peer_exchange"], "NCCL send/recv")
    return d


def strong_scaling_2p32(comm: Comm, dist, steps: int = 3, warmup: int = 2):
    """2^32 u32 keys in total (seed 7), uniform and Zipf(1.1) hashed, sharded
    evenly over the ranks: ms per distributed sort (max over ranks), and --
    on rank 0, alone, in the same job -- the single-GPU sort of the same
    2^32 keys of each distribution (the 1-GPU-equivalent runs)."""
    import torch

    from . import GEN_U32_UNIFORM, GEN_U32_ZIPF, testgen_fill
    G, r = dist.get_world_size(), dist.get_rank()
    total = 1 << 32
    n = total // G
    stream = torch.cuda.current_stream()
    res = {}
    for name, gen in (("uniform", GEN_U32_UNIFORM), ("zipf", GEN_U32_ZIPF)):
        keys = torch.empty(n, dtype=torch.uint32, device=comm.device)
        testgen_fill(keys, gen, seed=7, offset=r * n)
        out = torch.empty_like(keys)
        for _ in range(warmup):
            distributed_sort_keys(keys, comm, out=out)
        ms = _timed_steps(lambda: distributed_sort_keys(keys, comm, out=out), steps, dist, stream)
        res[name] = {"ms": ms, "gkeys_per_s": total / (ms * 1e-3) / 1e9,
                     "phases": _phase_times(comm, keys, out, dist)}
        del keys, out
        comm._temps.clear()
        torch.cuda.empty_cache()
    # the 1-GPU-equivalent runs: rank 0 alone sorts all 2^32 keys of each distribution
    one = torch.zeros(2, dtype=torch.float64, device="cuda")
    if r == 0:
        keys = torch.empty(total, dtype=torch.uint32, device=comm.device)
        out = torch.empty_like(keys)
        temp = alloc_temp(DeviceRadixSort.GetSortKeysTempStorageBytes(dtype_code(keys), total), comm.device)
        rs = DeviceRadixSort()
        for q, gen in enumerate((GEN_U32_UNIFORM, GEN_U32_ZIPF)):
            testgen_fill(keys, gen, seed=7)
            for _ in range(warmup):
                rs.SortKeys(temp, keys, out, total)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            torch.cuda.synchronize()
            e0.record(stream)
            for _ in range(steps):
                rs.SortKeys(temp, keys, out, total)
            e1.record(stream)
            torch.cuda.synchronize()
            one[q] = e0.elapsed_time(e1) / steps
        del keys, out, temp
        torch.cuda.empty_cache()
    dist.all_reduce(one)
    for q, name in enumerate(("uniform", "zipf")):
        t1 = one[q].item()
        res[name]["one_gpu_ms"] = t1
        res[name]["one_gpu_gkeys_per_s"] = total / (t1 * 1e-3) / 1e9
        res[name]["speedup_vs_one_gpu"] = t1 / res[name]["ms"]
    return res


def bench_distributed_sort(n_local, steps, warmup, dist, clock_sampler_cls, peak, seed=0, zipf=False,
                           metric="Gkeys/s uint32 SortKeys @2^28", scaling="weak", strong_2p32=False):
    """Benchmark of lcpp_dist_sort_keys: n_local u32 keys per rank (rank r
    holds elements [r n, (r+1) n) of the `seed` stream, uniform or Zipf(1.1)
    hashed).  Device time per step is the max over ranks.  Before timing,
    parity_check() compares three distributed sorts bit for bit with a
    stable sort of the gathered inputs."""
    import torch

    from . import GEN_U32_UNIFORM, GEN_U32_ZIPF, KERNEL_SORT_ONESWEEP, diag_timing_enable, diag_timing_read, \
        testgen_fill
    G, r = dist.get_world_size(), dist.get_rank()
    dev = torch.device("cuda", torch.cuda.current_device())
    all_cpus = os.sched_getaffinity(0)
    numa = bind_to_gpu_numa_node(dev.index)
    comm = Comm(dist)
    try:
        parity = parity_check(comm, dist)
        comm._temps.clear()
        keys = torch.empty(n_local, dtype=torch.uint32, device=dev)
        testgen_fill(keys, GEN_U32_ZIPF if zipf else GEN_U32_UNIFORM, seed=seed, offset=r * n_local)
        out = torch.empty_like(keys)
        for _ in range(warmup):
            distributed_sort_keys(keys, comm, out=out)
        torch.cuda.synchronize()
        stream = torch.cuda.current_stream()
        props = torch.cuda.get_device_properties(dev)
        bus = getattr(props, "pci_bus_id", None)
        # one nvidia-smi sampler (rank 0) for the whole job
        sampler = clock_sampler_cls(f"{bus:02x}:00.0" if isinstance(bus, int) else None) if r == 0 else _NoSampler()
        with sampler as clocks:
            diag_timing_enable(True)
            ms = _timed_steps(lambda: distributed_sort_keys(keys, comm, out=out), steps, dist, stream)
            recs = diag_timing_read()
            diag_timing_enable(False)
        value = G * n_local / (ms * 1e-3) / 1e9
        phases = _phase_times(comm, keys, out, dist)
        # the same call under each explicit exchange (every rank takes the
        # same branch: the condition is the auto choice, identical on all)
        on_one_host = G > 1 and not phases["exchange"].startswith("NCCL")
        by_exchange = {"nccl_send_recv": _phase_times(comm, keys, out, dist, exchange="nccl")}
        if on_one_host:
            by_exchange["peer_loads"] = _phase_times(comm, keys, out, dist, exchange="peer")
            by_exchange["copy_engine_pushes"] = _phase_times(comm, keys, out, dist, exchange="copy")

        # e2e: pinned host keys -> device, distributed sort, this rank's part
        # -> host, pipelined over three streams (upload of step s+1 and
        # download of step s-1 overlap the sort of step s).  Pinned buffers
        # are allocated after binding this process to its GPU's NUMA node.
        host_in = torch.empty(n_local, dtype=torch.uint32, pin_memory=True).copy_(keys)
        host_out = [torch.empty(n_local, dtype=torch.uint32, pin_memory=True) for _ in range(2)]
        d_in = [torch.empty_like(keys) for _ in range(2)]
        d_out = [torch.empty_like(keys) for _ in range(2)]
        k_e2e = max(3, min(steps, 10))
        s_in, s_out = torch.cuda.Stream(), torch.cuda.Stream()

        def e2e_run(k):
            ev_op, ev_out = {}, {}
            first, last = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            first.record(s_in)
            for st in range(k):
                b = st % 2
                with torch.cuda.stream(s_in):
                    if st >= 2:
                        s_in.wait_event(ev_op[st - 2])
                    d_in[b].copy_(host_in, non_blocking=True)
                    ev_in = torch.cuda.Event()
                    ev_in.record(s_in)
                stream.wait_event(ev_in)
                if st >= 2:
                    stream.wait_event(ev_out[st - 2])
                distributed_sort_keys(d_in[b], comm, out=d_out[b])
                ev_op[st] = torch.cuda.Event()
                ev_op[st].record(stream)
                with torch.cuda.stream(s_out):
                    s_out.wait_event(ev_op[st])
                    host_out[b].copy_(d_out[b], non_blocking=True)
                    ev_out[st] = torch.cuda.Event()
                    ev_out[st].record(s_out)
            last.record(s_out)
            torch.cuda.synchronize()
            return first.elapsed_time(last)

        e2e_run(2)
        dist.barrier()
        e2e_ms = torch.tensor([e2e_run(k_e2e) / k_e2e], dtype=torch.float64, device=dev)
        dist.all_reduce(e2e_ms, op=dist.ReduceOp.MAX)
        e2e_ms = e2e_ms.item()
        # host link alone: one 4 B/key upload and download per rank
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
        ev[0].record(stream)
        d_in[0].copy_(host_in, non_blocking=True)
        ev[1].record(stream)
        host_out[0].copy_(d_out[0], non_blocking=True)
        ev[2].record(stream)
        torch.cuda.synchronize()
        link = torch.tensor([4 * n_local / (ev[0].elapsed_time(ev[1]) * 1e-3) / 1e9,
                             4 * n_local / (ev[1].elapsed_time(ev[2]) * 1e-3) / 1e9], dtype=torch.float64,
                            device=dev)
        dist.all_reduce(link, op=dist.ReduceOp.MIN)
        del host_in, host_out, d_in, d_out
        strong = None
        if strong_2p32:
            del keys, out
            comm._temps.clear()
            torch.cuda.empty_cache()
            strong = strong_scaling_2p32(comm, dist)
    finally:
        comm.close(dist)
        os.sched_setaffinity(0, all_cpus)

    onesweep = [x[1] for x in recs if x[0] == KERNEL_SORT_ONESWEEP]
    avg_pass = sum(onesweep) / max(1, len(onesweep))
    achieved = 8 * n_local / (avg_pass * 1e-3) / 1e9
    peak_gbs, peak_src = peak
    # HBM bytes per GPU: the local sort (36 B/key: histogram read + 4 passes
    # x 8 B/key), the first merge level (reads 4 B/key where the runs lie,
    # writes 4 B/key), ceil(log2 G) - 1 local merge levels (8 B/key each);
    # (G-1)/G of the keys cross NVLink.
    levels = (G - 1).bit_length()
    hbm_bytes = (36 + 8 * levels) * n_local if G > 1 else 36 * n_local
    nvlink_bytes = (G - 1) / G * 4 * n_local
    dist_name = "Zipf(1.1) ranks hashed by fmix32" if zipf else "uniform"
    line = {
        "metric": metric, "value": value, "unit": "Gkeys/s", "n_gpus": G,
        "steps": steps, "warmup": warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": scaling,
        "vs_baseline": None, "dtype": "u32",
        "data": "synthetic (splitmix64 counter streams; see include/lcpp_b200_testgen.h)",
        "config": {"workload": f"distributed SortKeys u32 {dist_name}, seed {seed}, "
                               f"2^{n_local.bit_length() - 1} keys per GPU (global 2^{(G * n_local).bit_length() - 1})",
                   "items_per_gpu": n_local,
                   "parallelism": f"sort-partitioned over {G} GPUs ({phases['exchange']})" if G > 1 else "single GPU",
                   "algorithm": "lcpp_dist_sort_keys: local onesweep -> exact splitters refined 16 bits per round on "
                                "the device (NCCL all-reduce per round, all-gather of boundary ties) -> one host read "
                                "of the split matrix -> exchange: from 4 GPUs copy-engine pushes of every run into "
                                "the receivers' run buffers over NVLink, then local merge levels; with 2-3 GPUs a "
                                "first merge level reading the runs straight from the owners' memory",
                   "l2": "inputs larger than L2; no flush"},
        "parity_bit_exact": all(parity.values()), "parity_cases": parity,
        "phases_ms": phases,
        "phases_ms_by_exchange": by_exchange,
        "roofline": {"bound": "hbm", "kernel": "onesweep_bulk_kernel (one 8-bit pass)", "achieved": achieved,
                     "peak": peak_gbs, "peak_source": peak_src, "unit": "GB/s", "frac": achieved / peak_gbs,
                     "algorithmic_bytes_per_launch": 8 * n_local, "avg_launch_ms": avg_pass, "traffic": None},
        "op_roofline": {"hbm_bytes_per_gpu": hbm_bytes, "nvlink_bytes_per_gpu": nvlink_bytes,
                        "target_ms": max(hbm_bytes / (peak_gbs * 1e9), nvlink_bytes / 770e9) * 1e3,
                        "frac": max(hbm_bytes / (peak_gbs * 1e9), nvlink_bytes / 770e9) * 1e3 / ms},
        "e2e": {"value": G * n_local / (e2e_ms * 1e-3) / 1e9, "unit": "Gkeys/s",
                "h2d_bytes_per_step": 4 * n_local * G, "d2h_bytes_per_step": 4 * n_local * G, "steps": k_e2e,
                "ms_per_step": e2e_ms,
                "pipeline": "3 streams per rank: H2D of step s+1 and D2H of step s-1 overlap the sort of step s",
                "host_link_gb_per_s_per_rank_min": {"h2d": link[0].item(), "d2h": link[1].item()},
                "numa_node_rank0": numa},
        # per step: histogram + 4 passes (timed by the library) and, for G > 1,
        # split init + 2 rounds x (counts, select) + tie counts + positions +
        # the merge levels' split kernels (their block kernels are timed)
        "gpu_launches": len(recs) + (steps * (7 + levels) if G > 1 else 0), "clocks": clocks.summary(),
        "cpu_baseline": None,
    }
    if strong is not None:
        line["strong_scaling_2p32"] = strong
    return line
