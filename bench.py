#!/usr/bin/env python
"""Benchmark: uint32 SortKeys at 2^28 keys per GPU (BASELINE metric
"Gkeys/s uint32 SortKeys @2^28 (1/2/4/8 B200) and % of HBM roofline").

One step = one DeviceRadixSort::SortKeys (copy API) of 2^28 uniform uint32
keys (seed 0, bits [0,32)) through the library's C ABI.

Arms:
  default           our sm_100a library.  N = 1: device-resident `value`
                    (inputs in HBM), `e2e` through the same public call with
                    pinned host buffers (H2D of the keys + sort + D2H of the
                    sorted keys inside the timed region), live roofline of the
                    dominant kernel (onesweep pass) from CUDA events on the
                    library's launch stream, clocks sampled during the timed
                    region, and the CPU baseline (oracle port, all host
                    threads, bounded sample) on rank 0.
                    N > 1 (torchrun): the distributed sort, 2^28 keys per GPU
                    (weak scaling), max over ranks.
  --impl reference  the reference's own path on the host cores: its CPU
                    restatement (oracle port, the reference cannot be built
                    here), all host threads, a bounded sample of the same
                    workload per step.  Rank 0 only.
"""
from __future__ import annotations

import argparse
import json
import os
import re
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "luisacompute-parallelprimitive_b200"))
sys.path.insert(0, str(ROOT))

METRIC = "Gkeys/s uint32 SortKeys @2^28"
UNIT = "Gkeys/s"
BYTES_PER_KEY_SORT = 36       # k*(1+2P), k=4, P=4 (8-bit passes)
BYTES_PER_KEY_ONESWEEP = 8    # one pass reads and writes each 4-byte key
FALLBACK_HBM_GBS = 6650.0


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--log2n", type=int, default=28, help="keys per GPU = 2^log2n")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    return ap.parse_args()


def measured_peak():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
        except Exception:
            pass
    return FALLBACK_HBM_GBS, "fallback"


def profiled_traffic():
    """Per-launch DRAM bytes of the onesweep kernel from the committed ncu
    summary (line 'traffic_bytes_per_key: X'), scaled to the workload."""
    p = ROOT / "profiles" / "onesweep_u32_keys.md"
    if not p.exists():
        return None
    m = re.search(r"traffic_bytes_per_key:\s*([0-9.]+)", p.read_text())
    return float(m.group(1)) if m else None


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms while running."""

    FIELDS = ("pci.bus_id,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, bus_id: str | None):
        self.bus_id = (bus_id or "").lower()
        self.proc = None
        self.out = tempfile.NamedTemporaryFile(mode="w+", suffix=".csv", delete=False)

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=self.out, stderr=subprocess.DEVNULL)
        except FileNotFoundError:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        self.out.flush()
        rows = []
        for line in Path(self.out.name).read_text().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            if self.bus_id and not f[0].lower().endswith(self.bus_id[-12:]):
                continue
            try:
                rows.append((float(f[1]), float(f[2]), float(f[3]), f[4:9]))
            except ValueError:
                continue
        os.unlink(self.out.name)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        names = ["active", "hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(1, 5) if r[3][i].lower() == "active"})
        loaded = [r for r in rows if r[2] > 300] or rows
        return {"sm_mhz": statistics.median(r[0] for r in loaded), "sm_max_mhz": max(r[1] for r in rows),
                "reasons": reasons, "samples": len(rows), "power_w_max": max(r[2] for r in rows)}


def cpu_sort_sample(n_sample: int, threads: int, min_seconds: float):
    """Time the oracle port (multi-threaded LSD restatement) on a bounded
    sample of the workload; returns (Gkeys/s, reps)."""
    from oracle import oracle
    keys = oracle.generate(oracle.GEN_U32_UNIFORM, n_sample, seed=0)
    oracle.radix_sort(keys, threads=threads)  # warm
    reps, t0 = 0, time.perf_counter()
    while True:
        oracle.radix_sort(keys, threads=threads)
        reps += 1
        el = time.perf_counter() - t0
        if el >= min_seconds:
            break
    return n_sample * reps / el / 1e9, reps


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    from oracle import oracle
    threads = oracle.cpu_threads()
    n_sample = 1 << 22
    keys = oracle.generate(oracle.GEN_U32_UNIFORM, n_sample, seed=0)
    for _ in range(args.warmup):
        oracle.radix_sort(keys, threads=threads)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        oracle.radix_sort(keys, threads=threads)
    el = time.perf_counter() - t0
    v = n_sample * args.steps / el / 1e9
    line = {
        "impl": "reference", "metric": METRIC, "value": v, "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": el / args.steps * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "u32",
        "data": "synthetic (splitmix64 counter stream, seed 0)",
        "config": {"workload": f"SortKeys u32 uniform, 2^{args.log2n} keys per GPU; each step sorts a "
                               f"bounded 2^22-key sample of it on the host", "begin_bit": 0, "end_bit": 32},
        "cpu_baseline": {"value": v, "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": "2^22 uniform u32 keys (first 2^22 of the seed-0 stream) per step; "
                                   "multi-threaded LSD restatement of the onesweep semantics"},
        "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def run_ours(args):
    import torch

    import lcpp_b200 as L

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE {world}")
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import torch.distributed as dist
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
    n = 1 << args.log2n
    stream = torch.cuda.current_stream()

    if world > 1:
        from lcpp_b200 import distributed as D
        res = D.bench_distributed_sort(n, args.steps, args.warmup, dist)
        if rank == 0:
            print(json.dumps(res), flush=True)
        dist.barrier()
        dist.destroy_process_group()
        return 0

    rs = L.DeviceRadixSort()
    keys = torch.empty(n, dtype=torch.uint32, device="cuda")
    L.testgen_fill(keys, L.GEN_U32_UNIFORM, seed=0)
    out = torch.empty_like(keys)
    temp = L.alloc_temp(rs.GetSortKeysTempStorageBytes(L.U32, n))

    for _ in range(args.warmup):
        rs.SortKeys(temp, keys, out, n)
    torch.cuda.synchronize()
    assert L.device_status(temp) == L.OK

    bus = torch.cuda.get_device_properties(local).pci_bus_id if hasattr(
        torch.cuda.get_device_properties(local), "pci_bus_id") else None
    bus_id = f"{bus:02x}:00.0" if isinstance(bus, int) else None
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(bus_id) as clocks:
        L.diag_timing_enable(True)
        torch.cuda.synchronize()
        e0.record(stream)
        for _ in range(args.steps):
            rs.SortKeys(temp, keys, out, n)
        e1.record(stream)
        torch.cuda.synchronize()
        recs = L.diag_timing_read()
        L.diag_timing_enable(False)
    ms = e0.elapsed_time(e1) / args.steps
    assert L.device_status(temp) == L.OK
    value = n / (ms * 1e-3) / 1e9
    clk = clocks.summary()

    onesweep = [r[1] for r in recs if r[0] == L.KERNEL_SORT_ONESWEEP]
    hist = [r[1] for r in recs if r[0] == L.KERNEL_SORT_HISTOGRAM]
    avg_pass_ms = sum(onesweep) / len(onesweep)
    peak, peak_kind = measured_peak()
    achieved = BYTES_PER_KEY_ONESWEEP * n / (avg_pass_ms * 1e-3) / 1e9
    tpk = profiled_traffic()
    roofline = {"bound": "hbm", "kernel": "onesweep_kernel (one 8-bit pass)", "achieved": achieved,
                "peak": peak, "peak_source": peak_kind, "unit": "GB/s", "frac": achieved / peak,
                "algorithmic_bytes_per_launch": BYTES_PER_KEY_ONESWEEP * n,
                "avg_launch_ms": avg_pass_ms,
                "traffic": (tpk * n) if tpk is not None else None}
    sort_ach = BYTES_PER_KEY_SORT * n / (ms * 1e-3) / 1e9
    sort_roofline = {"bytes_per_key": BYTES_PER_KEY_SORT, "achieved": sort_ach, "peak": peak,
                     "unit": "GB/s", "frac": sort_ach / peak,
                     "histogram_ms": sum(hist) / len(hist), "onesweep_ms_per_pass": avg_pass_ms}

    # e2e: the same public call, host buffers, copies inside the timed region.
    host_in = torch.empty(n, dtype=torch.uint32, pin_memory=True)
    host_in.copy_(keys)
    host_out = torch.empty(n, dtype=torch.uint32, pin_memory=True)
    d_in = torch.empty_like(keys)
    k_e2e = max(3, min(args.steps, 20))
    for _ in range(2):
        d_in.copy_(host_in, non_blocking=True)
        rs.SortKeys(temp, d_in, out, n)
        host_out.copy_(out, non_blocking=True)
    torch.cuda.synchronize()
    e0.record(stream)
    for _ in range(k_e2e):
        d_in.copy_(host_in, non_blocking=True)
        rs.SortKeys(temp, d_in, out, n)
        host_out.copy_(out, non_blocking=True)
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1) / k_e2e
    e2e = {"value": n / (e2e_ms * 1e-3) / 1e9, "unit": UNIT, "h2d_bytes_per_step": 4 * n,
           "d2h_bytes_per_step": 4 * n, "steps": k_e2e, "ms_per_step": e2e_ms}
    # sanity: the result that came back is sorted
    ho = host_out.numpy()
    assert bool((ho[1:] >= ho[:-1]).all())

    cpu = None
    if not args.no_cpu_baseline and rank == 0:
        from oracle import oracle
        threads = oracle.cpu_threads()
        v, reps = cpu_sort_sample(1 << 24, threads, 10.0)
        cpu = {"value": v, "unit": UNIT, "cores": threads, "kind": "port",
               "sample": f"2^24 uniform u32 keys (first 2^24 of the seed-0 stream) x {reps} sorts; "
                         "multi-threaded LSD restatement of the onesweep semantics"}

    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "u32", "data": "synthetic (splitmix64 counter stream, seed 0)",
        "config": {"workload": f"SortKeys u32 uniform full range, n=2^{args.log2n} per GPU, bits [0,32)",
                   "keys_per_gpu": n, "parallelism": "single GPU",
                   "l2": "inputs larger than L2 (1 GiB of keys per step vs 126 MB L2); no flush"},
        "roofline": roofline, "sort_roofline": sort_roofline, "e2e": e2e,
        "gpu_launches": len(recs), "clocks": clk, "cpu_baseline": cpu,
    }
    print(json.dumps(line), flush=True)
    return 0


def main():
    args = parse_args()
    if args.impl == "reference":
        return run_reference(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
