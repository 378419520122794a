#!/usr/bin/env python
"""Benchmark of the sort / scan / reduce path (BASELINE metric "Gkeys/s
uint32 SortKeys @2^28 (1/2/4/8 B200) and % of HBM roofline").

Default (--op sort): one step = one DeviceRadixSort::SortKeys (copy API) of
2^28 uniform uint32 keys per GPU (seed 0, bits [0,32)) through the library's
C ABI.  The other BASELINE configurations are available with --op (pairs,
pairs_f32, pairs_u64, bits, scan, reduce, reduce_max, and the distributed
sort of 2^32 keys in total, dist / dist_zipf, at any N); the driver only
runs the default.

Arms:
  default           our sm_100a library.  N = 1: device-resident `value`
                    (inputs in HBM), `e2e` through the same public call with
                    pinned host buffers (H2D of the inputs + the op + D2H of
                    the result inside the timed region), live roofline of the
                    dominant kernel from CUDA events on the library's launch
                    stream, clocks sampled during the timed region, and the
                    CPU baseline (oracle port, all host threads, bounded
                    sample) on rank 0.
                    N > 1 (torchrun): the distributed sort
                    (lcpp_dist_sort_keys), 2^28 keys per GPU (weak scaling),
                    max over ranks; the line also carries a bit-exact parity
                    check of three gathered distributed sorts (the run exits
                    non-zero when it fails), per-phase times, and the 2^32-key
                    strong-scaling sort with the 1-GPU sort of the same keys
                    timed on rank 0 in the same job.
  --impl cub        NVIDIA CUB from the CUDA toolkit on the same GPU and the
                    same inputs (the comparison the reference's own benchmark
                    makes, tests/cub_bench_kernels.cu:20-75): ops sort, pairs,
                    scan, reduce; one GPU.
  --impl reference  the reference's own path on the host cores: its CPU
                    restatement (oracle port; the reference cannot be built
                    here), all host threads, a bounded sample of the same
                    workload per step.  Rank 0 only.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "luisacompute-parallelprimitive_b200"))
sys.path.insert(0, str(ROOT))

FALLBACK_HBM_GBS = 6650.0
DATA = "synthetic (splitmix64 counter streams; see include/lcpp_b200_testgen.h)"


# ---------------------------------------------------------------------------
# Workloads.  bytes: algorithmic HBM bytes per item of
# the whole op (k*(1+2P) + v*2P for sorts with P 8-bit passes); kbytes:
# algorithmic bytes per item of ONE launch of the dominant kernel.
# ---------------------------------------------------------------------------
OPS = {
    "sort": dict(metric="Gkeys/s uint32 SortKeys @2^28", unit="Gkeys/s", log2n=28, dtype="u32",
                 workload="SortKeys u32 uniform full range, bits [0,32), seed 0", bytes=36, kbytes=8,
                 kernel="onesweep_bulk_kernel (one 8-bit pass)"),
    "pairs": dict(metric="Gkeys/s uint32->uint32 SortPairs @2^28", unit="Gkeys/s", log2n=28, dtype="u32",
                  workload="SortPairs u32 uniform keys, u32 values = index, seed 1", bytes=68, kbytes=16,
                  kernel="onesweep_kernel (one 8-bit pass)"),
    "pairs_f32": dict(metric="Gkeys/s float32->uint32 SortPairs @2^27", unit="Gkeys/s", log2n=27, dtype="f32",
                      workload="SortPairs f32 N(0,1) keys with +-0.0, u32 values = index, seed 1",
                      bytes=68, kbytes=16, kernel="onesweep_kernel (one 8-bit pass)"),
    "pairs_u64": dict(metric="Gkeys/s uint64->int32 SortPairs @2^27", unit="Gkeys/s", log2n=27, dtype="u64",
                      workload="SortPairs u64 uniform keys, i32 values = index, seed 1", bytes=200, kbytes=24,
                      kernel="onesweep_kernel (one 8-bit pass)"),
    "bits": dict(metric="Gkeys/s uint32 SortKeys bits [8,24) @2^27", unit="Gkeys/s", log2n=27, dtype="u32",
                 workload="SortKeys u32 uniform, begin_bit 8, end_bit 24, seed 1", bytes=20, kbytes=8,
                 kernel="onesweep_bulk_kernel (one 8-bit pass)"),
    "scan": dict(metric="Gitems/s int32 InclusiveSum @2^30", unit="Gitems/s", log2n=30, dtype="i32",
                 workload="InclusiveSum i32 uniform in [-1000,1000], seed 1", bytes=8, kbytes=8,
                 kernel="scan_bulk_kernel"),
    "reduce": dict(metric="Gitems/s float32 Reduce Sum @2^30", unit="Gitems/s", log2n=30, dtype="f32",
                   workload="DeviceReduce::Sum f32 U[0,1), seed 1", bytes=4, kbytes=4, kernel="reduce_kernel"),
    "reduce_max": dict(metric="Gitems/s int64 Reduce Max @2^30", unit="Gitems/s", log2n=30, dtype="i64",
                       workload="DeviceReduce::Max i64 uniform, seed 1", bytes=8, kbytes=8, kernel="reduce_kernel"),
    # DeviceReduce::ArgMin: one read of every item (4 B), nothing written
    # but the (value, index) result.
    "argmin": dict(metric="Gitems/s float32 ArgMin @2^30", unit="Gitems/s", log2n=30, dtype="f32",
                   workload="DeviceReduce::ArgMin f32 U[0,1) (many tied minima), seed 1", bytes=4, kbytes=4,
                   kernel="arg_extremum_kernel"),
    # By-key family, keys i / 100 (segments of 100 as in the reference's
    # by-key tests), i32 values from the scan stream.  InclusiveSumByKey reads
    # keys and values and writes the output (12 B per item); ReduceByKey reads
    # both and writes one (key, aggregate) pair per 100 items (8.08 B).
    "scan_by_key": dict(metric="Gitems/s i32 by i32 InclusiveSumByKey @2^30", unit="Gitems/s", log2n=30,
                        dtype="i32", workload="InclusiveSumByKey i32 values by keys i/100, seed 1", bytes=12,
                        kbytes=12, kernel="by_key_kernel"),
    "reduce_by_key": dict(metric="Gitems/s i32 by i32 ReduceByKey Sum @2^30", unit="Gitems/s", log2n=30,
                          dtype="i32", workload="ReduceByKey Sum of i32 values by keys i/100, seed 1",
                          bytes=8.08, kbytes=8.08, kernel="by_key_kernel"),
    # DeviceSelect::If(x % 2 == 0) over uniform i32: reads every item, writes
    # the selected half (4 + 2 B per item).
    "select": dict(metric="Gitems/s i32 DeviceSelect::If(even) @2^30", unit="Gitems/s", log2n=30, dtype="i32",
                   workload="DeviceSelect::If x % 2 == 0 over uniform i32, seed 1", bytes=6, kbytes=6,
                   kernel="compact_kernel"),
    # DeviceSegmentedRadixSort: 2^27 u32 keys in
    # segments of 1..2047 keys (sizes uniform, seed 1), contiguous.  All
    # segments are short, so the one-block-per-segment kernel does the whole
    # sort: it reads and writes every key once (8 B per item, the op's and
    # the kernel's algorithmic bytes).
    "segsort": dict(metric="Gkeys/s uint32 SegmentedRadixSort SortKeys @2^27", unit="Gkeys/s", log2n=27,
                    dtype="u32", workload="SegmentedRadixSort SortKeys u32 uniform, segments of 1..2047 keys, seed 1",
                    bytes=8, kbytes=8, kernel="small_segment_kernel (one block per segment, shared-memory LSD)"),
    # DeviceRadixSort over decomposed keys (the decomposer overloads): 2^27
    # structs {u32 primary; i32 secondary} (uniform, seed 1), full 64-bit
    # window.  Algorithmic bytes as SortKeys of 8-byte keys (k(1+2P), P = 8);
    # the dominant launch is an onesweep pass over the 64-bit composite and
    # the 32-bit index: 24 B per item.
    "decomposed": dict(metric="Gkeys/s {u32,i32} decomposed SortKeys @2^27", unit="Gkeys/s", log2n=27,
                       dtype="u32+i32", workload="SortKeys of {u32 primary, i32 secondary} structs, uniform, seed 1",
                       bytes=136, kbytes=24, kernel="onesweep_kernel (one 8-bit pass of the 64-bit composite)"),
    # Merge path of the distributed sort (lcpp_dist_merge_sorted): two sorted
    # runs of 2^27 u32 keys (uniform, seed 1) into 2^28; reads and writes
    # every key once (8 B per output key).
    "merge": dict(metric="Gkeys/s uint32 merge of two sorted runs @2^28", unit="Gkeys/s", log2n=28, dtype="u32",
                  workload="merge path of two sorted u32 runs of 2^27 keys, uniform, seed 1", bytes=8, kbytes=8,
                  kernel="merge_bulk_kernel"),
    # Distributed SortKeys of 2^32 keys in total (seed 7), sharded evenly:
    # strong scaling over N GPUs (N = 1 is the 1-GPU-equivalent run).
    "dist": dict(metric="Gkeys/s uint32 distributed SortKeys @2^32", unit="Gkeys/s", log2n=32, dtype="u32",
                 workload="distributed SortKeys u32 uniform, seed 7", bytes=36, kbytes=8,
                 kernel="onesweep_bulk_kernel (one 8-bit pass)", distributed=True, seed=7, zipf=False),
    "dist_zipf": dict(metric="Gkeys/s uint32 distributed SortKeys Zipf(1.1) @2^32", unit="Gkeys/s", log2n=32,
                      dtype="u32", workload="distributed SortKeys u32 Zipf(1.1) hashed, seed 7", bytes=36, kbytes=8,
                      kernel="onesweep_bulk_kernel (one 8-bit pass)", distributed=True, seed=7, zipf=True),
}


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference", "cub"], default="ours")
    ap.add_argument("--op", choices=sorted(OPS), default="sort")
    ap.add_argument("--log2n", type=int, default=None, help="items per GPU = 2^log2n (default: the config's)")
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


def profiled_traffic(op: str):
    """DRAM bytes per item of one launch of the dominant kernel, from the
    committed ncu figures (profiles/traffic.json)."""
    p = ROOT / "profiles" / "traffic.json"
    if not p.exists():
        return None
    v = json.loads(p.read_text()).get(op)
    return float(v) if isinstance(v, (int, float)) else None


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


# ---------------------------------------------------------------------------
# Workload objects for our arm: inputs in HBM, one `step` = one public call.
# ---------------------------------------------------------------------------
class Workload:
    def __init__(self, op: str, n: int):
        import torch

        import lcpp_b200 as L
        self.op, self.n, self.L, self.torch = op, n, L, torch
        dev = "cuda"
        T = torch

        def fill(dt, dist, seed):
            t = T.empty(n, dtype=dt, device=dev)
            L.testgen_fill(t, dist, seed=seed)
            return t

        if op == "sort":
            self.inputs = [fill(T.uint32, L.GEN_U32_UNIFORM, 0)]
            self.outputs = [T.empty_like(self.inputs[0])]
            self.temp = L.alloc_temp(L.DeviceRadixSort.GetSortKeysTempStorageBytes(L.U32, n))
        elif op == "bits":
            self.inputs = [fill(T.uint32, L.GEN_U32_UNIFORM, 1)]
            self.outputs = [T.empty_like(self.inputs[0])]
            self.temp = L.alloc_temp(L.DeviceRadixSort.GetSortKeysTempStorageBytes(L.U32, n))
        elif op in ("pairs", "pairs_f32", "pairs_u64"):
            kdt, kdist, vdt, kc, vc = {
                "pairs": (T.uint32, L.GEN_U32_UNIFORM, T.uint32, L.U32, L.U32),
                "pairs_f32": (T.float32, L.GEN_F32_NORMAL, T.uint32, L.F32, L.U32),
                "pairs_u64": (T.uint64, L.GEN_U64_UNIFORM, T.int32, L.U64, L.I32),
            }[op]
            self.inputs = [fill(kdt, kdist, 1), fill(vdt, L.GEN_U32_INDEX, 1)]
            self.outputs = [T.empty_like(self.inputs[0]), T.empty_like(self.inputs[1])]
            self.temp = L.alloc_temp(L.DeviceRadixSort.GetSortPairsTempStorageBytes(kc, vc, n))
        elif op == "segsort":
            import numpy as np
            self.inputs = [fill(T.uint32, L.GEN_U32_UNIFORM, 1)]
            self.outputs = [T.empty_like(self.inputs[0])]
            b, e = segsort_offsets(n)
            self.seg = (T.from_numpy(b).to(dev), T.from_numpy(e).to(dev), int(b.size))
            self.temp = L.alloc_temp(L.DeviceSegmentedRadixSort.GetSortKeysTempStorageBytes(L.U32, n))
            self.ss = L.DeviceSegmentedRadixSort()
            del np
        elif op == "decomposed":
            words = fill(T.uint32, L.GEN_U32_UNIFORM, 1)
            more = fill(T.uint32, L.GEN_U32_UNIFORM, 2)
            self.inputs = [T.stack([words, more], dim=1).contiguous()]  # n structs of 8 bytes
            del words, more
            self.outputs = [T.empty_like(self.inputs[0])]
            self.dec = L.Decomposer(8, [(0, L.U32), (4, L.I32)])
            self.temp = L.alloc_temp(L.DeviceRadixSort.GetDecomposedTempStorageBytes(n))
        elif op == "merge":
            from lcpp_b200 import distributed as D
            self.merge_sorted = D.merge_sorted
            half = n // 2
            keys = fill(T.uint32, L.GEN_U32_UNIFORM, 1)
            self.inputs = [D.local_sort(keys[:half].clone()), D.local_sort(keys[half:].clone())]
            self.outputs = [T.empty(n, dtype=T.uint32, device=dev)]
            self.temp = None
            del keys
        elif op == "scan":
            self.inputs = [fill(T.int32, L.GEN_I32_SCAN, 1)]
            self.outputs = [T.empty_like(self.inputs[0])]
            self.temp = L.alloc_temp(L.DeviceScan.GetTempStorageBytes(L.I32, n))
        elif op == "reduce":
            self.inputs = [fill(T.float32, L.GEN_F32_UNIT, 1)]
            self.outputs = [T.empty(1, dtype=T.float32, device=dev)]
            self.temp = L.alloc_temp(L.DeviceReduce.GetTempStorageBytes(L.F32, n))
        elif op in ("scan_by_key", "reduce_by_key"):
            keys = T.arange(n, dtype=T.int64, device=dev).div_(100, rounding_mode="floor").to(T.int32)
            self.inputs = [keys, fill(T.int32, L.GEN_I32_SCAN, 1)]
            if op == "scan_by_key":
                self.outputs = [T.empty_like(self.inputs[1])]
                self.temp = L.alloc_temp(L.DeviceScan.GetScanByKeyTempStorageBytes(L.I32, L.I32, n))
            else:
                runs = (n + 99) // 100
                self.outputs = [T.empty(runs, dtype=T.int32, device=dev), T.empty(runs, dtype=T.int32, device=dev),
                                T.empty(1, dtype=T.int32, device=dev)]
                self.temp = L.alloc_temp(L.DeviceReduce.GetReduceByKeyTempStorageBytes(L.I32, L.I32, n))
        elif op == "select":
            self.inputs = [fill(T.uint32, L.GEN_U32_UNIFORM, 1).view(T.int32)]
            self.outputs = [T.empty_like(self.inputs[0]), T.empty(1, dtype=T.int32, device=dev)]
            self.temp = L.alloc_temp(L.DeviceSelect.GetTempStorageBytes(n))
            self.pred = L.Pred.mod_eq(2, 0)
        elif op == "argmin":
            self.inputs = [fill(T.float32, L.GEN_F32_UNIT, 1)]
            self.outputs = [T.empty(1, dtype=T.float32, device=dev), T.empty(1, dtype=T.int32, device=dev)]
            self.temp = L.alloc_temp(L.DeviceReduce.GetArgTempStorageBytes(L.F32, n))
        elif op == "reduce_max":
            self.inputs = [fill(T.int64, L.GEN_I64_UNIFORM, 1)]
            self.outputs = [T.empty(1, dtype=T.int64, device=dev)]
            self.temp = L.alloc_temp(L.DeviceReduce.GetTempStorageBytes(L.I64, n))
        self.rs, self.sc, self.rd = L.DeviceRadixSort(), L.DeviceScan(), L.DeviceReduce()
        self.sl = L.DeviceSelect()

    def step(self, inputs=None, outputs=None):
        op, n, i, o, t = self.op, self.n, inputs or self.inputs, outputs or self.outputs, self.temp
        if op == "sort":
            self.rs.SortKeys(t, i[0], o[0], n)
        elif op == "bits":
            self.rs.SortKeys(t, i[0], o[0], n, 8, 24)
        elif op.startswith("pairs"):
            self.rs.SortPairs(t, i[0], o[0], i[1], o[1], n)
        elif op == "merge":
            self.merge_sorted(i[0], i[1], o[0])
        elif op == "decomposed":
            self.rs.SortKeys(t, i[0], o[0], n, self.dec)
        elif op == "segsort":
            b, e, nseg = self.seg
            self.ss.SortKeys(t, i[0], o[0], n, nseg, b, e)
        elif op == "scan":
            self.sc.InclusiveSum(t, i[0], o[0], n)
        elif op == "reduce":
            self.rd.Sum(t, i[0], o[0], n)
        elif op == "reduce_max":
            self.rd.Max(t, i[0], o[0], n)
        elif op == "argmin":
            self.rd.ArgMin(t, i[0], o[0], o[1], n)
        elif op == "select":
            self.sl.If(t, i[0], o[0], o[1], n, self.pred)
        elif op == "scan_by_key":
            self.sc.InclusiveSumByKey(t, i[0], i[1], o[0], n)
        elif op == "reduce_by_key":
            self.rd.ReduceByKey(t, i[0], i[1], o[0], o[1], o[2], self.L.OP_SUM, n)

    def dominant_kind(self):
        L = self.L
        if self.op in ("scan",):
            return L.KERNEL_SCAN
        if self.op.endswith("by_key"):
            return L.KERNEL_BY_KEY
        if self.op.startswith("reduce"):
            return L.KERNEL_REDUCE
        if self.op == "segsort":
            return L.KERNEL_SEGMENT_BLOCK
        if self.op == "merge":
            return L.KERNEL_MERGE
        if self.op == "argmin":
            return L.KERNEL_ARG_REDUCE
        if self.op.endswith("by_key"):
            return L.KERNEL_BY_KEY
        if self.op == "select":
            return L.KERNEL_SELECT
        return L.KERNEL_SORT_ONESWEEP


def segsort_offsets(n: int):
    """Contiguous segments of 1..2047 keys covering [0, n) (seed 1)."""
    import numpy as np
    rng = np.random.default_rng(1)
    sizes = rng.integers(1, 2048, n // 1024 + 2)
    cum = np.concatenate([[0], np.cumsum(sizes)])
    cum = cum[cum < n]
    return cum.astype(np.uint32), np.concatenate([cum[1:], [n]]).astype(np.uint32)


def cpu_fn(op: str, n_sample: int, threads: int):
    """One run of the oracle port on a bounded sample of the workload (the
    reference tests' host algorithms restated)."""
    from oracle import oracle as O
    if op == "decomposed":
        p = O.generate(O.GEN_U32_UNIFORM, n_sample, seed=1)
        s = O.generate(O.GEN_U32_UNIFORM, n_sample, seed=2).view("int32")
        # the reference tests' host oracle: std::stable_sort by (primary, secondary)
        return lambda: O.decomposed_sort_order([p, s])
    if op == "merge":
        import numpy as np
        x = O.generate(O.GEN_U32_UNIFORM, n_sample, seed=1)
        a, b = np.sort(x[: n_sample // 2]), np.sort(x[n_sample // 2:])
        # the reference tests' host merge: std::merge (ties from the first run)
        return lambda: np.concatenate([a, b])[np.argsort(np.concatenate([a, b]), kind="stable")]
    if op == "segsort":
        x = O.generate(O.GEN_U32_UNIFORM, n_sample, seed=1)
        b, e = segsort_offsets(n_sample)
        return lambda: O.segmented_radix_sort(x, None, b, e)
    if op.startswith("dist"):
        # LSD radix sort time does not depend on the key distribution: the
        # uniform seed-7 stream stands in for both distributed workloads
        x = O.generate(O.GEN_U32_UNIFORM, n_sample, seed=7)
        return lambda: O.radix_sort(x, threads=threads)
    if op in ("sort", "bits"):
        x = O.generate(O.GEN_U32_UNIFORM, n_sample, seed=0 if op == "sort" else 1)
        kw = dict(begin_bit=8, end_bit=24) if op == "bits" else {}
        return lambda: O.radix_sort(x, threads=threads, **kw)
    if op.startswith("pairs"):
        dist = {"pairs": O.GEN_U32_UNIFORM, "pairs_f32": O.GEN_F32_UNIT, "pairs_u64": O.GEN_U64_UNIFORM}[op]
        x = O.generate(dist, n_sample, seed=1)
        v = O.generate(O.GEN_U32_INDEX, n_sample, seed=1)
        return lambda: O.radix_sort(x, v, threads=threads)
    if op == "scan":
        x = O.generate(O.GEN_I32_SCAN, n_sample, seed=1)
        return lambda: O.scan(x, "inclusive")
    if op == "reduce":
        x = O.generate(O.GEN_F32_UNIT, n_sample, seed=1)
        return lambda: O.sum_f64(x)
    if op == "argmin":
        x = O.generate(O.GEN_F32_UNIT, n_sample, seed=1)
        return lambda: O.arg_extremum(x, True)
    if op == "select":
        x = O.generate(O.GEN_U32_UNIFORM, n_sample, seed=1).view("int32")
        return lambda: O.select(x, O.clause_mask(x, [(6, 0, 2, 0)]))
    if op in ("scan_by_key", "reduce_by_key"):
        import numpy as np
        k = (np.arange(n_sample, dtype=np.int64) // 100).astype(np.int32)
        v = O.generate(O.GEN_I32_SCAN, n_sample, seed=1)
        if op == "scan_by_key":
            return lambda: O.scan_by_key(k, v, "inclusive")
        return lambda: O.reduce_by_key(k, v, O.OP_SUM)
    x = O.generate(O.GEN_I64_UNIFORM, n_sample, seed=1)
    return lambda: O.reduce(x, O.OP_MAX, -(1 << 63))


def cpu_sample(op: str, n_sample: int, threads: int, min_seconds: float):
    """Items per second of the oracle port over at least min_seconds."""
    fn = cpu_fn(op, n_sample, threads)
    fn()
    reps, t0 = 0, time.perf_counter()
    while True:
        fn()
        reps += 1
        el = time.perf_counter() - t0
        if el >= min_seconds:
            break
    return n_sample * reps / el, reps


def cpu_threads_for(op: str) -> int:
    from oracle import oracle as O
    # the sort restatement is multi-threaded; the scan / reduce host
    # references of the reference's tests are sequential
    # (the segmented restatement is a single-threaded numpy stable sort)
    return O.cpu_threads() if (op in ("sort", "bits") or op.startswith(("pairs", "dist"))) else 1


def reference_items(op: str, log2n: int) -> int:
    """Items one step of the reference arm processes: the full workload of the
    op's configuration when the host finishes it in about a second per step
    (the sorts up to 2^28 keys, the linear scans and reductions up to 2^30
    items), else a 2^26-item sample (the distributed 2^32-key sort,
    the segmented and decomposed sorts)."""
    if op in ("sort", "bits", "pairs", "pairs_f32", "pairs_u64", "merge"):
        return 1 << min(log2n, 28)
    if op in ("scan", "reduce", "reduce_max", "argmin", "select", "scan_by_key", "reduce_by_key"):
        return 1 << min(log2n, 30)
    return 1 << min(log2n, 26)


def single_thread_sort_leg(n: int, seed: int, min_seconds: float = 3.0):
    """The reference tests' own host check, a single-threaded comparison sort
    (std::sort, tests/device_radix_sort_one_sweep.cpp:169), restated with
    numpy's sort on one thread: keys per second over at least min_seconds."""
    from oracle import oracle as O
    x = O.generate(O.GEN_U32_UNIFORM, n, seed=seed)
    np_sort = __import__("numpy").sort
    reps, t0 = 0, time.perf_counter()
    while True:
        np_sort(x)
        reps += 1
        el = time.perf_counter() - t0
        if el >= min_seconds:
            break
    return n * reps / el, reps


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    cfg = OPS[args.op]
    log2n = args.log2n or cfg["log2n"]
    threads = cpu_threads_for(args.op)
    n_items = reference_items(args.op, log2n)
    fn = cpu_fn(args.op, n_items, threads)
    for _ in range(args.warmup):
        fn()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        fn()
    el = time.perf_counter() - t0
    v = n_items * args.steps / el / 1e9
    full = n_items == (1 << log2n) and not cfg.get("distributed")
    lg = n_items.bit_length() - 1
    how = ("multi-threaded LSD restatement of the onesweep semantics" if threads > 1
           else "sequential host reference of the reference's tests")
    sample = (f"the full workload (2^{lg} items) per step; {how}" if full
              else f"2^{lg} items of the {cfg['workload']} stream per step; {how}")
    line = {
        "impl": "reference", "metric": cfg["metric"], "value": v, "unit": cfg["unit"], "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": el / args.steps * 1e3,
        "higher_is_better": True, "scaling": "strong" if cfg.get("distributed") else "weak", "vs_baseline": None,
        "dtype": cfg["dtype"], "data": DATA,
        "config": {"workload": f"{cfg['workload']}, n=2^{log2n} " + ("in total" if cfg.get("distributed") else "per GPU"),
                   "items_per_step": n_items, "same_config": full},
        "cpu_baseline": {"value": v, "unit": cfg["unit"], "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": v, "unit": cfg["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    if args.op in ("sort", "bits"):
        ips, reps = single_thread_sort_leg(n_items, 0 if args.op == "sort" else 1)
        line["cpu_baseline"]["single_thread"] = {
            "value": ips / 1e9, "unit": cfg["unit"], "cores": 1, "kind": "port",
            "sample": f"2^{lg} keys x {reps} runs of numpy.sort on one thread (the reference tests' std::sort check)"}
    print(json.dumps(line), flush=True)
    return 0


CUB_OPS = {"sort": 0, "pairs": 1, "scan": 2, "reduce": 3}


def run_cub(args):
    """The same workload through cub::DeviceRadixSort / DeviceScan /
    DeviceReduce (luisacompute-parallelprimitive_b200/cub_arm), device-resident
    inputs, CUDA events around the timed steps."""
    import ctypes

    import torch
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    cfg = OPS[args.op]
    if args.op not in CUB_OPS:
        print(json.dumps({"impl": "cub", "unavailable": f"no CUB arm for --op {args.op}"}), flush=True)
        return 0
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
    log2n = args.log2n or cfg["log2n"]
    n = 1 << log2n
    so = ROOT / "luisacompute-parallelprimitive_b200" / "lcpp_b200" / "libcub_arm.so"
    lib = ctypes.CDLL(str(so))
    vp = ctypes.c_void_p
    lib.cub_arm_run.argtypes = [ctypes.c_int, vp, ctypes.POINTER(ctypes.c_size_t), vp, vp, vp, vp, ctypes.c_uint64,
                                vp]
    lib.cub_arm_run.restype = ctypes.c_int
    ver = lib.cub_arm_version()
    w = Workload(args.op, n)  # same generators and seeds as our arm
    i, o = w.inputs, w.outputs
    ptr = lambda lst, k: vp(lst[k].data_ptr()) if len(lst) > k else vp(0)  # noqa: E731
    op = CUB_OPS[args.op]
    stream = torch.cuda.current_stream()
    nbytes = ctypes.c_size_t(0)
    assert lib.cub_arm_run(op, None, ctypes.byref(nbytes), ptr(i, 0), ptr(o, 0), ptr(i, 1), ptr(o, 1), n,
                           vp(stream.cuda_stream)) == 0
    temp = torch.empty(max(nbytes.value, 1), dtype=torch.uint8, device="cuda")

    def step():
        assert lib.cub_arm_run(op, vp(temp.data_ptr()), ctypes.byref(nbytes), ptr(i, 0), ptr(o, 0), ptr(i, 1),
                               ptr(o, 1), n, vp(stream.cuda_stream)) == 0

    for _ in range(args.warmup):
        step()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e0.record(stream)
    for _ in range(args.steps):
        step()
    e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    value = n / (ms * 1e-3) / 1e9
    print(json.dumps({
        "impl": "cub", "metric": cfg["metric"], "value": value, "unit": cfg["unit"], "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": cfg["dtype"], "data": DATA,
        "config": {"workload": f"{cfg['workload']}, n=2^{log2n}", "library": f"CUB {ver // 100000}.{ver // 100 % 1000}.{ver % 100} "
                                                                           "(CUDA toolkit headers)",
                   "l2": "inputs larger than L2; no flush"},
        "op_roofline": {"bytes_per_item": cfg["bytes"], "achieved": cfg["bytes"] * n / (ms * 1e-3) / 1e9}}),
        flush=True)
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
    cfg = OPS[args.op]
    log2n = args.log2n or cfg["log2n"]
    n = 1 << log2n

    if world > 1 or cfg.get("distributed"):
        import socket

        import torch.distributed as dist
        from datetime import timedelta

        from lcpp_b200 import distributed as D
        # stdout carries exactly one JSON line: whatever NCCL prints on its own
        # (its version banner goes to file descriptor 1) is sent to stderr
        sys.stdout.flush()
        json_out = os.dup(1)
        os.dup2(2, 1)
        init = {}
        if world == 1 and "MASTER_ADDR" not in os.environ:  # one process, no torchrun
            with socket.socket() as sk:
                sk.bind(("127.0.0.1", 0))
                port = sk.getsockname()[1]
            init = dict(init_method=f"tcp://127.0.0.1:{port}", rank=0, world_size=1)
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local),
                                **init)
        rc = 0
        try:
            if cfg.get("distributed"):  # fixed total, sharded evenly (strong scaling)
                n_local = (1 << log2n) // world
                res = D.bench_distributed_sort(n_local, args.steps, args.warmup, dist, ClockSampler,
                                               measured_peak(), seed=cfg["seed"], zipf=cfg["zipf"],
                                               metric=cfg["metric"], scaling="strong")
            else:  # the default sort: 2^28 keys per GPU (weak scaling), plus 2^32 keys in total
                res = D.bench_distributed_sort(n, args.steps, args.warmup, dist, ClockSampler, measured_peak(),
                                               strong_2p32=world > 1)
            if rank == 0 and world == 1 and not args.no_cpu_baseline:
                threads = cpu_threads_for("sort")
                ips, reps = cpu_sample("sort", 1 << 24, threads, 10.0)
                res["cpu_baseline"] = {"value": ips / 1e9, "unit": "Gkeys/s", "cores": threads, "kind": "port",
                                       "sample": f"2^24 keys of the uniform u32 stream x {reps} runs; "
                                                 "multi-threaded LSD restatement of the onesweep semantics"}
            if rank == 0:
                os.write(json_out, (json.dumps(res) + "\n").encode())
            dist.barrier()
            if not res.get("parity_bit_exact", True):
                rc = 1
        finally:
            dist.destroy_process_group()
            sys.stdout.flush()
            os.dup2(json_out, 1)
            os.close(json_out)
        return rc

    w = Workload(args.op, n)
    stream = torch.cuda.current_stream()
    for _ in range(args.warmup):
        w.step()
    torch.cuda.synchronize()
    if w.temp is not None:
        assert L.device_status(w.temp) == L.OK

    props = torch.cuda.get_device_properties(local)
    bus = getattr(props, "pci_bus_id", None)
    bus_id = f"{bus:02x}:00.0" if isinstance(bus, int) else None
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(bus_id) as clocks:
        L.diag_timing_enable(True)
        torch.cuda.synchronize()
        e0.record(stream)
        for _ in range(args.steps):
            w.step()
        e1.record(stream)
        torch.cuda.synchronize()
        recs = L.diag_timing_read()
        L.diag_timing_enable(False)
    ms = e0.elapsed_time(e1) / args.steps
    if w.temp is not None:
        assert L.device_status(w.temp) == L.OK
    value = n / (ms * 1e-3) / 1e9
    clk = clocks.summary()

    kind = w.dominant_kind()
    dom = [r[1] for r in recs if r[0] == kind]
    avg_ms = sum(dom) / len(dom)
    peak, peak_kind = measured_peak()
    achieved = cfg["kbytes"] * n / (avg_ms * 1e-3) / 1e9
    tpi = profiled_traffic(args.op)
    roofline = {"bound": "hbm", "kernel": cfg["kernel"], "achieved": achieved, "peak": peak,
                "peak_source": peak_kind, "unit": "GB/s", "frac": achieved / peak,
                "algorithmic_bytes_per_launch": cfg["kbytes"] * n, "avg_launch_ms": avg_ms,
                "traffic": (tpi * n) if tpi is not None else None}
    op_ach = cfg["bytes"] * n / (ms * 1e-3) / 1e9
    op_roofline = {"bytes_per_item": cfg["bytes"], "achieved": op_ach, "peak": peak, "unit": "GB/s",
                   "frac": op_ach / peak}
    if kind == L.KERNEL_SORT_ONESWEEP:
        hist = [r[1] for r in recs if r[0] == L.KERNEL_SORT_HISTOGRAM]
        op_roofline.update({"histogram_ms": sum(hist) / len(hist), "onesweep_ms_per_pass": avg_ms})

    # e2e: the same public call with pinned host buffers; every step copies its
    # inputs host -> device, runs the op and copies the result device -> host,
    # pipelined over three streams the way a caller streams batches through the
    # library: the upload of step s+1 and the download of step s-1 overlap the
    # op of step s (double-buffered device buffers; the per-step time is the
    # whole run, fill and drain included, divided by the steps).
    # pinned host buffers are first touched on the GPU's NUMA node
    from lcpp_b200.distributed import bind_to_gpu_numa_node
    all_cpus = os.sched_getaffinity(0)
    numa = bind_to_gpu_numa_node(local)
    host_in = [torch.empty(t.shape, dtype=t.dtype, pin_memory=True).copy_(t) for t in w.inputs]
    host_out = [[torch.empty(t.shape, dtype=t.dtype, pin_memory=True) for t in w.outputs] for _ in range(2)]
    d_in = [[torch.empty_like(t) for t in w.inputs] for _ in range(2)]
    d_out = [[torch.empty_like(t) for t in w.outputs] for _ in range(2)]
    k_e2e = max(3, min(args.steps, 20))
    s_in, s_op, s_out = torch.cuda.Stream(), torch.cuda.Stream(), torch.cuda.Stream()

    def e2e_run(k):
        ev_in, ev_op, ev_out = {}, {}, {}
        first = torch.cuda.Event(enable_timing=True)
        last = torch.cuda.Event(enable_timing=True)
        first.record(s_in)
        for st in range(k):
            b = st % 2
            with torch.cuda.stream(s_in):
                if st >= 2:
                    s_in.wait_event(ev_op[st - 2])  # d_in[b] has been read
                for d, h in zip(d_in[b], host_in):
                    d.copy_(h, non_blocking=True)
                ev_in[st] = torch.cuda.Event()
                ev_in[st].record(s_in)
            with torch.cuda.stream(s_op):
                s_op.wait_event(ev_in[st])
                if st >= 2:
                    s_op.wait_event(ev_out[st - 2])  # d_out[b] has been downloaded
                w.step(d_in[b], d_out[b])
                ev_op[st] = torch.cuda.Event()
                ev_op[st].record(s_op)
            with torch.cuda.stream(s_out):
                s_out.wait_event(ev_op[st])
                for h, d in zip(host_out[b], d_out[b]):
                    h.copy_(d, non_blocking=True)
                ev_out[st] = torch.cuda.Event()
                ev_out[st].record(s_out)
        last.record(s_out)
        torch.cuda.synchronize()
        return first.elapsed_time(last)

    e2e_run(2)
    e2e_ms = e2e_run(k_e2e) / k_e2e
    e2e = {"value": n / (e2e_ms * 1e-3) / 1e9, "unit": cfg["unit"],
           "h2d_bytes_per_step": sum(t.numel() * t.element_size() for t in w.inputs),
           "d2h_bytes_per_step": sum(t.numel() * t.element_size() for t in w.outputs),
           "steps": k_e2e, "ms_per_step": e2e_ms,
           "pipeline": "3 streams: H2D of step s+1 and D2H of step s-1 overlap the op of step s",
           "numa_node": numa}
    os.sched_setaffinity(0, all_cpus)  # the CPU baseline below uses every host core
    host_out = host_out[(k_e2e - 1) % 2]
    if args.op in ("sort", "bits", "merge"):  # sanity: what came back is ordered
        ho = host_out[0].numpy()
        if args.op == "bits":
            ho = (ho >> 8) & 0xFFFF
        assert bool((ho[1:] >= ho[:-1]).all())

    cpu = None
    if not args.no_cpu_baseline and rank == 0:
        threads = cpu_threads_for(args.op)
        ips, reps = cpu_sample(args.op, 1 << 24, threads, 10.0)
        cpu = {"value": ips / 1e9, "unit": cfg["unit"], "cores": threads, "kind": "port",
               "sample": f"2^24 items of the {cfg['workload']} stream x {reps} runs; "
                         + ("multi-threaded LSD restatement of the onesweep semantics" if threads > 1
                            else "sequential host reference of the reference's tests")}
        if args.op in ("sort", "bits"):
            ips1, reps1 = single_thread_sort_leg(1 << 24, 0 if args.op == "sort" else 1)
            cpu["single_thread"] = {"value": ips1 / 1e9, "unit": cfg["unit"], "cores": 1, "kind": "port",
                                    "sample": f"2^24 keys x {reps1} runs of numpy.sort on one thread "
                                              "(the reference tests' std::sort check)"}

    line = {
        "metric": cfg["metric"], "value": value, "unit": cfg["unit"], "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": cfg["dtype"], "data": DATA,
        "config": {"workload": f"{cfg['workload']}, n=2^{log2n} per GPU", "items_per_gpu": n,
                   "parallelism": "single GPU",
                   "l2": f"inputs larger than L2 ({n * w.inputs[0].element_size() / 2**20:.0f} MiB per step "
                         "vs 126 MB L2); no flush"},
        "roofline": roofline, "op_roofline": op_roofline, "e2e": e2e,
        "gpu_launches": len(recs), "clocks": clk, "cpu_baseline": cpu,
    }
    print(json.dumps(line), flush=True)
    return 0


def main():
    args = parse_args()
    if args.impl == "reference":
        return run_reference(args)
    if args.impl == "cub":
        return run_cub(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
