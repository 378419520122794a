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
     rounds the prefix is the exact boundary key k_j (for 32-bit keys all
     of it in device tensors, one host wait at the end);
  3. keys equal to k_j are split between the ranks below and above the
     boundary in rank order, so every rank receives exactly its share even
     when one key value fills several ranks (heavy hitters);
  4. exchange and merge.  Ranks of one node whose GPUs reach each other
     (NVLink / NVSwitch peer access): the local sort writes into an exchange
     buffer shared with the other ranks through CUDA IPC, and each rank's
     first merge level reads its G incoming runs straight from the other
     ranks' buffers with plain loads over NVLink (no all-to-all buffer in
     between); the remaining ceil(log2 G) - 1 levels merge locally.
     Otherwise: one NCCL all-to-all of the sorted runs, then the pairwise
     merge of the G received runs.  Merging adjacent runs with ties taken
     from the left keeps equal keys in rank order (the result is the stable
     global sort).
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
        self._peer = None
        self._exchange = None

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

    def search_bits(self, sorted_keys, queries, upper: bool):
        """search() with the queries already a device tensor holding key images
        of the key width (int32 / int64 with the image's bits)."""
        torch = self.torch
        out = torch.empty(queries.numel(), dtype=torch.int64, device=self.device)
        if queries.numel():
            self.launches += 1
            check(lib().lcpp_dist_search_sorted(
                ctypes.c_void_p(sorted_keys.data_ptr()), sorted_keys.numel(), ctypes.c_void_p(queries.data_ptr()),
                queries.numel(), int(upper), ctypes.c_void_p(out.data_ptr()), dtype_code(sorted_keys),
                ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)), "lcpp_dist_search_sorted")
        return out

    def local_sort_into(self, keys, out_ptr):
        """SortKeys of `keys` (all bits) into the device buffer at out_ptr."""
        n = keys.numel()
        if n == 0:
            return
        code = dtype_code(keys)
        temp = self._temp("sort", DeviceRadixSort.GetSortKeysTempStorageBytes(code, n))
        check(lib().lcpp_radix_sort_keys(
            ctypes.c_void_p(temp.data_ptr()), temp.numel(), ctypes.c_void_p(keys.data_ptr()),
            ctypes.c_void_p(out_ptr), n, 0, keys.element_size() * 8, 0, code,
            ctypes.c_void_p(self.torch.cuda.current_stream().cuda_stream)), "lcpp_radix_sort_keys")

    def merge_batch(self, items, code):
        """One merge level: items = [(a_ptr, na, b_ptr, nb, out_ptr), ...],
        stable merges of sorted runs given as device pointers (local or mapped
        from a peer), all in one split launch and one merge launch (per 32)."""
        items = [it for it in items if it[1] + it[3] > 0]
        stream = ctypes.c_void_p(self.torch.cuda.current_stream().cuda_stream)
        for c0 in range(0, len(items), 32):
            chunk = items[c0:c0 + 32]
            k = len(chunk)
            pa = (ctypes.c_void_p * k)(*[it[0] for it in chunk])
            na = (ctypes.c_uint64 * k)(*[it[1] for it in chunk])
            pb = (ctypes.c_void_p * k)(*[it[2] for it in chunk])
            nb = (ctypes.c_uint64 * k)(*[it[3] for it in chunk])
            po = (ctypes.c_void_p * k)(*[it[4] for it in chunk])
            nbytes = ctypes.c_size_t(0)
            check(lib().lcpp_dist_merge_batch_temp_bytes(k, na, nb, ctypes.byref(nbytes)),
                  "lcpp_dist_merge_batch_temp_bytes")
            temp = self._temp("merge", nbytes.value)
            self.launches += 2
            check(lib().lcpp_dist_merge_sorted_batch(ctypes.c_void_p(temp.data_ptr()), temp.numel(), k, pa, na, pb,
                                                     nb, po, code, stream), "lcpp_dist_merge_sorted_batch")

    def merge_level(self, pairs):
        """pairs = [(a, b, out), ...] of tensors (b may be None: copy a)."""
        if not pairs:
            return
        self.merge_batch([(a.data_ptr(), a.numel(), b.data_ptr() if b is not None else 0,
                           b.numel() if b is not None else 0, o.data_ptr()) for a, b, o in pairs],
                         dtype_code(pairs[0][0]))

    def peer_capable(self, dist):
        """Whether every pair of ranks shares a node and has GPU peer access
        (decided once, collectively)."""
        if self._peer is None:
            import socket
            import zlib
            torch = self.torch
            G = dist.get_world_size()
            me = [zlib.crc32(socket.gethostname().encode()), self.device.index]
            rows = _all_gather_int64(dist, me, self.device)
            same_host = all(r[0] == rows[0][0] for r in rows)
            ok = same_host and all(torch.cuda.can_device_access_peer(self.device.index, r[1])
                                   for r in rows if r[1] != self.device.index)
            flag = torch.tensor([0 if ok else 1], dtype=torch.int64, device=self.device)
            dist.all_reduce(flag)  # peer mode only when every rank can use it
            self._peer = G > 1 and flag.item() == 0
        return self._peer

    def exchange(self, dist, nbytes):
        """The node's shared exchange buffers, with room for nbytes per rank
        (re-created, collectively, when some rank needs more)."""
        torch = self.torch
        need = torch.tensor([nbytes], dtype=torch.int64, device=self.device)
        dist.all_reduce(need, op=dist.ReduceOp.MAX)
        need = int(need.item())
        if self._exchange is None or self._exchange.capacity < need:
            if self._exchange is not None:
                self._exchange.close(dist)
            self._exchange = PeerExchange(dist, max(need, 256), self.device)
        return self._exchange

    def close(self, dist):
        """Releases the exchange buffers (collective; before the process
        group is destroyed)."""
        if self._exchange is not None:
            self._exchange.close(dist)
            self._exchange = None

    def merge(self, a, b, out):
        """out[:a.numel() + b.numel()] = stable merge of sorted runs a, b."""
        self.merge_level([(a, b, out)])

    def empty_like(self, t):
        return self.torch.empty_like(t)


class _DeviceArray:
    """A device buffer as __cuda_array_interface__ (for a zero-copy torch view)."""

    def __init__(self, ptr, n, itemsize):
        self.__cuda_array_interface__ = {"shape": (n,), "typestr": "<i4" if itemsize == 4 else "<i8",
                                         "data": (ptr, False), "version": 3, "strides": None}


def device_view(ptr, n, dtype):
    """torch tensor of n elements of dtype over device memory at ptr."""
    import torch
    itemsize = torch.empty(0, dtype=dtype).element_size()
    if n == 0:
        return torch.empty(0, dtype=dtype, device="cuda")
    return torch.as_tensor(_DeviceArray(ptr, n, itemsize), device="cuda").view(dtype)


class PeerExchange:
    """Two exchange buffers per rank, shared with every rank of the node
    through CUDA IPC.  Step s of the distributed sort writes this rank's
    sorted keys into buffer s % 2 and the other ranks read their runs from
    it; buffer s % 2 is written again only at step s + 2, after the
    collectives of step s + 1, which no rank passes before its step-s merge
    has run.  Set-up cost (cudaMalloc, handle exchange, mapping) is paid
    once per capacity."""

    def __init__(self, dist, capacity, device):
        import torch
        self.capacity = capacity
        self.rank, G = dist.get_rank(), dist.get_world_size()
        self.local = []
        raw = bytearray()
        for _ in range(2):
            p = ctypes.c_void_p()
            h = (ctypes.c_ubyte * 64)()
            check(lib().lcpp_dist_ipc_alloc(capacity, ctypes.byref(p), h), "lcpp_dist_ipc_alloc")
            self.local.append(p.value)
            raw += bytes(h)
        t = torch.tensor(list(raw), dtype=torch.uint8, device=device)
        parts = [torch.empty_like(t) for _ in range(G)]
        dist.all_gather(parts, t)
        self.ptrs, self.opened = [], []
        for r, part in enumerate(parts):
            if r == self.rank:
                self.ptrs.append(list(self.local))
                continue
            hb = bytes(part.cpu().tolist())
            row = []
            for slot in range(2):
                h = (ctypes.c_ubyte * 64).from_buffer_copy(hb[slot * 64:(slot + 1) * 64])
                p = ctypes.c_void_p()
                check(lib().lcpp_dist_ipc_open(h, ctypes.byref(p)), "lcpp_dist_ipc_open")
                row.append(p.value)
                self.opened.append(p.value)
            self.ptrs.append(row)
        self.step = 0

    def close(self, dist):
        import torch
        torch.cuda.synchronize()
        dist.barrier()  # every rank's reads of the buffers are done
        for p in self.opened:
            check(lib().lcpp_dist_ipc_close(ctypes.c_void_p(p)), "lcpp_dist_ipc_close")
        torch.cuda.synchronize()
        dist.barrier()  # every mapping is gone
        for p in self.local:
            check(lib().lcpp_dist_ipc_free(ctypes.c_void_p(p)), "lcpp_dist_ipc_free")
        self.opened, self.local, self.ptrs = [], [], []


def _all_gather_int64(dist, values, device):
    import torch
    t = torch.tensor(values, dtype=torch.int64, device=device)
    out = [torch.empty_like(t) for _ in range(dist.get_world_size())]
    dist.all_gather(out, t)
    return [o.tolist() for o in out]


def _split_indices(G, sizes, P, below, lo_hi):
    """idx[r][j]: split index of rank r before destination j.  Keys equal to
    boundary key k_j go below the boundary in rank order until the boundary
    holds exactly P_j keys.  lo_hi[r] = lo (G-1 values) ++ hi (G-1 values):
    counts of rank r's keys with image < k_j and <= k_j."""
    idx = [[0] * (G + 1) for _ in range(G)]
    for rr in range(G):
        idx[rr][G] = sizes[rr]
    for j in range(G - 1):
        remaining = P[j] - below[j]  # keys equal to k_j that go below boundary j, in rank order
        for rr in range(G):
            lo_r, hi_r = lo_hi[rr][j], lo_hi[rr][G - 1 + j]
            take = min(hi_r - lo_r, remaining)
            idx[rr][j + 1] = lo_r + take
            remaining -= take
        if remaining != 0:
            raise LcppError(7, "distributed splitter selection is inconsistent")
    return idx


def _exact_splits_32(sorted_keys, dist, ops):
    """exact_splits for 32-bit keys with every step on the device: the
    queries, counts, histograms, cumulative sums and prefix updates stay in
    device tensors, and the host waits once, for the final all-gather."""
    import torch
    G, r = dist.get_world_size(), dist.get_rank()
    dev = ops.device
    n_local = sorted_keys.numel()
    mine = torch.tensor([n_local], dtype=torch.int64, device=dev)
    parts = [torch.empty_like(mine) for _ in range(G)]
    dist.all_gather(parts, mine)
    sizes_t = torch.cat(parts)
    P = torch.arange(1, G, dtype=torch.int64, device=dev) * sizes_t.sum() // G
    prefix = torch.zeros(G - 1, dtype=torch.int64, device=dev)
    below = torch.zeros(G - 1, dtype=torch.int64, device=dev)
    sub = 1 << SUB_BITS
    l_all = torch.arange(sub + 1, dtype=torch.int64, device=dev)

    def as_bits(q):  # values in [0, 2^32) as the int32 with the same bits
        return torch.where(q >= (1 << 31), q - (1 << 32), q).to(torch.int32)

    for rnd in range(32 // SUB_BITS):
        shift = 32 - SUB_BITS * (rnd + 1)
        # query ((prefix << 16) | l) << shift for l in [0, 2^16]; 2^32 (the end
        # of the last prefix range) stands for the key count
        q = ((prefix[:, None] << SUB_BITS) + l_all[None, :]) << shift
        over = q >= (1 << 32)
        counts = ops.search_bits(sorted_keys, as_bits(torch.where(over, torch.zeros_like(q), q)).reshape(-1),
                                 upper=False).view(G - 1, sub + 1)
        counts = torch.where(over, torch.full_like(counts, n_local), counts)
        hist = (counts[:, 1:] - counts[:, :-1]).contiguous()
        dist.all_reduce(hist)
        cum = torch.cumsum(hist, dim=1)
        # first sub-bucket whose cumulative count exceeds the residual rank
        l = torch.searchsorted(cum, (P - below).unsqueeze(1), right=True).squeeze(1)
        below = below + torch.where(l > 0, cum.gather(1, (l - 1).clamp_min(0).unsqueeze(1)).squeeze(1),
                                    torch.zeros_like(l))
        prefix = (prefix << SUB_BITS) | l
    kq = as_bits(prefix)
    lo = ops.search_bits(sorted_keys, kq, upper=False)
    hi = ops.search_bits(sorted_keys, kq, upper=True)
    row = torch.cat([lo, hi, below, P, sizes_t])
    parts = [torch.empty_like(row) for _ in range(G)]
    dist.all_gather(parts, row)
    rows = torch.stack(parts).tolist()  # the one host wait
    m = G - 1
    below_l, P_l, sizes = rows[0][2 * m:3 * m], rows[0][3 * m:4 * m], rows[0][4 * m:]
    idx = _split_indices(G, sizes, P_l, below_l, [rw[:2 * m] for rw in rows])
    send = [idx[r][j + 1] - idx[r][j] for j in range(G)]
    recv = [idx[i][r + 1] - idx[i][r] for i in range(G)]
    return send, recv, idx


def exact_splits(sorted_keys, dist, ops):
    """Split indices of this rank's sorted keys so that rank j receives global
    sorted positions [P_j, P_{j+1}).  Returns (send_counts, recv_counts, idx)
    where idx[r][j] is the split index of rank r before destination j."""
    import torch
    if sorted_keys.element_size() == 4 and hasattr(ops, "search_bits"):
        return _exact_splits_32(sorted_keys, dist, ops)
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
    idx = _split_indices(G, sizes, P, below, gathered)
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


def distributed_sort_keys(keys_local, dist, ops=None, exchange="auto"):
    """Globally sort the keys held by all ranks; returns this rank's slice of
    the result (global positions [floor(r N / G), floor((r+1) N / G))).
    exchange: "peer" (merge straight from the other ranks' memory, ranks of
    one node with peer access), "nccl" (all-to-all, then merge) or "auto"."""
    import torch
    G, r = dist.get_world_size(), dist.get_rank()
    if ops is None:  # one-off call: the exchange buffers live for this call only
        ops = GpuOps()
        try:
            return distributed_sort_keys(keys_local, dist, ops, exchange)
        finally:
            ops.close(dist)
    if G == 1:
        return ops.local_sort(keys_local)
    peer = exchange == "peer" or (exchange == "auto" and hasattr(ops, "peer_capable") and ops.peer_capable(dist))
    if not peer:
        local = ops.local_sort(keys_local)
        send, recv, _ = exact_splits(local, dist, ops)
        out = torch.empty(sum(recv), dtype=local.dtype, device=local.device)
        dist.all_to_all_single(_bitcast_for_comm(out), _bitcast_for_comm(local), recv, send)
        return merge_runs(out, recv, ops)

    kb = keys_local.element_size()
    n = keys_local.numel()
    ex = ops.exchange(dist, n * kb)
    slot = ex.step & 1
    ex.step += 1
    ops.local_sort_into(keys_local, ex.ptrs[r][slot])
    local = device_view(ex.ptrs[r][slot], n, keys_local.dtype)
    _, recv, idx = exact_splits(local, dist, ops)
    code = dtype_code(keys_local)
    total = sum(recv)
    # first level straight from the owners' exchange buffers (run i = the
    # keys rank i sends here, in rank order), into `out`
    runs = [(ex.ptrs[i][slot] + idx[i][r] * kb, idx[i][r + 1] - idx[i][r]) for i in range(G)]
    out = torch.empty(total, dtype=keys_local.dtype, device=keys_local.device)
    counts, items, pos = [], [], 0
    for i in range(0, G, 2):
        (pa, na), (pb, nb) = runs[i], runs[i + 1] if i + 1 < G else (0, 0)
        items.append((pa, na, pb, nb, out.data_ptr() + pos * kb))
        counts.append(na + nb)
        pos += na + nb
    ops.merge_batch(items, code)
    return merge_runs(out, counts, ops)


def merge_runs(buf, counts, ops):
    """Merge the consecutive sorted runs of `buf` (lengths `counts`, in rank
    order) into one sorted run: pairwise merge-path levels ping-ponging
    between `buf` and one scratch buffer, each level one batch of merges (a
    run without a partner is copied).  Merging adjacent runs with ties taken
    from the left run keeps equal keys in rank order."""
    bounds = [0]
    for c in counts:
        bounds.append(bounds[-1] + int(c))
    runs = [(bounds[i], bounds[i + 1]) for i in range(len(counts))]
    src, dst = buf, None
    while len(runs) > 1:
        if dst is None:
            dst = ops.empty_like(buf)
        nxt, level = [], []
        for i in range(0, len(runs), 2):
            if i + 1 == len(runs):
                s0, s1 = runs[i]
                level.append((src[s0:s1], None, dst[s0:s1]))
                nxt.append(runs[i])
                continue
            (a0, a1), (b0, b1) = runs[i], runs[i + 1]
            level.append((src[a0:a1], src[b0:b1], dst[a0:b1]))
            nxt.append((a0, b1))
        ops.merge_level(level)
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
class _NoSampler:
    def __enter__(self):
        return self

    def __exit__(self, *exc):
        return False

    def summary(self):
        return None


def bench_distributed_sort(n_local, steps, warmup, dist, clock_sampler_cls, peak, seed=0, zipf=False,
                           metric="Gkeys/s uint32 SortKeys @2^28", scaling="weak"):
    """Benchmark of distributed_sort_keys: n_local u32 keys per rank (rank r
    holds elements [r n, (r+1) n) of the `seed` stream, uniform or Zipf(1.1)
    hashed).  Device time per step is the max over ranks.  Checks on the
    last warm-up result: every rank's slice is sorted, slices are ordered
    across ranks and balanced, and the order-independent fingerprints (sum,
    sum of squares, xor; 64-bit wrapping) of all outputs equal those of all
    inputs."""
    import torch

    from . import (GEN_U32_UNIFORM, GEN_U32_ZIPF, KERNEL_SORT_ONESWEEP, diag_timing_enable, diag_timing_read,
                   testgen_fill)
    G, r = dist.get_world_size(), dist.get_rank()
    dev = torch.device("cuda", torch.cuda.current_device())
    keys = torch.empty(n_local, dtype=torch.uint32, device=dev)
    testgen_fill(keys, GEN_U32_ZIPF if zipf else GEN_U32_UNIFORM, seed=seed, offset=r * n_local)
    ops = GpuOps()
    out = keys
    for _ in range(warmup):
        out = distributed_sort_keys(keys, dist, ops)
    torch.cuda.synchronize()
    dist.barrier()

    # checks in chunks of 2^26 keys (int64 copies of 2^32 keys would not fit)
    K = 0x9E3779B97F4A7C15 - (1 << 64)  # odd multiplier as a wrapping int64

    def fingerprint(t):
        f = torch.zeros(4, dtype=torch.int64, device=dev)
        for c in range(0, t.numel(), 1 << 26):
            x = t[c:c + (1 << 26)].view(torch.int32).to(torch.int64) & 0xFFFFFFFF
            f += torch.stack([x.sum(), (x * x).sum(), (x * K).sum(), torch.tensor(x.numel(), device=dev)])
        return f

    ok = out.numel() == n_local
    for c in range(0, out.numel(), 1 << 26):
        x = out[c:c + (1 << 26) + 1].view(torch.int32).to(torch.int64) & 0xFFFFFFFF
        ok = ok and bool((x[1:] >= x[:-1]).all())
    lo_hi = (out.view(torch.int32)[[0, -1]].to(torch.int64) & 0xFFFFFFFF if out.numel()
             else torch.zeros(2, dtype=torch.int64, device=dev))
    edges = torch.cat([lo_hi, torch.tensor([int(ok)], dtype=torch.int64, device=dev)])
    all_edges = [torch.empty_like(edges) for _ in range(G)]
    dist.all_gather(all_edges, edges)
    fp = torch.stack([fingerprint(keys), fingerprint(out)])
    dist.all_reduce(fp)
    e = [t.tolist() for t in all_edges]
    ordered = all(x[2] for x in e) and all(e[i][1] <= e[i + 1][0] for i in range(G - 1))
    same_multiset = bool(torch.equal(fp[0], fp[1]))
    props = torch.cuda.get_device_properties(dev)
    bus = getattr(props, "pci_bus_id", None)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    stream = torch.cuda.current_stream()
    # one nvidia-smi sampler (rank 0) for the whole job: a sampler per rank
    # adds NVML queries of every GPU while the ranks are being timed
    sampler = clock_sampler_cls(f"{bus:02x}:00.0" if isinstance(bus, int) else None) if r == 0 else _NoSampler()
    with sampler as clocks:
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

    # e2e: pinned host keys -> device, distributed sort, sorted slice -> host,
    # pipelined over three streams (upload of step s+1 and download of step
    # s-1 overlap the sort of step s; double-buffered device inputs).
    host_in = torch.empty(n_local, dtype=torch.uint32, pin_memory=True).copy_(keys)
    host_out = [torch.empty(n_local, dtype=torch.uint32, pin_memory=True) for _ in range(2)]
    d_in = [torch.empty_like(keys) for _ in range(2)]
    k_e2e = max(3, min(steps, 10))
    s_in, s_out = torch.cuda.Stream(), torch.cuda.Stream()

    def e2e_run(k):
        ev_in, ev_op = {}, {}
        first, last = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        first.record(s_in)

        def upload(st):
            with torch.cuda.stream(s_in):
                if st >= 2:
                    s_in.wait_event(ev_op[st - 2])  # d_in[st % 2] has been sorted
                d_in[st % 2].copy_(host_in, non_blocking=True)
                ev_in[st] = torch.cuda.Event()
                ev_in[st].record(s_in)

        upload(0)
        for st in range(k):
            if st + 1 < k:
                upload(st + 1)
            stream.wait_event(ev_in[st])
            res = distributed_sort_keys(d_in[st % 2], dist, ops)
            ev_op[st] = torch.cuda.Event()
            ev_op[st].record(stream)
            with torch.cuda.stream(s_out):
                s_out.wait_event(ev_op[st])
                res.record_stream(s_out)
                host_out[st % 2][: res.numel()].copy_(res, non_blocking=True)
        last.record(s_out)
        torch.cuda.synchronize()
        return first.elapsed_time(last)

    e2e_run(2)
    dist.barrier()
    e2e_ms = torch.tensor([e2e_run(k_e2e) / k_e2e], dtype=torch.float64, device=dev)
    dist.all_reduce(e2e_ms, op=dist.ReduceOp.MAX)
    e2e_ms = e2e_ms.item()

    ops.close(dist)
    onesweep = [x[1] for x in recs if x[0] == KERNEL_SORT_ONESWEEP]
    avg_pass = sum(onesweep) / max(1, len(onesweep))
    achieved = 8 * n_local / (avg_pass * 1e-3) / 1e9
    peak_gbs, peak_src = peak
    # per GPU in HBM: the local sort (4 passes x 8 B/key + 4 B/key histogram read); NCCL
    # exchange: the all-to-all (read + write 8 B/key) and ceil(log2 G) merge levels (8 B/key
    # each); peer exchange: the first merge level reads the runs where they lie (this GPU's
    # buffer is read once, by its owner or a peer: 4 B/key) and writes 4 B/key, then
    # ceil(log2 G) - 1 local levels.  (G-1)/G of the keys cross NVLink in each direction.
    levels = (G - 1).bit_length()
    if G == 1:
        hbm_bytes = 36 * n_local
    elif ops.peer_capable(dist):
        hbm_bytes = (36 + 8 + 8 * (levels - 1)) * n_local
    else:
        hbm_bytes = (36 + 8 + 8 * levels) * n_local
    nvlink_bytes = (G - 1) / G * 4 * n_local
    dist_name = "Zipf(1.1) ranks hashed by fmix32" if zipf else "uniform"
    return {
        "metric": metric, "value": value, "unit": "Gkeys/s", "n_gpus": G,
        "steps": steps, "warmup": warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": scaling,
        "vs_baseline": None, "dtype": "u32",
        "data": "synthetic (splitmix64 counter streams; see include/lcpp_b200_testgen.h)",
        "config": {"workload": f"distributed SortKeys u32 {dist_name}, seed {seed}, "
                               f"2^{n_local.bit_length() - 1} keys per GPU (global 2^{(G * n_local).bit_length() - 1})",
                   "items_per_gpu": n_local, "parallelism": f"sort-partitioned over {G} GPUs (NCCL all-to-all)",
                              "multiset_fingerprint_check": same_multiset,
                   "algorithm": "local onesweep into a CUDA-IPC exchange buffer -> exact 16-bit-refined splitters "
                                "(2 all-reduce rounds) -> merge-path merge reading the G runs straight from the "
                                "owners' memory over NVLink (then local merge levels)"
                                if ops.peer_capable(dist) else
                                "local onesweep -> exact 16-bit-refined splitters (2 all-reduce rounds) -> "
                                "NCCL all-to-all -> pairwise merge-path merge of the G received runs",
                   "l2": "inputs larger than L2; no flush", "globally_sorted_check": ordered},
        "roofline": {"bound": "hbm", "kernel": "onesweep_kernel (one 8-bit pass)", "achieved": achieved,
                     "peak": peak_gbs, "peak_source": peak_src, "unit": "GB/s", "frac": achieved / peak_gbs,
                     "algorithmic_bytes_per_launch": 8 * n_local, "avg_launch_ms": avg_pass, "traffic": None},
        "op_roofline": {"hbm_bytes_per_gpu": hbm_bytes, "nvlink_bytes_per_gpu": nvlink_bytes,
                        "target_ms": max(hbm_bytes / (peak_gbs * 1e9), nvlink_bytes / 770e9) * 1e3,
                        "frac": max(hbm_bytes / (peak_gbs * 1e9), nvlink_bytes / 770e9) * 1e3 / ms},
        "e2e": {"value": G * n_local / (e2e_ms * 1e-3) / 1e9, "unit": "Gkeys/s",
                "h2d_bytes_per_step": 4 * n_local * G, "d2h_bytes_per_step": 4 * n_local * G, "steps": k_e2e,
                "ms_per_step": e2e_ms,
                "pipeline": "3 streams per rank: H2D of step s+1 and D2H of step s-1 overlap the sort of step s"},
        "gpu_launches": len(recs) + other_launches, "clocks": clocks.summary(), "cpu_baseline": None,
    }
