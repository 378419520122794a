/*
 * lcpp_b200_dist.h -- device building blocks of the distributed sort.
 *
 * No counterpart in the reference (LCPP is single-GPU; it has no NCCL, MPI
 * or peer-copy code).  The distributed sort itself is orchestrated on the
 * host (luisacompute-parallelprimitive_b200/lcpp_b200/distributed.py) with
 * torch.distributed over NCCL for the exchange; these calls are the device
 * work it needs besides the local sorts.
 */
#ifndef LCPP_B200_DIST_H
#define LCPP_B200_DIST_H

#include <stdint.h>

#include "lcpp_b200.h"

#ifdef __cplusplus
extern "C" {
#endif

/* For each query q[i] (an order-preserving key image: the key after the
 * sort's ascending bijection, as unsigned 32-bit for 4-byte keys or 64-bit
 * for 8-byte keys), out[i] = number of keys of `sorted` (n keys of key_dtype,
 * sorted ascending by DeviceRadixSort) whose image is < q[i] (upper == 0)
 * or <= q[i] (upper != 0).  +-0.0 have the same image (as when sorting). */
lcpp_status lcpp_dist_search_sorted(const void* sorted, uint64_t n, const void* queries, uint64_t num_queries,
                                    int upper, uint64_t* out, lcpp_dtype key_dtype, lcpp_stream_t stream);

/* Temp bytes of lcpp_dist_merge_sorted for `total` = na + nb keys (the split
 * points of the output blocks). */
lcpp_status lcpp_dist_merge_temp_bytes(uint64_t total, size_t* temp_bytes);

/* Merge two runs sorted ascending by DeviceRadixSort (keys of key_dtype,
 * compared by the same order-preserving image): out[0, na + nb) receives the
 * merged keys; among equal images the keys of `a` come first.  `out` must not
 * overlap `a` or `b`; temp (256-byte aligned) holds the output blocks' split
 * points.  Merge path (Green, McColl & Bader, 2012): one small kernel finds
 * each output block's split point by binary search, a second merges each
 * block in shared memory. */
lcpp_status lcpp_dist_merge_sorted(void* temp, size_t temp_bytes, const void* a, uint64_t na, const void* b,
                                   uint64_t nb, void* out, lcpp_dtype key_dtype, lcpp_stream_t stream);

/* Batched form: `count` (1..LCPP_MERGE_BATCH_MAX) independent merges
 * out[i] = merge(a[i][0, na[i]), b[i][0, nb[i])) in one split launch and one
 * merge launch (one level of a merge tree).  Same ordering, overlap and
 * alignment rules as lcpp_dist_merge_sorted; the runs may live in another
 * GPU's memory (pointers from lcpp_dist_ipc_open). */
#define LCPP_MERGE_BATCH_MAX 32
lcpp_status lcpp_dist_merge_batch_temp_bytes(int count, const uint64_t* na, const uint64_t* nb, size_t* temp_bytes);
lcpp_status lcpp_dist_merge_sorted_batch(void* temp, size_t temp_bytes, int count, const void* const* a,
                                         const uint64_t* na, const void* const* b, const uint64_t* nb,
                                         void* const* out, lcpp_dtype key_dtype, lcpp_stream_t stream);

/* Exchange buffers shared between the processes of one node (CUDA IPC), so
 * that a rank's merge kernel reads the sorted runs of the other ranks straight
 * from their memory over NVLink (plain loads).  Set-up calls, not hot-path
 * calls: the distributed sort allocates its buffers once and reuses them.
 *
 * lcpp_dist_ipc_alloc: cudaMalloc of `bytes` on the current device and its
 *   IPC handle (LCPP_IPC_HANDLE_BYTES bytes written to `handle`).
 * lcpp_dist_ipc_open: maps another process's buffer from its handle on the
 *   current device (peer access enabled lazily); `*dptr` is usable by kernels
 *   on this device.
 * lcpp_dist_ipc_close: unmaps a buffer opened with lcpp_dist_ipc_open.
 * lcpp_dist_ipc_free: frees a buffer from lcpp_dist_ipc_alloc (after every
 *   peer has closed its mapping). */
#define LCPP_IPC_HANDLE_BYTES 64
lcpp_status lcpp_dist_ipc_alloc(size_t bytes, void** dptr, void* handle);
lcpp_status lcpp_dist_ipc_open(const void* handle, void** dptr);
lcpp_status lcpp_dist_ipc_close(void* dptr);
lcpp_status lcpp_dist_ipc_free(void* dptr);

#ifdef __cplusplus
} /* extern "C" */
#endif

#endif /* LCPP_B200_DIST_H */
