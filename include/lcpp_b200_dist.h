/*
 * lcpp_b200_dist.h -- sort, scan and reduce across GPUs, one process per GPU.
 *
 * No counterpart in the reference (LCPP is single-GPU; it has no NCCL, MPI
 * or peer-copy code).  Each distributed call shards one Device-level call of
 * the reference over the ranks of a communicator and gives the result that
 * call gives on the concatenation of the ranks' inputs in rank order:
 *   lcpp_dist_sort_keys       DeviceRadixSort::SortKeys (device_radix_sort.h:399-425)
 *   lcpp_dist_inclusive_sum   DeviceScan::InclusiveSum (device_scan.h:337-346)
 *   lcpp_dist_exclusive_sum   DeviceScan::ExclusiveSum (device_scan.h:321-336)
 *   lcpp_dist_reduce          DeviceReduce::Reduce (device_reduce.h:229-252)
 * The communicator wraps an NCCL communicator (libnccl.so.2 is loaded at
 * run time, only by these calls).  Every rank of the communicator makes the
 * same calls in the same order, each on its own GPU (the current device when
 * the communicator was created), with its own temp storage.  The lower part
 * of this header holds the device building blocks the calls use (sorted
 * search, merge path, CUDA IPC buffers), exported for callers that compose
 * their own exchange.
 */
#ifndef LCPP_B200_DIST_H
#define LCPP_B200_DIST_H

#include <stdint.h>

#include "lcpp_b200.h"

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------------------
 * Communicator
 * ---------------------------------------------------------------------- */
typedef struct lcpp_comm_s* lcpp_comm;

#define LCPP_COMM_ID_BYTES 128

/* A new communicator ID (an NCCL unique ID): one rank creates it and hands
 * the LCPP_COMM_ID_BYTES bytes to every rank by the caller's own means. */
lcpp_status lcpp_comm_unique_id(void* id);

/* Collective: every rank calls it with the same ID and nranks, its own rank,
 * and its GPU current.  Returns LCPP_ERR_COMM when NCCL cannot be loaded or
 * fails. */
lcpp_status lcpp_comm_init(const void* id, int nranks, int rank, lcpp_comm* comm);

/* Wraps a caller-owned ncclComm_t (not destroyed by lcpp_comm_destroy). */
lcpp_status lcpp_comm_from_nccl(void* nccl_comm, lcpp_comm* comm);

/* Releases the communicator and every peer mapping it opened.  Call it after
 * the last distributed call of every rank has completed. */
lcpp_status lcpp_comm_destroy(lcpp_comm comm);

lcpp_status lcpp_comm_rank(lcpp_comm comm, int* rank, int* nranks);

/* ------------------------------------------------------------------------
 * Distributed sort (keys only)
 *
 * Rank r passes its n_r keys and receives the keys at global sorted
 * positions [n_0 + ... + n_{r-1}, n_0 + ... + n_r) of the ascending stable
 * sort of all ranks' keys (concatenated in rank order): as many keys as it
 * passed, so keys_out has the size of keys_in and may be the same buffer.
 * Keys compare as DeviceRadixSort compares them (all bits; -0.0 and +0.0
 * equal, kept in input order).  Every step runs on the device; the call
 * waits on the host once, for the G x (G + 1) split matrix.
 *
 * exchange: LCPP_EXCHANGE_PEER -- ranks of one host read each other's
 *   sorted runs over NVLink (CUDA IPC mappings of the peers' temp storage,
 *   opened at the first call and again whenever a peer's temp allocation
 *   changes; temp must come from cudaMalloc, as PyTorch's caching allocator
 *   does); LCPP_EXCHANGE_NCCL -- NCCL send / receive of the runs;
 *   LCPP_EXCHANGE_COPY -- ranks of one host push their runs into the
 *   receivers' run buffers with copy-engine copies (cudaMemcpyAsync over the
 *   same IPC mappings, one stream per receiver), then every merge level is
 *   local;
 *   LCPP_EXCHANGE_AUTO -- when every rank is on one host and exported its
 *   buffer: copy-engine pushes (COPY) from 4 ranks on, peer loads (PEER)
 *   with 2 or 3 ranks; otherwise NCCL.
 * times (optional): per-phase device times of this call (the call then
 *   waits for its own completion). */
typedef enum lcpp_exchange {
    LCPP_EXCHANGE_AUTO = 0,
    LCPP_EXCHANGE_PEER = 1,
    LCPP_EXCHANGE_NCCL = 2,
    LCPP_EXCHANGE_COPY = 3
} lcpp_exchange;

typedef struct lcpp_dist_sort_times {
    float local_sort_ms;     /* histogram + onesweep passes of the local keys */
    float splitters_ms;      /* splitter rounds, tie split, split matrix */
    float host_wait_ms;      /* host blocked reading the split matrix */
    float exchange_merge_ms; /* first merge level over peer memory (or NCCL exchange + first level) */
    float local_merge_ms;    /* remaining merge levels */
    float total_ms;          /* device time of the whole call */
    float host_ms;           /* host time of the whole call */
    int peer_exchange;       /* 1: runs read over peer memory, 2: pushed by copy engines, 0: NCCL send / receive */
} lcpp_dist_sort_times;

lcpp_status lcpp_dist_sort_keys_temp_bytes(lcpp_comm comm, lcpp_dtype key_dtype, uint64_t n_local,
                                           size_t* temp_bytes);
lcpp_status lcpp_dist_sort_keys(lcpp_comm comm, void* temp, size_t temp_bytes, const void* keys_in,
                                void* keys_out, uint64_t n_local, lcpp_dtype key_dtype, int exchange,
                                lcpp_dist_sort_times* times, lcpp_stream_t stream);

/* ------------------------------------------------------------------------
 * Distributed scan and reduce
 *
 * Inclusive / exclusive sum over all ranks' items in rank order: rank r's
 * out[i] = (items of ranks < r) + in[0] + ... + in[i] (exclusive: up to
 * in[i - 1]); integer sums wrap.  Reduce: *d_out on every rank = init (op)
 * items of rank 0 (op) ... (op) items of rank G - 1, the per-rank results
 * combined in rank order (floating-point results identical on every rank
 * and from run to run).  No host wait.
 * ---------------------------------------------------------------------- */
lcpp_status lcpp_dist_scan_temp_bytes(lcpp_comm comm, lcpp_dtype dtype, uint64_t n_local, size_t* temp_bytes);
lcpp_status lcpp_dist_inclusive_sum(lcpp_comm comm, void* temp, size_t temp_bytes, const void* d_in, void* d_out,
                                    uint64_t n_local, lcpp_dtype dtype, lcpp_stream_t stream);
lcpp_status lcpp_dist_exclusive_sum(lcpp_comm comm, void* temp, size_t temp_bytes, const void* d_in, void* d_out,
                                    uint64_t n_local, lcpp_dtype dtype, lcpp_stream_t stream);
lcpp_status lcpp_dist_reduce_temp_bytes(lcpp_comm comm, lcpp_dtype dtype, uint64_t n_local, size_t* temp_bytes);
lcpp_status lcpp_dist_reduce(lcpp_comm comm, void* temp, size_t temp_bytes, const void* d_in, void* d_out,
                             uint64_t n_local, lcpp_op op, const void* init, lcpp_dtype dtype,
                             lcpp_stream_t stream);

/* ------------------------------------------------------------------------
 * Device building blocks
 * ---------------------------------------------------------------------- */

/* For each query q[i] (an order-preserving key image: the key after the
 * sort's ascending bijection, as unsigned 32-bit for 4-byte keys or 64-bit
 * for 8-byte keys), out[i] = number of keys of `sorted` (n keys of key_dtype,
 * sorted ascending by DeviceRadixSort) whose image is < q[i] (upper == 0)
 * or <= q[i] (upper != 0).  +-0.0 have the same image (as when sorting). */
lcpp_status lcpp_dist_search_sorted(const void* sorted, uint64_t n, const void* queries, uint64_t num_queries,
                                    int upper, uint64_t* out, lcpp_dtype key_dtype, lcpp_stream_t stream);

/* Temp bytes of lcpp_dist_merge_sorted for `total` = na + nb keys: a
 * 256-byte control area (byte 4: the device error word, as
 * lcpp_device_status reads it) and the split points of the output blocks. */
lcpp_status lcpp_dist_merge_temp_bytes(uint64_t total, size_t* temp_bytes);

/* Merge two runs sorted ascending by DeviceRadixSort (keys of key_dtype,
 * compared by the same order-preserving image): out[0, na + nb) receives the
 * merged keys; among equal images the keys of `a` come first.  `out` must not
 * overlap `a` or `b`; temp (256-byte aligned) holds the control area and the
 * output blocks' split points.  The runs must lie in device allocations (the
 * merge bulk-copies them from the 16-byte boundary at or below each range's
 * start).  Merge path (Green, McColl & Bader, 2012): one small kernel finds
 * each output block's split point by binary search, a second -- persistent,
 * the next block's inputs bulk-copied into shared memory while it merges the
 * current one -- merges each block in shared memory.  Every wait of the
 * second is bounded; on expiry LCPP_ERR_LOOKBACK_TIMEOUT is recorded in the
 * error word. */
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
