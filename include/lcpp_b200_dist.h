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

#ifdef __cplusplus
} /* extern "C" */
#endif

#endif /* LCPP_B200_DIST_H */
