/*
 * lcpp_b200_diag.h -- kernel timing hooks of liblcpp_b200.
 *
 * No counterpart in the reference (its timing lives in the benchmark,
 * tests/lcpp_cub_bench.cpp:225-260).  When enabled, every kernel the library
 * launches is bracketed by two CUDA events recorded on the launch stream, so
 * a benchmark can attribute device time to the individual kernels of one
 * sort / scan / reduce call.  Disabled by default; when disabled the hooks
 * cost one relaxed atomic load per launch.
 */
#ifndef LCPP_B200_DIAG_H
#define LCPP_B200_DIAG_H

#include "lcpp_b200.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef enum lcpp_kernel_kind {
    LCPP_KERNEL_SORT_HISTOGRAM = 0, /* all-pass digit histogram + digit offsets */
    LCPP_KERNEL_SORT_ONESWEEP = 1,  /* one 8-bit onesweep pass */
    LCPP_KERNEL_SCAN = 2,           /* decoupled look-back scan */
    LCPP_KERNEL_REDUCE = 3,         /* two-level reduce */
    LCPP_KERNEL_SEGMENT_BLOCK = 4,  /* segmented sort: one block per short segment */
    LCPP_KERNEL_MERGE = 5,          /* merge path (lcpp_dist_merge_sorted*) */
    LCPP_KERNEL_ARG_REDUCE = 6,     /* ArgMin / ArgMax */
    LCPP_KERNEL_BY_KEY = 7,         /* by-key scans and ReduceByKey */
    LCPP_KERNEL_SELECT = 8          /* DeviceSelect / DevicePartition */
} lcpp_kernel_kind;

typedef struct lcpp_kernel_time {
    int kind;          /* lcpp_kernel_kind */
    float ms;          /* device time between the launch's two events */
    uint64_t items;    /* items the launch processed */
} lcpp_kernel_time;

/* Enable (1) or disable (0) event recording, process-wide.  Enabling clears
 * earlier records. */
lcpp_status lcpp_diag_timing_enable(int enable);

/* Synchronise the recorded events and copy up to `capacity` records (in
 * launch order) to `out`; *count receives the number of records held. */
lcpp_status lcpp_diag_timing_read(lcpp_kernel_time* out, int capacity, int* count);

/* Wait-timeout probe (no reference counterpart: the reference's look-back
 * spins are unbounded, src/lcpp/agent/agent_radix_sort_onesweep.h:324-334).
 * One device thread waits on a status word that nothing publishes, with the
 * same bounded wait routine as the onesweep look-back but a limit of
 * `limit_ns` (at most 4 s).  The wait runs out, records
 * LCPP_ERR_LOOKBACK_TIMEOUT in temp's error word and the kernel returns, so
 * lcpp_device_status(temp, stream) reports the timeout and the context stays
 * usable.  temp: 256-byte aligned, at least 256 bytes. */
lcpp_status lcpp_diag_wait_timeout_probe(void* temp, size_t temp_bytes, uint64_t limit_ns, lcpp_stream_t stream);

#ifdef __cplusplus
} /* extern "C" */
#endif

#endif /* LCPP_B200_DIAG_H */
