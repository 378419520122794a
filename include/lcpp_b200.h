/*
 * lcpp_b200.h -- C ABI of the B200-native (sm_100a) sort / scan / reduce path.
 *
 * Drop-in boundary for LuisaCompute-ParallelPrimitive's Device-level modules
 * DeviceRadixSort, DeviceScan and DeviceReduce.  Every entry point below names
 * the reference member function it replaces (path:line inside the reference
 * project).  Conventions shared by all entry points:
 *
 *  - All pointers are device pointers owned by the caller.  The library never
 *    allocates device memory: scratch ("temp storage") is sized with the
 *    matching *_temp_bytes query and passed in, exactly like the reference's
 *    CUB-style GetTempStorageBytes + BufferView<uint> temp_storage pair.
 *  - Work is enqueued asynchronously on the given cudaStream_t (the reference
 *    records into a caller CommandList instead).  No host synchronisation
 *    happens on the hot path.
 *  - Counts are 64-bit (the reference takes `uint num_items`).
 *  - Misuse returns a status code instead of aborting (the reference aborts
 *    through LUISA_ASSERT, src/lcpp/device/device_radix_sort.h:976-1016).
 *  - Temp storage must be 256-byte aligned; it may be reused by consecutive
 *    calls on one stream, but two calls that may run concurrently need
 *    distinct temp storage.
 */
#ifndef LCPP_B200_H
#define LCPP_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* cudaStream_t without pulling in the CUDA headers. */
typedef struct CUstream_st* lcpp_stream_t;

typedef enum lcpp_status {
    LCPP_OK = 0,
    LCPP_ERR_INVALID_ARG = 1,       /* bad pointer, bit range, selector, ... */
    LCPP_ERR_TEMP_TOO_SMALL = 2,    /* temp_bytes below the *_temp_bytes query */
    LCPP_ERR_UNSUPPORTED_DTYPE = 3, /* dtype / op combination not provided */
    LCPP_ERR_CUDA = 4,              /* a CUDA runtime call failed */
    LCPP_ERR_LOOKBACK_TIMEOUT = 5,  /* a bounded device-side wait expired */
    LCPP_ERR_COMM = 6,              /* distributed exchange failed */
    LCPP_ERR_INTERNAL = 7           /* a device-side consistency check failed */
} lcpp_status;

/* Element types.  Numbering is part of the ABI. */
typedef enum lcpp_dtype {
    LCPP_U32 = 0,
    LCPP_I32 = 1,
    LCPP_F32 = 2,
    LCPP_U64 = 3,
    LCPP_I64 = 4,
    LCPP_F64 = 5,
    LCPP_U8 = 6,    /* 1-byte (bool) selection flags of DeviceSelect /
                       DevicePartition only; every other entry point rejects it */
    LCPP_NONE = 255 /* "no values" (keys-only) */
} lcpp_dtype;

/* Binary operators for scan / reduce (the reference takes DSL lambdas; the
 * ones its Device modules name are SumOp, MinOp and MaxOp,
 * src/lcpp/common/thread_operators.h:49-75). */
typedef enum lcpp_op {
    LCPP_OP_SUM = 0,
    LCPP_OP_MIN = 1,
    LCPP_OP_MAX = 2
} lcpp_op;

/* Human-readable status name (static storage). */
const char* lcpp_status_string(lcpp_status status);

/* Library version as MAJOR*10000 + MINOR*100 + PATCH. */
int lcpp_version(void);

/* ------------------------------------------------------------------------
 * DeviceRadixSort  (src/lcpp/device/device_radix_sort.h)
 *
 * Stable LSD radix sort over key bits [begin_bit, end_bit).  Keys are
 * compared through the reference's order-preserving bijection
 * (src/lcpp/common/util_type.h:97-175): unsigned keys as is, signed keys with
 * the sign bit flipped, floating-point keys with all bits flipped when
 * negative and only the sign bit otherwise; -0.0 and +0.0 produce identical
 * digits (src/lcpp/agent/radix_rank_sort_operations.h:31-43).  Descending
 * order inverts the transformed key (radix_rank_sort_operations.h:123-155).
 * Output keys and values are the original bit patterns.
 *
 * Key dtypes: U32, I32, F32, U64, I64, F64.  Value dtypes: any of those
 * (4- or 8-byte payload, moved bit-exactly).
 * ---------------------------------------------------------------------- */

/* Replaces DeviceRadixSort::GetSortKeysTempStorageBytes<K>
 * (device_radix_sort.h:358-362).  n == 0 gives 0 bytes, as the reference
 * (tests/device_radix_sort_interface_test.cpp:197-203). */
lcpp_status lcpp_radix_sort_keys_temp_bytes(lcpp_dtype key_dtype, uint64_t num_items,
                                            size_t* temp_bytes);

/* Replaces DeviceRadixSort::GetSortPairsTempStorageBytes<K,V>
 * (device_radix_sort.h:351-356). */
lcpp_status lcpp_radix_sort_pairs_temp_bytes(lcpp_dtype key_dtype, lcpp_dtype value_dtype,
                                             uint64_t num_items, size_t* temp_bytes);

/* Replaces DeviceRadixSort::SortKeys / SortKeysDescending, copy API
 * (device_radix_sort.h:399-425 and :457-483).  keys_in is not modified;
 * the sorted keys land in keys_out.  begin_bit == end_bit copies
 * (device_radix_sort.h:413-417); num_items == 0 is a no-op. */
lcpp_status lcpp_radix_sort_keys(void* temp, size_t temp_bytes,
                                 const void* keys_in, void* keys_out,
                                 uint64_t num_items, int begin_bit, int end_bit,
                                 int descending, lcpp_dtype key_dtype,
                                 lcpp_stream_t stream);

/* Replaces DeviceRadixSort::SortPairs / SortPairsDescending, copy API
 * (device_radix_sort.h:369-398 and :427-456). */
lcpp_status lcpp_radix_sort_pairs(void* temp, size_t temp_bytes,
                                  const void* keys_in, void* keys_out,
                                  const void* values_in, void* values_out,
                                  uint64_t num_items, int begin_bit, int end_bit,
                                  int descending, lcpp_dtype key_dtype,
                                  lcpp_dtype value_dtype, lcpp_stream_t stream);

/* Replaces the DoubleBuffer overloads of SortKeys / SortKeysDescending
 * (device_radix_sort.h:497-519 and :533-555).  key_buffers[2] are the two
 * slots of the reference's DoubleBuffer (src/lcpp/common/util_type.h:57-74);
 * *selector (0 or 1) names the slot holding the input and is flipped once per
 * 8-bit pass, so that on return key_buffers[*selector] holds the result.  Both
 * slots may be overwritten.  Zero items or begin_bit == end_bit leave the
 * selector unchanged (device_radix_sort.h:507-510). */
lcpp_status lcpp_radix_sort_keys_double_buffer(void* temp, size_t temp_bytes,
                                               void* key_buffers[2], int* selector,
                                               uint64_t num_items, int begin_bit, int end_bit,
                                               int descending, lcpp_dtype key_dtype,
                                               lcpp_stream_t stream);

/* Replaces the DoubleBuffer overloads of SortPairs / SortPairsDescending
 * (device_radix_sort.h:484-495, :520-531, dispatch_double_buffer :951-974).
 * One selector serves keys and values (the reference asserts they match). */
lcpp_status lcpp_radix_sort_pairs_double_buffer(void* temp, size_t temp_bytes,
                                                void* key_buffers[2], void* value_buffers[2],
                                                int* selector, uint64_t num_items,
                                                int begin_bit, int end_bit, int descending,
                                                lcpp_dtype key_dtype, lcpp_dtype value_dtype,
                                                lcpp_stream_t stream);

/* ------------------------------------------------------------------------
 * DeviceScan  (src/lcpp/device/device_scan.h)
 *
 * Single-pass decoupled look-back scan.  dtypes: I32, U32 (wrapping
 * two's-complement arithmetic), F32, I64, U64, F64.  In-place operation
 * (d_in == d_out) is allowed, as in the reference
 * (tests/device_scan_test.cpp:288-322).
 * ---------------------------------------------------------------------- */

/* Replaces DeviceScan::GetTempStorageBytes<T> (device_scan.h:295-308). */
lcpp_status lcpp_scan_temp_bytes(lcpp_dtype dtype, uint64_t num_items, size_t* temp_bytes);

/* Replaces DeviceScan::ExclusiveScan (device_scan.h:321-332):
 * out[i] = init (+) in[0] (+) ... (+) in[i-1].  `init` points to one host
 * value of `dtype`.  ExclusiveSum (device_scan.h:370-385) is op = SUM with a
 * zero init. */
lcpp_status lcpp_scan_exclusive(void* temp, size_t temp_bytes, const void* d_in, void* d_out,
                                uint64_t num_items, lcpp_op op, const void* init,
                                lcpp_dtype dtype, lcpp_stream_t stream);

/* Replaces DeviceScan::InclusiveScan without an initial value
 * (device_scan.h:333-344): out[i] = in[0] (+) ... (+) in[i].
 * InclusiveSum (device_scan.h:408-419) is op = SUM. */
lcpp_status lcpp_scan_inclusive(void* temp, size_t temp_bytes, const void* d_in, void* d_out,
                                uint64_t num_items, lcpp_op op, lcpp_dtype dtype,
                                lcpp_stream_t stream);

/* Replaces DeviceScan::InclusiveScanInit and the InclusiveScan overload with
 * an initial value (device_scan.h:346-368): out[i] = init (+) in[0] (+) ... (+) in[i]. */
lcpp_status lcpp_scan_inclusive_init(void* temp, size_t temp_bytes, const void* d_in,
                                     void* d_out, uint64_t num_items, lcpp_op op,
                                     const void* init, lcpp_dtype dtype, lcpp_stream_t stream);

/* Convenience forms of the two Sum entry points (device_scan.h:370-419). */
lcpp_status lcpp_scan_exclusive_sum(void* temp, size_t temp_bytes, const void* d_in, void* d_out,
                                    uint64_t num_items, lcpp_dtype dtype, lcpp_stream_t stream);
lcpp_status lcpp_scan_inclusive_sum(void* temp, size_t temp_bytes, const void* d_in, void* d_out,
                                    uint64_t num_items, lcpp_dtype dtype, lcpp_stream_t stream);

/* By-key scans: DeviceScan::GetScanByKeyTempStorageBytes,
 * ExclusiveScanByKey, InclusiveScanByKey (with and without an initial
 * value), ExclusiveSumByKey, InclusiveSumByKey (device_scan.h:310-597).
 * Segments are maximal runs of consecutive equal keys (== on the key type:
 * -0.0 equals +0.0, NaN starts a new run; signed and unsigned keys of one
 * width compare alike).  Within a segment starting at h:
 *   exclusive:      out[i] = init (i == h), init (+) v[h] (+) ... (+) v[i-1]
 *   inclusive:      out[i] = v[h] (+) ... (+) v[i]
 *   inclusive init: out[i] = init (+) v[h] (+) ... (+) v[i]
 * Keys and values may be of different types; d_values_out may equal
 * d_values_in.  `init` points to one host value of value_dtype.  Zero items
 * do nothing.  The Sum forms are op = SUM with a zero init. */
lcpp_status lcpp_scan_by_key_temp_bytes(lcpp_dtype key_dtype, lcpp_dtype value_dtype, uint64_t num_items,
                                        size_t* temp_bytes);
lcpp_status lcpp_scan_exclusive_by_key(void* temp, size_t temp_bytes, const void* d_keys_in,
                                       const void* d_values_in, void* d_values_out, uint64_t num_items,
                                       lcpp_op op, const void* init, lcpp_dtype key_dtype,
                                       lcpp_dtype value_dtype, lcpp_stream_t stream);
lcpp_status lcpp_scan_inclusive_by_key(void* temp, size_t temp_bytes, const void* d_keys_in,
                                       const void* d_values_in, void* d_values_out, uint64_t num_items,
                                       lcpp_op op, lcpp_dtype key_dtype, lcpp_dtype value_dtype,
                                       lcpp_stream_t stream);
lcpp_status lcpp_scan_inclusive_by_key_init(void* temp, size_t temp_bytes, const void* d_keys_in,
                                            const void* d_values_in, void* d_values_out, uint64_t num_items,
                                            lcpp_op op, const void* init, lcpp_dtype key_dtype,
                                            lcpp_dtype value_dtype, lcpp_stream_t stream);
lcpp_status lcpp_scan_exclusive_sum_by_key(void* temp, size_t temp_bytes, const void* d_keys_in,
                                           const void* d_values_in, void* d_values_out, uint64_t num_items,
                                           lcpp_dtype key_dtype, lcpp_dtype value_dtype, lcpp_stream_t stream);
lcpp_status lcpp_scan_inclusive_sum_by_key(void* temp, size_t temp_bytes, const void* d_keys_in,
                                           const void* d_values_in, void* d_values_out, uint64_t num_items,
                                           lcpp_dtype key_dtype, lcpp_dtype value_dtype, lcpp_stream_t stream);

/* No counterpart in the reference.  InclusiveSum for callers that cannot
 * allocate device memory when they scan (code running inside an allocator or
 * a memory-pool callback, a plugin host that hands out fixed buffers only, a
 * real-time loop that must not call cudaMalloc after start-up).  Same result
 * as lcpp_scan_inclusive_sum, but the scratch lives in a fixed 2 MiB + 4 KiB
 * device array inside the library, so the caller passes only input and
 * output.  Limits: at most 1,075,707,904 items of a 4-byte type or
 * 215,089,152 items of an 8-byte type; larger counts return
 * LCPP_ERR_TEMP_TOO_SMALL before any device work.  The first call on a
 * device looks up the array's device address (cudaGetSymbolAddress, with
 * that device current) and caches it with the context's unique ID; a call
 * that finds another context current on the device (after cudaDeviceReset)
 * looks it up again.  Make the first call on a device, and the first call
 * after a reset, before any stream capture.  All calls on one device share
 * the array: calls that may overlap
 * on the GPU (different streams, no ordering between them) race and give
 * wrong results.  Every GPU that loads the library holds the array until the
 * process exits.  Nothing in this call allocates memory. */
lcpp_status lcpp_scan_inclusive_sum_noalloc(const void* d_in, void* d_out, uint64_t num_items,
                                            lcpp_dtype dtype, lcpp_stream_t stream);

/* ------------------------------------------------------------------------
 * DeviceReduce  (src/lcpp/device/device_reduce.h)
 *
 * Deterministic two-level reduction: a fixed partition of the input over a
 * persistent grid, then a fixed-order fold of the per-block partials, so a
 * floating-point result is identical from run to run.
 * ---------------------------------------------------------------------- */

/* Replaces DeviceReduce::GetTempStorageBytes<T> (device_reduce.h:183-189). */
lcpp_status lcpp_reduce_temp_bytes(lcpp_dtype dtype, uint64_t num_items, size_t* temp_bytes);

/* Replaces DeviceReduce::Reduce (device_reduce.h:229-252):
 * *d_out = init (+) in[0] (+) ... (+) in[n-1]; n == 0 writes init. */
lcpp_status lcpp_reduce(void* temp, size_t temp_bytes, const void* d_in, void* d_out,
                        uint64_t num_items, lcpp_op op, const void* init, lcpp_dtype dtype,
                        lcpp_stream_t stream);

/* Replaces DeviceReduce::Sum (init 0), Min (init numeric max) and Max (init
 * numeric lowest) (device_reduce.h:280-308). */
lcpp_status lcpp_reduce_sum(void* temp, size_t temp_bytes, const void* d_in, void* d_out,
                            uint64_t num_items, lcpp_dtype dtype, lcpp_stream_t stream);
lcpp_status lcpp_reduce_min(void* temp, size_t temp_bytes, const void* d_in, void* d_out,
                            uint64_t num_items, lcpp_dtype dtype, lcpp_stream_t stream);
lcpp_status lcpp_reduce_max(void* temp, size_t temp_bytes, const void* d_in, void* d_out,
                            uint64_t num_items, lcpp_dtype dtype, lcpp_stream_t stream);

/* ------------------------------------------------------------------------
 * DeviceRadixSort over decomposed keys (the decomposer overloads,
 * src/lcpp/device/device_radix_sort.h:556-940)
 *
 * Keys are structs of key_bytes bytes; `members` (host array, at most
 * LCPP_MAX_KEY_MEMBERS) lists the members the reference's decomposer returns,
 * most significant first, by byte offset and dtype.  Keys are ordered by the
 * concatenation of the members' order-preserving bits (unsigned as is,
 * signed with the high bit flipped, floats sign-dependent with -0.0 sorted as
 * +0.0; the last member occupies bits [0, its width),
 * src/lcpp/block/block_radix_sort.h:251-318), compared on the bit window
 * [begin_bit, end_bit) only (end_bit at most the members' total width), in a
 * stable sort, ascending or descending.  Input and output must not overlap.
 * The DoubleBuffer forms read slot *selector, write the other slot and flip
 * *selector once (device_radix_sort.h:833-837); begin_bit == end_bit leaves
 * them unchanged and makes the copy forms copy.
 * ---------------------------------------------------------------------- */
#define LCPP_MAX_KEY_MEMBERS 8
typedef struct lcpp_key_member {
    uint32_t offset;  /* byte offset of the member in the key struct */
    lcpp_dtype dtype; /* LCPP_U32 ... LCPP_F64 */
} lcpp_key_member;

/* Temp bytes of the decomposed-key sorts for num_items keys (any key struct,
 * with or without values). */
lcpp_status lcpp_radix_sort_decomposed_temp_bytes(uint64_t num_items, size_t* temp_bytes);

lcpp_status lcpp_radix_sort_decomposed_keys(void* temp, size_t temp_bytes, const void* keys_in, void* keys_out,
                                            uint64_t num_items, uint32_t key_bytes, const lcpp_key_member* members,
                                            int num_members, int begin_bit, int end_bit, int descending,
                                            lcpp_stream_t stream);
lcpp_status lcpp_radix_sort_decomposed_pairs(void* temp, size_t temp_bytes, const void* keys_in, void* keys_out,
                                             const void* values_in, void* values_out, uint64_t num_items,
                                             uint32_t key_bytes, const lcpp_key_member* members, int num_members,
                                             int begin_bit, int end_bit, int descending, lcpp_dtype value_dtype,
                                             lcpp_stream_t stream);
lcpp_status lcpp_radix_sort_decomposed_keys_double_buffer(void* temp, size_t temp_bytes, void* key_buffers[2],
                                                          int* selector, uint64_t num_items, uint32_t key_bytes,
                                                          const lcpp_key_member* members, int num_members,
                                                          int begin_bit, int end_bit, int descending,
                                                          lcpp_stream_t stream);
lcpp_status lcpp_radix_sort_decomposed_pairs_double_buffer(void* temp, size_t temp_bytes, void* key_buffers[2],
                                                           void* value_buffers[2], int* selector, uint64_t num_items,
                                                           uint32_t key_bytes, const lcpp_key_member* members,
                                                           int num_members, int begin_bit, int end_bit,
                                                           int descending, lcpp_dtype value_dtype,
                                                           lcpp_stream_t stream);

/* ------------------------------------------------------------------------
 * DeviceSegmentedRadixSort  (src/lcpp/device/device_segmented_radix_sort.h)
 *
 * Stable sort of every segment by the key bits [begin_bit, end_bit) after the
 * radix bijection (unsigned as is, signed with the high bit flipped, floats
 * sign-dependent; here +0.0 and -0.0 are different keys, as in the
 * reference's comparator, device_segmented_radix_sort.h:216-243), ascending
 * or descending.  begin_offsets / end_offsets are device arrays of
 * num_segments uint32; item i belongs to the last segment s with
 * begin_offsets[s] <= i, when i < end_offsets[s] and
 * begin_offsets[s] <= end_offsets[s] <= num_items (the reference's rule,
 * device_segmented_sort.h:753-775): segments are expected in ascending order
 * of begin offset and not to overlap.  Items outside every segment are not
 * written.  num_items and num_segments are at most 2^32 - 1.  The temp size
 * depends on num_items only; lcpp_device_status(temp, stream) reports the
 * device error word of the sorting passes.  Segments of up to 2048 items are
 * sorted by one block each in shared memory; if longer segments exist, the
 * call reads their item count back (it synchronises `stream` once) and sorts
 * them with the onesweep sort of a (segment, key) composite. 
 * ---------------------------------------------------------------------- */

/* Replace DeviceSegmentedRadixSort::GetSortKeysTempStorageBytes /
 * GetSortPairsTempStorageBytes (device_segmented_radix_sort.h:28-38). */
lcpp_status lcpp_segmented_radix_sort_keys_temp_bytes(lcpp_dtype key_dtype, uint64_t num_items, size_t* temp_bytes);
lcpp_status lcpp_segmented_radix_sort_pairs_temp_bytes(lcpp_dtype key_dtype, lcpp_dtype value_dtype,
                                                      uint64_t num_items, size_t* temp_bytes);

/* Replaces SortKeys / SortKeysDescending, copy form
 * (device_segmented_radix_sort.h:40-56, :80-96). */
lcpp_status lcpp_segmented_radix_sort_keys(void* temp, size_t temp_bytes, const void* keys_in, void* keys_out,
                                           uint64_t num_items, uint64_t num_segments,
                                           const uint32_t* begin_offsets, const uint32_t* end_offsets,
                                           int begin_bit, int end_bit, int descending, lcpp_dtype key_dtype,
                                           lcpp_stream_t stream);

/* Replaces SortPairs / SortPairsDescending, copy form
 * (device_segmented_radix_sort.h:120-138, :163-181). */
lcpp_status lcpp_segmented_radix_sort_pairs(void* temp, size_t temp_bytes, const void* keys_in, void* keys_out,
                                            const void* values_in, void* values_out, uint64_t num_items,
                                            uint64_t num_segments, const uint32_t* begin_offsets,
                                            const uint32_t* end_offsets, int begin_bit, int end_bit, int descending,
                                            lcpp_dtype key_dtype, lcpp_dtype value_dtype, lcpp_stream_t stream);

/* Replace the DoubleBuffer forms (device_segmented_radix_sort.h:58-78,
 * :98-118, :140-161, :183-204).  As in the reference's segmented merge sort
 * (device_segmented_sort.h:229-246), the selector flips once per merge pass,
 * ceil(log2(num_items)) times, and key_buffers[*selector] holds the result on
 * return; nothing happens (selector unchanged) for num_items <= 1, no
 * segments or begin_bit == end_bit.  Positions outside every segment keep
 * what the result slot held. */
lcpp_status lcpp_segmented_radix_sort_keys_double_buffer(void* temp, size_t temp_bytes, void* key_buffers[2],
                                                         int* selector, uint64_t num_items, uint64_t num_segments,
                                                         const uint32_t* begin_offsets, const uint32_t* end_offsets,
                                                         int begin_bit, int end_bit, int descending,
                                                         lcpp_dtype key_dtype, lcpp_stream_t stream);
lcpp_status lcpp_segmented_radix_sort_pairs_double_buffer(void* temp, size_t temp_bytes, void* key_buffers[2],
                                                          void* value_buffers[2], int* selector, uint64_t num_items,
                                                          uint64_t num_segments, const uint32_t* begin_offsets,
                                                          const uint32_t* end_offsets, int begin_bit, int end_bit,
                                                          int descending, lcpp_dtype key_dtype,
                                                          lcpp_dtype value_dtype, lcpp_stream_t stream);

/* Replace DeviceReduce::GetArgTempStorageBytes / ArgMin / ArgMax
 * (device_reduce.h:192-204, :310-436): *d_out = the minimum (maximum) value
 * and *d_index_out = the first index holding it (ties go to the smaller
 * index, thread_operators.h:19-47; NaN never wins); zero items write the
 * numeric max (ArgMin) or lowest (ArgMax) value and index 1 (:318-323).
 * num_items at most 2^32 - 1 (uint32 indices, as the reference). */
lcpp_status lcpp_reduce_arg_temp_bytes(lcpp_dtype dtype, uint64_t num_items, size_t* temp_bytes);
lcpp_status lcpp_reduce_argmin(void* temp, size_t temp_bytes, const void* d_in, void* d_out, uint32_t* d_index_out,
                               uint64_t num_items, lcpp_dtype dtype, lcpp_stream_t stream);
lcpp_status lcpp_reduce_argmax(void* temp, size_t temp_bytes, const void* d_in, void* d_out, uint32_t* d_index_out,
                               uint64_t num_items, lcpp_dtype dtype, lcpp_stream_t stream);

/* Replace DeviceReduce::GetReduceByKeyTempStorageBytes / ReduceByKey
 * (device_reduce.h:208-223, :437-491): for every maximal run of consecutive
 * equal keys (as in the by-key scans) d_unique_out[r] = the run's first key,
 * d_aggregates_out[r] = v[first] (+) ... (+) v[last], and *d_num_runs_out =
 * the number of runs (uint32; zero items write 0 and nothing else).
 * num_items at most 2^32 - 1; d_unique_out must not overlap d_keys_in. */
lcpp_status lcpp_reduce_by_key_temp_bytes(lcpp_dtype key_dtype, lcpp_dtype value_dtype, uint64_t num_items,
                                          size_t* temp_bytes);
lcpp_status lcpp_reduce_by_key(void* temp, size_t temp_bytes, const void* d_keys_in, const void* d_values_in,
                               void* d_unique_out, void* d_aggregates_out, uint32_t* d_num_runs_out,
                               uint64_t num_items, lcpp_op op, lcpp_dtype key_dtype, lcpp_dtype value_dtype,
                               lcpp_stream_t stream);

/* ------------------------------------------------------------------------
 * DeviceSelect / DevicePartition  (src/lcpp/device/device_select.h,
 * src/lcpp/device/device_partition.h)
 *
 * The reference takes predicate lambdas; through the C ABI a predicate is
 * the AND of up to LCPP_MAX_CLAUSES clauses on the tested value (an item, or
 * a flag for FlaggedIf), each optionally negated.  a and b hold the bit
 * patterns of values of the tested type (4-byte types in the low half).
 * Zero clauses select everything.  C++ callers compiled with nvcc can pass
 * any __device__ callable instead (include/lcpp_b200_device.cuh).
 * All counts are uint32 (num_items at most 2^32 - 1, as the reference);
 * zero items write zero count(s) and nothing else.
 * ------------------------------------------------------------------------ */
#define LCPP_MAX_CLAUSES 4

typedef enum lcpp_clause_kind {
    LCPP_CLAUSE_LT = 0,      /* x <  a */
    LCPP_CLAUSE_LE = 1,      /* x <= a */
    LCPP_CLAUSE_GT = 2,      /* x >  a */
    LCPP_CLAUSE_GE = 3,      /* x >= a */
    LCPP_CLAUSE_EQ = 4,      /* x == a */
    LCPP_CLAUSE_NE = 5,      /* x != a */
    LCPP_CLAUSE_MOD_EQ = 6,  /* x % a == b (integer types, a != 0; C remainder) */
    LCPP_CLAUSE_BITS_ANY = 7 /* (x & a) != 0 (integer types) */
} lcpp_clause_kind;

typedef struct lcpp_clause {
    int32_t kind;   /* lcpp_clause_kind */
    int32_t negate; /* nonzero: the clause's result is inverted */
    uint64_t a;
    uint64_t b;
} lcpp_clause;

/* Replace DeviceSelect::GetTempStorageBytes and DevicePartition::
 * GetTempStorageBytes / GetThreeWayTempStorageBytes
 * (device_select.h:56-63, device_partition.h:55-71); item-type independent. */
lcpp_status lcpp_select_temp_bytes(uint64_t num_items, size_t* temp_bytes);
lcpp_status lcpp_partition_temp_bytes(uint64_t num_items, size_t* temp_bytes);
lcpp_status lcpp_partition_three_way_temp_bytes(uint64_t num_items, size_t* temp_bytes);

/* Replace DeviceSelect::Flagged (device_select.h:65-117): the items whose
 * flag != 0 (at flag_dtype; LCPP_U8 for bool flags), in input order, and
 * *d_num_selected_out = their count.  d_out may equal d_in (the in-place
 * overload). */
lcpp_status lcpp_select_flagged(void* temp, size_t temp_bytes, const void* d_in, const void* d_flags, void* d_out,
                                uint32_t* d_num_selected_out, uint64_t num_items, lcpp_dtype dtype,
                                lcpp_dtype flag_dtype, lcpp_stream_t stream);

/* Replace DeviceSelect::FlaggedIf (device_select.h:177-212): the items whose
 * flag satisfies the clauses (tested at flag_dtype).  d_out may equal d_in. */
lcpp_status lcpp_select_flagged_if(void* temp, size_t temp_bytes, const void* d_in, const void* d_flags,
                                   void* d_out, uint32_t* d_num_selected_out, uint64_t num_items, lcpp_dtype dtype,
                                   lcpp_dtype flag_dtype, const lcpp_clause* clauses, int num_clauses,
                                   lcpp_stream_t stream);

/* Replace DeviceSelect::If (device_select.h:119-175): the items that satisfy
 * the clauses.  d_out may equal d_in. */
lcpp_status lcpp_select_if(void* temp, size_t temp_bytes, const void* d_in, void* d_out,
                           uint32_t* d_num_selected_out, uint64_t num_items, lcpp_dtype dtype,
                           const lcpp_clause* clauses, int num_clauses, lcpp_stream_t stream);

/* Replace DeviceSelect::Unique (device_select.h:214-286): the first item of
 * every run of consecutive equal items (== at dtype: -0.0 equals +0.0, NaN
 * never equals).  d_out may equal d_in. */
lcpp_status lcpp_select_unique(void* temp, size_t temp_bytes, const void* d_in, void* d_out,
                               uint32_t* d_num_selected_out, uint64_t num_items, lcpp_dtype dtype,
                               lcpp_stream_t stream);

/* Replace DeviceSelect::UniqueByKey (device_select.h:288-333): the first
 * (key, value) of every run of equal consecutive keys. */
lcpp_status lcpp_select_unique_by_key(void* temp, size_t temp_bytes, const void* d_keys_in, const void* d_values_in,
                                      void* d_keys_out, void* d_values_out, uint32_t* d_num_selected_out,
                                      uint64_t num_items, lcpp_dtype key_dtype, lcpp_dtype value_dtype,
                                      lcpp_stream_t stream);

/* Replace DeviceScan::ExclusiveSumTransform and ExclusiveSumAdjacent
 * (device_scan.h:387-406; details/scan.h:127-240): d_out[i] (uint32) = the
 * number of j < i whose item satisfies the clauses (Transform), or that
 * starts a run of equal items, i.e. j == 0 or d_in[j] != d_in[j - 1]
 * (Adjacent; == at dtype).  The reference takes 4-byte inputs; 8-byte ones
 * work too.  Temp storage: lcpp_scan_transform_temp_bytes.  Zero items do
 * nothing. */
lcpp_status lcpp_scan_transform_temp_bytes(uint64_t num_items, size_t* temp_bytes);
lcpp_status lcpp_scan_exclusive_sum_transform(void* temp, size_t temp_bytes, const void* d_in, uint32_t* d_out,
                                              uint64_t num_items, lcpp_dtype dtype, const lcpp_clause* clauses,
                                              int num_clauses, lcpp_stream_t stream);
lcpp_status lcpp_scan_exclusive_sum_adjacent(void* temp, size_t temp_bytes, const void* d_in, uint32_t* d_out,
                                             uint64_t num_items, lcpp_dtype dtype, lcpp_stream_t stream);

/* Replace DevicePartition::Flagged / If (device_partition.h:73-155): the
 * selected items in input order from d_out[0], the rejected ones in REVERSE
 * input order from d_out[num_items - 1] down; *d_num_selected_out = the
 * selected count.  d_out must not equal d_in. */
lcpp_status lcpp_partition_flagged(void* temp, size_t temp_bytes, const void* d_in, const void* d_flags, void* d_out,
                                   uint32_t* d_num_selected_out, uint64_t num_items, lcpp_dtype dtype,
                                   lcpp_dtype flag_dtype, lcpp_stream_t stream);
lcpp_status lcpp_partition_if(void* temp, size_t temp_bytes, const void* d_in, void* d_out,
                              uint32_t* d_num_selected_out, uint64_t num_items, lcpp_dtype dtype,
                              const lcpp_clause* clauses, int num_clauses, lcpp_stream_t stream);

/* Replace the three-way DevicePartition::If (device_partition.h:157-227):
 * items satisfying the first clauses go to d_first_out, the others that
 * satisfy the second clauses to d_second_out (both in input order), the rest
 * to d_unselected_out in REVERSE input order; d_num_selected_out[0] / [1] =
 * the first / second counts.  Outputs must not overlap the input. */
lcpp_status lcpp_partition_if_three_way(void* temp, size_t temp_bytes, const void* d_in, void* d_first_out,
                                        void* d_second_out, void* d_unselected_out, uint32_t* d_num_selected_out,
                                        uint64_t num_items, lcpp_dtype dtype, const lcpp_clause* first_clauses,
                                        int num_first_clauses, const lcpp_clause* second_clauses,
                                        int num_second_clauses, lcpp_stream_t stream);

/* ------------------------------------------------------------------------
 * Device diagnostics (no reference counterpart: the reference's look-back
 * spins are unbounded, src/lcpp/agent/agent_radix_sort_onesweep.h:324-334).
 *
 * Every device-side wait in the kernels above is bounded.  When one expires
 * the kernel records LCPP_ERR_LOOKBACK_TIMEOUT in a status word inside the
 * temp storage of that call and returns normally.  This call synchronises
 * `stream`, reads that word and returns it (LCPP_OK when clear).  `temp` must
 * be the temp storage of the call being checked and must not have been
 * reused since.
 * ---------------------------------------------------------------------- */
lcpp_status lcpp_device_status(const void* temp, lcpp_stream_t stream);

#ifdef __cplusplus
} /* extern "C" */
#endif

#endif /* LCPP_B200_H */
