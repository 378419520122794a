// dist.cu -- device building blocks of the distributed sort
// (include/lcpp_b200_dist.h).
#include <cstring>

#include "../../include/lcpp_b200_device.cuh"
#include "../../include/lcpp_b200_dist.h"
#include "dist.cuh"

namespace lcpp {
namespace dist {

template <typename U>
__global__ void search_sorted_kernel(const U* __restrict__ sorted, uint64_t n, const U* __restrict__ queries,
                                     uint64_t nq, int upper, uint64_t* __restrict__ out, KeyCodec<U> codec)
{
    const uint64_t i = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= nq) return;
    out[i] = count_below(sorted, n, queries[i], upper != 0, codec);
}

}  // namespace dist
}  // namespace lcpp

extern "C" lcpp_status lcpp_dist_search_sorted(const void* sorted, uint64_t n, const void* queries,
                                               uint64_t num_queries, int upper, uint64_t* out,
                                               lcpp_dtype key_dtype, lcpp_stream_t stream)
{
    using namespace lcpp;
    using namespace lcpp::dist;
    const int kb = dtype_bytes(key_dtype);
    if (!kb) return LCPP_ERR_UNSUPPORTED_DTYPE;
    if (num_queries == 0) return LCPP_OK;
    if (!queries || !out || (n && !sorted)) return LCPP_ERR_INVALID_ARG;
    const unsigned block = 256;
    const uint64_t grid = ceil_div(num_queries, block);
    if (grid > 0x7fffffffull) return LCPP_ERR_INVALID_ARG;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    if (kb == 4) {
        search_sorted_kernel<uint32_t><<<unsigned(grid), block, 0, s>>>(
            static_cast<const uint32_t*>(sorted), n, static_cast<const uint32_t*>(queries), num_queries, upper, out,
            make_codec<uint32_t>(key_dtype, false));
    } else {
        search_sorted_kernel<uint64_t><<<unsigned(grid), block, 0, s>>>(
            static_cast<const uint64_t*>(sorted), n, static_cast<const uint64_t*>(queries), num_queries, upper, out,
            make_codec<uint64_t>(key_dtype, false));
    }
    return cudaGetLastError() == cudaSuccess ? LCPP_OK : LCPP_ERR_CUDA;
}

// ---------------------------------------------------------------------------
// Merge path of two sorted runs.
// ---------------------------------------------------------------------------
namespace lcpp {
namespace dist {

constexpr int kMergeBlock = 256;
constexpr int kMergeItems = 15;  // odd: the per-thread output rows in shared memory never conflict
constexpr uint64_t kMergeTile = uint64_t(kMergeBlock) * kMergeItems;

// Number of elements of a among the first o outputs of the merge (ties: a first).
template <typename U, typename LoadA, typename LoadB>
__device__ __forceinline__ uint64_t co_rank(uint64_t o, uint64_t na, uint64_t nb, LoadA la, LoadB lb)
{
    uint64_t lo = o > nb ? o - nb : 0;
    uint64_t hi = o < na ? o : na;
    while (lo < hi) {
        const uint64_t mid = lo + (hi - lo) / 2;
        if (la(mid) <= lb(o - mid - 1))
            lo = mid + 1;
        else
            hi = mid;
    }
    return lo;
}

// A batch of independent merges (one level of a merge tree), passed by value.
template <typename U>
struct MergeBatch {
    int count;
    uint64_t block_start[LCPP_MERGE_BATCH_MAX + 1];  // first output block of each merge (prefix sums)
    uint64_t split_start[LCPP_MERGE_BATCH_MAX + 1];  // first split entry of each merge (blocks + 1 each)
    const U* a[LCPP_MERGE_BATCH_MAX];
    const U* b[LCPP_MERGE_BATCH_MAX];
    U* out[LCPP_MERGE_BATCH_MAX];
    uint64_t na[LCPP_MERGE_BATCH_MAX];
    uint64_t nb[LCPP_MERGE_BATCH_MAX];
};

// Merge of an index (a block or a split entry) in a prefix-sum table.
__device__ __forceinline__ int batch_slot(const uint64_t* start, int count, uint64_t idx)
{
    int m = 0;
    while (m + 1 < count && start[m + 1] <= idx) ++m;
    return m;
}

// Split points: for merge m and output block k, the number of a-keys among
// its first k * kMergeTile outputs (ties: a first).
template <typename U>
__global__ void merge_split_kernel(const MergeBatch<U> mb, uint64_t* __restrict__ splits, KeyCodec<U> codec)
{
    const uint64_t e = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (e >= mb.split_start[mb.count]) return;
    const int m = batch_slot(mb.split_start, mb.count, e);
    const uint64_t k = e - mb.split_start[m];
    const uint64_t na = mb.na[m], nb = mb.nb[m];
    const U* a = mb.a[m];
    const U* b = mb.b[m];
    const uint64_t o = min(k * kMergeTile, na + nb);
    splits[e] = co_rank<U>(o, na, nb, [&](uint64_t i) { return key_image(a[i], codec); },
                           [&](uint64_t j) { return key_image(b[j], codec); });
}

// Comparison image of a key inside the merge: the identity for unsigned keys
// (PLAIN), else the sort's bijection with the +-0.0 fold.
template <bool PLAIN, typename U>
__device__ __forceinline__ U merge_image(U k, const KeyCodec<U>& c)
{
    if constexpr (PLAIN)
        return k;
    else
        return key_image(k, c);
}

/* ---- Persistent merge with bulk-copied inputs ------------------------------
 * Blocks take output tiles blockIdx.x, blockIdx.x + gridDim.x, ...; while a
 * block merges one tile, the inputs of its next kMergeStages - 1 tiles --
 * a[i0, i1) and b[j0, j1), contiguous ranges of the two runs, which may
 * live in another GPU's memory -- are bulk-copied (cp.async.bulk, no
 * multicast) into the other shared-memory stages.  A bulk copy needs
 * 16-byte aligned addresses and sizes: each range is copied from the
 * 16-byte boundary at or below its start (inside the same allocation) up
 * to the last boundary at or below its end, and the few keys past that
 * boundary are loaded by plain loads.  Per tile: each thread finds where
 * its kMergeItems outputs start (co-rank by binary search in shared memory,
 * 32-bit indices), merges them serially with one shared-memory load per
 * output, and the tile is stored coalesced through the same stage. */
// stages per block: one tile merging, the next one's inputs in flight (three
// stages measured slower locally and no faster over NVLink)
constexpr int kMergeStages = 2;
constexpr size_t kMergeCtrlBytes = 256;  // error word at byte 4 of the merge temp, split points after

template <typename U>
struct MergeStage {
    static constexpr int kVec = 16 / int(sizeof(U));
    // a part (from up to kVec - 1 keys before a[i0]), padding to 16 bytes, b part (likewise)
    static constexpr int kKeys = int(kMergeTile) + 3 * kVec;
};

template <typename U>
constexpr size_t merge_smem_bytes()
{
    return size_t(kMergeStages) * MergeStage<U>::kKeys * sizeof(U);
}

/* Where a tile's inputs sit in its stage. */
template <typename U>
struct MergeTileInfo {
    const U* a;      // a + lo_a: stage index 0
    const U* b;      // b + lo_b: stage index b_at
    U* out;          // out + o0
    int a_first;     // stage index of a[i0]
    int a_plain;     // stage indices [a_plain, a_end) come by plain loads
    int a_end;       // stage index past a[i1 - 1]
    int b_at;        // b part's first stage index (16-byte aligned)
    int b_first;     // stage index of b[j0] relative to b_at
    int b_plain;
    int b_end;
};

template <typename U, bool PLAIN>
__global__ void __launch_bounds__(kMergeBlock)
merge_bulk_kernel(const MergeBatch<U> mb, const uint64_t* __restrict__ all_splits, KeyCodec<U> codec,
                  uint64_t blocks, uint32_t* error)
{
    namespace bd = lcpp_b200::device::bulk_detail;
    constexpr int E = MergeStage<U>::kVec;
    constexpr int kStage = MergeStage<U>::kKeys;
    extern __shared__ __align__(128) unsigned char merge_smem[];
    U* const stages = reinterpret_cast<U*>(merge_smem);
    __shared__ __align__(8) uint64_t s_bar[kMergeStages];
    __shared__ MergeTileInfo<U> s_info[kMergeStages];
    const int tid = threadIdx.x;

    // thread 0: the inputs of output tile `blk` into stage st
    auto issue = [&](uint64_t blk, int st) {
        const int m = batch_slot(mb.block_start, mb.count, blk);
        const uint64_t local = blk - mb.block_start[m];
        const uint64_t* splits = all_splits + mb.split_start[m];
        const uint64_t total = mb.na[m] + mb.nb[m];
        const uint64_t o0 = local * kMergeTile;
        const uint64_t o1 = min(o0 + kMergeTile, total);
        const uint64_t i0 = splits[local], i1 = splits[local + 1];
        const uint64_t j0 = o0 - i0, j1 = o1 - i1;
        // the key index (signed: it may lie up to E - 1 keys before the run)
        // at the 16-byte boundary at or below p + i
        auto lower16 = [](const U* p, uint64_t i) -> int64_t {
            return int64_t(i) - int64_t((reinterpret_cast<uintptr_t>(p + i) & 15u) / sizeof(U));
        };
        const U* pa = mb.a[m];
        const U* pb = mb.b[m];
        const int64_t si0 = int64_t(i0), si1 = int64_t(i1), sj0 = int64_t(j0), sj1 = int64_t(j1);
        MergeTileInfo<U> t;
        const int64_t lo_a = si1 > si0 ? lower16(pa, i0) : si0;
        const int64_t hi_a = si1 > si0 ? max(lo_a, lower16(pa, i1)) : si0;
        const int64_t lo_b = sj1 > sj0 ? lower16(pb, j0) : sj0;
        const int64_t hi_b = sj1 > sj0 ? max(lo_b, lower16(pb, j1)) : sj0;
        t.a = pa + lo_a;
        t.a_first = int(si0 - lo_a);
        t.a_plain = int(max(hi_a, si0) - lo_a);
        t.a_end = int(si1 - lo_a);
        t.b_at = (t.a_end + E - 1) / E * E;
        t.b = pb + lo_b;
        t.b_first = int(sj0 - lo_b);
        t.b_plain = int(max(hi_b, sj0) - lo_b);
        t.b_end = int(sj1 - lo_b);
        t.out = mb.out[m] + o0;
        s_info[st] = t;
        const uint32_t bytes_a = uint32_t((hi_a - lo_a) * sizeof(U));
        const uint32_t bytes_b = uint32_t((hi_b - lo_b) * sizeof(U));
        U* dst = stages + size_t(st) * kStage;
        bd::expect_bytes(&s_bar[st], bytes_a + bytes_b);
        if (bytes_a) bd::bulk_copy(dst, t.a, bytes_a, &s_bar[st]);
        if (bytes_b) bd::bulk_copy(dst + t.b_at, t.b, bytes_b, &s_bar[st]);
    };

    uint64_t blk = blockIdx.x;
    uint32_t pending = 0;  // thread 0: bit st = a copy into stage st is in flight
    if (tid == 0) {
        for (int st = 0; st < kMergeStages; ++st) bd::init_barrier(&s_bar[st]);
        bd::fence_barrier_init();
        for (int q = 0; q + 1 < kMergeStages; ++q) {
            const uint64_t b = blk + uint64_t(q) * gridDim.x;
            if (b < blocks) {
                issue(b, q);
                pending |= 1u << q;
            }
        }
    }
    __syncthreads();
    uint32_t phase = 0;  // bit st: parity of the next completion of stage st
    for (uint32_t k = 0; blk < blocks; ++k, blk += gridDim.x) {
        const int st = int(k % kMergeStages);
        const uint64_t ahead = blk + uint64_t(kMergeStages - 1) * gridDim.x;
        if (tid == 0 && ahead < blocks) {
            // the stage of the previous tile: its reads and plain stores come first
            const int fs = int((k + kMergeStages - 1) % kMergeStages);
            bd::fence_proxy_async();
            issue(ahead, fs);
            pending |= 1u << fs;
        }
        if (!bd::wait(&s_bar[st], (phase >> st) & 1u, error, kWaitLimitNs)) atomicCAS(error, 0u, kDevErrTimeout);
        phase ^= 1u << st;
        pending &= ~(1u << st);
        U* const sm = stages + size_t(st) * kStage;
        const MergeTileInfo<U> t = s_info[st];
        // keys past the last 16-byte boundary of each range
        if (tid < E - 1) {
            const int i = t.a_plain + tid;
            if (i < t.a_end) sm[i] = t.a[i];
        } else if (tid >= 32 && tid < 32 + E - 1) {
            const int i = t.b_plain + tid - 32;
            if (i < t.b_end) sm[t.b_at + i] = t.b[i];
        }
        __syncthreads();
        if (*static_cast<volatile uint32_t*>(error)) break;
        const U* sa = sm + t.a_first;
        const U* sb = sm + t.b_at + t.b_first;
        const int la = t.a_end - t.a_first, lb = t.b_end - t.b_first, len = la + lb;
        U v[kMergeItems];
        const int ot = tid * kMergeItems;
        if (ot < len) {
            // co-rank: number of a-keys among this thread's first ot outputs
            int lo = ot > lb ? ot - lb : 0;
            int hi = ot < la ? ot : la;
            while (lo < hi) {
                const int mid = (lo + hi) >> 1;
                if (merge_image<PLAIN>(sa[mid], codec) <= merge_image<PLAIN>(sb[ot - mid - 1], codec))
                    lo = mid + 1;
                else
                    hi = mid;
            }
            // serial merge; reads past a run's end are clamped to its last key (or its first slot)
            const int a_last = la > 0 ? la - 1 : 0, b_last = lb > 0 ? lb - 1 : 0;
            int ia = lo, ib = ot - lo;
            U ka = sa[ia < la ? ia : a_last];
            U kb = sb[ib < lb ? ib : b_last];
#pragma unroll
            for (int k = 0; k < kMergeItems; ++k) {
                const bool take_a =
                    ib >= lb || (ia < la && merge_image<PLAIN>(ka, codec) <= merge_image<PLAIN>(kb, codec));
                v[k] = take_a ? ka : kb;
                if (take_a) {
                    ++ia;
                    ka = sa[ia < la ? ia : a_last];
                } else {
                    ++ib;
                    kb = sb[ib < lb ? ib : b_last];
                }
            }
        }
        __syncthreads();  // every thread is done reading the stage
        if (ot < len) {
#pragma unroll
            for (int k = 0; k < kMergeItems; ++k)
                if (ot + k < len) sm[ot + k] = v[k];
        }
        __syncthreads();
#pragma unroll
        for (int k = 0; k < kMergeItems; ++k) {
            const int idx = tid + k * kMergeBlock;
            if (idx < len) t.out[idx] = sm[idx];
        }
        __syncthreads();  // the stage is free for a later tile
    }
    // copies issued for tiles this block will not merge (only after an
    // error): wait for them, bounded, before the block's shared memory goes away
    if (tid == 0 && pending) {
        for (int st = 0; st < kMergeStages; ++st)
            if ((pending >> st) & 1u)
                if (!bd::wait(&s_bar[st], (phase >> st) & 1u, error, kWaitLimitNs))
                    atomicCAS(error, 0u, kDevErrTimeout);
    }
}

inline uint64_t merge_blocks(uint64_t total) { return ceil_div(total, kMergeTile); }

}  // namespace dist
}  // namespace lcpp

namespace lcpp {
namespace dist {
namespace {

// Split entries (blocks + 1) of every merge of a batch, in order.
bool batch_layout(int count, const uint64_t* na, const uint64_t* nb, uint64_t* block_start, uint64_t* split_start)
{
    block_start[0] = split_start[0] = 0;
    for (int m = 0; m < count; ++m) {
        const uint64_t blocks = merge_blocks(na[m] + nb[m]);
        block_start[m + 1] = block_start[m] + blocks;
        split_start[m + 1] = split_start[m] + blocks + 1;
    }
    return block_start[count] <= 0x7fffffffull && split_start[count] <= 0x7fffffffull * 256;
}

}  // namespace
}  // namespace dist
}  // namespace lcpp

extern "C" lcpp_status lcpp_dist_merge_batch_temp_bytes(int count, const uint64_t* na, const uint64_t* nb,
                                                        size_t* temp_bytes)
{
    using namespace lcpp;
    if (!temp_bytes || count < 0 || count > LCPP_MERGE_BATCH_MAX || (count && (!na || !nb)))
        return LCPP_ERR_INVALID_ARG;
    uint64_t bs[LCPP_MERGE_BATCH_MAX + 1], ss[LCPP_MERGE_BATCH_MAX + 1];
    if (!dist::batch_layout(count, na, nb, bs, ss)) return LCPP_ERR_INVALID_ARG;
    *temp_bytes = count ? dist::kMergeCtrlBytes + align_up(size_t(ss[count]) * 8, kTempAlign) : 0;
    return LCPP_OK;
}

extern "C" lcpp_status lcpp_dist_merge_sorted_batch(void* temp, size_t temp_bytes, int count, const void* const* a,
                                                    const uint64_t* na, const void* const* b, const uint64_t* nb,
                                                    void* const* out, lcpp_dtype key_dtype, lcpp_stream_t stream)
{
    using namespace lcpp;
    using namespace lcpp::dist;
    const int kb = dtype_bytes(key_dtype);
    if (!kb) return LCPP_ERR_UNSUPPORTED_DTYPE;
    if (count < 0 || count > LCPP_MERGE_BATCH_MAX) return LCPP_ERR_INVALID_ARG;
    if (count == 0) return LCPP_OK;
    if (!a || !na || !b || !nb || !out) return LCPP_ERR_INVALID_ARG;
    uint64_t grand = 0;
    for (int m = 0; m < count; ++m) {
        if ((na[m] && !a[m]) || (nb[m] && !b[m]) || (na[m] + nb[m] && !out[m])) return LCPP_ERR_INVALID_ARG;
        grand += na[m] + nb[m];
    }
    if (grand == 0) return LCPP_OK;
    size_t need = 0;
    lcpp_status st = lcpp_dist_merge_batch_temp_bytes(count, na, nb, &need);
    if (st != LCPP_OK) return st;
    if (!temp || (reinterpret_cast<uintptr_t>(temp) & (kTempAlign - 1))) return LCPP_ERR_INVALID_ARG;
    if (temp_bytes < need) return LCPP_ERR_TEMP_TOO_SMALL;
    // byte 4: the error word of the merge's bounded waits; split points after the control area
    uint32_t* error = reinterpret_cast<uint32_t*>(static_cast<unsigned char*>(temp) + 4);
    uint64_t* splits = reinterpret_cast<uint64_t*>(static_cast<unsigned char*>(temp) + kMergeCtrlBytes);
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    if (cudaMemsetAsync(temp, 0, kMergeCtrlBytes, s) != cudaSuccess) return LCPP_ERR_CUDA;
    int dev = 0, sms = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
        return LCPP_ERR_CUDA;
    const bool plain = key_dtype == LCPP_U32 || key_dtype == LCPP_U64;
    auto go = [&](auto tag) {
        using U = decltype(tag);
        MergeBatch<U> mb{};
        mb.count = count;
        batch_layout(count, na, nb, mb.block_start, mb.split_start);
        for (int m = 0; m < count; ++m) {
            mb.a[m] = static_cast<const U*>(a[m]);
            mb.b[m] = static_cast<const U*>(b[m]);
            mb.out[m] = static_cast<U*>(out[m]);
            mb.na[m] = na[m];
            mb.nb[m] = nb[m];
        }
        const auto c = make_codec<U>(key_dtype, false);
        const unsigned sgrid = unsigned(ceil_div(mb.split_start[count], 256));
        merge_split_kernel<U><<<sgrid, 256, 0, s>>>(mb, splits, c);
        const uint64_t blocks = mb.block_start[count];
        if (blocks == 0) return;
        // persistent: as many blocks as are resident
        auto launch = [&](auto kernel) {
            constexpr size_t smem = merge_smem_bytes<U>();
            int per_sm = 0;
            if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)) != cudaSuccess ||
                cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, kMergeBlock, smem) != cudaSuccess)
                return;  // reported by cudaGetLastError below
            const uint64_t resident = uint64_t(sms > 0 ? sms : 1) * uint64_t(per_sm > 0 ? per_sm : 1);
            diag::KernelTimer timer(5 /* LCPP_KERNEL_MERGE */, mb.split_start[count] - count, s);
            kernel<<<unsigned(std::min(blocks, resident)), kMergeBlock, smem, s>>>(mb, splits, c, blocks, error);
        };
        if (plain)
            launch(merge_bulk_kernel<U, true>);
        else
            launch(merge_bulk_kernel<U, false>);
    };
    if (kb == 4)
        go(uint32_t{});
    else
        go(uint64_t{});
    return cudaGetLastError() == cudaSuccess ? LCPP_OK : LCPP_ERR_CUDA;
}

extern "C" lcpp_status lcpp_dist_merge_temp_bytes(uint64_t total, size_t* temp_bytes)
{
    if (!temp_bytes) return LCPP_ERR_INVALID_ARG;
    const uint64_t zero = 0;
    return lcpp_dist_merge_batch_temp_bytes(total ? 1 : 0, &total, &zero, temp_bytes);
}

extern "C" lcpp_status lcpp_dist_merge_sorted(void* temp, size_t temp_bytes, const void* a, uint64_t na,
                                              const void* b, uint64_t nb, void* out, lcpp_dtype key_dtype,
                                              lcpp_stream_t stream)
{
    return lcpp_dist_merge_sorted_batch(temp, temp_bytes, 1, &a, &na, &b, &nb, &out, key_dtype, stream);
}

// ---------------------------------------------------------------------------
// Exchange buffers shared through CUDA IPC.
// ---------------------------------------------------------------------------
static_assert(sizeof(cudaIpcMemHandle_t) == LCPP_IPC_HANDLE_BYTES, "IPC handle size");

extern "C" lcpp_status lcpp_dist_ipc_alloc(size_t bytes, void** dptr, void* handle)
{
    if (!dptr || !handle || bytes == 0) return LCPP_ERR_INVALID_ARG;
    *dptr = nullptr;
    void* p = nullptr;
    if (cudaMalloc(&p, bytes) != cudaSuccess) {
        cudaGetLastError();
        return LCPP_ERR_CUDA;
    }
    cudaIpcMemHandle_t h;
    if (cudaIpcGetMemHandle(&h, p) != cudaSuccess) {
        cudaGetLastError();
        cudaFree(p);
        return LCPP_ERR_CUDA;
    }
    memcpy(handle, &h, sizeof(h));
    *dptr = p;
    return LCPP_OK;
}

extern "C" lcpp_status lcpp_dist_ipc_open(const void* handle, void** dptr)
{
    if (!dptr || !handle) return LCPP_ERR_INVALID_ARG;
    *dptr = nullptr;
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof(h));
    void* p = nullptr;
    if (cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
        cudaGetLastError();
        return LCPP_ERR_CUDA;
    }
    *dptr = p;
    return LCPP_OK;
}

extern "C" lcpp_status lcpp_dist_ipc_close(void* dptr)
{
    if (!dptr) return LCPP_ERR_INVALID_ARG;
    if (cudaIpcCloseMemHandle(dptr) != cudaSuccess) {
        cudaGetLastError();
        return LCPP_ERR_CUDA;
    }
    return LCPP_OK;
}

extern "C" lcpp_status lcpp_dist_ipc_free(void* dptr)
{
    if (!dptr) return LCPP_ERR_INVALID_ARG;
    if (cudaFree(dptr) != cudaSuccess) {
        cudaGetLastError();
        return LCPP_ERR_CUDA;
    }
    return LCPP_OK;
}
