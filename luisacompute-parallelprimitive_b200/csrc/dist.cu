// dist.cu -- device building blocks of the distributed sort
// (include/lcpp_b200_dist.h).
#include <cstring>

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

// One output tile per block: gather a[i0, i1) ++ b[j0, j1) into shared
// memory, each thread finds where its kMergeItems outputs start (co-rank by
// binary search in shared memory, 32-bit indices) and merges them serially
// with one shared-memory load per output, then the tile is stored coalesced.
template <typename U, bool PLAIN>
__global__ void __launch_bounds__(kMergeBlock)
merge_block_kernel(const MergeBatch<U> mb, const uint64_t* __restrict__ all_splits, KeyCodec<U> codec)
{
    __shared__ U s[kMergeTile];
    const int tid = threadIdx.x;
    const int m = batch_slot(mb.block_start, mb.count, blockIdx.x);
    const uint64_t blk = blockIdx.x - mb.block_start[m];
    const U* __restrict__ a = mb.a[m];
    const U* __restrict__ b = mb.b[m];
    U* __restrict__ out = mb.out[m];
    const uint64_t* splits = all_splits + mb.split_start[m];
    const uint64_t total = mb.na[m] + mb.nb[m];
    const uint64_t o0 = blk * kMergeTile;
    const uint64_t o1 = min(o0 + kMergeTile, total);
    const uint64_t i0 = splits[blk], i1 = splits[blk + 1];
    const uint64_t j0 = o0 - i0, j1 = o1 - i1;
    const int la = int(i1 - i0), lb = int(j1 - j0), len = int(o1 - o0);
    // Gather: all of a thread's loads are issued before any is stored, so
    // their latencies (HBM, or NVLink when a run lives in another GPU's
    // memory) overlap.
    {
        const U* pa = a + i0;
        const U* pb = b + j0 - la;  // pb[idx] = b[j0 + idx - la] for idx >= la
        U v[kMergeItems];
#pragma unroll
        for (int k = 0; k < kMergeItems; ++k) {
            const int idx = tid + k * kMergeBlock;
            if (idx < len) v[k] = (idx < la ? pa : pb)[idx];
        }
#pragma unroll
        for (int k = 0; k < kMergeItems; ++k) {
            const int idx = tid + k * kMergeBlock;
            if (idx < len) s[idx] = v[k];
        }
    }
    __syncthreads();
    U v[kMergeItems];
    const int ot = tid * kMergeItems;
    if (ot < len) {
        // co-rank: number of a-keys among this thread's first ot outputs
        int lo = ot > lb ? ot - lb : 0;
        int hi = ot < la ? ot : la;
        while (lo < hi) {
            const int mid = (lo + hi) >> 1;
            if (merge_image<PLAIN>(s[mid], codec) <= merge_image<PLAIN>(s[la + ot - mid - 1], codec))
                lo = mid + 1;
            else
                hi = mid;
        }
        // serial merge; ia / ib index s[] (the b part starts at la)
        int ia = lo, ib = la + ot - lo;
        const int a_end = la, b_end = la + lb;
        U ka = s[ia < b_end ? ia : b_end - 1];
        U kb = s[ib < b_end ? ib : b_end - 1];
#pragma unroll
        for (int k = 0; k < kMergeItems; ++k) {
            const bool take_a =
                ib >= b_end || (ia < a_end && merge_image<PLAIN>(ka, codec) <= merge_image<PLAIN>(kb, codec));
            v[k] = take_a ? ka : kb;
            int next = take_a ? ++ia : ++ib;
            next = next < b_end ? next : b_end - 1;
            const U x = s[next];
            ka = take_a ? x : ka;
            kb = take_a ? kb : x;
        }
    }
    __syncthreads();
    if (ot < len) {
#pragma unroll
        for (int k = 0; k < kMergeItems; ++k)
            if (ot + k < len) s[ot + k] = v[k];
    }
    __syncthreads();
#pragma unroll
    for (int k = 0; k < kMergeItems; ++k) {
        const int idx = tid + k * kMergeBlock;
        if (idx < len) out[o0 + idx] = s[idx];
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
    *temp_bytes = count ? align_up(size_t(ss[count]) * 8, kTempAlign) : 0;
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
    uint64_t* splits = static_cast<uint64_t*>(temp);
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
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
        const unsigned grid = unsigned(mb.block_start[count]);
        if (grid == 0) return;
        diag::KernelTimer timer(5 /* LCPP_KERNEL_MERGE */, mb.split_start[count] - count, s);
        if (plain)
            merge_block_kernel<U, true><<<grid, kMergeBlock, 0, s>>>(mb, splits, c);
        else
            merge_block_kernel<U, false><<<grid, kMergeBlock, 0, s>>>(mb, splits, c);
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
