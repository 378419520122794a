// dist.cu -- device building blocks of the distributed sort
// (include/lcpp_b200_dist.h).
#include "../../include/lcpp_b200_dist.h"
#include "common.cuh"

namespace lcpp {
namespace dist {

// Order-preserving image of a key (the ascending radix bijection) with the
// +-0.0 fold, i.e. the value whose order the radix sort realises.
template <typename U>
__device__ __forceinline__ U key_image(U k, const KeyCodec<U>& c)
{
    constexpr int kBits = sizeof(U) * 8;
    constexpr U kHigh = U(1) << (kBits - 1);
    using S = typename std::conditional<sizeof(U) == 4, int32_t, int64_t>::type;
    const U sign = U(S(k) >> (kBits - 1));
    U t = k ^ U(c.xor_pos ^ (sign & (c.xor_pos ^ c.xor_neg)));
    if (c.fold_zero && t == U(kHigh - 1)) t = kHigh;
    return t;
}

template <typename U>
__global__ void search_sorted_kernel(const U* __restrict__ sorted, uint64_t n, const U* __restrict__ queries,
                                     uint64_t nq, int upper, uint64_t* __restrict__ out, KeyCodec<U> codec)
{
    const uint64_t i = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= nq) return;
    const U q = queries[i];
    uint64_t lo = 0, hi = n;  // first index whose image is >= q (> q when upper)
    while (lo < hi) {
        const uint64_t mid = lo + (hi - lo) / 2;
        const U v = key_image(sorted[mid], codec);
        if (upper ? (v <= q) : (v < q))
            lo = mid + 1;
        else
            hi = mid;
    }
    out[i] = lo;
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

template <typename U>
__global__ void merge_split_kernel(const U* __restrict__ a, uint64_t na, const U* __restrict__ b, uint64_t nb,
                                   uint64_t* __restrict__ splits, uint64_t nsplits, KeyCodec<U> codec)
{
    const uint64_t k = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (k >= nsplits) return;
    const uint64_t o = min(k * kMergeTile, na + nb);
    splits[k] = co_rank<U>(o, na, nb, [&](uint64_t i) { return key_image(a[i], codec); },
                           [&](uint64_t j) { return key_image(b[j], codec); });
}

template <typename U>
__global__ void __launch_bounds__(kMergeBlock)
merge_block_kernel(const U* __restrict__ a, uint64_t na, const U* __restrict__ b, uint64_t nb,
                   const uint64_t* __restrict__ splits, U* __restrict__ out, KeyCodec<U> codec)
{
    __shared__ U s[kMergeTile];
    const int tid = threadIdx.x;
    const uint64_t total = na + nb;
    const uint64_t o0 = uint64_t(blockIdx.x) * kMergeTile;
    const uint64_t o1 = min(o0 + kMergeTile, total);
    const uint64_t i0 = splits[blockIdx.x], i1 = splits[blockIdx.x + 1];
    const uint64_t j0 = o0 - i0, j1 = o1 - i1;
    const int la = int(i1 - i0), lb = int(j1 - j0), len = int(o1 - o0);
    for (int k = tid; k < la; k += kMergeBlock) s[k] = a[i0 + k];
    for (int k = tid; k < lb; k += kMergeBlock) s[la + k] = b[j0 + k];
    __syncthreads();
    const U* sa = s;
    const U* sb = s + la;
    U v[kMergeItems];
    const int ot = tid * kMergeItems;
    if (ot < len) {
        int ia = int(co_rank<U>(uint64_t(ot), uint64_t(la), uint64_t(lb),
                                [&](uint64_t i) { return key_image(sa[i], codec); },
                                [&](uint64_t j) { return key_image(sb[j], codec); }));
        int ib = ot - ia;
#pragma unroll
        for (int k = 0; k < kMergeItems; ++k) {
            const bool take_a = ia < la && (ib >= lb || key_image(sa[ia], codec) <= key_image(sb[ib], codec));
            v[k] = take_a ? sa[ia] : sb[ib < lb ? ib : lb - 1];
            ia += take_a;
            ib += !take_a;
        }
    }
    __syncthreads();
    if (ot < len) {
#pragma unroll
        for (int k = 0; k < kMergeItems; ++k)
            if (ot + k < len) s[ot + k] = v[k];
    }
    __syncthreads();
    for (int k = tid; k < len; k += kMergeBlock) out[o0 + k] = s[k];
}

inline uint64_t merge_blocks(uint64_t total) { return ceil_div(total, kMergeTile); }

}  // namespace dist
}  // namespace lcpp

extern "C" lcpp_status lcpp_dist_merge_temp_bytes(uint64_t total, size_t* temp_bytes)
{
    if (!temp_bytes) return LCPP_ERR_INVALID_ARG;
    *temp_bytes = total ? lcpp::align_up(size_t(lcpp::dist::merge_blocks(total) + 1) * 8, lcpp::kTempAlign) : 0;
    return LCPP_OK;
}

extern "C" lcpp_status lcpp_dist_merge_sorted(void* temp, size_t temp_bytes, const void* a, uint64_t na,
                                              const void* b, uint64_t nb, void* out, lcpp_dtype key_dtype,
                                              lcpp_stream_t stream)
{
    using namespace lcpp;
    using namespace lcpp::dist;
    const int kb = dtype_bytes(key_dtype);
    if (!kb) return LCPP_ERR_UNSUPPORTED_DTYPE;
    const uint64_t total = na + nb;
    if (total == 0) return LCPP_OK;
    if (!out || (na && !a) || (nb && !b)) return LCPP_ERR_INVALID_ARG;
    size_t need = 0;
    lcpp_dist_merge_temp_bytes(total, &need);
    if (!temp || (reinterpret_cast<uintptr_t>(temp) & (kTempAlign - 1))) return LCPP_ERR_INVALID_ARG;
    if (temp_bytes < need) return LCPP_ERR_TEMP_TOO_SMALL;
    const uint64_t blocks = merge_blocks(total);
    if (blocks + 1 > 0x7fffffffull * 256) return LCPP_ERR_INVALID_ARG;
    uint64_t* splits = static_cast<uint64_t*>(temp);
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    const unsigned sgrid = unsigned(ceil_div(blocks + 1, 256));
    if (kb == 4) {
        const auto c = make_codec<uint32_t>(key_dtype, false);
        merge_split_kernel<uint32_t><<<sgrid, 256, 0, s>>>(static_cast<const uint32_t*>(a), na,
                                                          static_cast<const uint32_t*>(b), nb, splits, blocks + 1, c);
        merge_block_kernel<uint32_t><<<unsigned(blocks), kMergeBlock, 0, s>>>(
            static_cast<const uint32_t*>(a), na, static_cast<const uint32_t*>(b), nb, splits,
            static_cast<uint32_t*>(out), c);
    } else {
        const auto c = make_codec<uint64_t>(key_dtype, false);
        merge_split_kernel<uint64_t><<<sgrid, 256, 0, s>>>(static_cast<const uint64_t*>(a), na,
                                                          static_cast<const uint64_t*>(b), nb, splits, blocks + 1, c);
        merge_block_kernel<uint64_t><<<unsigned(blocks), kMergeBlock, 0, s>>>(
            static_cast<const uint64_t*>(a), na, static_cast<const uint64_t*>(b), nb, splits,
            static_cast<uint64_t*>(out), c);
    }
    return cudaGetLastError() == cudaSuccess ? LCPP_OK : LCPP_ERR_CUDA;
}
