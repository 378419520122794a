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
