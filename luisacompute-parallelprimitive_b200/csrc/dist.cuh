// dist.cuh -- device helpers shared by the distributed sort's kernels.
#pragma once

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

// Number of keys of sorted[0, n) (ascending by image) whose image is < q
// (upper: <= q).
template <typename U>
__device__ __forceinline__ uint64_t count_below(const U* __restrict__ sorted, uint64_t n, U q, bool upper,
                                                const KeyCodec<U>& c)
{
    uint64_t lo = 0, hi = n;
    while (lo < hi) {
        const uint64_t mid = lo + (hi - lo) / 2;
        const U v = key_image(sorted[mid], c);
        if (upper ? (v <= q) : (v < q))
            lo = mid + 1;
        else
            hi = mid;
    }
    return lo;
}

}  // namespace dist
}  // namespace lcpp
