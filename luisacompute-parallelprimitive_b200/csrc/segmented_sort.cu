// segmented_sort.cu -- DeviceSegmentedRadixSort for sm_100a.
//
// Replaces src/lcpp/device/device_segmented_radix_sort.h (a stable
// per-segment sort by the key bits [begin_bit, end_bit) after the radix
// bijection, ascending or descending, :216-243) of the reference, which runs
// it as a segmented merge sort (device_segmented_sort.h).  Segment rule, as
// in the reference (device_segmented_sort.h:753-775): item i belongs to the
// last segment s with begin[s] <= i, when i < end[s] and
// begin[s] <= end[s] <= num_items; other items are not written.  Unlike
// DeviceRadixSort, +0.0 and -0.0 are different keys here (no fold).
//
// B200 design.  Segments of at most kSmallMax (2048) items: one block each
// sorts its segment in shared memory (stable 8-bit LSD passes), reading and
// writing every key once.  Longer segments, when the blocks found any (their
// item count is read back: one host sync), are sorted together by one
// onesweep sort of the whole array, in which the items of short segments
// count as inactive:
//   1. build: one thread per item finds its segment by binary search over
//      the begin offsets and writes the composite key
//      (segment << kb) | key_bits (inactive items get segment =
//      num_segments and sort last) and its index;
//   2. one stable LSD pairs sort (onesweep, DoubleBuffer form in temp) of
//      the composite keys with the indices as values; when the composite
//      does not fit 64 bits, two stable sorts (key bits, then segment);
//   3. heads: first sorted position of each item's segment, by an inclusive
//      max-scan (DeviceScan) of "position if a segment starts here";
//   4. scatter: sorted item j of segment s goes to begin[s] + j - first[j]
//      (through a stash when the output buffer is the input buffer).
// Temp storage depends on num_items only (as the reference's query).
#include <cstdint>
#include <type_traits>

#include "../../include/lcpp_b200.h"
#include "common.cuh"
#include "radix_sort.cuh"
#include "scan.cuh"

namespace lcpp {
namespace seg {

constexpr int kBlock = 256;

constexpr int kSmallBlock = 256;
constexpr int kSmallItems = 8;
constexpr int kSmallMax = kSmallBlock * kSmallItems;  // keys of a segment sorted by one block

// Members of segment s under the reference's rule, for segments in
// ascending order of begin offset: [begin[s], min(end[s], begin[s + 1]))
// when begin[s] <= end[s] <= n, else none.
__device__ __forceinline__ void segment_members(uint32_t s, const uint32_t* __restrict__ begin,
                                                const uint32_t* __restrict__ end, uint32_t num_segments, uint64_t n,
                                                uint64_t& lo, uint64_t& hi)
{
    lo = begin[s];
    const uint64_t e = end[s];
    if (!(lo <= e && e <= n)) {
        hi = lo;
        return;
    }
    const uint64_t next = s + 1 < num_segments ? uint64_t(begin[s + 1]) : e;
    hi = next < e ? (next > lo ? next : lo) : e;
}

// Segment of item i under the reference's rule, or num_segments.  With
// `large_only`, segments of at most kSmallMax members (sorted by the
// one-block kernel) count as no segment.
__device__ __forceinline__ uint32_t segment_of(uint64_t i, const uint32_t* __restrict__ begin,
                                               const uint32_t* __restrict__ end, uint32_t num_segments, uint64_t n,
                                               bool large_only = false)
{
    uint32_t lo = 0, hi = num_segments;  // number of segments with begin <= i
    while (lo < hi) {
        const uint32_t mid = lo + (hi - lo) / 2;
        if (uint64_t(begin[mid]) <= i)
            lo = mid + 1;
        else
            hi = mid;
    }
    if (lo == 0) return num_segments;
    const uint32_t s = lo - 1;
    const uint64_t b = begin[s], e = end[s];
    if (!(b <= i && i < e && b <= e && e <= n)) return num_segments;
    if (large_only) {
        uint64_t mlo, mhi;
        segment_members(s, begin, end, num_segments, n, mlo, mhi);
        if (mhi - mlo <= uint64_t(kSmallMax)) return num_segments;
    }
    return s;
}

// Key bits [begin_bit, begin_bit + kb) of the radix bijection (no +-0 fold),
// inverted within the field for descending order.
template <typename U>
__device__ __forceinline__ uint64_t key_field(U k, const KeyCodec<U>& c, int begin_bit, uint64_t mask, bool desc)
{
    constexpr int kBits = sizeof(U) * 8;
    using S = typename std::conditional<sizeof(U) == 4, int32_t, int64_t>::type;
    const U sign = U(S(k) >> (kBits - 1));
    const U t = k ^ U(c.xor_pos ^ (sign & (c.xor_pos ^ c.xor_neg)));
    uint64_t f = (uint64_t(t) >> begin_bit) & mask;
    return desc ? (mask - f) : f;
}

template <typename U, typename CT>
__global__ void build_kernel(const U* __restrict__ keys, uint64_t n, const uint32_t* __restrict__ begin,
                             const uint32_t* __restrict__ end, uint32_t num_segments, KeyCodec<U> codec,
                             int begin_bit, uint64_t mask, int key_bits, int desc, int with_segment, int large_only,
                             CT* __restrict__ comp, uint32_t* __restrict__ idx)
{
    for (uint64_t i = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += uint64_t(gridDim.x) * blockDim.x) {
        uint64_t c = key_bits ? key_field(keys[i], codec, begin_bit, mask, desc != 0) : 0;
        if (with_segment) c |= uint64_t(segment_of(i, begin, end, num_segments, n, large_only != 0)) << key_bits;
        comp[i] = CT(c);
        idx[i] = uint32_t(i);
    }
}

// Second key of the two-sort path: the segment of each (key-sorted) item.
__global__ void segment_key_kernel(const uint32_t* __restrict__ idx, uint64_t n, const uint32_t* __restrict__ begin,
                                   const uint32_t* __restrict__ end, uint32_t num_segments, int large_only,
                                   uint64_t* __restrict__ comp)
{
    for (uint64_t j = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x; j < n; j += uint64_t(gridDim.x) * blockDim.x)
        comp[j] = segment_of(idx[j], begin, end, num_segments, n, large_only != 0);
}

// ---------------------------------------------------------------------------
// Short segments: one block sorts a segment of at most kSmallMax keys in
// shared memory -- a stable LSD radix sort over the key field, 8 bits per
// pass, ranked like the onesweep tile (lanes holding the same digit from
// low-5-bit shared mask words and 3 ballots, per-warp digit counters, a
// block scan over digits and warps), so every key is read and written once
// in global memory.
// Blocks of longer segments only add their length to *large_items.
// ---------------------------------------------------------------------------
template <typename U, typename V, bool PAIRS>
__global__ void __launch_bounds__(kSmallBlock)
small_segment_kernel(const U* __restrict__ keys_in, U* __restrict__ keys_out, const V* __restrict__ vals_in,
                     V* __restrict__ vals_out, uint64_t n, const uint32_t* __restrict__ begin,
                     const uint32_t* __restrict__ end, uint32_t num_segments, KeyCodec<U> codec, int begin_bit,
                     int key_bits, int desc, unsigned long long* __restrict__ large_items)
{
    constexpr int kWarps = kSmallBlock / 32;
    __shared__ U s_keys[kSmallMax];
    __shared__ V s_vals[PAIRS ? kSmallMax : 1];
    __shared__ uint32_t s_count[kWarps][256];
    __shared__ uint32_t s_masks[2][kWarps][32];  // per slot parity: lanes of each low-5-bit digit class
    __shared__ uint32_t s_warp_sum[kWarps];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const uint64_t mask = key_bits >= 64 ? ~uint64_t(0) : ((uint64_t(1) << key_bits) - 1);
    const int passes = (key_bits + 7) / 8;
    const uint32_t lt = (1u << lane) - 1u;
    const uint32_t counters_base = static_cast<uint32_t>(__cvta_generic_to_shared(&s_count[warp][0]));
    const uint32_t masks_base = static_cast<uint32_t>(__cvta_generic_to_shared(&s_masks[0][warp][0]));
    constexpr uint32_t kSetBytes = kWarps * 32 * 4;

    for (int d = tid; d < kWarps * 256; d += kSmallBlock) (&s_count[0][0])[d] = 0;
    for (int d = tid; d < 2 * kWarps * 32; d += kSmallBlock) (&s_masks[0][0][0])[d] = 0;
    __syncthreads();

    for (uint64_t seg = blockIdx.x; seg < num_segments; seg += gridDim.x) {
        uint64_t lo, hi;
        segment_members(uint32_t(seg), begin, end, num_segments, n, lo, hi);
        const int len = int(hi - lo > uint64_t(kSmallMax) ? kSmallMax + 1 : hi - lo);
        if (len > kSmallMax) {
            if (tid == 0) atomicAdd(large_items, (unsigned long long)(hi - lo));
            continue;
        }
        if (len == 0) continue;
        // load: slot i of lane l of warp w is position w * 8 * 32 + i * 32 + l
        U k[kSmallItems];
        V v[PAIRS ? kSmallItems : 1];
#pragma unroll
        for (int i = 0; i < kSmallItems; ++i) {
            const int p = warp * kSmallItems * 32 + i * 32 + lane;
            if (p < len) {
                k[i] = keys_in[lo + p];
                if constexpr (PAIRS) v[i] = vals_in[lo + p];
            }
        }
        // The digit counters are zero here (zeroed at start and after every
        // pass's scatter).
        for (int pass = 0; pass < passes && len > 1; ++pass) {
            uint32_t dig[kSmallItems], rank[kSmallItems];
#pragma unroll
            for (int i = 0; i < kSmallItems; ++i) {
                const int slot = warp * kSmallItems * 32 + i * 32;  // first position of this warp slot
                const int p = slot + lane;
                rank[i] = 0;
                dig[i] = 0;
                if (slot >= len) continue;  // warp-uniform: no key of this slot exists
                // positions past the end take digit 255 and rank after every key
                dig[i] = p < len ? uint32_t(key_field(k[i], codec, begin_bit, mask, desc != 0) >> (8 * pass)) & 0xffu
                                 : 0xffu;
                // lanes of the same digit: a shared mask word per low-5-bit
                // class (one per bank), narrowed by 3 ballots; the word is
                // cleared once every lane has read it (the shuffle below
                // depends on every lane's read), and the other parity's words
                // serve the next slot
                const uint32_t maddr = masks_base + uint32_t(i & 1) * kSetBytes + (dig[i] & 31u) * 4u;
                shared_red_or(maddr, 1u << lane);
                warp_barrier();
                uint32_t peers = shared_load(maddr);
#pragma unroll
                for (int b = 5; b < 8; ++b) {
                    const bool bit = (dig[i] >> b) & 1u;
                    const uint32_t vote = warp_ballot(bit);
                    peers &= bit ? vote : ~vote;
                }
                const int leader = 31 - __clz(peers);
                uint32_t base = shared_add_if(lane == leader, counters_base + dig[i] * 4u, uint32_t(__popc(peers)));
                base = warp_shfl(base, leader);
                shared_store_if(true, maddr, 0u);
                rank[i] = base + __popc(peers & lt);
            }
            __syncthreads();
            // digit d (one per thread): exclusive prefix over digits, then over warps
            {
                uint32_t tot = 0;
#pragma unroll
                for (int w = 0; w < kWarps; ++w) tot += s_count[w][tid];
                uint32_t incl = tot;
#pragma unroll
                for (int o = 1; o < 32; o <<= 1) {
                    const uint32_t y = __shfl_up_sync(0xffffffffu, incl, o);
                    if (lane >= o) incl += y;
                }
                if (lane == 31) s_warp_sum[warp] = incl;
                __syncthreads();
                uint32_t run = incl - tot;
                for (int w = 0; w < warp; ++w) run += s_warp_sum[w];
#pragma unroll
                for (int w = 0; w < kWarps; ++w) {
                    const uint32_t c = s_count[w][tid];
                    s_count[w][tid] = run;
                    run += c;
                }
            }
            __syncthreads();
#pragma unroll
            for (int i = 0; i < kSmallItems; ++i) {
                if (warp * kSmallItems * 32 + i * 32 >= len) continue;
                const uint32_t r = s_count[warp][dig[i]] + rank[i];
                s_keys[r] = k[i];
                if constexpr (PAIRS) s_vals[r] = v[i];
            }
            __syncthreads();
            // reload in the new order; the counters are free again
#pragma unroll
            for (int w = 0; w < kWarps; ++w) s_count[w][tid] = 0;
#pragma unroll
            for (int i = 0; i < kSmallItems; ++i) {
                const int p = warp * kSmallItems * 32 + i * 32 + lane;
                if (p - lane >= len) continue;
                k[i] = s_keys[p];
                if constexpr (PAIRS) v[i] = s_vals[p];
            }
            __syncthreads();
        }
#pragma unroll
        for (int i = 0; i < kSmallItems; ++i) {
            const int p = warp * kSmallItems * 32 + i * 32 + lane;
            if (p < len) {
                keys_out[lo + p] = k[i];
                if constexpr (PAIRS) vals_out[lo + p] = v[i];
            }
        }
    }
}

// heads[j] = j where a segment's run starts in sorted order, else 0.
template <typename CT>
__global__ void heads_kernel(const CT* __restrict__ comp, uint64_t n, int shift, uint32_t* __restrict__ heads)
{
    for (uint64_t j = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x; j < n; j += uint64_t(gridDim.x) * blockDim.x)
        heads[j] = (j == 0 || (uint64_t(comp[j]) >> shift) != (uint64_t(comp[j - 1]) >> shift)) ? uint32_t(j) : 0u;
}

template <typename T>
__global__ void gather_kernel(const T* __restrict__ src, const uint32_t* __restrict__ idx, uint64_t n,
                              T* __restrict__ dst)
{
    for (uint64_t j = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x; j < n; j += uint64_t(gridDim.x) * blockDim.x)
        dst[j] = src[idx[j]];
}

// out[begin[s] + j - first[j]] = item j in sorted order (items of the
// inactive class s == num_segments are skipped).  `src` is the stash
// (sorted order) when `idx` is null, else the input gathered through idx.
template <typename T, typename CT>
__global__ void scatter_kernel(const T* __restrict__ src, const uint32_t* __restrict__ idx,
                               const CT* __restrict__ comp, const uint32_t* __restrict__ first, uint64_t n, int shift,
                               uint32_t num_segments, const uint32_t* __restrict__ begin, T* __restrict__ out)
{
    for (uint64_t j = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x; j < n; j += uint64_t(gridDim.x) * blockDim.x) {
        const uint64_t s = uint64_t(comp[j]) >> shift;
        if (s >= num_segments) continue;
        out[uint64_t(begin[s]) + (j - first[j])] = idx ? src[idx[j]] : src[j];
    }
}

struct Layout {
    size_t comp0, comp1, idx0, idx1, heads, first, stash_k, stash_v, scan, sort, large, total;
};

Layout make_layout(int kb, int vb, uint64_t n)
{
    Layout L{};
    size_t off = 0;
    auto take = [&](size_t bytes) {
        const size_t at = off;
        off = align_up(off + bytes, kTempAlign);
        return at;
    };
    L.sort = take(radix::temp_bytes(8, 4, n));  // first: lcpp_device_status reads its error word
    L.comp0 = take(size_t(n) * 8);
    L.comp1 = take(size_t(n) * 8);
    L.idx0 = take(size_t(n) * 4);
    L.idx1 = take(size_t(n) * 4);
    L.heads = take(size_t(n) * 4);
    L.first = take(size_t(n) * 4);
    L.stash_k = take(size_t(n) * kb);
    L.stash_v = take(size_t(n) * vb);
    L.scan = take(scan::temp_bytes(LCPP_U32, n));
    L.large = take(sizeof(unsigned long long));  // items in segments too long for one block
    L.total = off;
    return L;
}

unsigned grid_for(uint64_t n)
{
    const uint64_t blocks = ceil_div(n, uint64_t(kBlock));
    const uint64_t cap = uint64_t(device_sm_count()) * 16;
    return unsigned(blocks < cap ? blocks : cap);
}

int bit_length(uint64_t v)
{
    int b = 0;
    while (v) {
        ++b;
        v >>= 1;
    }
    return b;
}

template <typename T>
void launch_gather(const void* src, const uint32_t* idx, uint64_t n, void* dst, cudaStream_t s)
{
    gather_kernel<T><<<grid_for(n), kBlock, 0, s>>>(static_cast<const T*>(src), idx, n, static_cast<T*>(dst));
}

template <typename CT>
void launch_scatter(int eb, const void* src, const uint32_t* idx, const CT* comp, const uint32_t* first, uint64_t n,
                    int shift, uint32_t num_segments, const uint32_t* begin, void* out, cudaStream_t s)
{
    if (eb == 4)
        scatter_kernel<uint32_t, CT><<<grid_for(n), kBlock, 0, s>>>(static_cast<const uint32_t*>(src), idx, comp,
                                                                     first, n, shift, num_segments, begin,
                                                                     static_cast<uint32_t*>(out));
    else
        scatter_kernel<uint64_t, CT><<<grid_for(n), kBlock, 0, s>>>(static_cast<const uint64_t*>(src), idx, comp,
                                                                     first, n, shift, num_segments, begin,
                                                                     static_cast<uint64_t*>(out));
}

template <typename U>
void launch_build(const void* keys, uint64_t n, const uint32_t* begin, const uint32_t* end, uint32_t num_segments,
                  lcpp_dtype kdt, int begin_bit, int key_bits, int desc, bool with_segment, bool wide,
                  void* comp, uint32_t* idx, cudaStream_t s, int large_only)
{
    const KeyCodec<U> codec = make_codec<U>(kdt, false);
    const uint64_t mask = key_bits >= 64 ? ~uint64_t(0) : ((uint64_t(1) << key_bits) - 1);
    if (wide)
        build_kernel<U, uint64_t><<<grid_for(n), kBlock, 0, s>>>(
            static_cast<const U*>(keys), n, begin, end, num_segments, codec, begin_bit, mask, key_bits, desc,
            with_segment, large_only, static_cast<uint64_t*>(comp), idx);
    else
        build_kernel<U, uint32_t><<<grid_for(n), kBlock, 0, s>>>(
            static_cast<const U*>(keys), n, begin, end, num_segments, codec, begin_bit, mask, key_bits, desc,
            with_segment, large_only, static_cast<uint32_t*>(comp), idx);
}

template <typename U, typename V, bool PAIRS>
void launch_small(const void* kin, void* kout, const void* vin, void* vout, uint64_t n, const uint32_t* begin,
                  const uint32_t* end, uint32_t num_segments, lcpp_dtype kdt, int begin_bit, int key_bits, int desc,
                  unsigned long long* large, cudaStream_t s)
{
    const KeyCodec<U> codec = make_codec<U>(kdt, false);
    const uint64_t cap = uint64_t(device_sm_count()) * 8;
    const unsigned grid = unsigned(num_segments < cap ? num_segments : cap);
    diag::KernelTimer timer(4 /* LCPP_KERNEL_SEGMENT_BLOCK */, n, s);
    small_segment_kernel<U, V, PAIRS><<<grid, kSmallBlock, 0, s>>>(
        static_cast<const U*>(kin), static_cast<U*>(kout), static_cast<const V*>(vin), static_cast<V*>(vout), n,
        begin, end, num_segments, codec, begin_bit, key_bits, desc, large);
}

}  // namespace seg

// Shared implementation of the segmented entry points (see the C ABI in
// include/lcpp_b200.h).
lcpp_status segmented_sort(void* temp, size_t temp_bytes_given, const void* keys_in, void* keys_out,
                           const void* vals_in, void* vals_out, void* key_bufs[2], void* val_bufs[2], int* selector,
                           uint64_t n, uint64_t num_segments, const uint32_t* begin_offsets,
                           const uint32_t* end_offsets, int begin_bit, int end_bit, int descending, lcpp_dtype kdt,
                           lcpp_dtype vdt, bool pairs, bool double_buffer, cudaStream_t stream)
{
    diag::Range nvtx_range("lcpp DeviceSegmentedRadixSort");
    using namespace seg;
    const int kb = dtype_bytes(kdt);
    const int vb = pairs ? dtype_bytes(vdt) : 0;
    if (!kb || (pairs && !vb)) return LCPP_ERR_UNSUPPORTED_DTYPE;
    if (begin_bit < 0 || begin_bit > end_bit || end_bit > kb * 8) return LCPP_ERR_INVALID_ARG;
    if (n > 0xffffffffull || num_segments > 0xffffffffull) return LCPP_ERR_INVALID_ARG;
    if (double_buffer) {
        if (!selector || (*selector != 0 && *selector != 1)) return LCPP_ERR_INVALID_ARG;
        if (!key_bufs || !key_bufs[0] || !key_bufs[1] || (pairs && (!val_bufs || !val_bufs[0] || !val_bufs[1])))
            return LCPP_ERR_INVALID_ARG;
        // the reference runs ceil(log2 n) merge passes, each flipping the
        // selector; nothing at all for n <= 1, no segments, or an empty bit
        // range (device_segmented_sort.h:229-246, device_segmented_radix_sort.h:69-73)
        if (n <= 1 || num_segments == 0 || begin_bit == end_bit) return LCPP_OK;
    } else if (n == 0 || num_segments == 0) {
        return LCPP_OK;
    }
    if (!begin_offsets || !end_offsets) return LCPP_ERR_INVALID_ARG;
    const int sel = double_buffer ? *selector : 0;
    const void* kin = double_buffer ? key_bufs[sel] : keys_in;
    const void* vin = double_buffer ? (pairs ? val_bufs[sel] : nullptr) : vals_in;
    const int flips = double_buffer ? bit_length(n - 1) : 0;
    void* kout = double_buffer ? key_bufs[sel ^ (flips & 1)] : keys_out;
    void* vout = double_buffer ? (pairs ? val_bufs[sel ^ (flips & 1)] : nullptr) : vals_out;
    if (!kin || !kout || (pairs && (!vin || !vout))) return LCPP_ERR_INVALID_ARG;
    if ((reinterpret_cast<uintptr_t>(kin) | reinterpret_cast<uintptr_t>(kout)) % kb) return LCPP_ERR_INVALID_ARG;
    if (pairs && (reinterpret_cast<uintptr_t>(vin) | reinterpret_cast<uintptr_t>(vout)) % vb)
        return LCPP_ERR_INVALID_ARG;
    if (!temp || (reinterpret_cast<uintptr_t>(temp) & (kTempAlign - 1))) return LCPP_ERR_INVALID_ARG;
    const Layout L = make_layout(kb, vb, n);
    if (temp_bytes_given < L.total) return LCPP_ERR_TEMP_TOO_SMALL;

    unsigned char* t = static_cast<unsigned char*>(temp);
    void* comp[2] = {t + L.comp0, t + L.comp1};
    void* idx[2] = {t + L.idx0, t + L.idx1};
    uint32_t* heads = reinterpret_cast<uint32_t*>(t + L.heads);
    uint32_t* first = reinterpret_cast<uint32_t*>(t + L.first);
    const uint32_t nseg = uint32_t(num_segments);
    const int key_bits = end_bit - begin_bit;
    const int seg_bits = bit_length(num_segments);  // segment ids 0..num_segments (inactive)
    const int total_bits = key_bits + seg_bits;
    const bool one_sort = total_bits <= 64;
    const bool wide = !one_sort || total_bits > 32;  // composite stored as u64
    const lcpp_dtype comp_dt = wide ? LCPP_U64 : LCPP_U32;
    int csel = 0;

    // Short segments: one block each, straight from input to output.
    unsigned long long* large = reinterpret_cast<unsigned long long*>(t + L.large);
    LCPP_CUDA_TRY(cudaMemsetAsync(large, 0, sizeof(unsigned long long), stream));
    {
        auto small = [&](auto ktag, auto vtag, auto pairs_tag) {
            using U = decltype(ktag);
            using V = decltype(vtag);
            launch_small<U, V, decltype(pairs_tag)::value>(kin, kout, vin, vout, n, begin_offsets, end_offsets, nseg,
                                                           kdt, begin_bit, key_bits, descending, large, stream);
        };
        using T_ = std::true_type;
        using F_ = std::false_type;
        if (!pairs)
            kb == 4 ? small(uint32_t{}, uint32_t{}, F_{}) : small(uint64_t{}, uint32_t{}, F_{});
        else if (kb == 4)
            vb == 4 ? small(uint32_t{}, uint32_t{}, T_{}) : small(uint32_t{}, uint64_t{}, T_{});
        else
            vb == 4 ? small(uint64_t{}, uint32_t{}, T_{}) : small(uint64_t{}, uint64_t{}, T_{});
    }
    // Longer segments (if any): the composite sort below, restricted to
    // them.  Reading their item count back is the call's one host sync.
    unsigned long long large_items = 0;
    LCPP_CUDA_TRY(cudaMemcpyAsync(&large_items, large, sizeof(large_items), cudaMemcpyDeviceToHost, stream));
    LCPP_CUDA_TRY(cudaStreamSynchronize(stream));
    if (large_items == 0) {
        if (cudaGetLastError() != cudaSuccess) return LCPP_ERR_CUDA;
        if (double_buffer) *selector ^= (flips & 1);
        return LCPP_OK;
    }
    
    auto run_sort = [&](int bits) -> lcpp_status {
        return radix::sort(t + L.sort, radix::temp_bytes(8, 4, n), nullptr, nullptr, nullptr, nullptr, comp, idx,
                           &csel, n, 0, bits, 0, comp_dt, LCPP_U32, true, true, stream);
    };

    if (one_sort) {
        if (kb == 4)
            launch_build<uint32_t>(kin, n, begin_offsets, end_offsets, nseg, kdt, begin_bit, key_bits, descending,
                                   true, wide, comp[0], static_cast<uint32_t*>(idx[0]), stream, 1);
        else
            launch_build<uint64_t>(kin, n, begin_offsets, end_offsets, nseg, kdt, begin_bit, key_bits, descending,
                                   true, wide, comp[0], static_cast<uint32_t*>(idx[0]), stream, 1);
        lcpp_status st = run_sort(total_bits);
        if (st != LCPP_OK) return st;
    } else {
        // key bits first, then a stable sort by segment
        if (kb == 4)
            launch_build<uint32_t>(kin, n, begin_offsets, end_offsets, nseg, kdt, begin_bit, key_bits, descending,
                                   false, true, comp[0], static_cast<uint32_t*>(idx[0]), stream, 1);
        else
            launch_build<uint64_t>(kin, n, begin_offsets, end_offsets, nseg, kdt, begin_bit, key_bits, descending,
                                   false, true, comp[0], static_cast<uint32_t*>(idx[0]), stream, 1);
        lcpp_status st = run_sort(key_bits);
        if (st != LCPP_OK) return st;
        segment_key_kernel<<<grid_for(n), kBlock, 0, stream>>>(static_cast<const uint32_t*>(idx[csel]), n,
                                                              begin_offsets, end_offsets, nseg, 1,
                                                              static_cast<uint64_t*>(comp[csel]));
        st = run_sort(seg_bits);
        if (st != LCPP_OK) return st;
    }
    const int shift = one_sort ? key_bits : 0;
    const uint32_t* sidx = static_cast<const uint32_t*>(idx[csel]);

    // first sorted position of each item's segment
    if (wide)
        heads_kernel<uint64_t><<<grid_for(n), kBlock, 0, stream>>>(static_cast<const uint64_t*>(comp[csel]), n, shift,
                                                                   heads);
    else
        heads_kernel<uint32_t><<<grid_for(n), kBlock, 0, stream>>>(static_cast<const uint32_t*>(comp[csel]), n, shift,
                                                                   heads);
    lcpp_status st = scan::run(t + L.scan, scan::temp_bytes(LCPP_U32, n), heads, first, n, LCPP_OP_MAX, nullptr,
                               LCPP_U32, 1, stream);
    if (st != LCPP_OK) return st;

    // keys (and values) into place; through a stash when the output may alias the input
    const bool alias = kout == kin || (pairs && vout == vin);
    auto place = [&](const void* src, void* dst, int eb, void* stash) {
        const uint32_t* use_idx = sidx;
        const void* from = src;
        if (alias) {
            if (eb == 4)
                launch_gather<uint32_t>(src, sidx, n, stash, stream);
            else
                launch_gather<uint64_t>(src, sidx, n, stash, stream);
            use_idx = nullptr;
            from = stash;
        }
        if (wide)
            launch_scatter<uint64_t>(eb, from, use_idx, static_cast<const uint64_t*>(comp[csel]), first, n, shift,
                                     nseg, begin_offsets, dst, stream);
        else
            launch_scatter<uint32_t>(eb, from, use_idx, static_cast<const uint32_t*>(comp[csel]), first, n, shift,
                                     nseg, begin_offsets, dst, stream);
    };
    place(kin, kout, kb, t + L.stash_k);
    if (pairs) place(vin, vout, vb, t + L.stash_v);
    if (cudaGetLastError() != cudaSuccess) return LCPP_ERR_CUDA;
    if (double_buffer) *selector ^= (flips & 1);
    return LCPP_OK;
}

size_t segmented_temp_bytes(int kb, int vb, uint64_t n)
{
    if (n == 0) return 0;
    return seg::make_layout(kb, vb, n).total;
}

}  // namespace lcpp

// ---------------------------------------------------------------------------
// C ABI
// ---------------------------------------------------------------------------
extern "C" lcpp_status lcpp_segmented_radix_sort_keys_temp_bytes(lcpp_dtype key_dtype, uint64_t num_items,
                                                                 size_t* temp_bytes)
{
    if (!temp_bytes) return LCPP_ERR_INVALID_ARG;
    const int kb = lcpp::dtype_bytes(key_dtype);
    if (!kb) return LCPP_ERR_UNSUPPORTED_DTYPE;
    *temp_bytes = lcpp::segmented_temp_bytes(kb, 0, num_items);
    return LCPP_OK;
}

extern "C" lcpp_status lcpp_segmented_radix_sort_pairs_temp_bytes(lcpp_dtype key_dtype, lcpp_dtype value_dtype,
                                                                  uint64_t num_items, size_t* temp_bytes)
{
    if (!temp_bytes) return LCPP_ERR_INVALID_ARG;
    const int kb = lcpp::dtype_bytes(key_dtype), vb = lcpp::dtype_bytes(value_dtype);
    if (!kb || !vb) return LCPP_ERR_UNSUPPORTED_DTYPE;
    *temp_bytes = lcpp::segmented_temp_bytes(kb, vb, num_items);
    return LCPP_OK;
}

extern "C" lcpp_status lcpp_segmented_radix_sort_keys(void* temp, size_t temp_bytes, const void* keys_in,
                                                      void* keys_out, uint64_t num_items, uint64_t num_segments,
                                                      const uint32_t* begin_offsets, const uint32_t* end_offsets,
                                                      int begin_bit, int end_bit, int descending,
                                                      lcpp_dtype key_dtype, lcpp_stream_t stream)
{
    return lcpp::segmented_sort(temp, temp_bytes, keys_in, keys_out, nullptr, nullptr, nullptr, nullptr, nullptr,
                                num_items, num_segments, begin_offsets, end_offsets, begin_bit, end_bit, descending,
                                key_dtype, LCPP_NONE, false, false, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" lcpp_status lcpp_segmented_radix_sort_pairs(void* temp, size_t temp_bytes, const void* keys_in,
                                                       void* keys_out, const void* values_in, void* values_out,
                                                       uint64_t num_items, uint64_t num_segments,
                                                       const uint32_t* begin_offsets, const uint32_t* end_offsets,
                                                       int begin_bit, int end_bit, int descending,
                                                       lcpp_dtype key_dtype, lcpp_dtype value_dtype,
                                                       lcpp_stream_t stream)
{
    return lcpp::segmented_sort(temp, temp_bytes, keys_in, keys_out, values_in, values_out, nullptr, nullptr,
                                nullptr, num_items, num_segments, begin_offsets, end_offsets, begin_bit, end_bit,
                                descending, key_dtype, value_dtype, true, false, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" lcpp_status lcpp_segmented_radix_sort_keys_double_buffer(void* temp, size_t temp_bytes,
                                                                    void* key_buffers[2], int* selector,
                                                                    uint64_t num_items, uint64_t num_segments,
                                                                    const uint32_t* begin_offsets,
                                                                    const uint32_t* end_offsets, int begin_bit,
                                                                    int end_bit, int descending,
                                                                    lcpp_dtype key_dtype, lcpp_stream_t stream)
{
    return lcpp::segmented_sort(temp, temp_bytes, nullptr, nullptr, nullptr, nullptr, key_buffers, nullptr, selector,
                                num_items, num_segments, begin_offsets, end_offsets, begin_bit, end_bit, descending,
                                key_dtype, LCPP_NONE, false, true, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" lcpp_status lcpp_segmented_radix_sort_pairs_double_buffer(
    void* temp, size_t temp_bytes, void* key_buffers[2], void* value_buffers[2], int* selector, uint64_t num_items,
    uint64_t num_segments, const uint32_t* begin_offsets, const uint32_t* end_offsets, int begin_bit, int end_bit,
    int descending, lcpp_dtype key_dtype, lcpp_dtype value_dtype, lcpp_stream_t stream)
{
    return lcpp::segmented_sort(temp, temp_bytes, nullptr, nullptr, nullptr, nullptr, key_buffers, value_buffers,
                                selector, num_items, num_segments, begin_offsets, end_offsets, begin_bit, end_bit,
                                descending, key_dtype, value_dtype, true, true, reinterpret_cast<cudaStream_t>(stream));
}
