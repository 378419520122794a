/* lcpp_b200_device.cuh -- CUDA templates for the operations whose reference
 * form takes a user callable (for programs compiled with nvcc).
 *
 * DeviceReduce::ArgMin / ArgMax with a comparator
 * (src/lcpp/device/device_reduce.h:360-371, :424-434): the reference
 * compiles the comparator into a one-thread shader that walks the input
 * from item 0 and lets item i replace the best so far when
 * compare(item, best) (ArgMin) or compare(best, item) (ArgMax), i.e. the
 * first index of the extreme equivalence class (:539-605).  Here the same
 * comparator drives a parallel two-level reduction: each thread folds its
 * strided share, warps and blocks combine with shuffles, the last block to
 * finish folds the per-block partials.  Partials combine with "b replaces a
 * when it is strictly better, or equivalent with a smaller index", which is
 * associative and commutative, so for a strict weak order the result is the
 * sequential fold's.  The library's own ArgMin / ArgMax (lcpp_reduce_argmin /
 * lcpp_reduce_argmax) instantiate this kernel with NaturalOrder.
 *
 * Temp storage: lcpp_reduce_arg_temp_bytes(dtype, num_items, &bytes), 256-byte
 * aligned; the comparator is any copyable type with a __device__
 * bool operator()(T, T) (a functor, or a __device__ lambda with
 * --extended-lambda). */
#ifndef LCPP_B200_DEVICE_CUH
#define LCPP_B200_DEVICE_CUH

#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include <algorithm>
#include <limits>

namespace lcpp_b200 {
namespace device {

/* Index of "no item yet"; never a real index, since num_items < 2^32. */
constexpr uint32_t kArgNone = 0xffffffffu;

/* <, == and "NaN never wins" (the reference's ArgMinOp / ArgMaxOp,
 * src/lcpp/common/thread_operators.h:19-47, compare values with < / > and
 * break ties by index with ==; a NaN input has no place in that order, and
 * its result there depends on the reduction tree). */
struct NaturalOrder {
    template <typename T>
    __device__ __forceinline__ bool less(T a, T b) const { return a < b; }
    template <typename T>
    __device__ __forceinline__ bool equiv(T a, T b) const { return a == b; }
    template <typename T>
    __device__ __forceinline__ bool skip(T x) const { return x != x; }
};

/* A user comparator: equivalence is "neither compares less". */
template <typename Compare>
struct CompareOrder {
    Compare compare;
    template <typename T>
    __device__ __forceinline__ bool less(T a, T b) const { return compare(a, b); }
    template <typename T>
    __device__ __forceinline__ bool equiv(T a, T b) const { return !compare(a, b) && !compare(b, a); }
    template <typename T>
    __device__ __forceinline__ bool skip(T) const { return false; }
};

namespace arg_detail {

constexpr int kBlock = 512;
constexpr int kUnroll = 4;
constexpr int kBlocksPerSm = 2;
constexpr uint64_t kMaxBlocks = 4096;
constexpr size_t kAlign = 256;

struct Layout {
    size_t ctrl, part_v, part_i, total;
    uint64_t blocks, chunk;
};

inline Layout layout(uint64_t n, int sm_count)
{
    Layout L{};
    const uint64_t step = uint64_t(kBlock) * kUnroll;
    const uint64_t max_blocks = std::min<uint64_t>(kMaxBlocks, uint64_t(sm_count > 0 ? sm_count : 1) * kBlocksPerSm);
    L.blocks = std::max<uint64_t>(1, std::min<uint64_t>(max_blocks, (n + step - 1) / step));
    L.chunk = ((n + L.blocks - 1) / L.blocks + kBlock - 1) / kBlock * kBlock;
    L.blocks = std::max<uint64_t>(1, (n + L.chunk - 1) / L.chunk);
    L.ctrl = 0;
    L.part_v = kAlign;
    L.part_i = L.part_v + size_t(kMaxBlocks) * 8;
    L.total = L.part_i + size_t(kMaxBlocks) * 4;
    L.total = (L.total + kAlign - 1) / kAlign * kAlign;
    return L;
}

/* (bv, bi) replaces (av, ai) as the best so far. */
template <bool IS_MIN, typename Order, typename T>
__device__ __forceinline__ bool better(const Order& ord, T bv, uint32_t bi, T av, uint32_t ai)
{
    if (bi == kArgNone) return false;
    if (ai == kArgNone) return true;
    const bool strictly = IS_MIN ? ord.less(bv, av) : ord.less(av, bv);
    return strictly || (bi < ai && ord.equiv(bv, av));
}

template <bool IS_MIN, typename Order, typename T>
__device__ __forceinline__ void warp_best(const Order& ord, T& v, uint32_t& i)
{
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const T ov = __shfl_xor_sync(0xffffffffu, v, o);
        const uint32_t oi = __shfl_xor_sync(0xffffffffu, i, o);
        if (better<IS_MIN>(ord, ov, oi, v, i)) {
            v = ov;
            i = oi;
        }
    }
}

/* Result in warp 0 (every lane). */
template <bool IS_MIN, int BLOCK, typename Order, typename T>
__device__ __forceinline__ void block_best(const Order& ord, T& v, uint32_t& i, T* s_v, uint32_t* s_i)
{
    constexpr int WARPS = BLOCK / 32;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    warp_best<IS_MIN>(ord, v, i);
    if (lane == 0) {
        s_v[warp] = v;
        s_i[warp] = i;
    }
    __syncthreads();
    if (warp == 0) {
        i = lane < WARPS ? s_i[lane] : kArgNone;
        v = lane < WARPS ? s_v[lane] : v;
        warp_best<IS_MIN>(ord, v, i);
    }
}

template <typename T>
__device__ __forceinline__ T load_cg(const T* p)
{
    T v;
    if constexpr (sizeof(T) == 4) {
        const unsigned int bits = __ldcg(reinterpret_cast<const unsigned int*>(p));
        memcpy(&v, &bits, 4);
    } else {
        static_assert(sizeof(T) == 8, "ArgMin / ArgMax take 4- or 8-byte values");
        const unsigned long long bits = __ldcg(reinterpret_cast<const unsigned long long*>(p));
        memcpy(&v, &bits, 8);
    }
    return v;
}

/* One pass over the input.  ctrl[0] counts finished blocks (zeroed before
 * the launch); the last one folds the partials and writes the result.
 * VECTOR: d_in is 16-byte aligned and is read with 16-byte loads. */
template <typename T, bool IS_MIN, int BLOCK, int UNROLL, bool VECTOR, typename Order>
__global__ void __launch_bounds__(BLOCK)
arg_extremum_kernel(const T* __restrict__ in, uint64_t n, uint64_t chunk, T* part_v, uint32_t* part_i,
                    unsigned int* ctrl, T* out_v, uint32_t* out_i, T none_value, Order ord)
{
    constexpr int VEC = 16 / sizeof(T);
    __shared__ T s_v[BLOCK / 32];
    __shared__ uint32_t s_i[BLOCK / 32];
    __shared__ int s_last;
    const int tid = threadIdx.x;
    T bv[UNROLL];
    uint32_t bi[UNROLL];
#pragma unroll
    for (int u = 0; u < UNROLL; ++u) {
        bv[u] = none_value;
        bi[u] = kArgNone;
    }
    /* Each slot u sees its items in increasing index order, so a later item
     * replaces the slot's best only when strictly better. */
    auto consider = [&](int u, T x, uint64_t idx) {
        if (ord.skip(x)) return;
        if (bi[u] == kArgNone || (IS_MIN ? ord.less(x, bv[u]) : ord.less(bv[u], x))) {
            bv[u] = x;
            bi[u] = uint32_t(idx);
        }
    };
    const uint64_t lo = uint64_t(blockIdx.x) * chunk;
    const uint64_t hi = lo + chunk < n ? lo + chunk : n;
    uint64_t rest = lo;
    if constexpr (VECTOR) {
        const uint64_t nvec = hi > lo ? (hi - lo) / VEC : 0;
        const uint4* vp = reinterpret_cast<const uint4*>(in + lo);
        uint64_t j = tid;
        for (; j + uint64_t(UNROLL - 1) * BLOCK < nvec; j += uint64_t(UNROLL) * BLOCK) {
            uint4 x[UNROLL];
#pragma unroll
            for (int u = 0; u < UNROLL; ++u) x[u] = vp[j + u * BLOCK];
#pragma unroll
            for (int u = 0; u < UNROLL; ++u) {
                T t[VEC];
                memcpy(t, &x[u], 16);
#pragma unroll
                for (int e = 0; e < VEC; ++e) consider(u, t[e], lo + (j + u * BLOCK) * VEC + e);
            }
        }
        for (; j < nvec; j += BLOCK) {
            const uint4 x = vp[j];
            T t[VEC];
            memcpy(t, &x, 16);
#pragma unroll
            for (int e = 0; e < VEC; ++e) consider(0, t[e], lo + j * VEC + e);
        }
        rest = lo + nvec * VEC;
    } else {
        uint64_t i = lo + tid;
        for (; i + uint64_t(UNROLL - 1) * BLOCK < hi; i += uint64_t(UNROLL) * BLOCK) {
            T x[UNROLL];
#pragma unroll
            for (int u = 0; u < UNROLL; ++u) x[u] = in[i + u * BLOCK];
#pragma unroll
            for (int u = 0; u < UNROLL; ++u) consider(u, x[u], i + u * BLOCK);
        }
        rest = i - tid;
    }
    for (uint64_t i = rest + tid; i < hi; i += BLOCK) consider(0, in[i], i);
    T v = bv[0];
    uint32_t vi = bi[0];
#pragma unroll
    for (int u = 1; u < UNROLL; ++u)
        if (better<IS_MIN>(ord, bv[u], bi[u], v, vi)) {
            v = bv[u];
            vi = bi[u];
        }
    block_best<IS_MIN, BLOCK>(ord, v, vi, s_v, s_i);
    if (tid == 0) {
        part_v[blockIdx.x] = v;
        part_i[blockIdx.x] = vi;
        __threadfence();
        s_last = atomicAdd(ctrl, 1u) == gridDim.x - 1;
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    T f = none_value;
    uint32_t fi = kArgNone;
    for (uint32_t b = tid; b < gridDim.x; b += BLOCK) {
        const T pv = load_cg(part_v + b);
        const uint32_t pi = __ldcg(part_i + b);
        if (better<IS_MIN>(ord, pv, pi, f, fi)) {
            f = pv;
            fi = pi;
        }
    }
    __syncthreads();
    block_best<IS_MIN, BLOCK>(ord, f, fi, s_v, s_i);
    if (tid == 0) {
        *out_v = f;
        *out_i = fi;
    }
}

template <typename T>
__global__ void arg_store_kernel(T* out_v, uint32_t* out_i, T v, uint32_t i)
{
    *out_v = v;
    *out_i = i;
}

}  // namespace arg_detail

/* d_out[0] / d_index_out[0] = the extreme value under `ord` and the first
 * index holding it.  num_items == 0 writes max() (ArgMin) or lowest()
 * (ArgMax) and index 1, as the reference (device_reduce.h:552-559); input
 * with no candidate at all (every item skipped: all NaN under NaturalOrder)
 * writes the same value and index kArgNone.  Returns cudaErrorInvalidValue
 * for a bad argument, before launching anything. */
template <bool IS_MIN, typename T, typename Order>
cudaError_t arg_extremum(void* temp, size_t temp_bytes, const T* d_in, T* d_out, uint32_t* d_index_out,
                         uint64_t num_items, Order ord, cudaStream_t stream)
{
    using namespace arg_detail;
    static_assert(sizeof(T) == 4 || sizeof(T) == 8, "ArgMin / ArgMax take 4- or 8-byte values");
    const T none_value = IS_MIN ? std::numeric_limits<T>::max() : std::numeric_limits<T>::lowest();
    if (!d_out || !d_index_out || num_items > 0xffffffffull) return cudaErrorInvalidValue;
    if (num_items == 0) {
        arg_store_kernel<T><<<1, 1, 0, stream>>>(d_out, d_index_out, none_value, 1u);
        return cudaGetLastError();
    }
    int dev = 0, sms = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return e;
    const Layout L = layout(num_items, sms);
    if (!d_in || !temp || (reinterpret_cast<uintptr_t>(temp) % kAlign) || temp_bytes < L.total)
        return cudaErrorInvalidValue;
    unsigned char* t = static_cast<unsigned char*>(temp);
    e = cudaMemsetAsync(t + L.ctrl, 0, sizeof(unsigned int), stream);
    if (e != cudaSuccess) return e;
    T* pv = reinterpret_cast<T*>(t + L.part_v);
    uint32_t* pi = reinterpret_cast<uint32_t*>(t + L.part_i);
    unsigned int* ctrl = reinterpret_cast<unsigned int*>(t + L.ctrl);
    if (reinterpret_cast<uintptr_t>(d_in) % 16 == 0)
        arg_extremum_kernel<T, IS_MIN, kBlock, kUnroll, true><<<unsigned(L.blocks), kBlock, 0, stream>>>(
            d_in, num_items, L.chunk, pv, pi, ctrl, d_out, d_index_out, none_value, ord);
    else
        arg_extremum_kernel<T, IS_MIN, kBlock, kUnroll, false><<<unsigned(L.blocks), kBlock, 0, stream>>>(
            d_in, num_items, L.chunk, pv, pi, ctrl, d_out, d_index_out, none_value, ord);
    return cudaGetLastError();
}

/* The reference's comparator overloads. */
template <typename T, typename Compare>
cudaError_t ArgMin(void* temp, size_t temp_bytes, const T* d_in, T* d_out, uint32_t* d_index_out,
                   uint64_t num_items, Compare compare, cudaStream_t stream = 0)
{
    return arg_extremum<true>(temp, temp_bytes, d_in, d_out, d_index_out, num_items, CompareOrder<Compare>{compare},
                              stream);
}

template <typename T, typename Compare>
cudaError_t ArgMax(void* temp, size_t temp_bytes, const T* d_in, T* d_out, uint32_t* d_index_out,
                   uint64_t num_items, Compare compare, cudaStream_t stream = 0)
{
    return arg_extremum<false>(temp, temp_bytes, d_in, d_out, d_index_out, num_items, CompareOrder<Compare>{compare},
                               stream);
}

}  // namespace device
}  // namespace lcpp_b200

#endif /* LCPP_B200_DEVICE_CUH */
