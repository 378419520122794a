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
#include <type_traits>

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

/* A user comparator: equivalence is "neither compares less".  The parallel
 * combine (b replaces a when strictly better, or equivalent with a smaller
 * index) equals the reference's sequential fold from item 0
 * (src/lcpp/device/device_reduce.h:571-600) for every strict weak order.
 * Comparators that are not strict weak orders are outside that parity
 * domain; `<` over floating-point input holding NaN is one: NaN is then
 * "equivalent" to every value, so [5, NaN, 3] may give (NaN, 1) here where
 * the sequential fold gives (3, 2).  The comparator-free ArgMin / ArgMax
 * (NaturalOrder) skip NaN items instead. */
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


/* ---------------------------------------------------------------------------
 * Scans and reductions by key.
 *
 * DeviceScan::ExclusiveScanByKey / InclusiveScanByKey (and the ...SumByKey
 * forms; src/lcpp/device/device_scan.h:425-597) and
 * DeviceReduce::ReduceByKey (src/lcpp/device/device_reduce.h:437-491,
 * details/reduce_by_key.h).  A segment (run) is a maximal stretch of
 * consecutive items whose keys compare equal with `equal` (default ==, so
 * -0.0 and +0.0 share a run and every NaN starts one).  Per item i of a
 * segment starting at h:
 *   exclusive:       out[i] = init                          (i == h)
 *                             init op v[h] op ... op v[i-1]  (i > h)
 *   inclusive:       out[i] = v[h] op ... op v[i]
 *   inclusive init:  out[i] = init op v[h] op ... op v[i]
 *   reduce by key:   unique_out[r] = key[h_r], aggregates_out[r] = the fold of
 *                    run r, *num_runs_out = number of runs (0 for no items).
 *
 * One decoupled look-back pass scans (count, value) pairs under
 * (c1, v1) + (c2, v2) = (c1 + c2, c2 ? v2 : v1 op v2), where c counts segment
 * heads; the pair operator is associative whenever `op` is, so tiles, warps
 * and lanes combine in any grouping with left-to-right operand order.  The
 * count gives ReduceByKey each head's run index (its unique key and the
 * previous run's aggregate are written at the head; the last item writes the
 * last run and the run count).  The scans only need "some head", so their
 * look-back stops at the nearest predecessor tile that holds a head.
 * Tile = 256 threads x 4 groups x 4 consecutive items (4096 items); a lane's
 * group is one 16-byte load for 4-byte types (two for 8-byte types) when
 * keys, values and output are 16-byte aligned.  Tiles take ids from an atomic
 * counter in launch order, so a tile's predecessors are always running or
 * done; every wait is bounded by %globaltimer (4 s) and records error 5
 * (LCPP_ERR_LOOKBACK_TIMEOUT) at byte 4 of temp storage.
 * ------------------------------------------------------------------------- */

/* Bulk asynchronous copies global -> shared (cp.async.bulk, completion on an
 * mbarrier, no multicast) for the persistent kernels below. */
namespace bulk_detail {

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return uint32_t(__cvta_generic_to_shared(p)); }

/* dst, src and bytes multiples of 16 */
__device__ __forceinline__ void bulk_copy(void* dst, const void* src, uint32_t bytes, uint64_t* bar)
{
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ bool try_wait(uint64_t* bar, uint32_t parity)
{
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return done != 0;
}

__device__ __forceinline__ uint64_t now_ns()
{
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

/* Bounded wait for phase `parity` of `bar`: false after limit_ns, or as soon
 * as another thread of the call has recorded an error in *error. */
__device__ __forceinline__ bool wait(uint64_t* bar, uint32_t parity, const unsigned int* error, uint64_t limit_ns)
{
    uint64_t t0 = 0;
    uint32_t spins = 0;
    while (!try_wait(bar, parity)) {
        if (++spins == 16) {
            spins = 0;
            if (*static_cast<const volatile unsigned int*>(error)) return false;
            const uint64_t now = now_ns();
            if (t0 == 0)
                t0 = now;
            else if (now - t0 > limit_ns)
                return false;
        }
    }
    return true;
}

__device__ __forceinline__ void init_barrier(uint64_t* bar)
{
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_u32(bar)) : "memory");
}

/* thread 0 before the block's first copy, after init_barrier */
__device__ __forceinline__ void fence_barrier_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }

/* one arrival that expects `bytes` of copies on bar */
__device__ __forceinline__ void expect_bytes(uint64_t* bar, uint32_t bytes)
{
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}

/* orders this thread's (and, after a barrier, the block's) generic-proxy
 * accesses to shared memory before a later bulk copy into it */
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

}  // namespace bulk_detail

/* key equality (the reference's default `lhs == rhs`) */
struct EqualTo {
    template <typename K>
    __device__ __forceinline__ bool operator()(K a, K b) const { return a == b; }
};

namespace bykey_detail {

constexpr int kBlock = 256;
constexpr int kWarps = kBlock / 32;
constexpr int kChunks = 4;
constexpr int kGroup = 4;
constexpr uint64_t kTileItems = uint64_t(kBlock) * kChunks * kGroup;
constexpr uint64_t kWaitLimitNs = 4000000000ull;
constexpr unsigned int kErrTimeout = 5;
constexpr size_t kAlign = 256;
enum : uint32_t { kInvalid = 0, kPartial = 1, kInclusive = 2 };
enum : int { kModeExclusive = 0, kModeInclusive = 1, kModeInclusiveInit = 2, kModeReduce = 3 };

struct Ctrl {
    unsigned int tile_counter;
    unsigned int error;  // byte 4 of temp storage
};

/* A (head count, value) pair, or nothing (has == false). */
template <typename V>
struct Acc {
    uint32_t c;
    uint32_t has;
    V v;
};

template <bool COUNT, typename V, typename Op>
__device__ __forceinline__ Acc<V> seg(const Acc<V>& a, const Acc<V>& b, const Op& op)
{
    if (!a.has) return b;
    if (!b.has) return a;
    Acc<V> r;
    r.c = COUNT ? a.c + b.c : (a.c | b.c);
    r.has = 1;
    r.v = b.c ? b.v : op(a.v, b.v);
    return r;
}

template <typename V>
__device__ __forceinline__ Acc<V> shfl_acc(const Acc<V>& a, int src)
{
    return {__shfl_sync(0xffffffffu, a.c, src), __shfl_sync(0xffffffffu, a.has, src),
            __shfl_sync(0xffffffffu, a.v, src)};
}
template <typename V>
__device__ __forceinline__ Acc<V> shfl_up_acc(const Acc<V>& a, int d)
{
    return {__shfl_up_sync(0xffffffffu, a.c, d), __shfl_up_sync(0xffffffffu, a.has, d),
            __shfl_up_sync(0xffffffffu, a.v, d)};
}
template <typename V>
__device__ __forceinline__ Acc<V> shfl_down_acc(const Acc<V>& a, int d)
{
    return {__shfl_down_sync(0xffffffffu, a.c, d), __shfl_down_sync(0xffffffffu, a.has, d),
            __shfl_down_sync(0xffffffffu, a.v, d)};
}

__device__ __forceinline__ uint64_t ld_acquire_u64(const uint64_t* p)
{
    uint64_t v;
    asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_u64(uint64_t* p, uint64_t v)
{
    asm volatile("st.release.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ uint64_t global_ns()
{
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ uint64_t ld_relaxed_u64(const uint64_t* p)
{
    uint64_t v;
    asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_relaxed_u64(uint64_t* p, uint64_t v)
{
    asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

/* Consecutive tiles' status words sit one 128-byte line apart: the few
 * dozen most recent words are read by every block's look-back at once, and
 * packed into two or three lines those reads queue at one L2 slice. */
constexpr uint64_t kMetaStride = 16;

/* Tile status (tile t's word at meta[t * kMetaStride]).  Packed (4-byte
 * values, head counts below 2^30): meta =
 * (value << 32) | (head count << 2) | status, one word published and read
 * with relaxed accesses.  Otherwise meta = (head count << 32) | status,
 * released after the value it announces (partial[t] or inclusive[t]) is
 * stored, and read with acquire. */
template <typename V>
struct TileStatus {
    uint64_t* meta;
    V* partial;
    V* inclusive;
    bool packed;
    __device__ __forceinline__ void publish(uint64_t t, uint32_t status, const Acc<V>& a) const
    {
        if constexpr (sizeof(V) == 4) {
            if (packed) {
                uint32_t bits;
                memcpy(&bits, &a.v, 4);
                st_relaxed_u64(meta + t * kMetaStride, (uint64_t(bits) << 32) | (uint64_t(a.c) << 2) | status);
                return;
            }
        }
        *static_cast<volatile V*>(status == kPartial ? partial + t : inclusive + t) = a.v;
        st_release_u64(meta + t * kMetaStride, (uint64_t(a.c) << 32) | status);
    }
    /* tile t's status word (0 = not published yet) */
    __device__ __forceinline__ uint64_t word(uint64_t t) const
    {
        return packed ? ld_relaxed_u64(meta + t * kMetaStride) : ld_acquire_u64(meta + t * kMetaStride);
    }
    /* the pair a published word announces */
    __device__ __forceinline__ Acc<V> pair(uint64_t t, uint64_t m) const
    {
        Acc<V> r;
        r.has = 1;
        if constexpr (sizeof(V) == 4) {
            if (packed) {
                r.c = uint32_t(m >> 2) & 0x3fffffffu;
                const uint32_t bits = uint32_t(m >> 32);
                memcpy(&r.v, &bits, 4);
                return r;
            }
        }
        r.c = uint32_t(m >> 32);
        r.v = *static_cast<const volatile V*>((m & 3u) == kPartial ? partial + t : inclusive + t);
        return r;
    }
};

/* Exclusive prefix of `tile` (> 0), run by one whole warp: lane l inspects
 * tile base - l; the walk ends at the nearest inclusive tile (or, for the
 * scans, the nearest tile holding a head). */
template <bool COUNT, typename V, typename Op>
__device__ __forceinline__ Acc<V> look_back(uint64_t tile, const TileStatus<V>& ts, Ctrl* ctrl, const Op& op)
{
    const int lane = threadIdx.x & 31;
    Acc<V> prefix{0, 0, V{}};
    int64_t base = int64_t(tile) - 1;
    while (true) {
        const int64_t j = base - lane;
        Acc<V> val{0, 0, V{}};
        uint32_t status = kInclusive;  // lanes before tile 0 end the walk
        if (j >= 0) {
            uint64_t m;
            uint32_t spins = 0;
            uint64_t t0 = 0;
            bool gave_up = false;
            while (((m = ts.word(uint64_t(j))) & 3u) == kInvalid) {
                if (++spins == 64) {
                    spins = 0;
                    const uint64_t now = global_ns();
                    if (t0 == 0) {
                        t0 = now;
                    } else if (now - t0 > kWaitLimitNs || *static_cast<volatile unsigned int*>(&ctrl->error)) {
                        atomicCAS(&ctrl->error, 0u, kErrTimeout);
                        gave_up = true;  // stop here, contributing nothing
                        break;
                    }
                }
            }
            if (!gave_up) {
                status = uint32_t(m & 3u);
                val = ts.pair(uint64_t(j), m);
            }
        }
        const bool stop = status == kInclusive || (!COUNT && val.has && val.c != 0);
        const uint32_t mask = __ballot_sync(0xffffffffu, stop);
        const int last = mask ? __ffs(mask) - 1 : 31;
        Acc<V> x = lane <= last ? val : Acc<V>{0, 0, V{}};
        /* ordered fold of lanes 0..last: farther tiles (higher lanes) first */
#pragma unroll
        for (int d = 1; d < 32; d <<= 1) {
            const Acc<V> y = shfl_down_acc(x, d);
            if (lane + d < 32) x = seg<COUNT>(y, x, op);
        }
        prefix = seg<COUNT>(shfl_acc(x, 0), prefix, op);
        if (mask) return prefix;
        base -= 32;
    }
}

template <typename T>
__device__ __forceinline__ void load_group(const T* p, uint64_t n, uint64_t g, bool vector, T (&x)[kGroup])
{
    if (vector && g + kGroup <= n) {
        constexpr int W = int(sizeof(T)) * kGroup / 16;
        const uint4* q = reinterpret_cast<const uint4*>(p + g);
        uint4 w[W];
#pragma unroll
        for (int i = 0; i < W; ++i) w[i] = q[i];
        memcpy(x, w, sizeof(x));
    } else {
#pragma unroll
        for (int e = 0; e < kGroup; ++e) x[e] = g + e < n ? p[g + e] : T{};
    }
}

template <typename T>
__device__ __forceinline__ void store_group(T* p, uint64_t n, uint64_t g, bool vector, const T (&x)[kGroup])
{
    if (vector && g + kGroup <= n) {
        constexpr int W = int(sizeof(T)) * kGroup / 16;
        uint4 w[W];
        memcpy(w, x, sizeof(x));
        uint4* q = reinterpret_cast<uint4*>(p + g);
#pragma unroll
        for (int i = 0; i < W; ++i) q[i] = w[i];
    } else {
#pragma unroll
        for (int e = 0; e < kGroup; ++e)
            if (g + e < n) p[g + e] = x[e];
    }
}

/* Head flags of a thread's items (bit j * kGroup + e); padding past n is a
 * head of its own.  `before` is the key preceding the warp's first item
 * (ignored for item 0). */
template <typename K, typename Equal>
__device__ __forceinline__ uint32_t head_bits(const K (&k)[kChunks][kGroup], K before, uint64_t n,
                                              uint64_t warp_base, int lane, const Equal& equal)
{
    uint32_t heads = 0;
#pragma unroll
    for (int j = 0; j < kChunks; ++j) {
        const K prev_lane = __shfl_up_sync(0xffffffffu, k[j][kGroup - 1], 1);
        const K prev_chunk = __shfl_sync(0xffffffffu, k[j > 0 ? j - 1 : 0][kGroup - 1], 31);
        const uint64_t g = warp_base + uint64_t(j * 32 + lane) * kGroup;
#pragma unroll
        for (int e = 0; e < kGroup; ++e) {
            const uint64_t i = g + e;
            bool h;
            if (i >= n)
                h = true;
            else if (e > 0)
                h = !equal(k[j][e - 1], k[j][e]);
            else if (lane > 0)
                h = !equal(prev_lane, k[j][0]);
            else if (j > 0)
                h = !equal(prev_chunk, k[j][0]);
            else
                h = i == 0 || !equal(before, k[j][0]);
            heads |= uint32_t(h) << (j * kGroup + e);
        }
    }
    return heads;
}

/* Per-lane group folds, then warp scans chunk by chunk: pre[j] = the
 * exclusive prefix of chunk j's group within the warp; returns the warp's
 * total (every lane). */
template <bool COUNT, typename V, typename Op>
__device__ __forceinline__ Acc<V> group_scans(const V (&v)[kChunks][kGroup], uint32_t heads, int lane,
                                              Acc<V> (&pre)[kChunks], const Op& op)
{
    Acc<V> carry{0, 0, V{}};
#pragma unroll
    for (int j = 0; j < kChunks; ++j) {
        Acc<V> x{(heads >> (j * kGroup)) & 1u, 1, v[j][0]};
#pragma unroll
        for (int e = 1; e < kGroup; ++e) {
            if ((heads >> (j * kGroup + e)) & 1u) {
                x.c = COUNT ? x.c + 1 : 1;
                x.v = v[j][e];
            } else {
                x.v = op(x.v, v[j][e]);
            }
        }
#pragma unroll
        for (int d = 1; d < 32; d <<= 1) {
            const Acc<V> y = shfl_up_acc(x, d);
            if (lane >= d) x = seg<COUNT>(y, x, op);
        }
        Acc<V> ex = shfl_up_acc(x, 1);
        if (lane == 0) ex = Acc<V>{0, 0, V{}};
        pre[j] = seg<COUNT>(carry, ex, op);
        carry = seg<COUNT>(carry, shfl_acc(x, 31), op);
    }
    return carry;
}

/* Warp 0: the tile's warp totals folded in order; excl[w] = the prefix of
 * warp w within the tile; returns the tile's aggregate (every lane). */
template <bool COUNT, int WARPS, typename V, typename Op>
__device__ __forceinline__ Acc<V> block_fold(const Acc<V>* total, Acc<V>* excl, int lane, const Op& op)
{
    Acc<V> x = lane < WARPS ? total[lane] : Acc<V>{0, 0, V{}};
#pragma unroll
    for (int d = 1; d < WARPS; d <<= 1) {
        const Acc<V> y = shfl_up_acc(x, d);
        if (lane >= d) x = seg<COUNT>(y, x, op);
    }
    Acc<V> ex = shfl_up_acc(x, 1);
    if (lane == 0) ex = Acc<V>{0, 0, V{}};
    if (lane < WARPS) excl[lane] = ex;
    return shfl_acc(x, WARPS - 1);
}

/* Outputs of a thread's items once the exclusive prefix of its warp is
 * known.  mode: kModeExclusive / kModeInclusive / kModeInclusiveInit write
 * out[]; kModeReduce (COUNT only; k holds the keys) writes unique_out[],
 * out[] (= the aggregates) and *num_runs. */
template <bool COUNT, int KC, typename K, typename V, typename Op>
__device__ __forceinline__ void emit(const K (&k)[KC][kGroup], const V (&v)[kChunks][kGroup], uint32_t heads,
                                     const Acc<V> (&pre)[kChunks], const Acc<V>& warp_prefix, uint64_t warp_base,
                                     int lane, uint64_t n, int mode, V init, V* out, K* unique_out,
                                     uint32_t* num_runs, bool vector, const Op& op)
{
#pragma unroll
    for (int j = 0; j < kChunks; ++j) {
        const uint64_t g = warp_base + uint64_t(j * 32 + lane) * kGroup;
        Acc<V> E = seg<COUNT>(warp_prefix, pre[j], op);
        V o[kGroup];
#pragma unroll
        for (int e = 0; e < kGroup; ++e) {
            const uint64_t i = g + e;
            const bool h = (heads >> (j * kGroup + e)) & 1u;
            Acc<V> P;
            P.has = 1;
            if (h || !E.has) {
                P.c = COUNT ? (E.has ? E.c : 0u) + uint32_t(h) : uint32_t(h);
                P.v = v[j][e];
            } else {
                P.c = E.c;
                P.v = op(E.v, v[j][e]);
            }
            if (mode == kModeExclusive) {
                o[e] = h ? init : op(init, E.v);
            } else if (mode == kModeInclusive) {
                o[e] = P.v;
            } else if (mode == kModeInclusiveInit) {
                o[e] = op(init, P.v);
            } else if constexpr (COUNT) {
                if (i < n) {
                    if (h) {
                        const uint32_t r = P.c - 1;
                        unique_out[r] = k[j][e];
                        if (r > 0) out[r - 1] = E.v;
                    }
                    if (i == n - 1) {
                        out[P.c - 1] = P.v;
                        *num_runs = P.c;
                    }
                }
            }
            E = P;
        }
        if (mode != kModeReduce) store_group(out, n, g, vector, o);
    }
}

/* One tile per block (any alignment). */
template <typename K, typename V, bool COUNT, typename Equal, typename Op>
__global__ void __launch_bounds__(kBlock, (sizeof(K) + sizeof(V) <= 8) ? 3 : 2)
by_key_kernel(const K* keys, const V* values, V* out, K* unique_out, uint32_t* num_runs, uint64_t n, int mode,
              V init, bool vector, Ctrl* ctrl, TileStatus<V> ts, Equal equal, Op op)
{
    __shared__ uint32_t s_tile;
    __shared__ Acc<V> s_total[kWarps];
    __shared__ Acc<V> s_excl[kWarps];
    __shared__ Acc<V> s_prefix;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (threadIdx.x == 0) s_tile = atomicAdd(&ctrl->tile_counter, 1u);
    __syncthreads();
    const uint64_t tile = s_tile;
    const uint64_t warp_base = tile * kTileItems + uint64_t(warp) * (32 * kChunks * kGroup);

    K k[kChunks][kGroup];
    V v[kChunks][kGroup];
#pragma unroll
    for (int j = 0; j < kChunks; ++j) {
        const uint64_t g = warp_base + uint64_t(j * 32 + lane) * kGroup;
        load_group(keys, n, g, vector, k[j]);
        load_group(values, n, g, vector, v[j]);
    }
    const K before = lane == 0 && warp_base > 0 && warp_base < n ? keys[warp_base - 1] : K{};
    const uint32_t heads = head_bits(k, before, n, warp_base, lane, equal);
    Acc<V> pre[kChunks];
    const Acc<V> carry = group_scans<COUNT>(v, heads, lane, pre, op);
    if (lane == 0) s_total[warp] = carry;
    __syncthreads();

    if (warp == 0) {
        const Acc<V> aggregate = block_fold<COUNT, kWarps>(s_total, s_excl, lane, op);
        Acc<V> prefix{0, 0, V{}};
        if (tile == 0) {
            if (lane == 0) ts.publish(0, kInclusive, aggregate);
        } else {
            if (lane == 0) ts.publish(tile, kPartial, aggregate);
            prefix = look_back<COUNT>(tile, ts, ctrl, op);
            if (lane == 0) ts.publish(tile, kInclusive, seg<COUNT>(prefix, aggregate, op));
        }
        if (lane == 0) s_prefix = prefix;
    }
    __syncthreads();
    emit<COUNT>(k, v, heads, pre, seg<COUNT>(s_prefix, s_excl[warp], op), warp_base, lane, n, mode, init, out,
                unique_out, num_runs, vector, op);
}

/* ---- Persistent variant for 16-byte aligned keys and values ---------------
 * Like the compaction's: tiles are taken from the atomic counter and their
 * keys and values bulk-copied into a three-stage shared-memory ring.  Eight
 * data warps and one look-back warp; per iteration, concurrently:
 *   data warps -- A(k+1): heads and warp scans of tile k+1 from its stage
 *           (heads and per-chunk prefixes stay in registers), its partial
 *           published;
 *   look-back warp -- the look-back of tile k, its inclusive published;
 * then, with tile k's prefix known, the data warps re-read tile k's values
 * (and keys) from its stage, write its outputs, and the stage is refilled
 * with the block's next tile.  The two register sets alternate. */
template <int BLOCK>
struct KeyShape {
    static constexpr int kBlock = BLOCK;  // data threads; one more warp runs the look-backs
    static constexpr int kWarps = BLOCK / 32;
    static constexpr int kThreads = BLOCK + 32;
    static constexpr uint64_t kTile = uint64_t(BLOCK) * kChunks * kGroup;
};
/* ReduceByKey's look-back walks to an inclusive tile past every tile in
 * flight (about one round trip per 32 of them), so its throughput grows
 * with the tile: 8192 items (16 data warps) when a key and a value take at
 * most 8 bytes (192 KB of stages); the scans stop at the first predecessor
 * holding a head and keep 4096-item tiles (two blocks per SM). */
template <bool COUNT, typename K, typename V>
using KeyBulkOf = KeyShape<(COUNT && sizeof(K) + sizeof(V) <= 8) ? 512 : 256>;
constexpr int kBulkStages = 3;
constexpr int kIdSlots = 4;  // tile ids of tiles k .. k+3 (k+3: acquired at the end of iteration k)

template <typename K, typename V, bool COUNT>
constexpr size_t bulk_smem_bytes()
{
    return size_t(kBulkStages) * KeyBulkOf<COUNT, K, V>::kTile * (sizeof(K) + sizeof(V));
}

/* What A(k) leaves in registers for the output phase of tile k. */
template <typename V>
struct TileRegs {
    uint64_t tile;
    uint32_t heads;
    Acc<V> pre[kChunks];
};

template <typename K, typename V, bool COUNT, typename Equal, typename Op>
__global__ void __launch_bounds__(KeyBulkOf<COUNT, K, V>::kThreads, (!COUNT && sizeof(K) + sizeof(V) <= 8) ? 2 : 1)
by_key_bulk_kernel(const K* keys, const V* values, V* out, K* unique_out, uint32_t* num_runs, uint64_t n, int mode,
                   V init, bool vector, uint64_t tiles, Ctrl* ctrl, TileStatus<V> ts, Equal equal, Op op)
{
    using S = KeyBulkOf<COUNT, K, V>;
    constexpr uint32_t kKeyBytes = uint32_t(S::kTile * sizeof(K));
    constexpr uint32_t kValueBytes = uint32_t(S::kTile * sizeof(V));
    extern __shared__ __align__(128) unsigned char bulk_smem[];
    K* sk = reinterpret_cast<K*>(bulk_smem);                                     // [stage][tile]
    V* sv = reinterpret_cast<V*>(bulk_smem + size_t(kBulkStages) * kKeyBytes);  // [stage][tile]
    __shared__ __align__(8) uint64_t s_bar[kBulkStages];
    __shared__ uint64_t s_id[kIdSlots];  // tile id of the block's i-th tile at i % kIdSlots
    __shared__ uint32_t s_pending;       // bit s: a copy into stage s is in flight
    __shared__ uint32_t s_phase;         // bit s: parity of the next completion of stage s
    __shared__ Acc<V> s_total[kBulkStages][S::kWarps];
    __shared__ Acc<V> s_excl[kBulkStages][S::kWarps];
    __shared__ Acc<V> s_agg[kBulkStages];
    __shared__ Acc<V> s_prefix[kBulkStages];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const bool data = warp < S::kWarps;
    const int toff = warp * (32 * kChunks * kGroup);  // the warp's first item in the tile
    auto data_sync = [] { asm volatile("bar.sync 1, %0;" ::"n"(S::kBlock) : "memory"); };

    // the block's i-th tile: its id, and its copy into stage i % 3 when full (thread 0)
    auto acquire = [&](uint32_t i) {
        const int s = int(i % kBulkStages);
        if (*static_cast<volatile unsigned int*>(&ctrl->error)) {
            s_id[i % kIdSlots] = tiles;
            return;
        }
        const uint64_t t = atomicAdd(&ctrl->tile_counter, 1u);
        s_id[i % kIdSlots] = t;
        if (t < tiles && (t + 1) * S::kTile <= n) {
            s_pending |= 1u << s;
            bulk_detail::expect_bytes(&s_bar[s], kKeyBytes + kValueBytes);
            bulk_detail::bulk_copy(sk + size_t(s) * S::kTile, keys + t * S::kTile, kKeyBytes, &s_bar[s]);
            bulk_detail::bulk_copy(sv + size_t(s) * S::kTile, values + t * S::kTile, kValueBytes, &s_bar[s]);
        }
    };
    // this thread's keys and values of the block's i-th tile
    auto load = [&](uint32_t i, uint64_t tile, bool wait, K (&k)[kChunks][kGroup], V (&v)[kChunks][kGroup],
                    bool want_keys) {
        const int s = int(i % kBulkStages);
        const uint64_t warp_base = tile * S::kTile + uint64_t(toff);
        if ((tile + 1) * S::kTile <= n) {
            if (wait && !bulk_detail::wait(&s_bar[s], (s_phase >> s) & 1u, &ctrl->error, kWaitLimitNs))
                atomicCAS(&ctrl->error, 0u, kErrTimeout);
#pragma unroll
            for (int j = 0; j < kChunks; ++j) {
                const int at = toff + (j * 32 + lane) * kGroup;
                if (want_keys) memcpy(k[j], sk + size_t(s) * S::kTile + at, sizeof(k[j]));
                memcpy(v[j], sv + size_t(s) * S::kTile + at, sizeof(v[j]));
            }
        } else {
#pragma unroll
            for (int j = 0; j < kChunks; ++j) {
                const uint64_t g = warp_base + uint64_t(j * 32 + lane) * kGroup;
                if (want_keys) load_group(keys, n, g, false, k[j]);
                load_group(values, n, g, false, v[j]);
            }
        }
    };
    // A(i): heads and warp scans of the block's i-th tile into r, its warp totals into s_total
    auto phase_a = [&](uint32_t i, TileRegs<V>& r) {
        const int s = int(i % kBulkStages);
        const uint64_t tile = s_id[i % kIdSlots];
        const uint64_t warp_base = tile * S::kTile + uint64_t(toff);
        K k[kChunks][kGroup];
        V v[kChunks][kGroup];
        load(i, tile, true, k, v, true);
        K before{};
        if (lane == 0 && warp_base > 0 && warp_base < n) {
            const bool staged = (tile + 1) * S::kTile <= n && toff > 0;
            before = staged ? sk[size_t(s) * S::kTile + toff - 1] : keys[warp_base - 1];
        }
        r.tile = tile;
        r.heads = head_bits(k, before, n, warp_base, lane, equal);
        const Acc<V> carry = group_scans<COUNT>(v, r.heads, lane, r.pre, op);
        if (lane == 0) s_total[s][warp] = carry;
    };
    // after A(i) and a barrier of the data warps: warp 0 folds the warp
    // totals and publishes the tile's partial, thread 0 retires its copy
    auto after_a = [&](uint32_t i) {
        const int s = int(i % kBulkStages);
        if (warp != 0) return;
        const uint64_t tile = s_id[i % kIdSlots];
        const Acc<V> aggregate = block_fold<COUNT, S::kWarps>(s_total[s], s_excl[s], lane, op);
        if (lane == 0) {
            s_agg[s] = aggregate;
            ts.publish(tile, tile == 0 ? kInclusive : kPartial, aggregate);
            if (((s_pending >> s) & 1u) && !*static_cast<volatile unsigned int*>(&ctrl->error)) {
                s_phase ^= 1u << s;
                s_pending &= ~(1u << s);
            }
        }
    };
    // the look-back warp: tile i's exclusive prefix, its inclusive published
    auto look = [&](uint32_t i) {
        const int s = int(i % kBulkStages);
        const uint64_t tile = s_id[i % kIdSlots];
        Acc<V> prefix{0, 0, V{}};
        if (tile > 0) {
            prefix = look_back<COUNT>(tile, ts, ctrl, op);
            if (lane == 0) ts.publish(tile, kInclusive, seg<COUNT>(prefix, s_agg[s], op));
        }
        if (lane == 0) s_prefix[s] = prefix;
    };
    // Hand-offs between the data warps and the look-back warp (named
    // barriers over the whole block: one side arrives, the other waits).
    // Barrier 3, "aggregate ready": tile i+1's aggregate is published and
    // tile i's prefix has been consumed; barrier 2, "prefix ready".  Each
    // side arrives once per tile and only after the other side's previous
    // arrival was consumed, so no barrier ever sees two arrivals of a side.
    auto agg_ready_signal = [] { asm volatile("bar.arrive 3, %0;" ::"n"(S::kThreads) : "memory"); };
    auto agg_ready_wait = [] { asm volatile("bar.sync 3, %0;" ::"n"(S::kThreads) : "memory"); };
    auto prefix_ready_signal = [] { asm volatile("bar.arrive 2, %0;" ::"n"(S::kThreads) : "memory"); };
    auto prefix_ready_wait = [] { asm volatile("bar.sync 2, %0;" ::"n"(S::kThreads) : "memory"); };
    // data warps, one iteration: A(i + 1) into nxt, then, once tile i's
    // prefix is known, tile i's outputs from cur and its stage, and the
    // stage refilled; false after the block's last tile
    auto step = [&](uint32_t i, const TileRegs<V>& cur, TileRegs<V>& nxt) -> bool {
        const bool has_next = s_id[(i + 1) % kIdSlots] < tiles;
        if (has_next) {
            phase_a(i + 1, nxt);
            data_sync();
            after_a(i + 1);
        }
        prefix_ready_wait();  // tile i's prefix
        if (has_next) agg_ready_signal();
        const int s = int(i % kBulkStages);
        K k[kChunks][kGroup];
        V v[kChunks][kGroup];
        load(i, cur.tile, false, k, v, COUNT);
        emit<COUNT>(k, v, cur.heads, cur.pre, seg<COUNT>(s_prefix[s], s_excl[s][warp], op),
                    cur.tile * S::kTile + uint64_t(toff), lane, n, mode, init, out, unique_out, num_runs, vector,
                    op);
        data_sync();  // stage i % 3 is free
        if (tid == 0) {
            bulk_detail::fence_proxy_async();
            acquire(i + kBulkStages);
        }
        return has_next;
    };

    if (tid == 0) {
        s_pending = 0;
        s_phase = 0;
        for (int s = 0; s < kBulkStages; ++s) bulk_detail::init_barrier(&s_bar[s]);
        bulk_detail::fence_barrier_init();
        for (uint32_t i = 0; i < uint32_t(kBulkStages); ++i) acquire(i);
    }
    __syncthreads();
    if (s_id[0] < tiles) {
        if (data) {
            TileRegs<V> ra, rb;
            phase_a(0, ra);
            data_sync();
            after_a(0);
            agg_ready_signal();
            for (uint32_t i = 0;; i += 2) {
                if (!step(i, ra, rb)) break;
                if (!step(i + 1, rb, ra)) break;
            }
        } else {
            // the look-back warp: one tile after the other, as their aggregates appear
            for (uint32_t i = 0;; ++i) {
                agg_ready_wait();
                look(i);
                prefix_ready_signal();
                if (s_id[(i + 1) % kIdSlots] >= tiles) break;
            }
        }
    }
    __syncthreads();
    // copies not retired (only after an error): wait for them, bounded,
    // before the block's shared memory goes away
    if (tid == 0 && s_pending) {
        for (int s = 0; s < kBulkStages; ++s)
            if ((s_pending >> s) & 1u)
                if (!bulk_detail::wait(&s_bar[s], (s_phase >> s) & 1u, &ctrl->error, kWaitLimitNs))
                    atomicCAS(&ctrl->error, 0u, kErrTimeout);
    }
}

struct Layout {
    size_t ctrl, meta, partial, inclusive, total;
    uint64_t tiles;
};

inline Layout layout(uint64_t n, size_t value_bytes)
{
    Layout L{};
    L.tiles = n ? (n + kTileItems - 1) / kTileItems : 0;
    auto up = [](size_t x) { return (x + kAlign - 1) / kAlign * kAlign; };
    L.ctrl = 0;
    L.meta = kAlign;
    L.partial = up(L.meta + size_t(L.tiles) * 8 * kMetaStride);
    L.inclusive = up(L.partial + size_t(L.tiles) * value_bytes);
    L.total = up(L.inclusive + size_t(L.tiles) * value_bytes);
    return L;
}

inline bool aligned16(const void* p) { return reinterpret_cast<uintptr_t>(p) % 16 == 0; }

template <bool COUNT, typename K, typename V, typename Equal, typename Op>
cudaError_t launch(void* temp, size_t temp_bytes, const K* keys, const V* values, V* out, K* unique_out,
                   uint32_t* num_runs, uint64_t n, int mode, V init, Equal equal, Op op, cudaStream_t stream)
{
    const Layout L = layout(n, sizeof(V));
    if (!keys || !values || !out || !temp || reinterpret_cast<uintptr_t>(temp) % kAlign || temp_bytes < L.total)
        return cudaErrorInvalidValue;
    if (L.tiles > 0xffffffffull) return cudaErrorInvalidValue;
    unsigned char* t = static_cast<unsigned char*>(temp);
    cudaError_t e = cudaMemsetAsync(t, 0, L.meta + size_t(L.tiles) * 8 * kMetaStride, stream);
    if (e != cudaSuccess) return e;
    // head counts stay below 2^30 for the scans (0 or 1) and below n for ReduceByKey
    const bool packed = sizeof(V) == 4 && (!COUNT || n < (uint64_t(1) << 30));
    TileStatus<V> ts{reinterpret_cast<uint64_t*>(t + L.meta), reinterpret_cast<V*>(t + L.partial),
                     reinterpret_cast<V*>(t + L.inclusive), packed};
    Ctrl* ctrl = reinterpret_cast<Ctrl*>(t);
    const bool vector = aligned16(keys) && aligned16(values) && (mode == kModeReduce || aligned16(out));
    if (aligned16(keys) && aligned16(values)) {
        // the persistent bulk-copy kernel, as many blocks as are resident
        using S = KeyBulkOf<COUNT, K, V>;
        auto kernel = by_key_bulk_kernel<K, V, COUNT, Equal, Op>;
        constexpr size_t smem = bulk_smem_bytes<K, V, COUNT>();
        int dev = 0, sms = 0, per_sm = 0;
        e = cudaGetDevice(&dev);
        if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        if (e == cudaSuccess) e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
        if (e == cudaSuccess) e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, S::kThreads, smem);
        if (e != cudaSuccess) return e;
        const uint64_t tiles = (n + S::kTile - 1) / S::kTile;  // <= L.tiles status rows
        const uint64_t resident = uint64_t(sms > 0 ? sms : 1) * uint64_t(per_sm > 0 ? per_sm : 1);
        kernel<<<unsigned(std::min(tiles, resident)), S::kThreads, smem, stream>>>(
            keys, values, out, unique_out, num_runs, n, mode, init, vector, tiles, ctrl, ts, equal, op);
    } else {
        by_key_kernel<K, V, COUNT><<<unsigned(L.tiles), kBlock, 0, stream>>>(
            keys, values, out, unique_out, num_runs, n, mode, init, vector, ctrl, ts, equal, op);
    }
    return cudaGetLastError();
}

}  // namespace bykey_detail

/* Temp storage bytes of the by-key scans and ReduceByKey (any key type). */
inline size_t by_key_temp_bytes(uint64_t num_items, size_t value_bytes)
{
    return num_items ? bykey_detail::layout(num_items, value_bytes).total : 0;
}

/* mode: 0 exclusive (init), 1 inclusive, 2 inclusive with init.  Values may
 * be scanned in place (d_values_out == d_values_in).  No items: nothing. */
template <typename K, typename V, typename Op, typename Equal = EqualTo>
cudaError_t scan_by_key(void* temp, size_t temp_bytes, const K* d_keys_in, const V* d_values_in, V* d_values_out,
                        uint64_t num_items, int mode, V init, Op op, Equal equal = Equal{}, cudaStream_t stream = 0)
{
    static_assert(sizeof(K) == 4 || sizeof(K) == 8, "keys: 4- or 8-byte types");
    static_assert(sizeof(V) == 4 || sizeof(V) == 8, "values: 4- or 8-byte types");
    if (mode < 0 || mode > 2) return cudaErrorInvalidValue;
    if (num_items == 0) return cudaSuccess;
    return bykey_detail::launch<false>(temp, temp_bytes, d_keys_in, d_values_in, d_values_out,
                                       static_cast<K*>(nullptr), nullptr, num_items, mode, init, equal, op, stream);
}

/* ReduceByKey; num_items < 2^32 (the run count is a uint32, as the
 * reference's); d_unique_out must not overlap d_keys_in.  No items: writes
 * *d_num_runs_out = 0. */
template <typename K, typename V, typename Op, typename Equal = EqualTo>
cudaError_t reduce_by_key(void* temp, size_t temp_bytes, const K* d_keys_in, const V* d_values_in, K* d_unique_out,
                          V* d_aggregates_out, uint32_t* d_num_runs_out, uint64_t num_items, Op op,
                          Equal equal = Equal{}, cudaStream_t stream = 0)
{
    static_assert(sizeof(K) == 4 || sizeof(K) == 8, "keys: 4- or 8-byte types");
    static_assert(sizeof(V) == 4 || sizeof(V) == 8, "values: 4- or 8-byte types");
    if (!d_num_runs_out || num_items > 0xffffffffull) return cudaErrorInvalidValue;
    if (num_items == 0) return cudaMemsetAsync(d_num_runs_out, 0, sizeof(uint32_t), stream);
    if (!d_unique_out || static_cast<const void*>(d_unique_out) == static_cast<const void*>(d_keys_in))
        return cudaErrorInvalidValue;
    return bykey_detail::launch<true>(temp, temp_bytes, d_keys_in, d_values_in, d_aggregates_out, d_unique_out,
                                      d_num_runs_out, num_items, bykey_detail::kModeReduce, V{}, equal, op, stream);
}

/* ---------------------------------------------------------------------------
 * Compaction: DeviceSelect::Flagged / If / FlaggedIf / Unique / UniqueByKey
 * (src/lcpp/device/device_select.h:56-345) and DevicePartition::Flagged / If
 * and the three-way If (src/lcpp/device/device_partition.h:55-227).
 *
 * Selection per item: Flagged -- flag != 0 at the flag's type (bool flags are
 * 1-byte); If -- select(item); FlaggedIf -- select(flag); Unique /
 * UniqueByKey -- item 0 and every item whose key differs from its
 * predecessor's (`equal`, default ==).  Select writes the selected items in
 * input order and the count; Partition writes the selected items in order
 * from the front and the rejected ones in REVERSE order from the back
 * (output[n - 1 - rejected_before], device_partition.h:531-575); the
 * three-way form writes items with select_first to first_out, the remaining
 * ones with select_second to second_out (both in order) and the rest in
 * reverse order into unselected_out (device_partition.h:582-660), and the two
 * counts.  Select may run in place (d_out == d_in; Unique too): an item only
 * ever moves to a lower index, and a tile writes only after its look-back,
 * i.e. after every lower tile has loaded its items.
 *
 * One pass: tiles of 512 threads x 4 groups x 4 consecutive items (8192
 * items), tile ids from an atomic counter; the per-group selected counts are
 * scanned across lanes, warps and (decoupled look-back, every wait bounded
 * by %globaltimer at 4 s, error 5 at byte 4 of temp) tiles; each selected
 * item is stored at its rank.  The tile status word is
 * (count << 32) | status; the three-way form keeps its second count in two
 * more arrays (partial, inclusive) written before the word is released, and
 * learns both totals from a counting pass first (its unselected output is
 * placed from the end of a region whose size is n minus both totals).
 * ------------------------------------------------------------------------- */

/* "no values" for the value arrays of the keys-only forms */
struct NoValue {};

/* flag != 0 at the flag's type */
struct NonZero {
    template <typename F>
    __device__ __forceinline__ bool operator()(F f) const { return f != F(0); }
};

namespace select_detail {

constexpr int kBlock = 512;  // 8192-item tiles: fewer look-back windows per item
constexpr int kWarps = kBlock / 32;
constexpr int kChunks = 4;
constexpr int kGroup = 4;
constexpr uint64_t kTileItems = uint64_t(kBlock) * kChunks * kGroup;
constexpr uint64_t kWaitLimitNs = 4000000000ull;
constexpr unsigned int kErrTimeout = 5;
constexpr size_t kAlign = 256;
enum : uint32_t { kInvalid = 0, kPartial = 1, kInclusive = 2 };
enum : int { kSelFlag = 0, kSelIf = 1, kSelUnique = 2 };
enum : int { kOutSelect = 0, kOutPartition = 1, kOutThreeWay = 2, kOutRanks = 3 };

struct Ctrl {
    unsigned int tile_counter;
    unsigned int error;      // byte 4 of temp storage
    unsigned int totals[2];  // three-way: both selected counts (counting pass)
};

__device__ __forceinline__ uint64_t ld_relaxed_u64(const uint64_t* p)
{
    uint64_t v;
    asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_relaxed_u64(uint64_t* p, uint64_t v)
{
    asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ void st_release_u64(uint64_t* p, uint64_t v)
{
    asm volatile("st.release.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ uint64_t global_ns()
{
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

/* 4 consecutive items at g: one 4-, 16- or two 16-byte loads when vector */
template <typename T>
__device__ __forceinline__ void load4(const T* p, uint64_t n, uint64_t g, bool vector, T (&x)[kGroup])
{
    if (vector && g + kGroup <= n) {
        if constexpr (sizeof(T) == 1) {
            const uint32_t w = *reinterpret_cast<const uint32_t*>(p + g);
            memcpy(x, &w, 4);
        } else {
            constexpr int W = int(sizeof(T)) * kGroup / 16;
            const uint4* q = reinterpret_cast<const uint4*>(p + g);
            uint4 w[W];
#pragma unroll
            for (int i = 0; i < W; ++i) w[i] = q[i];
            memcpy(x, w, sizeof(x));
        }
    } else {
#pragma unroll
        for (int e = 0; e < kGroup; ++e) x[e] = g + e < n ? p[g + e] : T{};
    }
}

/* Counts of one range: selected (first) in the low half, second-selected in
 * the high half.  Both stay below 2^32, so packed sums never carry. */
__device__ __forceinline__ uint64_t warp_sum(uint64_t v)
{
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

/* Consecutive tiles' status words sit one 128-byte line apart: the few
 * dozen most recent words are read by every block's look-back at once, and
 * packed into two or three lines those reads queue at one L2 slice. */
constexpr uint64_t kStatusStride = 16;

template <bool THREE>
struct Status {
    uint64_t* word;       // (first count << 32) | status, tile t at word[t * kStatusStride]
    uint32_t* second_p;   // three-way: second count of the partial
    uint32_t* second_i;   // three-way: second count of the inclusive prefix
    // The word carries the first count, so a relaxed store publishes it; the
    // three-way form's second count is stored first and released by the word.
    __device__ __forceinline__ void publish(uint64_t t, uint32_t status, uint64_t packed) const
    {
        const uint64_t w = (uint64_t(uint32_t(packed)) << 32) | status;
        if constexpr (THREE) {
            *static_cast<volatile uint32_t*>((status == kPartial ? second_p : second_i) + t) = uint32_t(packed >> 32);
            st_release_u64(word + t * kStatusStride, w);
        } else {
            st_relaxed_u64(word + t * kStatusStride, w);
        }
    }
};

/* Exclusive packed count of `tile` (> 0), run by one whole warp: lane l
 * inspects tile base - l, so one round trip covers 32 predecessors; the walk
 * ends at the nearest inclusive tile.  Status words are read relaxed: the
 * first count travels in the word itself, and the three-way form's second
 * count is read after an acquire fence.  Every wait is bounded; on timeout
 * the error is recorded and the walk stops. */
template <bool THREE>
__device__ __forceinline__ uint64_t look_back(uint64_t tile, const Status<THREE>& st, Ctrl* ctrl)
{
    const int lane = threadIdx.x & 31;
    uint64_t prefix = 0;
    int64_t base = int64_t(tile) - 1;
    while (true) {
        const int64_t j = base - lane;
        uint64_t val = 0;
        uint32_t status = kInclusive;  // lanes before tile 0 end the walk
        if (j >= 0) {
            uint64_t m;
            uint32_t spins = 0;
            uint64_t t0 = 0;
            bool gave_up = false;
            while (((m = ld_relaxed_u64(st.word + uint64_t(j) * kStatusStride)) & 3u) == kInvalid) {
                if (++spins == 64) {
                    spins = 0;
                    const uint64_t now = global_ns();
                    if (t0 == 0) {
                        t0 = now;
                    } else if (now - t0 > kWaitLimitNs || *static_cast<volatile unsigned int*>(&ctrl->error)) {
                        atomicCAS(&ctrl->error, 0u, kErrTimeout);
                        gave_up = true;  // stop here, contributing nothing
                        break;
                    }
                }
            }
            if (!gave_up) {
                status = uint32_t(m & 3u);
                val = m >> 32;
                if constexpr (THREE) {
                    asm volatile("fence.acq_rel.gpu;" ::: "memory");
                    val |= uint64_t(*static_cast<const volatile uint32_t*>(
                               (status == kPartial ? st.second_p : st.second_i) + j))
                           << 32;
                }
            }
        }
        const uint32_t mask = __ballot_sync(0xffffffffu, status == kInclusive);
        const int last = mask ? __ffs(mask) - 1 : 31;
        prefix += warp_sum(lane <= last ? val : 0);
        if (mask) return prefix;
        base -= 32;
    }
}

/* Counting pass of the three-way partition: ctrl->totals[0..1]. */
template <typename T, typename P1, typename P2>
__global__ void __launch_bounds__(kBlock) count_kernel(const T* in, uint64_t n, Ctrl* ctrl, P1 first, P2 second)
{
    uint32_t c1 = 0, c2 = 0;
    for (uint64_t i = uint64_t(blockIdx.x) * kBlock + threadIdx.x; i < n; i += uint64_t(gridDim.x) * kBlock) {
        const T x = in[i];
        const bool s1 = first(x);
        c1 += s1;
        c2 += !s1 && second(x);
    }
    const uint64_t w = warp_sum(uint64_t(c1) | (uint64_t(c2) << 32));
    if ((threadIdx.x & 31) == 0 && w) {
        atomicAdd(&ctrl->totals[0], uint32_t(w));
        atomicAdd(&ctrl->totals[1], uint32_t(w >> 32));
    }
}

template <typename T, typename F, typename V>
struct Args {
    const T* in;
    const F* flags;
    const V* vin;
    T* out;
    T* out2;
    T* out3;
    V* vout;
    uint32_t* num_selected;  // may be null for kOutRanks
    uint64_t n;
    bool vector;
    uint32_t* ranks;  // kOutRanks: the exclusive count of selected items before each item
};

/* Selection mask of one thread's items (bit j * G + e set when pick holds;
 * bits at and above C * G are unspecified).  A predicate type may provide
 * its own select_mask overload, found by argument-dependent lookup, that
 * evaluates it over all the items at once. */
template <typename Pick, typename X, int C, int G>
__device__ __forceinline__ uint32_t select_mask(const Pick& pick, const X (&x)[C][G])
{
    uint32_t m = 0;
#pragma unroll
    for (int j = 0; j < C; ++j)
#pragma unroll
        for (int e = 0; e < G; ++e)
            if (pick(x[j][e])) m |= 1u << (j * G + e);
    return m;
}

/* Bits of a thread's items that lie below n (bit j * kGroup + e). */
__device__ __forceinline__ uint32_t valid_mask(uint64_t warp_base, int lane, uint64_t n)
{
    constexpr uint32_t kAll = (kChunks * kGroup == 32) ? ~0u : ((1u << (kChunks * kGroup)) - 1u);
    if (warp_base + uint64_t(32 * kChunks * kGroup) <= n) return kAll;
    uint32_t m = 0;
#pragma unroll
    for (int j = 0; j < kChunks; ++j) {
        const uint64_t g = warp_base + uint64_t(j * 32 + lane) * kGroup;
#pragma unroll
        for (int e = 0; e < kGroup; ++e)
            if (g + e < n) m |= 1u << (j * kGroup + e);
    }
    return m;
}

/* Selection bits of one warp's items x (bit j * kGroup + e): pick(flag)
 * (kSelFlag), pick(item) (kSelIf; three-way: sel2 = !pick && pick2), or a
 * key change against the previous item by `equal` (kSelUnique: neighbours
 * from registers, shuffles, or one load for the warp's first item). */
template <typename T, typename F, int SEL, bool THREE, typename Pick, typename Pick2, typename Equal>
__device__ __forceinline__ void select_bits(const T (&x)[kChunks][kGroup], const F (&f)[kChunks][kGroup], const T* in,
                                            uint64_t n, uint64_t warp_base, int lane, Pick pick, Pick2 pick2,
                                            Equal equal, uint32_t& sel1, uint32_t& sel2)
{
    sel1 = sel2 = 0;
    if constexpr (SEL == kSelFlag) {
        sel1 = select_mask(pick, f) & valid_mask(warp_base, lane, n);
    } else if constexpr (SEL == kSelIf) {
        const uint32_t valid = valid_mask(warp_base, lane, n);
        sel1 = select_mask(pick, x) & valid;
        if constexpr (THREE) sel2 = select_mask(pick2, x) & valid & ~sel1;
    }
    if constexpr (SEL == kSelUnique) {
#pragma unroll
        for (int j = 0; j < kChunks; ++j) {
            const T prev_lane = __shfl_up_sync(0xffffffffu, x[j][kGroup - 1], 1);
            const T prev_chunk = __shfl_sync(0xffffffffu, x[j > 0 ? j - 1 : 0][kGroup - 1], 31);
            const uint64_t g = warp_base + uint64_t(j * 32 + lane) * kGroup;
#pragma unroll
            for (int e = 0; e < kGroup; ++e) {
                const uint64_t i = g + e;
                if (i >= n) continue;
                bool h;
                if (e > 0)
                    h = !equal(x[j][e - 1], x[j][e]);
                else if (lane > 0)
                    h = !equal(prev_lane, x[j][0]);
                else if (j > 0)
                    h = !equal(prev_chunk, x[j][0]);
                else
                    h = i == 0 || !equal(in[i - 1], x[j][0]);
                if (h) sel1 |= 1u << (j * kGroup + e);
            }
        }
    }
}

/* Per chunk: this lane's exclusive packed count within the warp (group
 * columns scanned across lanes, carried across columns); returns the warp's
 * packed total. */
template <bool THREE>
__device__ __forceinline__ uint64_t chunk_prefixes(uint32_t sel1, uint32_t sel2, int lane, uint64_t (&pre)[kChunks])
{
    uint64_t carry = 0;
#pragma unroll
    for (int j = 0; j < kChunks; ++j) {
        uint64_t c = uint64_t(__popc((sel1 >> (j * kGroup)) & 0xFu));
        if constexpr (THREE) c |= uint64_t(__popc((sel2 >> (j * kGroup)) & 0xFu)) << 32;
        uint64_t incl = c;
#pragma unroll
        for (int d = 1; d < 32; d <<= 1) {
            const uint64_t y = __shfl_up_sync(0xffffffffu, incl, d);
            if (lane >= d) incl += y;
        }
        pre[j] = carry + incl - c;
        carry += __shfl_sync(0xffffffffu, incl, 31);
    }
    return carry;
}

/* Stores one warp's items once their output positions are known:
 * warp_prefix = selected items before the warp (packed), pre = per chunk. */
template <typename T, typename F, typename V, int OUT>
__device__ __forceinline__ void scatter_items(const Args<T, F, V>& a, const T (&x)[kChunks][kGroup], uint32_t sel1,
                                              uint32_t sel2, const uint64_t (&pre)[kChunks], uint64_t warp_prefix,
                                              uint64_t warp_base, int lane, uint64_t unsel_end)
{
    constexpr bool THREE = OUT == kOutThreeWay;
    constexpr bool HAS_V = !std::is_same<V, NoValue>::value;
    const uint64_t n = a.n;
    V v[kGroup];
#pragma unroll
    for (int j = 0; j < kChunks; ++j) {
        const uint64_t g = warp_base + uint64_t(j * 32 + lane) * kGroup;
        if constexpr (HAS_V) load4(a.vin, n, g, a.vector, v);
        const uint64_t base = warp_prefix + pre[j];
        uint64_t pos1 = uint32_t(base), pos2 = base >> 32;
        if constexpr (OUT == kOutRanks) {
            uint32_t r[kGroup];
#pragma unroll
            for (int e = 0; e < kGroup; ++e) {
                r[e] = uint32_t(pos1);
                pos1 += (sel1 >> (j * kGroup + e)) & 1u;
            }
            if (a.vector && g + kGroup <= n) {
                *reinterpret_cast<uint4*>(a.ranks + g) = make_uint4(r[0], r[1], r[2], r[3]);
            } else {
#pragma unroll
                for (int e = 0; e < kGroup; ++e)
                    if (g + e < n) a.ranks[g + e] = r[e];
            }
        } else {
#pragma unroll
            for (int e = 0; e < kGroup; ++e) {
                const uint64_t i = g + e;
                if (i >= n) continue;
                const int b = j * kGroup + e;
                if ((sel1 >> b) & 1u) {
                    a.out[pos1] = x[j][e];
                    if constexpr (HAS_V) a.vout[pos1] = v[e];
                    ++pos1;
                } else if constexpr (THREE) {
                    if ((sel2 >> b) & 1u) {
                        a.out2[pos2++] = x[j][e];
                    } else {
                        a.out3[unsel_end - 1 - (i - pos1 - pos2)] = x[j][e];
                    }
                } else if constexpr (OUT == kOutPartition) {
                    a.out[n - 1 - (i - pos1)] = x[j][e];
                }
            }
        }
    }
}

/* SEL: kSelFlag (pick(flag)), kSelIf (pick(item)), kSelUnique (key change by
 * `equal`); OUT: kOutSelect, kOutPartition, kOutThreeWay (pick = first,
 * pick2 = second).  One 8192-item tile per block, register loads (any
 * alignment). */
template <typename T, typename F, typename V, int SEL, int OUT, typename Pick, typename Pick2, typename Equal>
__global__ void __launch_bounds__(kBlock)
compact_kernel(Args<T, F, V> a, Ctrl* ctrl, Status<OUT == kOutThreeWay> st, Pick pick, Pick2 pick2, Equal equal)
{
    constexpr bool THREE = OUT == kOutThreeWay;
    __shared__ uint32_t s_tile;
    __shared__ uint64_t s_total[kWarps];
    __shared__ uint64_t s_excl[kWarps];
    __shared__ uint64_t s_prefix;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (threadIdx.x == 0) s_tile = atomicAdd(&ctrl->tile_counter, 1u);
    __syncthreads();
    const uint64_t tile = s_tile;
    const uint64_t n = a.n;
    const uint64_t warp_base = tile * kTileItems + uint64_t(warp) * (32 * kChunks * kGroup);

    T x[kChunks][kGroup];
    F f[kChunks][kGroup];
#pragma unroll
    for (int j = 0; j < kChunks; ++j) {
        const uint64_t g = warp_base + uint64_t(j * 32 + lane) * kGroup;
        load4(a.in, n, g, a.vector, x[j]);
        if constexpr (SEL == kSelFlag) load4(a.flags, n, g, a.vector, f[j]);
    }
    uint32_t sel1, sel2;
    select_bits<T, F, SEL, THREE>(x, f, a.in, n, warp_base, lane, pick, pick2, equal, sel1, sel2);
    uint64_t pre[kChunks];
    const uint64_t carry = chunk_prefixes<THREE>(sel1, sel2, lane, pre);
    if (lane == 0) s_total[warp] = carry;
    __syncthreads();
    if (warp == 0) {
        const uint64_t t = lane < kWarps ? s_total[lane] : 0;
        uint64_t incl = t;
#pragma unroll
        for (int d = 1; d < kWarps; d <<= 1) {
            const uint64_t y = __shfl_up_sync(0xffffffffu, incl, d);
            if (lane >= d) incl += y;
        }
        if (lane < kWarps) s_excl[lane] = incl - t;
        const uint64_t aggregate = __shfl_sync(0xffffffffu, incl, kWarps - 1);
        uint64_t prefix = 0;
        if (tile == 0) {
            if (lane == 0) st.publish(0, kInclusive, aggregate);
        } else {
            if (lane == 0) st.publish(tile, kPartial, aggregate);
            prefix = look_back<THREE>(tile, st, ctrl);
            if (lane == 0) st.publish(tile, kInclusive, prefix + aggregate);
        }
        if (lane == 0) {
            s_prefix = prefix;
            if (tile == gridDim.x - 1 && a.num_selected) {
                a.num_selected[0] = uint32_t(prefix + aggregate);
                if constexpr (THREE) a.num_selected[1] = uint32_t((prefix + aggregate) >> 32);
            }
        }
    }
    __syncthreads();
    const uint64_t unsel_end = THREE ? n - ctrl->totals[0] - ctrl->totals[1] : 0;
    scatter_items<T, F, V, OUT>(a, x, sel1, sel2, pre, s_prefix + s_excl[warp], warp_base, lane, unsel_end);
}

/* ---- Persistent variant for 16-byte aligned data ---------------------------
 * Like the plain scan's persistent kernel: each block keeps kBulkStages tiles
 * of items (and flags) in flight in shared memory, filled by bulk
 * asynchronous copies (cp.async.bulk, completion on an mbarrier, no
 * multicast) up to two tiles ahead.  8 or 16 data warps (BulkShape) and
 * one look-back warp; per iteration, concurrently:
 *   data warps -- A(k+1): selection bits and counts of tile k+1 as soon as
 *           its data is in, and its partial count published; staged outputs
 *           (select / partition / three-way without values): tile k+1
 *           compacted in place in its shared-memory stage (its items are in
 *           registers since A) -- selected items first, then the second
 *           category, then the rest in reverse;
 *   look-back warp -- the look-back of tile k, its inclusive count
 *           published;
 * then, with tile k's prefix known: tile k written out with contiguous
 * stores (staged), or its items re-read from shared memory and scattered to
 * their positions (values, ranks); and tile k's stage refilled with the
 * block's next tile.
 * Tile ids come from the atomic counter in increasing order per block, so
 * the smallest unfinished tile is always one a block is working on.  The
 * last (partial) tile is loaded with guarded plain loads. */
template <int BLOCK>
struct BulkShape {
    static constexpr int kBlock = BLOCK;  // data threads; one more warp runs the look-backs
    static constexpr int kWarps = BLOCK / 32;
    static constexpr int kThreads = BLOCK + 32;
    static constexpr uint64_t kTile = uint64_t(BLOCK) * kChunks * kGroup;
};
/* 512 data threads (8192-item tiles) when an item and its flag take at most
 * 4 bytes, else 256 (4096-item tiles): bigger tiles mean fewer look-backs,
 * and fewer tiles in flight for each look-back to walk past. */
template <typename T, typename F, int SEL>
constexpr int bulk_block()
{
    return sizeof(T) + (SEL == kSelFlag ? sizeof(F) : 0) <= 4 ? 512 : 256;
}
template <typename T, typename F, int SEL>
using BulkOf = BulkShape<bulk_block<T, F, SEL>()>;
constexpr uint64_t kBulkTileMin = uint64_t(256) * kChunks * kGroup;  // status rows are sized for it
constexpr int kBulkStages = 3;

using bulk_detail::bulk_copy;
using bulk_detail::smem_u32;

/* Bounded wait for phase `parity` of `bar`; false on timeout or when another
 * thread of the call recorded an error. */
__device__ __forceinline__ bool bulk_wait(uint64_t* bar, uint32_t parity, Ctrl* ctrl)
{
    return bulk_detail::wait(bar, parity, &ctrl->error, kWaitLimitNs);
}

template <typename T, typename F, int SEL>
constexpr size_t bulk_smem_bytes()
{
    return size_t(kBulkStages) * BulkOf<T, F, SEL>::kTile * (sizeof(T) + (SEL == kSelFlag ? sizeof(F) : 0));
}

template <typename T, typename F, typename V, int SEL, int OUT, typename Pick, typename Pick2, typename Equal>
__global__ void __launch_bounds__(BulkOf<T, F, SEL>::kThreads)
compact_bulk_kernel(Args<T, F, V> a, Ctrl* ctrl, Status<OUT == kOutThreeWay> st, uint64_t tiles, Pick pick,
                    Pick2 pick2, Equal equal)
{
    using S = BulkOf<T, F, SEL>;
    constexpr bool THREE = OUT == kOutThreeWay;
    constexpr bool FLAGS = SEL == kSelFlag;
    constexpr bool STAGED = std::is_same<V, NoValue>::value && OUT != kOutRanks;
    constexpr int kSelRows = STAGED ? 1 : kBulkStages;
    constexpr int kSelCols = STAGED ? 1 : S::kBlock;
    constexpr uint32_t kItemBytes = uint32_t(S::kTile * sizeof(T));
    constexpr uint32_t kFlagBytes = FLAGS ? uint32_t(S::kTile * sizeof(F)) : 0u;
    extern __shared__ __align__(128) unsigned char bulk_smem[];
    T* sx = reinterpret_cast<T*>(bulk_smem);                                            // [stage][tile]
    F* sf = reinterpret_cast<F*>(bulk_smem + size_t(kBulkStages) * kItemBytes);         // [stage][tile]
    __shared__ __align__(8) uint64_t s_bar[kBulkStages];
    __shared__ uint64_t s_tile[kBulkStages];
    __shared__ uint32_t s_pending;  // bit s: a copy into stage s is in flight
    __shared__ uint32_t s_phase;    // bit s: parity of the next completion of stage s
    __shared__ uint32_t s_sel[kSelRows][2][kSelCols];  // unstaged outputs: selection bits from A to B
    __shared__ uint64_t s_total[kBulkStages][S::kWarps];
    __shared__ uint64_t s_excl[kBulkStages][S::kWarps];
    __shared__ uint64_t s_agg[kBulkStages];
    __shared__ uint64_t s_prefix[kBulkStages];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const uint64_t n = a.n;
    const int toff = warp * (32 * kChunks * kGroup);  // the warp's first item in the tile
    // barrier of the data warps alone (the look-back warp runs on meanwhile)
    auto data_sync = [] { asm volatile("bar.sync 1, %0;" ::"n"(S::kBlock) : "memory"); };

    // next tile id for stage s, and its copy when the tile is full (thread 0)
    auto acquire = [&](int s) {
        if (*static_cast<volatile unsigned int*>(&ctrl->error)) {
            s_tile[s] = tiles;
            return;
        }
        const uint64_t t = atomicAdd(&ctrl->tile_counter, 1u);
        s_tile[s] = t;
        if (t < tiles && (t + 1) * S::kTile <= n) {
            s_pending |= 1u << s;
            bulk_detail::expect_bytes(&s_bar[s], kItemBytes + kFlagBytes);
            bulk_copy(sx + size_t(s) * S::kTile, a.in + t * S::kTile, kItemBytes, &s_bar[s]);
            if constexpr (FLAGS)
                bulk_copy(sf + size_t(s) * S::kTile, a.flags + t * S::kTile, kFlagBytes, &s_bar[s]);
        }
    };
    auto retire = [&](int s) {  // thread 0, after the barrier that follows the wait
        if (((s_pending >> s) & 1u) && !*static_cast<volatile unsigned int*>(&ctrl->error)) {
            s_phase ^= 1u << s;
            s_pending &= ~(1u << s);
        }
    };
    // this thread's items of the tile in stage s
    auto load = [&](int s, uint64_t tile, bool wait, T (&x)[kChunks][kGroup], F (&f)[kChunks][kGroup]) {
        const uint64_t warp_base = tile * S::kTile + uint64_t(toff);
        if ((tile + 1) * S::kTile <= n) {
            if (wait && !bulk_wait(&s_bar[s], (s_phase >> s) & 1u, ctrl)) atomicCAS(&ctrl->error, 0u, kErrTimeout);
#pragma unroll
            for (int j = 0; j < kChunks; ++j) {
                const int at = toff + (j * 32 + lane) * kGroup;
                memcpy(x[j], sx + size_t(s) * S::kTile + at, sizeof(x[j]));
                if constexpr (FLAGS) memcpy(f[j], sf + size_t(s) * S::kTile + at, sizeof(f[j]));
            }
        } else {
#pragma unroll
            for (int j = 0; j < kChunks; ++j) {
                const uint64_t g = warp_base + uint64_t(j * 32 + lane) * kGroup;
                load4(a.in, n, g, false, x[j]);
                if constexpr (FLAGS) load4(a.flags, n, g, false, f[j]);
            }
        }
    };
    // A: selection bits and the warp's count (all threads); the items stay
    // in x for the staged outputs
    auto phase_a = [&](int s, uint64_t tile, T (&x)[kChunks][kGroup], uint32_t& sel1, uint32_t& sel2) {
        F f[kChunks][kGroup];
        load(s, tile, true, x, f);
        select_bits<T, F, SEL, THREE>(x, f, a.in, n, tile * S::kTile + uint64_t(toff), lane, pick, pick2, equal,
                                      sel1, sel2);
        if constexpr (!STAGED) {
            s_sel[s][0][tid] = sel1;
            s_sel[s][1][tid] = sel2;
        }
        uint64_t c = uint64_t(__popc(sel1));
        if constexpr (THREE) c |= uint64_t(__popc(sel2)) << 32;
        c = warp_sum(c);
        if (lane == 0) s_total[s][warp] = c;
    };
    // A, warp 0 after a barrier: the tile's aggregate and its partial status
    auto publish = [&](int s, uint64_t tile) {
        const uint64_t t = lane < S::kWarps ? s_total[s][lane] : 0;
        uint64_t incl = t;
#pragma unroll
        for (int d = 1; d < S::kWarps; d <<= 1) {
            const uint64_t y = __shfl_up_sync(0xffffffffu, incl, d);
            if (lane >= d) incl += y;
        }
        if (lane < S::kWarps) s_excl[s][lane] = incl - t;
        const uint64_t aggregate = __shfl_sync(0xffffffffu, incl, S::kWarps - 1);
        if (lane == 0) {
            s_agg[s] = aggregate;
            st.publish(tile, tile == 0 ? kInclusive : kPartial, aggregate);
        }
    };
    // staged outputs, all threads after the barrier that follows publish(s):
    // the tile's items compacted in place in stage s -- selected at [0, c1),
    // second category at [c1, c1 + c2), the rest at [c1 + c2, items) in
    // reverse order -- from the registers phase A left them in
    auto stage = [&](int s, uint64_t tile, const T (&x)[kChunks][kGroup], uint32_t sel1, uint32_t sel2) {
        const uint32_t items = uint32_t(n - tile * S::kTile < S::kTile ? n - tile * S::kTile : S::kTile);
        // per-lane counts of each chunk packed in bytes (a chunk holds 128 items of the warp)
        uint32_t c1 = 0, c2 = 0;
#pragma unroll
        for (int j = 0; j < kChunks; ++j) {
            c1 |= uint32_t(__popc((sel1 >> (j * kGroup)) & 0xFu)) << (8 * j);
            if constexpr (THREE) c2 |= uint32_t(__popc((sel2 >> (j * kGroup)) & 0xFu)) << (8 * j);
        }
        uint32_t i1 = c1, i2 = c2;
#pragma unroll
        for (int d = 1; d < 32; d <<= 1) {
            const uint32_t y1 = __shfl_up_sync(0xffffffffu, i1, d);
            uint32_t y2 = 0;
            if constexpr (THREE) y2 = __shfl_up_sync(0xffffffffu, i2, d);
            if (lane >= d) {
                i1 += y1;
                if constexpr (THREE) i2 += y2;
            }
        }
        const uint32_t t1 = __shfl_sync(0xffffffffu, i1, 31);
        uint32_t t2 = 0;
        if constexpr (THREE) t2 = __shfl_sync(0xffffffffu, i2, 31);
        const uint32_t e1 = i1 - c1, e2 = i2 - c2;
        const uint64_t we = s_excl[s][warp];
        const uint32_t agg1 = uint32_t(s_agg[s]);
        uint32_t b1 = uint32_t(we), b2 = agg1 + uint32_t(we >> 32);  // chunk bases
        T* out = sx + size_t(s) * S::kTile;
#pragma unroll
        for (int j = 0; j < kChunks; ++j) {
            uint32_t p1 = b1 + ((e1 >> (8 * j)) & 0xFFu), p2 = b2 + ((e2 >> (8 * j)) & 0xFFu);
            b1 += (t1 >> (8 * j)) & 0xFFu;
            if constexpr (THREE) b2 += (t2 >> (8 * j)) & 0xFFu;
            const uint32_t t0 = uint32_t(toff + (j * 32 + lane) * kGroup);
#pragma unroll
            for (int e = 0; e < kGroup; ++e) {
                const int b = j * kGroup + e;
                if ((sel1 >> b) & 1u) {
                    out[p1++] = x[j][e];
                } else if (THREE && ((sel2 >> b) & 1u)) {
                    out[p2++] = x[j][e];
                } else if constexpr (OUT != kOutSelect) {
                    // rank among the tile's unselected items: t minus the selected ones before it
                    const uint32_t t = t0 + uint32_t(e);
                    const uint32_t q = t - p1 - (THREE ? p2 - agg1 : 0u);
                    if (t < items) out[items - 1 - q] = x[j][e];
                }
            }
        }
    };
    // staged outputs, after the look-back of the tile in stage s: its
    // compacted items written with contiguous stores
    auto write_out = [&](int s, uint64_t tile, uint64_t unsel_end) {
        const uint64_t start = tile * S::kTile;
        const uint32_t items = uint32_t(n - start < S::kTile ? n - start : S::kTile);
        const uint64_t agg = s_agg[s], prefix = s_prefix[s];
        const uint32_t c1 = uint32_t(agg);
        const T* in = sx + size_t(s) * S::kTile;
        if constexpr (OUT == kOutSelect) {
            T* o1 = a.out + uint32_t(prefix);
            for (uint32_t m = uint32_t(tid); m < c1; m += S::kBlock) o1[m] = in[m];
        } else if constexpr (OUT == kOutPartition) {
            // unselected rank q (in order) goes to n - 1 - (start - prefix + q), staged at items - 1 - q
            T* o1 = a.out + prefix;
            T* o0 = a.out + (n - start - items + prefix);
            for (uint32_t m = uint32_t(tid); m < items; m += S::kBlock) (m < c1 ? o1 : o0)[m] = in[m];
        } else {
            const uint32_t c2 = uint32_t(agg >> 32);
            const uint64_t p1 = uint32_t(prefix), p2 = prefix >> 32;
            const uint64_t u = start - p1 - p2;  // unselected items before the tile
            for (uint32_t m = uint32_t(tid); m < items; m += S::kBlock) {
                if (m < c1)
                    a.out[p1 + m] = in[m];
                else if (m < c1 + c2)
                    a.out2[p2 + (m - c1)] = in[m];
                else
                    a.out3[unsel_end - u - items + m] = in[m];
            }
        }
    };

    T x[kChunks][kGroup];
    uint32_t sel1 = 0, sel2 = 0;
    const bool data = warp < S::kWarps;
    // Hand-offs between the data warps and the look-back warp (named
    // barriers over the whole block: one side arrives, the other waits).
    // Barrier 3, "aggregate ready": tile k+1's aggregate is published and
    // tile k's prefix has been consumed; barrier 2, "prefix ready".  Each
    // side arrives once per tile and only after the other side's previous
    // arrival was consumed, so no barrier ever sees two arrivals of a side.
    auto agg_ready_signal = [] { asm volatile("bar.arrive 3, %0;" ::"n"(S::kThreads) : "memory"); };
    auto agg_ready_wait = [] { asm volatile("bar.sync 3, %0;" ::"n"(S::kThreads) : "memory"); };
    auto prefix_ready_signal = [] { asm volatile("bar.arrive 2, %0;" ::"n"(S::kThreads) : "memory"); };
    auto prefix_ready_wait = [] { asm volatile("bar.sync 2, %0;" ::"n"(S::kThreads) : "memory"); };
    if (tid == 0) {
        s_pending = 0;
        s_phase = 0;
        for (int s = 0; s < kBulkStages; ++s) bulk_detail::init_barrier(&s_bar[s]);
        bulk_detail::fence_barrier_init();
        for (int s = 0; s < kBulkStages; ++s) acquire(s);
    }
    __syncthreads();

    const uint64_t unsel_end = THREE ? n - ctrl->totals[0] - ctrl->totals[1] : 0;
    if (s_tile[0] < tiles) {
        if (data) {
            phase_a(0, s_tile[0], x, sel1, sel2);
            data_sync();
            if (warp == 0) {
                if (lane == 0) retire(0);
                publish(0, s_tile[0]);
            }
            if constexpr (STAGED) {
                data_sync();
                stage(0, s_tile[0], x, sel1, sel2);
            }
            agg_ready_signal();
            for (uint32_t k = 0;; ++k) {
                const int s = int(k % kBulkStages);
                const int ns = int((k + 1) % kBulkStages);
                const uint64_t tile = s_tile[s];
                const uint64_t next = s_tile[ns];
                const bool has_next = next < tiles;
                if (has_next) {
                    phase_a(ns, next, x, sel1, sel2);
                    data_sync();  // counts of tile k+1 visible
                    if (warp == 0) {
                        if (lane == 0) retire(ns);
                        publish(ns, next);
                    }
                    if constexpr (STAGED) {
                        data_sync();  // offsets of tile k+1 visible
                        stage(ns, next, x, sel1, sel2);
                    }
                }
                prefix_ready_wait();  // tile k's prefix
                if (has_next) agg_ready_signal();
                if constexpr (STAGED) {
                    write_out(s, tile, unsel_end);
                } else {
                    T xs[kChunks][kGroup];
                    F f[kChunks][kGroup];
                    load(s, tile, false, xs, f);
                    const uint32_t b1 = s_sel[s][0][tid], b2 = s_sel[s][1][tid];
                    uint64_t pre[kChunks];
                    chunk_prefixes<THREE>(b1, b2, lane, pre);
                    scatter_items<T, F, V, OUT>(a, xs, b1, b2, pre, s_prefix[s] + s_excl[s][warp],
                                                tile * S::kTile + uint64_t(toff), lane, unsel_end);
                }
                data_sync();  // stage s is free
                if (tid == 0) {
                    // the stage's generic-proxy accesses are ordered before the copy that refills it
                    bulk_detail::fence_proxy_async();
                    acquire(s);
                }
                if (!has_next) break;
            }
        } else {
            // the look-back warp: one tile after the other, as their aggregates appear
            for (uint32_t k = 0;; ++k) {
                const int s = int(k % kBulkStages);
                agg_ready_wait();
                const uint64_t tile = s_tile[s];
                uint64_t prefix = 0;
                if (tile > 0) {
                    prefix = look_back<THREE>(tile, st, ctrl);
                    if (lane == 0) st.publish(tile, kInclusive, prefix + s_agg[s]);
                }
                if (lane == 0) {
                    s_prefix[s] = prefix;
                    if (tile == tiles - 1 && a.num_selected) {
                        a.num_selected[0] = uint32_t(prefix + s_agg[s]);
                        if constexpr (THREE) a.num_selected[1] = uint32_t((prefix + s_agg[s]) >> 32);
                    }
                }
                prefix_ready_signal();
                if (s_tile[(k + 1) % kBulkStages] >= tiles) break;
            }
        }
    }
    __syncthreads();
    // copies not retired (only after an error): wait for them, bounded,
    // before the block's shared memory goes away
    if (tid == 0 && s_pending) {
        for (int s = 0; s < kBulkStages; ++s)
            if ((s_pending >> s) & 1u)
                if (!bulk_wait(&s_bar[s], (s_phase >> s) & 1u, ctrl)) atomicCAS(&ctrl->error, 0u, kErrTimeout);
    }
}

struct Layout {
    size_t ctrl, word, second_p, second_i, total;
    uint64_t tiles;
};

inline Layout layout(uint64_t n, bool three)
{
    Layout L{};
    // status rows for the smaller tile of the two kernels
    L.tiles = n ? (n + kBulkTileMin - 1) / kBulkTileMin : 0;
    auto up = [](size_t x) { return (x + kAlign - 1) / kAlign * kAlign; };
    L.ctrl = 0;
    L.word = kAlign;
    L.second_p = up(L.word + size_t(L.tiles) * 8 * kStatusStride);
    L.second_i = up(L.second_p + (three ? size_t(L.tiles) * 4 : 0));
    L.total = up(L.second_i + (three ? size_t(L.tiles) * 4 : 0));
    return L;
}

inline bool aligned16(const void* p) { return p == nullptr || reinterpret_cast<uintptr_t>(p) % 16 == 0; }

template <int SEL, int OUT, typename T, typename F, typename V, typename Pick, typename Pick2, typename Equal>
cudaError_t launch(void* temp, size_t temp_bytes, Args<T, F, V> a, Pick pick, Pick2 pick2, Equal equal,
                   cudaStream_t stream)
{
    constexpr bool THREE = OUT == kOutThreeWay;
    constexpr bool RANKS = OUT == kOutRanks;
    if (!a.num_selected && !RANKS) return cudaErrorInvalidValue;
    if (a.n == 0)
        return a.num_selected ? cudaMemsetAsync(a.num_selected, 0, (THREE ? 2 : 1) * sizeof(uint32_t), stream)
                              : cudaSuccess;
    if (a.n > 0xffffffffull || !a.in || (RANKS ? !a.ranks : !a.out) || (THREE && (!a.out2 || !a.out3)))
        return cudaErrorInvalidValue;
    if (SEL == kSelFlag && !a.flags) return cudaErrorInvalidValue;
    const Layout L = layout(a.n, THREE);
    if (!temp || reinterpret_cast<uintptr_t>(temp) % kAlign || temp_bytes < L.total) return cudaErrorInvalidValue;
    unsigned char* t = static_cast<unsigned char*>(temp);
    cudaError_t e = cudaMemsetAsync(t, 0, L.word + size_t(L.tiles) * 8 * kStatusStride, stream);
    if (e != cudaSuccess) return e;
    Ctrl* ctrl = reinterpret_cast<Ctrl*>(t);
    int dev = 0, sms = 0;
    e = cudaGetDevice(&dev);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return e;
    if constexpr (THREE) {
        const uint64_t want = (a.n + kBlock - 1) / kBlock;
        const unsigned grid = unsigned(std::min<uint64_t>(want, uint64_t(sms > 0 ? sms : 1) * 8));
        count_kernel<<<grid, kBlock, 0, stream>>>(a.in, a.n, ctrl, pick, pick2);
        e = cudaGetLastError();
        if (e != cudaSuccess) return e;
    }
    a.vector = aligned16(a.in) && aligned16(a.flags) && aligned16(a.vin) && aligned16(a.out) &&
               aligned16(a.vout) && aligned16(a.out2) && aligned16(a.out3) && aligned16(a.ranks);
    Status<THREE> st{reinterpret_cast<uint64_t*>(t + L.word), reinterpret_cast<uint32_t*>(t + L.second_p),
                     reinterpret_cast<uint32_t*>(t + L.second_i)};
    if (a.vector) {
        // 16-byte aligned: the persistent bulk-copy kernel, as many blocks as are resident
        using Shape = BulkOf<T, F, SEL>;
        auto kernel = compact_bulk_kernel<T, F, V, SEL, OUT, Pick, Pick2, Equal>;
        constexpr size_t smem = bulk_smem_bytes<T, F, SEL>();
        e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
        int per_sm = 0;
        if (e == cudaSuccess) e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, Shape::kThreads, smem);
        if (e != cudaSuccess) return e;
        const uint64_t tiles = (a.n + Shape::kTile - 1) / Shape::kTile;
        const uint64_t resident = uint64_t(sms > 0 ? sms : 1) * uint64_t(per_sm > 0 ? per_sm : 1);
        kernel<<<unsigned(std::min(tiles, resident)), Shape::kThreads, smem, stream>>>(a, ctrl, st, tiles, pick, pick2,
                                                                                 equal);
    } else {
        const uint64_t tiles = (a.n + kTileItems - 1) / kTileItems;
        compact_kernel<T, F, V, SEL, OUT><<<unsigned(tiles), kBlock, 0, stream>>>(a, ctrl, st, pick, pick2, equal);
    }
    return cudaGetLastError();
}

struct Never {
    template <typename X>
    __device__ __forceinline__ bool operator()(X) const { return false; }
};

}  // namespace select_detail

/* Temp storage bytes of the select / partition forms (any item type);
 * three_way: the three-way partition. */
inline size_t select_temp_bytes(uint64_t num_items, bool three_way = false)
{
    return num_items ? select_detail::layout(num_items, three_way).total : 0;
}

/* DeviceSelect / DevicePartition with user callables.  num_items < 2^32
 * (uint32 counts, as the reference); zero items write zero count(s).
 * d_out may equal d_in for the select forms. */
template <typename T, typename F, typename Pick = NonZero>
cudaError_t select_flagged(void* temp, size_t temp_bytes, const T* d_in, const F* d_flags, T* d_out,
                           uint32_t* d_num_selected_out, uint64_t num_items, Pick pick = Pick{},
                           cudaStream_t stream = 0)
{
    using namespace select_detail;
    Args<T, F, NoValue> a{d_in, d_flags, nullptr, d_out, nullptr, nullptr, nullptr, d_num_selected_out, num_items,
                          false, nullptr};
    return launch<kSelFlag, kOutSelect>(temp, temp_bytes, a, pick, Never{}, EqualTo{}, stream);
}

template <typename T, typename Pick>
cudaError_t select_if(void* temp, size_t temp_bytes, const T* d_in, T* d_out, uint32_t* d_num_selected_out,
                      uint64_t num_items, Pick pick, cudaStream_t stream = 0)
{
    using namespace select_detail;
    Args<T, T, NoValue> a{d_in, nullptr, nullptr, d_out, nullptr, nullptr, nullptr, d_num_selected_out, num_items,
                          false, nullptr};
    return launch<kSelIf, kOutSelect>(temp, temp_bytes, a, pick, Never{}, EqualTo{}, stream);
}

template <typename T, typename Equal = EqualTo>
cudaError_t select_unique(void* temp, size_t temp_bytes, const T* d_in, T* d_out, uint32_t* d_num_selected_out,
                          uint64_t num_items, Equal equal = Equal{}, cudaStream_t stream = 0)
{
    using namespace select_detail;
    Args<T, T, NoValue> a{d_in, nullptr, nullptr, d_out, nullptr, nullptr, nullptr, d_num_selected_out, num_items,
                          false, nullptr};
    return launch<kSelUnique, kOutSelect>(temp, temp_bytes, a, Never{}, Never{}, equal, stream);
}

template <typename K, typename V, typename Equal = EqualTo>
cudaError_t select_unique_by_key(void* temp, size_t temp_bytes, const K* d_keys_in, const V* d_values_in,
                                 K* d_keys_out, V* d_values_out, uint32_t* d_num_selected_out, uint64_t num_items,
                                 Equal equal = Equal{}, cudaStream_t stream = 0)
{
    using namespace select_detail;
    if (num_items && (!d_values_in || !d_values_out)) return cudaErrorInvalidValue;
    Args<K, K, V> a{d_keys_in, nullptr, d_values_in, d_keys_out, nullptr, nullptr, d_values_out, d_num_selected_out,
                    num_items, false, nullptr};
    return launch<kSelUnique, kOutSelect>(temp, temp_bytes, a, Never{}, Never{}, equal, stream);
}

template <typename T, typename F, typename Pick = NonZero>
cudaError_t partition_flagged(void* temp, size_t temp_bytes, const T* d_in, const F* d_flags, T* d_out,
                              uint32_t* d_num_selected_out, uint64_t num_items, Pick pick = Pick{},
                              cudaStream_t stream = 0)
{
    using namespace select_detail;
    if (num_items && d_out == d_in) return cudaErrorInvalidValue;
    Args<T, F, NoValue> a{d_in, d_flags, nullptr, d_out, nullptr, nullptr, nullptr, d_num_selected_out, num_items,
                          false, nullptr};
    return launch<kSelFlag, kOutPartition>(temp, temp_bytes, a, pick, Never{}, EqualTo{}, stream);
}

template <typename T, typename Pick>
cudaError_t partition_if(void* temp, size_t temp_bytes, const T* d_in, T* d_out, uint32_t* d_num_selected_out,
                         uint64_t num_items, Pick pick, cudaStream_t stream = 0)
{
    using namespace select_detail;
    if (num_items && d_out == d_in) return cudaErrorInvalidValue;
    Args<T, T, NoValue> a{d_in, nullptr, nullptr, d_out, nullptr, nullptr, nullptr, d_num_selected_out, num_items,
                          false, nullptr};
    return launch<kSelIf, kOutPartition>(temp, temp_bytes, a, pick, Never{}, EqualTo{}, stream);
}

/* DeviceScan::ExclusiveSumTransform / ExclusiveSumAdjacent
 * (src/lcpp/device/device_scan.h:387-406, details/scan.h:127-240):
 * d_out[i] = the number of j < i with pick(d_in[j]), or with j == 0 ||
 * !equal(d_in[j - 1], d_in[j]).  Temp storage: select_temp_bytes. */
template <typename T, typename Pick>
cudaError_t exclusive_sum_transform(void* temp, size_t temp_bytes, const T* d_in, uint32_t* d_out,
                                    uint64_t num_items, Pick pick, cudaStream_t stream = 0)
{
    using namespace select_detail;
    Args<T, T, NoValue> a{d_in, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, num_items, false,
                          d_out};
    return launch<kSelIf, kOutRanks>(temp, temp_bytes, a, pick, Never{}, EqualTo{}, stream);
}

template <typename T, typename Equal = EqualTo>
cudaError_t exclusive_sum_adjacent(void* temp, size_t temp_bytes, const T* d_in, uint32_t* d_out,
                                   uint64_t num_items, Equal equal = Equal{}, cudaStream_t stream = 0)
{
    using namespace select_detail;
    Args<T, T, NoValue> a{d_in, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, num_items, false,
                          d_out};
    return launch<kSelUnique, kOutRanks>(temp, temp_bytes, a, Never{}, Never{}, equal, stream);
}

/* d_num_selected_out[0] = first count, [1] = second count. */
template <typename T, typename Pick1, typename Pick2>
cudaError_t partition_three_way(void* temp, size_t temp_bytes, const T* d_in, T* d_first_out, T* d_second_out,
                                T* d_unselected_out, uint32_t* d_num_selected_out, uint64_t num_items,
                                Pick1 select_first, Pick2 select_second, cudaStream_t stream = 0)
{
    using namespace select_detail;
    Args<T, T, NoValue> a{d_in, nullptr, nullptr, d_first_out, d_second_out, d_unselected_out, nullptr,
                          d_num_selected_out, num_items, false, nullptr};
    return launch<kSelIf, kOutThreeWay>(temp, temp_bytes, a, select_first, select_second, EqualTo{}, stream);
}

/* ---------------------------------------------------------------------------
 * Reduce / TransformReduce and the plain scans with a user operator
 * (src/lcpp/device/device_reduce.h:229-308, :493-516; device_scan.h:321-368).
 *
 * Reduce: d_out[0] = init op (transform(d_in[0]) op ... op transform(d_in[n-1]));
 * op must be associative and commutative (the partial results of blocks and
 * warps combine in a fixed but not left-to-right order).  Two levels as
 * ArgMin / ArgMax: each block folds an equal contiguous chunk, the last block
 * to finish folds the partials.  Zero items write init.
 *
 * The scans with a user operator run the by-key pass with every key equal
 * (one segment), so they keep left-to-right operand order: op need only be
 * associative.  Temp storage: by_key_temp_bytes(num_items, sizeof(T)).
 * ------------------------------------------------------------------------- */

/* "all keys equal": the by-key pass over one segment is a plain scan */
struct AlwaysEqual {
    template <typename K>
    __device__ __forceinline__ bool operator()(K, K) const { return true; }
};

struct Identity {
    template <typename T>
    __device__ __forceinline__ T operator()(T x) const { return x; }
};

namespace reduce_detail {

constexpr int kBlock = 256;
constexpr int kBlocksPerSm = 4;
constexpr uint64_t kMaxBlocks = 4096;
constexpr size_t kAlign = 256;

inline size_t temp_bytes(size_t value_bytes) { return kAlign + size_t(kMaxBlocks) * value_bytes; }

template <typename T, typename Op>
__device__ __forceinline__ T warp_fold(T v, bool has, bool& out_has, const Op& op)
{
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const T ov = __shfl_down_sync(0xffffffffu, v, o);
        const bool oh = __shfl_down_sync(0xffffffffu, int(has), o) != 0;
        if ((threadIdx.x & 31) + o < 32 && oh) {
            v = has ? op(v, ov) : ov;
            has = true;
        }
    }
    out_has = has;
    return v;
}

/* Result in thread 0. */
template <typename T, typename Op>
__device__ __forceinline__ T block_fold(T v, bool has, bool& out_has, const Op& op, T* s_v, int* s_h)
{
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    v = warp_fold(v, has, has, op);
    if (lane == 0) {
        s_v[warp] = v;
        s_h[warp] = has;
    }
    __syncthreads();
    if (warp == 0) {
        const bool h = lane < kBlock / 32 && s_h[lane];
        v = warp_fold(h ? s_v[lane] : v, h, has, op);
    }
    out_has = has;
    return v;
}

template <typename T, typename U, typename Op, typename Tr>
__global__ void __launch_bounds__(kBlock)
reduce_kernel(const U* in, uint64_t n, uint64_t chunk, T* partials, unsigned int* done, T* out, T init, Op op, Tr tr)
{
    __shared__ T s_v[kBlock / 32];
    __shared__ int s_h[kBlock / 32];
    __shared__ int s_last;
    const uint64_t lo = uint64_t(blockIdx.x) * chunk;
    const uint64_t hi = lo + chunk < n ? lo + chunk : n;
    T acc{};
    bool has = false;
    for (uint64_t i = lo + threadIdx.x; i < hi; i += kBlock) {
        const T x = tr(in[i]);
        acc = has ? op(acc, x) : x;
        has = true;
    }
    acc = block_fold(acc, has, has, op, s_v, s_h);
    if (threadIdx.x == 0) {
        partials[blockIdx.x] = acc;  // every block holds at least one item
        __threadfence();
        s_last = atomicAdd(done, 1u) == gridDim.x - 1;
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    T f{};
    bool fh = false;
    for (uint32_t b = threadIdx.x; b < gridDim.x; b += kBlock) {
        const T p = *static_cast<const volatile T*>(partials + b);
        f = fh ? op(f, p) : p;
        fh = true;
    }
    __syncthreads();
    f = block_fold(f, fh, fh, op, s_v, s_h);
    if (threadIdx.x == 0) *out = op(init, f);
}

template <typename T>
__global__ void store_kernel(T* out, T v)
{
    *out = v;
}

}  // namespace reduce_detail

/* Temp storage bytes of transform_reduce / reduce (any item count). */
inline size_t reduce_temp_bytes(size_t value_bytes) { return reduce_detail::temp_bytes(value_bytes); }

template <typename T, typename U, typename Op, typename Transform>
cudaError_t transform_reduce(void* temp, size_t temp_bytes, const U* d_in, T* d_out, uint64_t num_items, Op op,
                             Transform transform, T init, cudaStream_t stream = 0)
{
    using namespace reduce_detail;
    if (!d_out) return cudaErrorInvalidValue;
    if (num_items == 0) {
        store_kernel<T><<<1, 1, 0, stream>>>(d_out, init);
        return cudaGetLastError();
    }
    if (!d_in || !temp || reinterpret_cast<uintptr_t>(temp) % kAlign || temp_bytes < reduce_detail::temp_bytes(sizeof(T)))
        return cudaErrorInvalidValue;
    int dev = 0, sms = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return e;
    const uint64_t max_blocks = std::min<uint64_t>(kMaxBlocks, uint64_t(sms > 0 ? sms : 1) * kBlocksPerSm);
    uint64_t blocks = std::max<uint64_t>(1, std::min<uint64_t>(max_blocks, (num_items + kBlock - 1) / kBlock));
    const uint64_t chunk = (num_items + blocks - 1) / blocks;
    blocks = (num_items + chunk - 1) / chunk;
    unsigned char* t = static_cast<unsigned char*>(temp);
    e = cudaMemsetAsync(t, 0, sizeof(unsigned int), stream);
    if (e != cudaSuccess) return e;
    reduce_kernel<T, U><<<unsigned(blocks), kBlock, 0, stream>>>(d_in, num_items, chunk,
                                                                 reinterpret_cast<T*>(t + kAlign),
                                                                 reinterpret_cast<unsigned int*>(t), d_out, init,
                                                                 op, transform);
    return cudaGetLastError();
}

template <typename T, typename Op>
cudaError_t reduce(void* temp, size_t temp_bytes, const T* d_in, T* d_out, uint64_t num_items, Op op, T init,
                   cudaStream_t stream = 0)
{
    return transform_reduce(temp, temp_bytes, d_in, d_out, num_items, op, Identity{}, init, stream);
}

/* mode: 0 exclusive (init), 1 inclusive, 2 inclusive with init. */
template <typename T, typename Op>
cudaError_t scan(void* temp, size_t temp_bytes, const T* d_in, T* d_out, uint64_t num_items, int mode, T init, Op op,
                 cudaStream_t stream = 0)
{
    return scan_by_key(temp, temp_bytes, d_in, d_in, d_out, num_items, mode, init, op, AlwaysEqual{}, stream);
}

}  // namespace device
}  // namespace lcpp_b200

#endif /* LCPP_B200_DEVICE_CUH */
