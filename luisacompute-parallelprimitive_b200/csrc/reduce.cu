// reduce.cu -- deterministic two-level reduction for sm_100a.
//
// Replaces DeviceReduce's multi-level recursion (src/lcpp/device/
// device_reduce.h:728-1020, details/reduce.h:197-241, agent/agent_reduce.h).
// A persistent grid of a few blocks per SM splits the input into equal
// contiguous chunks (16-byte vector loads, UNROLL independent accumulators per
// thread), reduces each chunk with a fixed tree, and the last block to finish
// folds the per-block partials in index order and applies the initial value.
// The partition depends only on n and the SM count, so floating-point
// results are identical from run to run.  The reference's grid overruns past
// 10240 tiles (src/lcpp/common/grid_even_shared.h:82-87); this partition is
// exact for any 64-bit n.
#include "common.cuh"
#include "ops.cuh"
#include "reduce.cuh"

namespace lcpp {
namespace reduce {

struct Ctrl {
    uint32_t done;
    uint32_t error;
};

template <typename T>
struct VecOf;
template <> struct VecOf<uint32_t> { using type = uint4; };
template <> struct VecOf<int32_t> { using type = int4; };
template <> struct VecOf<float> { using type = float4; };
template <> struct VecOf<uint64_t> { using type = ulonglong2; };
template <> struct VecOf<int64_t> { using type = longlong2; };
template <> struct VecOf<double> { using type = double2; };

template <typename T, typename Op, int BLOCK>
__device__ __forceinline__ T block_reduce(T v, T* s_warp, Op op, T ident)
{
    constexpr int WARPS = BLOCK / kWarp;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    v = warp_reduce(v, op);
    if (lane == 0) s_warp[warp] = v;
    __syncthreads();
    T r = ident;
    if (warp == 0) r = warp_reduce(lane < WARPS ? s_warp[lane] : ident, op);
    return r;  // valid in warp 0
}

template <typename T, typename Op, int BLOCK, int UNROLL, bool VECTOR>
__global__ void __launch_bounds__(BLOCK)
reduce_kernel(const T* __restrict__ in, uint64_t n, uint64_t chunk, T* partials, Ctrl* ctrl,
              T* out, T init)
{
    constexpr int VEC = 16 / sizeof(T);
    using VT = typename VecOf<T>::type;
    __shared__ T s_warp[BLOCK / kWarp];
    __shared__ int s_last;
    const Op op;
    const T ident = Identity<Op, T>::value();
    const int tid = threadIdx.x;

    T acc[UNROLL][VEC];
#pragma unroll
    for (int u = 0; u < UNROLL; ++u)
#pragma unroll
        for (int e = 0; e < VEC; ++e) acc[u][e] = ident;

    const uint64_t lo = uint64_t(blockIdx.x) * chunk;
    const uint64_t hi = min(lo + chunk, n);
    if (lo < hi) {
        if constexpr (VECTOR) {
            const uint64_t nvec = (hi - lo) / VEC;
            const VT* vp = reinterpret_cast<const VT*>(in + lo);
            uint64_t j = tid;
            for (; j + uint64_t(UNROLL - 1) * BLOCK < nvec; j += uint64_t(UNROLL) * BLOCK) {
                VT x[UNROLL];
#pragma unroll
                for (int u = 0; u < UNROLL; ++u) x[u] = vp[j + u * BLOCK];
#pragma unroll
                for (int u = 0; u < UNROLL; ++u) {
                    T t[VEC];
                    memcpy(t, &x[u], 16);
#pragma unroll
                    for (int e = 0; e < VEC; ++e) acc[u][e] = op(acc[u][e], t[e]);
                }
            }
            for (; j < nvec; j += BLOCK) {
                const VT x = vp[j];
                T t[VEC];
                memcpy(t, &x, 16);
#pragma unroll
                for (int e = 0; e < VEC; ++e) acc[0][e] = op(acc[0][e], t[e]);
            }
            for (uint64_t i = lo + nvec * VEC + tid; i < hi; i += BLOCK) acc[0][0] = op(acc[0][0], in[i]);
        } else {
            uint64_t i = lo + tid;
            for (; i + uint64_t(UNROLL - 1) * BLOCK < hi; i += uint64_t(UNROLL) * BLOCK) {
                T x[UNROLL];
#pragma unroll
                for (int u = 0; u < UNROLL; ++u) x[u] = in[i + u * BLOCK];
#pragma unroll
                for (int u = 0; u < UNROLL; ++u) acc[u][0] = op(acc[u][0], x[u]);
            }
            for (; i < hi; i += BLOCK) acc[0][0] = op(acc[0][0], in[i]);
        }
    }
    // Fixed combination order of the accumulators.
    T t = acc[0][0];
#pragma unroll
    for (int e = 1; e < VEC; ++e) t = op(t, acc[0][e]);
#pragma unroll
    for (int u = 1; u < UNROLL; ++u)
#pragma unroll
        for (int e = 0; e < VEC; ++e) t = op(t, acc[u][e]);
    t = block_reduce<T, Op, BLOCK>(t, s_warp, op, ident);
    if (tid == 0) partials[blockIdx.x] = t;
    __threadfence();
    __syncthreads();
    if (tid == 0) s_last = atomicAdd(&ctrl->done, 1u) == gridDim.x - 1;
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    // Last block: fold the partials in index order per thread, then the tree.
    T f = ident;
    for (uint32_t i = tid; i < gridDim.x; i += BLOCK) {
        T p;
        if constexpr (sizeof(T) == 4) {
            const uint32_t b = __ldcg(reinterpret_cast<const uint32_t*>(partials) + i);
            memcpy(&p, &b, 4);
        } else {
            const unsigned long long b = __ldcg(reinterpret_cast<const unsigned long long*>(partials) + i);
            memcpy(&p, &b, 8);
        }
        f = op(f, p);
    }
    __syncthreads();
    f = block_reduce<T, Op, BLOCK>(f, s_warp, op, ident);
    if (tid == 0) *out = op(init, f);
}

template <typename B>
__global__ void store_value(B* out, B v)
{
    *out = v;
}

namespace {

constexpr int kBlock = 512;
constexpr int kUnroll = 4;
constexpr int kBlocksPerSm = 2;
// Upper bound of the grid; fixes the temp size independently of the device.
constexpr uint64_t kMaxBlocks = 4096;

struct Layout {
    size_t ctrl, partials, total;
    uint64_t blocks, chunk;
};

Layout make_layout(int tb, uint64_t n)
{
    Layout L{};
    const uint64_t vec = 16 / tb;
    const uint64_t step = uint64_t(kBlock) * vec * kUnroll;
    const uint64_t max_blocks = std::min<uint64_t>(kMaxBlocks, uint64_t(device_sm_count()) * kBlocksPerSm);
    L.blocks = std::max<uint64_t>(1, std::min(max_blocks, ceil_div(n, step)));
    L.chunk = align_up(ceil_div(n, L.blocks), vec * kBlock);
    L.blocks = std::max<uint64_t>(1, ceil_div(n, L.chunk));
    size_t off = 0;
    L.ctrl = off; off += kTempAlign;
    L.partials = off; off = align_up(off + size_t(kMaxBlocks) * tb, kTempAlign);
    L.total = off;
    return L;
}

template <typename T, typename Op>
lcpp_status launch(unsigned char* temp, const Layout& L, const T* in, T* out, uint64_t n, T init,
                   cudaStream_t stream)
{
    LCPP_CUDA_TRY(cudaMemsetAsync(temp + L.ctrl, 0, sizeof(Ctrl), stream));
    Ctrl* ctrl = reinterpret_cast<Ctrl*>(temp + L.ctrl);
    T* partials = reinterpret_cast<T*>(temp + L.partials);
    const bool aligned = (reinterpret_cast<uintptr_t>(in) & 15) == 0;
    diag::KernelTimer timer(3 /* LCPP_KERNEL_REDUCE */, n, stream);
    if (aligned)
        reduce_kernel<T, Op, kBlock, kUnroll, true><<<unsigned(L.blocks), kBlock, 0, stream>>>(
            in, n, L.chunk, partials, ctrl, out, init);
    else
        reduce_kernel<T, Op, kBlock, kUnroll, false><<<unsigned(L.blocks), kBlock, 0, stream>>>(
            in, n, L.chunk, partials, ctrl, out, init);
    return cudaGetLastError() == cudaSuccess ? LCPP_OK : LCPP_ERR_CUDA;
}

template <typename T>
lcpp_status by_op(unsigned char* temp, const Layout& L, const void* in, void* out, uint64_t n,
                  lcpp_op op, const void* init, cudaStream_t stream)
{
    T init_v;
    memcpy(&init_v, init, sizeof(T));
    const T* i = static_cast<const T*>(in);
    T* o = static_cast<T*>(out);
    switch (op) {
    case LCPP_OP_SUM: return launch<T, SumOp>(temp, L, i, o, n, init_v, stream);
    case LCPP_OP_MIN: return launch<T, MinOp>(temp, L, i, o, n, init_v, stream);
    case LCPP_OP_MAX: return launch<T, MaxOp>(temp, L, i, o, n, init_v, stream);
    default: return LCPP_ERR_UNSUPPORTED_DTYPE;
    }
}

}  // namespace

size_t temp_bytes(lcpp_dtype dt, uint64_t n)
{
    const int tb = dtype_bytes(dt);
    if (n == 0 || tb == 0) return 0;
    return make_layout(tb, n).total;
}

lcpp_status run(void* temp, size_t temp_bytes_given, const void* in, void* out, uint64_t n,
                lcpp_op op, const void* init, lcpp_dtype dt, cudaStream_t stream)
{
    diag::Range nvtx_range("lcpp DeviceReduce");
    const int tb = dtype_bytes(dt);
    if (tb == 0) return LCPP_ERR_UNSUPPORTED_DTYPE;
    if (op != LCPP_OP_SUM && op != LCPP_OP_MIN && op != LCPP_OP_MAX) return LCPP_ERR_UNSUPPORTED_DTYPE;
    if (!init || !out) return LCPP_ERR_INVALID_ARG;
    if (n == 0) {
        // Empty input writes the initial value (device_reduce.h:238-242).
        if (reinterpret_cast<uintptr_t>(out) % tb) return LCPP_ERR_INVALID_ARG;
        if (tb == 4) {
            uint32_t v;
            memcpy(&v, init, 4);
            store_value<uint32_t><<<1, 1, 0, stream>>>(static_cast<uint32_t*>(out), v);
        } else {
            unsigned long long v;
            memcpy(&v, init, 8);
            store_value<unsigned long long><<<1, 1, 0, stream>>>(static_cast<unsigned long long*>(out), v);
        }
        return cudaGetLastError() == cudaSuccess ? LCPP_OK : LCPP_ERR_CUDA;
    }
    if (!in) return LCPP_ERR_INVALID_ARG;
    if (reinterpret_cast<uintptr_t>(in) % tb || reinterpret_cast<uintptr_t>(out) % tb) return LCPP_ERR_INVALID_ARG;
    if (!temp || (reinterpret_cast<uintptr_t>(temp) & (kTempAlign - 1))) return LCPP_ERR_INVALID_ARG;
    const Layout L = make_layout(tb, n);
    if (temp_bytes_given < L.total) return LCPP_ERR_TEMP_TOO_SMALL;
    unsigned char* t = static_cast<unsigned char*>(temp);
    switch (dt) {
    case LCPP_I32: return by_op<int32_t>(t, L, in, out, n, op, init, stream);
    case LCPP_U32: return by_op<uint32_t>(t, L, in, out, n, op, init, stream);
    case LCPP_F32: return by_op<float>(t, L, in, out, n, op, init, stream);
    case LCPP_I64: return by_op<int64_t>(t, L, in, out, n, op, init, stream);
    case LCPP_U64: return by_op<uint64_t>(t, L, in, out, n, op, init, stream);
    case LCPP_F64: return by_op<double>(t, L, in, out, n, op, init, stream);
    default: return LCPP_ERR_UNSUPPORTED_DTYPE;
    }
}

}  // namespace reduce
}  // namespace lcpp
