// scan.cu -- single-pass decoupled look-back scan for sm_100a.
//
// Replaces DeviceScan's CUDA path (src/lcpp/device/device_scan.h:606-697,
// details/scan.h:242-335, details/single_pass_scan_operator.h:119-332).
//
// Tile = BLOCK threads x CHUNKS chunks x one 16-byte vector per thread and
// chunk.  Warp w owns a contiguous segment of the tile; within it, chunk j of
// lane l is the 16-byte vector at segment + (j*32 + l) * VEC, so every load
// and store is a fully coalesced 512-byte warp access and the items of each
// thread are consecutive in memory.  The scan is built bottom-up: vector
// (sequential) -> warp (shuffle scan of vector totals) -> chunk carry ->
// block (shared memory) -> tile prefix (decoupled look-back).
//
// Tile status: for 4-byte types one 64-bit word {value:32 | flag:32} per tile
// read and written with single relaxed GPU-scope accesses (the reference's
// PackedScanTileStateViewer, single_pass_scan_operator.h:119-172).  For
// 8-byte types separate flag / partial / inclusive arrays with release /
// acquire on the flag (the reference's triple-buffer ScanTileStateViewer,
// :61-114).  Tile ids are taken from an atomic counter so that a tile only
// ever waits on tiles that are already running; waits are bounded.
#include "common.cuh"
#include "ops.cuh"
#include "scan.cuh"

namespace lcpp {
namespace scan {

struct Ctrl {
    uint32_t tile_counter;
    uint32_t error;
};

enum : uint32_t { kInvalid = 0, kPartial = 1, kInclusive = 2 };

__device__ __forceinline__ uint32_t ld_acquire(const uint32_t* p)
{
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release(uint32_t* p, uint32_t v)
{
    asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

template <typename T>
__device__ __forceinline__ uint64_t to_bits(T v)
{
    if constexpr (sizeof(T) == 4) {
        uint32_t b;
        memcpy(&b, &v, 4);
        return b;
    } else {
        uint64_t b;
        memcpy(&b, &v, 8);
        return b;
    }
}
template <typename T>
__device__ __forceinline__ T from_bits(uint64_t b)
{
    T v;
    if constexpr (sizeof(T) == 4) {
        const uint32_t b32 = uint32_t(b);
        memcpy(&v, &b32, 4);
    } else {
        memcpy(&v, &b, 8);
    }
    return v;
}

template <typename T, bool PACKED>
struct TileState;

template <typename T>
struct TileState<T, true> {
    uint64_t* words;
    __device__ __forceinline__ void publish(uint64_t tile, uint32_t flag, T v) const
    {
        st_relaxed(words + tile, (to_bits(v) << 32) | flag);
    }
    __device__ __forceinline__ uint32_t read(uint64_t tile, T& v) const
    {
        const uint64_t w = ld_relaxed(words + tile);
        v = from_bits<T>(w >> 32);
        return uint32_t(w);
    }
};

template <typename T>
struct TileState<T, false> {
    uint32_t* flags;
    uint64_t* partial;
    uint64_t* inclusive;
    __device__ __forceinline__ void publish(uint64_t tile, uint32_t flag, T v) const
    {
        st_relaxed((flag == kPartial ? partial : inclusive) + tile, to_bits(v));
        st_release(flags + tile, flag);
    }
    __device__ __forceinline__ uint32_t read(uint64_t tile, T& v) const
    {
        const uint32_t f = ld_acquire(flags + tile);
        if (f != kInvalid) v = from_bits<T>(ld_relaxed((f == kPartial ? partial : inclusive) + tile));
        return f;
    }
};

// A value paired with "is empty" so that the first inclusive element is never
// combined with a padding identity.
template <typename T>
struct Maybe {
    T v;
    bool has;
};
template <typename T, typename Op>
__device__ __forceinline__ Maybe<T> combine(Maybe<T> a, Maybe<T> b, Op op)
{
    if (!a.has) return b;
    if (!b.has) return a;
    return {op(a.v, b.v), true};
}

template <typename T>
struct VecOf;
template <> struct VecOf<uint32_t> { using type = uint4; };
template <> struct VecOf<int32_t> { using type = int4; };
template <> struct VecOf<float> { using type = float4; };
template <> struct VecOf<uint64_t> { using type = ulonglong2; };
template <> struct VecOf<int64_t> { using type = longlong2; };
template <> struct VecOf<double> { using type = double2; };

// MODE: 0 exclusive (with init), 1 inclusive, 2 inclusive with init.
template <typename T, typename Op, int MODE, int BLOCK, int CHUNKS, bool PACKED, bool VECTOR>
__global__ void __launch_bounds__(BLOCK)
scan_kernel(const T* in, T* out, uint64_t n, T init, TileState<T, PACKED> ts, Ctrl* ctrl)
{
    constexpr int VEC = 16 / sizeof(T);
    constexpr int WARPS = BLOCK / kWarp;
    constexpr int WARP_ITEMS = kWarp * VEC * CHUNKS;
    constexpr uint64_t TILE = uint64_t(WARPS) * WARP_ITEMS;
    using VT = typename VecOf<T>::type;
    static_assert(sizeof(VT) == 16, "16-byte vectors");

    __shared__ uint32_t s_tile;
    __shared__ T s_warp_total[WARPS];
    __shared__ T s_warp_excl[WARPS];
    __shared__ T s_tile_prefix;
    __shared__ int s_tile_has;

    const Op op;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if (tid == 0) s_tile = atomicAdd(&ctrl->tile_counter, 1u);
    __syncthreads();
    const uint64_t tile = s_tile;
    const uint64_t tile_base = tile * TILE;
    const bool full = tile_base + TILE <= n;
    const T ident = Identity<Op, T>::value();
    const uint64_t tbase = tile_base + uint64_t(warp) * WARP_ITEMS + uint64_t(lane) * VEC;

    T v[CHUNKS][VEC];
    if (VECTOR && full) {
#pragma unroll
        for (int j = 0; j < CHUNKS; ++j) {
            const VT x = *reinterpret_cast<const VT*>(in + tbase + j * kWarp * VEC);
            memcpy(&v[j][0], &x, 16);
        }
    } else {
#pragma unroll
        for (int j = 0; j < CHUNKS; ++j)
#pragma unroll
            for (int e = 0; e < VEC; ++e) {
                const uint64_t idx = tbase + j * kWarp * VEC + e;
                v[j][e] = idx < n ? in[idx] : ident;
            }
    }

    // Thread- and warp-level scans; pre[j] = prefix of chunk j's vector
    // within the warp segment.
    Maybe<T> pre[CHUNKS];
    Maybe<T> carry{ident, false};
#pragma unroll
    for (int j = 0; j < CHUNKS; ++j) {
#pragma unroll
        for (int e = 1; e < VEC; ++e) v[j][e] = op(v[j][e - 1], v[j][e]);
        const T incl = warp_inclusive_scan(v[j][VEC - 1], op);
        const T excl = shfl_up(incl, 1);
        pre[j] = combine(carry, Maybe<T>{excl, lane > 0}, op);
        carry = combine(carry, Maybe<T>{shfl_idx(incl, 31), true}, op);
    }
    if (lane == 0) s_warp_total[warp] = carry.v;
    __syncthreads();

    if (warp == 0) {
        // Block aggregate and exclusive prefix of each warp.
        const T x = lane < WARPS ? s_warp_total[lane] : ident;
        const T incl = warp_inclusive_scan(x, op);
        const T excl = shfl_up(incl, 1);
        if (lane < WARPS) s_warp_excl[lane] = excl;
        const T aggregate = shfl_idx(incl, WARPS - 1);

        Maybe<T> prefix{ident, false};
        if (tile == 0) {
            if (MODE != 1) prefix = {init, true};
            if (lane == 0) ts.publish(0, kInclusive, MODE != 1 ? op(init, aggregate) : aggregate);
        } else {
            if (lane == 0) ts.publish(tile, kPartial, aggregate);
            // Warp-wide look-back: lane l inspects tile (base - l).
            int64_t base = int64_t(tile) - 1;
            while (true) {
                const int64_t j = base - lane;
                T val = ident;
                uint32_t flag = kInclusive;  // lanes before tile 0 never count
                if (j >= 0) {
                    uint32_t spins = 0;
                    uint64_t t0 = 0;
                    while ((flag = ts.read(uint64_t(j), val)) == kInvalid) {
                        if (++spins == 64) {
                            spins = 0;
                            const uint64_t now = global_timer_ns();
                            if (t0 == 0) {
                                t0 = now;
                            } else if (now - t0 > kWaitLimitNs || error_raised(&ctrl->error)) {
                                report_error(&ctrl->error, kDevErrTimeout);
                                flag = kInclusive;
                                val = ident;
                                break;
                            }
                        }
                    }
                }
                const uint32_t inc_mask = __ballot_sync(0xffffffffu, flag == kInclusive);
                const int stop = inc_mask ? __ffs(inc_mask) - 1 : 31;
                const T window = warp_reduce(lane <= stop ? val : ident, op);
                prefix = combine(Maybe<T>{window, true}, prefix, op);
                if (inc_mask) break;
                base -= 32;
            }
            if (lane == 0) ts.publish(tile, kInclusive, op(prefix.v, aggregate));
        }
        if (lane == 0) {
            s_tile_prefix = prefix.v;
            s_tile_has = prefix.has;
        }
    }
    __syncthreads();

    const Maybe<T> warp_prefix =
        combine(Maybe<T>{s_tile_prefix, s_tile_has != 0}, Maybe<T>{s_warp_excl[warp], warp > 0}, op);
    T o[CHUNKS][VEC];
#pragma unroll
    for (int j = 0; j < CHUNKS; ++j) {
        const Maybe<T> p = combine(warp_prefix, pre[j], op);
        if (MODE == 0) {
            o[j][0] = p.v;  // exclusive scans always have a prefix (init)
#pragma unroll
            for (int e = 1; e < VEC; ++e) o[j][e] = op(p.v, v[j][e - 1]);
        } else {
#pragma unroll
            for (int e = 0; e < VEC; ++e) o[j][e] = p.has ? op(p.v, v[j][e]) : v[j][e];
        }
    }
    if (VECTOR && full) {
#pragma unroll
        for (int j = 0; j < CHUNKS; ++j) {
            VT x;
            memcpy(&x, &o[j][0], 16);
            *reinterpret_cast<VT*>(out + tbase + j * kWarp * VEC) = x;
        }
    } else {
#pragma unroll
        for (int j = 0; j < CHUNKS; ++j)
#pragma unroll
            for (int e = 0; e < VEC; ++e) {
                const uint64_t idx = tbase + j * kWarp * VEC + e;
                if (idx < n) out[idx] = o[j][e];
            }
    }
}

namespace {

constexpr int kBlock = 256;
template <typename T>
constexpr int chunks() { return sizeof(T) == 4 ? 8 : 8; }
template <typename T>
constexpr uint64_t tile_items() { return uint64_t(kBlock) * (16 / sizeof(T)) * chunks<T>(); }

struct Layout {
    size_t ctrl, flags, partial, inclusive, total;
    uint64_t tiles;
};

Layout make_layout(int tb, uint64_t n)
{
    Layout L{};
    const uint64_t tile = tb == 4 ? tile_items<uint32_t>() : tile_items<uint64_t>();
    L.tiles = ceil_div(n, tile);
    size_t off = 0;
    L.ctrl = off; off += kTempAlign;
    if (tb == 4) {
        L.flags = off; off = align_up(off + size_t(L.tiles) * 8, kTempAlign);  // packed words
        L.partial = L.inclusive = 0;
    } else {
        L.flags = off; off = align_up(off + size_t(L.tiles) * 4, kTempAlign);
        L.partial = off; off = align_up(off + size_t(L.tiles) * 8, kTempAlign);
        L.inclusive = off; off = align_up(off + size_t(L.tiles) * 8, kTempAlign);
    }
    L.total = off;
    return L;
}

template <typename T, typename Op, int MODE>
lcpp_status launch(unsigned char* temp, const Layout& L, const T* in, T* out, uint64_t n, T init,
                   cudaStream_t stream)
{
    constexpr bool PACKED = sizeof(T) == 4;
    constexpr int CH = chunks<T>();
    const size_t zero = (PACKED ? L.flags + size_t(L.tiles) * 8 : L.flags + size_t(L.tiles) * 4) - L.ctrl;
    LCPP_CUDA_TRY(cudaMemsetAsync(temp + L.ctrl, 0, zero, stream));
    Ctrl* ctrl = reinterpret_cast<Ctrl*>(temp + L.ctrl);
    TileState<T, PACKED> ts;
    if constexpr (PACKED) {
        ts.words = reinterpret_cast<uint64_t*>(temp + L.flags);
    } else {
        ts.flags = reinterpret_cast<uint32_t*>(temp + L.flags);
        ts.partial = reinterpret_cast<uint64_t*>(temp + L.partial);
        ts.inclusive = reinterpret_cast<uint64_t*>(temp + L.inclusive);
    }
    const bool aligned = ((reinterpret_cast<uintptr_t>(in) | reinterpret_cast<uintptr_t>(out)) & 15) == 0;
    const unsigned grid = unsigned(L.tiles);
    diag::KernelTimer timer(2 /* LCPP_KERNEL_SCAN */, n, stream);
    if (aligned)
        scan_kernel<T, Op, MODE, kBlock, CH, PACKED, true><<<grid, kBlock, 0, stream>>>(in, out, n, init, ts, ctrl);
    else
        scan_kernel<T, Op, MODE, kBlock, CH, PACKED, false><<<grid, kBlock, 0, stream>>>(in, out, n, init, ts, ctrl);
    return cudaGetLastError() == cudaSuccess ? LCPP_OK : LCPP_ERR_CUDA;
}

template <typename T, int MODE>
lcpp_status by_op(unsigned char* temp, const Layout& L, const void* in, void* out, uint64_t n,
                  lcpp_op op, const void* init, cudaStream_t stream)
{
    T init_v{};
    if (init) memcpy(&init_v, init, sizeof(T));
    const T* i = static_cast<const T*>(in);
    T* o = static_cast<T*>(out);
    switch (op) {
    case LCPP_OP_SUM: return launch<T, SumOp, MODE>(temp, L, i, o, n, init_v, stream);
    case LCPP_OP_MIN: return launch<T, MinOp, MODE>(temp, L, i, o, n, init_v, stream);
    case LCPP_OP_MAX: return launch<T, MaxOp, MODE>(temp, L, i, o, n, init_v, stream);
    default: return LCPP_ERR_UNSUPPORTED_DTYPE;
    }
}

template <int MODE>
lcpp_status by_type(unsigned char* temp, const Layout& L, const void* in, void* out, uint64_t n,
                    lcpp_op op, const void* init, lcpp_dtype dt, cudaStream_t stream)
{
    switch (dt) {
    case LCPP_I32: return by_op<int32_t, MODE>(temp, L, in, out, n, op, init, stream);
    case LCPP_U32: return by_op<uint32_t, MODE>(temp, L, in, out, n, op, init, stream);
    case LCPP_F32: return by_op<float, MODE>(temp, L, in, out, n, op, init, stream);
    case LCPP_I64: return by_op<int64_t, MODE>(temp, L, in, out, n, op, init, stream);
    case LCPP_U64: return by_op<uint64_t, MODE>(temp, L, in, out, n, op, init, stream);
    case LCPP_F64: return by_op<double, MODE>(temp, L, in, out, n, op, init, stream);
    default: return LCPP_ERR_UNSUPPORTED_DTYPE;
    }
}

}  // namespace

size_t temp_bytes(lcpp_dtype dt, uint64_t n)
{
    if (n == 0) return 0;
    return make_layout(dtype_bytes(dt), n).total;
}

lcpp_status run(void* temp, size_t temp_bytes_given, const void* in, void* out, uint64_t n,
                lcpp_op op, const void* init, lcpp_dtype dt, int mode, cudaStream_t stream)
{
    const int tb = dtype_bytes(dt);
    if (tb == 0) return LCPP_ERR_UNSUPPORTED_DTYPE;
    if (op != LCPP_OP_SUM && op != LCPP_OP_MIN && op != LCPP_OP_MAX) return LCPP_ERR_UNSUPPORTED_DTYPE;
    if (mode != 1 && !init) return LCPP_ERR_INVALID_ARG;
    if (n == 0) return LCPP_OK;
    if (!in || !out) return LCPP_ERR_INVALID_ARG;
    if ((reinterpret_cast<uintptr_t>(in) | reinterpret_cast<uintptr_t>(out)) % tb) return LCPP_ERR_INVALID_ARG;
    if (!temp || (reinterpret_cast<uintptr_t>(temp) & (kTempAlign - 1))) return LCPP_ERR_INVALID_ARG;
    const Layout L = make_layout(tb, n);
    if (temp_bytes_given < L.total) return LCPP_ERR_TEMP_TOO_SMALL;
    if (L.tiles > 0x7fffffffull) return LCPP_ERR_INVALID_ARG;
    unsigned char* t = static_cast<unsigned char*>(temp);
    switch (mode) {
    case 0: return by_type<0>(t, L, in, out, n, op, init, dt, stream);
    case 1: return by_type<1>(t, L, in, out, n, op, init, dt, stream);
    default: return by_type<2>(t, L, in, out, n, op, init, dt, stream);
    }
}

size_t error_word_offset() { return offsetof(Ctrl, error); }

}  // namespace scan
}  // namespace lcpp
