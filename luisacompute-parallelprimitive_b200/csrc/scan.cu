// scan.cu -- single-pass decoupled look-back scan for sm_100a.
//
// Replaces DeviceScan's CUDA path (src/lcpp/device/device_scan.h:606-697,
// details/scan.h:242-335, details/single_pass_scan_operator.h:119-332).
//
// Two kernels share the tile layout and the look-back: scan_bulk_kernel
// (persistent blocks, tiles brought into shared memory by bulk asynchronous
// copies several tiles ahead; used for 16-byte aligned data) and scan_kernel
// (one tile per block, loads straight into registers; any alignment).
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
#include <cstdlib>

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

// Exclusive prefix of `tile` (> 0) by decoupled look-back, run by one whole
// warp: lane l inspects tile base - l, so one round trip covers 32
// predecessors; the walk stops at the nearest tile that has published its
// inclusive prefix.  Every wait is bounded; on timeout the error is recorded
// and the walk stops.  (Wider windows, 64 or 128 tiles per round trip,
// measured slower on B200.)
template <typename T, typename Op, bool PACKED>
__device__ __forceinline__ T look_back(uint64_t tile, const TileState<T, PACKED>& ts, Ctrl* ctrl)
{
    const Op op;
    const int lane = threadIdx.x & 31;
    const T ident = Identity<Op, T>::value();
    Maybe<T> prefix{ident, false};
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
        if (inc_mask) return prefix.v;
        base -= 32;
    }
}

// Shared memory of one tile's block-level scan.
template <typename T, int WARPS>
struct BlockScanSmem {
    T warp_total[WARPS];
    T warp_excl[WARPS];
    T tile_prefix;
    int tile_has;
};

// Thread- and warp-level scans of one thread's CHUNKS x VEC items (in place,
// inclusive within each vector); pre[j] = prefix of chunk j's vector within
// the warp segment; returns the warp segment's total (valid in every lane).
template <typename T, typename Op, int CHUNKS, int VEC>
__device__ __forceinline__ T warp_segment_scan(T (&v)[CHUNKS][VEC], Maybe<T> (&pre)[CHUNKS], Op op)
{
    const int lane = threadIdx.x & 31;
    const T ident = Identity<Op, T>::value();
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
    return carry.v;
}

// Run by warp 0 after the warp totals are in shared memory: the block
// aggregate, each warp's exclusive prefix, and the tile's exclusive prefix
// from the decoupled look-back (lane l inspects tile base - l, so one round
// trip covers 32 predecessors).  Publishes the tile's partial and then
// inclusive status; writes the results to shared memory.
template <typename T, typename Op, int MODE, int WARPS, bool PACKED>
__device__ __forceinline__ void resolve_tile_prefix(uint64_t tile, T init, const TileState<T, PACKED>& ts,
                                                    Ctrl* ctrl, BlockScanSmem<T, WARPS>& sm)
{
    const Op op;
    const int lane = threadIdx.x & 31;
    const T ident = Identity<Op, T>::value();
    const T x = lane < WARPS ? sm.warp_total[lane] : ident;
    const T incl = warp_inclusive_scan(x, op);
    const T excl = shfl_up(incl, 1);
    if (lane < WARPS) sm.warp_excl[lane] = excl;
    const T aggregate = shfl_idx(incl, WARPS - 1);

    Maybe<T> prefix{ident, false};
    if (tile == 0) {
        if (MODE != 1) prefix = {init, true};
        if (lane == 0) ts.publish(0, kInclusive, MODE != 1 ? op(init, aggregate) : aggregate);
    } else {
        if (lane == 0) ts.publish(tile, kPartial, aggregate);
        prefix = {look_back<T, Op, PACKED>(tile, ts, ctrl), true};
        if (lane == 0) ts.publish(tile, kInclusive, op(prefix.v, aggregate));
    }
    if (lane == 0) {
        sm.tile_prefix = prefix.v;
        sm.tile_has = prefix.has;
    }
}

// Final values of one thread's items from the scanned vectors, the tile's
// exclusive prefix (`tile_has`: whether there is one) and the warp's
// exclusive prefix within the tile.
template <typename T, typename Op, int MODE, int CHUNKS, int VEC>
__device__ __forceinline__ void finish_items(const T (&v)[CHUNKS][VEC], const Maybe<T> (&pre)[CHUNKS], T tile_prefix,
                                             bool tile_has, T warp_excl, T (&o)[CHUNKS][VEC])
{
    const Op op;
    const int warp = threadIdx.x >> 5;
    const Maybe<T> warp_prefix = combine(Maybe<T>{tile_prefix, tile_has}, Maybe<T>{warp_excl, warp > 0}, op);
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
}

// Tile = BLOCK threads x CHUNKS x one 16-byte vector; warp w owns a
// contiguous segment, chunk j of lane l is the vector at
// segment + (j * 32 + l) * VEC.
template <typename T, int BLOCK, int CHUNKS>
struct TileShape {
    static constexpr int kVec = 16 / sizeof(T);
    static constexpr int kWarps = BLOCK / kWarp;
    static constexpr int kWarpItems = kWarp * kVec * CHUNKS;
    static constexpr uint64_t kTile = uint64_t(kWarps) * kWarpItems;
    __device__ static uint64_t thread_offset()
    {
        return uint64_t(threadIdx.x >> 5) * kWarpItems + uint64_t(threadIdx.x & 31) * kVec;
    }
};

template <typename T, int CHUNKS, int VEC>
__device__ __forceinline__ void load_guarded(const T* in, uint64_t n, uint64_t tbase, T ident, T (&v)[CHUNKS][VEC])
{
#pragma unroll
    for (int j = 0; j < CHUNKS; ++j)
#pragma unroll
        for (int e = 0; e < VEC; ++e) {
            const uint64_t idx = tbase + j * kWarp * VEC + e;
            v[j][e] = idx < n ? in[idx] : ident;
        }
}

template <typename T, int CHUNKS, int VEC>
__device__ __forceinline__ void store_items(T* out, uint64_t n, uint64_t tbase, bool vector, const T (&o)[CHUNKS][VEC])
{
    using VT = typename VecOf<T>::type;
    if (vector) {
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

// One tile per block, loads straight into registers (any alignment).
// MODE: 0 exclusive (with init), 1 inclusive, 2 inclusive with init.
template <typename T, typename Op, int MODE, int BLOCK, int CHUNKS, bool PACKED, bool VECTOR>
__global__ void __launch_bounds__(BLOCK)
scan_kernel(const T* in, T* out, uint64_t n, T init, const T* init_dev, TileState<T, PACKED> ts, Ctrl* ctrl)
{
    if (init_dev) init = *init_dev;  // initial value held in device memory
    using Shape = TileShape<T, BLOCK, CHUNKS>;
    constexpr int VEC = Shape::kVec;
    constexpr int WARPS = Shape::kWarps;
    using VT = typename VecOf<T>::type;
    static_assert(sizeof(VT) == 16, "16-byte vectors");

    __shared__ uint32_t s_tile;
    __shared__ BlockScanSmem<T, WARPS> sm;

    const Op op;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if (tid == 0) s_tile = atomicAdd(&ctrl->tile_counter, 1u);
    __syncthreads();
    const uint64_t tile = s_tile;
    const uint64_t tile_base = tile * Shape::kTile;
    const bool full = tile_base + Shape::kTile <= n;
    const T ident = Identity<Op, T>::value();
    const uint64_t tbase = tile_base + Shape::thread_offset();

    T v[CHUNKS][VEC];
    if (VECTOR && full) {
#pragma unroll
        for (int j = 0; j < CHUNKS; ++j) {
            const VT x = *reinterpret_cast<const VT*>(in + tbase + j * kWarp * VEC);
            memcpy(&v[j][0], &x, 16);
        }
    } else {
        load_guarded(in, n, tbase, ident, v);
    }

    Maybe<T> pre[CHUNKS];
    const T total = warp_segment_scan(v, pre, op);
    if (lane == 0) sm.warp_total[warp] = total;
    __syncthreads();
    if (warp == 0) resolve_tile_prefix<T, Op, MODE, WARPS, PACKED>(tile, init, ts, ctrl, sm);
    __syncthreads();

    T o[CHUNKS][VEC];
    finish_items<T, Op, MODE>(v, pre, sm.tile_prefix, sm.tile_has != 0, sm.warp_excl[warp], o);
    store_items(out, n, tbase, VECTOR && full, o);
}

// ---------------------------------------------------------------------------
// Persistent variant for 16-byte aligned input and output: each block keeps
// STAGES tiles in flight in shared memory, filled by bulk asynchronous copies
// (cp.async.bulk, completion on an mbarrier), so that the loads of the next
// tiles proceed while the block waits for the look-back of the current one.
// Tile ids still come from the atomic counter, in increasing order per
// block, so the smallest unfinished tile is always one a block is working
// on and only waits on finished or running tiles.  The last (partial) tile is
// loaded with guarded plain loads.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count)
{
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(uint32_t(__cvta_generic_to_shared(bar))),
                 "r"(count)
                 : "memory");
}

__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar)
{
    const uint32_t b = uint32_t(__cvta_generic_to_shared(bar));
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(b), "r"(bytes) : "memory");
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            uint32_t(__cvta_generic_to_shared(dst))),
        "l"(src), "r"(bytes), "r"(b)
        : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity)
{
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(uint32_t(__cvta_generic_to_shared(bar))), "r"(parity)
        : "memory");
    return done != 0;
}

// Bounded wait for phase `parity` of `bar`; false on timeout, or as soon as
// `error` (when given) reports an error.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, const uint32_t* error = nullptr)
{
    uint64_t t0 = 0;
    uint32_t spins = 0;
    while (!mbar_try_wait(bar, parity)) {
        if (++spins == 16) {
            spins = 0;
            if (error && error_raised(error)) return false;
            const uint64_t now = global_timer_ns();
            if (t0 == 0)
                t0 = now;
            else if (now - t0 > kWaitLimitNs)
                return false;
        }
    }
    return true;
}

// Per stage: the tile's block-level results between its two phases.
template <typename T, int WARPS>
struct StageSmem {
    T warp_total[WARPS];
    T warp_excl[WARPS];
    T aggregate;
    T tile_prefix;
    int tile_has;
};

// Pipelined persistent scan.  Iteration k of a block, with tiles k, k+1, ...
// in its stages:
//   A(k+1): reduce tile k+1 as soon as its data is in, publish its partial
//           aggregate (so that no later tile's look-back waits for a tile that
//           is merely queued behind this block's current one);
//   look-back of tile k (warp 0), publish its inclusive prefix;
//   B(k):   scan tile k from shared memory again, add the prefix, store;
//   refill tile k's stage with the next tile id (STAGES - 1 tiles ahead).
template <typename T, typename Op, int MODE, int BLOCK, int CHUNKS, bool PACKED, int STAGES>
__global__ void __launch_bounds__(BLOCK)
scan_bulk_kernel(const T* in, T* out, uint64_t n, uint64_t tiles, T init, const T* init_dev, TileState<T, PACKED> ts,
                 Ctrl* ctrl)
{
    if (init_dev) init = *init_dev;  // initial value held in device memory
    using Shape = TileShape<T, BLOCK, CHUNKS>;
    constexpr int VEC = Shape::kVec;
    constexpr int WARPS = Shape::kWarps;
    constexpr uint64_t TILE = Shape::kTile;
    constexpr uint32_t kTileBytes = uint32_t(TILE * sizeof(T));
    using VT = typename VecOf<T>::type;
    // three or more: a stage is refilled while the next two are read
    static_assert(STAGES >= 3 && STAGES <= 8, "stages");

    extern __shared__ __align__(128) unsigned char smem_raw[];
    T* stage_buf = reinterpret_cast<T*>(smem_raw);  // [STAGES][TILE]
    __shared__ __align__(8) uint64_t s_bar[STAGES];
    __shared__ uint64_t s_tile[STAGES];
    __shared__ uint32_t s_pending;  // bit s: a bulk copy into stage s is in flight
    __shared__ uint32_t s_phase;    // bit s: parity of the next completion of stage s
    __shared__ StageSmem<T, WARPS> sm[STAGES];

    const Op op;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const T ident = Identity<Op, T>::value();
    const uint64_t toff = Shape::thread_offset();

    // Takes the next tile id for stage st and starts its copy if it is full
    // (thread 0 only).  After an error no new copies start and the block
    // winds down.
    auto acquire = [&](int st) {
        if (error_raised(&ctrl->error)) {
            s_tile[st] = tiles;
            return;
        }
        const uint64_t t = atomicAdd(&ctrl->tile_counter, 1u);
        s_tile[st] = t;
        if (t < tiles && (t + 1) * TILE <= n) {
            s_pending |= 1u << st;
            bulk_load(stage_buf + size_t(st) * TILE, in + t * TILE, kTileBytes, &s_bar[st]);
        }
    };
    // After the barrier that follows the wait for stage st's copy (thread 0):
    // the copy has landed unless a wait timed out (then the error is set and
    // the bit stays pending, with the parity of the copy still in flight).
    auto retire = [&](int st) {
        if (((s_pending >> st) & 1u) && !error_raised(&ctrl->error)) {
            s_phase ^= 1u << st;
            s_pending &= ~(1u << st);
        }
    };

    // This thread's items of the tile in stage st: from shared memory for a
    // full tile (waiting for its copy the first time, `wait`), else guarded
    // loads from global memory.
    auto load = [&](int st, uint64_t tile, bool wait, T(&v)[CHUNKS][VEC]) {
        const uint64_t tile_base = tile * TILE;
        if (tile_base + TILE <= n) {
            if (wait) {
                const uint32_t parity = (s_phase >> st) & 1u;
                if (!mbar_wait(&s_bar[st], parity)) report_error(&ctrl->error, kDevErrTimeout);
            }
            const T* src = stage_buf + size_t(st) * TILE + toff;
#pragma unroll
            for (int j = 0; j < CHUNKS; ++j) {
                const VT x = *reinterpret_cast<const VT*>(src + j * kWarp * VEC);
                memcpy(&v[j][0], &x, 16);
            }
        } else {
            load_guarded(in, n, tile_base + toff, ident, v);
        }
    };

    // Phase A of the tile in stage st: warp totals (all threads), then
    // (warp 0, after a barrier) the aggregate and its partial status.
    auto phase_a_totals = [&](int st, uint64_t tile) {
        T v[CHUNKS][VEC];
        load(st, tile, true, v);
        T acc = v[0][0];
#pragma unroll
        for (int j = 0; j < CHUNKS; ++j)
#pragma unroll
            for (int e = 0; e < VEC; ++e)
                if (j + e > 0) acc = op(acc, v[j][e]);
        acc = warp_reduce(acc, op);
        if (lane == 0) sm[st].warp_total[warp] = acc;
    };
    auto phase_a_publish = [&](int st, uint64_t tile) {  // warp 0
        const T x = lane < WARPS ? sm[st].warp_total[lane] : ident;
        const T incl = warp_inclusive_scan(x, op);
        const T excl = shfl_up(incl, 1);
        if (lane < WARPS) sm[st].warp_excl[lane] = excl;
        const T aggregate = shfl_idx(incl, WARPS - 1);
        if (lane == 0) {
            sm[st].aggregate = aggregate;
            if (tile == 0)
                ts.publish(0, kInclusive, MODE != 1 ? op(init, aggregate) : aggregate);
            else
                ts.publish(tile, kPartial, aggregate);
        }
    };

    if (tid == 0) {
        s_pending = 0;
        s_phase = 0;
        for (int st = 0; st < STAGES; ++st) mbar_init(&s_bar[st], 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        for (int st = 0; st < STAGES; ++st) acquire(st);
    }
    __syncthreads();
    if (s_tile[0] < tiles) phase_a_totals(0, s_tile[0]);
    __syncthreads();
    if (tid == 0) retire(0);
    if (warp == 0 && s_tile[0] < tiles) phase_a_publish(0, s_tile[0]);

    for (uint32_t k = 0;; ++k) {
        const int st = int(k % STAGES);
        const int nst = int((k + 1) % STAGES);
        const uint64_t tile = s_tile[st];
        if (tile >= tiles) break;
        const uint64_t next = s_tile[nst];

        if (next < tiles) phase_a_totals(nst, next);
        __syncthreads();  // (1) warp totals of tile k+1 visible; stage phases read
        if (warp == 0) {
            if (lane == 0) retire(nst);
            if (next < tiles) phase_a_publish(nst, next);
            // look-back of tile k
            Maybe<T> prefix{ident, false};
            if (tile == 0) {
                if (MODE != 1) prefix = {init, true};
            } else {
                prefix = {look_back<T, Op, PACKED>(tile, ts, ctrl), true};
                if (lane == 0) ts.publish(tile, kInclusive, op(prefix.v, sm[st].aggregate));
            }
            if (lane == 0) {
                sm[st].tile_prefix = prefix.v;
                sm[st].tile_has = prefix.has;
            }
        }
        __syncthreads();  // (2) prefix of tile k visible

        {
            T v[CHUNKS][VEC];
            load(st, tile, false, v);
            Maybe<T> pre[CHUNKS];
            warp_segment_scan(v, pre, op);
            T o[CHUNKS][VEC];
            finish_items<T, Op, MODE>(v, pre, sm[st].tile_prefix, sm[st].tile_has != 0, sm[st].warp_excl[warp], o);
            store_items(out, n, tile * TILE + toff, tile * TILE + TILE <= n, o);
        }
        __syncthreads();  // (3) stage st and sm[st] are free
        if (tid == 0) {
            // the stage's generic-proxy reads are ordered before the
            // asynchronous copy that refills it
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            acquire(st);
        }
    }

    // Copies not retired (only after an error): wait for them, again
    // bounded, before the block's shared memory goes away.
    if (tid == 0 && s_pending) {
        for (int st = 0; st < STAGES; ++st)
            if ((s_pending >> st) & 1u) {
                if (!mbar_wait(&s_bar[st], (s_phase >> st) & 1u)) report_error(&ctrl->error, kDevErrTimeout);
            }
    }
}

namespace {

constexpr int kBlock = 256;

// Tile = kBlock threads x kChunks x one 16-byte vector (16 KB: 4096 4-byte
// or 2048 8-byte items).  16 KB tiles with three stages (four blocks per SM)
// measured faster on B200 than 32 KB tiles (two blocks per SM), four stages,
// or a dedicated look-back warp.
constexpr int kChunks = 4;
constexpr int kStages = 3;

uint64_t tile_items(int tb) { return uint64_t(kBlock) * uint64_t(16 / tb) * kChunks; }

struct Layout {
    size_t ctrl, flags, partial, inclusive, total;
    uint64_t tiles;
};

Layout make_layout(int tb, uint64_t n)
{
    Layout L{};
    L.tiles = ceil_div(n, tile_items(tb));
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

template <typename T, typename Op, int MODE, bool PACKED>
void launch_kernel(const T* in, T* out, uint64_t n, uint64_t tiles, T init, const T* init_dev,
                   const TileState<T, PACKED>& ts, Ctrl* ctrl, bool aligned, cudaStream_t stream)
{
    // 16-byte aligned input and output: the persistent bulk-copy kernel;
    // otherwise one tile per block with register loads.
    if (aligned) {
        auto kernel = scan_bulk_kernel<T, Op, MODE, kBlock, kChunks, PACKED, kStages>;
        constexpr size_t smem = size_t(kStages) * kBlock * 16 * kChunks;
        set_max_dynamic_smem(reinterpret_cast<const void*>(kernel), smem);
        const uint64_t resident =
            uint64_t(device_sm_count()) * resident_blocks(reinterpret_cast<const void*>(kernel), kBlock, smem);
        const unsigned grid = unsigned(tiles < resident ? tiles : resident);
        kernel<<<grid, kBlock, smem, stream>>>(in, out, n, tiles, init, init_dev, ts, ctrl);
    } else {
        scan_kernel<T, Op, MODE, kBlock, kChunks, PACKED, false><<<unsigned(tiles), kBlock, 0, stream>>>(
            in, out, n, init, init_dev, ts, ctrl);
    }
}

template <typename T, typename Op, int MODE>
lcpp_status launch(unsigned char* temp, const Layout& L, const T* in, T* out, uint64_t n, T init,
                   const T* init_dev, cudaStream_t stream)
{
    constexpr bool PACKED = sizeof(T) == 4;
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
    diag::KernelTimer timer(2 /* LCPP_KERNEL_SCAN */, n, stream);
    launch_kernel<T, Op, MODE>(in, out, n, L.tiles, init, init_dev, ts, ctrl, aligned, stream);
    return cudaGetLastError() == cudaSuccess ? LCPP_OK : LCPP_ERR_CUDA;
}

template <typename T, int MODE>
lcpp_status by_op(unsigned char* temp, const Layout& L, const void* in, void* out, uint64_t n,
                  lcpp_op op, const void* init, const void* init_dev, cudaStream_t stream)
{
    T init_v{};
    if (init) memcpy(&init_v, init, sizeof(T));
    const T* i = static_cast<const T*>(in);
    T* o = static_cast<T*>(out);
    const T* id = static_cast<const T*>(init_dev);
    switch (op) {
    case LCPP_OP_SUM: return launch<T, SumOp, MODE>(temp, L, i, o, n, init_v, id, stream);
    case LCPP_OP_MIN: return launch<T, MinOp, MODE>(temp, L, i, o, n, init_v, id, stream);
    case LCPP_OP_MAX: return launch<T, MaxOp, MODE>(temp, L, i, o, n, init_v, id, stream);
    default: return LCPP_ERR_UNSUPPORTED_DTYPE;
    }
}

template <int MODE>
lcpp_status by_type(unsigned char* temp, const Layout& L, const void* in, void* out, uint64_t n,
                    lcpp_op op, const void* init, const void* init_dev, lcpp_dtype dt, cudaStream_t stream)
{
    switch (dt) {
    case LCPP_I32: return by_op<int32_t, MODE>(temp, L, in, out, n, op, init, init_dev, stream);
    case LCPP_U32: return by_op<uint32_t, MODE>(temp, L, in, out, n, op, init, init_dev, stream);
    case LCPP_F32: return by_op<float, MODE>(temp, L, in, out, n, op, init, init_dev, stream);
    case LCPP_I64: return by_op<int64_t, MODE>(temp, L, in, out, n, op, init, init_dev, stream);
    case LCPP_U64: return by_op<uint64_t, MODE>(temp, L, in, out, n, op, init, init_dev, stream);
    case LCPP_F64: return by_op<double, MODE>(temp, L, in, out, n, op, init, init_dev, stream);
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
    return run_with_init(temp, temp_bytes_given, in, out, n, op, init, nullptr, dt, mode, stream);
}

lcpp_status run_with_init(void* temp, size_t temp_bytes_given, const void* in, void* out, uint64_t n, lcpp_op op,
                          const void* init, const void* init_dev, lcpp_dtype dt, int mode, cudaStream_t stream)
{
    diag::Range nvtx_range("lcpp DeviceScan");
    const int tb = dtype_bytes(dt);
    if (tb == 0) return LCPP_ERR_UNSUPPORTED_DTYPE;
    if (op != LCPP_OP_SUM && op != LCPP_OP_MIN && op != LCPP_OP_MAX) return LCPP_ERR_UNSUPPORTED_DTYPE;
    if (mode != 1 && !init && !init_dev) return LCPP_ERR_INVALID_ARG;
    if (n == 0) return LCPP_OK;
    if (init_dev && reinterpret_cast<uintptr_t>(init_dev) % tb) return LCPP_ERR_INVALID_ARG;
    if (!in || !out) return LCPP_ERR_INVALID_ARG;
    if ((reinterpret_cast<uintptr_t>(in) | reinterpret_cast<uintptr_t>(out)) % tb) return LCPP_ERR_INVALID_ARG;
    if (!temp || (reinterpret_cast<uintptr_t>(temp) & (kTempAlign - 1))) return LCPP_ERR_INVALID_ARG;
    const Layout L = make_layout(tb, n);
    if (temp_bytes_given < L.total) return LCPP_ERR_TEMP_TOO_SMALL;
    if (L.tiles > 0x7fffffffull) return LCPP_ERR_INVALID_ARG;
    unsigned char* t = static_cast<unsigned char*>(temp);
    switch (mode) {
    case 0: return by_type<0>(t, L, in, out, n, op, init, init_dev, dt, stream);
    case 1: return by_type<1>(t, L, in, out, n, op, init, init_dev, dt, stream);
    default: return by_type<2>(t, L, in, out, n, op, init, init_dev, dt, stream);
    }
}

size_t error_word_offset() { return offsetof(Ctrl, error); }

}  // namespace scan
}  // namespace lcpp
