// radix_sort.cu -- onesweep LSD radix sort for sm_100a.
//
// Replaces DeviceRadixSort (src/lcpp/device/device_radix_sort.h) of the
// reference.  One call runs:
//   1. cudaMemsetAsync of the control block, histograms and the pass-0
//      look-back rows;
//   2. histogram_kernel: ONE read of the keys produces the 256-bin digit
//      histograms of every pass (the reference's AgentRadixSortHistogram,
//      src/lcpp/agent/agent_radix_sort_histogram.h:116-187); the last block to
//      finish turns them into exclusive digit offsets (the reference runs a
//      separate RadixSortExclusiveSumModule, details/radix_sort.h:81-123);
//   3. one onesweep_kernel per 8-bit pass: load a tile, rank it stably with
//      warp match-any and per-warp shared-memory counters, publish per-digit
//      tile counts, resolve the global digit offsets with a bounded decoupled
//      look-back, stage the tile in shared memory in digit order and write it
//      out so that each digit's run is stored contiguously (the reference's
//      AgentRadixSortOneSweep, agent_radix_sort_onesweep.h:224-511, with
//      BlockRadixRankMatchEarlyCounts, block_radix_rank.h:207-486).
//
// Differences from the reference that are part of this design:
//  - look-back status rows are double-buffered and each pass clears the rows
//    the next pass will use, instead of a separate reset kernel per pass and
//    portion (device_radix_sort.h:1389-1398);
//  - one portion at any size: counts and offsets are 64-bit above 2^30 keys
//    (the reference splits at 2^28 keys into portions, :1056, and its
//    portion carry is never written, agent_radix_sort_onesweep.h:362);
//  - every spin is bounded (kWaitLimitNs) and reports LCPP_ERR_LOOKBACK_TIMEOUT.
#include <mutex>

#include "common.cuh"
#include "radix_sort.cuh"

namespace lcpp {
namespace radix {

// ---------------------------------------------------------------------------
// Status words of the per-digit decoupled look-back.  One word per
// (tile, digit): two flag bits and the count, so a single relaxed load sees a
// consistent {flag, value} pair.  0 means "not published yet".
// ---------------------------------------------------------------------------
template <typename ST>
struct StatusBits;
template <>
struct StatusBits<uint32_t> {
    static constexpr uint32_t kPartial = 1u << 30;
    static constexpr uint32_t kInclusive = 1u << 31;
    static constexpr uint32_t kFlags = kPartial | kInclusive;
    static constexpr uint32_t kValue = kPartial - 1u;
};
template <>
struct StatusBits<uint64_t> {
    static constexpr uint64_t kPartial = 1ull << 62;
    static constexpr uint64_t kInclusive = 1ull << 63;
    static constexpr uint64_t kFlags = kPartial | kInclusive;
    static constexpr uint64_t kValue = kPartial - 1ull;
};

struct Ctrl {
    uint32_t hist_done;
    uint32_t error;
    uint32_t tile_counter[kMaxPasses];
};
static_assert(sizeof(Ctrl) <= 256, "control block must fit 256 bytes");

// Exclusive scan of one value per thread over threads [0, 256) of a block of
// BLOCK >= 256 threads.  Every thread of the block must call it.
template <typename T, int BLOCK>
__device__ __forceinline__ T exclusive_scan_256(T v, T* s_warp_sums)
{
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    T incl = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        T y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
    }
    if (lane == 31 && warp < 8) s_warp_sums[warp] = incl;
    __syncthreads();
    T base = 0;
#pragma unroll
    for (int w = 0; w < 8; ++w)
        if (w < warp) base += s_warp_sums[w];
    __syncthreads();
    return base + incl - v;
}

// ---------------------------------------------------------------------------
// Histogram of every pass in one read.
// Shared counters are replicated COPIES times and lane i uses copy i % COPIES,
// which bounds same-address conflicts of a warp's shared atomics to
// 32 / COPIES even when every key has the same digit.
// ---------------------------------------------------------------------------
template <typename U, int BLOCK, int COPIES, bool VECTOR>
__global__ void __launch_bounds__(BLOCK)
histogram_kernel(const U* __restrict__ keys, uint64_t n, KeyCodec<U> codec, int begin_bit,
                 int end_bit, int passes, uint64_t chunk, Ctrl* ctrl,
                 unsigned long long* __restrict__ g_hist, unsigned long long* __restrict__ g_bins)
{
    extern __shared__ __align__(16) uint32_t s_hist[];  // [passes * 256][COPIES]
    __shared__ unsigned long long s_sums[8];
    __shared__ int s_last;
    const int tid = threadIdx.x;
    const int copy = (tid & 31) % COPIES;
    for (int i = tid; i < passes * kDigits * COPIES; i += BLOCK) s_hist[i] = 0;
    __syncthreads();

    auto count = [&](U k) {
        const U t = transform_key(k, codec);
#pragma unroll
        for (int p = 0; p < kMaxPasses; ++p) {
            if (p < passes) {
                const int shift = begin_bit + kRadixBits * p;
                const int nb = min(kRadixBits, end_bit - shift);
                const uint32_t d = uint32_t(t >> shift) & ((1u << nb) - 1u);
                atomicAdd(&s_hist[(p * kDigits + d) * COPIES + copy], 1u);
            }
        }
    };

    const uint64_t lo = uint64_t(blockIdx.x) * chunk;
    const uint64_t hi = min(lo + chunk, n);
    if (lo < hi) {
        if constexpr (VECTOR) {
            constexpr int VEC = 16 / sizeof(U);
            using V = typename std::conditional<sizeof(U) == 4, uint4, ulonglong2>::type;
            const uint64_t nvec = (hi - lo) / VEC;
            const V* vp = reinterpret_cast<const V*>(keys + lo);
            uint64_t j = tid;
            for (; j + 3 * BLOCK < nvec; j += 4 * BLOCK) {
                V a = vp[j], b = vp[j + BLOCK], c = vp[j + 2 * BLOCK], d = vp[j + 3 * BLOCK];
                const U* pa = reinterpret_cast<const U*>(&a);
                const U* pb = reinterpret_cast<const U*>(&b);
                const U* pc = reinterpret_cast<const U*>(&c);
                const U* pd = reinterpret_cast<const U*>(&d);
#pragma unroll
                for (int e = 0; e < VEC; ++e) { count(pa[e]); count(pb[e]); count(pc[e]); count(pd[e]); }
            }
            for (; j < nvec; j += BLOCK) {
                V a = vp[j];
                const U* pa = reinterpret_cast<const U*>(&a);
#pragma unroll
                for (int e = 0; e < VEC; ++e) count(pa[e]);
            }
            for (uint64_t i = lo + nvec * VEC + tid; i < hi; i += BLOCK) count(keys[i]);
        } else {
            for (uint64_t i = lo + tid; i < hi; i += BLOCK) count(keys[i]);
        }
    }
    __syncthreads();
    for (int i = tid; i < passes * kDigits; i += BLOCK) {
        uint32_t s = 0;
#pragma unroll
        for (int c = 0; c < COPIES; ++c) s += s_hist[i * COPIES + c];
        if (s) atomicAdd(&g_hist[i], (unsigned long long)s);
    }
    __threadfence();
    __syncthreads();
    if (tid == 0) s_last = atomicAdd(&ctrl->hist_done, 1u) == gridDim.x - 1;
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    // Last block: exclusive digit offsets of every pass.
    for (int p = 0; p < passes; ++p) {
        const unsigned long long v = tid < kDigits ? __ldcg(&g_hist[p * kDigits + tid]) : 0ull;
        const unsigned long long ex = exclusive_scan_256<unsigned long long, BLOCK>(v, s_sums);
        if (tid < kDigits) g_bins[p * kDigits + tid] = ex;
    }
}

// ---------------------------------------------------------------------------
// One onesweep pass.
// ---------------------------------------------------------------------------
template <typename U, typename V, typename ST, typename OffT>
struct OnesweepArgs {
    const U* keys_in;
    U* keys_out;
    const V* vals_in;
    V* vals_out;
    uint64_t n;
    KeyCodec<U> codec;
    int shift;
    int nbits;
    const unsigned long long* bins;  // [256] exclusive global digit offsets of this pass
    ST* status;                      // [tiles][256] look-back rows of this pass
    ST* status_next;                 // rows the next pass uses (cleared here), or null
    uint32_t* tile_counter;
    uint32_t* error;
};

template <typename U, typename V, bool PAIRS, int BLOCK, int ITEMS, typename OffT>
struct OnesweepSmem {
    static constexpr int kTile = BLOCK * ITEMS;
    static constexpr int kWarps = BLOCK / kWarp;
    union {
        U keys[kTile];
        uint32_t counters[kWarps * kDigits];  // per-warp digit counters while ranking
    } u;
    V vals[PAIRS ? kTile : 1];
    uint32_t digit_start[kDigits];  // first tile position of each digit
    OffT gofs[kDigits];             // output index = gofs[digit] + tile position
    uint32_t warp_sums[8];
    uint32_t tile_id;
};

template <typename U, typename V, bool PAIRS, int BLOCK, int ITEMS, typename ST, typename OffT>
__global__ void __launch_bounds__(BLOCK)
onesweep_kernel(OnesweepArgs<U, V, ST, OffT> a)
{
    using Smem = OnesweepSmem<U, V, PAIRS, BLOCK, ITEMS, OffT>;
    using SB = StatusBits<ST>;
    constexpr int kTile = Smem::kTile;
    constexpr int kWarps = Smem::kWarps;
    static_assert(BLOCK >= kDigits, "one thread per digit");
    static_assert(kTile <= 65536, "tile positions are packed in 16 bits");
    static_assert(sizeof(U) * kTile >= sizeof(uint32_t) * kWarps * kDigits, "counter overlay");
    extern __shared__ __align__(16) unsigned char smem_raw[];
    Smem& s = *reinterpret_cast<Smem*>(smem_raw);

    const int tid = threadIdx.x;
    const int lane = tid & 31;
    const int warp = tid >> 5;

    if (tid == 0) s.tile_id = atomicAdd(a.tile_counter, 1u);
    for (int i = tid; i < kWarps * kDigits; i += BLOCK) s.u.counters[i] = 0;
    __syncthreads();
    const uint32_t tile = s.tile_id;
    const uint64_t tile_base = uint64_t(tile) * kTile;
    const int valid = int(a.n - tile_base < uint64_t(kTile) ? a.n - tile_base : uint64_t(kTile));
    const uint32_t max_digit = (1u << a.nbits) - 1u;

    // Warp-striped load: warp w owns positions [w*ITEMS*32, (w+1)*ITEMS*32) of
    // the tile, slot i of lane l is position w*ITEMS*32 + i*32 + l.
    U keys[ITEMS];
    V vals[PAIRS ? ITEMS : 1];
    uint32_t packed[ITEMS];
    const int warp_base = warp * ITEMS * kWarp + lane;
#pragma unroll
    for (int i = 0; i < ITEMS; ++i) {
        const int pos = warp_base + i * kWarp;
        keys[i] = pos < valid ? a.keys_in[tile_base + pos] : U(0);
    }
    if constexpr (PAIRS) {
#pragma unroll
        for (int i = 0; i < ITEMS; ++i) {
            const int pos = warp_base + i * kWarp;
            vals[i] = pos < valid ? a.vals_in[tile_base + pos] : V(0);
        }
    }

    // Stable in-warp ranking: keys of one slot are ranked in lane order among
    // equal digits, slots in order; the digit's leader lane bumps the warp's
    // shared counter by the number of peers.
    const uint32_t lt = lanemask_lt();
    uint32_t* my_counters = s.u.counters + warp * kDigits;
#pragma unroll
    for (int i = 0; i < ITEMS; ++i) {
        const int pos = warp_base + i * kWarp;
        const uint32_t d =
            pos < valid ? uint32_t(transform_key(keys[i], a.codec) >> a.shift) & max_digit : max_digit;
        const uint32_t peers = __match_any_sync(0xffffffffu, d);
        const int leader = 31 - __clz(peers);
        uint32_t base = 0;
        if (lane == leader) base = atomicAdd(&my_counters[d], uint32_t(__popc(peers)));
        base = __shfl_sync(0xffffffffu, base, leader);
        packed[i] = (d << 16) | (base + __popc(peers & lt));
    }
    __syncthreads();

    // Per digit: exclusive prefix over warps, tile total, early publication.
    uint32_t total = 0;
    if (tid < kDigits) {
#pragma unroll
        for (int w = 0; w < kWarps; ++w) {
            const uint32_t c = s.u.counters[w * kDigits + tid];
            s.u.counters[w * kDigits + tid] = total;
            total += c;
        }
        ST* mine = a.status + uint64_t(tile) * kDigits + tid;
        st_relaxed(mine, ST(total) | (tile == 0 ? SB::kInclusive : SB::kPartial));
    }
    const uint32_t dstart = exclusive_scan_256<uint32_t, BLOCK>(total, s.warp_sums);
    if (tid < kDigits) s.digit_start[tid] = dstart;
    __syncthreads();

    // Tile rank = digit start + earlier warps' count of the digit + in-warp rank.
#pragma unroll
    for (int i = 0; i < ITEMS; ++i) {
        const uint32_t d = packed[i] >> 16;
        packed[i] = s.digit_start[d] + s.u.counters[warp * kDigits + d] + (packed[i] & 0xffffu);
    }
    __syncthreads();  // counters are dead; the key tile reuses their storage

    // Decoupled look-back, one digit per thread.
    if (tid < kDigits) {
        OffT prefix = 0;
        if (tile > 0) {
            int64_t j = int64_t(tile) - 1;
            uint32_t spins = 0;
            uint64_t t0 = 0;
            while (true) {
                const ST w = ld_relaxed(a.status + uint64_t(j) * kDigits + tid);
                if ((w & SB::kFlags) == 0) {
                    if (++spins == 64) {
                        spins = 0;
                        const uint64_t now = global_timer_ns();
                        if (t0 == 0) {
                            t0 = now;
                        } else if (now - t0 > kWaitLimitNs) {
                            report_error(a.error, kDevErrTimeout);
                            break;
                        }
                        if (error_raised(a.error)) break;  // another waiter gave up
                    }
                    continue;
                }
                prefix += OffT(w & SB::kValue);
                if ((w & SB::kInclusive) || j == 0) break;
                --j;
            }
            st_relaxed(a.status + uint64_t(tile) * kDigits + tid,
                       ST(prefix + total) | SB::kInclusive);
        }
        s.gofs[tid] = OffT(a.bins[tid]) + prefix - OffT(dstart);
        if (a.status_next) a.status_next[uint64_t(tile) * kDigits + tid] = 0;
    }

    // Tile ranks are a permutation of [0, kTile) by construction; the check
    // turns a broken invariant into an error code instead of a wild write.
    bool rank_ok = true;
#pragma unroll
    for (int i = 0; i < ITEMS; ++i) rank_ok &= packed[i] < uint32_t(kTile);
    if (rank_ok) {
#pragma unroll
        for (int i = 0; i < ITEMS; ++i) s.u.keys[packed[i]] = keys[i];
        if constexpr (PAIRS) {
#pragma unroll
            for (int i = 0; i < ITEMS; ++i) s.vals[packed[i]] = vals[i];
        }
    } else {
        report_error(a.error, kDevErrInternal);
    }
    __syncthreads();

    // Digit-ordered tile -> global: consecutive threads write consecutive
    // positions of one digit run.
#pragma unroll
    for (int i = 0; i < ITEMS; ++i) {
        const int idx = i * BLOCK + tid;
        if (idx < valid) {
            const U k = s.u.keys[idx];
            const uint32_t d = uint32_t(transform_key(k, a.codec) >> a.shift) & max_digit;
            const OffT pos = s.gofs[d] + OffT(idx);
            if (uint64_t(pos) < a.n) {  // always true when the offsets are consistent
                a.keys_out[pos] = k;
                if constexpr (PAIRS) a.vals_out[pos] = s.vals[idx];
            } else {
                report_error(a.error, kDevErrInternal);
            }
        }
    }
}

// ---------------------------------------------------------------------------
// Host side.
// ---------------------------------------------------------------------------
namespace {

// Tile geometry per (key bytes, value bytes).
struct Geometry {
    int block;
    int items;
    int tile() const { return block * items; }
};

Geometry geometry(int kb, int vb)
{
    if (kb == 4 && vb == 0) return {384, 20};
    if (kb == 4 && vb == 4) return {384, 15};
    if (kb == 4 && vb == 8) return {256, 16};
    if (kb == 8 && vb == 0) return {256, 16};
    if (kb == 8 && vb == 4) return {256, 14};
    return {256, 12};  // 8-byte keys, 8-byte values
}

constexpr int kHistBlock = 512;

int hist_copies(int kb) { return kb == 4 ? 8 : 4; }

struct Layout {
    size_t ctrl, hist, bins, status_a, status_b, keys_alt, vals_alt, total;
    size_t status_bytes;  // per buffer
    uint64_t tiles;
    bool wide;
};

Layout make_layout(int kb, int vb, uint64_t n)
{
    Layout L{};
    const Geometry g = geometry(kb, vb);
    L.wide = n >= (1ull << 30);
    L.tiles = ceil_div(n, uint64_t(g.tile()));
    const size_t st = L.wide ? 8 : 4;
    const int max_passes = kb;  // 8-bit passes over the full key width
    size_t off = 0;
    L.ctrl = off; off += kTempAlign;
    L.hist = off; off = align_up(off + size_t(max_passes) * kDigits * 8, kTempAlign);
    L.bins = off; off = align_up(off + size_t(max_passes) * kDigits * 8, kTempAlign);
    L.status_bytes = align_up(size_t(L.tiles) * kDigits * st, kTempAlign);
    L.status_a = off; off += L.status_bytes;
    L.status_b = off; off += L.status_bytes;
    L.keys_alt = off; off = align_up(off + size_t(n) * kb, kTempAlign);
    L.vals_alt = off; off = align_up(off + size_t(n) * vb, kTempAlign);
    L.total = off;
    return L;
}

template <typename F>
void set_smem_once(F* kernel, size_t bytes)
{
    set_max_dynamic_smem(reinterpret_cast<const void*>(kernel), bytes);
}

struct SortCall {
    const void* keys_src[kMaxPasses];
    void* keys_dst[kMaxPasses];
    const void* vals_src[kMaxPasses];
    void* vals_dst[kMaxPasses];
};

template <typename U, typename V, bool PAIRS, int BLOCK, int ITEMS, typename ST, typename OffT>
lcpp_status launch_passes(const Layout& L, unsigned char* temp, const SortCall& c, uint64_t n,
                          const KeyCodec<U>& codec, int begin_bit, int end_bit, int passes,
                          cudaStream_t stream)
{
    using Smem = OnesweepSmem<U, V, PAIRS, BLOCK, ITEMS, OffT>;
    auto kernel = onesweep_kernel<U, V, PAIRS, BLOCK, ITEMS, ST, OffT>;
    const size_t smem = sizeof(Smem);
    set_smem_once(kernel, smem);
    Ctrl* ctrl = reinterpret_cast<Ctrl*>(temp + L.ctrl);
    const unsigned long long* bins = reinterpret_cast<const unsigned long long*>(temp + L.bins);
    ST* status[2] = {reinterpret_cast<ST*>(temp + L.status_a), reinterpret_cast<ST*>(temp + L.status_b)};
    const unsigned grid = unsigned(L.tiles);
    for (int p = 0; p < passes; ++p) {
        OnesweepArgs<U, V, ST, OffT> a;
        a.keys_in = static_cast<const U*>(c.keys_src[p]);
        a.keys_out = static_cast<U*>(c.keys_dst[p]);
        a.vals_in = static_cast<const V*>(c.vals_src[p]);
        a.vals_out = static_cast<V*>(c.vals_dst[p]);
        a.n = n;
        a.codec = codec;
        a.shift = begin_bit + kRadixBits * p;
        a.nbits = min(kRadixBits, end_bit - a.shift);
        a.bins = bins + p * kDigits;
        a.status = status[p & 1];
        a.status_next = (p + 1 < passes) ? status[(p + 1) & 1] : nullptr;
        a.tile_counter = &ctrl->tile_counter[p];
        a.error = &ctrl->error;
        diag::KernelTimer timer(1 /* LCPP_KERNEL_SORT_ONESWEEP */, n, stream);
        kernel<<<grid, BLOCK, smem, stream>>>(a);
        timer.stop();
    }
    return cudaGetLastError() == cudaSuccess ? LCPP_OK : LCPP_ERR_CUDA;
}

template <typename U>
lcpp_status launch_histogram(const Layout& L, unsigned char* temp, const U* keys, uint64_t n,
                             const KeyCodec<U>& codec, int begin_bit, int end_bit, int passes,
                             cudaStream_t stream)
{
    constexpr int COPIES = sizeof(U) == 4 ? 8 : 4;
    const int vec = 16 / int(sizeof(U));
    const bool aligned = (reinterpret_cast<uintptr_t>(keys) & 15) == 0;
    const uint64_t per_block_min = uint64_t(kHistBlock) * vec * 4;
    const uint64_t max_blocks = uint64_t(device_sm_count()) * 2;
    uint64_t blocks = std::max<uint64_t>(1, std::min(max_blocks, ceil_div(n, per_block_min)));
    uint64_t chunk = align_up(ceil_div(n, blocks), size_t(vec) * kHistBlock);
    blocks = ceil_div(n, chunk);
    const size_t smem = size_t(passes) * kDigits * COPIES * sizeof(uint32_t);
    Ctrl* ctrl = reinterpret_cast<Ctrl*>(temp + L.ctrl);
    auto* hist = reinterpret_cast<unsigned long long*>(temp + L.hist);
    auto* bins = reinterpret_cast<unsigned long long*>(temp + L.bins);
    diag::KernelTimer timer(0 /* LCPP_KERNEL_SORT_HISTOGRAM */, n, stream);
    if (aligned) {
        auto k = histogram_kernel<U, kHistBlock, COPIES, true>;
        set_smem_once(k, smem);
        k<<<unsigned(blocks), kHistBlock, smem, stream>>>(keys, n, codec, begin_bit, end_bit, passes,
                                                          chunk, ctrl, hist, bins);
    } else {
        auto k = histogram_kernel<U, kHistBlock, COPIES, false>;
        set_smem_once(k, smem);
        k<<<unsigned(blocks), kHistBlock, smem, stream>>>(keys, n, codec, begin_bit, end_bit, passes,
                                                          chunk, ctrl, hist, bins);
    }
    return cudaGetLastError() == cudaSuccess ? LCPP_OK : LCPP_ERR_CUDA;
}

template <typename U, typename V, bool PAIRS>
lcpp_status run_typed(const Layout& L, unsigned char* temp, const SortCall& c, uint64_t n,
                      lcpp_dtype kdt, bool descending, int begin_bit, int end_bit, int passes,
                      cudaStream_t stream)
{
    const KeyCodec<U> codec = make_codec<U>(kdt, descending);
    // Zero control block, histograms, offsets and the pass-0 look-back rows
    // (contiguous in the layout).
    const size_t zero_bytes = L.status_a + size_t(L.tiles) * kDigits * (L.wide ? 8 : 4) - L.ctrl;
    LCPP_CUDA_TRY(cudaMemsetAsync(temp + L.ctrl, 0, zero_bytes, stream));
    lcpp_status st = launch_histogram<U>(L, temp, static_cast<const U*>(c.keys_src[0]), n, codec,
                                         begin_bit, end_bit, passes, stream);
    if (st != LCPP_OK) return st;
    const int kb = sizeof(U), vb = PAIRS ? int(sizeof(V)) : 0;
    const Geometry g = geometry(kb, vb);
#define LCPP_PASSES(B, I)                                                                       \
    (L.wide ? launch_passes<U, V, PAIRS, B, I, uint64_t, uint64_t>(L, temp, c, n, codec,         \
                                                                   begin_bit, end_bit, passes,  \
                                                                   stream)                      \
            : launch_passes<U, V, PAIRS, B, I, uint32_t, uint32_t>(L, temp, c, n, codec,         \
                                                                   begin_bit, end_bit, passes,  \
                                                                   stream))
    if constexpr (sizeof(U) == 4 && !PAIRS) {
        return LCPP_PASSES(384, 20);
    } else if constexpr (sizeof(U) == 4 && sizeof(V) == 4) {
        return LCPP_PASSES(384, 15);
    } else if constexpr (sizeof(U) == 4) {
        return LCPP_PASSES(256, 16);
    } else if constexpr (!PAIRS) {
        return LCPP_PASSES(256, 16);
    } else if constexpr (sizeof(V) == 4) {
        return LCPP_PASSES(256, 14);
    } else {
        return LCPP_PASSES(256, 12);
    }
#undef LCPP_PASSES
    (void)g;
}

bool key_dtype_ok(lcpp_dtype dt) { return dtype_bytes(dt) != 0; }

}  // namespace

size_t temp_bytes(int kb, int vb, uint64_t n)
{
    if (n == 0) return 0;
    return make_layout(kb, vb, n).total;
}

lcpp_status sort(void* temp, size_t temp_bytes_given, const void* keys_in, void* keys_out,
                 const void* vals_in, void* vals_out, void* key_bufs[2], void* val_bufs[2],
                 int* selector, uint64_t n, int begin_bit, int end_bit, int descending,
                 lcpp_dtype kdt, lcpp_dtype vdt, bool pairs, bool double_buffer, cudaStream_t stream)
{
    if (!key_dtype_ok(kdt)) return LCPP_ERR_UNSUPPORTED_DTYPE;
    if (pairs && !key_dtype_ok(vdt)) return LCPP_ERR_UNSUPPORTED_DTYPE;
    const int kb = dtype_bytes(kdt);
    const int vb = pairs ? dtype_bytes(vdt) : 0;
    if (begin_bit < 0 || begin_bit > end_bit || end_bit > kb * 8) return LCPP_ERR_INVALID_ARG;
    if (double_buffer) {
        if (!selector || (*selector != 0 && *selector != 1)) return LCPP_ERR_INVALID_ARG;
        if (n && (!key_bufs || !key_bufs[0] || !key_bufs[1])) return LCPP_ERR_INVALID_ARG;
        if (n && pairs && (!val_bufs || !val_bufs[0] || !val_bufs[1])) return LCPP_ERR_INVALID_ARG;
    } else if (n && (!keys_in || !keys_out || (pairs && (!vals_in || !vals_out)))) {
        return LCPP_ERR_INVALID_ARG;
    }
    if (n == 0) return LCPP_OK;
    if (begin_bit == end_bit) {
        // Zero-width range: the copy API copies, the DoubleBuffer API leaves
        // the selector and the data alone (device_radix_sort.h:381-390, 507-510).
        if (!double_buffer) {
            if (keys_out != keys_in)
                LCPP_CUDA_TRY(cudaMemcpyAsync(keys_out, keys_in, size_t(n) * kb, cudaMemcpyDeviceToDevice, stream));
            if (pairs && vals_out != vals_in)
                LCPP_CUDA_TRY(cudaMemcpyAsync(vals_out, vals_in, size_t(n) * vb, cudaMemcpyDeviceToDevice, stream));
        }
        return LCPP_OK;
    }
    if (!temp || (reinterpret_cast<uintptr_t>(temp) & (kTempAlign - 1))) return LCPP_ERR_INVALID_ARG;
    const Layout L = make_layout(kb, vb, n);
    if (temp_bytes_given < L.total) return LCPP_ERR_TEMP_TOO_SMALL;
    unsigned char* t = static_cast<unsigned char*>(temp);

    const int passes = (end_bit - begin_bit + kRadixBits - 1) / kRadixBits;
    SortCall c{};
    if (double_buffer) {
        int sel = *selector;
        for (int p = 0; p < passes; ++p) {
            c.keys_src[p] = key_bufs[sel];
            c.keys_dst[p] = key_bufs[sel ^ 1];
            if (pairs) {
                c.vals_src[p] = val_bufs[sel];
                c.vals_dst[p] = val_bufs[sel ^ 1];
            }
            sel ^= 1;
        }
    } else {
        // The last pass writes keys_out; earlier passes ping-pong between
        // keys_out and the temp copy so that keys_in is never written.
        void* kalt = t + L.keys_alt;
        void* valt = t + L.vals_alt;
        const void* ksrc = keys_in;
        const void* vsrc = vals_in;
        for (int p = 0; p < passes; ++p) {
            const bool to_out = ((passes - 1 - p) % 2) == 0;
            c.keys_src[p] = ksrc;
            c.keys_dst[p] = to_out ? keys_out : kalt;
            ksrc = c.keys_dst[p];
            if (pairs) {
                c.vals_src[p] = vsrc;
                c.vals_dst[p] = to_out ? vals_out : valt;
                vsrc = c.vals_dst[p];
            }
        }
    }

    lcpp_status st;
    const bool desc = descending != 0;
    if (kb == 4) {
        if (!pairs) st = run_typed<uint32_t, uint32_t, false>(L, t, c, n, kdt, desc, begin_bit, end_bit, passes, stream);
        else if (vb == 4) st = run_typed<uint32_t, uint32_t, true>(L, t, c, n, kdt, desc, begin_bit, end_bit, passes, stream);
        else st = run_typed<uint32_t, uint64_t, true>(L, t, c, n, kdt, desc, begin_bit, end_bit, passes, stream);
    } else {
        if (!pairs) st = run_typed<uint64_t, uint32_t, false>(L, t, c, n, kdt, desc, begin_bit, end_bit, passes, stream);
        else if (vb == 4) st = run_typed<uint64_t, uint32_t, true>(L, t, c, n, kdt, desc, begin_bit, end_bit, passes, stream);
        else st = run_typed<uint64_t, uint64_t, true>(L, t, c, n, kdt, desc, begin_bit, end_bit, passes, stream);
    }
    if (st == LCPP_OK && double_buffer) *selector ^= (passes & 1);
    return st;
}

size_t error_word_offset() { return offsetof(Ctrl, error); }

}  // namespace radix
}  // namespace lcpp
