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
//      warp ballots and per-warp shared-memory counters, publish per-digit
//      tile counts, resolve the global digit offsets with a bounded decoupled
//      look-back, stage the tile in shared memory in digit order and write it
//      out so that each digit's run is stored contiguously (the reference's
//      AgentRadixSortOneSweep, agent_radix_sort_onesweep.h:224-511, with
//      BlockRadixRankMatchEarlyCounts, block_radix_rank.h:207-486).  Keys-only
//      sorts of 4-byte keys whose buffers are 16-byte aligned run the same
//      tile work in onesweep_bulk_kernel: persistent blocks that bulk-copy
//      their next tile into shared memory while the current one is ranked.
//
// B200 budget: at the measured ~6.5 TB/s an 8-bit pass over 4-byte keys has
// about 11 SM cycles per 32 keys, and the integer ALU pipe issues about two
// warp instructions per cycle, so the kernels are written for instruction
// count: keys are transformed once on load and once on store (not at every
// digit extraction), the key kind is a template parameter (unsigned
// ascending keys need no transform at all), full tiles use unguarded loads
// with immediate offsets, the tile-base and per-warp offsets are merged into
// one table (one shared load per key), and consistency checks run per digit
// rather than per key.
//
// Differences from the reference that are part of this design:
//  - look-back status rows are double-buffered and each pass clears the rows
//    the next pass will use, instead of a separate reset kernel per pass and
//    portion (device_radix_sort.h:1389-1398);
//  - one portion at any size: counts and offsets are 64-bit from 2^30 keys
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

// ---------------------------------------------------------------------------
// Key transform, specialised by kind (see KeyCodec in common.cuh):
//   kPlain : unsigned keys, ascending   -> identity
//   kXor   : unsigned descending, signed ascending / descending -> k ^ xor_pos
//   kFloat : floating point -> sign-dependent XOR, and +-0.0 share digits
// ---------------------------------------------------------------------------
enum : int { kPlain = 0, kXor = 1, kFloat = 2 };

template <int KIND, typename U>
__device__ __forceinline__ U twiddle_in(U k, const KeyCodec<U>& c)
{
    if constexpr (KIND == kPlain) {
        return k;
    } else if constexpr (KIND == kXor) {
        return k ^ c.xor_pos;
    } else {
        // Pure bijection (no +-0 fold: the stored key keeps its bits; the
        // fold only applies to digits, see digit_of).
        constexpr int kBits = sizeof(U) * 8;
        using S = typename std::conditional<sizeof(U) == 4, int32_t, int64_t>::type;
        const U sign = U(S(k) >> (kBits - 1));
        return k ^ U(c.xor_pos ^ (sign & (c.xor_pos ^ c.xor_neg)));
    }
}

template <int KIND, typename U>
__device__ __forceinline__ U twiddle_out(U t, const KeyCodec<U>& c)
{
    if constexpr (KIND == kPlain) {
        return t;
    } else if constexpr (KIND == kXor) {
        return t ^ c.xor_pos;
    } else {
        // Undo the optional descending inversion, then the float bijection:
        // a transformed key with the high bit set came from a non-negative
        // key (flip the high bit back), otherwise from a negative one (flip all).
        constexpr int kBits = sizeof(U) * 8;
        constexpr U kHigh = U(1) << (kBits - 1);
        using S = typename std::conditional<sizeof(U) == 4, int32_t, int64_t>::type;
        const U u = t ^ U(c.xor_pos ^ kHigh);  // xor_pos is kHigh ascending, ~kHigh descending
        const U sign = U(S(u) >> (kBits - 1));
        return u ^ U(~U(0) ^ (sign & ~kHigh));
    }
}

// Digit of a transformed key.  For floats, the transformed -0.0 (ascending)
// or +0.0 (descending), kHigh - 1, takes the digits of kHigh, the value the
// other zero maps to (radix_rank_sort_operations.h:31-43).
template <int KIND, typename U>
__device__ __forceinline__ uint32_t digit_of(U t, int shift, uint32_t mask)
{
    if constexpr (KIND == kFloat) {
        constexpr U kHigh = U(1) << (sizeof(U) * 8 - 1);
        t = t == U(kHigh - 1) ? kHigh : t;
    }
    return uint32_t(t >> shift) & mask;
}

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
// Shared counters are replicated COPIES times, interleaved so that copy c of
// bin b sits at word b * COPIES + c, and lane l counts into copy l % COPIES.
// With COPIES = 32 every lane of a warp hits its own bank, so the shared
// atomics never conflict, whatever the key distribution.
// ---------------------------------------------------------------------------
template <typename U, int KIND, int PASSES, int BLOCK, int COPIES>
__global__ void __launch_bounds__(BLOCK, 1)
histogram_kernel(const U* __restrict__ keys, uint64_t n, KeyCodec<U> codec, int begin_bit,
                 uint32_t last_mask, uint64_t chunk, Ctrl* ctrl,
                 unsigned long long* __restrict__ g_hist, unsigned long long* __restrict__ g_bins)
{
    extern __shared__ __align__(16) uint32_t s_hist[];  // [PASSES * 256][COPIES]
    __shared__ unsigned long long s_sums[8];
    __shared__ int s_last;
    const int tid = threadIdx.x;
    const int copy = (tid & 31) % COPIES;
    for (int i = tid; i < PASSES * kDigits * COPIES; i += BLOCK) s_hist[i] = 0;
    __syncthreads();

    auto count = [&](U k) {
        const U t = twiddle_in<KIND>(k, codec);
#pragma unroll
        for (int p = 0; p < PASSES; ++p) {
            const uint32_t d = digit_of<KIND>(t, begin_bit + kRadixBits * p, p + 1 == PASSES ? last_mask : 0xffu);
            atomicAdd(&s_hist[(p * kDigits + d) * COPIES + copy], 1u);
        }
    };

    constexpr int VEC = 16 / sizeof(U);
    using VT = typename std::conditional<sizeof(U) == 4, uint4, ulonglong2>::type;
    const uint64_t lo = uint64_t(blockIdx.x) * chunk;
    const uint64_t hi = min(lo + chunk, n);
    if (lo < hi) {
        // Scalar head up to the first 16-byte boundary, vector body, scalar tail.
        const uint64_t mis = (reinterpret_cast<uintptr_t>(keys + lo) & 15) / sizeof(U);
        const uint64_t head = min(hi - lo, uint64_t(mis ? VEC - mis : 0));
        if (uint64_t(tid) < head) count(keys[lo + tid]);
        const uint64_t vlo = lo + head;
        const uint64_t nvec = (hi - vlo) / VEC;
        const VT* vp = reinterpret_cast<const VT*>(keys + vlo);
        uint64_t j = tid;
        for (; j + 3 * BLOCK < nvec; j += 4 * BLOCK) {
            VT v[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) v[u] = vp[j + u * BLOCK];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const U* e = reinterpret_cast<const U*>(&v[u]);
#pragma unroll
                for (int q = 0; q < VEC; ++q) count(e[q]);
            }
        }
        for (; j < nvec; j += BLOCK) {
            const VT v = vp[j];
            const U* e = reinterpret_cast<const U*>(&v);
#pragma unroll
            for (int q = 0; q < VEC; ++q) count(e[q]);
        }
        for (uint64_t i = vlo + nvec * VEC + tid; i < hi; i += BLOCK) count(keys[i]);
    }
    __syncthreads();
    for (int i = tid; i < PASSES * kDigits; i += BLOCK) {
        uint32_t s = 0;
#pragma unroll
        for (int c = 0; c < COPIES; ++c) s += s_hist[i * COPIES + ((c + i) & (COPIES - 1))];  // rotated: no bank conflicts
        if (s) atomicAdd(&g_hist[i], (unsigned long long)s);
    }
    __threadfence();
    __syncthreads();
    if (tid == 0) s_last = atomicAdd(&ctrl->hist_done, 1u) == gridDim.x - 1;
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    // Last block: exclusive digit offsets of every pass.
    for (int p = 0; p < PASSES; ++p) {
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
    uint32_t digit_mask;             // (1 << bits of this pass) - 1
    const unsigned long long* bins;  // [256] exclusive global digit offsets of this pass
    ST* status;                      // [tiles][256] look-back rows of this pass
    ST* status_next;                 // rows the next pass uses (cleared here), or null
    uint32_t* tile_counter;
    uint32_t* error;
};

// Tile policy of one onesweep configuration: BLOCK x ITEMS keys per tile
// (warp-striped, ITEMS slots per lane), WINDOW predecessor tiles read per
// look-back round trip, MIN_BLOCKS resident blocks per SM asked of the
// register allocator.
template <int BLOCK, int ITEMS, int WINDOW, int MIN_BLOCKS>
struct Policy {
    static constexpr int kBlock = BLOCK;
    static constexpr int kItems = ITEMS;
    static constexpr int kWindow = WINDOW;
    static constexpr int kMinBlocks = MIN_BLOCKS;
    static constexpr int kTile = BLOCK * ITEMS;
    static constexpr int kWarps = BLOCK / kWarp;
    static constexpr int kSleepNs = 32;  // back-off between polls of an unpublished status word
    // Peer masks: one word per low-5-bit digit class and slot, two slots per
    // set, two sets alternating by slot pair.
    static constexpr int kMaskWords = 2 * 32;
};

// Shared memory of one onesweep block.  The staging tile (keys, and values
// for pairs) has its own storage, so every key is written to its tile rank
// as soon as it is ranked: no rank array stays live in registers, and the
// digit threads start their look-back while other warps are still ranking.
template <typename U, typename V, bool PAIRS, typename P, typename OffT>
struct OnesweepSmem {
    static constexpr int kTile = P::kTile;
    static constexpr int kWarps = P::kWarps;
    U keys[kTile];                        // transformed keys in tile-rank order
    V vals[PAIRS ? kTile : 1];
    alignas(16) uint32_t counters[kWarps * kDigits];  // per-warp digit counters, then rank bases
    uint32_t peer_masks[2 * kWarps * P::kMaskWords];
    OffT gofs[kDigits];         // output index = gofs[digit] + tile position
    uint32_t totals[kDigits];   // keys of each digit in the tile
    uint32_t dstarts[kDigits];  // first tile rank of each digit
    uint32_t warp_sums[8];
    uint32_t tile_id;
    int bad;
};

// Bounded wait until a status word is published (flag bits set).  Backs off
// with __nanosleep so that waiting warps leave issue slots to the warps of
// other tiles on the same SM.  On timeout (or when another thread already
// reported an error) returns an inclusive zero so that the caller finishes.
template <int SLEEP_NS, typename ST>
__device__ __forceinline__ ST wait_status(const ST* p, ST w, uint32_t* error, uint64_t limit_ns = kWaitLimitNs)
{
    using SB = StatusBits<ST>;
    uint32_t spins = 0;
    uint64_t t0 = 0;
    while ((w & SB::kFlags) == 0) {
        if constexpr (SLEEP_NS > 0) __nanosleep(SLEEP_NS);
        w = ld_relaxed(p);
        if (++spins == 32) {
            spins = 0;
            const uint64_t now = global_timer_ns();
            if (t0 == 0) {
                t0 = now;
            } else if (now - t0 > limit_ns) {
                report_error(error, kDevErrTimeout);
                return SB::kInclusive;
            }
            if (error_raised(error)) return SB::kInclusive;
        }
    }
    return w;
}

// Exclusive prefix of one digit over tiles [0, tile): walk back from
// tile - 1, W tiles per round trip, adding partial counts until an inclusive
// count is found.  Tile 0 always publishes an inclusive count.
template <typename ST, typename OffT, int W, int SLEEP_NS>
__device__ __forceinline__ OffT lookback_digit(const ST* status, uint32_t tile, int digit, uint32_t* error)
{
    using SB = StatusBits<ST>;
    OffT prefix = 0;
    int64_t base = int64_t(tile) - 1;
    while (true) {
        ST w[W];
#pragma unroll
        for (int q = 0; q < W; ++q) {
            const int64_t j = base - q;
            w[q] = j >= 0 ? ld_relaxed(status + uint64_t(j) * kDigits + digit) : SB::kInclusive;
        }
        bool done = false;
#pragma unroll
        for (int q = 0; q < W; ++q) {
            if (!done) {
                const int64_t j = base - q;
                if (j >= 0) w[q] = wait_status<SLEEP_NS>(status + uint64_t(j) * kDigits + digit, w[q], error);
                prefix += OffT(w[q] & SB::kValue);
                done = (w[q] & SB::kInclusive) != 0;
            }
        }
        if (done) return prefix;
        base -= W;
    }
}

// Digit extraction for the onesweep kernel.  BYTE: the pass covers a whole
// byte of a 4-byte key (shift % 8 == 0, 8 bits), so one byte permute
// extracts it.
template <int KIND, bool BYTE, typename U>
__device__ __forceinline__ uint32_t pass_digit(U t, int shift, uint32_t mask, uint32_t byte_sel)
{
    if constexpr (BYTE && sizeof(U) == 4) {
        if constexpr (KIND == kFloat) {
            constexpr U kHigh = U(1) << 31;
            t = t == U(kHigh - 1) ? kHigh : t;
        }
        return __byte_perm(uint32_t(t), 0u, byte_sel);
    } else {
        return digit_of<KIND>(t, shift, mask);
    }
}

struct NoHook {
    __device__ __forceinline__ void operator()() const {}
};

// Everything after the tile id is known.  FULL: the tile has kTile keys (all
// but possibly the last tile), compiled without any per-key bounds logic.
// staged: the tile's keys already sit in shared memory (bulk-copied, same
// order as in global memory), or null to load them from global memory.
// after_counts runs on every thread right after the block barrier that
// follows the early counts, the first point at which every thread has its
// keys in registers.  PERSIST: the block goes on to another tile, so the
// rank counters are cleared before returning.  Returns false when the tile
// broke an invariant (the error word is set and nothing was stored).
template <bool FULL, bool BYTE, bool PERSIST, typename P, typename U, typename V, bool PAIRS, int KIND, typename ST,
          typename OffT, typename Hook = NoHook>
__device__ __forceinline__ bool process_tile(const OnesweepArgs<U, V, ST, OffT>& a,
                                             OnesweepSmem<U, V, PAIRS, P, OffT>& s, uint32_t tile, int valid,
                                             const U* staged = nullptr, Hook after_counts = Hook())
{
    using SB = StatusBits<ST>;
    constexpr int BLOCK = P::kBlock;
    constexpr int ITEMS = P::kItems;
    constexpr int kTile = P::kTile;
    constexpr int kWarps = P::kWarps;
    const int tid = threadIdx.x;
    const int lane = tid & 31;
    const int warp = tid >> 5;
    const uint64_t tile_base = uint64_t(tile) * kTile;
    const uint32_t dmask = a.digit_mask;
    const uint32_t byte_sel = 0x4440u | uint32_t(a.shift >> 3);
    auto digit = [&](U t) { return pass_digit<KIND, BYTE>(t, a.shift, dmask, byte_sel); };
    auto in_tile = [&](int i) { return FULL || warp * ITEMS * kWarp + lane + i * kWarp < valid; };

    // Warp-striped load: warp w owns positions [w*ITEMS*32, (w+1)*ITEMS*32) of
    // the tile, slot i of lane l is position w*ITEMS*32 + i*32 + l.
    U keys[ITEMS];
    V vals[PAIRS ? ITEMS : 1];
    const uint32_t counters_base = static_cast<uint32_t>(__cvta_generic_to_shared(s.counters + warp * kDigits));
    {
        const int warp_base = warp * ITEMS * kWarp + lane;
        if (staged) {
#pragma unroll
            for (int i = 0; i < ITEMS; ++i) keys[i] = staged[warp_base + i * kWarp];
        } else {
            const U* src = a.keys_in + tile_base + warp_base;
#pragma unroll
            for (int i = 0; i < ITEMS; ++i) keys[i] = in_tile(i) ? src[i * kWarp] : U(0);
        }
        if constexpr (PAIRS) {
            const V* vsrc = a.vals_in + tile_base + warp_base;
#pragma unroll
            for (int i = 0; i < ITEMS; ++i) vals[i] = in_tile(i) ? vsrc[i * kWarp] : V(0);
        }
#pragma unroll
        for (int i = 0; i < ITEMS; ++i) keys[i] = twiddle_in<KIND>(keys[i], a.codec);
        // Early counts: per-warp digit histograms.  Positions past the end
        // of the last tile take the largest digit, so they rank after every
        // real key and are never stored.
#pragma unroll
        for (int i = 0; i < ITEMS; ++i)
            shared_red_add(counters_base + (in_tile(i) ? digit(keys[i]) : dmask) * 4u, 1u);
    }
    __syncthreads();
    after_counts();

    // Per digit: tile total (published at once), block-wide digit start,
    // then counters[w][d] := digit start + count of d in warps < w, the
    // first tile rank of warp w's keys with digit d.
    uint32_t total = 0;
    if (tid < kDigits) {
#pragma unroll
        for (int w = 0; w < kWarps; ++w) total += s.counters[w * kDigits + tid];
        st_relaxed(a.status + uint64_t(tile) * kDigits + tid,
                   ST(total) | (tile == 0 ? SB::kInclusive : SB::kPartial));
    }
    const uint32_t dstart = exclusive_scan_256<uint32_t, BLOCK>(total, s.warp_sums);
    if (tid < kDigits) {
        uint32_t run = dstart;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) {
            const uint32_t c = s.counters[w * kDigits + tid];
            s.counters[w * kDigits + tid] = run;
            run += c;
        }
        s.totals[tid] = total;
        s.dstarts[tid] = dstart;
    }
    __syncthreads();

    // Stable ranking, each key written to the staging tile at its rank: keys
    // of one slot are ranked in lane order among equal digits, slots in
    // order; the digit's leader lane advances the warp's rank counter by the
    // number of peers and the returned value is the first tile rank of the
    // group.  The leader's atomic is predicated rather than branched around,
    // so the atomics of both slots of a pair are issued back to back;
    // shared-memory operations of one warp complete in issue order, which
    // keeps consecutive slots consistent.
    {
        const uint32_t lt = lanemask_lt();
        constexpr uint32_t kSetBytes = uint32_t(kWarps * P::kMaskWords) * 4u;
        const uint32_t masks_base =
            static_cast<uint32_t>(__cvta_generic_to_shared(s.peer_masks + warp * P::kMaskWords));
#pragma unroll
        for (int i0 = 0; i0 < ITEMS; i0 += 2) {
            uint32_t d[2], peers[2], maddr[2], base[2];
            // Each lane ORs its bit into the mask word of its digit's low 5
            // bits (32 words, one per bank, so these accesses never
            // conflict), and one ballot per remaining bit narrows the class
            // to the digit.  Slot g of a pair uses half g of the pair's mask
            // set; every lane clears its word once all lanes have read it
            // (the shuffle below depends on every lane's read), and the next
            // pair's warp barrier orders the clears before the pair after it
            // reuses the set.
#pragma unroll
            for (int g = 0; g < 2; ++g) {
                if (i0 + g < ITEMS) {
                    const int i = i0 + g;
                    d[g] = in_tile(i) ? digit(keys[i]) : dmask;
                    maddr[g] = masks_base + uint32_t((i0 >> 1) & 1) * kSetBytes + (uint32_t(g) * 32u + (d[g] & 31u)) * 4u;
                    shared_red_or(maddr[g], 1u << lane);
                }
            }
            warp_barrier();
#pragma unroll
            for (int g = 0; g < 2; ++g) {
                if (i0 + g < ITEMS) {
                    peers[g] = shared_load(maddr[g]);
#pragma unroll
                    for (int b = 5; b < kRadixBits; ++b) {
                        const bool bit = (d[g] >> b) & 1u;
                        const uint32_t vote = warp_ballot(bit);
                        peers[g] &= bit ? vote : ~vote;
                    }
                }
            }
#pragma unroll
            for (int g = 0; g < 2; ++g) {
                if (i0 + g < ITEMS) {
                    const int leader = 31 - __clz(peers[g]);
                    base[g] = shared_add_if(lane == leader, counters_base + d[g] * 4u, uint32_t(__popc(peers[g])));
                }
            }
#pragma unroll
            for (int g = 0; g < 2; ++g) {
                if (i0 + g < ITEMS) {
                    base[g] = warp_shfl(base[g], 31 - __clz(peers[g]));
                    shared_store_if(true, maddr[g], 0u);
                    const uint32_t r = base[g] + __popc(peers[g] & lt);
                    s.keys[r] = keys[i0 + g];
                    if constexpr (PAIRS) s.vals[r] = vals[i0 + g];
                }
            }
        }
    }

    // Publishes the inclusive count of digit d and its output base, and
    // checks that the digit's keys land inside the output (a broken
    // invariant becomes an error code, never a wild write).
    auto finish_digit = [&](int d, OffT prefix) {
        const uint32_t tot = s.totals[d];
        if (tile > 0) st_relaxed(a.status + uint64_t(tile) * kDigits + d, ST(prefix + tot) | SB::kInclusive);
        s.gofs[d] = OffT(a.bins[d]) + prefix - OffT(s.dstarts[d]);
        // positions past the end of the last tile all carry the largest digit
        const uint32_t stored = tot - ((!FULL && uint32_t(d) == dmask) ? uint32_t(kTile - valid) : 0u);
        if (uint64_t(a.bins[d]) + uint64_t(prefix) + stored > a.n) s.bad = 1;
        if (a.status_next) a.status_next[uint64_t(tile) * kDigits + d] = 0;
    };

    // Decoupled look-back, one digit per thread, P::kWindow predecessor tiles
    // per round trip.  A digit thread starts as soon as its own warp has
    // ranked its keys, while other warps may still be ranking.
    if (tid < kDigits) {
        OffT prefix = 0;
        if (tile > 0) prefix = lookback_digit<ST, OffT, P::kWindow, P::kSleepNs>(a.status, tile, tid, a.error);
        finish_digit(tid, prefix);
    }
    __syncthreads();
    if (s.bad) {
        if (tid == 0) report_error(a.error, kDevErrInternal);
        return false;
    }
    if constexpr (PERSIST) {
        // The rank counters are dead from here on (the stores use gofs):
        // clear them for the next tile's early counts.
        static_assert((kWarps * kDigits) % 4 == 0, "16-byte clears");
        uint4* c4 = reinterpret_cast<uint4*>(s.counters);
        for (int i = tid; i < kWarps * kDigits / 4; i += BLOCK) c4[i] = make_uint4(0u, 0u, 0u, 0u);
    }

    // Digit-ordered tile -> global: consecutive threads write consecutive
    // positions of one digit run.  Loads, offset lookups and stores are done
    // in separate unrolled phases so that their latencies overlap.
    {
        OffT out_pos[ITEMS];
#pragma unroll
        for (int i = 0; i < ITEMS; ++i) keys[i] = s.keys[i * BLOCK + tid];
#pragma unroll
        for (int i = 0; i < ITEMS; ++i) out_pos[i] = s.gofs[digit(keys[i])] + OffT(i * BLOCK + tid);
        if constexpr (PAIRS) {
#pragma unroll
            for (int i = 0; i < ITEMS; ++i) vals[i] = s.vals[i * BLOCK + tid];
        }
#pragma unroll
        for (int i = 0; i < ITEMS; ++i) {
            if (FULL || i * BLOCK + tid < valid) {
                a.keys_out[out_pos[i]] = twiddle_out<KIND>(keys[i], a.codec);
                if constexpr (PAIRS) a.vals_out[out_pos[i]] = vals[i];
            }
        }
    }
    return true;
}

template <typename U, typename V, bool PAIRS, typename P, int KIND, bool BYTE, typename ST, typename OffT>
__global__ void __launch_bounds__(P::kBlock, P::kMinBlocks)
onesweep_kernel(OnesweepArgs<U, V, ST, OffT> a)
{
    using Smem = OnesweepSmem<U, V, PAIRS, P, OffT>;
    constexpr int BLOCK = P::kBlock;
    constexpr int kTile = Smem::kTile;
    constexpr int kWarps = Smem::kWarps;
    static_assert(BLOCK >= kDigits, "one thread per digit");
    static_assert(kTile <= 65536, "tile ranks fit 16 bits");
    extern __shared__ __align__(16) unsigned char smem_raw[];
    Smem& s = *reinterpret_cast<Smem*>(smem_raw);

    const int tid = threadIdx.x;
    if (tid == 0) {
        s.tile_id = atomicAdd(a.tile_counter, 1u);
        s.bad = 0;
    }
    for (int i = tid; i < kWarps * kDigits; i += BLOCK) s.counters[i] = 0;
    for (int i = tid; i < 2 * kWarps * P::kMaskWords; i += BLOCK) s.peer_masks[i] = 0;
    __syncthreads();
    const uint32_t tile = s.tile_id;
    const uint64_t tile_base = uint64_t(tile) * kTile;
    if (tile_base + kTile <= a.n)
        process_tile<true, BYTE, false, P, U, V, PAIRS, KIND, ST, OffT>(a, s, tile, kTile);
    else
        process_tile<false, BYTE, false, P, U, V, PAIRS, KIND, ST, OffT>(a, s, tile, int(a.n - tile_base));
}

// ---------------------------------------------------------------------------
// Persistent onesweep pass for keys-only sorts whose key buffers are 16-byte
// aligned.  One block per resident slot; each block takes tile ids from the
// pass's atomic counter in increasing order.  As soon as every thread holds
// its keys of tile k in registers (the barrier after the early counts), one
// thread takes the block's next tile id and starts a bulk asynchronous copy
// (cp.async.bulk global -> shared, completion on an mbarrier, no multicast)
// of that tile into the block's input buffer, so the HBM read of tile k+1
// runs during the ranking, look-back and stores of tile k.  The last tile,
// when partial, is read with guarded plain loads.
//
// Forward progress: a block's next tile is taken while its current tile is in
// flight, so every tile id below the smallest unpublished one belongs to a
// block that has published it or is about to (the current tile of a running
// block publishes its partial counts before any wait), as with one tile per
// block.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void os_mbar_init(uint64_t* bar)
{
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(uint32_t(__cvta_generic_to_shared(bar))) : "memory");
}

// one arrival expecting `bytes`, then the copy that delivers them
__device__ __forceinline__ void os_bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar)
{
    const uint32_t b = uint32_t(__cvta_generic_to_shared(bar));
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(b), "r"(bytes) : "memory");
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            uint32_t(__cvta_generic_to_shared(dst))),
        "l"(src), "r"(bytes), "r"(b)
        : "memory");
}

// Bounded wait for phase `parity` of `bar`: false after kWaitLimitNs.
__device__ __forceinline__ bool os_mbar_wait(uint64_t* bar, uint32_t parity)
{
    const uint32_t b = uint32_t(__cvta_generic_to_shared(bar));
    uint64_t t0 = 0;
    uint32_t spins = 0;
    while (true) {
        uint32_t done;
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(done)
            : "r"(b), "r"(parity)
            : "memory");
        if (done) return true;
        if (++spins == 16) {
            spins = 0;
            const uint64_t now = global_timer_ns();
            if (t0 == 0)
                t0 = now;
            else if (now - t0 > kWaitLimitNs)
                return false;
        }
    }
}

template <typename U, typename V, typename P, typename OffT>
struct OnesweepBulkSmem {
    alignas(16) U in[P::kTile];  // the next tile, bulk-copied in global order
    OnesweepSmem<U, V, false, P, OffT> s;
    uint64_t bar;
    uint32_t next_tile;
};

template <typename U, typename V, typename P, int KIND, bool BYTE, typename ST, typename OffT>
__global__ void __launch_bounds__(P::kBlock, P::kMinBlocks)
onesweep_bulk_kernel(OnesweepArgs<U, V, ST, OffT> a, uint32_t tiles)
{
    using Smem = OnesweepBulkSmem<U, V, P, OffT>;
    constexpr int BLOCK = P::kBlock;
    constexpr int kTile = P::kTile;
    constexpr int kWarps = P::kWarps;
    constexpr uint32_t kTileBytes = uint32_t(kTile * sizeof(U));
    static_assert(BLOCK >= kDigits, "one thread per digit");
    static_assert(kTile <= 65536, "tile ranks fit 16 bits");
    static_assert(kTileBytes % 16 == 0, "bulk copies move multiples of 16 bytes");
    extern __shared__ __align__(16) unsigned char smem_raw[];
    Smem& m = *reinterpret_cast<Smem*>(smem_raw);

    const int tid = threadIdx.x;
    const uint64_t full_tiles = a.n / kTile;
    // thread 0: take the next tile id and, for a full tile, start its copy
    auto acquire = [&]() {
        const uint32_t t = atomicAdd(a.tile_counter, 1u);
        m.next_tile = t;
        if (t < full_tiles) os_bulk_load(m.in, a.keys_in + uint64_t(t) * kTile, kTileBytes, &m.bar);
    };
    if (tid == 0) {
        m.s.bad = 0;
        os_mbar_init(&m.bar);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        acquire();
    }
    for (int i = tid; i < kWarps * kDigits; i += BLOCK) m.s.counters[i] = 0;
    for (int i = tid; i < 2 * kWarps * P::kMaskWords; i += BLOCK) m.s.peer_masks[i] = 0;
    __syncthreads();

    uint32_t phase = 0;
    bool in_flight = false;  // a copy this block started has not been waited for
    while (true) {
        const uint32_t tile = m.next_tile;
        if (tile >= tiles) break;
        // The hook runs after every thread has read the input buffer: the
        // buffer's generic-proxy reads are ordered before the copy that
        // refills it.
        auto refill = [&]() {
            if (tid == 0) {
                m.s.bad = 0;
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                acquire();
            }
        };
        bool ok;
        if (tile < full_tiles) {
            // every thread observes the copy's completion; the block leaves
            // together if any of them gave up
            if (__syncthreads_or(!os_mbar_wait(&m.bar, phase))) {
                if (tid == 0) report_error(a.error, kDevErrTimeout);
                in_flight = true;
                break;
            }
            phase ^= 1u;
            ok = process_tile<true, BYTE, true, P, U, V, false, KIND, ST, OffT>(a, m.s, tile, kTile, m.in, refill);
        } else {
            ok = process_tile<false, BYTE, true, P, U, V, false, KIND, ST, OffT>(
                a, m.s, tile, int(a.n - uint64_t(tile) * kTile), nullptr, refill);
        }
        // the copy started by refill, if any, is for m.next_tile
        if (!ok) {
            in_flight = m.next_tile < full_tiles;
            break;
        }
        __syncthreads();  // staging tile, counters and next_tile are free / visible
    }
    // Only after an error: wait (bounded) for this block's copy in flight
    // before its shared memory is released.
    if (tid == 0 && in_flight && !os_mbar_wait(&m.bar, phase)) report_error(a.error, kDevErrTimeout);
}

// Wait-timeout probe: one thread waits, with the look-back's bounded wait
// routine, on a status word that nothing publishes.  The wait runs out after
// limit_ns, records LCPP_ERR_LOOKBACK_TIMEOUT and the kernel returns.
__global__ void wait_timeout_probe_kernel(const uint32_t* never_published, uint32_t* error, uint64_t limit_ns)
{
    if (threadIdx.x == 0 && blockIdx.x == 0) wait_status<32>(never_published, 0u, error, limit_ns);
}

// ---------------------------------------------------------------------------
// Host side.
// ---------------------------------------------------------------------------
namespace {

// Smallest tile (keys per onesweep block) of any configuration; sizes the
// look-back rows in temp storage.
constexpr uint64_t kMinTile = 5120;
constexpr int kHistBlock = 1024;

struct Layout {
    size_t ctrl, hist, bins, status_a, status_b, keys_alt, vals_alt, total;
    bool wide;  // 64-bit status words and offsets (n >= 2^30)
};

Layout make_layout(int kb, int vb, uint64_t n)
{
    Layout L{};
    L.wide = n >= (1ull << 30);
    const uint64_t max_tiles = ceil_div(n, kMinTile);
    const size_t st = L.wide ? 8 : 4;
    const int max_passes = kb;  // 8-bit passes over the full key width
    size_t off = 0;
    L.ctrl = off; off += kTempAlign;
    L.hist = off; off = align_up(off + size_t(max_passes) * kDigits * 8, kTempAlign);
    L.bins = off; off = align_up(off + size_t(max_passes) * kDigits * 8, kTempAlign);
    const size_t status_bytes = align_up(size_t(max_tiles) * kDigits * st, kTempAlign);
    L.status_a = off; off += status_bytes;
    L.status_b = off; off += status_bytes;
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

template <typename U, int KIND, int PASSES>
void launch_histogram_p(unsigned grid, size_t smem, uint64_t chunk, const U* keys, uint64_t n,
                        const KeyCodec<U>& codec, int begin_bit, uint32_t last_mask, Ctrl* ctrl,
                        unsigned long long* hist, unsigned long long* bins, cudaStream_t stream)
{
    constexpr int COPIES = sizeof(U) == 4 ? 32 : 16;
    auto k = histogram_kernel<U, KIND, PASSES, kHistBlock, COPIES>;
    set_smem_once(k, smem);
    k<<<grid, kHistBlock, smem, stream>>>(keys, n, codec, begin_bit, last_mask, chunk, ctrl, hist, bins);
}

template <typename U, int KIND>
lcpp_status launch_histogram(const Layout& L, unsigned char* temp, const U* keys, uint64_t n,
                             const KeyCodec<U>& codec, int begin_bit, int end_bit, int passes,
                             cudaStream_t stream)
{
    // 128 KB of counters at most (4 passes x 32 copies, or 8 passes x 16
    // copies): one block of kHistBlock threads per SM.
    constexpr int COPIES = sizeof(U) == 4 ? 32 : 16;
    const int vec = 16 / int(sizeof(U));
    const uint64_t per_block_min = uint64_t(kHistBlock) * vec * 4;
    const uint64_t max_blocks = uint64_t(device_sm_count());
    uint64_t blocks = std::max<uint64_t>(1, std::min(max_blocks, ceil_div(n, per_block_min)));
    const uint64_t chunk = align_up(ceil_div(n, blocks), size_t(vec) * kHistBlock);
    blocks = ceil_div(n, chunk);
    const size_t smem = size_t(passes) * kDigits * COPIES * sizeof(uint32_t);
    Ctrl* ctrl = reinterpret_cast<Ctrl*>(temp + L.ctrl);
    auto* hist = reinterpret_cast<unsigned long long*>(temp + L.hist);
    auto* bins = reinterpret_cast<unsigned long long*>(temp + L.bins);
    const int last_bits = end_bit - begin_bit - kRadixBits * (passes - 1);
    const uint32_t last_mask = (1u << last_bits) - 1u;
    const unsigned grid = unsigned(blocks);
    diag::KernelTimer timer(0 /* LCPP_KERNEL_SORT_HISTOGRAM */, n, stream);
#define LCPP_HIST(P) launch_histogram_p<U, KIND, P>(grid, smem, chunk, keys, n, codec, begin_bit, last_mask, ctrl, hist, bins, stream)
    switch (passes) {
    case 1: LCPP_HIST(1); break;
    case 2: LCPP_HIST(2); break;
    case 3: LCPP_HIST(3); break;
    case 4: LCPP_HIST(4); break;
    default:
        if constexpr (sizeof(U) == 8) {
            switch (passes) {
            case 5: LCPP_HIST(5); break;
            case 6: LCPP_HIST(6); break;
            case 7: LCPP_HIST(7); break;
            default: LCPP_HIST(8); break;
            }
        }
        break;
    }
#undef LCPP_HIST
    return cudaGetLastError() == cudaSuccess ? LCPP_OK : LCPP_ERR_CUDA;
}

template <typename U, typename V, bool PAIRS, typename P, int KIND, typename ST, typename OffT, bool BYTE, bool BULK>
void launch_pass(const OnesweepArgs<U, V, ST, OffT>& a, uint64_t tiles, cudaStream_t stream)
{
    if constexpr (BULK) {
        static_assert(!PAIRS, "the persistent pass sorts keys only");
        using Smem = OnesweepBulkSmem<U, V, P, OffT>;
        auto kernel = onesweep_bulk_kernel<U, V, P, KIND, BYTE, ST, OffT>;
        set_smem_once(kernel, sizeof(Smem));
        const uint64_t slots =
            uint64_t(device_sm_count()) *
            uint64_t(std::max(1, resident_blocks(reinterpret_cast<const void*>(kernel), P::kBlock, sizeof(Smem))));
        kernel<<<unsigned(std::min<uint64_t>(tiles, slots)), P::kBlock, sizeof(Smem), stream>>>(a, uint32_t(tiles));
    } else {
        using Smem = OnesweepSmem<U, V, PAIRS, P, OffT>;
        auto kernel = onesweep_kernel<U, V, PAIRS, P, KIND, BYTE, ST, OffT>;
        set_smem_once(kernel, sizeof(Smem));
        kernel<<<unsigned(tiles), P::kBlock, sizeof(Smem), stream>>>(a);
    }
}

template <typename U, typename V, bool PAIRS, typename P, int KIND, typename ST, typename OffT, bool BULK>
lcpp_status launch_passes(const Layout& L, unsigned char* temp, const SortCall& c, uint64_t n,
                          const KeyCodec<U>& codec, int begin_bit, int end_bit, int passes,
                          cudaStream_t stream)
{
    static_assert(P::kTile >= kMinTile, "look-back rows are sized for kMinTile");
    Ctrl* ctrl = reinterpret_cast<Ctrl*>(temp + L.ctrl);
    const unsigned long long* bins = reinterpret_cast<const unsigned long long*>(temp + L.bins);
    ST* status[2] = {reinterpret_cast<ST*>(temp + L.status_a), reinterpret_cast<ST*>(temp + L.status_b)};
    const uint64_t tiles = ceil_div(n, uint64_t(P::kTile));
    // Control block, histograms, offsets and the pass-0 look-back rows are
    // contiguous in the layout: one memset clears them.
    LCPP_CUDA_TRY(cudaMemsetAsync(temp + L.ctrl, 0, L.status_a + size_t(tiles) * kDigits * sizeof(ST) - L.ctrl,
                                  stream));
    lcpp_status st = launch_histogram<U, KIND>(L, temp, static_cast<const U*>(c.keys_src[0]), n, codec,
                                               begin_bit, end_bit, passes, stream);
    if (st != LCPP_OK) return st;
    for (int p = 0; p < passes; ++p) {
        OnesweepArgs<U, V, ST, OffT> a;
        a.keys_in = static_cast<const U*>(c.keys_src[p]);
        a.keys_out = static_cast<U*>(c.keys_dst[p]);
        a.vals_in = static_cast<const V*>(c.vals_src[p]);
        a.vals_out = static_cast<V*>(c.vals_dst[p]);
        a.n = n;
        a.codec = codec;
        a.shift = begin_bit + kRadixBits * p;
        a.digit_mask = (1u << min(kRadixBits, end_bit - a.shift)) - 1u;
        a.bins = bins + p * kDigits;
        a.status = status[p & 1];
        a.status_next = (p + 1 < passes) ? status[(p + 1) & 1] : nullptr;
        a.tile_counter = &ctrl->tile_counter[p];
        a.error = &ctrl->error;
        diag::KernelTimer timer(1 /* LCPP_KERNEL_SORT_ONESWEEP */, n, stream);
        if (sizeof(U) == 4 && a.shift % 8 == 0 && a.digit_mask == 0xffu)
            launch_pass<U, V, PAIRS, P, KIND, ST, OffT, true, BULK>(a, tiles, stream);
        else
            launch_pass<U, V, PAIRS, P, KIND, ST, OffT, false, BULK>(a, tiles, stream);
        timer.stop();
    }
    return cudaGetLastError() == cudaSuccess ? LCPP_OK : LCPP_ERR_CUDA;
}

// Tile policies (block threads, keys per thread, look-back window, blocks
// per SM), one per key / value size class, measured on B200 (2^28 4-byte,
// 2^27 8-byte keys): 4-byte keys 448 x 28, 70.3 Gkeys/s (512 x 24: 69.0);
// 4-byte pairs 512 x 16, 46.5 (512 x 14: 44.1); 8-byte keys 384 x 16, 21.3
// (256 x 20: 19.5); pairs with an 8-byte key or value 256 x 20, 16.6
// (384 x 16: 16.3).  The persistent bulk-copy pass for 4-byte keys holds two
// tiles per block (input and staging), so its tile is 448 x 24 to keep two
// blocks per SM: 0.9095 ms per pass at 2^28 (512 x 20: 0.949; 384 x 28:
// 0.918).  A build may define these macros to other values; only the chosen
// policy of each class is compiled.
#ifndef LCPP_ONESWEEP_4B_KEYS
#define LCPP_ONESWEEP_4B_KEYS 448, 28, 8, 2
#endif
#ifndef LCPP_ONESWEEP_4B_KEYS_BULK
#define LCPP_ONESWEEP_4B_KEYS_BULK 448, 24, 8, 2
#endif
#ifndef LCPP_ONESWEEP_4B_PAIRS
#define LCPP_ONESWEEP_4B_PAIRS 512, 16, 8, 2
#endif
#ifndef LCPP_ONESWEEP_8B_KEYS
#define LCPP_ONESWEEP_8B_KEYS 384, 16, 8, 2
#endif
#ifndef LCPP_ONESWEEP_8B_PAIRS
#define LCPP_ONESWEEP_8B_PAIRS 256, 20, 8, 2
#endif

template <typename U, typename V, bool PAIRS, typename P, int KIND, bool BULK = false>
lcpp_status run_policy(const Layout& L, unsigned char* temp, const SortCall& c, uint64_t n,
                       const KeyCodec<U>& codec, int begin_bit, int end_bit, int passes, cudaStream_t stream)
{
    // 64-bit status words and offsets from 2^30 keys on
    if (L.wide)
        return launch_passes<U, V, PAIRS, P, KIND, uint64_t, uint64_t, BULK>(L, temp, c, n, codec, begin_bit,
                                                                             end_bit, passes, stream);
    return launch_passes<U, V, PAIRS, P, KIND, uint32_t, uint32_t, BULK>(L, temp, c, n, codec, begin_bit, end_bit,
                                                                         passes, stream);
}

// Every pass of the call reads its keys from a 16-byte aligned buffer, so
// the persistent pass can bulk-copy whole tiles.  One tile shape for all of
// a call's passes: each pass clears the look-back rows of the next one for
// its own tile count.
bool sources_aligned(const SortCall& c, int passes)
{
    for (int p = 0; p < passes; ++p)
        if (reinterpret_cast<uintptr_t>(c.keys_src[p]) % 16 != 0) return false;
    return true;
}

template <typename U, typename V, bool PAIRS, int KIND>
lcpp_status run_kind(const Layout& L, unsigned char* temp, const SortCall& c, uint64_t n,
                     const KeyCodec<U>& codec, int begin_bit, int end_bit, int passes, cudaStream_t stream)
{
    if constexpr (sizeof(U) == 4 && !PAIRS) {
        if (sources_aligned(c, passes))
            return run_policy<U, V, PAIRS, Policy<LCPP_ONESWEEP_4B_KEYS_BULK>, KIND, true>(
                L, temp, c, n, codec, begin_bit, end_bit, passes, stream);
        return run_policy<U, V, PAIRS, Policy<LCPP_ONESWEEP_4B_KEYS>, KIND>(L, temp, c, n, codec, begin_bit, end_bit,
                                                                            passes, stream);
    } else if constexpr (sizeof(U) == 4 && sizeof(V) == 4)
        return run_policy<U, V, PAIRS, Policy<LCPP_ONESWEEP_4B_PAIRS>, KIND>(L, temp, c, n, codec, begin_bit,
                                                                             end_bit, passes, stream);
    else if constexpr (!PAIRS)
        return run_policy<U, V, PAIRS, Policy<LCPP_ONESWEEP_8B_KEYS>, KIND>(L, temp, c, n, codec, begin_bit,
                                                                            end_bit, passes, stream);
    else
        return run_policy<U, V, PAIRS, Policy<LCPP_ONESWEEP_8B_PAIRS>, KIND>(L, temp, c, n, codec, begin_bit,
                                                                             end_bit, passes, stream);
}

template <typename U, typename V, bool PAIRS>
lcpp_status run_typed(const Layout& L, unsigned char* temp, const SortCall& c, uint64_t n,
                      lcpp_dtype kdt, bool descending, int begin_bit, int end_bit, int passes,
                      cudaStream_t stream)
{
    const KeyCodec<U> codec = make_codec<U>(kdt, descending);
    const bool is_float = kdt == LCPP_F32 || kdt == LCPP_F64;
    const bool is_plain = !is_float && codec.xor_pos == U(0);
    if (is_float) return run_kind<U, V, PAIRS, kFloat>(L, temp, c, n, codec, begin_bit, end_bit, passes, stream);
    if (is_plain) return run_kind<U, V, PAIRS, kPlain>(L, temp, c, n, codec, begin_bit, end_bit, passes, stream);
    return run_kind<U, V, PAIRS, kXor>(L, temp, c, n, codec, begin_bit, end_bit, passes, stream);
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
    diag::Range nvtx_range("lcpp DeviceRadixSort");
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
    // Element alignment of every key / value buffer.
    auto misaligned = [](const void* p, int bytes) { return (reinterpret_cast<uintptr_t>(p) % bytes) != 0; };
    if (double_buffer) {
        if (misaligned(key_bufs[0], kb) || misaligned(key_bufs[1], kb)) return LCPP_ERR_INVALID_ARG;
        if (pairs && (misaligned(val_bufs[0], vb) || misaligned(val_bufs[1], vb))) return LCPP_ERR_INVALID_ARG;
    } else {
        if (misaligned(keys_in, kb) || misaligned(keys_out, kb)) return LCPP_ERR_INVALID_ARG;
        if (pairs && (misaligned(vals_in, vb) || misaligned(vals_out, vb))) return LCPP_ERR_INVALID_ARG;
    }
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

namespace lcpp {
namespace radix {

lcpp_status wait_timeout_probe(void* temp, size_t temp_bytes, uint64_t limit_ns, cudaStream_t stream)
{
    if (!temp || (reinterpret_cast<uintptr_t>(temp) & (kTempAlign - 1)) || temp_bytes < kTempAlign)
        return LCPP_ERR_INVALID_ARG;
    if (limit_ns > kWaitLimitNs) return LCPP_ERR_INVALID_ARG;
    // word 0: the status word nothing publishes; word 1: the error word (the
    // offset lcpp_device_status reads)
    uint32_t* words = static_cast<uint32_t*>(temp);
    LCPP_CUDA_TRY(cudaMemsetAsync(words, 0, 2 * sizeof(uint32_t), stream));
    wait_timeout_probe_kernel<<<1, 32, 0, stream>>>(words, words + 1, limit_ns);
    return cudaGetLastError() == cudaSuccess ? LCPP_OK : LCPP_ERR_CUDA;
}

}  // namespace radix
}  // namespace lcpp
