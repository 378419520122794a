// dist_sort.cu -- sort, scan and reduce across the GPUs of an NCCL
// communicator, one process per GPU (include/lcpp_b200_dist.h).
//
// No counterpart in the reference, which is single-GPU: each call shards the
// path it replaces (DeviceRadixSort::SortKeys, device_radix_sort.h:399-425;
// DeviceScan::InclusiveSum / ExclusiveSum, device_scan.h:321-346;
// DeviceReduce::Reduce, device_reduce.h:229-252) over the ranks, with the
// same semantics over the concatenation of the ranks' inputs in rank order.
//
// Sort (keys only):
//   1. local onesweep sort of the rank's keys into its exchange buffer (part
//      of the caller's temp storage);
//   2. exact splitters on the device: rank r ends with global sorted
//      positions [P_r, P_{r+1}), P_r = keys held by ranks below r.  The key
//      image of position P_j is found 16 bits per round: every rank counts
//      its keys below each of the 65537 sub-bucket edges of each boundary's
//      current prefix (binary searches), one NCCL all-reduce sums the
//      counts, and a select kernel extends each prefix by the sub-bucket
//      holding P_j (2 rounds for 32-bit keys, 4 for 64-bit keys);
//   3. keys equal to a boundary key are split in rank order, so that every
//      rank receives exactly as many keys as it holds even when one value
//      fills several ranks (one NCCL all-gather of per-rank counts);
//   4. the host reads the G x (G+1) split matrix (the call's one host wait)
//      and the other ranks' exchange-buffer handles;
//   5. ranks of one host: the first level of a merge tree reads the runs
//      that belong to this rank straight from the other ranks' exchange
//      buffers over NVLink (CUDA IPC mappings, plain loads), followed by an
//      NCCL all-reduce of one word that keeps every exchange buffer intact
//      until all ranks have read it; otherwise NCCL send / receive of the
//      runs, then the merge tree over the local copies;
//   6. the remaining ceil(log2 G) - 1 merge levels run locally.  Merges take
//      ties from the run of the lower rank, so the result is the stable sort
//      of the concatenated inputs, bit for bit.
// Scan: local reduce, all-gather of the per-rank totals, carry-in (the
// totals of lower ranks, added in rank order) kept in device memory and
// read by the local scan as its initial value.  Reduce: local reduce,
// all-gather, fold in rank order from the caller's initial value.
#include <dlfcn.h>
#include <unistd.h>

#include <array>
#include <chrono>
#include <cstring>
#include <limits>
#include <type_traits>
#include <vector>

#include <cudaTypedefs.h>
#include <nccl.h>

#include "../../include/lcpp_b200_dist.h"
#include "dist.cuh"
#include "radix_sort.cuh"
#include "reduce.cuh"
#include "scan.cuh"

namespace lcpp {
namespace dist {
namespace {

// ---------------------------------------------------------------------------
// NCCL, resolved at run time: the library has no link-time dependency on it,
// and in a process that already loaded libnccl.so.2 (a PyTorch process) the
// same copy is used.
// ---------------------------------------------------------------------------
struct Nccl {
    decltype(&ncclGetUniqueId) get_unique_id = nullptr;
    decltype(&ncclCommInitRank) comm_init_rank = nullptr;
    decltype(&ncclCommDestroy) comm_destroy = nullptr;
    decltype(&ncclCommCount) comm_count = nullptr;
    decltype(&ncclCommUserRank) comm_user_rank = nullptr;
    decltype(&ncclAllReduce) all_reduce = nullptr;
    decltype(&ncclAllGather) all_gather = nullptr;
    decltype(&ncclSend) send = nullptr;
    decltype(&ncclRecv) recv = nullptr;
    decltype(&ncclGroupStart) group_start = nullptr;
    decltype(&ncclGroupEnd) group_end = nullptr;
    bool ok = false;
};

const Nccl& nccl()
{
    static const Nccl n = [] {
        Nccl r;
        void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
        if (!h) return r;
        auto sym = [&](auto& f, const char* name) {
            f = reinterpret_cast<std::remove_reference_t<decltype(f)>>(dlsym(h, name));
            return f != nullptr;
        };
        r.ok = sym(r.get_unique_id, "ncclGetUniqueId") && sym(r.comm_init_rank, "ncclCommInitRank") &&
               sym(r.comm_destroy, "ncclCommDestroy") && sym(r.comm_count, "ncclCommCount") &&
               sym(r.comm_user_rank, "ncclCommUserRank") && sym(r.all_reduce, "ncclAllReduce") &&
               sym(r.all_gather, "ncclAllGather") && sym(r.send, "ncclSend") && sym(r.recv, "ncclRecv") &&
               sym(r.group_start, "ncclGroupStart") && sym(r.group_end, "ncclGroupEnd");
        return r;
    }();
    return n;
}

// Base of the device allocation holding p (for its IPC handle), through the
// runtime's driver entry-point query.
bool allocation_base(const void* p, void** base)
{
    static const PFN_cuMemGetAddressRange get_range = [] {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &f, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            return static_cast<PFN_cuMemGetAddressRange>(nullptr);
        return reinterpret_cast<PFN_cuMemGetAddressRange>(f);
    }();
    if (!get_range) return false;
    CUdeviceptr b = 0;
    size_t size = 0;
    if (get_range(&b, &size, reinterpret_cast<CUdeviceptr>(p)) != CUDA_SUCCESS) return false;
    *base = reinterpret_cast<void*>(b);
    return true;
}

uint64_t host_hash()
{
    char name[256] = {};
    gethostname(name, sizeof(name) - 1);
    uint64_t h = 1469598103934665603ull;  // FNV-1a
    for (const char* c = name; *c; ++c) h = (h ^ uint64_t(uint8_t(*c))) * 1099511628211ull;
    return h;
}

// What every rank publishes about its part of a distributed sort.
struct alignas(16) Desc {
    unsigned char ipc[64];  // IPC handle of the allocation holding the exchange buffer
    uint64_t offset;        // exchange buffer - allocation base
    uint64_t n;             // keys this rank holds
    uint64_t host;          // hash of the host name
    uint64_t ipc_ok;        // 1 when ipc / offset are valid
    uint64_t pad[4];
};
static_assert(sizeof(Desc) == 128, "descriptor size");

constexpr int kSubBits = 16;
constexpr uint32_t kSubEdges = (1u << kSubBits) + 1;  // sub-bucket edges per boundary and round
constexpr int kMaxRanks = 64;
constexpr int kPushMinRanks = 4;  // AUTO exchange: copy-engine pushes from this many ranks on
constexpr uint64_t kMergeTileKeys = 3840;  // output keys per merge block (dist.cu)
constexpr size_t kMergeCtrlBytes = 256;    // the merge temp's control area (dist.cu)

}  // namespace
}  // namespace dist
}  // namespace lcpp

struct lcpp_comm_s {
    ncclComm_t nccl = nullptr;
    bool owned = false;
    int rank = 0, nranks = 1, device = 0;
    std::vector<std::array<unsigned char, 64>> handle;  // per rank: handle of the mapping in `base`
    std::vector<void*> base;                            // per rank: mapped allocation, or null
    cudaEvent_t ev[5] = {};
    // LCPP_EXCHANGE_COPY: one stream per receiving rank for the pushes, the
    // fork event and one join event per receiver (created at first use)
    std::vector<cudaStream_t> push_stream;
    std::vector<cudaEvent_t> push_done;
    cudaEvent_t push_fork = nullptr;
};

namespace lcpp {
namespace dist {
namespace {

#define LCPP_NCCL_TRY(expr)                              \
    do {                                                 \
        if ((expr) != ncclSuccess) return LCPP_ERR_COMM; \
    } while (0)

// ---------------------------------------------------------------------------
// Splitter kernels.
// ---------------------------------------------------------------------------
// P[j] = keys held by ranks 0..j (boundary j + 1); prefixes and counts start
// empty.
__global__ void split_init_kernel(const Desc* __restrict__ desc, int nb, uint64_t* P, uint64_t* prefix,
                                  uint64_t* below)
{
    const int j = blockIdx.x * blockDim.x + threadIdx.x;
    if (j >= nb) return;
    uint64_t p = 0;
    for (int s = 0; s <= j; ++s) p += desc[s].n;
    P[j] = p;
    prefix[j] = 0;
    below[j] = 0;
}

// Round `round`: L[j][e] = number of this rank's keys whose image is below
// sub-bucket edge e of boundary j's prefix (edge 65536 is the end of the
// prefix range, i.e. the key count when that range reaches the top).
template <typename U>
__global__ void bound_counts_kernel(const U* __restrict__ x, uint64_t n, KeyCodec<U> c,
                                    const uint64_t* __restrict__ prefix, int round, int nb, uint64_t* __restrict__ L)
{
    constexpr int kBits = int(sizeof(U)) * 8;
    const uint64_t idx = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (idx >= uint64_t(nb) * kSubEdges) return;
    const int j = int(idx / kSubEdges);
    const uint32_t e = uint32_t(idx % kSubEdges);
    const uint64_t p = prefix[j];
    const int pbits = kSubBits * round;
    const uint64_t all_ones = pbits == 0 ? 0ull : ((1ull << pbits) - 1ull);
    if (e == (1u << kSubBits) && p == all_ones) {
        L[idx] = n;
        return;
    }
    const int sh = kBits - kSubBits * (round + 1);
    const uint64_t q = ((p << kSubBits) + e) << sh;
    L[idx] = count_below<U>(x, n, U(q), false, c);
}

// G[j][e] (summed over ranks) is monotone in e; the new sub-bucket of
// boundary j is the last e in [0, 65535] with G[j][e] <= P[j].
__global__ void split_select_kernel(const uint64_t* __restrict__ G, int nb, const uint64_t* __restrict__ P,
                                    uint64_t* prefix, uint64_t* below)
{
    const int j = blockIdx.x * blockDim.x + threadIdx.x;
    if (j >= nb) return;
    const uint64_t* g = G + uint64_t(j) * kSubEdges;
    const uint64_t target = P[j];
    uint32_t lo = 0, hi = (1u << kSubBits) - 1;
    while (lo < hi) {
        const uint32_t mid = (lo + hi + 1) >> 1;
        if (g[mid] <= target)
            lo = mid;
        else
            hi = mid - 1;
    }
    below[j] = g[lo];
    prefix[j] = (prefix[j] << kSubBits) | lo;
}

// tie[j] = {keys with image < k_j, keys with image == k_j} on this rank.
template <typename U>
__global__ void tie_counts_kernel(const U* __restrict__ x, uint64_t n, KeyCodec<U> c,
                                  const uint64_t* __restrict__ prefix, int nb, uint64_t* __restrict__ tie)
{
    const int j = blockIdx.x * blockDim.x + threadIdx.x;
    if (j >= nb) return;
    const U k = U(prefix[j]);
    const uint64_t less = count_below<U>(x, n, k, false, c);
    const uint64_t le = count_below<U>(x, n, k, true, c);
    tie[2 * j] = less;
    tie[2 * j + 1] = le - less;
}

// pos[s][j]: where rank s's sorted keys split before destination j.  Keys
// equal to boundary key k_j go below boundary j in rank order until it
// holds exactly P_j keys.  A broken invariant records LCPP_ERR_INTERNAL.
__global__ void split_positions_kernel(const uint64_t* __restrict__ tie_all, const Desc* __restrict__ desc,
                                       const uint64_t* __restrict__ P, const uint64_t* __restrict__ below, int G,
                                       uint64_t* __restrict__ pos, uint32_t* error)
{
    if (threadIdx.x != 0 || blockIdx.x != 0) return;
    for (int s = 0; s < G; ++s) {
        pos[s * (G + 1)] = 0;
        pos[s * (G + 1) + G] = desc[s].n;
    }
    for (int j = 0; j < G - 1; ++j) {
        uint64_t need = P[j] - below[j];
        uint64_t sum_less = 0;
        for (int s = 0; s < G; ++s) {
            const uint64_t less = tie_all[(uint64_t(s) * (G - 1) + j) * 2];
            const uint64_t eq = tie_all[(uint64_t(s) * (G - 1) + j) * 2 + 1];
            sum_less += less;
            const uint64_t take = eq < need ? eq : need;
            need -= take;
            pos[s * (G + 1) + j + 1] = less + take;
        }
        if (need != 0 || sum_less != below[j]) report_error(error, kDevErrInternal);
    }
}

// ---------------------------------------------------------------------------
// Scan / reduce helpers.
// ---------------------------------------------------------------------------
// Integer sums wrap (two's complement), as the reference's: they are done in
// the unsigned type of the same width.
template <typename T, bool INTEGRAL = std::is_integral<T>::value>
struct WrapOf {
    using type = T;
};
template <typename T>
struct WrapOf<T, true> {
    using type = typename std::make_unsigned<T>::type;
};
template <typename T>
struct Arith {
    using W = typename WrapOf<T>::type;
    __device__ static T add(T a, T b) { return T(W(a) + W(b)); }
};

template <typename T>
__device__ __forceinline__ T apply_op(lcpp_op op, T a, T b)
{
    if (op == LCPP_OP_SUM) return Arith<T>::add(a, b);
    if (op == LCPP_OP_MIN) return b < a ? b : a;
    return a < b ? b : a;
}

// carry = totals[0] + ... + totals[rank - 1], added in rank order.
template <typename T>
__global__ void carry_kernel(const T* __restrict__ totals, int rank, T* carry)
{
    T acc = T(0);
    for (int s = 0; s < rank; ++s) acc = Arith<T>::add(acc, totals[s]);
    *carry = acc;
}

// out = init (op) parts[0] (op) ... (op) parts[G - 1], in rank order.
template <typename T>
__global__ void fold_kernel(const T* __restrict__ parts, int G, lcpp_op op, T init, T* out)
{
    T acc = init;
    for (int s = 0; s < G; ++s) acc = apply_op(op, acc, parts[s]);
    *out = acc;
}

template <typename F>
lcpp_status with_type(lcpp_dtype dt, F&& f)
{
    switch (dt) {
    case LCPP_I32: return f(int32_t{});
    case LCPP_U32: return f(uint32_t{});
    case LCPP_F32: return f(float{});
    case LCPP_I64: return f(int64_t{});
    case LCPP_U64: return f(uint64_t{});
    case LCPP_F64: return f(double{});
    default: return LCPP_ERR_UNSUPPORTED_DTYPE;
    }
}

template <typename T>
T op_identity(lcpp_op op)
{
    if (op == LCPP_OP_MIN) return std::numeric_limits<T>::max();
    if (op == LCPP_OP_MAX) return std::numeric_limits<T>::lowest();
    return T(0);
}

// ---------------------------------------------------------------------------
// Temp layouts.
// ---------------------------------------------------------------------------
struct SortLayout {
    size_t sort, sort_bytes, xbuf, rbuf, desc_send, desc_recv, bounds, P, prefix, below, tie_send, tie_recv, pos,
        barrier, splits, splits_bytes, total;
};

SortLayout sort_layout(int kb, uint64_t n, int G)
{
    SortLayout L{};
    size_t off = 0;
    auto take = [&](size_t bytes) {
        const size_t at = off;
        off = align_up(off + bytes, kTempAlign);
        return at;
    };
    // The local sort's temp comes first: its error word (temp + 4) is the
    // one lcpp_device_status reads, and the later steps report into it.
    L.sort_bytes = std::max<size_t>(radix::temp_bytes(kb, 0, n), kTempAlign);
    L.sort = take(L.sort_bytes);
    L.xbuf = take(size_t(n) * kb);
    L.rbuf = take(size_t(n) * kb);
    L.desc_send = take(sizeof(Desc));
    L.desc_recv = take(sizeof(Desc) * G);
    const int nb = G > 1 ? G - 1 : 0;
    L.bounds = take(size_t(nb) * kSubEdges * 8);
    L.P = take(8 * size_t(G));
    L.prefix = take(8 * size_t(G));
    L.below = take(8 * size_t(G));
    L.tie_send = take(16 * size_t(G));
    L.tie_recv = take(16 * size_t(G) * G);
    L.pos = take(8 * size_t(G) * (G + 1));
    L.barrier = take(8);
    // split points of one merge level: lcpp_dist_merge_batch_temp_bytes gives
    // 256 + align_up(8 (blocks + merges), 256) with blocks <= ceil(n / tile) +
    // merges and merges <= G
    L.splits_bytes = kMergeCtrlBytes + align_up(8 * size_t(ceil_div(n, kMergeTileKeys) + 2 * uint64_t(G)), kTempAlign);
    L.splits = take(L.splits_bytes);
    L.total = off;
    return L;
}

struct ScanLayout {
    size_t scan, scan_bytes, red, red_bytes, part, parts, carry, total;
};

ScanLayout scan_layout(lcpp_dtype dt, uint64_t n, int G)
{
    ScanLayout L{};
    size_t off = 0;
    auto take = [&](size_t bytes) {
        const size_t at = off;
        off = align_up(off + bytes, kTempAlign);
        return at;
    };
    L.scan_bytes = std::max<size_t>(scan::temp_bytes(dt, n), kTempAlign);  // first: error word at temp + 4
    L.scan = take(L.scan_bytes);
    L.red_bytes = std::max<size_t>(reduce::temp_bytes(dt, n), kTempAlign);
    L.red = take(L.red_bytes);
    L.part = take(8);
    L.parts = take(8 * size_t(G));
    L.carry = take(8);
    L.total = off;
    return L;
}

bool ok_temp(const void* temp) { return temp && (reinterpret_cast<uintptr_t>(temp) & (kTempAlign - 1)) == 0; }

// ---------------------------------------------------------------------------
// Merge tree over G sorted runs.
// ---------------------------------------------------------------------------
struct Run {
    const void* ptr;
    uint64_t n;
};

// One merge level: pairs of adjacent runs into `dst` (contiguous, in run
// order); an odd last run is copied.  `out` receives the new runs.
lcpp_status merge_level(const std::vector<Run>& runs, void* dst, int kb, lcpp_dtype dt, void* splits,
                        size_t splits_bytes, std::vector<Run>& out, cudaStream_t s)
{
    out.clear();
    const void* a[LCPP_MERGE_BATCH_MAX];
    const void* b[LCPP_MERGE_BATCH_MAX];
    void* o[LCPP_MERGE_BATCH_MAX];
    uint64_t na[LCPP_MERGE_BATCH_MAX], nb[LCPP_MERGE_BATCH_MAX];
    int count = 0;
    uint64_t at = 0;
    for (size_t i = 0; i < runs.size(); i += 2) {
        const Run& x = runs[i];
        const Run y = i + 1 < runs.size() ? runs[i + 1] : Run{nullptr, 0};
        a[count] = x.ptr;
        na[count] = x.n;
        b[count] = y.ptr;
        nb[count] = y.n;
        o[count] = static_cast<unsigned char*>(dst) + at * kb;
        out.push_back(Run{o[count], x.n + y.n});
        at += x.n + y.n;
        ++count;
    }
    size_t need = 0;
    lcpp_status st = lcpp_dist_merge_batch_temp_bytes(count, na, nb, &need);
    if (st != LCPP_OK) return st;
    if (need > splits_bytes) return LCPP_ERR_INTERNAL;
    return lcpp_dist_merge_sorted_batch(splits, splits_bytes, count, a, na, b, nb, o, dt,
                                        reinterpret_cast<lcpp_stream_t>(s));
}

template <typename U>
void launch_counts(const U* x, uint64_t n, lcpp_dtype dt, int G, int round, const SortLayout& L, unsigned char* t,
                   cudaStream_t s)
{
    const int nb = G - 1;
    const uint64_t threads = uint64_t(nb) * kSubEdges;
    bound_counts_kernel<U><<<unsigned(ceil_div(threads, 256)), 256, 0, s>>>(
        x, n, make_codec<U>(dt, false), reinterpret_cast<const uint64_t*>(t + L.prefix), round, nb,
        reinterpret_cast<uint64_t*>(t + L.bounds));
}

}  // namespace
}  // namespace dist
}  // namespace lcpp

using namespace lcpp;
using namespace lcpp::dist;

namespace {

lcpp_status finish_comm(ncclComm_t c, bool owned, lcpp_comm* out)
{
    const Nccl& N = nccl();
    auto* comm = new lcpp_comm_s();
    comm->nccl = c;
    comm->owned = owned;
    if (N.comm_user_rank(c, &comm->rank) != ncclSuccess || N.comm_count(c, &comm->nranks) != ncclSuccess ||
        comm->nranks < 1 || comm->nranks > kMaxRanks || cudaGetDevice(&comm->device) != cudaSuccess) {
        const lcpp_status st = comm->nranks > kMaxRanks ? LCPP_ERR_INVALID_ARG : LCPP_ERR_COMM;
        if (owned) N.comm_destroy(c);
        delete comm;
        return st;
    }
    comm->handle.assign(comm->nranks, {});
    comm->base.assign(comm->nranks, nullptr);
    for (auto& e : comm->ev) {
        if (cudaEventCreate(&e) != cudaSuccess) {
            for (auto& f : comm->ev)
                if (f) cudaEventDestroy(f);
            if (owned) N.comm_destroy(c);
            delete comm;
            return LCPP_ERR_CUDA;
        }
    }
    *out = comm;
    return LCPP_OK;
}

lcpp_status dist_scan(lcpp_comm comm, void* temp, size_t temp_bytes, const void* d_in, void* d_out,
                      uint64_t n_local, lcpp_dtype dtype, bool exclusive, lcpp_stream_t stream)
{
    diag::Range nvtx_range("lcpp dist scan");
    if (!comm) return LCPP_ERR_INVALID_ARG;
    const int tb = dtype_bytes(dtype);
    if (!tb) return LCPP_ERR_UNSUPPORTED_DTYPE;
    if (n_local && (!d_in || !d_out)) return LCPP_ERR_INVALID_ARG;
    if (!ok_temp(temp)) return LCPP_ERR_INVALID_ARG;
    const ScanLayout L = scan_layout(dtype, n_local, comm->nranks);
    if (temp_bytes < L.total) return LCPP_ERR_TEMP_TOO_SMALL;
    const Nccl& N = nccl();
    if (comm->nranks > 1 && !N.ok) return LCPP_ERR_COMM;
    unsigned char* t = static_cast<unsigned char*>(temp);
    const cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    if (n_local == 0) LCPP_CUDA_TRY(cudaMemsetAsync(t, 0, kTempAlign, s));
    // local total (0 items give 0), every rank's total, carry-in
    const uint64_t zero = 0;
    lcpp_status st = reduce::run(t + L.red, L.red_bytes, d_in, t + L.part, n_local, LCPP_OP_SUM, &zero, dtype, s);
    if (st != LCPP_OK) return st;
    if (comm->nranks > 1)
        LCPP_NCCL_TRY(N.all_gather(t + L.part, t + L.parts, size_t(tb), ncclUint8, comm->nccl, s));
    else
        LCPP_CUDA_TRY(cudaMemcpyAsync(t + L.parts, t + L.part, tb, cudaMemcpyDeviceToDevice, s));
    st = with_type(dtype, [&](auto tag) {
        using T = decltype(tag);
        carry_kernel<T><<<1, 1, 0, s>>>(reinterpret_cast<const T*>(t + L.parts), comm->rank,
                                        reinterpret_cast<T*>(t + L.carry));
        return cudaGetLastError() == cudaSuccess ? LCPP_OK : LCPP_ERR_CUDA;
    });
    if (st != LCPP_OK) return st;
    if (n_local == 0) return LCPP_OK;
    return scan::run_with_init(t + L.scan, L.scan_bytes, d_in, d_out, n_local, LCPP_OP_SUM, nullptr, t + L.carry,
                               dtype, exclusive ? 0 : 2, s);
}

}  // namespace

extern "C" {

lcpp_status lcpp_comm_unique_id(void* id)
{
    if (!id) return LCPP_ERR_INVALID_ARG;
    const Nccl& N = nccl();
    if (!N.ok) return LCPP_ERR_COMM;
    ncclUniqueId u;
    LCPP_NCCL_TRY(N.get_unique_id(&u));
    static_assert(sizeof(ncclUniqueId) == LCPP_COMM_ID_BYTES, "NCCL unique id size");
    memcpy(id, &u, sizeof(u));
    return LCPP_OK;
}

lcpp_status lcpp_comm_init(const void* id, int nranks, int rank, lcpp_comm* comm)
{
    if (!id || !comm || nranks < 1 || nranks > kMaxRanks || rank < 0 || rank >= nranks) return LCPP_ERR_INVALID_ARG;
    const Nccl& N = nccl();
    if (!N.ok) return LCPP_ERR_COMM;
    ncclUniqueId u;
    memcpy(&u, id, sizeof(u));
    ncclComm_t c = nullptr;
    LCPP_NCCL_TRY(N.comm_init_rank(&c, nranks, u, rank));
    return finish_comm(c, true, comm);
}

lcpp_status lcpp_comm_from_nccl(void* nccl_comm, lcpp_comm* comm)
{
    if (!nccl_comm || !comm) return LCPP_ERR_INVALID_ARG;
    if (!nccl().ok) return LCPP_ERR_COMM;
    return finish_comm(static_cast<ncclComm_t>(nccl_comm), false, comm);
}

lcpp_status lcpp_comm_destroy(lcpp_comm comm)
{
    if (!comm) return LCPP_ERR_INVALID_ARG;
    lcpp_status st = LCPP_OK;
    for (void* b : comm->base)
        if (b && cudaIpcCloseMemHandle(b) != cudaSuccess) st = LCPP_ERR_CUDA;
    for (auto& e : comm->ev)
        if (e) cudaEventDestroy(e);
    for (auto& e : comm->push_done)
        if (e) cudaEventDestroy(e);
    for (auto& q : comm->push_stream)
        if (q) cudaStreamDestroy(q);
    if (comm->push_fork) cudaEventDestroy(comm->push_fork);
    if (comm->owned && nccl().comm_destroy(comm->nccl) != ncclSuccess) st = LCPP_ERR_COMM;
    delete comm;
    return st;
}

lcpp_status lcpp_comm_rank(lcpp_comm comm, int* rank, int* nranks)
{
    if (!comm) return LCPP_ERR_INVALID_ARG;
    if (rank) *rank = comm->rank;
    if (nranks) *nranks = comm->nranks;
    return LCPP_OK;
}

lcpp_status lcpp_dist_sort_keys_temp_bytes(lcpp_comm comm, lcpp_dtype key_dtype, uint64_t n_local,
                                           size_t* temp_bytes)
{
    if (!comm || !temp_bytes) return LCPP_ERR_INVALID_ARG;
    const int kb = dtype_bytes(key_dtype);
    if (!kb) return LCPP_ERR_UNSUPPORTED_DTYPE;
    *temp_bytes = sort_layout(kb, n_local, comm->nranks).total;
    return LCPP_OK;
}

lcpp_status lcpp_dist_sort_keys(lcpp_comm comm, void* temp, size_t temp_bytes, const void* keys_in, void* keys_out,
                                uint64_t n_local, lcpp_dtype key_dtype, int exchange, lcpp_dist_sort_times* times,
                                lcpp_stream_t stream)
{
    diag::Range nvtx_range("lcpp dist sort_keys");
    using clock = std::chrono::steady_clock;
    if (!comm) return LCPP_ERR_INVALID_ARG;
    const int kb = dtype_bytes(key_dtype);
    if (!kb) return LCPP_ERR_UNSUPPORTED_DTYPE;
    if (exchange < LCPP_EXCHANGE_AUTO || exchange > LCPP_EXCHANGE_COPY) return LCPP_ERR_INVALID_ARG;
    if (n_local && (!keys_in || !keys_out)) return LCPP_ERR_INVALID_ARG;
    if ((reinterpret_cast<uintptr_t>(keys_in) | reinterpret_cast<uintptr_t>(keys_out)) % kb) return LCPP_ERR_INVALID_ARG;
    if (!ok_temp(temp)) return LCPP_ERR_INVALID_ARG;
    const int G = comm->nranks, r = comm->rank;
    const SortLayout L = sort_layout(kb, n_local, G);
    if (temp_bytes < L.total) return LCPP_ERR_TEMP_TOO_SMALL;
    unsigned char* t = static_cast<unsigned char*>(temp);
    {  // keys_out must not overlap temp storage
        const unsigned char* o = static_cast<const unsigned char*>(keys_out);
        if (n_local && o < t + L.total && t < o + size_t(n_local) * kb) return LCPP_ERR_INVALID_ARG;
    }
    const cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    const Nccl& N = nccl();
    uint32_t* error = reinterpret_cast<uint32_t*>(t + 4);
    const auto t0 = clock::now();
    LCPP_CUDA_TRY(cudaEventRecord(comm->ev[0], s));

    // 1. local sort (one rank: straight into the output)
    void* x = G == 1 ? keys_out : static_cast<void*>(t + L.xbuf);
    if (n_local) {
        void* no_bufs[2] = {nullptr, nullptr};
        const lcpp_status st = radix::sort(t + L.sort, L.sort_bytes, keys_in, x, nullptr, nullptr, no_bufs, no_bufs,
                                           nullptr, n_local, 0, kb * 8, 0, key_dtype, LCPP_NONE, false, false, s);
        if (st != LCPP_OK) return st;
    } else {
        LCPP_CUDA_TRY(cudaMemsetAsync(t, 0, kTempAlign, s));
    }
    LCPP_CUDA_TRY(cudaEventRecord(comm->ev[1], s));
    if (G == 1) {
        for (int e = 2; e < 5; ++e) LCPP_CUDA_TRY(cudaEventRecord(comm->ev[e], s));
        if (times) {
            LCPP_CUDA_TRY(cudaEventSynchronize(comm->ev[4]));
            lcpp_dist_sort_times z{};
            cudaEventElapsedTime(&z.local_sort_ms, comm->ev[0], comm->ev[1]);
            z.total_ms = z.local_sort_ms;
            z.host_ms = std::chrono::duration<float, std::milli>(clock::now() - t0).count();
            *times = z;
        }
        return cudaGetLastError() == cudaSuccess ? LCPP_OK : LCPP_ERR_CUDA;
    }
    if (!N.ok) return LCPP_ERR_COMM;

    // descriptors: size, host and (ranks of one host) the exchange buffer's handle
    Desc mine{};
    mine.n = n_local;
    mine.host = host_hash();
    void* base = nullptr;
    cudaIpcMemHandle_t h;
    if (exchange != LCPP_EXCHANGE_NCCL && allocation_base(x, &base) && cudaIpcGetMemHandle(&h, base) == cudaSuccess) {
        memcpy(mine.ipc, &h, sizeof(h));
        mine.offset = uint64_t(static_cast<unsigned char*>(x) - static_cast<unsigned char*>(base));
        mine.ipc_ok = 1;
    }
    cudaGetLastError();  // a failed handle query only rules the peer exchange out
    LCPP_CUDA_TRY(cudaMemcpyAsync(t + L.desc_send, &mine, sizeof(mine), cudaMemcpyHostToDevice, s));
    LCPP_NCCL_TRY(N.all_gather(t + L.desc_send, t + L.desc_recv, sizeof(Desc), ncclUint8, comm->nccl, s));

    // 2. exact splitters, 16 bits per round, on the device
    const int nb = G - 1;
    const Desc* desc_d = reinterpret_cast<const Desc*>(t + L.desc_recv);
    auto* P = reinterpret_cast<uint64_t*>(t + L.P);
    auto* prefix = reinterpret_cast<uint64_t*>(t + L.prefix);
    auto* below = reinterpret_cast<uint64_t*>(t + L.below);
    auto* bounds = reinterpret_cast<uint64_t*>(t + L.bounds);
    split_init_kernel<<<1, 64, 0, s>>>(desc_d, nb, P, prefix, below);
    const int rounds = kb * 8 / kSubBits;
    for (int round = 0; round < rounds; ++round) {
        if (kb == 4)
            launch_counts<uint32_t>(static_cast<const uint32_t*>(x), n_local, key_dtype, G, round, L, t, s);
        else
            launch_counts<uint64_t>(static_cast<const uint64_t*>(x), n_local, key_dtype, G, round, L, t, s);
        LCPP_NCCL_TRY(N.all_reduce(bounds, bounds, size_t(nb) * kSubEdges, ncclUint64, ncclSum, comm->nccl, s));
        split_select_kernel<<<1, 64, 0, s>>>(bounds, nb, P, prefix, below);
    }
    // 3. ties with the boundary keys, split in rank order
    auto* tie_send = reinterpret_cast<uint64_t*>(t + L.tie_send);
    auto* tie_recv = reinterpret_cast<uint64_t*>(t + L.tie_recv);
    if (kb == 4)
        tie_counts_kernel<uint32_t><<<1, 64, 0, s>>>(static_cast<const uint32_t*>(x), n_local,
                                                     make_codec<uint32_t>(key_dtype, false), prefix, nb, tie_send);
    else
        tie_counts_kernel<uint64_t><<<1, 64, 0, s>>>(static_cast<const uint64_t*>(x), n_local,
                                                     make_codec<uint64_t>(key_dtype, false), prefix, nb, tie_send);
    LCPP_NCCL_TRY(N.all_gather(tie_send, tie_recv, size_t(2) * nb, ncclUint64, comm->nccl, s));
    auto* pos_d = reinterpret_cast<uint64_t*>(t + L.pos);
    split_positions_kernel<<<1, 1, 0, s>>>(tie_recv, desc_d, P, below, G, pos_d, error);
    LCPP_CUDA_TRY(cudaEventRecord(comm->ev[2], s));

    // 4. the host reads the split matrix and the descriptors
    std::vector<uint64_t> pos(size_t(G) * (G + 1));
    std::vector<Desc> desc(G);
    uint32_t err = 0;
    LCPP_CUDA_TRY(cudaMemcpyAsync(pos.data(), pos_d, pos.size() * 8, cudaMemcpyDeviceToHost, s));
    LCPP_CUDA_TRY(cudaMemcpyAsync(desc.data(), desc_d, sizeof(Desc) * G, cudaMemcpyDeviceToHost, s));
    LCPP_CUDA_TRY(cudaMemcpyAsync(&err, error, 4, cudaMemcpyDeviceToHost, s));
    const auto w0 = clock::now();
    LCPP_CUDA_TRY(cudaStreamSynchronize(s));
    const auto w1 = clock::now();
    if (err) return lcpp_status(err);
    auto seg = [&](int src, int dst) { return pos[size_t(src) * (G + 1) + dst]; };
    bool mapped = exchange != LCPP_EXCHANGE_NCCL;
    for (int q = 0; q < G; ++q) mapped = mapped && desc[q].ipc_ok && desc[q].host == desc[0].host;
    if ((exchange == LCPP_EXCHANGE_PEER || exchange == LCPP_EXCHANGE_COPY) && !mapped) return LCPP_ERR_COMM;
    // AUTO on one host: copy-engine pushes from kPushMinRanks ranks on (at 4
    // ranks on B200, exchange and first merge 1.70 ms against 2.31 ms with
    // peer loads for 2^28 keys per rank), peer loads below that
    const bool push = mapped && (exchange == LCPP_EXCHANGE_COPY ||
                                 (exchange == LCPP_EXCHANGE_AUTO && G >= kPushMinRanks));
    const bool peer = mapped && !push;

    // 5. exchange and the first merge level
    std::vector<Run> runs(G), next;
    void* bufs[2];
    int levels = 0;
    while ((1 << levels) < G) ++levels;
    // rank q's exchange buffer as seen from this rank (its IPC mapping)
    auto exchange_buffer = [&](int q, const unsigned char** xq) -> lcpp_status {
        if (q == r) {
            *xq = static_cast<const unsigned char*>(x);
            return LCPP_OK;
        }
        if (!comm->base[q] || memcmp(comm->handle[q].data(), desc[q].ipc, 64) != 0) {
            if (comm->base[q]) cudaIpcCloseMemHandle(comm->base[q]);
            comm->base[q] = nullptr;
            cudaIpcMemHandle_t hq;
            memcpy(&hq, desc[q].ipc, sizeof(hq));
            void* bq = nullptr;
            if (cudaIpcOpenMemHandle(&bq, hq, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
                cudaGetLastError();
                return LCPP_ERR_COMM;
            }
            comm->base[q] = bq;
            memcpy(comm->handle[q].data(), desc[q].ipc, 64);
        }
        *xq = static_cast<const unsigned char*>(comm->base[q]) + desc[q].offset;
        return LCPP_OK;
    };
    if (peer) {
        for (int q = 0; q < G; ++q) {
            const unsigned char* xq = nullptr;
            const lcpp_status st = exchange_buffer(q, &xq);
            if (st != LCPP_OK) return st;
            runs[q] = Run{xq + seg(q, r) * kb, seg(q, r + 1) - seg(q, r)};
        }
        // levels alternate between the run buffer and the output, ending in the output
        bufs[0] = (levels & 1) ? keys_out : static_cast<void*>(t + L.rbuf);
        bufs[1] = (levels & 1) ? static_cast<void*>(t + L.rbuf) : keys_out;
        const lcpp_status st = merge_level(runs, bufs[0], kb, key_dtype, t + L.splits, L.splits_bytes, next, s);
        if (st != LCPP_OK) return st;
        runs.swap(next);
        // no rank overwrites its exchange buffer (its next call's local sort)
        // before every rank has read its runs from it
        LCPP_NCCL_TRY(N.all_reduce(t + L.barrier, t + L.barrier, 1, ncclInt32, ncclSum, comm->nccl, s));
    } else if (push) {
        // Copy engines push this rank's run for every receiver q into q's run
        // buffer (through the IPC mapping of q's temp storage, at the place
        // q expects it: runs in source-rank order), one stream per receiver
        // so the copies to different peers run at the same time; then every
        // merge level is local.  A receiver does not touch its run buffer
        // before the exchange, and the splitter collectives above order this
        // call's pushes after the receiver's previous call.
        if (comm->push_stream.empty()) {
            comm->push_stream.assign(G, nullptr);
            comm->push_done.assign(G, nullptr);
            LCPP_CUDA_TRY(cudaEventCreateWithFlags(&comm->push_fork, cudaEventDisableTiming));
            for (int q = 0; q < G; ++q) {
                LCPP_CUDA_TRY(cudaStreamCreateWithFlags(&comm->push_stream[q], cudaStreamNonBlocking));
                LCPP_CUDA_TRY(cudaEventCreateWithFlags(&comm->push_done[q], cudaEventDisableTiming));
            }
        }
        LCPP_CUDA_TRY(cudaEventRecord(comm->push_fork, s));
        for (int i = 0; i < G; ++i) {
            const int q = (r + i) % G;  // receivers in a different order on every rank
            const unsigned char* xq = nullptr;
            const lcpp_status st = exchange_buffer(q, &xq);
            if (st != LCPP_OK) return st;
            const SortLayout Lq = sort_layout(kb, desc[q].n, G);
            unsigned char* rq = const_cast<unsigned char*>(xq) - Lq.xbuf + Lq.rbuf;
            uint64_t at = 0;  // keys of lower source ranks ahead of this rank's run in q's buffer
            for (int p2 = 0; p2 < r; ++p2) at += seg(p2, q + 1) - seg(p2, q);
            const uint64_t cnt = seg(r, q + 1) - seg(r, q);
            const cudaStream_t ps = comm->push_stream[q];
            LCPP_CUDA_TRY(cudaStreamWaitEvent(ps, comm->push_fork, 0));
            if (cnt)
                LCPP_CUDA_TRY(cudaMemcpyAsync(rq + at * kb, static_cast<const unsigned char*>(x) + seg(r, q) * kb,
                                              cnt * kb, cudaMemcpyDeviceToDevice, ps));
            LCPP_CUDA_TRY(cudaEventRecord(comm->push_done[q], ps));
            LCPP_CUDA_TRY(cudaStreamWaitEvent(s, comm->push_done[q], 0));
        }
        unsigned char* rb = t + L.rbuf;
        uint64_t at = 0;
        for (int q = 0; q < G; ++q) {
            const uint64_t cnt_in = seg(q, r + 1) - seg(q, r);
            runs[q] = Run{rb + at * kb, cnt_in};
            at += cnt_in;
        }
        // every rank's pushes have landed before any rank merges its run
        // buffer or overwrites its exchange buffer (merge scratch below)
        LCPP_NCCL_TRY(N.all_reduce(t + L.barrier, t + L.barrier, 1, ncclInt32, ncclSum, comm->nccl, s));
        bufs[0] = (levels & 1) ? keys_out : x;
        bufs[1] = (levels & 1) ? x : keys_out;
        const lcpp_status st = merge_level(runs, bufs[0], kb, key_dtype, t + L.splits, L.splits_bytes, next, s);
        if (st != LCPP_OK) return st;
        runs.swap(next);
    } else {
        unsigned char* rb = t + L.rbuf;
        uint64_t at = 0;
        LCPP_NCCL_TRY(N.group_start());
        for (int q = 0; q < G; ++q) {
            const uint64_t cnt_in = seg(q, r + 1) - seg(q, r);
            const uint64_t cnt_out = seg(r, q + 1) - seg(r, q);
            if (q == r) {
                if (cnt_in)
                    LCPP_CUDA_TRY(cudaMemcpyAsync(rb + at * kb, static_cast<const unsigned char*>(x) + seg(r, r) * kb,
                                                  cnt_in * kb, cudaMemcpyDeviceToDevice, s));
            } else {
                if (cnt_out)
                    LCPP_NCCL_TRY(N.send(static_cast<const unsigned char*>(x) + seg(r, q) * kb, cnt_out * kb,
                                         ncclUint8, q, comm->nccl, s));
                if (cnt_in) LCPP_NCCL_TRY(N.recv(rb + at * kb, cnt_in * kb, ncclUint8, q, comm->nccl, s));
            }
            runs[q] = Run{rb + at * kb, cnt_in};
            at += cnt_in;
        }
        LCPP_NCCL_TRY(N.group_end());
        // the exchange buffer is free once the sends are done: levels
        // alternate between it and the output, ending in the output
        bufs[0] = (levels & 1) ? keys_out : x;
        bufs[1] = (levels & 1) ? x : keys_out;
        const lcpp_status st = merge_level(runs, bufs[0], kb, key_dtype, t + L.splits, L.splits_bytes, next, s);
        if (st != LCPP_OK) return st;
        runs.swap(next);
    }
    LCPP_CUDA_TRY(cudaEventRecord(comm->ev[3], s));

    // 6. remaining merge levels, locally
    for (int level = 1; level < levels; ++level) {
        const lcpp_status st =
            merge_level(runs, bufs[level & 1], kb, key_dtype, t + L.splits, L.splits_bytes, next, s);
        if (st != LCPP_OK) return st;
        runs.swap(next);
    }
    LCPP_CUDA_TRY(cudaEventRecord(comm->ev[4], s));
    if (times) {
        LCPP_CUDA_TRY(cudaEventSynchronize(comm->ev[4]));
        lcpp_dist_sort_times z{};
        cudaEventElapsedTime(&z.local_sort_ms, comm->ev[0], comm->ev[1]);
        cudaEventElapsedTime(&z.splitters_ms, comm->ev[1], comm->ev[2]);
        cudaEventElapsedTime(&z.exchange_merge_ms, comm->ev[2], comm->ev[3]);
        cudaEventElapsedTime(&z.local_merge_ms, comm->ev[3], comm->ev[4]);
        cudaEventElapsedTime(&z.total_ms, comm->ev[0], comm->ev[4]);
        z.host_wait_ms = std::chrono::duration<float, std::milli>(w1 - w0).count();
        z.host_ms = std::chrono::duration<float, std::milli>(clock::now() - t0).count();
        z.peer_exchange = peer ? 1 : push ? 2 : 0;
        *times = z;
    }
    return cudaGetLastError() == cudaSuccess ? LCPP_OK : LCPP_ERR_CUDA;
}

lcpp_status lcpp_dist_scan_temp_bytes(lcpp_comm comm, lcpp_dtype dtype, uint64_t n_local, size_t* temp_bytes)
{
    if (!comm || !temp_bytes) return LCPP_ERR_INVALID_ARG;
    if (!dtype_bytes(dtype)) return LCPP_ERR_UNSUPPORTED_DTYPE;
    *temp_bytes = scan_layout(dtype, n_local, comm->nranks).total;
    return LCPP_OK;
}

lcpp_status lcpp_dist_inclusive_sum(lcpp_comm comm, void* temp, size_t temp_bytes, const void* d_in, void* d_out,
                                    uint64_t n_local, lcpp_dtype dtype, lcpp_stream_t stream)
{
    return dist_scan(comm, temp, temp_bytes, d_in, d_out, n_local, dtype, false, stream);
}

lcpp_status lcpp_dist_exclusive_sum(lcpp_comm comm, void* temp, size_t temp_bytes, const void* d_in, void* d_out,
                                    uint64_t n_local, lcpp_dtype dtype, lcpp_stream_t stream)
{
    return dist_scan(comm, temp, temp_bytes, d_in, d_out, n_local, dtype, true, stream);
}

lcpp_status lcpp_dist_reduce_temp_bytes(lcpp_comm comm, lcpp_dtype dtype, uint64_t n_local, size_t* temp_bytes)
{
    return lcpp_dist_scan_temp_bytes(comm, dtype, n_local, temp_bytes);
}

lcpp_status lcpp_dist_reduce(lcpp_comm comm, void* temp, size_t temp_bytes, const void* d_in, void* d_out,
                             uint64_t n_local, lcpp_op op, const void* init, lcpp_dtype dtype, lcpp_stream_t stream)
{
    diag::Range nvtx_range("lcpp dist reduce");
    if (!comm || !init || !d_out) return LCPP_ERR_INVALID_ARG;
    const int tb = dtype_bytes(dtype);
    if (!tb) return LCPP_ERR_UNSUPPORTED_DTYPE;
    if (op != LCPP_OP_SUM && op != LCPP_OP_MIN && op != LCPP_OP_MAX) return LCPP_ERR_UNSUPPORTED_DTYPE;
    if (n_local && !d_in) return LCPP_ERR_INVALID_ARG;
    if (reinterpret_cast<uintptr_t>(d_out) % tb) return LCPP_ERR_INVALID_ARG;
    if (!ok_temp(temp)) return LCPP_ERR_INVALID_ARG;
    const ScanLayout L = scan_layout(dtype, n_local, comm->nranks);
    if (temp_bytes < L.total) return LCPP_ERR_TEMP_TOO_SMALL;
    const Nccl& N = nccl();
    if (comm->nranks > 1 && !N.ok) return LCPP_ERR_COMM;
    unsigned char* t = static_cast<unsigned char*>(temp);
    const cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    LCPP_CUDA_TRY(cudaMemsetAsync(t, 0, kTempAlign, s));  // error word of this call
    return with_type(dtype, [&](auto tag) {
        using T = decltype(tag);
        const T ident = op_identity<T>(op);
        lcpp_status st = reduce::run(t + L.red, L.red_bytes, d_in, t + L.part, n_local, op, &ident, dtype, s);
        if (st != LCPP_OK) return st;
        if (comm->nranks > 1)
            LCPP_NCCL_TRY(N.all_gather(t + L.part, t + L.parts, size_t(tb), ncclUint8, comm->nccl, s));
        else
            LCPP_CUDA_TRY(cudaMemcpyAsync(t + L.parts, t + L.part, tb, cudaMemcpyDeviceToDevice, s));
        T init_v;
        memcpy(&init_v, init, sizeof(T));
        fold_kernel<T><<<1, 1, 0, s>>>(reinterpret_cast<const T*>(t + L.parts), comm->nranks, op, init_v,
                                       static_cast<T*>(d_out));
        return cudaGetLastError() == cudaSuccess ? LCPP_OK : LCPP_ERR_CUDA;
    });
}

}  // extern "C"
