// decomposed_sort.cu -- DeviceRadixSort over decomposed (struct) keys for
// sm_100a.
//
// Replaces the decomposer overloads of DeviceRadixSort
// (src/lcpp/device/device_radix_sort.h:556-940).  The reference orders keys
// by the concatenation of their members' order-preserving bits (TwiddleIn
// and the -0.0 fold per member, src/lcpp/block/block_radix_sort.h:251-318):
// the first member is the most significant, the last occupies bits
// [0, its width); only the bit window [begin_bit, end_bit) of the
// concatenation is compared; the sort is stable (ties keep input order,
// descending included); the DoubleBuffer form writes the alternate slot and
// flips the selector once (:759-838).  The reference ranks every key against
// every other one (O(n^2), :806-823).
//
// B200 design: the window is cut into 64-bit chunks; from the least
// significant chunk up, a build kernel writes each item's chunk (through the
// current index order) and one stable onesweep pairs sort orders the
// (chunk, index) pairs, so the index order after the last chunk is the
// stable lexicographic order.  A gather kernel then copies the key structs
// (and values) into place.
#include <cstdint>
#include <cstring>

#include "../../include/lcpp_b200.h"
#include "common.cuh"
#include "radix_sort.cuh"

namespace lcpp {
namespace dec {

constexpr int kBlock = 256;

// Members as the kernels see them: byte offset, width in bytes, kind
// (0 unsigned, 1 signed, 2 float) and the position of the member's lowest
// bit in the concatenation.
struct Members {
    int count;
    uint32_t key_bytes;
    uint32_t offset[LCPP_MAX_KEY_MEMBERS];
    uint32_t bytes[LCPP_MAX_KEY_MEMBERS];
    uint32_t kind[LCPP_MAX_KEY_MEMBERS];
    uint32_t low_bit[LCPP_MAX_KEY_MEMBERS];
};

// Order-preserving bits of one member (the sort's bijection with the
// -0.0 fold), as the low bytes*8 bits of a uint64.
__device__ __forceinline__ uint64_t member_bits(const unsigned char* key, uint32_t offset, uint32_t bytes,
                                                uint32_t kind)
{
    if (bytes == 4) {
        uint32_t u;
        memcpy(&u, key + offset, 4);
        if (kind == 1) {
            u ^= 0x80000000u;
        } else if (kind == 2) {
            u = (u & 0x80000000u) ? ~u : (u ^ 0x80000000u);
            if (u == 0x7fffffffu) u = 0x80000000u;  // -0.0 sorts as +0.0
        }
        return u;
    }
    uint64_t u;
    memcpy(&u, key + offset, 8);
    constexpr uint64_t kHigh = uint64_t(1) << 63;
    if (kind == 1) {
        u ^= kHigh;
    } else if (kind == 2) {
        u = (u & kHigh) ? ~u : (u ^ kHigh);
        if (u == kHigh - 1) u = kHigh;
    }
    return u;
}

// comp[j] = bits [lo, lo + width) of the concatenation of key idx[j] (or key
// j on the first chunk), inverted within the width for descending order.
__global__ void chunk_kernel(const unsigned char* __restrict__ keys, uint64_t n, const Members m, uint32_t lo,
                             uint32_t width, int desc, const uint32_t* __restrict__ idx, uint64_t* __restrict__ comp,
                             uint32_t* __restrict__ idx_init)
{
    const uint64_t wmask = width >= 64 ? ~uint64_t(0) : ((uint64_t(1) << width) - 1);
    for (uint64_t j = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x; j < n; j += uint64_t(gridDim.x) * blockDim.x) {
        const uint64_t item = idx ? idx[j] : j;
        if (idx_init) idx_init[j] = uint32_t(j);
        const unsigned char* key = keys + item * m.key_bytes;
        uint64_t c = 0;
        for (int k = 0; k < m.count; ++k) {
            const uint32_t mlo = m.low_bit[k], mhi = mlo + m.bytes[k] * 8;
            const uint32_t olo = mlo > lo ? mlo : lo;
            const uint32_t ohi = mhi < lo + width ? mhi : lo + width;
            if (olo >= ohi) continue;
            const uint64_t bits = member_bits(key, m.offset[k], m.bytes[k], m.kind[k]);
            const uint32_t w = ohi - olo;
            const uint64_t part = (bits >> (olo - mlo)) & (w >= 64 ? ~uint64_t(0) : ((uint64_t(1) << w) - 1));
            c |= part << (olo - lo);
        }
        comp[j] = desc ? (wmask - c) : c;
    }
}

// dst[j] = src[idx[j]] for elements of `bytes` bytes (4-byte words when the
// size and both pointers allow it).
__global__ void gather_words_kernel(const uint32_t* __restrict__ src, uint32_t* __restrict__ dst,
                                    const uint32_t* __restrict__ idx, uint64_t n, uint32_t words)
{
    const uint64_t total = n * words;
    for (uint64_t t = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x; t < total;
         t += uint64_t(gridDim.x) * blockDim.x) {
        const uint64_t j = t / words, w = t - j * words;
        dst[t] = src[uint64_t(idx[j]) * words + w];
    }
}

__global__ void gather_bytes_kernel(const unsigned char* __restrict__ src, unsigned char* __restrict__ dst,
                                    const uint32_t* __restrict__ idx, uint64_t n, uint32_t bytes)
{
    const uint64_t total = n * bytes;
    for (uint64_t t = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x; t < total;
         t += uint64_t(gridDim.x) * blockDim.x) {
        const uint64_t j = t / bytes, b = t - j * bytes;
        dst[t] = src[uint64_t(idx[j]) * bytes + b];
    }
}

unsigned grid_for(uint64_t work)
{
    const uint64_t blocks = ceil_div(work, uint64_t(kBlock));
    const uint64_t cap = uint64_t(device_sm_count()) * 16;
    return unsigned(blocks < cap ? blocks : cap);
}

void gather(const void* src, void* dst, const uint32_t* idx, uint64_t n, uint32_t bytes, cudaStream_t s)
{
    const bool words = bytes % 4 == 0 && (reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst)) % 4 == 0;
    if (words)
        gather_words_kernel<<<grid_for(n * (bytes / 4)), kBlock, 0, s>>>(static_cast<const uint32_t*>(src),
                                                                        static_cast<uint32_t*>(dst), idx, n, bytes / 4);
    else
        gather_bytes_kernel<<<grid_for(n * bytes), kBlock, 0, s>>>(static_cast<const unsigned char*>(src),
                                                                  static_cast<unsigned char*>(dst), idx, n, bytes);
}

struct Layout {
    size_t sort, comp0, comp1, idx0, idx1, total;
};

Layout make_layout(uint64_t n)
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
    L.total = off;
    return L;
}

bool members_from(const lcpp_key_member* in, int count, uint32_t key_bytes, Members& m, uint32_t& total_bits)
{
    if (!in || count < 1 || count > LCPP_MAX_KEY_MEMBERS || key_bytes == 0) return false;
    m.count = count;
    m.key_bytes = key_bytes;
    total_bits = 0;
    for (int k = count - 1; k >= 0; --k) {  // the last member holds the lowest bits
        const int b = dtype_bytes(in[k].dtype);
        if (!b || uint64_t(in[k].offset) + b > key_bytes) return false;
        m.offset[k] = in[k].offset;
        m.bytes[k] = uint32_t(b);
        m.kind[k] = (in[k].dtype == LCPP_I32 || in[k].dtype == LCPP_I64) ? 1u
                  : (in[k].dtype == LCPP_F32 || in[k].dtype == LCPP_F64) ? 2u : 0u;
        m.low_bit[k] = total_bits;
        total_bits += uint32_t(b) * 8;
    }
    return true;
}

}  // namespace dec

lcpp_status decomposed_sort(void* temp, size_t temp_bytes_given, const void* keys_in, void* keys_out,
                            const void* vals_in, void* vals_out, void* key_bufs[2], void* val_bufs[2], int* selector,
                            uint64_t n, uint32_t key_bytes, const lcpp_key_member* members, int num_members,
                            int begin_bit, int end_bit, int descending, lcpp_dtype vdt, bool pairs, bool double_buffer,
                            cudaStream_t stream)
{
    diag::Range nvtx_range("lcpp DeviceRadixSort (decomposed keys)");
    using namespace dec;
    Members m{};
    uint32_t total_bits = 0;
    if (!members_from(members, num_members, key_bytes, m, total_bits)) return LCPP_ERR_INVALID_ARG;
    const int vb = pairs ? dtype_bytes(vdt) : 0;
    if (pairs && !vb) return LCPP_ERR_UNSUPPORTED_DTYPE;
    if (begin_bit < 0 || begin_bit > end_bit || uint32_t(end_bit) > total_bits) return LCPP_ERR_INVALID_ARG;
    if (n > 0xffffffffull) return LCPP_ERR_INVALID_ARG;
    if (double_buffer) {
        if (!selector || (*selector != 0 && *selector != 1)) return LCPP_ERR_INVALID_ARG;
        if (!key_bufs || !key_bufs[0] || !key_bufs[1] || (pairs && (!val_bufs || !val_bufs[0] || !val_bufs[1])))
            return LCPP_ERR_INVALID_ARG;
    }
    // nothing to do: no items; an empty bit window copies (copy form) or
    // leaves everything alone (DoubleBuffer form), device_radix_sort.h:780-787
    if (n == 0) return LCPP_OK;
    const int sel = double_buffer ? *selector : 0;
    const void* kin = double_buffer ? key_bufs[sel] : keys_in;
    void* kout = double_buffer ? key_bufs[sel ^ 1] : keys_out;
    const void* vin = pairs ? (double_buffer ? val_bufs[sel] : vals_in) : nullptr;
    void* vout = pairs ? (double_buffer ? val_bufs[sel ^ 1] : vals_out) : nullptr;
    if (!kin || !kout || (pairs && (!vin || !vout))) return LCPP_ERR_INVALID_ARG;
    if (kin == kout || (pairs && vin == vout)) return LCPP_ERR_INVALID_ARG;  // the reference rejects overlap
    if (begin_bit == end_bit) {
        if (double_buffer) return LCPP_OK;
        LCPP_CUDA_TRY(cudaMemcpyAsync(kout, kin, size_t(n) * key_bytes, cudaMemcpyDeviceToDevice, stream));
        if (pairs) LCPP_CUDA_TRY(cudaMemcpyAsync(vout, vin, size_t(n) * vb, cudaMemcpyDeviceToDevice, stream));
        return LCPP_OK;
    }
    if (!temp || (reinterpret_cast<uintptr_t>(temp) & (kTempAlign - 1))) return LCPP_ERR_INVALID_ARG;
    const Layout L = make_layout(n);
    if (temp_bytes_given < L.total) return LCPP_ERR_TEMP_TOO_SMALL;

    unsigned char* t = static_cast<unsigned char*>(temp);
    void* comp[2] = {t + L.comp0, t + L.comp1};
    void* idx[2] = {t + L.idx0, t + L.idx1};
    int csel = 0;
    for (uint32_t lo = uint32_t(begin_bit); lo < uint32_t(end_bit); lo += 64) {
        const uint32_t width = uint32_t(end_bit) - lo < 64 ? uint32_t(end_bit) - lo : 64;
        const bool first = lo == uint32_t(begin_bit);
        // chunk of each item in the current order; the first chunk also
        // seeds the index order
        chunk_kernel<<<grid_for(n), kBlock, 0, stream>>>(
            static_cast<const unsigned char*>(kin), n, m, lo, width, descending,
            first ? nullptr : static_cast<const uint32_t*>(idx[csel]), static_cast<uint64_t*>(comp[csel]),
            first ? static_cast<uint32_t*>(idx[csel]) : nullptr);
        const lcpp_status st = radix::sort(t + L.sort, radix::temp_bytes(8, 4, n), nullptr, nullptr, nullptr,
                                           nullptr, comp, idx, &csel, n, 0, int(width), 0, LCPP_U64, LCPP_U32, true,
                                           true, stream);
        if (st != LCPP_OK) return st;
    }
    const uint32_t* order = static_cast<const uint32_t*>(idx[csel]);
    gather(kin, kout, order, n, key_bytes, stream);
    if (pairs) gather(vin, vout, order, n, uint32_t(vb), stream);
    if (cudaGetLastError() != cudaSuccess) return LCPP_ERR_CUDA;
    if (double_buffer) *selector ^= 1;
    return LCPP_OK;
}

}  // namespace lcpp

extern "C" lcpp_status lcpp_radix_sort_decomposed_temp_bytes(uint64_t num_items, size_t* temp_bytes)
{
    if (!temp_bytes) return LCPP_ERR_INVALID_ARG;
    *temp_bytes = num_items ? lcpp::dec::make_layout(num_items).total : 0;
    return LCPP_OK;
}

extern "C" lcpp_status lcpp_radix_sort_decomposed_keys(void* temp, size_t temp_bytes, const void* keys_in,
                                                       void* keys_out, uint64_t num_items, uint32_t key_bytes,
                                                       const lcpp_key_member* members, int num_members, int begin_bit,
                                                       int end_bit, int descending, lcpp_stream_t stream)
{
    return lcpp::decomposed_sort(temp, temp_bytes, keys_in, keys_out, nullptr, nullptr, nullptr, nullptr, nullptr,
                                 num_items, key_bytes, members, num_members, begin_bit, end_bit, descending, LCPP_NONE,
                                 false, false, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" lcpp_status lcpp_radix_sort_decomposed_pairs(void* temp, size_t temp_bytes, const void* keys_in,
                                                        void* keys_out, const void* values_in, void* values_out,
                                                        uint64_t num_items, uint32_t key_bytes,
                                                        const lcpp_key_member* members, int num_members,
                                                        int begin_bit, int end_bit, int descending,
                                                        lcpp_dtype value_dtype, lcpp_stream_t stream)
{
    return lcpp::decomposed_sort(temp, temp_bytes, keys_in, keys_out, values_in, values_out, nullptr, nullptr,
                                 nullptr, num_items, key_bytes, members, num_members, begin_bit, end_bit, descending,
                                 value_dtype, true, false, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" lcpp_status lcpp_radix_sort_decomposed_keys_double_buffer(void* temp, size_t temp_bytes,
                                                                     void* key_buffers[2], int* selector,
                                                                     uint64_t num_items, uint32_t key_bytes,
                                                                     const lcpp_key_member* members, int num_members,
                                                                     int begin_bit, int end_bit, int descending,
                                                                     lcpp_stream_t stream)
{
    return lcpp::decomposed_sort(temp, temp_bytes, nullptr, nullptr, nullptr, nullptr, key_buffers, nullptr, selector,
                                 num_items, key_bytes, members, num_members, begin_bit, end_bit, descending, LCPP_NONE,
                                 false, true, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" lcpp_status lcpp_radix_sort_decomposed_pairs_double_buffer(
    void* temp, size_t temp_bytes, void* key_buffers[2], void* value_buffers[2], int* selector, uint64_t num_items,
    uint32_t key_bytes, const lcpp_key_member* members, int num_members, int begin_bit, int end_bit, int descending,
    lcpp_dtype value_dtype, lcpp_stream_t stream)
{
    return lcpp::decomposed_sort(temp, temp_bytes, nullptr, nullptr, nullptr, nullptr, key_buffers, value_buffers,
                                 selector, num_items, key_bytes, members, num_members, begin_bit, end_bit, descending,
                                 value_dtype, true, true, reinterpret_cast<cudaStream_t>(stream));
}
