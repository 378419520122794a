/*
 * lcpp_b200.hpp -- C++ surface of the B200 sort / scan / reduce library,
 * shaped like the reference's Device-level classes so that a caller of
 * lcpp::DeviceRadixSort / DeviceScan / DeviceReduce switches by changing
 * types, not call sites.  Header-only; every call forwards to the C ABI in
 * lcpp_b200.h.
 *
 * Mapping (reference -> here):
 *   CommandList& cmdlist            -> lcpp_stream_t stream (a cudaStream_t;
 *                                      work is enqueued, not recorded)
 *   BufferView<T>                   -> lcpp_b200::BufferView<T> {T* ptr, size}
 *   BufferView<uint> temp_storage   -> lcpp_b200::BufferView<uint32_t>
 *                                      (size in 4-byte words, like the
 *                                      reference's uint temp buffer)
 *   DoubleBuffer<T>                 -> lcpp_b200::DoubleBuffer<T> (same
 *                                      members and selector semantics)
 *   scan / reduce operators         -> SumOp, MinOp, MaxOp tag types (the
 *                                      reference's thread_operators.h names;
 *                                      DSL lambdas have no counterpart)
 *   LUISA_ASSERT on misuse          -> throws lcpp_b200::Error (status code)
 *
 * Reference: src/lcpp/device/device_radix_sort.h:351-554 (temp queries,
 * SortKeys / SortPairs / ...Descending, DoubleBuffer overloads),
 * src/lcpp/device/device_scan.h:295-420 (GetTempStorageBytes,
 * ExclusiveScan / InclusiveScan / InclusiveScanInit / ExclusiveSum /
 * InclusiveSum), src/lcpp/device/device_reduce.h:183-308
 * (GetTempStorageBytes, Reduce / Sum / Min / Max),
 * src/lcpp/common/util_type.h:57-74 (DoubleBuffer),
 * src/lcpp/device/device_segmented_radix_sort.h:28-204
 * (DeviceSegmentedRadixSort).
 */
#ifndef LCPP_B200_HPP
#define LCPP_B200_HPP

#include <algorithm>
#include <cstddef>
#include <cstdint>
#include <cstring>
#include <stdexcept>
#include <string>
#include <type_traits>

#include "lcpp_b200.h"
#ifdef __CUDACC__
#include "lcpp_b200_device.cuh"
#endif

namespace lcpp_b200 {

// ---------------------------------------------------------------------------
// Views, double buffers, operators, errors
// ---------------------------------------------------------------------------
template <typename T>
struct BufferView {
    T* ptr = nullptr;
    size_t count = 0;  // elements

    BufferView() = default;
    BufferView(T* p, size_t n) noexcept : ptr(p), count(n) {}
    [[nodiscard]] size_t size() const noexcept { return count; }
    [[nodiscard]] size_t size_bytes() const noexcept { return count * sizeof(T); }
    [[nodiscard]] T* data() const noexcept { return ptr; }
    [[nodiscard]] BufferView subview(size_t offset, size_t n) const noexcept { return {ptr + offset, n}; }
};

template <typename T>
struct DoubleBuffer {
    BufferView<T> d_buffer[2];
    int selector = 0;

    DoubleBuffer() = default;
    DoubleBuffer(BufferView<T> d_current, BufferView<T> d_alternate) noexcept
        : d_buffer{d_current, d_alternate}, selector{0}
    {
    }
    [[nodiscard]] BufferView<T> current() const noexcept { return d_buffer[selector]; }
    [[nodiscard]] BufferView<T> alternate() const noexcept { return d_buffer[selector ^ 1]; }
};

#ifdef __CUDACC__
#define LCPP_B200_HD __host__ __device__
#else
#define LCPP_B200_HD
#endif

/// The reference's SumOp / MinOp / MaxOp (thread_operators.h:49-75): tags
/// for the C ABI operators, and callable (also on the device under nvcc) for
/// the template paths.  Integer sums wrap.
struct SumOp {
    template <typename T>
    LCPP_B200_HD T operator()(T a, T b) const
    {
        if constexpr (std::is_integral_v<T>)
            return T(std::make_unsigned_t<T>(a) + std::make_unsigned_t<T>(b));
        else
            return a + b;
    }
};
struct MinOp {
    template <typename T>
    LCPP_B200_HD T operator()(T a, T b) const { return b < a ? b : a; }
};
struct MaxOp {
    template <typename T>
    LCPP_B200_HD T operator()(T a, T b) const { return a < b ? b : a; }
};

class Error : public std::runtime_error {
public:
    Error(lcpp_status s, const std::string& what)
        : std::runtime_error(what + ": " + lcpp_status_string(s)), status_(s)
    {
    }
    [[nodiscard]] lcpp_status status() const noexcept { return status_; }

private:
    lcpp_status status_;
};

namespace detail {

template <typename T>
constexpr lcpp_dtype dtype_of()
{
    if constexpr (std::is_same_v<T, float>)
        return LCPP_F32;
    else if constexpr (std::is_same_v<T, double>)
        return LCPP_F64;
    else if constexpr (std::is_integral_v<T> && sizeof(T) == 4)
        return std::is_signed_v<T> ? LCPP_I32 : LCPP_U32;
    else if constexpr (std::is_integral_v<T> && sizeof(T) == 8)
        return std::is_signed_v<T> ? LCPP_I64 : LCPP_U64;
    else
        return LCPP_NONE;
}

template <typename T>
constexpr lcpp_dtype checked_dtype()
{
    constexpr lcpp_dtype d = dtype_of<T>();
    static_assert(d != LCPP_NONE, "element types: 4- or 8-byte integers, float, double");
    return d;
}

template <typename Op>
constexpr bool is_builtin_op = std::is_same_v<Op, SumOp> || std::is_same_v<Op, MinOp> || std::is_same_v<Op, MaxOp>;

template <typename Op>
constexpr lcpp_op op_of()
{
    if constexpr (std::is_same_v<Op, SumOp>)
        return LCPP_OP_SUM;
    else if constexpr (std::is_same_v<Op, MinOp>)
        return LCPP_OP_MIN;
    else {
        static_assert(std::is_same_v<Op, MaxOp>, "operators: SumOp, MinOp, MaxOp");
        return LCPP_OP_MAX;
    }
}

inline void check(lcpp_status s, const char* what)
{
    if (s != LCPP_OK) throw Error(s, what);
}

inline void require(bool ok, const char* what)
{
    if (!ok) throw Error(LCPP_ERR_INVALID_ARG, what);
}

inline size_t temp_bytes(BufferView<uint32_t> t) { return t.size_bytes(); }

// "keys equal by ==" for the by-key scans (selects the C ABI)
struct KeyEq {};
constexpr const KeyEq* kKeyEq = nullptr;

#ifdef __CUDACC__
inline void check_cuda(cudaError_t e, const char* what)
{
    if (e == cudaErrorInvalidValue) throw Error(LCPP_ERR_INVALID_ARG, what);
    if (e != cudaSuccess) throw Error(LCPP_ERR_CUDA, what);
}
#endif

}  // namespace detail

// ---------------------------------------------------------------------------
// Decomposed (struct) keys: the reference's decomposer returns a tuple of
// the key's members, most significant first; here `members(&Key::a,
// &Key::b, ...)` names the same members by pointer-to-member.
// ---------------------------------------------------------------------------
template <typename Key>
struct Decomposer {
    lcpp_key_member member[LCPP_MAX_KEY_MEMBERS];
    int count = 0;
    int bits = 0;  // total width of the members (the default end_bit)
};

template <typename Key, typename... M>
Decomposer<Key> members(M Key::*... ptrs)
{
    static_assert(sizeof...(M) >= 1 && sizeof...(M) <= LCPP_MAX_KEY_MEMBERS, "1 to 8 key members");
    static_assert(std::is_default_constructible_v<Key>, "the key struct must be default constructible");
    Decomposer<Key> d{};
    const Key probe{};
    auto add = [&](auto ptr) {
        using T = std::remove_cv_t<std::remove_reference_t<decltype(probe.*ptr)>>;
        const auto offset = reinterpret_cast<const char*>(&(probe.*ptr)) - reinterpret_cast<const char*>(&probe);
        d.member[d.count++] = lcpp_key_member{uint32_t(offset), detail::checked_dtype<T>()};
        d.bits += int(sizeof(T) * 8);
    };
    (add(ptrs), ...);
    return d;
}

// ---------------------------------------------------------------------------
// DeviceRadixSort
// ---------------------------------------------------------------------------
class DeviceRadixSort {
public:
    /// Temp storage bytes for the decomposed-key sorts.
    static size_t GetDecomposedTempStorageBytes(uint64_t num_items)
    {
        size_t b = 0;
        detail::check(lcpp_radix_sort_decomposed_temp_bytes(num_items, &b), "GetDecomposedTempStorageBytes");
        return b;
    }

    // Decomposer overloads (device_radix_sort.h:556-940): end_bit = -1 means
    // the members' total width.
    template <typename Key>
    void SortKeys(lcpp_stream_t stream, BufferView<uint32_t> temp_storage, BufferView<Key> d_keys_in,
                  BufferView<Key> d_keys_out, uint64_t num_items, const Decomposer<Key>& decomposer,
                  int begin_bit = 0, int end_bit = -1)
    {
        dec_keys(stream, temp_storage, d_keys_in, d_keys_out, num_items, decomposer, begin_bit, end_bit, 0);
    }

    template <typename Key>
    void SortKeysDescending(lcpp_stream_t stream, BufferView<uint32_t> temp_storage, BufferView<Key> d_keys_in,
                            BufferView<Key> d_keys_out, uint64_t num_items, const Decomposer<Key>& decomposer,
                            int begin_bit = 0, int end_bit = -1)
    {
        dec_keys(stream, temp_storage, d_keys_in, d_keys_out, num_items, decomposer, begin_bit, end_bit, 1);
    }

    template <typename Key, typename ValueType>
    void SortPairs(lcpp_stream_t stream, BufferView<uint32_t> temp_storage, BufferView<Key> d_keys_in,
                   BufferView<Key> d_keys_out, BufferView<ValueType> d_values_in, BufferView<ValueType> d_values_out,
                   uint64_t num_items, const Decomposer<Key>& decomposer, int begin_bit = 0, int end_bit = -1)
    {
        dec_pairs(stream, temp_storage, d_keys_in, d_keys_out, d_values_in, d_values_out, num_items, decomposer,
                  begin_bit, end_bit, 0);
    }

    template <typename Key, typename ValueType>
    void SortPairsDescending(lcpp_stream_t stream, BufferView<uint32_t> temp_storage, BufferView<Key> d_keys_in,
                             BufferView<Key> d_keys_out, BufferView<ValueType> d_values_in,
                             BufferView<ValueType> d_values_out, uint64_t num_items,
                             const Decomposer<Key>& decomposer, int begin_bit = 0, int end_bit = -1)
    {
        dec_pairs(stream, temp_storage, d_keys_in, d_keys_out, d_values_in, d_values_out, num_items, decomposer,
                  begin_bit, end_bit, 1);
    }

    template <typename Key>
    void SortKeys(lcpp_stream_t stream, BufferView<uint32_t> temp_storage, DoubleBuffer<Key>& d_keys,
                  uint64_t num_items, const Decomposer<Key>& decomposer, int begin_bit = 0, int end_bit = -1)
    {
        dec_keys_db(stream, temp_storage, d_keys, num_items, decomposer, begin_bit, end_bit, 0);
    }

    template <typename Key>
    void SortKeysDescending(lcpp_stream_t stream, BufferView<uint32_t> temp_storage, DoubleBuffer<Key>& d_keys,
                            uint64_t num_items, const Decomposer<Key>& decomposer, int begin_bit = 0, int end_bit = -1)
    {
        dec_keys_db(stream, temp_storage, d_keys, num_items, decomposer, begin_bit, end_bit, 1);
    }

    /// Temp storage bytes for SortPairs / SortPairsDescending (0 for 0 items).
    template <typename KeyType, typename ValueType>
    static size_t GetSortPairsTempStorageBytes(uint64_t num_items)
    {
        size_t b = 0;
        detail::check(lcpp_radix_sort_pairs_temp_bytes(detail::checked_dtype<KeyType>(),
                                                       detail::checked_dtype<ValueType>(), num_items, &b),
                      "GetSortPairsTempStorageBytes");
        return b;
    }

    /// Temp storage bytes for SortKeys / SortKeysDescending (0 for 0 items).
    template <typename KeyType>
    static size_t GetSortKeysTempStorageBytes(uint64_t num_items)
    {
        size_t b = 0;
        detail::check(lcpp_radix_sort_keys_temp_bytes(detail::checked_dtype<KeyType>(), num_items, &b),
                      "GetSortKeysTempStorageBytes");
        return b;
    }

    template <typename KeyType, typename ValueType>
    void SortPairs(lcpp_stream_t stream, BufferView<uint32_t> temp_storage, BufferView<KeyType> d_keys_in,
                   BufferView<KeyType> d_keys_out, BufferView<ValueType> d_values_in,
                   BufferView<ValueType> d_values_out, uint64_t num_items, int begin_bit = 0,
                   int end_bit = sizeof(KeyType) * 8)
    {
        pairs(stream, temp_storage, d_keys_in, d_keys_out, d_values_in, d_values_out, num_items, begin_bit, end_bit,
              0);
    }

    template <typename KeyType, typename ValueType>
    void SortPairsDescending(lcpp_stream_t stream, BufferView<uint32_t> temp_storage, BufferView<KeyType> d_keys_in,
                             BufferView<KeyType> d_keys_out, BufferView<ValueType> d_values_in,
                             BufferView<ValueType> d_values_out, uint64_t num_items, int begin_bit = 0,
                             int end_bit = sizeof(KeyType) * 8)
    {
        pairs(stream, temp_storage, d_keys_in, d_keys_out, d_values_in, d_values_out, num_items, begin_bit, end_bit,
              1);
    }

    template <typename KeyType>
    void SortKeys(lcpp_stream_t stream, BufferView<uint32_t> temp_storage, BufferView<KeyType> d_keys_in,
                  BufferView<KeyType> d_keys_out, uint64_t num_items, int begin_bit = 0,
                  int end_bit = sizeof(KeyType) * 8)
    {
        keys(stream, temp_storage, d_keys_in, d_keys_out, num_items, begin_bit, end_bit, 0);
    }

    template <typename KeyType>
    void SortKeysDescending(lcpp_stream_t stream, BufferView<uint32_t> temp_storage, BufferView<KeyType> d_keys_in,
                            BufferView<KeyType> d_keys_out, uint64_t num_items, int begin_bit = 0,
                            int end_bit = sizeof(KeyType) * 8)
    {
        keys(stream, temp_storage, d_keys_in, d_keys_out, num_items, begin_bit, end_bit, 1);
    }

    // DoubleBuffer overloads: the result ends in d_keys.current() (and
    // d_values.current()); the selector flips once per 8-bit pass and is
    // unchanged for zero items or begin_bit == end_bit.
    template <typename KeyType, typename ValueType>
    void SortPairs(lcpp_stream_t stream, BufferView<uint32_t> temp_storage, DoubleBuffer<KeyType>& d_keys,
                   DoubleBuffer<ValueType>& d_values, uint64_t num_items, int begin_bit = 0,
                   int end_bit = sizeof(KeyType) * 8)
    {
        pairs_db(stream, temp_storage, d_keys, d_values, num_items, begin_bit, end_bit, 0);
    }

    template <typename KeyType, typename ValueType>
    void SortPairsDescending(lcpp_stream_t stream, BufferView<uint32_t> temp_storage, DoubleBuffer<KeyType>& d_keys,
                             DoubleBuffer<ValueType>& d_values, uint64_t num_items, int begin_bit = 0,
                             int end_bit = sizeof(KeyType) * 8)
    {
        pairs_db(stream, temp_storage, d_keys, d_values, num_items, begin_bit, end_bit, 1);
    }

    template <typename KeyType>
    void SortKeys(lcpp_stream_t stream, BufferView<uint32_t> temp_storage, DoubleBuffer<KeyType>& d_keys,
                  uint64_t num_items, int begin_bit = 0, int end_bit = sizeof(KeyType) * 8)
    {
        keys_db(stream, temp_storage, d_keys, num_items, begin_bit, end_bit, 0);
    }

    template <typename KeyType>
    void SortKeysDescending(lcpp_stream_t stream, BufferView<uint32_t> temp_storage, DoubleBuffer<KeyType>& d_keys,
                            uint64_t num_items, int begin_bit = 0, int end_bit = sizeof(KeyType) * 8)
    {
        keys_db(stream, temp_storage, d_keys, num_items, begin_bit, end_bit, 1);
    }

private:
    template <typename Key>
    static void dec_keys(lcpp_stream_t s, BufferView<uint32_t> t, BufferView<Key> ki, BufferView<Key> ko, uint64_t n,
                         const Decomposer<Key>& d, int b, int e, int desc)
    {
        detail::require(ki.size() >= n && ko.size() >= n, "SortKeys: a key view is shorter than num_items");
        detail::check(lcpp_radix_sort_decomposed_keys(t.data(), detail::temp_bytes(t), ki.data(), ko.data(), n,
                                                      uint32_t(sizeof(Key)), d.member, d.count, b,
                                                      e < 0 ? d.bits : e, desc, s),
                      "SortKeys(decomposer)");
    }

    template <typename Key, typename V>
    static void dec_pairs(lcpp_stream_t s, BufferView<uint32_t> t, BufferView<Key> ki, BufferView<Key> ko,
                          BufferView<V> vi, BufferView<V> vo, uint64_t n, const Decomposer<Key>& d, int b, int e,
                          int desc)
    {
        detail::require(ki.size() >= n && ko.size() >= n && vi.size() >= n && vo.size() >= n,
                        "SortPairs: a key or value view is shorter than num_items");
        detail::check(lcpp_radix_sort_decomposed_pairs(t.data(), detail::temp_bytes(t), ki.data(), ko.data(),
                                                       vi.data(), vo.data(), n, uint32_t(sizeof(Key)), d.member,
                                                       d.count, b, e < 0 ? d.bits : e, desc,
                                                       detail::checked_dtype<V>(), s),
                      "SortPairs(decomposer)");
    }

    template <typename Key>
    static void dec_keys_db(lcpp_stream_t s, BufferView<uint32_t> t, DoubleBuffer<Key>& kd, uint64_t n,
                            const Decomposer<Key>& d, int b, int e, int desc)
    {
        detail::require(kd.d_buffer[0].size() >= n && kd.d_buffer[1].size() >= n,
                        "SortKeys: a double-buffer view is shorter than num_items");
        void* kb[2] = {kd.d_buffer[0].data(), kd.d_buffer[1].data()};
        int sel = kd.selector;
        detail::check(lcpp_radix_sort_decomposed_keys_double_buffer(t.data(), detail::temp_bytes(t), kb, &sel, n,
                                                                    uint32_t(sizeof(Key)), d.member, d.count, b,
                                                                    e < 0 ? d.bits : e, desc, s),
                      "SortKeys(decomposer)");
        kd.selector = sel;
    }

    template <typename K, typename V>
    static void pairs(lcpp_stream_t s, BufferView<uint32_t> t, BufferView<K> ki, BufferView<K> ko, BufferView<V> vi,
                      BufferView<V> vo, uint64_t n, int b, int e, int desc)
    {
        detail::require(ki.size() >= n && ko.size() >= n && vi.size() >= n && vo.size() >= n,
                        "SortPairs: a key or value view is shorter than num_items");
        detail::check(lcpp_radix_sort_pairs(t.data(), detail::temp_bytes(t), ki.data(), ko.data(), vi.data(),
                                            vo.data(), n, b, e, desc, detail::checked_dtype<K>(),
                                            detail::checked_dtype<V>(), s),
                      "SortPairs");
    }

    template <typename K>
    static void keys(lcpp_stream_t s, BufferView<uint32_t> t, BufferView<K> ki, BufferView<K> ko, uint64_t n, int b,
                     int e, int desc)
    {
        detail::require(ki.size() >= n && ko.size() >= n, "SortKeys: a key view is shorter than num_items");
        detail::check(lcpp_radix_sort_keys(t.data(), detail::temp_bytes(t), ki.data(), ko.data(), n, b, e, desc,
                                           detail::checked_dtype<K>(), s),
                      "SortKeys");
    }

    template <typename K, typename V>
    static void pairs_db(lcpp_stream_t s, BufferView<uint32_t> t, DoubleBuffer<K>& kd, DoubleBuffer<V>& vd,
                         uint64_t n, int b, int e, int desc)
    {
        detail::require(kd.d_buffer[0].size() >= n && kd.d_buffer[1].size() >= n && vd.d_buffer[0].size() >= n &&
                            vd.d_buffer[1].size() >= n,
                        "SortPairs: a double-buffer view is shorter than num_items");
        detail::require(kd.selector == vd.selector, "SortPairs: key and value selectors differ");
        void* kb[2] = {kd.d_buffer[0].data(), kd.d_buffer[1].data()};
        void* vb[2] = {vd.d_buffer[0].data(), vd.d_buffer[1].data()};
        int sel = kd.selector;
        detail::check(lcpp_radix_sort_pairs_double_buffer(t.data(), detail::temp_bytes(t), kb, vb, &sel, n, b, e, desc,
                                                          detail::checked_dtype<K>(), detail::checked_dtype<V>(), s),
                      "SortPairs");
        kd.selector = vd.selector = sel;
    }

    template <typename K>
    static void keys_db(lcpp_stream_t s, BufferView<uint32_t> t, DoubleBuffer<K>& kd, uint64_t n, int b, int e,
                        int desc)
    {
        detail::require(kd.d_buffer[0].size() >= n && kd.d_buffer[1].size() >= n,
                        "SortKeys: a double-buffer view is shorter than num_items");
        void* kb[2] = {kd.d_buffer[0].data(), kd.d_buffer[1].data()};
        int sel = kd.selector;
        detail::check(lcpp_radix_sort_keys_double_buffer(t.data(), detail::temp_bytes(t), kb, &sel, n, b, e, desc,
                                                         detail::checked_dtype<K>(), s),
                      "SortKeys");
        kd.selector = sel;
    }
};

// ---------------------------------------------------------------------------
// DeviceSegmentedRadixSort (src/lcpp/device/device_segmented_radix_sort.h)
// ---------------------------------------------------------------------------
class DeviceSegmentedRadixSort {
public:
    template <typename KeyType>
    static size_t GetSortKeysTempStorageBytes(uint64_t num_items)
    {
        size_t b = 0;
        detail::check(lcpp_segmented_radix_sort_keys_temp_bytes(detail::checked_dtype<KeyType>(), num_items, &b),
                      "GetSortKeysTempStorageBytes");
        return b;
    }

    template <typename KeyType, typename ValueType>
    static size_t GetSortPairsTempStorageBytes(uint64_t num_items)
    {
        size_t b = 0;
        detail::check(lcpp_segmented_radix_sort_pairs_temp_bytes(detail::checked_dtype<KeyType>(),
                                                                 detail::checked_dtype<ValueType>(), num_items, &b),
                      "GetSortPairsTempStorageBytes");
        return b;
    }

    template <typename KeyType>
    void SortKeys(lcpp_stream_t stream, BufferView<uint32_t> temp_storage, BufferView<KeyType> keys_input,
                  BufferView<KeyType> keys_output, uint64_t num_items, uint64_t num_segments,
                  BufferView<uint32_t> begin_offsets, BufferView<uint32_t> end_offsets, int begin_bit = 0,
                  int end_bit = sizeof(KeyType) * 8)
    {
        keys(stream, temp_storage, keys_input, keys_output, num_items, num_segments, begin_offsets, end_offsets,
             begin_bit, end_bit, 0);
    }

    template <typename KeyType>
    void SortKeysDescending(lcpp_stream_t stream, BufferView<uint32_t> temp_storage, BufferView<KeyType> keys_input,
                            BufferView<KeyType> keys_output, uint64_t num_items, uint64_t num_segments,
                            BufferView<uint32_t> begin_offsets, BufferView<uint32_t> end_offsets, int begin_bit = 0,
                            int end_bit = sizeof(KeyType) * 8)
    {
        keys(stream, temp_storage, keys_input, keys_output, num_items, num_segments, begin_offsets, end_offsets,
             begin_bit, end_bit, 1);
    }

    template <typename KeyType, typename ValueType>
    void SortPairs(lcpp_stream_t stream, BufferView<uint32_t> temp_storage, BufferView<KeyType> keys_input,
                   BufferView<KeyType> keys_output, BufferView<ValueType> values_input,
                   BufferView<ValueType> values_output, uint64_t num_items, uint64_t num_segments,
                   BufferView<uint32_t> begin_offsets, BufferView<uint32_t> end_offsets, int begin_bit = 0,
                   int end_bit = sizeof(KeyType) * 8)
    {
        pairs(stream, temp_storage, keys_input, keys_output, values_input, values_output, num_items, num_segments,
              begin_offsets, end_offsets, begin_bit, end_bit, 0);
    }

    template <typename KeyType, typename ValueType>
    void SortPairsDescending(lcpp_stream_t stream, BufferView<uint32_t> temp_storage, BufferView<KeyType> keys_input,
                             BufferView<KeyType> keys_output, BufferView<ValueType> values_input,
                             BufferView<ValueType> values_output, uint64_t num_items, uint64_t num_segments,
                             BufferView<uint32_t> begin_offsets, BufferView<uint32_t> end_offsets, int begin_bit = 0,
                             int end_bit = sizeof(KeyType) * 8)
    {
        pairs(stream, temp_storage, keys_input, keys_output, values_input, values_output, num_items, num_segments,
              begin_offsets, end_offsets, begin_bit, end_bit, 1);
    }

    // DoubleBuffer forms: the selector flips ceil(log2 num_items) times, as
    // in the reference's segmented merge sort.
    template <typename KeyType>
    void SortKeys(lcpp_stream_t stream, BufferView<uint32_t> temp_storage, DoubleBuffer<KeyType>& keys_db,
                  uint64_t num_items, uint64_t num_segments, BufferView<uint32_t> begin_offsets,
                  BufferView<uint32_t> end_offsets, int begin_bit = 0, int end_bit = sizeof(KeyType) * 8)
    {
        keys_db_(stream, temp_storage, keys_db, num_items, num_segments, begin_offsets, end_offsets, begin_bit,
                 end_bit, 0);
    }

    template <typename KeyType>
    void SortKeysDescending(lcpp_stream_t stream, BufferView<uint32_t> temp_storage, DoubleBuffer<KeyType>& keys_db,
                            uint64_t num_items, uint64_t num_segments, BufferView<uint32_t> begin_offsets,
                            BufferView<uint32_t> end_offsets, int begin_bit = 0, int end_bit = sizeof(KeyType) * 8)
    {
        keys_db_(stream, temp_storage, keys_db, num_items, num_segments, begin_offsets, end_offsets, begin_bit,
                 end_bit, 1);
    }

    template <typename KeyType, typename ValueType>
    void SortPairs(lcpp_stream_t stream, BufferView<uint32_t> temp_storage, DoubleBuffer<KeyType>& keys_db,
                   DoubleBuffer<ValueType>& values_db, uint64_t num_items, uint64_t num_segments,
                   BufferView<uint32_t> begin_offsets, BufferView<uint32_t> end_offsets, int begin_bit = 0,
                   int end_bit = sizeof(KeyType) * 8)
    {
        pairs_db_(stream, temp_storage, keys_db, values_db, num_items, num_segments, begin_offsets, end_offsets,
                  begin_bit, end_bit, 0);
    }

    template <typename KeyType, typename ValueType>
    void SortPairsDescending(lcpp_stream_t stream, BufferView<uint32_t> temp_storage, DoubleBuffer<KeyType>& keys_db,
                             DoubleBuffer<ValueType>& values_db, uint64_t num_items, uint64_t num_segments,
                             BufferView<uint32_t> begin_offsets, BufferView<uint32_t> end_offsets, int begin_bit = 0,
                             int end_bit = sizeof(KeyType) * 8)
    {
        pairs_db_(stream, temp_storage, keys_db, values_db, num_items, num_segments, begin_offsets, end_offsets,
                  begin_bit, end_bit, 1);
    }

private:
    static void offsets(BufferView<uint32_t> b, BufferView<uint32_t> e, uint64_t nseg)
    {
        detail::require(b.size() >= nseg && e.size() >= nseg, "segment offset views are shorter than num_segments");
    }

    template <typename K>
    static void keys(lcpp_stream_t s, BufferView<uint32_t> t, BufferView<K> ki, BufferView<K> ko, uint64_t n,
                     uint64_t nseg, BufferView<uint32_t> b, BufferView<uint32_t> e, int bb, int eb, int desc)
    {
        offsets(b, e, nseg);
        detail::require(ki.size() >= n && ko.size() >= n, "SortKeys: a key view is shorter than num_items");
        detail::check(lcpp_segmented_radix_sort_keys(t.data(), detail::temp_bytes(t), ki.data(), ko.data(), n, nseg,
                                                     b.data(), e.data(), bb, eb, desc, detail::checked_dtype<K>(), s),
                      "SortKeys");
    }

    template <typename K, typename V>
    static void pairs(lcpp_stream_t s, BufferView<uint32_t> t, BufferView<K> ki, BufferView<K> ko, BufferView<V> vi,
                      BufferView<V> vo, uint64_t n, uint64_t nseg, BufferView<uint32_t> b, BufferView<uint32_t> e,
                      int bb, int eb, int desc)
    {
        offsets(b, e, nseg);
        detail::require(ki.size() >= n && ko.size() >= n && vi.size() >= n && vo.size() >= n,
                        "SortPairs: a key or value view is shorter than num_items");
        detail::check(lcpp_segmented_radix_sort_pairs(t.data(), detail::temp_bytes(t), ki.data(), ko.data(),
                                                      vi.data(), vo.data(), n, nseg, b.data(), e.data(), bb, eb, desc,
                                                      detail::checked_dtype<K>(), detail::checked_dtype<V>(), s),
                      "SortPairs");
    }

    template <typename K>
    static void keys_db_(lcpp_stream_t s, BufferView<uint32_t> t, DoubleBuffer<K>& kd, uint64_t n, uint64_t nseg,
                         BufferView<uint32_t> b, BufferView<uint32_t> e, int bb, int eb, int desc)
    {
        offsets(b, e, nseg);
        detail::require(kd.d_buffer[0].size() >= n && kd.d_buffer[1].size() >= n,
                        "SortKeys: a double-buffer view is shorter than num_items");
        void* kb[2] = {kd.d_buffer[0].data(), kd.d_buffer[1].data()};
        int sel = kd.selector;
        detail::check(lcpp_segmented_radix_sort_keys_double_buffer(t.data(), detail::temp_bytes(t), kb, &sel, n,
                                                                   nseg, b.data(), e.data(), bb, eb, desc,
                                                                   detail::checked_dtype<K>(), s),
                      "SortKeys");
        kd.selector = sel;
    }

    template <typename K, typename V>
    static void pairs_db_(lcpp_stream_t s, BufferView<uint32_t> t, DoubleBuffer<K>& kd, DoubleBuffer<V>& vd,
                          uint64_t n, uint64_t nseg, BufferView<uint32_t> b, BufferView<uint32_t> e, int bb, int eb,
                          int desc)
    {
        offsets(b, e, nseg);
        detail::require(kd.d_buffer[0].size() >= n && kd.d_buffer[1].size() >= n && vd.d_buffer[0].size() >= n &&
                            vd.d_buffer[1].size() >= n,
                        "SortPairs: a double-buffer view is shorter than num_items");
        detail::require(kd.selector == vd.selector, "SortPairs: key and value selectors differ");
        void* kb[2] = {kd.d_buffer[0].data(), kd.d_buffer[1].data()};
        void* vb[2] = {vd.d_buffer[0].data(), vd.d_buffer[1].data()};
        int sel = kd.selector;
        detail::check(lcpp_segmented_radix_sort_pairs_double_buffer(t.data(), detail::temp_bytes(t), kb, vb, &sel, n,
                                                                    nseg, b.data(), e.data(), bb, eb, desc,
                                                                    detail::checked_dtype<K>(),
                                                                    detail::checked_dtype<V>(), s),
                      "SortPairs");
        kd.selector = vd.selector = sel;
    }
};

// ---------------------------------------------------------------------------
// DeviceScan
// ---------------------------------------------------------------------------
class DeviceScan {
public:
    /// Temp storage bytes for ExclusiveScan / InclusiveScan / ExclusiveSum /
    /// InclusiveSum (0 for 0 items).
    template <typename T>
    static size_t GetTempStorageBytes(uint64_t num_items)
    {
        size_t b = 0;
        detail::check(lcpp_scan_temp_bytes(detail::checked_dtype<T>(), num_items, &b), "GetTempStorageBytes");
#ifdef __CUDACC__
        b = std::max(b, device::by_key_temp_bytes(num_items, sizeof(T)));  // user operators
#endif
        return b;
    }

    /// ScanOp: SumOp / MinOp / MaxOp (C ABI), or under nvcc any associative
    /// __device__ callable (operand order is kept).
    template <typename T, typename ScanOp>
    void ExclusiveScan(lcpp_stream_t stream, BufferView<uint32_t> temp_storage, BufferView<T> d_in,
                       BufferView<T> d_out, uint64_t num_items, ScanOp op, T initial_value)
    {
        views(d_in, d_out, num_items);
        if constexpr (!detail::is_builtin_op<ScanOp>) {
            user_scan(stream, temp_storage, d_in, d_out, num_items, 0, initial_value, op, "ExclusiveScan");
        } else {
            detail::check(lcpp_scan_exclusive(temp_storage.data(), detail::temp_bytes(temp_storage), d_in.data(),
                                              d_out.data(), num_items, detail::op_of<ScanOp>(), &initial_value,
                                              detail::checked_dtype<T>(), stream),
                          "ExclusiveScan");
        }
    }

    /// Inclusive scan without an initial value (CUB semantics).
    template <typename T, typename ScanOp>
    void InclusiveScan(lcpp_stream_t stream, BufferView<uint32_t> temp_storage, BufferView<T> d_in,
                       BufferView<T> d_out, uint64_t num_items, ScanOp op)
    {
        views(d_in, d_out, num_items);
        if constexpr (!detail::is_builtin_op<ScanOp>) {
            user_scan(stream, temp_storage, d_in, d_out, num_items, 1, T{}, op, "InclusiveScan");
        } else {
            detail::check(lcpp_scan_inclusive(temp_storage.data(), detail::temp_bytes(temp_storage), d_in.data(),
                                              d_out.data(), num_items, detail::op_of<ScanOp>(),
                                              detail::checked_dtype<T>(), stream),
                          "InclusiveScan");
        }
    }

    /// Inclusive scan with the initial value folded in front.
    template <typename T, typename ScanOp>
    void InclusiveScan(lcpp_stream_t stream, BufferView<uint32_t> temp_storage, BufferView<T> d_in,
                       BufferView<T> d_out, uint64_t num_items, ScanOp op, T initial_value)
    {
        InclusiveScanInit(stream, temp_storage, d_in, d_out, num_items, op, initial_value);
    }

    template <typename T, typename ScanOp>
    void InclusiveScanInit(lcpp_stream_t stream, BufferView<uint32_t> temp_storage, BufferView<T> d_in,
                           BufferView<T> d_out, uint64_t num_items, ScanOp op, T initial_value)
    {
        views(d_in, d_out, num_items);
        if constexpr (!detail::is_builtin_op<ScanOp>) {
            user_scan(stream, temp_storage, d_in, d_out, num_items, 2, initial_value, op, "InclusiveScanInit");
        } else {
            detail::check(lcpp_scan_inclusive_init(temp_storage.data(), detail::temp_bytes(temp_storage),
                                                   d_in.data(), d_out.data(), num_items, detail::op_of<ScanOp>(),
                                                   &initial_value, detail::checked_dtype<T>(), stream),
                          "InclusiveScanInit");
        }
    }

    template <typename T>
    void ExclusiveSum(lcpp_stream_t stream, BufferView<uint32_t> temp_storage, BufferView<T> d_in,
                      BufferView<T> d_out, uint64_t num_items)
    {
        views(d_in, d_out, num_items);
        detail::check(lcpp_scan_exclusive_sum(temp_storage.data(), detail::temp_bytes(temp_storage), d_in.data(),
                                              d_out.data(), num_items, detail::checked_dtype<T>(), stream),
                      "ExclusiveSum");
    }

    template <typename T>
    void InclusiveSum(lcpp_stream_t stream, BufferView<uint32_t> temp_storage, BufferView<T> d_in,
                      BufferView<T> d_out, uint64_t num_items)
    {
        views(d_in, d_out, num_items);
        detail::check(lcpp_scan_inclusive_sum(temp_storage.data(), detail::temp_bytes(temp_storage), d_in.data(),
                                              d_out.data(), num_items, detail::checked_dtype<T>(), stream),
                      "InclusiveSum");
    }

    // ---- by key (device_scan.h:310-597; argument order as the reference's).
    // ScanOp: SumOp / MinOp / MaxOp through the C ABI; under nvcc also any
    // __device__ callable, and the overloads with an EqualityOp (a
    // __device__ callable "same segment"), through lcpp_b200_device.cuh.

    template <typename K, typename V>
    static size_t GetScanByKeyTempStorageBytes(uint64_t num_items)
    {
        size_t b = 0;
        detail::check(lcpp_scan_by_key_temp_bytes(detail::checked_dtype<K>(), detail::checked_dtype<V>(), num_items,
                                                  &b),
                      "GetScanByKeyTempStorageBytes");
        return b;
    }

    template <typename K, typename V, typename ScanOp>
    void ExclusiveScanByKey(lcpp_stream_t stream, BufferView<uint32_t> temp_storage, BufferView<K> d_keys_in,
                            BufferView<V> d_values_in, BufferView<V> d_values_out, ScanOp scan_op, uint64_t num_items,
                            V initial_value)
    {
        by_key(stream, temp_storage, d_keys_in, d_values_in, d_values_out, scan_op, num_items, 0, initial_value,
               detail::kKeyEq, "ExclusiveScanByKey");
    }

    template <typename K, typename V, typename ScanOp>
    void InclusiveScanByKey(lcpp_stream_t stream, BufferView<uint32_t> temp_storage, BufferView<K> d_keys_in,
                            BufferView<V> d_values_in, BufferView<V> d_values_out, ScanOp scan_op, uint64_t num_items)
    {
        by_key(stream, temp_storage, d_keys_in, d_values_in, d_values_out, scan_op, num_items, 1, V{},
               detail::kKeyEq, "InclusiveScanByKey");
    }

    /// The reference's extension: init prepended to every segment.
    template <typename K, typename V, typename ScanOp>
    void InclusiveScanByKey(lcpp_stream_t stream, BufferView<uint32_t> temp_storage, BufferView<K> d_keys_in,
                            BufferView<V> d_values_in, BufferView<V> d_values_out, ScanOp scan_op, uint64_t num_items,
                            V initial_value)
    {
        by_key(stream, temp_storage, d_keys_in, d_values_in, d_values_out, scan_op, num_items, 2, initial_value,
               detail::kKeyEq, "InclusiveScanByKey");
    }

    template <typename K, typename V>
    void ExclusiveSumByKey(lcpp_stream_t stream, BufferView<uint32_t> temp_storage, BufferView<K> d_keys_in,
                           BufferView<V> d_values_in, BufferView<V> d_values_out, uint64_t num_items)
    {
        ExclusiveScanByKey(stream, temp_storage, d_keys_in, d_values_in, d_values_out, SumOp{}, num_items, V(0));
    }

    template <typename K, typename V>
    void InclusiveSumByKey(lcpp_stream_t stream, BufferView<uint32_t> temp_storage, BufferView<K> d_keys_in,
                           BufferView<V> d_values_in, BufferView<V> d_values_out, uint64_t num_items)
    {
        InclusiveScanByKey(stream, temp_storage, d_keys_in, d_values_in, d_values_out, SumOp{}, num_items);
    }

#ifdef __CUDACC__
    template <typename K, typename V, typename ScanOp, typename EqualityOp>
    void ExclusiveScanByKey(lcpp_stream_t stream, BufferView<uint32_t> temp_storage, BufferView<K> d_keys_in,
                            BufferView<V> d_values_in, BufferView<V> d_values_out, ScanOp scan_op, uint64_t num_items,
                            V initial_value, EqualityOp equality_op)
    {
        by_key(stream, temp_storage, d_keys_in, d_values_in, d_values_out, scan_op, num_items, 0, initial_value,
               &equality_op, "ExclusiveScanByKey");
    }

    template <typename K, typename V, typename ScanOp, typename EqualityOp,
              typename = std::enable_if_t<!std::is_arithmetic_v<EqualityOp>>>
    void InclusiveScanByKey(lcpp_stream_t stream, BufferView<uint32_t> temp_storage, BufferView<K> d_keys_in,
                            BufferView<V> d_values_in, BufferView<V> d_values_out, ScanOp scan_op, uint64_t num_items,
                            EqualityOp equality_op)
    {
        by_key(stream, temp_storage, d_keys_in, d_values_in, d_values_out, scan_op, num_items, 1, V{}, &equality_op,
               "InclusiveScanByKey");
    }

    template <typename K, typename V, typename ScanOp, typename EqualityOp>
    void InclusiveScanByKey(lcpp_stream_t stream, BufferView<uint32_t> temp_storage, BufferView<K> d_keys_in,
                            BufferView<V> d_values_in, BufferView<V> d_values_out, ScanOp scan_op, uint64_t num_items,
                            V initial_value, EqualityOp equality_op)
    {
        by_key(stream, temp_storage, d_keys_in, d_values_in, d_values_out, scan_op, num_items, 2, initial_value,
               &equality_op, "InclusiveScanByKey");
    }

    template <typename K, typename V, typename EqualityOp>
    void ExclusiveSumByKey(lcpp_stream_t stream, BufferView<uint32_t> temp_storage, BufferView<K> d_keys_in,
                           BufferView<V> d_values_in, BufferView<V> d_values_out, uint64_t num_items,
                           EqualityOp equality_op)
    {
        ExclusiveScanByKey(stream, temp_storage, d_keys_in, d_values_in, d_values_out, SumOp{}, num_items, V(0),
                           equality_op);
    }

    template <typename K, typename V, typename EqualityOp>
    void InclusiveSumByKey(lcpp_stream_t stream, BufferView<uint32_t> temp_storage, BufferView<K> d_keys_in,
                           BufferView<V> d_values_in, BufferView<V> d_values_out, uint64_t num_items,
                           EqualityOp equality_op)
    {
        InclusiveScanByKey(stream, temp_storage, d_keys_in, d_values_in, d_values_out, SumOp{}, num_items,
                           equality_op);
    }
#endif

private:
    // A user scan operator: the by-key pass over one segment (nvcc only).
    template <typename T, typename Op>
    void user_scan(lcpp_stream_t stream, BufferView<uint32_t> temp_storage, BufferView<T> in, BufferView<T> out,
                   uint64_t n, int mode, T init, Op op, const char* what)
    {
#ifdef __CUDACC__
        detail::check_cuda(device::scan(temp_storage.data(), detail::temp_bytes(temp_storage), in.data(), out.data(),
                                        n, mode, init, op, reinterpret_cast<cudaStream_t>(stream)),
                           what);
#else
        (void)stream, (void)temp_storage, (void)in, (void)out, (void)n, (void)mode, (void)init, (void)op, (void)what;
        static_assert(detail::is_builtin_op<Op>, "scan operators other than SumOp / MinOp / MaxOp need nvcc");
#endif
    }

    // mode 0 exclusive, 1 inclusive, 2 inclusive with init; eq: a
    // detail::KeyEq pointer for == (the C ABI), else the user's equality.
    template <typename K, typename V, typename ScanOp, typename EqualityOp>
    void by_key(lcpp_stream_t stream, BufferView<uint32_t> temp_storage, BufferView<K> keys, BufferView<V> vin,
                BufferView<V> vout, ScanOp scan_op, uint64_t n, int mode, V init, const EqualityOp* eq,
                const char* what)
    {
        detail::require(keys.size() >= n && vin.size() >= n && vout.size() >= n,
                        "DeviceScan: a key or value view is shorter than num_items");
        constexpr bool custom_eq = !std::is_same_v<EqualityOp, detail::KeyEq>;
        if constexpr (detail::is_builtin_op<ScanOp> && !custom_eq) {
            (void)scan_op;
            (void)eq;
            const void* tb = temp_storage.data();
            const size_t nb = detail::temp_bytes(temp_storage);
            const lcpp_dtype kd = detail::checked_dtype<K>(), vd = detail::checked_dtype<V>();
            const lcpp_op op = detail::op_of<ScanOp>();
            lcpp_status s;
            if (mode == 0)
                s = lcpp_scan_exclusive_by_key(const_cast<void*>(tb), nb, keys.data(), vin.data(), vout.data(), n, op,
                                               &init, kd, vd, stream);
            else if (mode == 1)
                s = lcpp_scan_inclusive_by_key(const_cast<void*>(tb), nb, keys.data(), vin.data(), vout.data(), n, op,
                                               kd, vd, stream);
            else
                s = lcpp_scan_inclusive_by_key_init(const_cast<void*>(tb), nb, keys.data(), vin.data(), vout.data(),
                                                    n, op, &init, kd, vd, stream);
            detail::check(s, what);
        } else {
#ifdef __CUDACC__
            const auto st = reinterpret_cast<cudaStream_t>(stream);
            cudaError_t e;
            if constexpr (custom_eq)
                e = device::scan_by_key(temp_storage.data(), detail::temp_bytes(temp_storage), keys.data(), vin.data(),
                                        vout.data(), n, mode, init, scan_op, *eq, st);
            else
                e = device::scan_by_key(temp_storage.data(), detail::temp_bytes(temp_storage), keys.data(), vin.data(),
                                        vout.data(), n, mode, init, scan_op, device::EqualTo{}, st);
            detail::check_cuda(e, what);
#else
            static_assert(detail::is_builtin_op<ScanOp>, "custom scan operators need nvcc (lcpp_b200_device.cuh)");
#endif
        }
    }

    template <typename T>
    static void views(BufferView<T> i, BufferView<T> o, uint64_t n)
    {
        detail::require(i.size() >= n && o.size() >= n, "DeviceScan: a view is shorter than num_items");
    }
};

// ---------------------------------------------------------------------------
// DeviceReduce
// ---------------------------------------------------------------------------
class DeviceReduce {
public:
    /// Temp storage bytes for Reduce / Sum / Min / Max.
    template <typename T>
    static size_t GetTempStorageBytes(uint64_t num_items)
    {
        size_t b = 0;
        detail::check(lcpp_reduce_temp_bytes(detail::checked_dtype<T>(), num_items, &b), "GetTempStorageBytes");
#ifdef __CUDACC__
        if (num_items) b = std::max(b, device::reduce_temp_bytes(sizeof(T)));  // user operators
#endif
        return b;
    }

    /// d_out[0] = initial_value op d_in[0] op ... (initial_value alone for 0
    /// items).  ReduceOp: SumOp / MinOp / MaxOp (C ABI), or under nvcc any
    /// associative and commutative __device__ callable.
    template <typename T, typename ReduceOp>
    void Reduce(lcpp_stream_t stream, BufferView<uint32_t> temp_storage, BufferView<T> d_in, BufferView<T> d_out,
                uint64_t num_items, ReduceOp op, T initial_value)
    {
        views(d_in, d_out, num_items);
        if constexpr (!detail::is_builtin_op<ReduceOp>) {
#ifdef __CUDACC__
            detail::check_cuda(device::reduce(temp_storage.data(), detail::temp_bytes(temp_storage), d_in.data(),
                                              d_out.data(), num_items, op, initial_value,
                                              reinterpret_cast<cudaStream_t>(stream)),
                               "Reduce");
#else
            static_assert(detail::is_builtin_op<ReduceOp>, "reduce operators other than SumOp / MinOp / MaxOp need nvcc");
#endif
        } else {
            (void)op;
            detail::check(lcpp_reduce(temp_storage.data(), detail::temp_bytes(temp_storage), d_in.data(),
                                      d_out.data(), num_items, detail::op_of<ReduceOp>(), &initial_value,
                                      detail::checked_dtype<T>(), stream),
                          "Reduce");
        }
    }

#ifdef __CUDACC__
    /// TransformReduce (device_reduce.h:493-516): d_out[0] = initial_value op
    /// transform(d_in[0]) op ...; transform and op are __device__ callables,
    /// op associative and commutative.  nvcc only.
    template <typename T, typename ReduceOp, typename TransformOp>
    void TransformReduce(lcpp_stream_t stream, BufferView<uint32_t> temp_storage, BufferView<T> d_in,
                         BufferView<T> d_out, uint64_t num_items, ReduceOp reduce_op, TransformOp transform_op,
                         T initial_value)
    {
        views(d_in, d_out, num_items);
        detail::check_cuda(device::transform_reduce(temp_storage.data(), detail::temp_bytes(temp_storage), d_in.data(),
                                                    d_out.data(), num_items, reduce_op, transform_op, initial_value,
                                                    reinterpret_cast<cudaStream_t>(stream)),
                           "TransformReduce");
    }
#endif

    template <typename T>
    void Sum(lcpp_stream_t stream, BufferView<uint32_t> temp_storage, BufferView<T> d_in, BufferView<T> d_out,
             uint64_t num_items)
    {
        views(d_in, d_out, num_items);
        detail::check(lcpp_reduce_sum(temp_storage.data(), detail::temp_bytes(temp_storage), d_in.data(),
                                      d_out.data(), num_items, detail::checked_dtype<T>(), stream),
                      "Sum");
    }

    template <typename T>
    void Min(lcpp_stream_t stream, BufferView<uint32_t> temp_storage, BufferView<T> d_in, BufferView<T> d_out,
             uint64_t num_items)
    {
        views(d_in, d_out, num_items);
        detail::check(lcpp_reduce_min(temp_storage.data(), detail::temp_bytes(temp_storage), d_in.data(),
                                      d_out.data(), num_items, detail::checked_dtype<T>(), stream),
                      "Min");
    }

    template <typename T>
    void Max(lcpp_stream_t stream, BufferView<uint32_t> temp_storage, BufferView<T> d_in, BufferView<T> d_out,
             uint64_t num_items)
    {
        views(d_in, d_out, num_items);
        detail::check(lcpp_reduce_max(temp_storage.data(), detail::temp_bytes(temp_storage), d_in.data(),
                                      d_out.data(), num_items, detail::checked_dtype<T>(), stream),
                      "Max");
    }

    /// Temp storage bytes for ReduceByKey (device_reduce.h:208-223).
    template <typename K, typename V>
    static size_t GetReduceByKeyTempStorageBytes(uint64_t num_items)
    {
        size_t b = 0;
        detail::check(lcpp_reduce_by_key_temp_bytes(detail::checked_dtype<K>(), detail::checked_dtype<V>(),
                                                    num_items, &b),
                      "GetReduceByKeyTempStorageBytes");
        return b;
    }

    /// One (first key, aggregate) per run of equal consecutive keys, and the
    /// run count (device_reduce.h:437-491).  ReduceOp: SumOp / MinOp / MaxOp,
    /// or under nvcc any __device__ callable.
    template <typename K, typename V, typename ReduceOp>
    void ReduceByKey(lcpp_stream_t stream, BufferView<uint32_t> temp_storage, BufferView<K> d_keys_in,
                     BufferView<V> d_values_in, BufferView<K> d_unique_out, BufferView<V> d_aggregates_out,
                     BufferView<uint32_t> d_num_runs_out, ReduceOp reduce_op, uint64_t num_elements)
    {
        detail::require(d_keys_in.size() >= num_elements && d_values_in.size() >= num_elements &&
                            d_num_runs_out.size() >= 1,
                        "DeviceReduce: a by-key input view is shorter than num_elements, or no run-count view");
        detail::require(num_elements == 0 || (d_unique_out.size() >= 1 && d_aggregates_out.size() >= 1),
                        "DeviceReduce: a by-key output view is empty");
        if constexpr (detail::is_builtin_op<ReduceOp>) {
            (void)reduce_op;
            detail::check(lcpp_reduce_by_key(temp_storage.data(), detail::temp_bytes(temp_storage), d_keys_in.data(),
                                             d_values_in.data(), d_unique_out.data(), d_aggregates_out.data(),
                                             d_num_runs_out.data(), num_elements, detail::op_of<ReduceOp>(),
                                             detail::checked_dtype<K>(), detail::checked_dtype<V>(), stream),
                          "ReduceByKey");
        } else {
#ifdef __CUDACC__
            detail::check_cuda(device::reduce_by_key(temp_storage.data(), detail::temp_bytes(temp_storage),
                                                     d_keys_in.data(), d_values_in.data(), d_unique_out.data(),
                                                     d_aggregates_out.data(), d_num_runs_out.data(), num_elements,
                                                     reduce_op, device::EqualTo{},
                                                     reinterpret_cast<cudaStream_t>(stream)),
                               "ReduceByKey");
#else
            static_assert(detail::is_builtin_op<ReduceOp>, "custom reduce operators need nvcc (lcpp_b200_device.cuh)");
#endif
        }
    }

    /// Temp storage bytes for ArgMin / ArgMax (the reference's
    /// GetArgTempStorageBytes, device_reduce.h:192-204).
    template <typename T>
    static size_t GetArgTempStorageBytes(uint64_t num_items)
    {
        size_t b = 0;
        detail::check(lcpp_reduce_arg_temp_bytes(detail::checked_dtype<T>(), num_items, &b), "GetArgTempStorageBytes");
        return b;
    }

    /// d_out[0] = the minimum, d_index_out[0] = the first index holding it;
    /// 0 items: max() and index 1 (device_reduce.h:310-358).
    template <typename T>
    void ArgMin(lcpp_stream_t stream, BufferView<uint32_t> temp_storage, BufferView<T> d_in, BufferView<T> d_out,
                BufferView<uint32_t> d_index_out, uint64_t num_items)
    {
        arg_views(d_in, d_out, d_index_out, num_items);
        detail::check(lcpp_reduce_argmin(temp_storage.data(), detail::temp_bytes(temp_storage), d_in.data(),
                                         d_out.data(), d_index_out.data(), num_items, detail::checked_dtype<T>(),
                                         stream),
                      "ArgMin");
    }

    /// d_out[0] = the maximum, d_index_out[0] = the first index holding it;
    /// 0 items: lowest() and index 1 (device_reduce.h:373-422).
    template <typename T>
    void ArgMax(lcpp_stream_t stream, BufferView<uint32_t> temp_storage, BufferView<T> d_in, BufferView<T> d_out,
                BufferView<uint32_t> d_index_out, uint64_t num_items)
    {
        arg_views(d_in, d_out, d_index_out, num_items);
        detail::check(lcpp_reduce_argmax(temp_storage.data(), detail::temp_bytes(temp_storage), d_in.data(),
                                         d_out.data(), d_index_out.data(), num_items, detail::checked_dtype<T>(),
                                         stream),
                      "ArgMax");
    }

#ifdef __CUDACC__
    /// The comparator overloads (device_reduce.h:360-371, :424-434):
    /// `compare` is a __device__ callable "a orders before b"; the result is
    /// the first index of the extreme equivalence class.  Needs nvcc; the
    /// kernel is instantiated in the caller's translation unit
    /// (lcpp_b200_device.cuh).
    template <typename T, typename Compare>
    void ArgMin(lcpp_stream_t stream, BufferView<uint32_t> temp_storage, BufferView<T> d_in, BufferView<T> d_out,
                BufferView<uint32_t> d_index_out, uint64_t num_items, Compare compare)
    {
        arg_views(d_in, d_out, d_index_out, num_items);
        detail::check_cuda(device::ArgMin(temp_storage.data(), detail::temp_bytes(temp_storage), d_in.data(),
                                          d_out.data(), d_index_out.data(), num_items, compare,
                                          reinterpret_cast<cudaStream_t>(stream)),
                           "ArgMin");
    }

    template <typename T, typename Compare>
    void ArgMax(lcpp_stream_t stream, BufferView<uint32_t> temp_storage, BufferView<T> d_in, BufferView<T> d_out,
                BufferView<uint32_t> d_index_out, uint64_t num_items, Compare compare)
    {
        arg_views(d_in, d_out, d_index_out, num_items);
        detail::check_cuda(device::ArgMax(temp_storage.data(), detail::temp_bytes(temp_storage), d_in.data(),
                                          d_out.data(), d_index_out.data(), num_items, compare,
                                          reinterpret_cast<cudaStream_t>(stream)),
                           "ArgMax");
    }
#endif

private:
    template <typename T>
    static void views(BufferView<T> i, BufferView<T> o, uint64_t n)
    {
        detail::require(i.size() >= n && o.size() >= 1, "DeviceReduce: the input view is shorter than num_items "
                                                        "or the output view is empty");
    }

    template <typename T>
    static void arg_views(BufferView<T> i, BufferView<T> o, BufferView<uint32_t> idx, uint64_t n)
    {
        detail::require(o.size() >= 1 && idx.size() >= 1, "DeviceReduce: extremum output view is empty");
        detail::require(i.size() >= n, "DeviceReduce: the input view is shorter than num_items");
    }
};

// ---------------------------------------------------------------------------
// DeviceSelect / DevicePartition
// ---------------------------------------------------------------------------

/// A predicate that crosses the C ABI: the AND of up to LCPP_MAX_CLAUSES
/// clauses on a value of type T (lt, le, gt, ge, eq, ne against a constant;
/// mod_eq(m, r): x % m == r; bits_any(mask): (x & mask) != 0), each negatable
/// with `!`.  Under nvcc the DeviceSelect / DevicePartition methods also take
/// any __device__ callable bool(T).
template <typename T>
class Predicate {
public:
    static Predicate lt(T a) { return one(LCPP_CLAUSE_LT, a); }
    static Predicate le(T a) { return one(LCPP_CLAUSE_LE, a); }
    static Predicate gt(T a) { return one(LCPP_CLAUSE_GT, a); }
    static Predicate ge(T a) { return one(LCPP_CLAUSE_GE, a); }
    static Predicate eq(T a) { return one(LCPP_CLAUSE_EQ, a); }
    static Predicate ne(T a) { return one(LCPP_CLAUSE_NE, a); }
    static Predicate mod_eq(T m, T r) { return one(LCPP_CLAUSE_MOD_EQ, m, r); }
    static Predicate bits_any(T mask) { return one(LCPP_CLAUSE_BITS_ANY, mask); }
    static Predicate always() { return Predicate{}; }

    Predicate operator&(const Predicate& o) const
    {
        detail::require(n_ + o.n_ <= LCPP_MAX_CLAUSES, "Predicate: too many clauses");
        Predicate r = *this;
        for (int i = 0; i < o.n_; ++i) r.c_[r.n_++] = o.c_[i];
        return r;
    }
    Predicate operator!() const
    {
        detail::require(n_ == 1, "Predicate: ! applies to a single clause");
        Predicate r = *this;
        r.c_[0].negate = !r.c_[0].negate;
        return r;
    }
    const lcpp_clause* data() const { return c_; }
    int size() const { return n_; }

private:
    static uint64_t bits(T v)
    {
        static_assert(sizeof(T) == 1 || sizeof(T) == 4 || sizeof(T) == 8, "1-, 4- or 8-byte values");
        uint64_t b = 0;
        std::memcpy(&b, &v, sizeof(T));
        return b;
    }
    static Predicate one(int kind, T a, T b = T(0))
    {
        Predicate p;
        p.c_[0] = lcpp_clause{kind, 0, bits(a), bits(b)};
        p.n_ = 1;
        return p;
    }
    lcpp_clause c_[LCPP_MAX_CLAUSES] = {};
    int n_ = 0;
};

namespace detail {
template <typename P>
struct is_predicate : std::false_type {};
template <typename T>
struct is_predicate<Predicate<T>> : std::true_type {};

template <typename F>
constexpr lcpp_dtype flag_dtype()
{
    if constexpr (std::is_same_v<F, bool> || (std::is_integral_v<F> && sizeof(F) == 1))
        return LCPP_U8;
    else
        return checked_dtype<F>();
}

inline void require_views(bool ok) { require(ok, "a view is shorter than num_items, or a count view is empty"); }
}  // namespace detail

class DeviceSelect {
public:
    static size_t GetTempStorageBytes(uint64_t num_items)
    {
        size_t b = 0;
        detail::check(lcpp_select_temp_bytes(num_items, &b), "GetTempStorageBytes");
        return b;
    }

    /// Items whose flag != 0, in order (device_select.h:65-104).
    template <typename T, typename F>
    void Flagged(lcpp_stream_t stream, BufferView<uint32_t> temp_storage, BufferView<T> input,
                 BufferView<F> selection_flags, BufferView<T> output, BufferView<uint32_t> num_selected_out,
                 uint64_t num_items)
    {
        detail::require_views(input.size() >= num_items && selection_flags.size() >= num_items &&
                              output.size() >= num_items && num_selected_out.size() >= 1);
        detail::check(lcpp_select_flagged(temp_storage.data(), detail::temp_bytes(temp_storage), input.data(),
                                          selection_flags.data(), output.data(), num_selected_out.data(), num_items,
                                          detail::checked_dtype<T>(), detail::flag_dtype<F>(), stream),
                      "Flagged");
    }

    /// In place (device_select.h:106-117).
    template <typename T, typename F>
    void Flagged(lcpp_stream_t stream, BufferView<uint32_t> temp_storage, BufferView<T> data,
                 BufferView<F> selection_flags, BufferView<uint32_t> num_selected_out, uint64_t num_items)
    {
        Flagged(stream, temp_storage, data, selection_flags, data, num_selected_out, num_items);
    }

    /// Items with pred(item) (device_select.h:119-158).
    template <typename T, typename P>
    void If(lcpp_stream_t stream, BufferView<uint32_t> temp_storage, BufferView<T> input, BufferView<T> output,
            BufferView<uint32_t> num_selected_out, uint64_t num_items, const P& pred)
    {
        detail::require_views(input.size() >= num_items && output.size() >= num_items && num_selected_out.size() >= 1);
        if constexpr (detail::is_predicate<P>::value) {
            static_assert(std::is_same_v<P, Predicate<T>>, "If: the Predicate's type must be the item type");
            detail::check(lcpp_select_if(temp_storage.data(), detail::temp_bytes(temp_storage), input.data(),
                                         output.data(), num_selected_out.data(), num_items,
                                         detail::checked_dtype<T>(), pred.data(), pred.size(), stream),
                          "If");
        } else {
#ifdef __CUDACC__
            detail::check_cuda(device::select_if(temp_storage.data(), detail::temp_bytes(temp_storage), input.data(),
                                                 output.data(), num_selected_out.data(), num_items, pred,
                                                 reinterpret_cast<cudaStream_t>(stream)),
                               "If");
#else
            static_assert(detail::is_predicate<P>::value, "callable predicates need nvcc (lcpp_b200_device.cuh)");
#endif
        }
    }

    /// In place (device_select.h:160-175).
    template <typename T, typename P>
    void If(lcpp_stream_t stream, BufferView<uint32_t> temp_storage, BufferView<T> data,
            BufferView<uint32_t> num_selected_out, uint64_t num_items, const P& pred)
    {
        If(stream, temp_storage, data, data, num_selected_out, num_items, pred);
    }

    /// Items whose flag satisfies pred (device_select.h:177-199).
    template <typename T, typename F, typename P>
    void FlaggedIf(lcpp_stream_t stream, BufferView<uint32_t> temp_storage, BufferView<T> input,
                   BufferView<F> selection_flags, BufferView<T> output, BufferView<uint32_t> num_selected_out,
                   uint64_t num_items, const P& pred)
    {
        detail::require_views(input.size() >= num_items && selection_flags.size() >= num_items &&
                              output.size() >= num_items && num_selected_out.size() >= 1);
        if constexpr (detail::is_predicate<P>::value) {
            detail::check(lcpp_select_flagged_if(temp_storage.data(), detail::temp_bytes(temp_storage), input.data(),
                                                 selection_flags.data(), output.data(), num_selected_out.data(),
                                                 num_items, detail::checked_dtype<T>(), detail::flag_dtype<F>(),
                                                 pred.data(), pred.size(), stream),
                          "FlaggedIf");
        } else {
#ifdef __CUDACC__
            detail::check_cuda(device::select_flagged(temp_storage.data(), detail::temp_bytes(temp_storage),
                                                      input.data(), selection_flags.data(), output.data(),
                                                      num_selected_out.data(), num_items, pred,
                                                      reinterpret_cast<cudaStream_t>(stream)),
                               "FlaggedIf");
#else
            static_assert(detail::is_predicate<P>::value, "callable predicates need nvcc (lcpp_b200_device.cuh)");
#endif
        }
    }

    /// In place (device_select.h:201-212).
    template <typename T, typename F, typename P>
    void FlaggedIf(lcpp_stream_t stream, BufferView<uint32_t> temp_storage, BufferView<T> data,
                   BufferView<F> selection_flags, BufferView<uint32_t> num_selected_out, uint64_t num_items,
                   const P& pred)
    {
        FlaggedIf(stream, temp_storage, data, selection_flags, data, num_selected_out, num_items, pred);
    }

    /// First item of every run of equal items (device_select.h:214-286).
    template <typename T>
    void Unique(lcpp_stream_t stream, BufferView<uint32_t> temp_storage, BufferView<T> input, BufferView<T> output,
                BufferView<uint32_t> num_selected_out, uint64_t num_items)
    {
        detail::require_views(input.size() >= num_items && output.size() >= num_items && num_selected_out.size() >= 1);
        detail::check(lcpp_select_unique(temp_storage.data(), detail::temp_bytes(temp_storage), input.data(),
                                         output.data(), num_selected_out.data(), num_items,
                                         detail::checked_dtype<T>(), stream),
                      "Unique");
    }

    template <typename T>
    void Unique(lcpp_stream_t stream, BufferView<uint32_t> temp_storage, BufferView<T> data,
                BufferView<uint32_t> num_selected_out, uint64_t num_items)
    {
        Unique(stream, temp_storage, data, data, num_selected_out, num_items);
    }

    /// First (key, value) of every run of equal keys (device_select.h:288-333).
    template <typename K, typename V>
    void UniqueByKey(lcpp_stream_t stream, BufferView<uint32_t> temp_storage, BufferView<K> keys_input,
                     BufferView<V> values_input, BufferView<K> keys_output, BufferView<V> values_output,
                     BufferView<uint32_t> num_selected_out, uint64_t num_items)
    {
        detail::require_views(keys_input.size() >= num_items && values_input.size() >= num_items &&
                              keys_output.size() >= num_items && values_output.size() >= num_items &&
                              num_selected_out.size() >= 1);
        detail::check(lcpp_select_unique_by_key(temp_storage.data(), detail::temp_bytes(temp_storage),
                                                keys_input.data(), values_input.data(), keys_output.data(),
                                                values_output.data(), num_selected_out.data(), num_items,
                                                detail::checked_dtype<K>(), detail::checked_dtype<V>(), stream),
                      "UniqueByKey");
    }

#ifdef __CUDACC__
    /// The equality overloads (device_select.h:233-333): `equality` is a
    /// __device__ callable bool(T, T) "same run".
    template <typename T, typename Eq, typename = std::enable_if_t<!std::is_arithmetic_v<Eq>>>
    void Unique(lcpp_stream_t stream, BufferView<uint32_t> temp_storage, BufferView<T> input, BufferView<T> output,
                BufferView<uint32_t> num_selected_out, uint64_t num_items, Eq equality)
    {
        detail::require_views(input.size() >= num_items && output.size() >= num_items && num_selected_out.size() >= 1);
        detail::check_cuda(device::select_unique(temp_storage.data(), detail::temp_bytes(temp_storage), input.data(),
                                                 output.data(), num_selected_out.data(), num_items, equality,
                                                 reinterpret_cast<cudaStream_t>(stream)),
                           "Unique");
    }

    template <typename T, typename Eq, typename = std::enable_if_t<!std::is_arithmetic_v<Eq>>>
    void Unique(lcpp_stream_t stream, BufferView<uint32_t> temp_storage, BufferView<T> data,
                BufferView<uint32_t> num_selected_out, uint64_t num_items, Eq equality)
    {
        Unique(stream, temp_storage, data, data, num_selected_out, num_items, equality);
    }

    template <typename K, typename V, typename Eq>
    void UniqueByKey(lcpp_stream_t stream, BufferView<uint32_t> temp_storage, BufferView<K> keys_input,
                     BufferView<V> values_input, BufferView<K> keys_output, BufferView<V> values_output,
                     BufferView<uint32_t> num_selected_out, uint64_t num_items, Eq equality)
    {
        detail::require_views(keys_input.size() >= num_items && values_input.size() >= num_items &&
                              keys_output.size() >= num_items && values_output.size() >= num_items &&
                              num_selected_out.size() >= 1);
        detail::check_cuda(device::select_unique_by_key(temp_storage.data(), detail::temp_bytes(temp_storage),
                                                        keys_input.data(), values_input.data(), keys_output.data(),
                                                        values_output.data(), num_selected_out.data(), num_items,
                                                        equality, reinterpret_cast<cudaStream_t>(stream)),
                           "UniqueByKey");
    }
#endif
};

class DevicePartition {
public:
    static size_t GetTempStorageBytes(uint64_t num_items)
    {
        size_t b = 0;
        detail::check(lcpp_partition_temp_bytes(num_items, &b), "GetTempStorageBytes");
        return b;
    }
    static size_t GetThreeWayTempStorageBytes(uint64_t num_items)
    {
        size_t b = 0;
        detail::check(lcpp_partition_three_way_temp_bytes(num_items, &b), "GetThreeWayTempStorageBytes");
        return b;
    }

    /// Selected items in order, then the rejected ones in reverse order
    /// (device_partition.h:73-113).
    template <typename T, typename F>
    void Flagged(lcpp_stream_t stream, BufferView<uint32_t> temp_storage, BufferView<T> input,
                 BufferView<F> selection_flags, BufferView<T> output, BufferView<uint32_t> num_selected_out,
                 uint64_t num_items)
    {
        detail::require_views(input.size() >= num_items && selection_flags.size() >= num_items &&
                              output.size() >= num_items && num_selected_out.size() >= 1);
        detail::check(lcpp_partition_flagged(temp_storage.data(), detail::temp_bytes(temp_storage), input.data(),
                                             selection_flags.data(), output.data(), num_selected_out.data(),
                                             num_items, detail::checked_dtype<T>(), detail::flag_dtype<F>(), stream),
                      "Flagged");
    }

    /// device_partition.h:115-155.
    template <typename T, typename P>
    void If(lcpp_stream_t stream, BufferView<uint32_t> temp_storage, BufferView<T> input, BufferView<T> output,
            BufferView<uint32_t> num_selected_out, uint64_t num_items, const P& pred)
    {
        detail::require_views(input.size() >= num_items && output.size() >= num_items && num_selected_out.size() >= 1);
        if constexpr (detail::is_predicate<P>::value) {
            detail::check(lcpp_partition_if(temp_storage.data(), detail::temp_bytes(temp_storage), input.data(),
                                            output.data(), num_selected_out.data(), num_items,
                                            detail::checked_dtype<T>(), pred.data(), pred.size(), stream),
                          "If");
        } else {
#ifdef __CUDACC__
            detail::check_cuda(device::partition_if(temp_storage.data(), detail::temp_bytes(temp_storage),
                                                    input.data(), output.data(), num_selected_out.data(), num_items,
                                                    pred, reinterpret_cast<cudaStream_t>(stream)),
                               "If");
#else
            static_assert(detail::is_predicate<P>::value, "callable predicates need nvcc (lcpp_b200_device.cuh)");
#endif
        }
    }

    /// Three-way (device_partition.h:157-227): num_selected_out[0] / [1] =
    /// the first / second counts; unselected items in reverse order.
    template <typename T, typename P1, typename P2>
    void If(lcpp_stream_t stream, BufferView<uint32_t> temp_storage, BufferView<T> input, BufferView<T> first_output,
            BufferView<T> second_output, BufferView<T> unselected_output, BufferView<uint32_t> num_selected_out,
            uint64_t num_items, const P1& select_first, const P2& select_second)
    {
        detail::require_views(input.size() >= num_items && first_output.size() >= num_items &&
                              second_output.size() >= num_items && unselected_output.size() >= num_items &&
                              num_selected_out.size() >= 2);
        if constexpr (detail::is_predicate<P1>::value && detail::is_predicate<P2>::value) {
            detail::check(lcpp_partition_if_three_way(temp_storage.data(), detail::temp_bytes(temp_storage),
                                                      input.data(), first_output.data(), second_output.data(),
                                                      unselected_output.data(), num_selected_out.data(), num_items,
                                                      detail::checked_dtype<T>(), select_first.data(),
                                                      select_first.size(), select_second.data(),
                                                      select_second.size(), stream),
                          "If");
        } else {
#ifdef __CUDACC__
            detail::check_cuda(device::partition_three_way(temp_storage.data(), detail::temp_bytes(temp_storage),
                                                           input.data(), first_output.data(), second_output.data(),
                                                           unselected_output.data(), num_selected_out.data(),
                                                           num_items, select_first, select_second,
                                                           reinterpret_cast<cudaStream_t>(stream)),
                               "If");
#else
            static_assert(detail::is_predicate<P1>::value, "callable predicates need nvcc (lcpp_b200_device.cuh)");
#endif
        }
    }
};

/// Words of a uint32 temp buffer that hold `bytes` (the reference's
/// bytes_to_uint_count).
inline size_t bytes_to_uint_count(size_t bytes) { return (bytes + 3) / 4; }

}  // namespace lcpp_b200

#endif /* LCPP_B200_HPP */
