// CUDA caller of the overloads that take a user callable -- the comparator
// forms of DeviceReduce::ArgMin / ArgMax, the by-key scans with a key
// equality and custom operators, ReduceByKey with a custom operator
// (include/lcpp_b200.hpp with nvcc, kernels from lcpp_b200_device.cuh),
// written like the reference's tests/device_reduce_test.cpp:290-345: device
// results against the reference's sequential comparator fold
// (src/lcpp/device/device_reduce.h:580-603) on the host.  Built and run by
// tests/test_cpp_api.py on a GPU box; compiled (not run) on the CPU.  Prints
// "OK <checks>" and exits 0 on success.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <iterator>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <limits>
#include <random>
#include <utility>
#include <vector>

#include "lcpp_b200.hpp"

using namespace lcpp_b200;

namespace {

int g_checks = 0;

#define CHECK(cond)                                                                  \
    do {                                                                             \
        ++g_checks;                                                                  \
        if (!(cond)) {                                                               \
            std::fprintf(stderr, "FAILED %s at %s:%d\n", #cond, __FILE__, __LINE__); \
            std::exit(1);                                                            \
        }                                                                            \
    } while (0)

#define CUDA(call) CHECK((call) == cudaSuccess)

template <typename T>
struct DeviceArray {
    T* p = nullptr;
    size_t n = 0;
    explicit DeviceArray(size_t count) : n(count) { CUDA(cudaMalloc(&p, std::max<size_t>(count, 1) * sizeof(T))); }
    ~DeviceArray() { cudaFree(p); }
    BufferView<T> view() const { return {p, n}; }
    void upload(const std::vector<T>& h) { CUDA(cudaMemcpy(p, h.data(), h.size() * sizeof(T), cudaMemcpyHostToDevice)); }
    T first() const
    {
        T v;
        CUDA(cudaMemcpy(&v, p, sizeof(T), cudaMemcpyDeviceToHost));
        return v;
    }
};

DeviceArray<uint32_t> temp_for(size_t bytes) { return DeviceArray<uint32_t>(bytes_to_uint_count(std::max<size_t>(bytes, 4))); }

struct LastDigitLess {
    __host__ __device__ bool operator()(int a, int b) const { return a % 10 < b % 10; }
};

// |a| < |b| with a modulus carried in the functor (a stateful comparator).
struct ModAbsLess {
    int64_t m;
    __host__ __device__ bool operator()(int64_t a, int64_t b) const
    {
        const int64_t x = (a < 0 ? -a : a) % m, y = (b < 0 ? -b : b) % m;
        return x < y;
    }
};

// The reference's comparator fold: item i replaces the best when
// compare(item, best) (ArgMin) or compare(best, item) (ArgMax).
template <typename T, typename C>
std::pair<T, uint32_t> fold(const std::vector<T>& h, bool is_min, C c)
{
    T best = h[0];
    uint32_t bi = 0;
    for (size_t i = 1; i < h.size(); ++i)
        if (is_min ? c(h[i], best) : c(best, h[i])) {
            best = h[i];
            bi = uint32_t(i);
        }
    return {best, bi};
}

template <typename T, typename C>
void check_both(lcpp_stream_t s, const std::vector<T>& h, C c, size_t offset = 0)
{
    const size_t n = h.size() - offset;
    DeviceArray<T> in(h.size()), value(1);
    DeviceArray<uint32_t> index(1);
    in.upload(h);
    auto temp = temp_for(DeviceReduce::GetArgTempStorageBytes<T>(n));
    BufferView<T> view{in.p + offset, n};
    const std::vector<T> sub(h.begin() + offset, h.end());
    DeviceReduce rd;
    rd.ArgMin(s, temp.view(), view, value.view(), index.view(), n, c);
    CUDA(cudaStreamSynchronize(s));
    auto want = fold(sub, true, c);
    CHECK(value.first() == want.first && index.first() == want.second);
    rd.ArgMax(s, temp.view(), view, value.view(), index.view(), n, c);
    CUDA(cudaStreamSynchronize(s));
    want = fold(sub, false, c);
    CHECK(value.first() == want.first && index.first() == want.second);
}

void reference_case(lcpp_stream_t s)
{
    // device_reduce_test.cpp:290-330: last-digit comparator, first ties
    const std::vector<int> h{21, 11, 33, 23, 8, 28};
    DeviceArray<int> in(h.size()), mn(1), mx(1);
    DeviceArray<uint32_t> mni(1), mxi(1);
    in.upload(h);
    auto temp = temp_for(DeviceReduce::GetArgTempStorageBytes<int>(h.size()));
    DeviceReduce rd;
    rd.ArgMin(s, temp.view(), in.view(), mn.view(), mni.view(), h.size(), LastDigitLess{});
    rd.ArgMax(s, temp.view(), in.view(), mx.view(), mxi.view(), h.size(), LastDigitLess{});
    CUDA(cudaStreamSynchronize(s));
    CHECK(mn.first() == 21 && mni.first() == 0u);
    CHECK(mx.first() == 8 && mxi.first() == 4u);
}

void empty_sentinels(lcpp_stream_t s)
{
    // device_reduce_test.cpp:332-345: the comparator forms keep the sentinels
    DeviceArray<int> in(0), mn(1), mx(1);
    DeviceArray<uint32_t> mni(1), mxi(1);
    DeviceReduce rd;
    rd.ArgMin(s, BufferView<uint32_t>{}, in.view(), mn.view(), mni.view(), 0, LastDigitLess{});
    rd.ArgMax(s, BufferView<uint32_t>{}, in.view(), mx.view(), mxi.view(), 0, LastDigitLess{});
    CUDA(cudaStreamSynchronize(s));
    CHECK(mn.first() == std::numeric_limits<int>::max() && mni.first() == 1u);
    CHECK(mx.first() == std::numeric_limits<int>::lowest() && mxi.first() == 1u);
}

void random_cases(lcpp_stream_t s)
{
    std::mt19937 rng(114521);
    for (size_t n : {size_t(1), size_t(7), size_t(2049), size_t(1000003), size_t(20000003)}) {
        std::vector<int> h(n);
        for (auto& x : h) x = int(rng() % 2000001) - 1000000;
        check_both(s, h, LastDigitLess{});
        if (n > 8) check_both(s, h, LastDigitLess{}, 3);  // misaligned start
    }
    std::mt19937_64 rng64(7);
    std::vector<int64_t> h(3000001);
    for (auto& x : h) x = int64_t(rng64());
    check_both(s, h, ModAbsLess{1000});
    check_both(s, h, ModAbsLess{1000}, 1);
#ifdef __CUDACC_EXTENDED_LAMBDA__
    std::vector<float> f(1000003);
    std::normal_distribution<float> nd;
    for (auto& x : f) x = std::round(nd(rng) * 8.0f);
    check_both(s, f, [] __host__ __device__(float a, float b) { return std::fabs(a) < std::fabs(b); });
#endif
}

struct SameParity {
    __host__ __device__ bool operator()(int a, int b) const { return (a & 1) == (b & 1); }
};

// a non-commutative associative operator: affine maps x -> a*x + b packed as
// (a, b) in the two halves of a uint64 (mod 2^32); (f then g)(x) = g(f(x))
struct Compose {
    __host__ __device__ uint64_t operator()(uint64_t f, uint64_t g) const
    {
        const uint32_t fa = uint32_t(f >> 32), fb = uint32_t(f), ga = uint32_t(g >> 32), gb = uint32_t(g);
        return (uint64_t(ga * fa) << 32) | uint32_t(ga * fb + gb);
    }
};

template <typename K, typename V, typename Op, typename Eq>
std::vector<V> host_scan_by_key(const std::vector<K>& k, const std::vector<V>& v, int mode, V init, Op op, Eq eq)
{
    std::vector<V> out(v.size());
    V run{};
    for (size_t i = 0; i < v.size(); ++i) {
        const bool head = i == 0 || !eq(k[i - 1], k[i]);
        if (mode == 0) {
            out[i] = head ? init : op(init, run);
            run = head ? v[i] : op(run, v[i]);
        } else {
            run = head ? v[i] : op(run, v[i]);
            out[i] = mode == 2 ? op(init, run) : run;
        }
    }
    return out;
}

void by_key_cases(lcpp_stream_t s)
{
    // device_scan_test.cpp:419-446: keys {1, 3, 5, 2, 4} under "same parity"
    {
        const std::vector<int> keys{1, 3, 5, 2, 4}, ones(5, 1);
        DeviceArray<int> dk(5), dv(5), out(5);
        dk.upload(keys);
        dv.upload(ones);
        auto temp = temp_for(DeviceScan::GetScanByKeyTempStorageBytes<int, int>(5));
        DeviceScan sc;
        sc.InclusiveSumByKey(s, temp.view(), dk.view(), dv.view(), out.view(), 5, SameParity{});
        CUDA(cudaStreamSynchronize(s));
        std::vector<int> got(5);
        CUDA(cudaMemcpy(got.data(), out.p, 5 * sizeof(int), cudaMemcpyDeviceToHost));
        CHECK((got == std::vector<int>{1, 2, 3, 1, 2}));
    }
    // random keys, parity equality, and a non-commutative operator
    std::mt19937 rng(7);
    for (size_t n : {size_t(1), size_t(4097), size_t(1000003)}) {
        std::vector<int> keys(n);
        std::vector<uint64_t> maps(n);
        for (size_t i = 0; i < n; ++i) {
            keys[i] = int(rng() % 5) * (rng() % 50 == 0 ? 1 : 2);  // mostly even: long parity runs
            maps[i] = (uint64_t(rng() | 1u) << 32) | rng();
        }
        DeviceArray<int> dk(n);
        DeviceArray<uint64_t> dv(n), out(n);
        dk.upload(keys);
        dv.upload(maps);
        auto temp = temp_for(DeviceScan::GetScanByKeyTempStorageBytes<int, uint64_t>(n));
        DeviceScan sc;
        const uint64_t ident_shift = (uint64_t(1) << 32) | 5u;  // x -> x + 5
        std::vector<uint64_t> got(n);
        for (int mode = 0; mode < 3; ++mode) {
            if (mode == 0)
                sc.ExclusiveScanByKey(s, temp.view(), dk.view(), dv.view(), out.view(), Compose{}, n, ident_shift,
                                      SameParity{});
            else if (mode == 1)
                sc.InclusiveScanByKey(s, temp.view(), dk.view(), dv.view(), out.view(), Compose{}, n, SameParity{});
            else
                sc.InclusiveScanByKey(s, temp.view(), dk.view(), dv.view(), out.view(), Compose{}, n, ident_shift,
                                      SameParity{});
            CUDA(cudaStreamSynchronize(s));
            CUDA(cudaMemcpy(got.data(), out.p, n * sizeof(uint64_t), cudaMemcpyDeviceToHost));
            CHECK(got == host_scan_by_key(keys, maps, mode, ident_shift, Compose{}, SameParity{}));
        }
        // ReduceByKey with the non-commutative operator (== on keys)
        DeviceArray<int> uniq(n);
        DeviceArray<uint64_t> agg(n);
        DeviceArray<uint32_t> runs(1);
        auto rtemp = temp_for(DeviceReduce::GetReduceByKeyTempStorageBytes<int, uint64_t>(n));
        DeviceReduce rd;
        rd.ReduceByKey(s, rtemp.view(), dk.view(), dv.view(), uniq.view(), agg.view(), runs.view(), Compose{}, n);
        CUDA(cudaStreamSynchronize(s));
        std::vector<int> wu;
        std::vector<uint64_t> wa;
        for (size_t i = 0; i < n; ++i) {
            if (i == 0 || keys[i] != keys[i - 1]) {
                wu.push_back(keys[i]);
                wa.push_back(maps[i]);
            } else {
                wa.back() = Compose{}(wa.back(), maps[i]);
            }
        }
        CHECK(runs.first() == uint32_t(wu.size()));
        std::vector<int> gu(wu.size());
        std::vector<uint64_t> ga(wa.size());
        CUDA(cudaMemcpy(gu.data(), uniq.p, gu.size() * sizeof(int), cudaMemcpyDeviceToHost));
        CUDA(cudaMemcpy(ga.data(), agg.p, ga.size() * sizeof(uint64_t), cudaMemcpyDeviceToHost));
        CHECK(gu == wu);
        CHECK(ga == wa);
    }
}

struct PositiveOdd {
    __host__ __device__ bool operator()(int f) const { return f > 0 && f % 2 != 0; }
};
struct DivisibleBy {
    int d;
    __host__ __device__ bool operator()(int x) const { return x % d == 0; }
};
struct Below {
    int b;
    __host__ __device__ bool operator()(int x) const { return x < b; }
};

void select_cases(lcpp_stream_t s)
{
    DeviceSelect sel;
    // device_select_test.cpp:432-500: Unique in place under "same parity"
    {
        const std::vector<int> data{1, 3, 2, 4, 5, 7, 8, 10};
        DeviceArray<int> d(8);
        DeviceArray<uint32_t> cnt(1);
        d.upload(data);
        auto temp = temp_for(DeviceSelect::GetTempStorageBytes(8));
        sel.Unique(s, temp.view(), d.view(), cnt.view(), 8, SameParity{});
        CUDA(cudaStreamSynchronize(s));
        std::vector<int> got(4);
        CUDA(cudaMemcpy(got.data(), d.p, 4 * sizeof(int), cudaMemcpyDeviceToHost));
        CHECK(cnt.first() == 4u);
        CHECK((got == std::vector<int>{1, 2, 5, 8}));
    }
    // :374-430: FlaggedIf with a functor over flags -3..5
    {
        std::vector<int> in(9), flags(9);
        for (int i = 0; i < 9; ++i) {
            in[i] = 100 + i;
            flags[i] = i - 3;
        }
        DeviceArray<int> din(9), df(9), out(9);
        DeviceArray<uint32_t> cnt(1);
        din.upload(in);
        df.upload(flags);
        auto temp = temp_for(DeviceSelect::GetTempStorageBytes(9));
        sel.FlaggedIf(s, temp.view(), din.view(), df.view(), out.view(), cnt.view(), 9, PositiveOdd{});
        CUDA(cudaStreamSynchronize(s));
        std::vector<int> got(3);
        CUDA(cudaMemcpy(got.data(), out.p, 3 * sizeof(int), cudaMemcpyDeviceToHost));
        CHECK(cnt.first() == 3u);
        CHECK((got == std::vector<int>{104, 106, 108}));
    }
    // random: If with a stateful functor vs std::copy_if; partition three-way
    std::mt19937 rng(5);
    for (size_t n : {size_t(1), size_t(4097), size_t(1000003)}) {
        std::vector<int> in(n);
        for (auto& x : in) x = int(rng() % 1000) - 500;
        DeviceArray<int> din(n), o1(n), o2(n), o3(n);
        DeviceArray<uint32_t> cnt(2);
        din.upload(in);
        auto temp = temp_for(DevicePartition::GetThreeWayTempStorageBytes(n));
        sel.If(s, temp.view(), din.view(), o1.view(), cnt.view(), n, DivisibleBy{7});
        CUDA(cudaStreamSynchronize(s));
        std::vector<int> want, got(n);
        std::copy_if(in.begin(), in.end(), std::back_inserter(want), DivisibleBy{7});
        CHECK(cnt.first() == want.size());
        CUDA(cudaMemcpy(got.data(), o1.p, n * sizeof(int), cudaMemcpyDeviceToHost));
        CHECK(std::equal(want.begin(), want.end(), got.begin()));
        DevicePartition part;
        part.If(s, temp.view(), din.view(), o1.view(), o2.view(), o3.view(), cnt.view(), n, DivisibleBy{3}, Below{0});
        CUDA(cudaStreamSynchronize(s));
        std::vector<int> w1, w2, w3;
        for (int x : in) {
            if (x % 3 == 0) w1.push_back(x);
            else if (x < 0) w2.push_back(x);
        }
        for (size_t i = n; i-- > 0;)
            if (in[i] % 3 != 0 && in[i] >= 0) w3.push_back(in[i]);
        std::vector<uint32_t> c(2);
        CUDA(cudaMemcpy(c.data(), cnt.p, 8, cudaMemcpyDeviceToHost));
        CHECK(c[0] == w1.size() && c[1] == w2.size());
        std::vector<int> g1(n), g2(n), g3(n);
        CUDA(cudaMemcpy(g1.data(), o1.p, n * sizeof(int), cudaMemcpyDeviceToHost));
        CUDA(cudaMemcpy(g2.data(), o2.p, n * sizeof(int), cudaMemcpyDeviceToHost));
        CUDA(cudaMemcpy(g3.data(), o3.p, n * sizeof(int), cudaMemcpyDeviceToHost));
        CHECK(std::equal(w1.begin(), w1.end(), g1.begin()));
        CHECK(std::equal(w2.begin(), w2.end(), g2.begin()));
        CHECK(std::equal(w3.begin(), w3.end(), g3.begin()));
    }
}

struct Xor {
    __host__ __device__ uint64_t operator()(uint64_t a, uint64_t b) const { return a ^ b; }
};
struct Square {
    __host__ __device__ int64_t operator()(int64_t x) const { return int64_t(uint64_t(x) * uint64_t(x)); }
};

void user_operator_cases(lcpp_stream_t s)
{
    // Reduce / TransformReduce (device_reduce.h:229-308, :493-516) and the
    // plain scans (device_scan.h:321-368) with user operators, against host folds
    std::mt19937_64 rng(17);
    for (size_t n : {size_t(1), size_t(4097), size_t(1000003)}) {
        std::vector<uint64_t> maps(n);
        std::vector<int64_t> ints(n);
        for (size_t i = 0; i < n; ++i) {
            maps[i] = (uint64_t(uint32_t(rng()) | 1u) << 32) | uint32_t(rng());
            ints[i] = int64_t(rng() % 2001) - 1000;
        }
        DeviceArray<uint64_t> dm(n), out(n), one(1);
        DeviceArray<int64_t> di(n), ione(1);
        dm.upload(maps);
        di.upload(ints);
        DeviceReduce rd;
        auto rtemp = temp_for(DeviceReduce::GetTempStorageBytes<uint64_t>(n));
        rd.Reduce(s, rtemp.view(), dm.view(), one.view(), n, Xor{}, uint64_t(0x5a5a));
        CUDA(cudaStreamSynchronize(s));
        uint64_t x = 0x5a5a;
        for (uint64_t m : maps) x ^= m;
        CHECK(one.first() == x);
        auto itemp = temp_for(DeviceReduce::GetTempStorageBytes<int64_t>(n));
        rd.TransformReduce(s, itemp.view(), di.view(), ione.view(), n, SumOp{}, Square{}, int64_t(7));
        CUDA(cudaStreamSynchronize(s));
        int64_t sq = 7;
        for (int64_t v : ints) sq += v * v;
        CHECK(ione.first() == sq);

        DeviceScan sc;
        auto stemp = temp_for(DeviceScan::GetTempStorageBytes<uint64_t>(n));
        const uint64_t shift = (uint64_t(1) << 32) | 9u;  // x -> x + 9
        std::vector<uint64_t> got(n), want(n);
        for (int mode = 0; mode < 3; ++mode) {
            if (mode == 0) sc.ExclusiveScan(s, stemp.view(), dm.view(), out.view(), n, Compose{}, shift);
            else if (mode == 1) sc.InclusiveScan(s, stemp.view(), dm.view(), out.view(), n, Compose{});
            else sc.InclusiveScanInit(s, stemp.view(), dm.view(), out.view(), n, Compose{}, shift);
            CUDA(cudaStreamSynchronize(s));
            CUDA(cudaMemcpy(got.data(), out.p, n * sizeof(uint64_t), cudaMemcpyDeviceToHost));
            uint64_t run = mode == 1 ? maps[0] : shift;
            for (size_t i = 0; i < n; ++i) {
                if (mode == 0) {
                    want[i] = run;
                    run = Compose{}(run, maps[i]);
                } else {
                    if (mode == 2 || i > 0) run = Compose{}(run, maps[i]);
                    want[i] = run;
                }
            }
            CHECK(got == want);
        }
    }
}

}  // namespace

int main()
{
    cudaStream_t stream;
    CUDA(cudaStreamCreate(&stream));
    const auto s = reinterpret_cast<lcpp_stream_t>(stream);
    reference_case(s);
    empty_sentinels(s);
    random_cases(s);
    by_key_cases(s);
    select_cases(s);
    user_operator_cases(s);
    CUDA(cudaStreamDestroy(stream));
    std::printf("OK %d\n", g_checks);
    return 0;
}
