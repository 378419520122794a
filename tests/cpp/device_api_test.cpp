// C++ caller of include/lcpp_b200.hpp, written like the reference's own
// tests (tests/device_radix_sort_one_sweep.cpp, tests/device_scan_test.cpp,
// tests/device_reduce_test.cpp): device results against std:: host
// algorithms.  Built and run by tests/test_cpp_api.py on a GPU box; also
// compiled (not run) on the CPU.  Prints "OK <checks>" and exits 0 on success.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <cstdio>
#include <limits>
#include <numeric>
#include <random>
#include <tuple>
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
    std::vector<T> download() const
    {
        std::vector<T> h(n);
        CUDA(cudaMemcpy(h.data(), p, n * sizeof(T), cudaMemcpyDeviceToHost));
        return h;
    }
};

DeviceArray<uint32_t> temp_for(size_t bytes) { return DeviceArray<uint32_t>(bytes_to_uint_count(bytes)); }

void sort_keys_float(lcpp_stream_t s)
{
    // device_radix_sort_one_sweep.cpp: float keys U[0,1), mt19937(114521), asc and desc
    for (size_t n : {size_t(1) << 5, size_t(1) << 16, size_t(1) << 20}) {
        std::mt19937 rng(114521);
        std::uniform_real_distribution<float> dist(0.f, 1.f);
        std::vector<float> h(n);
        for (auto& x : h) x = dist(rng);
        DeviceArray<float> in(n), out(n);
        in.upload(h);
        auto temp = temp_for(DeviceRadixSort::GetSortKeysTempStorageBytes<float>(n));
        DeviceRadixSort rs;
        rs.SortKeys(s, temp.view(), in.view(), out.view(), n);
        CUDA(cudaStreamSynchronize(s));
        auto expect = h;
        std::sort(expect.begin(), expect.end());
        CHECK(out.download() == expect);
        rs.SortKeysDescending(s, temp.view(), in.view(), out.view(), n);
        CUDA(cudaStreamSynchronize(s));
        std::sort(expect.begin(), expect.end(), std::greater<float>());
        CHECK(out.download() == expect);
    }
}

void sort_pairs_shuffled(lcpp_stream_t s)
{
    // shuffled permutation keys with float values, asc and desc
    const size_t n = 524288;
    std::vector<uint32_t> keys(n);
    std::iota(keys.begin(), keys.end(), 0u);
    std::shuffle(keys.begin(), keys.end(), std::mt19937(114521));
    std::vector<float> vals(n);
    for (size_t i = 0; i < n; ++i) vals[i] = float(keys[i]) * 0.5f;
    DeviceArray<uint32_t> ki(n), ko(n);
    DeviceArray<float> vi(n), vo(n);
    ki.upload(keys);
    vi.upload(vals);
    auto temp = temp_for(DeviceRadixSort::GetSortPairsTempStorageBytes<uint32_t, float>(n));
    DeviceRadixSort rs;
    for (int desc = 0; desc < 2; ++desc) {
        if (desc)
            rs.SortPairsDescending(s, temp.view(), ki.view(), ko.view(), vi.view(), vo.view(), n);
        else
            rs.SortPairs(s, temp.view(), ki.view(), ko.view(), vi.view(), vo.view(), n);
        CUDA(cudaStreamSynchronize(s));
        auto k = ko.download();
        auto v = vo.download();
        for (size_t i = 0; i < n; ++i) {
            CHECK(k[i] == (desc ? uint32_t(n - 1 - i) : uint32_t(i)));
            CHECK(v[i] == float(k[i]) * 0.5f);
            if (!(k[i] == (desc ? uint32_t(n - 1 - i) : uint32_t(i)))) break;
        }
    }
}

void sort_bits_stable_double_buffer(lcpp_stream_t s)
{
    // device_radix_sort_interface_test.cpp: 257 keys, bits [1,6), stable; DoubleBuffer selector
    const size_t n = 257;
    std::vector<uint32_t> keys(n), idx(n);
    for (size_t i = 0; i < n; ++i) {
        keys[i] = uint32_t(((i * 53) % 64) | (((i * 17) % 11) << 8));
        idx[i] = uint32_t(i);
    }
    std::vector<size_t> order(n);
    std::iota(order.begin(), order.end(), 0);
    auto bits = [](uint32_t k) { return (k >> 1) & 31u; };
    std::stable_sort(order.begin(), order.end(), [&](size_t a, size_t b) { return bits(keys[a]) < bits(keys[b]); });
    DeviceArray<uint32_t> k0(n), k1(n), v0(n), v1(n);
    k0.upload(keys);
    v0.upload(idx);
    DoubleBuffer<uint32_t> dk(k0.view(), k1.view());
    DoubleBuffer<uint32_t> dv(v0.view(), v1.view());
    auto temp = temp_for(DeviceRadixSort::GetSortPairsTempStorageBytes<uint32_t, uint32_t>(n));
    DeviceRadixSort rs;
    rs.SortPairs(s, temp.view(), dk, dv, n, 1, 6);
    CUDA(cudaStreamSynchronize(s));
    CHECK(dk.selector == 1 && dv.selector == 1);  // one 5-bit pass
    const auto& kc = dk.selector ? k1 : k0;
    const auto& vc = dv.selector ? v1 : v0;
    auto k = kc.download();
    auto v = vc.download();
    for (size_t i = 0; i < n; ++i) {
        CHECK(v[i] == uint32_t(order[i]));
        CHECK(k[i] == keys[order[i]]);
    }
    // zero-width range: selector unchanged
    rs.SortKeys(s, temp.view(), dk, n, 3, 3);
    CHECK(dk.selector == 1);
}

void scans(lcpp_stream_t s)
{
    // device_scan_test.cpp: (i % 7) - 3 at 320*25*3+17 items; wrapping int arithmetic
    const size_t n = 320 * 25 * 3 + 17;
    std::vector<int32_t> h(n);
    for (size_t i = 0; i < n; ++i) h[i] = int32_t(i % 7) - 3;
    DeviceArray<int32_t> in(n), out(n);
    in.upload(h);
    auto temp = temp_for(DeviceScan::GetTempStorageBytes<int32_t>(n));
    DeviceScan sc;
    std::vector<int32_t> expect(n);
    sc.InclusiveSum(s, temp.view(), in.view(), out.view(), n);
    CUDA(cudaStreamSynchronize(s));
    std::inclusive_scan(h.begin(), h.end(), expect.begin());
    CHECK(out.download() == expect);
    sc.ExclusiveSum(s, temp.view(), in.view(), out.view(), n);
    CUDA(cudaStreamSynchronize(s));
    std::exclusive_scan(h.begin(), h.end(), expect.begin(), 0);
    CHECK(out.download() == expect);
    sc.InclusiveScanInit(s, temp.view(), in.view(), out.view(), n, SumOp{}, int32_t(100));
    CUDA(cudaStreamSynchronize(s));
    std::inclusive_scan(h.begin(), h.end(), expect.begin(), std::plus<int32_t>(), 100);
    CHECK(out.download() == expect);
    sc.ExclusiveScan(s, temp.view(), in.view(), out.view(), n, MaxOp{}, std::numeric_limits<int32_t>::lowest());
    CUDA(cudaStreamSynchronize(s));
    int32_t run = std::numeric_limits<int32_t>::lowest();
    for (size_t i = 0; i < n; ++i) {
        expect[i] = run;
        run = std::max(run, h[i]);
    }
    CHECK(out.download() == expect);
    sc.InclusiveScan(s, temp.view(), in.view(), out.view(), n, MinOp{});
    CUDA(cudaStreamSynchronize(s));
    run = std::numeric_limits<int32_t>::max();
    for (size_t i = 0; i < n; ++i) expect[i] = run = std::min(run, h[i]);
    CHECK(out.download() == expect);
}

void arg_reductions(lcpp_stream_t s)
{
    // device_reduce_test.cpp:238-288: first of equal maxima; negative floats
    {
        const std::vector<int32_t> h{1, 9, 4, 9, 3};
        DeviceArray<int32_t> in(h.size()), value(1);
        DeviceArray<uint32_t> index(1);
        in.upload(h);
        auto temp = temp_for(DeviceReduce::GetArgTempStorageBytes<int32_t>(h.size()));
        DeviceReduce rd;
        rd.ArgMax(s, temp.view(), in.view(), value.view(), index.view(), h.size());
        CUDA(cudaStreamSynchronize(s));
        CHECK(value.download()[0] == 9 && index.download()[0] == 1u);
    }
    {
        const std::vector<float> h{-7.0f, -3.0f, -5.0f};
        DeviceArray<float> in(h.size()), value(1);
        DeviceArray<uint32_t> index(1);
        in.upload(h);
        auto temp = temp_for(DeviceReduce::GetArgTempStorageBytes<float>(h.size()));
        DeviceReduce rd;
        rd.ArgMax(s, temp.view(), in.view(), value.view(), index.view(), h.size());
        CUDA(cudaStreamSynchronize(s));
        CHECK(value.download()[0] == -3.0f && index.download()[0] == 1u);
    }
    // empty input: max() / lowest() and index 1 (device_reduce.h:318-323)
    {
        DeviceArray<int64_t> in(0), value(1);
        DeviceArray<uint32_t> index(1);
        DeviceReduce rd;
        rd.ArgMin(s, BufferView<uint32_t>{}, in.view(), value.view(), index.view(), 0);
        CUDA(cudaStreamSynchronize(s));
        CHECK(value.download()[0] == std::numeric_limits<int64_t>::max() && index.download()[0] == 1u);
    }
    // random doubles against std::min_element / std::max_element (first index)
    {
        const size_t n = 3000017;
        std::vector<double> h(n);
        std::mt19937_64 rng(11);
        std::uniform_int_distribution<int> dist(-500, 500);
        for (auto& x : h) x = dist(rng) * 0.25;
        DeviceArray<double> in(n), value(1);
        DeviceArray<uint32_t> index(1);
        in.upload(h);
        auto temp = temp_for(DeviceReduce::GetArgTempStorageBytes<double>(n));
        DeviceReduce rd;
        const auto mn = std::min_element(h.begin(), h.end());
        const auto mx = std::max_element(h.begin(), h.end());
        rd.ArgMin(s, temp.view(), in.view(), value.view(), index.view(), n);
        CUDA(cudaStreamSynchronize(s));
        CHECK(value.download()[0] == *mn && index.download()[0] == uint32_t(mn - h.begin()));
        rd.ArgMax(s, temp.view(), in.view(), value.view(), index.view(), n);
        CUDA(cudaStreamSynchronize(s));
        CHECK(value.download()[0] == *mx && index.download()[0] == uint32_t(mx - h.begin()));
    }
}

void by_key(lcpp_stream_t s)
{
    // device_scan_test.cpp:324-380: ExclusiveSumByKey over ones, keys i / 100
    for (int k : {5, 12, 20}) {
        const size_t n = size_t(1) << k;
        std::vector<int32_t> keys(n), ones(n, 1), expect(n);
        for (size_t i = 0; i < n; ++i) {
            keys[i] = int32_t(i / 100);
            expect[i] = int32_t(i % 100);
        }
        DeviceArray<int32_t> dk(n), dv(n), out(n);
        dk.upload(keys);
        dv.upload(ones);
        auto temp = temp_for(DeviceScan::GetScanByKeyTempStorageBytes<int32_t, int32_t>(n));
        DeviceScan sc;
        sc.ExclusiveSumByKey(s, temp.view(), dk.view(), dv.view(), out.view(), n);
        CUDA(cudaStreamSynchronize(s));
        CHECK(out.download() == expect);
    }
    // :382-417: int keys, int64 values, segments cut one past each 1024-item tile
    {
        const size_t tile = 1024, n = tile * 2 + 2;
        std::vector<int32_t> keys(n);
        std::vector<int64_t> ones(n, 1), expect(n);
        int64_t run = 0;
        for (size_t i = 0; i < n; ++i) {
            keys[i] = i < tile + 1 ? 1 : i < tile * 2 + 1 ? 2 : 3;
            if (i == 0 || keys[i] != keys[i - 1]) run = 0;
            expect[i] = ++run;
        }
        DeviceArray<int32_t> dk(n);
        DeviceArray<int64_t> dv(n), out(n);
        dk.upload(keys);
        dv.upload(ones);
        auto temp = temp_for(DeviceScan::GetScanByKeyTempStorageBytes<int32_t, int64_t>(n));
        DeviceScan sc;
        sc.InclusiveSumByKey(s, temp.view(), dk.view(), dv.view(), out.view(), n);
        CUDA(cudaStreamSynchronize(s));
        CHECK(out.download() == expect);
    }
    // device_reduce_test.cpp:422-513: ReduceByKey Sum by key i / 100; empty input
    {
        const int n = 1 << 12;
        std::vector<int32_t> keys(n), data(n);
        for (int i = 0; i < n; ++i) {
            keys[i] = i / 100;
            data[i] = i;
        }
        std::mt19937 rng(114521);
        std::shuffle(data.begin(), data.end(), rng);
        const int runs = (n + 99) / 100;
        DeviceArray<int32_t> dk(n), dv(n), uniq(runs), agg(runs);
        DeviceArray<uint32_t> nruns(1);
        dk.upload(keys);
        dv.upload(data);
        auto temp = temp_for(DeviceReduce::GetReduceByKeyTempStorageBytes<int32_t, int32_t>(n));
        DeviceReduce rd;
        rd.ReduceByKey(s, temp.view(), dk.view(), dv.view(), uniq.view(), agg.view(), nruns.view(), SumOp{},
                       uint64_t(n));
        CUDA(cudaStreamSynchronize(s));
        CHECK(nruns.download()[0] == uint32_t(runs));
        const auto u = uniq.download(), a = agg.download();
        for (int r = 0; r < runs; ++r) {
            CHECK(u[r] == r);
            CHECK(a[r] == std::accumulate(data.begin() + r * 100, data.begin() + std::min(r * 100 + 100, n), 0));
        }
        nruns.upload({17u});
        rd.ReduceByKey(s, BufferView<uint32_t>{}, dk.view(), dv.view(), uniq.view(), agg.view(), nruns.view(),
                       SumOp{}, 0);
        CUDA(cudaStreamSynchronize(s));
        CHECK(nruns.download()[0] == 0u);
    }
}

void select_partition(lcpp_stream_t s)
{
    // device_select_test.cpp:254-320: Flagged (7 at i % 3 == 1) and If(even)
    {
        const size_t n = 17;
        std::vector<int32_t> in(n);
        std::vector<uint32_t> flags(n);
        std::vector<int32_t> want_f, want_e;
        for (size_t i = 0; i < n; ++i) {
            in[i] = int32_t(100 + i);
            flags[i] = i % 3 == 1 ? 7u : 0u;
            if (flags[i]) want_f.push_back(in[i]);
            if (in[i] % 2 == 0) want_e.push_back(in[i]);
        }
        DeviceArray<int32_t> din(n), out(n);
        DeviceArray<uint32_t> df(n), cnt(1);
        din.upload(in);
        df.upload(flags);
        auto temp = temp_for(DeviceSelect::GetTempStorageBytes(n));
        DeviceSelect sel;
        sel.Flagged(s, temp.view(), din.view(), df.view(), out.view(), cnt.view(), n);
        CUDA(cudaStreamSynchronize(s));
        auto got = out.download();
        CHECK(cnt.download()[0] == want_f.size());
        CHECK(std::equal(want_f.begin(), want_f.end(), got.begin()));
        sel.If(s, temp.view(), din.view(), out.view(), cnt.view(), n, Predicate<int32_t>::mod_eq(2, 0));
        CUDA(cudaStreamSynchronize(s));
        got = out.download();
        CHECK(cnt.download()[0] == want_e.size());
        CHECK(std::equal(want_e.begin(), want_e.end(), got.begin()));
        // in place: If(> 0 and odd) on the input itself
        sel.If(s, temp.view(), din.view(), cnt.view(), n, Predicate<int32_t>::gt(0) & !Predicate<int32_t>::mod_eq(2, 0));
        CUDA(cudaStreamSynchronize(s));
        got = din.download();
        CHECK(cnt.download()[0] == 8u);
        for (int i = 0; i < 8; ++i) CHECK(got[i] == 101 + 2 * i);
    }
    // :322-372: Unique / UniqueByKey keep the first item of each run
    {
        const std::vector<int32_t> keys{1, 1, 2, 2, 2, 4, 7, 7, 9}, values{10, 11, 20, 21, 22, 40, 70, 71, 90};
        const size_t n = keys.size();
        DeviceArray<int32_t> dk(n), dv(n), ko(n), vo(n);
        DeviceArray<uint32_t> cnt(1);
        dk.upload(keys);
        dv.upload(values);
        auto temp = temp_for(DeviceSelect::GetTempStorageBytes(n));
        DeviceSelect sel;
        sel.UniqueByKey(s, temp.view(), dk.view(), dv.view(), ko.view(), vo.view(), cnt.view(), n);
        CUDA(cudaStreamSynchronize(s));
        CHECK(cnt.download()[0] == 5u);
        const auto gk = ko.download(), gv = vo.download();
        const int32_t ek[5] = {1, 2, 4, 7, 9}, ev[5] = {10, 20, 40, 70, 90};
        for (int i = 0; i < 5; ++i) CHECK(gk[i] == ek[i] && gv[i] == ev[i]);
        sel.Unique(s, temp.view(), dk.view(), cnt.view(), n);  // in place
        CUDA(cudaStreamSynchronize(s));
        const auto gu = dk.download();
        CHECK(cnt.download()[0] == 5u);
        for (int i = 0; i < 5; ++i) CHECK(gu[i] == ek[i]);
    }
    // device_partition_test.cpp:122-204 and :293-353
    {
        const size_t n = 12;
        std::vector<int32_t> in(n);
        std::vector<uint8_t> flags(n);
        std::vector<int32_t> want;
        for (size_t i = 0; i < n; ++i) {
            in[i] = int32_t(i);
            flags[i] = i % 3 == 0;
            if (flags[i]) want.push_back(in[i]);
        }
        for (size_t i = n; i-- > 0;)
            if (!flags[i]) want.push_back(in[i]);
        DeviceArray<int32_t> din(n), out(n), o1(n), o2(n), o3(n);
        DeviceArray<uint8_t> df(n);
        DeviceArray<uint32_t> cnt(2);
        din.upload(in);
        df.upload(flags);
        auto temp = temp_for(DevicePartition::GetThreeWayTempStorageBytes(n));
        DevicePartition part;
        part.Flagged(s, temp.view(), din.view(), df.view(), out.view(), cnt.view().subview(0, 1), n);
        CUDA(cudaStreamSynchronize(s));
        CHECK(cnt.download()[0] == 4u);
        CHECK(out.download() == want);
        part.If(s, temp.view(), din.view(), o1.view(), o2.view(), o3.view(), cnt.view(), n,
                Predicate<int32_t>::mod_eq(3, 0), Predicate<int32_t>::lt(8));
        CUDA(cudaStreamSynchronize(s));
        const auto c = cnt.download();
        CHECK(c[0] == 4u && c[1] == 5u);
        const auto g1 = o1.download(), g2 = o2.download(), g3 = o3.download();
        const int32_t e1[4] = {0, 3, 6, 9}, e2[5] = {1, 2, 4, 5, 7}, e3[3] = {11, 10, 8};
        for (int i = 0; i < 4; ++i) CHECK(g1[i] == e1[i]);
        for (int i = 0; i < 5; ++i) CHECK(g2[i] == e2[i]);
        for (int i = 0; i < 3; ++i) CHECK(g3[i] == e3[i]);
    }
}

void reductions(lcpp_stream_t s)
{
    // device_reduce_test.cpp: ones at 2^k + 1; float max identity on empty input
    for (int k : {0, 10, 20}) {
        const size_t n = (size_t(1) << k) + 1;
        std::vector<int32_t> h(n, 1);
        DeviceArray<int32_t> in(n), out(1);
        in.upload(h);
        auto temp = temp_for(DeviceReduce::GetTempStorageBytes<int32_t>(n));
        DeviceReduce rd;
        rd.Sum(s, temp.view(), in.view(), out.view(), n);
        CUDA(cudaStreamSynchronize(s));
        CHECK(out.download()[0] == int32_t(n));
    }
    {
        DeviceArray<float> in(1), out(1);
        auto temp = temp_for(std::max<size_t>(DeviceReduce::GetTempStorageBytes<float>(0), 4));
        DeviceReduce rd;
        rd.Max(s, temp.view(), in.view(), out.view(), 0);
        CUDA(cudaStreamSynchronize(s));
        CHECK(out.download()[0] == std::numeric_limits<float>::lowest());
    }
    {
        const size_t n = 1000003;
        std::vector<int64_t> h(n);
        std::mt19937_64 rng(7);
        for (auto& x : h) x = int64_t(rng());
        DeviceArray<int64_t> in(n), out(1);
        in.upload(h);
        auto temp = temp_for(DeviceReduce::GetTempStorageBytes<int64_t>(n));
        DeviceReduce rd;
        rd.Reduce(s, temp.view(), in.view(), out.view(), n, MinOp{}, std::numeric_limits<int64_t>::max());
        CUDA(cudaStreamSynchronize(s));
        CHECK(out.download()[0] == *std::min_element(h.begin(), h.end()));
    }
}

void segmented(lcpp_stream_t s)
{
    // device_segmented_sort_test.cpp: 19 items, segments [1,4) [5,5) [5,9) [10,19)
    const size_t n = 19, nseg = 4;
    const std::vector<uint32_t> begin{1u, 5u, 5u, 10u}, end{4u, 5u, 9u, 19u};
    std::vector<int32_t> keys{91, 3, -2, 3, 92, 8, 1, 8, 4, 93, 5, -1, 5, 2, -1, 7, 2, 5, 0};
    std::vector<uint32_t> vals(n);
    std::iota(vals.begin(), vals.end(), 0u);
    std::vector<int32_t> expect_k(n, -777);
    std::vector<uint32_t> expect_v(n, 0xffffffffu);
    for (size_t g = 0; g < nseg; ++g) {
        std::vector<uint32_t> o(end[g] - begin[g]);
        std::iota(o.begin(), o.end(), begin[g]);
        std::stable_sort(o.begin(), o.end(), [&](uint32_t l, uint32_t r) { return keys[l] > keys[r]; });
        for (size_t i = 0; i < o.size(); ++i) {
            expect_k[begin[g] + i] = keys[o[i]];
            expect_v[begin[g] + i] = vals[o[i]];
        }
    }
    DeviceArray<int32_t> ki(n), ko(n);
    DeviceArray<uint32_t> vi(n), vo(n), db(nseg), de(nseg);
    ki.upload(keys);
    vi.upload(vals);
    ko.upload(std::vector<int32_t>(n, -777));
    vo.upload(std::vector<uint32_t>(n, 0xffffffffu));
    db.upload(begin);
    de.upload(end);
    auto temp = temp_for(DeviceSegmentedRadixSort::GetSortPairsTempStorageBytes<int32_t, uint32_t>(n));
    DeviceSegmentedRadixSort ss;
    ss.SortPairsDescending(s, temp.view(), ki.view(), ko.view(), vi.view(), vo.view(), n, nseg, db.view(), de.view());
    CUDA(cudaStreamSynchronize(s));
    CHECK(ko.download() == expect_k);
    CHECK(vo.download() == expect_v);
}

struct RadixCompositeKey {
    uint32_t primary;
    int32_t secondary;
    bool operator==(const RadixCompositeKey& o) const { return primary == o.primary && secondary == o.secondary; }
};

void decomposed(lcpp_stream_t s)
{
    // device_radix_sort_interface_test.cpp:285-330: decomposed as (primary, secondary)
    const std::vector<RadixCompositeKey> keys{{1u, -1}, {0u, 7}, {1u, -1}, {2u, -8}, {0u, 3}, {1u, 4}, {2u, 0}, {0u, 7}};
    const size_t n = keys.size();
    std::vector<RadixCompositeKey> expect = keys;
    std::stable_sort(expect.begin(), expect.end(), [](const RadixCompositeKey& l, const RadixCompositeKey& r) {
        return std::tie(l.primary, l.secondary) < std::tie(r.primary, r.secondary);
    });
    DeviceArray<RadixCompositeKey> in(n), out(n);
    in.upload(keys);
    auto temp = temp_for(DeviceRadixSort::GetDecomposedTempStorageBytes(n));
    DeviceRadixSort rs;
    const auto dec = members(&RadixCompositeKey::primary, &RadixCompositeKey::secondary);
    CHECK(dec.bits == 64);
    rs.SortKeys(s, temp.view(), in.view(), out.view(), n, dec);
    CUDA(cudaStreamSynchronize(s));
    CHECK(out.download() == expect);
    DeviceArray<RadixCompositeKey> alt(n);
    DoubleBuffer<RadixCompositeKey> db(in.view(), alt.view());
    rs.SortKeysDescending(s, temp.view(), db, n, dec);
    CUDA(cudaStreamSynchronize(s));
    CHECK(db.selector == 1);
    std::stable_sort(expect.begin(), expect.end(), [](const RadixCompositeKey& l, const RadixCompositeKey& r) {
        return std::tie(l.primary, l.secondary) > std::tie(r.primary, r.secondary);
    });
    CHECK(alt.download() == expect);
}

void misuse_throws(lcpp_stream_t s)
{
    DeviceArray<uint32_t> a(16), b(16);
    auto temp = temp_for(DeviceRadixSort::GetSortKeysTempStorageBytes<uint32_t>(16));
    DeviceRadixSort rs;
    bool threw = false;
    try {
        rs.SortKeys(s, temp.view(), a.view(), b.view(), 16, 4, 40);  // end_bit past the key
    } catch (const Error& e) {
        threw = e.status() == LCPP_ERR_INVALID_ARG;
    }
    CHECK(threw);
    threw = false;
    try {
        rs.SortKeys(s, temp.view().subview(0, 1), a.view(), b.view(), 16);  // temp too small
    } catch (const Error& e) {
        threw = e.status() == LCPP_ERR_TEMP_TOO_SMALL;
    }
    CHECK(threw);
    threw = false;
    try {
        rs.SortKeys(s, temp.view(), a.view(), b.view().subview(0, 8), 16);  // output view too short
    } catch (const Error& e) {
        threw = e.status() == LCPP_ERR_INVALID_ARG;
    }
    CHECK(threw);
    CHECK(DeviceRadixSort::GetSortKeysTempStorageBytes<uint32_t>(0) == 0);
}

}  // namespace

int main()
{
    cudaStream_t stream;
    CUDA(cudaStreamCreate(&stream));
    const auto s = reinterpret_cast<lcpp_stream_t>(stream);
    sort_keys_float(s);
    sort_pairs_shuffled(s);
    sort_bits_stable_double_buffer(s);
    scans(s);
    reductions(s);
    arg_reductions(s);
    by_key(s);
    select_partition(s);
    segmented(s);
    decomposed(s);
    misuse_throws(s);
    CUDA(cudaStreamDestroy(stream));
    std::printf("OK %d\n", g_checks);
    return 0;
}
