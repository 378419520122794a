// make_golden.cpp -- writes the golden fixtures for the sort / scan / reduce
// parity tests.
//
// Inputs follow the input generators of the reference project's own tests and
// expected outputs come from the host algorithms those tests check the GPU
// against (std::sort, std::stable_sort with a selected-bits comparator,
// std::inclusive_scan / std::exclusive_scan, std::min_element ...).  Each case
// names the reference test it follows (path:line inside the reference
// project).  Sizes are cut down where the reference's would make the fixture
// file large; the generator formulas are unchanged.
//
// Output: one raw file per array into the directory given as argv[1], plus
// an index file "arrays.txt" with lines "<name> <dtype> <count>".
// tests/golden/make_golden.py compiles and runs this program and packs the
// result into golden.npz.
#include <algorithm>
#include <cstdint>
#include <cstdio>
#include <functional>
#include <iterator>
#include <numeric>
#include <tuple>
#include <random>
#include <string>
#include <vector>

static std::string g_dir;
static FILE* g_index = nullptr;

template <typename T>
static const char* dtype_name();
template <> const char* dtype_name<uint32_t>() { return "u32"; }
template <> const char* dtype_name<int32_t>() { return "i32"; }
template <> const char* dtype_name<float>() { return "f32"; }
template <> const char* dtype_name<uint64_t>() { return "u64"; }
template <> const char* dtype_name<int64_t>() { return "i64"; }
template <> const char* dtype_name<uint8_t>() { return "u8"; }

template <typename T>
static void emit(const std::string& name, const std::vector<T>& v)
{
    std::string path = g_dir + "/" + name + ".bin";
    FILE* f = std::fopen(path.c_str(), "wb");
    if (!f) { std::perror(path.c_str()); std::exit(1); }
    if (!v.empty()) std::fwrite(v.data(), sizeof(T), v.size(), f);
    std::fclose(f);
    std::fprintf(g_index, "%s %s %zu\n", name.c_str(), dtype_name<T>(), v.size());
}

// tests/device_radix_sort_one_sweep.cpp:79-136 -- float keys U[0,1) from
// std::mt19937(114521); the ascending and descending inputs are drawn
// alternately from one engine; expected = std::sort and std::sort(greater).
static void float_keys()
{
    for (unsigned loop = 5; loop <= 14; ++loop) {
        const unsigned n = 1u << loop;
        std::vector<float> asc(n), desc(n);
        std::mt19937 rng(114521);
        std::uniform_real_distribution<float> dist(0.0f, 1.0f);
        for (unsigned i = 0; i < n; ++i) {
            asc[i] = dist(rng);
            desc[i] = dist(rng);
        }
        emit("float_keys_asc_in_" + std::to_string(n), asc);
        emit("float_keys_desc_in_" + std::to_string(n), desc);
        std::sort(asc.begin(), asc.end());
        std::sort(desc.begin(), desc.end(), std::greater<float>());
        emit("float_keys_asc_out_" + std::to_string(n), asc);
        emit("float_keys_desc_out_" + std::to_string(n), desc);
    }
}

// tests/device_radix_sort_one_sweep.cpp:175-205 -- u64 keys (n-i-1)*2654435761,
// n = 65536, expected = std::sort.
static void u64_keys()
{
    const unsigned n = 65536;
    std::vector<uint64_t> keys(n);
    for (unsigned i = 0; i < n; ++i) keys[i] = static_cast<uint64_t>((n - i - 1) * 2654435761ull);
    emit("u64_keys_in", keys);
    std::sort(keys.begin(), keys.end());
    emit("u64_keys_out", keys);
}

// tests/device_radix_sort_one_sweep.cpp:207-333 -- pairs: shuffled index keys
// (std::shuffle with std::mt19937(114521), ascending input first, then the
// descending one), float values U[0,1) drawn afterwards from the same engine;
// expected = std::sort of (key, value) by key, ascending and descending.
// The reference uses 524288 items; 32768 keeps the fixture small.
static void pairs_u32_f32()
{
    const int n = 32768;
    std::vector<uint32_t> key(n), dkey(n);
    std::vector<float> val(n), dval(n);
    std::mt19937 rng(114521);
    std::uniform_real_distribution<float> dist(0.0f, 1.0f);
    for (int i = 0; i < n; ++i) key[i] = dkey[i] = static_cast<uint32_t>(i);
    std::shuffle(key.begin(), key.end(), rng);
    std::shuffle(dkey.begin(), dkey.end(), rng);
    for (int i = 0; i < n; ++i) {
        val[i] = dist(rng);
        dval[i] = dist(rng);
    }
    emit("pairs_asc_keys_in", key);
    emit("pairs_asc_vals_in", val);
    emit("pairs_desc_keys_in", dkey);
    emit("pairs_desc_vals_in", dval);
    std::vector<std::pair<uint32_t, float>> a(n), d(n);
    for (int i = 0; i < n; ++i) {
        a[i] = {key[i], val[i]};
        d[i] = {dkey[i], dval[i]};
    }
    std::sort(a.begin(), a.end(), [](auto& x, auto& y) { return x.first < y.first; });
    std::sort(d.begin(), d.end(), [](auto& x, auto& y) { return x.first > y.first; });
    std::vector<uint32_t> ak(n), dk(n);
    std::vector<float> av(n), dv(n);
    for (int i = 0; i < n; ++i) {
        ak[i] = a[i].first; av[i] = a[i].second;
        dk[i] = d[i].first; dv[i] = d[i].second;
    }
    emit("pairs_asc_keys_out", ak);
    emit("pairs_asc_vals_out", av);
    emit("pairs_desc_keys_out", dk);
    emit("pairs_desc_vals_out", dv);
}

// Stable order of indices by the selected bits, ascending / descending.
static void stable_orders(const std::vector<uint32_t>& keys, unsigned begin, unsigned end,
                          std::vector<uint32_t>& asc, std::vector<uint32_t>& desc)
{
    auto sel = [&](uint32_t k) { return (k >> begin) & ((1u << (end - begin)) - 1u); };
    asc.resize(keys.size());
    desc.resize(keys.size());
    std::iota(asc.begin(), asc.end(), 0u);
    std::iota(desc.begin(), desc.end(), 0u);
    std::stable_sort(asc.begin(), asc.end(), [&](uint32_t l, uint32_t r) { return sel(keys[l]) < sel(keys[r]); });
    std::stable_sort(desc.begin(), desc.end(), [&](uint32_t l, uint32_t r) { return sel(keys[l]) > sel(keys[r]); });
}

// tests/device_radix_sort_interface_test.cpp:68-158 -- 257 keys
// ((i*53)%64) | (((i*17)%11)<<8), values = i, bits [1,6).
// tests/device_radix_sort_interface_test.cpp:205-283 -- 65 keys
// ((i*19)%32) | ((i%7)<<8), bits [0,5), DoubleBuffer.
static void interface_cases()
{
    {
        const unsigned n = 257;
        std::vector<uint32_t> keys(n), vals(n), asc, desc;
        for (unsigned i = 0; i < n; ++i) {
            keys[i] = ((i * 53u) % 64u) | (((i * 17u) % 11u) << 8u);
            vals[i] = i;
        }
        stable_orders(keys, 1, 6, asc, desc);
        emit("partial_bits_keys", keys);
        emit("partial_bits_vals", vals);
        emit("partial_bits_asc_order", asc);
        emit("partial_bits_desc_order", desc);
    }
    {
        const unsigned n = 65;
        std::vector<uint32_t> keys(n), vals(n), asc, desc;
        for (unsigned i = 0; i < n; ++i) {
            keys[i] = ((i * 19u) % 32u) | ((i % 7u) << 8u);
            vals[i] = i;
        }
        stable_orders(keys, 0, 5, asc, desc);
        emit("double_buffer_keys", keys);
        emit("double_buffer_vals", vals);
        emit("double_buffer_asc_order", asc);
        emit("double_buffer_desc_order", desc);
    }
}

// tests/device_scan_test.cpp:189-265 -- (i%7)-3 at 384*22*3+17 and
// 320*25*3+17, expected = running (inclusive) sum.
// tests/scan_optimization_regression_test.cpp:124-190 -- tile-boundary sizes,
// value(i) = i%7+1, exclusive / inclusive sums and init-3 forms at 16003.
static void scan_cases()
{
    for (size_t n : {size_t(384 * 22 * 3 + 17), size_t(320 * 25 * 3 + 17)}) {
        std::vector<int32_t> in(n), out(n);
        for (size_t i = 0; i < n; ++i) in[i] = static_cast<int32_t>(i % 7u) - 3;
        std::inclusive_scan(in.begin(), in.end(), out.begin());
        emit("scan_mod7_in_" + std::to_string(n), in);
        emit("scan_mod7_inclusive_" + std::to_string(n), out);
    }
    const size_t sizes[] = {0, 1, 31, 32, 33, 255, 256, 257, 3839, 3840, 3841, 4095, 4096, 4097,
                            7999, 8000, 8001, 16003, 262147};
    for (size_t n : sizes) {
        std::vector<int32_t> in(n), ex(n), inc(n);
        for (size_t i = 0; i < n; ++i) in[i] = static_cast<int32_t>(i % 7u + 1u);
        std::exclusive_scan(in.begin(), in.end(), ex.begin(), 0);
        std::inclusive_scan(in.begin(), in.end(), inc.begin());
        emit("scan_tiles_exclusive_" + std::to_string(n), ex);
        emit("scan_tiles_inclusive_" + std::to_string(n), inc);
        if (n == 16003) {
            std::vector<int32_t> ex3(n), inc3(n);
            std::exclusive_scan(in.begin(), in.end(), ex3.begin(), 3);
            std::inclusive_scan(in.begin(), in.end(), inc3.begin(), std::plus<int32_t>(), 3);
            emit("scan_tiles_exclusive_init3_16003", ex3);
            emit("scan_tiles_inclusive_init3_16003", inc3);
        }
    }
    // tests/device_scan_test.cpp:288-322 -- InclusiveScanInit {1,2,3,4}, init 10.
    std::vector<int32_t> in{1, 2, 3, 4}, out(4);
    std::inclusive_scan(in.begin(), in.end(), out.begin(), std::plus<int32_t>(), 10);
    emit("scan_init_in", in);
    emit("scan_init_out", out);
}

// tests/device_reduce_test.cpp:78-91 and :160-217 -- 0..4095 shuffled with
// std::mt19937(114521); expected min / max via std::min_element /
// std::max_element.
static void reduce_cases()
{
    const int n = 1 << 12;
    std::vector<int32_t> data(n);
    for (int i = 0; i < n; ++i) data[i] = i;
    std::mt19937 rng(114521);
    std::shuffle(data.begin(), data.end(), rng);
    emit("reduce_shuffled_in", data);
    std::vector<int32_t> mm{*std::min_element(data.begin(), data.end()),
                            *std::max_element(data.begin(), data.end())};
    emit("reduce_shuffled_minmax", mm);
}

// tests/device_reduce_test.cpp:238-330 -- ArgMax of {1, 9, 4, 9, 3} is
// (9, 1) (first of equal maxima); float ArgMax of {-7, -3, -5} is (-3, 1);
// with the comparator "last decimal digit less", {21, 11, 33, 23, 8, 28}
// gives ArgMin (21, 0) and ArgMax (8, 4).  Expected pairs come from a
// first-index scan with std::min_element / std::max_element semantics.
static void arg_cases()
{
    const std::vector<int32_t> ties{1, 9, 4, 9, 3};
    emit("arg_ties_in", ties);
    const auto mx = std::max_element(ties.begin(), ties.end());  // first of equal maxima
    emit("arg_ties_max", std::vector<int32_t>{*mx, int32_t(mx - ties.begin())});
    const std::vector<float> neg{-7.0f, -3.0f, -5.0f};
    emit("arg_negative_in", neg);
    const auto nmx = std::max_element(neg.begin(), neg.end());
    emit("arg_negative_max", std::vector<float>{*nmx, float(nmx - neg.begin())});
    const std::vector<int32_t> digits{21, 11, 33, 23, 8, 28};
    emit("arg_digit_in", digits);
    auto last_digit_less = [](int32_t l, int32_t r) { return l % 10 < r % 10; };
    const auto dmn = std::min_element(digits.begin(), digits.end(), last_digit_less);
    const auto dmx = std::max_element(digits.begin(), digits.end(), last_digit_less);
    emit("arg_digit_minmax", std::vector<int32_t>{*dmn, int32_t(dmn - digits.begin()), *dmx,
                                                  int32_t(dmx - digits.begin())});
}

// tests/device_scan_test.cpp:324-380 -- ExclusiveSumByKey over ones with
// keys i / 100 (one size of the reference's 2^5..2^23 loop: 2^12); expected
// = std::exclusive_scan per segment.  :382-417 -- InclusiveSumByKey of int64
// ones over int keys 1 | 2 | 3 split at one item past each of the
// reference's 1024-item tiles (2050 items); expected = the running count in
// each segment.  :419-446 -- keys {1, 3, 5, 2, 4} under "same parity"
// equality: InclusiveSumByKey of ones = {1, 2, 3, 1, 2}.
// tests/device_reduce_test.cpp:422-483 -- ReduceByKey (Sum) of the shuffled
// 0..4095 of reduce_cases over keys i / 100; expected = per-segment sums.
static void by_key_cases()
{
    const int n = 1 << 12, per = 100;
    std::vector<int32_t> keys(n), ones(n, 1), excl(n);
    for (int i = 0; i < n; ++i) keys[i] = i / per;
    for (int s0 = 0; s0 < n; s0 += per)
        std::exclusive_scan(ones.begin() + s0, ones.begin() + std::min(s0 + per, n), excl.begin() + s0, 0);
    emit("sbk_segment_keys", keys);
    emit("sbk_exclusive_sum_out", excl);

    const size_t tile = 256 * 4, m = tile * 2 + 2;
    std::vector<int32_t> k3(m);
    std::vector<int64_t> incl(m);
    int64_t run = 0;
    for (size_t i = 0; i < m; ++i) {
        k3[i] = i < tile + 1 ? 1 : i < tile * 2 + 1 ? 2 : 3;
        if (i == 0 || k3[i] != k3[i - 1]) run = 0;
        incl[i] = ++run;
    }
    emit("sbk_three_tiles_keys", k3);
    emit("sbk_three_tiles_inclusive_out", incl);

    emit("sbk_parity_keys", std::vector<int32_t>{1, 3, 5, 2, 4});
    emit("sbk_parity_inclusive_out", std::vector<int32_t>{1, 2, 3, 1, 2});

    std::vector<int32_t> data(n);
    for (int i = 0; i < n; ++i) data[i] = i;
    std::mt19937 rng(114521);
    std::shuffle(data.begin(), data.end(), rng);
    std::vector<int32_t> uniq, agg;
    for (int s0 = 0; s0 < n; s0 += per) {
        uniq.push_back(keys[s0]);
        agg.push_back(std::accumulate(data.begin() + s0, data.begin() + std::min(s0 + per, n), 0));
    }
    emit("rbk_unique_out", uniq);
    emit("rbk_aggregates_out", agg);
}

// tests/device_select_test.cpp and tests/device_partition_test.cpp: the
// select / partition cases with their host expectations (std::copy_if,
// std::unique, and the reverse walk for rejected items).
template <typename T, typename P>
static std::vector<T> keep(const std::vector<T>& v, P p)
{
    std::vector<T> out;
    std::copy_if(v.begin(), v.end(), std::back_inserter(out), p);
    return out;
}

static void select_cases()
{
    // device_select_test.cpp:254-320: Flagged (flags 7 at i % 3 == 1) and If(even), 17 items
    std::vector<int32_t> in(17);
    std::vector<uint32_t> flags(17);
    for (int i = 0; i < 17; ++i) {
        in[i] = 100 + i;
        flags[i] = i % 3 == 1 ? 7u : 0u;
    }
    emit("sel_stable_in", in);
    emit("sel_stable_flags", flags);
    std::vector<int32_t> fl;
    for (int i = 0; i < 17; ++i)
        if (flags[i]) fl.push_back(in[i]);
    emit("sel_stable_flagged_out", fl);
    emit("sel_stable_if_even_out", keep(in, [](int32_t x) { return x % 2 == 0; }));

    // :322-372: Unique and UniqueByKey keep the first item of each run
    const std::vector<int32_t> keys{1, 1, 2, 2, 2, 4, 7, 7, 9}, values{10, 11, 20, 21, 22, 40, 70, 71, 90};
    emit("sel_unique_keys", keys);
    emit("sel_unique_values", values);
    std::vector<int32_t> uk, uv;
    for (size_t i = 0; i < keys.size(); ++i)
        if (i == 0 || keys[i] != keys[i - 1]) {
            uk.push_back(keys[i]);
            uv.push_back(values[i]);
        }
    emit("sel_unique_keys_out", uk);
    emit("sel_unique_values_out", uv);

    // :374-430: FlaggedIf with "flag > 0 and odd" over flags -3..5
    std::vector<int32_t> fin(9), ff(9), fif;
    for (int i = 0; i < 9; ++i) {
        fin[i] = 100 + i;
        ff[i] = i - 3;
        if (ff[i] > 0 && ff[i] % 2 != 0) fif.push_back(fin[i]);
    }
    emit("sel_flaggedif_in", fin);
    emit("sel_flaggedif_flags", ff);
    emit("sel_flaggedif_out", fif);

    // :432-500: in place -- Flagged with the data as its own flags, If(> 0),
    // Unique under "same parity" and under ==
    const std::vector<int32_t> aliased{0, 2, 0, 3, 4, 0, 5, 0}, pred{-3, 4, -1, 6, 0, 2, 7, -8},
        uniq_par{1, 3, 2, 4, 5, 7, 8, 10}, uniq_def{1, 1, 2, 2, 2, 4, 4, 9};
    emit("sel_inplace_aliased", aliased);
    emit("sel_inplace_aliased_out", keep(aliased, [](int32_t x) { return x != 0; }));
    emit("sel_inplace_pred", pred);
    emit("sel_inplace_pred_out", keep(pred, [](int32_t x) { return x > 0; }));
    std::vector<int32_t> up;
    for (size_t i = 0; i < uniq_par.size(); ++i)
        if (i == 0 || uniq_par[i] % 2 != uniq_par[i - 1] % 2) up.push_back(uniq_par[i]);
    emit("sel_inplace_unique_parity", uniq_par);
    emit("sel_inplace_unique_parity_out", up);
    std::vector<int32_t> ud = uniq_def;
    ud.erase(std::unique(ud.begin(), ud.end()), ud.end());
    emit("sel_inplace_unique", uniq_def);
    emit("sel_inplace_unique_out", ud);

    // :114-172: wide values (1 << 40 | i / 3) with bool flags (i % 3 == 1)
    std::vector<uint64_t> wide(17);
    std::vector<uint8_t> bflags(17);
    for (int i = 0; i < 17; ++i) {
        wide[i] = (uint64_t(1) << 40) | uint64_t(i / 3);
        bflags[i] = i % 3 == 1;
    }
    emit("sel_wide_in", wide);
    emit("sel_wide_flags", bflags);
    std::vector<uint64_t> wf;
    for (int i = 0; i < 17; ++i)
        if (bflags[i]) wf.push_back(wide[i]);
    emit("sel_wide_flagged_out", wf);
    emit("sel_wide_if_even_out", keep(wide, [](uint64_t x) { return x % 2 == 0; }));
    std::vector<uint64_t> wu = wide;
    wu.erase(std::unique(wu.begin(), wu.end()), wu.end());
    emit("sel_wide_unique_out", wu);

    // device_partition_test.cpp:122-204: Flagged (i % 3 == 0) and If(< 7) over 0..11,
    // rejected items in reverse order after the selected ones
    std::vector<int32_t> pin(12), pf_out, pi_out;
    std::vector<uint32_t> pflags(12);
    for (int i = 0; i < 12; ++i) {
        pin[i] = i;
        pflags[i] = i % 3 == 0;
    }
    for (int i = 0; i < 12; ++i) {
        if (pflags[i]) pf_out.push_back(pin[i]);
        if (pin[i] < 7) pi_out.push_back(pin[i]);
    }
    for (int i = 12; i-- > 0;) {
        if (!pflags[i]) pf_out.push_back(pin[i]);
        if (pin[i] >= 7) pi_out.push_back(pin[i]);
    }
    emit("part_in", pin);
    emit("part_flags", pflags);
    emit("part_flagged_out", pf_out);
    emit("part_if_lt7_out", pi_out);

    // :293-353: three-way, first = divisible by 3, second = < 8
    std::vector<int32_t> first, second, rest;
    for (int i = 0; i < 12; ++i) {
        if (i % 3 == 0) first.push_back(i);
        else if (i < 8) second.push_back(i);
    }
    for (int i = 12; i-- > 0;)
        if (i % 3 != 0 && i >= 8) rest.push_back(i);
    emit("part3_first_out", first);
    emit("part3_second_out", second);
    emit("part3_unselected_out", rest);
}

// tests/device_segmented_sort_test.cpp:22-56 and :260-268 -- 19 items in
// segments [1,4) [5,5) [5,9) [10,19); keys outside every segment are -777
// and their values UINT_MAX; expected = std::stable_sort per segment with
// std::less / std::greater (the reference's segmented_order helper).
static void segmented_cases()
{
    const unsigned n = 19, segments = 4;
    const std::vector<uint32_t> begin{1u, 5u, 5u, 10u}, end{4u, 5u, 9u, 19u};
    std::vector<int32_t> keys{91, 3, -2, 3, 92, 8, 1, 8, 4, 93, 5, -1, 5, 2, -1, 7, 2, 5, 0};
    std::vector<uint32_t> vals(n);
    std::iota(vals.begin(), vals.end(), 0u);
    auto in_segment = [&](unsigned i) {
        for (unsigned s = 0; s < segments; ++s)
            if (i >= begin[s] && i < end[s]) return true;
        return false;
    };
    for (unsigned i = 0; i < n; ++i)
        if (!in_segment(i)) {
            keys[i] = -777;
            vals[i] = 0xffffffffu;
        }
    auto order = [&](bool desc) {
        std::vector<uint32_t> ord(n, 0xffffffffu);
        for (unsigned s = 0; s < segments; ++s) {
            std::vector<uint32_t> o(end[s] - begin[s]);
            std::iota(o.begin(), o.end(), begin[s]);
            std::stable_sort(o.begin(), o.end(), [&](uint32_t l, uint32_t r) {
                return desc ? keys[l] > keys[r] : keys[l] < keys[r];
            });
            std::copy(o.begin(), o.end(), ord.begin() + begin[s]);
        }
        return ord;
    };
    emit("segmented_keys", keys);
    emit("segmented_vals", vals);
    emit("segmented_begin", begin);
    emit("segmented_end", end);
    emit("segmented_asc_order", order(false));
    emit("segmented_desc_order", order(true));
}

// tests/device_radix_sort_interface_test.cpp:285-330 -- 8 keys
// {uint primary; int secondary}, decomposed as (primary, secondary); full
// stable orders by std::tie and the window [28, 36) (low 4 bits of primary,
// top 4 bits of the twiddled secondary).
static void decomposed_cases()
{
    const std::vector<uint32_t> primary{1u, 0u, 1u, 2u, 0u, 1u, 2u, 0u};
    const std::vector<int32_t> secondary{-1, 7, -1, -8, 3, 4, 0, 7};
    const unsigned n = 8;
    auto cross = [&](unsigned i) {
        const uint32_t sb = static_cast<uint32_t>(secondary[i]) ^ 0x80000000u;
        return ((primary[i] & 0x0fu) << 4u) | ((sb >> 28u) & 0x0fu);
    };
    auto order = [&](auto less) {
        std::vector<uint32_t> o(n);
        std::iota(o.begin(), o.end(), 0u);
        std::stable_sort(o.begin(), o.end(), less);
        return o;
    };
    emit("decomposed_primary", primary);
    emit("decomposed_secondary", secondary);
    emit("decomposed_full_asc_order", order([&](uint32_t l, uint32_t r) {
        return std::tie(primary[l], secondary[l]) < std::tie(primary[r], secondary[r]);
    }));
    emit("decomposed_full_desc_order", order([&](uint32_t l, uint32_t r) {
        return std::tie(primary[l], secondary[l]) > std::tie(primary[r], secondary[r]);
    }));
    emit("decomposed_window_asc_order", order([&](uint32_t l, uint32_t r) { return cross(l) < cross(r); }));
    emit("decomposed_window_desc_order", order([&](uint32_t l, uint32_t r) { return cross(l) > cross(r); }));
}

int main(int argc, char** argv)
{
    if (argc != 2) {
        std::fprintf(stderr, "usage: %s <out_dir>\n", argv[0]);
        return 2;
    }
    g_dir = argv[1];
    g_index = std::fopen((g_dir + "/arrays.txt").c_str(), "w");
    if (!g_index) { std::perror("arrays.txt"); return 1; }
    float_keys();
    u64_keys();
    pairs_u32_f32();
    interface_cases();
    scan_cases();
    reduce_cases();
    arg_cases();
    by_key_cases();
    select_cases();
    segmented_cases();
    decomposed_cases();
    std::fclose(g_index);
    return 0;
}
