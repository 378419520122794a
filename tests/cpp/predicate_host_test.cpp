// Host-only checks of lcpp_b200::Predicate<T> (include/lcpp_b200.hpp): the
// lcpp_clause encoding that crosses the C ABI in place of the reference's
// predicate lambdas.  Needs no GPU: built and run by tests/test_cpp_api.py on
// the CPU.  Prints "OK <checks>" and exits 0 on success.
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>

#include "lcpp_b200.hpp"

using namespace lcpp_b200;

static int g_checks = 0;
#define CHECK(cond)                                                                  \
    do {                                                                             \
        ++g_checks;                                                                  \
        if (!(cond)) {                                                               \
            std::fprintf(stderr, "FAILED %s at %s:%d\n", #cond, __FILE__, __LINE__); \
            std::exit(1);                                                            \
        }                                                                            \
    } while (0)

int main()
{
    // device_select_test.cpp's "value % 2 == 0" and device_partition_test.cpp's "value < 7"
    const auto even = Predicate<int32_t>::mod_eq(2, 0);
    CHECK(even.size() == 1 && even.data()[0].kind == LCPP_CLAUSE_MOD_EQ);
    CHECK(even.data()[0].a == 2u && even.data()[0].b == 0u && even.data()[0].negate == 0);
    const auto lt7 = Predicate<int32_t>::lt(7);
    CHECK(lt7.data()[0].kind == LCPP_CLAUSE_LT && lt7.data()[0].a == 7u);
    // negative integers: the low bytes of the two's-complement pattern
    CHECK(Predicate<int32_t>::gt(-1).data()[0].a == 0xffffffffu);
    CHECK(Predicate<int64_t>::gt(-1).data()[0].a == ~uint64_t(0));
    // floats: their bit patterns
    const float f = 1.5f;
    uint32_t fb = 0;
    std::memcpy(&fb, &f, 4);
    CHECK(Predicate<float>::lt(1.5f).data()[0].a == fb);
    const double d = -2.25;
    uint64_t db = 0;
    std::memcpy(&db, &d, 8);
    CHECK(Predicate<double>::ge(-2.25).data()[0].a == db);
    // "flag > 0 and odd" (device_select_test.cpp:387-388): AND of two clauses, one negated
    const auto pos_odd = Predicate<int32_t>::gt(0) & !Predicate<int32_t>::mod_eq(2, 0);
    CHECK(pos_odd.size() == 2);
    CHECK(pos_odd.data()[0].kind == LCPP_CLAUSE_GT && pos_odd.data()[0].negate == 0);
    CHECK(pos_odd.data()[1].kind == LCPP_CLAUSE_MOD_EQ && pos_odd.data()[1].negate == 1);
    CHECK((!!Predicate<int32_t>::eq(3)).data()[0].negate == 0);
    CHECK(Predicate<uint8_t>::bits_any(0x80).data()[0].a == 0x80u);
    CHECK(Predicate<int32_t>::always().size() == 0);
    // more than LCPP_MAX_CLAUSES clauses, and ! of a conjunction, are misuse
    bool threw = false;
    try {
        auto p = Predicate<int32_t>::gt(0);
        for (int i = 0; i < LCPP_MAX_CLAUSES; ++i) p = p & Predicate<int32_t>::lt(i);
    } catch (const Error& e) {
        threw = e.status() == LCPP_ERR_INVALID_ARG;
    }
    CHECK(threw);
    threw = false;
    try {
        (void)!(Predicate<int32_t>::gt(0) & Predicate<int32_t>::lt(9));
    } catch (const Error& e) {
        threw = e.status() == LCPP_ERR_INVALID_ARG;
    }
    CHECK(threw);
    std::printf("OK %d\n", g_checks);
    return 0;
}
