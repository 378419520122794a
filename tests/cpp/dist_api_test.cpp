// C++ caller of the distributed C ABI (include/lcpp_b200_dist.h) with no
// Python involved: the parent forks one process per GPU (it makes no CUDA
// call itself), rank 0 creates the communicator ID and hands it to the other
// ranks through pipes, and every rank sorts, scans and reduces its share.
// Each rank regenerates all ranks' inputs on the host and checks its part
// against std::stable_sort / std::inclusive_scan of the concatenation.
// Built and run by tests/test_cpp_api.py on a GPU box (also compiled, not
// run, on the CPU).  Usage: dist_api_test <ranks>; prints "OK <ranks>".
#include <cuda_runtime.h>
#include <sys/wait.h>
#include <unistd.h>

#include <algorithm>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <numeric>
#include <vector>

#include "lcpp_b200.h"
#include "lcpp_b200_dist.h"

namespace {

#define CHECK(cond)                                                                           \
    do {                                                                                      \
        if (!(cond)) {                                                                        \
            std::fprintf(stderr, "rank %d: FAILED %s at %s:%d\n", g_rank, #cond, __FILE__, __LINE__); \
            std::_Exit(1);                                                                    \
        }                                                                                     \
    } while (0)

int g_rank = -1;

uint64_t mix(uint64_t z)
{
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

uint64_t keys_of(int rank) { return (1u << 18) + 1000u * uint64_t(rank); }

// rank r's u32 keys: uniform with one value (a heavy hitter) in 1 of 3
std::vector<uint32_t> u32_keys(int rank)
{
    std::vector<uint32_t> k(keys_of(rank));
    for (size_t i = 0; i < k.size(); ++i) {
        const uint64_t z = mix(uint64_t(rank) << 32 | i);
        k[i] = (z % 3 == 0) ? 0x9E3779B9u : uint32_t(z >> 32);
    }
    return k;
}

// rank r's f32 keys: values in [-8, 8) and both signed zeros
std::vector<float> f32_keys(int rank)
{
    std::vector<float> k(keys_of(rank) / 2 + 7 * rank);
    for (size_t i = 0; i < k.size(); ++i) {
        const uint64_t z = mix(0xF00Dull << 40 | uint64_t(rank) << 32 | i);
        k[i] = (i % 17 == 0) ? 0.0f : (i % 19 == 0) ? -0.0f : float(int64_t(z % 16000) - 8000) / 1000.0f;
    }
    return k;
}

// order-preserving image of a float (the sort's bijection, +-0.0 folded)
uint32_t image(float f)
{
    uint32_t b;
    std::memcpy(&b, &f, 4);
    uint32_t t = (b & 0x80000000u) ? ~b : (b ^ 0x80000000u);
    return t == 0x7FFFFFFFu ? 0x80000000u : t;
}

template <typename T>
T* to_device(const std::vector<T>& h)
{
    T* d = nullptr;
    CHECK(cudaMalloc(&d, std::max<size_t>(h.size(), 1) * sizeof(T)) == cudaSuccess);
    CHECK(cudaMemcpy(d, h.data(), h.size() * sizeof(T), cudaMemcpyHostToDevice) == cudaSuccess);
    return d;
}

template <typename T>
std::vector<T> to_host(const T* d, size_t n)
{
    std::vector<T> h(n);
    CHECK(cudaMemcpy(h.data(), d, n * sizeof(T), cudaMemcpyDeviceToHost) == cudaSuccess);
    return h;
}

// this rank's part of the stable sort (by `less`) of all ranks' keys
template <typename T, typename Gen, typename Less>
std::vector<T> expected_part(int rank, int ranks, Gen gen, Less less)
{
    std::vector<T> all;
    size_t lo = 0, n = 0;
    for (int q = 0; q < ranks; ++q) {
        const std::vector<T> k = gen(q);
        if (q == rank) {
            lo = all.size();
            n = k.size();
        }
        all.insert(all.end(), k.begin(), k.end());
    }
    std::stable_sort(all.begin(), all.end(), less);
    return std::vector<T>(all.begin() + lo, all.begin() + lo + n);
}

template <typename T>
void sort_and_check(lcpp_comm comm, int rank, int ranks, const std::vector<T>& keys, const std::vector<T>& want,
                    lcpp_dtype dt, int exchange)
{
    size_t bytes = 0;
    CHECK(lcpp_dist_sort_keys_temp_bytes(comm, dt, keys.size(), &bytes) == LCPP_OK);
    void* temp = nullptr;
    CHECK(cudaMalloc(&temp, bytes) == cudaSuccess);
    T* d = to_device(keys);
    lcpp_dist_sort_times times{};
    CHECK(lcpp_dist_sort_keys(comm, temp, bytes, d, d, keys.size(), dt, exchange, &times, nullptr) == LCPP_OK);
    const std::vector<T> got = to_host(d, keys.size());
    CHECK(std::memcmp(got.data(), want.data(), want.size() * sizeof(T)) == 0);
    CHECK(lcpp_device_status(temp, nullptr) == LCPP_OK);
    // one host: peer loads (2-3 ranks under AUTO, or PEER) or copy-engine
    // pushes (4+ ranks under AUTO)
    if (ranks > 1 && exchange == LCPP_EXCHANGE_PEER) CHECK(times.peer_exchange == 1);
    if (ranks > 1 && exchange == LCPP_EXCHANGE_AUTO) CHECK(times.peer_exchange == (ranks >= 4 ? 2 : 1));
    cudaFree(d);
    cudaFree(temp);
    (void)rank;
}

int run_rank(int rank, int ranks, int id_in, const std::vector<int>& id_out)
{
    g_rank = rank;
    CHECK(cudaSetDevice(rank) == cudaSuccess);
    unsigned char id[LCPP_COMM_ID_BYTES];
    if (rank == 0) {
        CHECK(lcpp_comm_unique_id(id) == LCPP_OK);
        for (int fd : id_out) CHECK(write(fd, id, sizeof(id)) == ssize_t(sizeof(id)));
    } else {
        CHECK(read(id_in, id, sizeof(id)) == ssize_t(sizeof(id)));
    }
    lcpp_comm comm = nullptr;
    CHECK(lcpp_comm_init(id, ranks, rank, &comm) == LCPP_OK);
    int r = -1, g = 0;
    CHECK(lcpp_comm_rank(comm, &r, &g) == LCPP_OK && r == rank && g == ranks);

    // SortKeys, u32 with a heavy hitter that spans ranks, both exchanges
    const auto want_u = expected_part<uint32_t>(rank, ranks, u32_keys, std::less<uint32_t>());
    for (int ex : {LCPP_EXCHANGE_AUTO, LCPP_EXCHANGE_NCCL})
        sort_and_check(comm, rank, ranks, u32_keys(rank), want_u, LCPP_U32, ex);
    // f32: equal keys with different bits (+-0.0) keep rank / input order
    const auto want_f = expected_part<float>(rank, ranks, f32_keys,
                                             [](float a, float b) { return image(a) < image(b); });
    sort_and_check(comm, rank, ranks, f32_keys(rank), want_f, LCPP_F32, LCPP_EXCHANGE_AUTO);

    // InclusiveSum / ExclusiveSum and Reduce over all ranks' items
    auto vals = [](int q) {
        std::vector<int32_t> v(keys_of(q) / 4);
        for (size_t i = 0; i < v.size(); ++i) v[i] = int32_t(mix(0xABCull << 40 | uint64_t(q) << 32 | i) % 2001) - 1000;
        return v;
    };
    int64_t before = 0, total = 0;
    for (int q = 0; q < ranks; ++q) {
        const auto v = vals(q);
        const int64_t s = std::accumulate(v.begin(), v.end(), int64_t(0));
        if (q < rank) before += s;
        total += s;
    }
    const auto mine = vals(rank);
    int32_t* din = to_device(mine);
    int32_t* dout = nullptr;
    CHECK(cudaMalloc(&dout, mine.size() * 4) == cudaSuccess);
    size_t bytes = 0;
    CHECK(lcpp_dist_scan_temp_bytes(comm, LCPP_I32, mine.size(), &bytes) == LCPP_OK);
    void* temp = nullptr;
    CHECK(cudaMalloc(&temp, bytes) == cudaSuccess);
    CHECK(lcpp_dist_inclusive_sum(comm, temp, bytes, din, dout, mine.size(), LCPP_I32, nullptr) == LCPP_OK);
    std::vector<int32_t> got = to_host(dout, mine.size());
    int64_t run = before;
    for (size_t i = 0; i < mine.size(); ++i) {
        run += mine[i];
        CHECK(got[i] == int32_t(run));
    }
    CHECK(lcpp_dist_exclusive_sum(comm, temp, bytes, din, dout, mine.size(), LCPP_I32, nullptr) == LCPP_OK);
    got = to_host(dout, mine.size());
    CHECK(got[0] == int32_t(before));
    const int32_t init = 3;
    CHECK(lcpp_dist_reduce(comm, temp, bytes, din, dout, mine.size(), LCPP_OP_SUM, &init, LCPP_I32, nullptr) ==
          LCPP_OK);
    CHECK(to_host(dout, 1)[0] == int32_t(total + 3));
    cudaFree(temp);
    cudaFree(din);
    cudaFree(dout);
    CHECK(cudaDeviceSynchronize() == cudaSuccess);
    CHECK(lcpp_comm_destroy(comm) == LCPP_OK);
    return 0;
}

}  // namespace

int main(int argc, char** argv)
{
    const int ranks = argc > 1 ? std::atoi(argv[1]) : 1;
    if (ranks < 1 || ranks > 8) return 2;
    std::vector<int> rd(ranks, -1), wr;
    for (int q = 1; q < ranks; ++q) {
        int fd[2];
        if (pipe(fd) != 0) return 2;
        rd[q] = fd[0];
        wr.push_back(fd[1]);
    }
    std::vector<pid_t> kids;
    for (int q = 0; q < ranks; ++q) {
        const pid_t p = fork();
        if (p == 0) std::_Exit(run_rank(q, ranks, rd[q], q == 0 ? wr : std::vector<int>()));
        kids.push_back(p);
    }
    int bad = 0;
    for (pid_t p : kids) {
        int st = 0;
        waitpid(p, &st, 0);
        bad += !(WIFEXITED(st) && WEXITSTATUS(st) == 0);
    }
    if (bad) return 1;
    std::printf("OK %d\n", ranks);
    return 0;
}
