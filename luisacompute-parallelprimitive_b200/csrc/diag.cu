// diag.cu -- optional per-kernel CUDA-event timing (include/lcpp_b200_diag.h).
#include <atomic>
#include <mutex>
#include <vector>

#include "../../include/lcpp_b200_diag.h"
#include "common.cuh"
#include "radix_sort.cuh"

namespace lcpp {
namespace diag {
namespace {

struct Record {
    int kind;
    uint64_t items;
    cudaEvent_t start, stop;
};

std::atomic<int> g_enabled{0};
std::mutex g_mu;
std::vector<Record> g_records;
std::vector<cudaEvent_t> g_pool;

cudaEvent_t take_event()
{
    if (!g_pool.empty()) {
        cudaEvent_t e = g_pool.back();
        g_pool.pop_back();
        return e;
    }
    cudaEvent_t e = nullptr;
    cudaEventCreate(&e);
    return e;
}

void recycle_all()
{
    for (auto& r : g_records) {
        g_pool.push_back(r.start);
        g_pool.push_back(r.stop);
    }
    g_records.clear();
}

}  // namespace

KernelTimer::KernelTimer(int kind, uint64_t items, cudaStream_t stream) : index_(-1), stream_(stream)
{
    if (!g_enabled.load(std::memory_order_relaxed)) return;
    std::lock_guard<std::mutex> lk(g_mu);
    Record r{kind, items, take_event(), take_event()};
    if (!r.start || !r.stop) return;
    cudaEventRecord(r.start, stream);
    g_records.push_back(r);
    index_ = int(g_records.size()) - 1;
}

void KernelTimer::stop()
{
    if (index_ < 0) return;
    std::lock_guard<std::mutex> lk(g_mu);
    if (index_ < int(g_records.size())) cudaEventRecord(g_records[index_].stop, stream_);
    index_ = -1;
}

}  // namespace diag
}  // namespace lcpp

extern "C" lcpp_status lcpp_diag_timing_enable(int enable)
{
    using namespace lcpp::diag;
    std::lock_guard<std::mutex> lk(g_mu);
    if (enable) recycle_all();
    g_enabled.store(enable ? 1 : 0);
    return LCPP_OK;
}

extern "C" lcpp_status lcpp_diag_timing_read(lcpp_kernel_time* out, int capacity, int* count)
{
    using namespace lcpp::diag;
    if (!count || (capacity > 0 && !out)) return LCPP_ERR_INVALID_ARG;
    std::lock_guard<std::mutex> lk(g_mu);
    *count = int(g_records.size());
    for (int i = 0; i < capacity && i < int(g_records.size()); ++i) {
        const Record& r = g_records[i];
        if (cudaEventSynchronize(r.stop) != cudaSuccess) return LCPP_ERR_CUDA;
        float ms = 0.f;
        if (cudaEventElapsedTime(&ms, r.start, r.stop) != cudaSuccess) return LCPP_ERR_CUDA;
        out[i].kind = r.kind;
        out[i].ms = ms;
        out[i].items = r.items;
    }
    return LCPP_OK;
}

extern "C" lcpp_status lcpp_diag_wait_timeout_probe(void* temp, size_t temp_bytes, uint64_t limit_ns,
                                                   lcpp_stream_t stream)
{
    return lcpp::radix::wait_timeout_probe(temp, temp_bytes, limit_ns, reinterpret_cast<cudaStream_t>(stream));
}
