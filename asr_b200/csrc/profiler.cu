// Event-based kernel timer behind asr_profiler_enable / asr_profiler_report.
#include <cstdio>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <vector>

#include "asr_b200.h"
#include "profiler.cuh"

namespace asr {
namespace {

struct Record {
    const char* name;
    cudaEvent_t start, stop;
};

std::mutex g_mu;
bool g_on = false;
std::vector<Record> g_records;
std::vector<cudaEvent_t> g_pool;

cudaEvent_t take_event() {
    if (!g_pool.empty()) {
        cudaEvent_t e = g_pool.back();
        g_pool.pop_back();
        return e;
    }
    cudaEvent_t e = nullptr;
    if (cudaEventCreate(&e) != cudaSuccess) return nullptr;
    return e;
}

}  // namespace

KernelTimer::KernelTimer(const char* name, cudaStream_t stream) : name_(name), stream_(stream) {
    nvtxRangePushA(name);
    std::lock_guard<std::mutex> lock(g_mu);
    if (!g_on) return;
    start_ = take_event();
    if (start_) cudaEventRecord(start_, stream_);
}

KernelTimer::~KernelTimer() {
    nvtxRangePop();
    if (!start_) return;
    std::lock_guard<std::mutex> lock(g_mu);
    cudaEvent_t stop = take_event();
    if (!stop) return;
    cudaEventRecord(stop, stream_);
    g_records.push_back({name_, start_, stop});
}

}  // namespace asr

using namespace asr;

extern "C" int asr_profiler_enable(int on) {
    std::lock_guard<std::mutex> lock(g_mu);
    g_on = on != 0;
    return ASR_OK;
}

extern "C" int asr_profiler_report(char* buf, size_t len, int clear) {
    std::lock_guard<std::mutex> lock(g_mu);
    std::map<std::string, std::pair<long, double>> agg;
    for (const Record& r : g_records) {
        if (cudaEventSynchronize(r.stop) != cudaSuccess) return -ASR_ERR_CUDA;
        float ms = 0.f;
        if (cudaEventElapsedTime(&ms, r.start, r.stop) != cudaSuccess) return -ASR_ERR_CUDA;
        auto& a = agg[r.name];
        a.first += 1;
        a.second += ms;
    }
    std::string out;
    char line[256];
    for (const auto& kv : agg) {
        std::snprintf(line, sizeof(line), "%s %ld %.6f\n", kv.first.c_str(), kv.second.first, kv.second.second);
        out += line;
    }
    if (clear) {
        for (const Record& r : g_records) {
            g_pool.push_back(r.start);
            g_pool.push_back(r.stop);
        }
        g_records.clear();
    }
    if (buf && len > 0) {
        const size_t n = out.size() < len - 1 ? out.size() : len - 1;
        std::memcpy(buf, out.data(), n);
        buf[n] = '\0';
    }
    return (int)out.size();
}
