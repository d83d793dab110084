// trace.cu -- optional per-kernel CUDA-event timing (dc_kernel_timing / _report).
#include <cuda_runtime.h>

#include <cstdio>
#include <map>
#include <mutex>
#include <string>
#include <vector>

#include "common.cuh"
#include "trace.h"

namespace dc {
namespace {

struct Record {
    const char *name;
    cudaEvent_t start, stop;
};

std::mutex g_mu;
bool g_enabled = false;
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

bool trace_enabled() {
    std::lock_guard<std::mutex> lk(g_mu);
    return g_enabled;
}

KernelTrace::KernelTrace(const char *name, cudaStream_t stream) : name_(name), stream_(stream) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g_enabled) return;
    start_ = take_event();
    if (start_) cudaEventRecord(start_, stream_);
}

KernelTrace::~KernelTrace() {
    if (!start_) return;
    std::lock_guard<std::mutex> lk(g_mu);
    cudaEvent_t stop = take_event();
    if (!stop) return;
    cudaEventRecord(stop, stream_);
    g_records.push_back({name_, start_, stop});
}

}  // namespace dc

using namespace dc;

extern "C" {

int dc_kernel_timing(int enable) {
    std::lock_guard<std::mutex> lk(g_mu);
    g_enabled = enable != 0;
    return DC_OK;
}

int dc_kernel_timing_report(char *buf, size_t len, int reset) {
    std::lock_guard<std::mutex> lk(g_mu);
    std::map<std::string, std::pair<long, double>> agg;
    long n = 0;
    for (auto &r : g_records) {
        if (cudaEventSynchronize(r.stop) != cudaSuccess) return -1;
        float ms = 0.f;
        if (cudaEventElapsedTime(&ms, r.start, r.stop) != cudaSuccess) return -1;
        auto &a = agg[r.name];
        a.first += 1;
        a.second += ms;
        n++;
    }
    std::string out = "{";
    bool first = true;
    for (auto &kv : agg) {
        char item[256];
        snprintf(item, sizeof item, "%s\"%s\": [%ld, %.6f]", first ? "" : ", ", kv.first.c_str(),
                 kv.second.first, kv.second.second);
        out += item;
        first = false;
    }
    out += "}";
    if (buf && len) {
        size_t m = out.size() < len - 1 ? out.size() : len - 1;
        out.copy(buf, m);
        buf[m] = 0;
    }
    if (reset) {
        for (auto &r : g_records) {
            g_pool.push_back(r.start);
            g_pool.push_back(r.stop);
        }
        g_records.clear();
    }
    return (int)n;
}

}  // extern "C"
