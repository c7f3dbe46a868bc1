// Per-kernel-class CUDA-event timers (see include/veda/profile.hpp).
#include "veda/profile.hpp"

#include "veda/tensor.hpp"

#include <cuda_runtime.h>

#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <mutex>
#include <stdexcept>
#include <vector>

namespace veda::profile
{

namespace
{
struct Record
{
    std::string name;
    double flops, bytes;
    cudaEvent_t start, stop;
};

std::mutex g_mu;
bool g_enabled = false;

// VEDA_HOST_PROFILE=1: every scope also sums the host (wall-clock) time spent inside it, and the
// totals per name are printed to stderr when the process exits — where the host's issue time
// goes, independent of the device timers.
struct HostTotals
{
    std::map<std::string, std::pair<double, uint64_t>> by_name;   // ms, count
    ~HostTotals()
    {
        if (by_name.empty())
        {
            return;
        }
        std::fprintf(stderr, "veda host profile (ms total, scopes):\n");
        for (const auto& [name, v] : by_name)
        {
            std::fprintf(stderr, "  %-20s %12.3f %10llu\n", name.c_str(), v.first,
                         static_cast<unsigned long long>(v.second));
        }
    }
};
HostTotals g_host;
const bool g_host_enabled = [] {
    const char* v = std::getenv("VEDA_HOST_PROFILE");
    return v != nullptr && v[0] == '1';
}();
std::vector<Record> g_records;     // recorded since the last collect
std::vector<cudaEvent_t> g_free;   // pooled events
std::map<std::string, Totals> g_totals;

cudaEvent_t take()
{
    if (!g_free.empty())
    {
        cudaEvent_t e = g_free.back();
        g_free.pop_back();
        return e;
    }
    cudaEvent_t e = nullptr;
    if (cudaEventCreate(&e) != cudaSuccess)
    {
        throw std::runtime_error("profile: cudaEventCreate failed");
    }
    return e;
}
} // namespace

void enable(bool on)
{
    std::lock_guard<std::mutex> lock(g_mu);
    g_enabled = on;
}

bool enabled() { return g_enabled; }

Scope::Scope(const char* name, double flops, double bytes)
{
    if (g_host_enabled)
    {
        name_ = name;
        host_start_ = std::chrono::duration<double, std::milli>(
                          std::chrono::steady_clock::now().time_since_epoch())
                          .count();
    }
    if (!g_enabled)
    {
        return;
    }
    std::lock_guard<std::mutex> lock(g_mu);
    Record r{name, flops, bytes, take(), take()};
    cudaEventRecord(r.start, reinterpret_cast<cudaStream_t>(current_stream()));
    g_records.push_back(std::move(r));
    slot_ = static_cast<int>(g_records.size()) - 1;
}

Scope::~Scope()
{
    if (name_ != nullptr)
    {
        const double now = std::chrono::duration<double, std::milli>(
                               std::chrono::steady_clock::now().time_since_epoch())
                               .count();
        std::lock_guard<std::mutex> lock(g_mu);
        auto& v = g_host.by_name[name_];
        v.first += now - host_start_;
        v.second += 1;
    }
    if (slot_ < 0)
    {
        return;
    }
    std::lock_guard<std::mutex> lock(g_mu);
    if (slot_ < static_cast<int>(g_records.size()))
    {
        cudaEventRecord(g_records[slot_].stop, reinterpret_cast<cudaStream_t>(current_stream()));
    }
}

namespace
{
double now_ms()
{
    return std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now().time_since_epoch())
        .count();
}
void add_host(const char* name, double ms)
{
    std::lock_guard<std::mutex> lock(g_mu);
    auto& v = g_host.by_name[name];
    v.first += ms;
    v.second += 1;
}
} // namespace

HostScope::HostScope(const char* name)
{
    if (g_host_enabled)
    {
        name_ = name;
        start_ = now_ms();
    }
}

HostScope::~HostScope()
{
    if (name_ != nullptr)
    {
        add_host(name_, now_ms() - start_);
    }
}

std::map<std::string, Totals> collect(bool reset)
{
    std::lock_guard<std::mutex> lock(g_mu);
    for (Record& r : g_records)
    {
        cudaEventSynchronize(r.stop);
        float ms = 0.0f;
        cudaEventElapsedTime(&ms, r.start, r.stop);
        Totals& t = g_totals[r.name];
        t.ms += ms;
        t.flops += r.flops;
        t.bytes += r.bytes;
        t.launches += 1;
        g_free.push_back(r.start);
        g_free.push_back(r.stop);
    }
    g_records.clear();
    std::map<std::string, Totals> out = g_totals;
    if (reset)
    {
        g_totals.clear();
    }
    return out;
}

} // namespace veda::profile
