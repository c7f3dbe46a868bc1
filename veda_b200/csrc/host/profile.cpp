// Per-kernel-class CUDA-event timers (see include/veda/profile.hpp).
#include "veda/profile.hpp"

#include "veda/tensor.hpp"

#include <cuda_runtime.h>

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
