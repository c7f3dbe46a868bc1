// veda::profile — per-kernel-class device timers. The reference's profiler (src/libs/profile/
// Profile.h:50-73) is an RAII wall-clock scope that is off by default; this one records a CUDA
// event pair on the current stream around each region while enabled, so device time (not host
// time) is what gets summed, and nothing is synchronised until collect(). With
// VEDA_HOST_PROFILE=1 each scope also sums its host wall-clock time (printed at exit).
#pragma once

#include <cstdint>
#include <map>
#include <string>

namespace veda::profile
{

struct Totals
{
    double ms = 0.0;        // summed device time
    double flops = 0.0;     // summed algorithmic FLOPs
    double bytes = 0.0;     // summed algorithmic bytes
    uint64_t launches = 0;
};

void enable(bool on);
bool enabled();
// Synchronises on the recorded events and returns the per-class totals; reset clears them.
std::map<std::string, Totals> collect(bool reset = true);

class Scope
{
public:
    Scope(const char* name, double flops, double bytes);
    ~Scope();
    Scope(const Scope&) = delete;
    Scope& operator=(const Scope&) = delete;

private:
    int slot_ = -1;
    const char* name_ = nullptr;   // set when host timing is on (VEDA_HOST_PROFILE=1)
    double host_start_ = 0.0;
};

// Host wall-clock time of a region (no device events), summed per name when VEDA_HOST_PROFILE=1.
class HostScope
{
public:
    explicit HostScope(const char* name);
    ~HostScope();
    HostScope(const HostScope&) = delete;
    HostScope& operator=(const HostScope&) = delete;

private:
    const char* name_ = nullptr;
    double start_ = 0.0;
};

} // namespace veda::profile
