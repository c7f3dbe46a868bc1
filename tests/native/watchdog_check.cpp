// Drives the data-parallel watchdog (veda_b200/csrc/host/watchdog.hpp) with fake stream and
// communicator polls and a fake clock: no GPU, no NCCL. Prints one line per scenario.
#include "watchdog.hpp"

#include <cstdio>

using veda::train::detail::WaitOutcome;
using veda::train::detail::watch;

namespace
{
struct Fake
{
    int stream_done_after = -1;   // polls until the stream completes (-1: never)
    int stream_error_at = -1;     // poll at which the stream reports an error
    int comm_error_at = -1;       // poll at which the communicator reports an error
    int polls = 0, aborts = 0;
    double clock = 0.0;
};

const char* name(WaitOutcome o)
{
    switch (o)
    {
    case WaitOutcome::done: return "done";
    case WaitOutcome::stream_error: return "stream_error";
    case WaitOutcome::comm_error: return "comm_error";
    case WaitOutcome::timeout: return "timeout";
    }
    return "?";
}

void run(const char* label, Fake f, double timeout)
{
    const WaitOutcome o = watch(
        [&] {
            ++f.polls;
            if (f.stream_error_at >= 0 && f.polls >= f.stream_error_at) return -1;
            if (f.stream_done_after >= 0 && f.polls >= f.stream_done_after) return 0;
            return 1;
        },
        [&] { return (f.comm_error_at >= 0 && f.polls >= f.comm_error_at) ? -1 : 1; },
        [&] { ++f.aborts; }, [&] { return f.clock; }, [&] { f.clock += 0.25; }, timeout);
    std::printf("%s %s polls=%d aborts=%d\n", label, name(o), f.polls, f.aborts);
}
} // namespace

int main()
{
    Fake a;
    a.stream_done_after = 5;
    run("completes", a, 10.0);
    Fake b;
    b.comm_error_at = 3;
    run("peer_error", b, 10.0);
    Fake c;
    run("no_progress", c, 2.0);
    Fake d;
    d.stream_error_at = 2;
    run("stream_fault", d, 10.0);
    return 0;
}
