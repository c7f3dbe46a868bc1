// Host-side wait on work that may include collectives with other processes.
//
// A blocking wait (cudaStreamSynchronize) on a stream whose NCCL collective waits for a peer that
// has failed never returns. watch() polls instead: the stream (done / pending / failed) and the
// communicator's asynchronous error state (ncclCommGetAsyncError), pausing between polls, and
// calls abort (ncclCommAbort, which makes NCCL's kernels give up so the stream drains) when the
// communicator reports an error or when nothing completes within the timeout. The poll, abort,
// clock and pause functions are parameters so the logic runs against fakes without a GPU.
#pragma once

#include <chrono>
#include <string>
#include <thread>

namespace veda::train::detail
{

enum class WaitOutcome
{
    done,           // the stream completed
    stream_error,   // the stream reported a CUDA error
    comm_error,     // the communicator reported an asynchronous error; it has been aborted
    timeout         // nothing completed within the timeout; the communicator has been aborted
};

// stream_poll() -> 0 done, 1 still running, -1 failed.
// comm_poll()   -> 0 no error, 1 an operation still in progress (non-blocking communicator),
//                  -1 an asynchronous error.
// abort()       -> aborts the communicator (called at most once).
// now()         -> seconds on a monotonic clock; pause() waits a little before the next poll.
template <class StreamPoll, class CommPoll, class Abort, class Now, class Pause>
WaitOutcome watch(StreamPoll stream_poll, CommPoll comm_poll, Abort abort, Now now, Pause pause,
                  double timeout_s)
{
    const double start = now();
    for (;;)
    {
        const int s = stream_poll();
        if (s == 0)
        {
            return WaitOutcome::done;
        }
        if (s < 0)
        {
            return WaitOutcome::stream_error;
        }
        if (comm_poll() < 0)
        {
            abort();
            return WaitOutcome::comm_error;
        }
        if (now() - start > timeout_s)
        {
            abort();
            return WaitOutcome::timeout;
        }
        pause();
    }
}

inline double monotonic_seconds()
{
    return std::chrono::duration<double>(std::chrono::steady_clock::now().time_since_epoch()).count();
}

inline void short_pause()
{
    std::this_thread::sleep_for(std::chrono::microseconds(50));
}

inline const char* describe(WaitOutcome o)
{
    switch (o)
    {
    case WaitOutcome::done: return "completed";
    case WaitOutcome::stream_error: return "the stream reported a CUDA error";
    case WaitOutcome::comm_error:
        return "the communicator reported an asynchronous error (a peer failed); it was aborted";
    case WaitOutcome::timeout:
        return "no progress within the communication timeout (a peer may have failed); the "
               "communicator was aborted";
    }
    return "unknown";
}

} // namespace veda::train::detail
