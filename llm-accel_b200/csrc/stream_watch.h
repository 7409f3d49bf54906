// Host wait with a deadline for a stream that carries NCCL collectives.
//
// An NCCL kernel whose peer never enters the collective waits on the GPU with
// no limit of its own (the peer all-reduce kernels bound their own waits, NCCL's
// do not). A rank of a tensor-parallel group therefore does not block in
// cudaStreamSynchronize: it polls the stream, the communicator's asynchronous
// error and a deadline, and on an error or on expiry aborts the communicator,
// which ends its kernels. Header only, with the CUDA / NCCL calls passed in, so
// the loop itself runs on the host without a GPU.
#pragma once

#include <cstdint>
#include <thread>

namespace llmx {

enum WatchOutcome {
    kWatchDone = 0,         // every operation on the stream finished
    kWatchStreamError = 1,  // the stream reported a CUDA error (no abort)
    kWatchCommError = 2,    // the communicator reported an asynchronous error; aborted
    kWatchTimeout = 3,      // the deadline passed with work still pending; aborted
};

// query():      0 = the stream is idle, 1 = work pending, -1 = CUDA error
// comm_error(): true when the communicator holds an asynchronous error
// abort():      abort the communicator; called at most once, just before returning
// now_ms():     a monotonic clock in milliseconds
template <class Query, class CommError, class Abort, class Clock>
WatchOutcome watch_stream(Query query, CommError comm_error, Abort abort, Clock now_ms, double timeout_ms) {
    const double t0 = now_ms();
    for (uint64_t n = 0;; n++) {
        const int q = query();
        if (q == 0) return kWatchDone;
        if (q < 0) return kWatchStreamError;
        if (comm_error()) {
            abort();
            return kWatchCommError;
        }
        if (now_ms() - t0 > timeout_ms) {
            abort();
            return kWatchTimeout;
        }
        // spin for short waits (a decode step), then give the core away
        if (n >= 256) std::this_thread::yield();
    }
}

}  // namespace llmx
