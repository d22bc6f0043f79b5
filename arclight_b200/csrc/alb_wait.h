// Bounded host wait for a stream whose work includes collectives.
//
// The reference's ranks wait on each other in spin barriers with no way out
// (thread.cpp:239-268; errors abort the process, nnml.h:97-111).  Here a rank
// whose peer died would otherwise block in cudaStreamSynchronize forever, its
// NCCL kernels spinning on the peer.  bounded_wait polls the stream and the
// communicator's asynchronous error instead and gives up after timeout_ms; on
// kCommError or kTimeout the caller aborts the communicator (ncclCommAbort),
// which makes the spinning collective kernels return, and reports the error.
//
// Host code only, templated on its probes so the policy is tested on the CPU
// with fakes:
//   query()    -> 0 when the stream's work is done, 1 while it runs, < 0 on a
//                 stream error;
//   comm_err() -> 0, or non-zero once the communicator reports an error.
#pragma once

#include <chrono>
#include <thread>

namespace alb {

enum class WaitResult { kDone = 0, kStreamError = 1, kCommError = 2, kTimeout = 3 };

template <class Query, class CommErr>
WaitResult bounded_wait(Query query, CommErr comm_err, double timeout_ms) {
    using clk = std::chrono::steady_clock;
    const auto t0 = clk::now();
    while (true) {
        const int q = query();
        if (q == 0) return WaitResult::kDone;
        if (q < 0) return WaitResult::kStreamError;
        if (comm_err() != 0) return WaitResult::kCommError;
        const double ms = std::chrono::duration<double, std::milli>(clk::now() - t0).count();
        if (ms > timeout_ms) return WaitResult::kTimeout;
        // a step ends within milliseconds: poll at full rate (yielding) for the
        // first 50 ms so the step's latency is not stretched, then nap
        if (ms < 50.0) {
            std::this_thread::yield();
        } else {
            std::this_thread::sleep_for(std::chrono::microseconds(20));
        }
    }
}

}  // namespace alb
