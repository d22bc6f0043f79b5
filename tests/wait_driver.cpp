// Drives alb::bounded_wait (arclight_b200/csrc/alb_wait.h) with fake stream and
// communicator probes; built and run by tests/test_wait_host.py.  Prints one
// line per case: name, result code (0 done, 1 stream error, 2 comm error,
// 3 timeout), polls, elapsed ms.
#include <chrono>
#include <cstdio>

#include "alb_wait.h"

static void run(const char * name, int done_at, int serr_at, int cerr_at, double timeout_ms) {
    int polls = 0;
    auto query = [&]() {
        ++polls;
        if (serr_at >= 0 && polls >= serr_at) return -1;
        if (done_at >= 0 && polls >= done_at) return 0;
        return 1;
    };
    auto comm = [&]() { return (cerr_at >= 0 && polls >= cerr_at) ? 1 : 0; };
    const auto t0 = std::chrono::steady_clock::now();
    const alb::WaitResult r = alb::bounded_wait(query, comm, timeout_ms);
    const double ms = std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
    std::printf("%s %d %d %.3f\n", name, (int)r, polls, ms);
}

int main() {
    run("done", 100, -1, -1, 10000.0);          // the stream finishes after 100 polls
    run("stream_error", -1, 10, -1, 10000.0);   // a failed kernel
    run("comm_error", -1, -1, 50, 10000.0);     // NCCL reports an asynchronous error
    run("timeout", -1, -1, -1, 50.0);           // a peer never answers
    run("done_first", 1, -1, 5, 10000.0);       // done wins over a later comm error
    return 0;
}
