// watchdog.h -- bounded host-side waits for work that another party (a peer rank, the device)
// has to finish.  Pure C++: the engine plugs in NCCL and CUDA queries; the tests plug in fakes.
//
// A wait polls `state()` until it reports Done.  It gives up, calls `abort()` once and returns
// the reason when the state reports Failed, or when `timeout_ms` (> 0) passes first.  The
// engine uses it for NCCL's non-blocking communicator (ncclCommInitRankConfig with
// blocking = 0, then ncclCommGetAsyncError until ncclSuccess) and for stream synchronisation
// while a communicator is live: a rank that died or stalled ends in ncclCommAbort and an error
// status instead of a host thread blocked forever.
#pragma once

#include <chrono>
#include <cstdint>
#include <functional>
#include <thread>

namespace act {

enum class WaitState { Pending, Done, Failed };
enum class WaitResult { Done, Failed, TimedOut };

inline WaitResult bounded_wait(const std::function<WaitState()>& state, const std::function<void()>& abort,
                               int64_t timeout_ms, int64_t poll_us = 50) {
    const auto t0 = std::chrono::steady_clock::now();
    for (;;) {
        const WaitState s = state();
        if (s == WaitState::Done) return WaitResult::Done;
        if (s == WaitState::Failed) {
            if (abort) abort();
            return WaitResult::Failed;
        }
        if (timeout_ms > 0) {
            const auto ms =
                std::chrono::duration_cast<std::chrono::milliseconds>(std::chrono::steady_clock::now() - t0).count();
            if (ms >= timeout_ms) {
                if (abort) abort();
                return WaitResult::TimedOut;
            }
        }
        std::this_thread::sleep_for(std::chrono::microseconds(poll_us));
    }
}

}  // namespace act
