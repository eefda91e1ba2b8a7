"""The bounded wait behind the library's NCCL handling (csrc/watchdog.h), driven by fakes on the
CPU: the engine polls ncclCommGetAsyncError / cudaStreamQuery through it and calls
ncclCommAbort when it gives up.  Here a fake state stands for a communicator that finishes, one
that reports an error, and one whose peer never answers."""
import os
import subprocess

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CSRC = os.path.join(ROOT, "audiocraft.cpp_b200", "csrc")

PROGRAM = r"""
#include <chrono>
#include <cstdio>
#include "watchdog.h"
using namespace act;
int main() {
    int aborts = 0, polls = 0;
    auto abort = [&] { ++aborts; };
    // 1: pending three times, then done (NCCL init that completes)
    auto r1 = bounded_wait([&] { return ++polls < 4 ? WaitState::Pending : WaitState::Done; }, abort, 1000);
    std::printf("done %d %d %d\n", (int)(r1 == WaitResult::Done), aborts, polls);
    // 2: an asynchronous error (ncclCommGetAsyncError != success / in progress)
    aborts = 0;
    auto r2 = bounded_wait([&] { return WaitState::Failed; }, abort, 1000);
    std::printf("failed %d %d\n", (int)(r2 == WaitResult::Failed), aborts);
    // 3: a peer that never answers: expires after the limit, aborts once
    aborts = 0;
    const auto t0 = std::chrono::steady_clock::now();
    auto r3 = bounded_wait([&] { return WaitState::Pending; }, abort, 50);
    const long ms = (long)std::chrono::duration_cast<std::chrono::milliseconds>(std::chrono::steady_clock::now() - t0).count();
    std::printf("timeout %d %d %ld\n", (int)(r3 == WaitResult::TimedOut), aborts, ms);
    return 0;
}
"""


def test_bounded_wait_with_fake_communicator(tmp_path):
    src = tmp_path / "wd.cpp"
    src.write_text(PROGRAM)
    exe = tmp_path / "wd"
    subprocess.run(["g++", "-std=c++17", "-O1", "-I" + CSRC, str(src), "-o", str(exe)], check=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True, check=True, timeout=30).stdout.split("\n")
    done, failed, timeout = (l.split() for l in out[:3])
    assert done == ["done", "1", "0", "4"]
    assert failed == ["failed", "1", "1"]
    assert timeout[:3] == ["timeout", "1", "1"] and 50 <= int(timeout[3]) < 2000
