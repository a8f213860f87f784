// Bounded waits for work that depends on other ranks (host code only).
//
// A sharded network's collectives finish only when every rank reaches them.  A
// rank that died, hung or left the step between calls leaves the survivors'
// NCCL kernels waiting for data that never comes, and a plain
// cudaStreamSynchronize would then block forever.  bounded_wait instead polls
// two things until a deadline:
//   * ready():      the rank's streams have drained (cudaStreamQuery),
//   * async_error(): the communicator's asynchronous error
//                    (ncclCommGetAsyncError: a peer's connection dropped, a
//                    remote error, ...), non-zero = failed.
// On an error or at the deadline it calls abort() exactly once
// (ncclCommAbort, which makes the waiting NCCL kernels return) and then waits
// up to `drain_ms` more for the streams to drain, so that the context stays
// usable when the abort released them.
//
// The poll functions are template parameters so that the same loop runs
// against the CUDA/NCCL calls in the library and against fakes in the CPU
// tests.  Nothing here touches a device.
#pragma once

#include <chrono>
#include <thread>

namespace kl {

enum class WaitResult : int {
  kDone = 0,         // the streams drained with no communicator error
  kCommError = 1,    // the communicator reported an error; it was aborted
  kTimeout = 2,      // the deadline passed; the communicator was aborted
};

struct WaitReport {
  WaitResult result = WaitResult::kDone;
  bool drained = true;   // the streams drained (after the abort, for errors)
  int polls = 0;         // poll rounds, for the tests
  int comm_error = 0;    // the communicator's error code, if any
};

inline double wall_ms() {
  using namespace std::chrono;
  return duration<double, std::milli>(steady_clock::now().time_since_epoch()).count();
}

// ready() -> bool, async_error() -> int (0 = fine), abort() -> void,
// now() -> double (ms), sleep(double ms) -> void.
template <class Ready, class AsyncError, class Abort, class Now, class Sleep>
WaitReport bounded_wait(Ready ready, AsyncError async_error, Abort abort, Now now, Sleep sleep, double timeout_ms,
                        double drain_ms, double poll_ms = 0.05) {
  WaitReport rep;
  const double t0 = now();
  double nap = poll_ms;
  for (;;) {
    ++rep.polls;
    const int e = async_error();
    if (e != 0) {
      rep.result = WaitResult::kCommError;
      rep.comm_error = e;
      break;
    }
    if (ready()) return rep;
    if (now() - t0 >= timeout_ms) {
      rep.result = WaitResult::kTimeout;
      break;
    }
    sleep(nap);
    if (nap < 1.0) nap *= 2.0;  // back off to 1 ms polls: steps are sub-ms, hangs are long
  }
  abort();
  const double t1 = now();
  rep.drained = false;
  while (now() - t1 < drain_ms) {
    if (ready()) {
      rep.drained = true;
      break;
    }
    sleep(1.0);
  }
  return rep;
}

inline void sleep_ms(double ms) {
  std::this_thread::sleep_for(std::chrono::duration<double, std::milli>(ms));
}

}  // namespace kl
