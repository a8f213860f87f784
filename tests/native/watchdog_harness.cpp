// CPU check of kl::bounded_wait (klearu_b200/csrc/watchdog.h) against fake
// streams, a fake communicator and a fake clock.  Prints one line per case:
//   <case> <result> <aborts> <drained>
// tests/test_failure_detection.py compiles and runs it.
#include <cstdio>

#include "watchdog.h"

struct Fake {
  double t = 0;             // fake clock, ms
  int polls = 0;            // ready() calls
  int ready_at = -1;        // ready() turns true from this poll on (-1: never)
  int ready_after_abort = 0;  // 1: ready() is true once aborted
  int err_at = -1;          // async_error() reports 5 from this poll on
  int aborts = 0;
};

static void run(const char* name, Fake f, double timeout_ms) {
  int errpolls = 0;
  const kl::WaitReport r = kl::bounded_wait(
      [&] {
        ++f.polls;
        if (f.aborts && f.ready_after_abort) return true;
        return f.ready_at >= 0 && f.polls >= f.ready_at;
      },
      [&] { return (f.err_at >= 0 && ++errpolls >= f.err_at) ? 5 : 0; }, [&] { ++f.aborts; },
      [&] { return f.t; }, [&](double ms) { f.t += ms; }, timeout_ms, timeout_ms);
  std::printf("%s %d %d %d %d\n", name, (int)r.result, f.aborts, (int)r.drained, r.comm_error);
}

int main() {
  Fake a; a.ready_at = 5;
  run("done", a, 100.0);
  Fake b; b.err_at = 3; b.ready_after_abort = 1;
  run("comm_error", b, 100.0);
  Fake c; c.ready_after_abort = 1;
  run("timeout", c, 10.0);
  Fake d;
  run("stuck", d, 10.0);
  Fake e; e.ready_at = 1; e.err_at = 1;
  run("error_first", e, 10.0);
  return 0;
}
