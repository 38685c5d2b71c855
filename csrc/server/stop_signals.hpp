// SIGINT / SIGTERM as a synchronous event for the servers' main functions.
//
// The constructor blocks both signals in the calling thread; every thread started afterwards (HTTP
// threads, the CUDA runtime's own threads) inherits the mask, so the signals stay pending until
// wait() takes them with sigtimedwait. No asynchronous handler runs, so nothing is shared with
// signal context (ThreadSanitizer reports a handler that writes a flag another thread reads).
// Construct it first thing in main(), before any thread exists.
#pragma once
#include <pthread.h>
#include <signal.h>
#include <time.h>

namespace vmc {

class StopSignals {
 public:
  StopSignals() {
    sigemptyset(&set_);
    sigaddset(&set_, SIGINT);
    sigaddset(&set_, SIGTERM);
    pthread_sigmask(SIG_BLOCK, &set_, nullptr);
  }
  // True once SIGINT or SIGTERM arrived (waits at most timeout_ms).
  bool wait(int timeout_ms) {
    timespec ts{timeout_ms / 1000, (timeout_ms % 1000) * 1000000L};
    return sigtimedwait(&set_, nullptr, &ts) > 0;
  }

 private:
  sigset_t set_;
};

}  // namespace vmc
