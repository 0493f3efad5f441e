// watchdog.h -- host-side failure detection for work that waits on NCCL peers.
//
// A collective whose peer has died or left never completes: its kernel keeps
// waiting on the device and a plain cudaStreamSynchronize would block the
// host for good.  Every host wait on a stream that may hold collectives goes
// through wait_with_watchdog instead.  It polls the stream and the
// communicator's asynchronous error state until the stream drains, the
// communicator reports an error, or a deadline passes; in the last two cases
// the caller aborts the communicator (which ends its kernels, so the stream
// drains and the context stays usable) and returns AF2_ERR_NCCL.  No device
// code is involved and nothing here faults a GPU.
//
// Plain C++ on purpose: the loop takes its three probes as callables, so the
// same code runs against fakes in a host-only unit test.
#pragma once

#include <chrono>
#include <thread>

namespace af2 {

enum class StreamState { kDone, kPending, kError };  // cudaStreamQuery: success / not ready / error
enum class PeerState { kOk, kError };                // ncclCommGetAsyncError: success or in progress / error

enum class WaitOutcome {
  kDone,         // the stream drained
  kStreamError,  // the stream reported a CUDA error
  kPeerError,    // the communicator reported an asynchronous error (a peer failed or left)
  kTimeout       // neither before the deadline
};

// Polls `stream_state()` and `peer_state()` until one of the outcomes above.
// The first polls spin (a healthy step finishes within microseconds of the
// host reaching the wait); later ones sleep up to `max_sleep_us` between polls.
// timeout_s <= 0 waits without a deadline (the communicator's errors still end the wait).
template <class StreamProbe, class PeerProbe, class Clock = std::chrono::steady_clock>
WaitOutcome wait_with_watchdog(StreamProbe stream_state, PeerProbe peer_state, double timeout_s,
                               int max_sleep_us = 1000) {
  const auto start = Clock::now();
  int sleep_us = 0;
  for (int poll = 0;; ++poll) {
    switch (stream_state()) {
      case StreamState::kDone: return WaitOutcome::kDone;
      case StreamState::kError: return WaitOutcome::kStreamError;
      case StreamState::kPending: break;
    }
    if (peer_state() == PeerState::kError) return WaitOutcome::kPeerError;
    if (timeout_s > 0 && std::chrono::duration<double>(Clock::now() - start).count() > timeout_s)
      return WaitOutcome::kTimeout;
    if (poll < 64) continue;
    sleep_us = sleep_us < max_sleep_us ? sleep_us + 10 : max_sleep_us;
    std::this_thread::sleep_for(std::chrono::microseconds(sleep_us));
  }
}

inline const char *wait_outcome_text(WaitOutcome w) {
  switch (w) {
    case WaitOutcome::kDone: return "done";
    case WaitOutcome::kStreamError: return "the stream reported an error";
    case WaitOutcome::kPeerError: return "the communicator reported an asynchronous error (a rank failed or left)";
    case WaitOutcome::kTimeout: return "the communicator's work did not finish before the deadline";
  }
  return "unknown";
}

}  // namespace af2
