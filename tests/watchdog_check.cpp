// Host-only check of the library's watchdog loop (csrc/watchdog.h) against fake
// stream and communicator probes: a stream that drains, a stream error, a
// communicator error while the stream waits, and a deadline.  Built and run by
// tests/test_failure_detection.py with g++; prints "ok" on success.
#include <chrono>
#include <cstdio>

#include "watchdog.h"

using namespace af2;

static int failures = 0;
#define EXPECT(cond)                                            \
  do {                                                          \
    if (!(cond)) {                                              \
      std::printf("FAILED line %d: %s\n", __LINE__, #cond);     \
      ++failures;                                               \
    }                                                           \
  } while (0)

int main() {
  // drains at once
  EXPECT(wait_with_watchdog([] { return StreamState::kDone; }, [] { return PeerState::kOk; }, 1.0) ==
         WaitOutcome::kDone);
  // drains after 2000 polls, including sleeping ones
  int polls = 0;
  EXPECT(wait_with_watchdog([&] { return ++polls > 2000 ? StreamState::kDone : StreamState::kPending; },
                            [] { return PeerState::kOk; }, 10.0, 20) == WaitOutcome::kDone);
  EXPECT(polls == 2001);
  // a stream error ends the wait
  EXPECT(wait_with_watchdog([] { return StreamState::kError; }, [] { return PeerState::kOk; }, 1.0) ==
         WaitOutcome::kStreamError);
  // the communicator reports an error while the stream still waits (a peer left)
  int peer_polls = 0;
  EXPECT(wait_with_watchdog([] { return StreamState::kPending; },
                            [&] { return ++peer_polls >= 300 ? PeerState::kError : PeerState::kOk; }, 0.0, 20) ==
         WaitOutcome::kPeerError);
  EXPECT(peer_polls == 300);
  // nothing ever finishes: the deadline ends the wait, close to it
  const auto t0 = std::chrono::steady_clock::now();
  EXPECT(wait_with_watchdog([] { return StreamState::kPending; }, [] { return PeerState::kOk; }, 0.05, 200) ==
         WaitOutcome::kTimeout);
  const double waited = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
  EXPECT(waited >= 0.05 && waited < 1.0);
  // a stream that drains in the same poll as a peer error counts as drained
  EXPECT(wait_with_watchdog([] { return StreamState::kDone; }, [] { return PeerState::kError; }, 1.0) ==
         WaitOutcome::kDone);
  if (failures == 0) std::printf("ok\n");
  return failures == 0 ? 0 : 1;
}
