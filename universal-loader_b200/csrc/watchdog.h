/*
 * watchdog.h — bounded host-side wait for a stream that may hold collectives.
 *
 * A tensor-parallel forward enqueues NCCL all-reduces on the context stream; if a peer rank
 * is gone, the collective never completes and a plain cudaStreamSynchronize would block the
 * survivor forever.  bounded_wait polls instead: it returns once the stream's work is done,
 * and gives up at a deadline (or at the first asynchronous communicator error), calling the
 * abort hook exactly once first so the device-side collective stops waiting (ncclCommAbort
 * in the library).  The reference has no multi-GPU data path to guard; its only failure
 * handling is an init-time CPU fallback (src/inference/inference_engine.cpp:128-143).
 *
 * Host-only and free of CUDA / NCCL types: the hooks are passed in, so the logic is unit
 * tested on the CPU with fakes (tests/test_watchdog_cpu.py).
 */
#pragma once

#include <chrono>
#include <thread>

#include "../../include/ulb.h"

namespace ulb {

enum class Poll { kDone, kPending, kError };

/*
 *   query()       Poll::kDone / kPending / kError (the stream's state)
 *   comm_error()  true once the communicator reports an asynchronous error
 *   abort()       called once on a timeout or a communicator error
 *   timeout_s     > 0; the wait gives up this long after it starts
 * Returns ULB_OK, ULB_ECUDA (query error; no abort), ULB_ENCCL (communicator error, aborted)
 * or ULB_ETIMEOUT (deadline, aborted).  Polls every `poll_us` microseconds.
 */
template <class Query, class CommError, class Abort>
int bounded_wait(Query query, CommError comm_error, Abort abort, double timeout_s, int poll_us = 50) {
  using clk = std::chrono::steady_clock;
  const auto deadline = clk::now() + std::chrono::duration_cast<clk::duration>(std::chrono::duration<double>(timeout_s));
  for (;;) {
    const Poll p = query();
    if (p == Poll::kDone) return ULB_OK;
    if (p == Poll::kError) return ULB_ECUDA;
    if (comm_error()) {
      abort();
      return ULB_ENCCL;
    }
    if (clk::now() >= deadline) {
      abort();
      return ULB_ETIMEOUT;
    }
    std::this_thread::sleep_for(std::chrono::microseconds(poll_us));
  }
}

}  // namespace ulb
