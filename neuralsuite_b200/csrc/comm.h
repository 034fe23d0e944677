// NCCL communicator used by the data-parallel GPT step.  NCCL is resolved at
// run time with dlopen (preferring the copy already loaded in the process,
// e.g. PyTorch's), so the kernel library has no link-time NCCL dependency.
#pragma once

#include <cuda_runtime.h>
#include <nccl.h>

#include <string>

#include "ns_b200.h"

struct ns_comm {
  ncclComm_t comm = nullptr;
  int world = 1;
  int rank = 0;
  bool aborted = false;
};

namespace nsb {
namespace comm {

// Sum-allreduce of `count` floats in place on `stream`.
ns_status allreduce(ns_comm* c, float* buf, int64_t count, cudaStream_t stream);
// Non-blocking health poll.
ns_status check(ns_comm* c);
// Waits for `ev` with a host deadline, polling the communicator; aborts the
// communicator and returns NS_ERR_TIMEOUT when the deadline passes.
ns_status wait_event(ns_comm* c, cudaEvent_t ev, double timeout_s);

}  // namespace comm
}  // namespace nsb
