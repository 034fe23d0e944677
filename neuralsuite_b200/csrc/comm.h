// NCCL communicator used by the data-parallel GPT step.  NCCL is resolved at
// run time with dlopen (preferring the copy already loaded in the process,
// e.g. PyTorch's), so the kernel library has no link-time NCCL dependency.
//
// Every host wait on the communicator is a poll with a deadline: creation
// (the communicator is created non-blocking), collectives NCCL reports as
// still being enqueued, and the end-of-step event.  On a deadline or an
// asynchronous NCCL error the communicator is aborted and the call returns
// NS_ERR_TIMEOUT / NS_ERR_COMM, so a rank that died never leaves the others
// blocked inside NCCL.
#pragma once

#include <cuda_runtime.h>
#include <nccl.h>

#include <string>

#include "ns_b200.h"

namespace nsb {
namespace comm {

// The NCCL entry points a communicator calls: the run-time loaded library,
// or a fake one in the host-side self-test (ns_comm_selftest).
struct Api {
  bool ok = false;
  ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
  ncclResult_t (*CommInitRankConfig)(ncclComm_t*, int, ncclUniqueId, int, ncclConfig_t*) = nullptr;
  ncclResult_t (*AllReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                            cudaStream_t) = nullptr;
  ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t*) = nullptr;
  ncclResult_t (*CommFinalize)(ncclComm_t) = nullptr;
  ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
  ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
  const char* (*GetErrorString)(ncclResult_t) = nullptr;
};

}  // namespace comm
}  // namespace nsb

struct ns_comm {
  ncclComm_t comm = nullptr;
  int world = 1;
  int rank = 0;
  bool aborted = false;
  const nsb::comm::Api* api = nullptr;
  double timeout_s = 300.0;  // deadline of creation and of a collective's enqueue
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
