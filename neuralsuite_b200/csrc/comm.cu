// NCCL (run-time loaded) communicator for the data-parallel step.
#include "comm.h"

#include <dlfcn.h>

#include <chrono>
#include <cstring>
#include <mutex>
#include <thread>

#include "common.cuh"

namespace nsb {
namespace comm {
namespace {

struct Api {
  bool ok = false;
  ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
  ncclResult_t (*CommInitRank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*AllReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                            cudaStream_t) = nullptr;
  ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t*) = nullptr;
  ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
  ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
  const char* (*GetErrorString)(ncclResult_t) = nullptr;
};

Api& api() {
  static Api a;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!h) return;
    a.GetUniqueId = reinterpret_cast<decltype(a.GetUniqueId)>(dlsym(h, "ncclGetUniqueId"));
    a.CommInitRank = reinterpret_cast<decltype(a.CommInitRank)>(dlsym(h, "ncclCommInitRank"));
    a.AllReduce = reinterpret_cast<decltype(a.AllReduce)>(dlsym(h, "ncclAllReduce"));
    a.CommGetAsyncError =
        reinterpret_cast<decltype(a.CommGetAsyncError)>(dlsym(h, "ncclCommGetAsyncError"));
    a.CommAbort = reinterpret_cast<decltype(a.CommAbort)>(dlsym(h, "ncclCommAbort"));
    a.CommDestroy = reinterpret_cast<decltype(a.CommDestroy)>(dlsym(h, "ncclCommDestroy"));
    a.GetErrorString = reinterpret_cast<decltype(a.GetErrorString)>(dlsym(h, "ncclGetErrorString"));
    a.ok = a.GetUniqueId && a.CommInitRank && a.AllReduce && a.CommGetAsyncError && a.CommAbort &&
           a.CommDestroy && a.GetErrorString;
  });
  return a;
}

ns_status nccl_fail(ncclResult_t r, const char* what) {
  const char* s = api().GetErrorString ? api().GetErrorString(r) : "?";
  return fail(NS_ERR_COMM, std::string(what) + ": " + s);
}

}  // namespace

ns_status allreduce(ns_comm* c, float* buf, int64_t count, cudaStream_t stream) {
  if (!c || c->aborted) return fail(NS_ERR_COMM, "allreduce on an aborted communicator");
  if (count <= 0) return NS_OK;
  ncclResult_t r = api().AllReduce(buf, buf, (size_t)count, ncclFloat32, ncclSum, c->comm, stream);
  if (r != ncclSuccess) return nccl_fail(r, "ncclAllReduce");
  return NS_OK;
}

ns_status check(ns_comm* c) {
  if (!c) return NS_OK;
  if (c->aborted) return fail(NS_ERR_COMM, "communicator aborted");
  ncclResult_t async = ncclSuccess;
  ncclResult_t r = api().CommGetAsyncError(c->comm, &async);
  if (r != ncclSuccess) return nccl_fail(r, "ncclCommGetAsyncError");
  if (async != ncclSuccess && async != ncclInProgress) return nccl_fail(async, "NCCL async error");
  return NS_OK;
}

ns_status wait_event(ns_comm* c, cudaEvent_t ev, double timeout_s) {
  const auto t0 = std::chrono::steady_clock::now();
  for (;;) {
    cudaError_t e = cudaEventQuery(ev);
    if (e == cudaSuccess) return NS_OK;
    if (e != cudaErrorNotReady) return cuda_fail(e, "waiting for the step");
    ns_status s = check(c);
    if (s != NS_OK) {
      if (c && !c->aborted) {
        api().CommAbort(c->comm);
        c->aborted = true;
      }
      return s;
    }
    const double dt = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
    if (dt > timeout_s) {
      if (c && !c->aborted) {
        api().CommAbort(c->comm);
        c->aborted = true;
      }
      return fail(NS_ERR_TIMEOUT, "step did not finish before the deadline; communicator aborted");
    }
    std::this_thread::sleep_for(std::chrono::microseconds(50));
  }
}

}  // namespace comm
}  // namespace nsb

using namespace nsb;

extern "C" {

ns_status ns_comm_unique_id(uint8_t host_id_out[128]) {
  if (!comm::api().ok) return fail(NS_ERR_UNSUPPORTED, "libnccl.so.2 could not be loaded");
  ncclUniqueId id;
  ncclResult_t r = comm::api().GetUniqueId(&id);
  if (r != ncclSuccess) return fail(NS_ERR_COMM, "ncclGetUniqueId failed");
  static_assert(sizeof(ncclUniqueId) == 128, "ncclUniqueId is 128 bytes");
  std::memcpy(host_id_out, &id, 128);
  return NS_OK;
}

ns_status ns_comm_init(const uint8_t host_id[128], int world_size, int rank, ns_comm** out) {
  NS_REQUIRE(out && host_id && world_size >= 1 && rank >= 0 && rank < world_size,
             "ns_comm_init: bad arguments");
  if (!comm::api().ok) return fail(NS_ERR_UNSUPPORTED, "libnccl.so.2 could not be loaded");
  ncclUniqueId id;
  std::memcpy(&id, host_id, 128);
  ns_comm* c = new ns_comm();
  c->world = world_size;
  c->rank = rank;
  ncclResult_t r = comm::api().CommInitRank(&c->comm, world_size, id, rank);
  if (r != ncclSuccess) {
    delete c;
    return fail(NS_ERR_COMM, "ncclCommInitRank failed");
  }
  *out = c;
  return NS_OK;
}

ns_status ns_comm_allreduce_sum(ns_comm* c, float* buf, int64_t count, void* stream) {
  return comm::allreduce(c, buf, count, as_stream(stream));
}

ns_status ns_comm_check(ns_comm* c) { return comm::check(c); }

ns_status ns_comm_abort(ns_comm* c) {
  if (!c) return NS_OK;
  if (!c->aborted && comm::api().ok) comm::api().CommAbort(c->comm);
  c->aborted = true;
  return NS_OK;
}

ns_status ns_comm_destroy(ns_comm* c) {
  if (!c) return NS_OK;
  if (!c->aborted && comm::api().ok) comm::api().CommDestroy(c->comm);
  delete c;
  return NS_OK;
}

}  // extern "C"
