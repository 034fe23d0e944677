// NCCL (run-time loaded) communicator for the data-parallel step, with host
// waits that always end: see comm.h.
#include "comm.h"

#include <dlfcn.h>

#include <chrono>
#include <climits>
#include <cstring>
#include <mutex>
#include <thread>

#include "common.cuh"

namespace nsb {
namespace comm {
namespace {

const Api& nccl() {
  static Api a;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!h) return;
    a.GetUniqueId = reinterpret_cast<decltype(a.GetUniqueId)>(dlsym(h, "ncclGetUniqueId"));
    a.CommInitRankConfig =
        reinterpret_cast<decltype(a.CommInitRankConfig)>(dlsym(h, "ncclCommInitRankConfig"));
    a.AllReduce = reinterpret_cast<decltype(a.AllReduce)>(dlsym(h, "ncclAllReduce"));
    a.CommGetAsyncError =
        reinterpret_cast<decltype(a.CommGetAsyncError)>(dlsym(h, "ncclCommGetAsyncError"));
    a.CommFinalize = reinterpret_cast<decltype(a.CommFinalize)>(dlsym(h, "ncclCommFinalize"));
    a.CommAbort = reinterpret_cast<decltype(a.CommAbort)>(dlsym(h, "ncclCommAbort"));
    a.CommDestroy = reinterpret_cast<decltype(a.CommDestroy)>(dlsym(h, "ncclCommDestroy"));
    a.GetErrorString = reinterpret_cast<decltype(a.GetErrorString)>(dlsym(h, "ncclGetErrorString"));
    a.ok = a.GetUniqueId && a.CommInitRankConfig && a.AllReduce && a.CommGetAsyncError &&
           a.CommAbort && a.CommDestroy && a.GetErrorString;
  });
  return a;
}

ns_status nccl_fail(const Api* api, ncclResult_t r, const char* what) {
  const char* s = api && api->GetErrorString ? api->GetErrorString(r) : "?";
  return fail(NS_ERR_COMM, std::string(what) + ": " + s);
}

void abort_comm(ns_comm* c) {
  if (c && !c->aborted) {
    c->api->CommAbort(c->comm);
    c->aborted = true;
  }
}

// Polls done() (1 = finished, 0 = not yet, -1 = failed with *err set) and the
// communicator's asynchronous error state until done, an error, or
// timeout_s.  On an error or the deadline the communicator is aborted.
template <typename Done>
ns_status poll_until(ns_comm* c, Done&& done, double timeout_s, const char* what) {
  const auto t0 = std::chrono::steady_clock::now();
  for (;;) {
    ns_status err = NS_OK;
    const int d = done(&err);
    if (d > 0) return NS_OK;
    if (d < 0) {
      abort_comm(c);
      return err;
    }
    ns_status s = check(c);
    if (s != NS_OK) {
      abort_comm(c);
      return s;
    }
    const double dt = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
    if (dt > timeout_s) {
      abort_comm(c);
      return fail(NS_ERR_TIMEOUT, std::string(what) +
                                      " did not finish before the deadline; communicator aborted");
    }
    std::this_thread::sleep_for(std::chrono::microseconds(50));
  }
}

// done() of a non-blocking NCCL call: finished once the communicator's
// asynchronous state leaves ncclInProgress.
int nccl_settled(ns_comm* c, ns_status* err) {
  ncclResult_t async = ncclSuccess;
  ncclResult_t r = c->api->CommGetAsyncError(c->comm, &async);
  if (r != ncclSuccess) {
    *err = nccl_fail(c->api, r, "ncclCommGetAsyncError");
    return -1;
  }
  if (async == ncclInProgress) return 0;
  if (async != ncclSuccess) {
    *err = nccl_fail(c->api, async, "NCCL async error");
    return -1;
  }
  return 1;
}

// Creates c->comm non-blocking and waits (bounded) for it to be ready.
ns_status init_comm(ns_comm* c, const ncclUniqueId& id) {
  ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
  cfg.blocking = 0;
  ncclResult_t r = c->api->CommInitRankConfig(&c->comm, c->world, id, c->rank, &cfg);
  if (r != ncclSuccess && r != ncclInProgress) {
    if (c->comm) abort_comm(c);
    return nccl_fail(c->api, r, "ncclCommInitRankConfig");
  }
  return poll_until(c, [&](ns_status* err) { return nccl_settled(c, err); }, c->timeout_s,
                    "NCCL communicator creation");
}

}  // namespace

ns_status allreduce(ns_comm* c, float* buf, int64_t count, cudaStream_t stream) {
  if (!c || c->aborted) return fail(NS_ERR_COMM, "allreduce on an aborted communicator");
  if (count <= 0) return NS_OK;
  ncclResult_t r =
      c->api->AllReduce(buf, buf, (size_t)count, ncclFloat32, ncclSum, c->comm, stream);
  if (r == ncclInProgress)  // a non-blocking communicator still enqueueing
    return poll_until(c, [&](ns_status* err) { return nccl_settled(c, err); }, c->timeout_s,
                      "ncclAllReduce enqueue");
  if (r != ncclSuccess) return nccl_fail(c->api, r, "ncclAllReduce");
  return NS_OK;
}

ns_status check(ns_comm* c) {
  if (!c) return NS_OK;
  if (c->aborted) return fail(NS_ERR_COMM, "communicator aborted");
  ncclResult_t async = ncclSuccess;
  ncclResult_t r = c->api->CommGetAsyncError(c->comm, &async);
  if (r != ncclSuccess) return nccl_fail(c->api, r, "ncclCommGetAsyncError");
  if (async != ncclSuccess && async != ncclInProgress) return nccl_fail(c->api, async, "NCCL async error");
  return NS_OK;
}

ns_status wait_event(ns_comm* c, cudaEvent_t ev, double timeout_s) {
  return poll_until(
      c,
      [&](ns_status* err) {
        cudaError_t e = cudaEventQuery(ev);
        if (e == cudaSuccess) return 1;
        if (e == cudaErrorNotReady) return 0;
        *err = cuda_fail(e, "waiting for the step");
        return -1;
      },
      timeout_s, "the step");
}

// ------------------------------------------------------------ self-test fake
//
// A fake NCCL for ns_comm_selftest: no GPU, no library.  Its communicator
// handle is a dummy; the scenario decides what the asynchronous state reports.
namespace fake {

int g_scenario = 0;
int g_polls = 0;
int g_aborts = 0;

ncclComm_t handle() { return reinterpret_cast<ncclComm_t>(static_cast<uintptr_t>(0x1000)); }

ncclResult_t get_unique_id(ncclUniqueId* id) {
  std::memset(id, 0, sizeof(*id));
  return ncclSuccess;
}
ncclResult_t init(ncclComm_t* comm, int, ncclUniqueId, int, ncclConfig_t* cfg) {
  *comm = handle();
  return cfg && cfg->blocking == 0 ? ncclInProgress : ncclSuccess;
}
ncclResult_t all_reduce(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                        cudaStream_t) {
  return ncclSuccess;
}
ncclResult_t get_async_error(ncclComm_t, ncclResult_t* async) {
  ++g_polls;
  switch (g_scenario) {
    case 2: *async = g_polls > 2 ? ncclRemoteError : ncclSuccess; break;  // a peer failed
    case 3: *async = ncclInProgress; break;                                // creation never ends
    case 4: *async = g_polls > 3 ? ncclSuccess : ncclInProgress; break;    // creation ends
    default: *async = ncclSuccess;
  }
  return ncclSuccess;
}
ncclResult_t finalize(ncclComm_t) { return ncclSuccess; }
ncclResult_t comm_abort(ncclComm_t) {
  ++g_aborts;
  return ncclSuccess;
}
ncclResult_t destroy(ncclComm_t) { return ncclSuccess; }
const char* error_string(ncclResult_t r) { return r == ncclRemoteError ? "remote error (fake)" : "fake"; }

const Api& api() {
  static Api a = [] {
    Api f;
    f.ok = true;
    f.GetUniqueId = get_unique_id;
    f.CommInitRankConfig = init;
    f.AllReduce = all_reduce;
    f.CommGetAsyncError = get_async_error;
    f.CommFinalize = finalize;
    f.CommAbort = comm_abort;
    f.CommDestroy = destroy;
    f.GetErrorString = error_string;
    return f;
  }();
  return a;
}

}  // namespace fake

}  // namespace comm
}  // namespace nsb

using namespace nsb;

extern "C" {

ns_status ns_comm_unique_id(uint8_t host_id_out[128]) {
  NS_REQUIRE(host_id_out, "ns_comm_unique_id: NULL argument");
  const comm::Api& a = comm::nccl();
  if (!a.ok) return fail(NS_ERR_UNSUPPORTED, "libnccl.so.2 could not be loaded");
  ncclUniqueId id;
  ncclResult_t r = a.GetUniqueId(&id);
  if (r != ncclSuccess) return fail(NS_ERR_COMM, "ncclGetUniqueId failed");
  static_assert(sizeof(ncclUniqueId) == 128, "ncclUniqueId is 128 bytes");
  std::memcpy(host_id_out, &id, 128);
  return NS_OK;
}

ns_status ns_comm_init(const uint8_t host_id[128], int world_size, int rank, ns_comm** out) {
  NS_REQUIRE(out && host_id && world_size >= 1 && rank >= 0 && rank < world_size,
             "ns_comm_init: bad arguments");
  const comm::Api& a = comm::nccl();
  if (!a.ok) return fail(NS_ERR_UNSUPPORTED, "libnccl.so.2 could not be loaded");
  ncclUniqueId id;
  std::memcpy(&id, host_id, 128);
  ns_comm* c = new ns_comm();
  c->world = world_size;
  c->rank = rank;
  c->api = &a;
  ns_status rc = comm::init_comm(c, id);
  if (rc != NS_OK) {
    delete c;
    return rc;
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
  comm::abort_comm(c);
  return NS_OK;
}

ns_status ns_comm_destroy(ns_comm* c) {
  if (!c) return NS_OK;
  ns_status rc = NS_OK;
  if (!c->aborted) {
    // A non-blocking communicator is finalised (bounded) before it is destroyed.
    if (c->api->CommFinalize) {
      ncclResult_t r = c->api->CommFinalize(c->comm);
      if (r == ncclInProgress)
        rc = comm::poll_until(c, [&](ns_status* err) { return comm::nccl_settled(c, err); },
                              c->timeout_s, "NCCL communicator finalisation");
      else if (r != ncclSuccess)
        comm::abort_comm(c);
    }
    if (!c->aborted) c->api->CommDestroy(c->comm);
  }
  delete c;
  return rc;
}

ns_status ns_comm_selftest(int scenario, double timeout_s, int* aborts) {
  NS_REQUIRE(scenario >= 0 && scenario <= 4, "ns_comm_selftest: scenario must be 0..4");
  comm::fake::g_scenario = scenario;
  comm::fake::g_polls = 0;
  comm::fake::g_aborts = 0;
  ns_comm c;
  c.api = &comm::fake::api();
  c.timeout_s = timeout_s;
  ns_status rc;
  if (scenario >= 3) {
    ncclUniqueId id;
    comm::fake::get_unique_id(&id);
    rc = comm::init_comm(&c, id);
  } else {
    c.comm = comm::fake::handle();
    int polls = 0;
    rc = comm::poll_until(
        &c,
        [&](ns_status*) { return scenario == 0 && ++polls >= 3 ? 1 : 0; },  // 1: never done
        timeout_s, "the fake step");
  }
  if (aborts) *aborts = comm::fake::g_aborts;
  return rc;
}

}  // extern "C"
