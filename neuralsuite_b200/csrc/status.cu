// Status plumbing of the C ABI: thread-local last error, device queries.
#include <atomic>
#include <cstdio>
#include <mutex>
#include <string>

#include "common.cuh"

namespace nsb {

namespace {
thread_local std::string t_last_error;
}

namespace {
std::atomic<long long> g_launches{0};
}

void count_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

void set_error(const std::string& msg) { t_last_error = msg; }

ns_status fail(ns_status code, const std::string& msg) {
  t_last_error = msg;
  return code;
}

ns_status cuda_fail(cudaError_t err, const char* what) {
  t_last_error = std::string(what) + ": " + cudaGetErrorName(err) + " (" +
                 cudaGetErrorString(err) + ")";
  return NS_ERR_CUDA;
}

int sm_count() {
  static int cached[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (cached[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      n = 148;
    cached[dev] = n;
  }
  return cached[dev];
}

}  // namespace nsb

extern "C" {

const char* ns_last_error(void) { return nsb::t_last_error.c_str(); }

int ns_version(void) { return 1; }

long long ns_launch_count(void) { return nsb::g_launches.load(std::memory_order_relaxed); }

int ns_device_supported(void) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  int major = 0, minor = 0;
  if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess)
    return 0;
  if (cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev) != cudaSuccess)
    return 0;
  return (major == 10 && minor == 0) ? 1 : 0;
}

}  // extern "C"
