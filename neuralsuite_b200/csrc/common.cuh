// Shared helpers for the sm_100a kernels and the C ABI: status plumbing,
// launch checks and small device utilities.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "ns_b200.h"

namespace nsb {

// Thread-local last-error string behind ns_last_error().
void set_error(const std::string& msg);
ns_status fail(ns_status code, const std::string& msg);
ns_status cuda_fail(cudaError_t err, const char* what);

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

// Kernels launched by this library in this process (host-side count).
void count_launch();

// Checks (and counts) the launch that was just issued.
inline ns_status check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, what);
  count_launch();
  return NS_OK;
}

inline int ceil_div(int a, int b) { return (a + b - 1) / b; }
inline int64_t ceil_div64(int64_t a, int64_t b) { return (a + b - 1) / b; }

int sm_count();  // multiprocessors of the current device (cached per device)

// Programmatic dependent launch: a kernel launched by launch_pdl may be
// scheduled while the kernel before it in the stream is still running, so it
// must call pdl_wait() before it reads anything an earlier kernel wrote (the
// wait returns once those kernels have finished and their writes are
// visible); pdl_trigger() then lets the next kernel's CTAs be scheduled.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Asynchronous global -> shared copies (cp.async, through L2 only): every
// copy of a staging round is in flight at once, then one wait.  stage_async
// spreads n floats over the CTA's threads: 16-byte copies where both
// addresses allow, 4-byte copies otherwise.
__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void cp_async16(float* dst, const float* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(dst)), "l"(src)
               : "memory");
}
__device__ __forceinline__ void cp_async4(float* dst, const float* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_addr(dst)), "l"(src)
               : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.wait_all;" ::: "memory");
}
__device__ __forceinline__ void stage_async(float* dst, const float* src, int n) {
  const bool vec = ((n & 3) == 0) && ((reinterpret_cast<uintptr_t>(src) & 15) == 0) &&
                   ((smem_addr(dst) & 15) == 0);
  if (vec) {
    for (int i = threadIdx.x * 4; i < n; i += blockDim.x * 4) cp_async16(dst + i, src + i);
  } else {
    for (int i = threadIdx.x; i < n; i += blockDim.x) cp_async4(dst + i, src + i);
  }
}

template <typename... KArgs, typename... Args>
ns_status launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                     cudaStream_t s, const char* what, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, static_cast<Args&&>(args)...);
  if (e != cudaSuccess) return cuda_fail(e, what);
  count_launch();
  return NS_OK;
}

}  // namespace nsb

#define NS_TRY_CUDA(call, what)                          \
  do {                                                   \
    cudaError_t _e = (call);                             \
    if (_e != cudaSuccess) return nsb::cuda_fail(_e, what); \
  } while (0)

#define NS_REQUIRE(cond, msg) \
  do {                        \
    if (!(cond)) return nsb::fail(NS_ERR_INVALID_ARGUMENT, msg); \
  } while (0)

// ----------------------------------------------------------------- device side
namespace nsb {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// The reference's tanh GELU and its derivative (src/tensor.cpp:436-458), with
// the products written as separate IEEE multiplies and adds (no FMA
// contraction) to stay as close to the reference's arithmetic as the device
// tanhf allows.
__device__ __forceinline__ float gelu_f(float x) {
  const float cube = __fmul_rn(__fmul_rn(__fmul_rn(0.044715f, x), x), x);
  const float inner = __fmul_rn(0.7978845608f, __fadd_rn(x, cube));
  return __fmul_rn(__fmul_rn(0.5f, x), __fadd_rn(1.0f, tanhf(inner)));
}

__device__ __forceinline__ float gelu_grad_f(float x) {
  const float cube = __fmul_rn(__fmul_rn(__fmul_rn(0.044715f, x), x), x);
  const float inner = __fmul_rn(0.7978845608f, __fadd_rn(x, cube));
  const float th = tanhf(inner);
  const float d_inner =
      __fmul_rn(0.7978845608f, __fadd_rn(1.0f, __fmul_rn(__fmul_rn(3.0f * 0.044715f, x), x)));
  const float a = __fmul_rn(0.5f, __fadd_rn(1.0f, th));
  const float b = __fmul_rn(__fmul_rn(__fmul_rn(0.5f, x), __fsub_rn(1.0f, __fmul_rn(th, th))),
                            d_inner);
  return __fadd_rn(a, b);
}

}  // namespace nsb
