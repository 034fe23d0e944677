// K3: GELU, residual add, fused cross-entropy forward+backward, gradient
// sum-of-squares and clip.  All HBM-bound; float4 grid-stride loops, one warp
// per row for the cross-entropy, deterministic fixed-order reductions.
#include <algorithm>
#include <cuda.h>

#include <mutex>

#include "common.cuh"

namespace nsb {
namespace {

int pointwise_grid(int64_t n4) {
  const int64_t want = ceil_div64(n4, 256);
  return (int)std::max<int64_t>(1, std::min<int64_t>(want, (int64_t)sm_count() * 8));
}

__global__ void gelu_fwd_k(const float* __restrict__ x, float* __restrict__ y, int64_t n) {
  pdl_wait();     // the previous kernel's writes are visible (launched by launch_pdl)
  pdl_trigger();  // the next kernel, if launched as a programmatic dependent, may start
  const int64_t n4 = n >> 2;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n4; i += stride) {
    float4 v = reinterpret_cast<const float4*>(x)[i];
    v.x = gelu_f(v.x); v.y = gelu_f(v.y); v.z = gelu_f(v.z); v.w = gelu_f(v.w);
    reinterpret_cast<float4*>(y)[i] = v;
  }
  for (int64_t i = (n4 << 2) + blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += stride)
    y[i] = gelu_f(x[i]);
}

// y = gelu(x) and y_lo = y - trunc_tf32(y) (the next GEMM's operand split).
__global__ void gelu_fwd_lo_k(const float* __restrict__ x, float* __restrict__ y,
                              float* __restrict__ y_lo, int64_t n) {
  pdl_wait();     // the previous kernel's writes are visible (launched by launch_pdl)
  pdl_trigger();  // the next kernel, if launched as a programmatic dependent, may start
  const int64_t n4 = n >> 2;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  auto lo = [](float v) { return v - __uint_as_float(__float_as_uint(v) & 0xFFFFE000u); };
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n4; i += stride) {
    float4 v = reinterpret_cast<const float4*>(x)[i];
    v.x = gelu_f(v.x); v.y = gelu_f(v.y); v.z = gelu_f(v.z); v.w = gelu_f(v.w);
    reinterpret_cast<float4*>(y)[i] = v;
    reinterpret_cast<float4*>(y_lo)[i] = make_float4(lo(v.x), lo(v.y), lo(v.z), lo(v.w));
  }
  for (int64_t i = (n4 << 2) + blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += stride) {
    const float v = gelu_f(x[i]);
    y[i] = v;
    y_lo[i] = lo(v);
  }
}

__global__ void gelu_bwd_k(const float* __restrict__ d, const float* __restrict__ x,
                           float* __restrict__ dx, int64_t n) {
  pdl_wait();     // the previous kernel's writes are visible (launched by launch_pdl)
  pdl_trigger();  // the next kernel, if launched as a programmatic dependent, may start
  const int64_t n4 = n >> 2;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n4; i += stride) {
    const float4 v = reinterpret_cast<const float4*>(x)[i];
    const float4 g = reinterpret_cast<const float4*>(d)[i];
    float4 o;
    o.x = __fmul_rn(g.x, gelu_grad_f(v.x)); o.y = __fmul_rn(g.y, gelu_grad_f(v.y));
    o.z = __fmul_rn(g.z, gelu_grad_f(v.z)); o.w = __fmul_rn(g.w, gelu_grad_f(v.w));
    reinterpret_cast<float4*>(dx)[i] = o;
  }
  for (int64_t i = (n4 << 2) + blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += stride)
    dx[i] = __fmul_rn(d[i], gelu_grad_f(x[i]));
}

__global__ void add_k(const float* __restrict__ a, const float* __restrict__ b,
                      float* __restrict__ o, int64_t n) {
  pdl_wait();     // the previous kernel's writes are visible (launched by launch_pdl)
  pdl_trigger();  // the next kernel, if launched as a programmatic dependent, may start
  const int64_t n4 = n >> 2;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n4; i += stride) {
    const float4 u = reinterpret_cast<const float4*>(a)[i];
    const float4 v = reinterpret_cast<const float4*>(b)[i];
    reinterpret_cast<float4*>(o)[i] =
        make_float4(__fadd_rn(u.x, v.x), __fadd_rn(u.y, v.y), __fadd_rn(u.z, v.z), __fadd_rn(u.w, v.w));
  }
  for (int64_t i = (n4 << 2) + blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += stride)
    o[i] = __fadd_rn(a[i], b[i]);
}

// CrossEntropyLoss (include/losses.h:34-86), one warp per row:
//   row_loss = -((x_t - max) - log(sum exp(x - max)))
//   dlogits  = (exp(x - max)/sum - onehot) / denom
__global__ void __launch_bounds__(256) ce_rows_k(const float* __restrict__ logits,
                                                 const int32_t* __restrict__ targets, int rows,
                                                 int classes, float denom,
                                                 float* __restrict__ dlogits,
                                                 float* __restrict__ row_loss,
                                                 int32_t* __restrict__ err) {
  pdl_wait();     // the previous kernel's writes are visible (launched by launch_pdl)
  pdl_trigger();  // the next kernel, if launched as a programmatic dependent, may start
  const int row = blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const float* p = logits + (size_t)row * classes;
  float* d = dlogits + (size_t)row * classes;
  const int t = targets[row];
  const bool bad = t < 0 || t >= classes;
  float mx = -INFINITY;
  for (int c = lane; c < classes; c += 32) mx = fmaxf(mx, p[c]);
  mx = warp_max(mx);
  float s = 0.f;
  for (int c = lane; c < classes; c += 32) s += expf(__fsub_rn(p[c], mx));
  s = warp_sum(s);
  for (int c = lane; c < classes; c += 32) {
    const float prob = __fdiv_rn(expf(__fsub_rn(p[c], mx)), s);
    const float tv = (c == t) ? 1.0f : 0.0f;
    d[c] = __fdiv_rn(__fsub_rn(prob, tv), denom);
  }
  if (lane == 0) {
    if (bad) {
      if (err) atomicExch(err, 1);
      row_loss[row] = 0.0f;
    } else {
      row_loss[row] = -__fsub_rn(__fsub_rn(p[t], mx), logf(s));
    }
  }
}

// Ordered single-CTA reduction: out[0] = (sum of x[0..n)) / div.
__global__ void __launch_bounds__(1024) sum_finish_k(const float* __restrict__ x, int64_t n,
                                                     float div, float* __restrict__ out) {
  pdl_wait();     // the previous kernel's writes are visible (launched by launch_pdl)
  pdl_trigger();  // the next kernel, if launched as a programmatic dependent, may start
  __shared__ float sh[32];
  float s = 0.f;
  for (int64_t i = threadIdx.x; i < n; i += blockDim.x) s += x[i];
  s = warp_sum(s);
  if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x >> 5) ? sh[threadIdx.x] : 0.f;
    v = warp_sum(v);
    if (threadIdx.x == 0) out[0] = __fdiv_rn(v, div);
  }
}

// Per-CTA partial sums of squares (grid-stride, float4), one float per CTA.
__global__ void __launch_bounds__(256) sumsq_partial_k(const float* __restrict__ x, int64_t n,
                                                       float* __restrict__ part) {
  pdl_wait();     // the previous kernel's writes are visible (launched by launch_pdl)
  pdl_trigger();  // the next kernel, if launched as a programmatic dependent, may start
  __shared__ float sh[8];
  const int64_t n4 = n >> 2;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  float s = 0.f;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n4; i += stride) {
    const float4 v = reinterpret_cast<const float4*>(x)[i];
    s += (v.x * v.x + v.y * v.y) + (v.z * v.z + v.w * v.w);
  }
  for (int64_t i = (n4 << 2) + blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += stride)
    s += x[i] * x[i];
  s = warp_sum(s);
  if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int w = 0; w < 8; ++w) t += sh[w];
    part[blockIdx.x] = t;
  }
}

// ClipGradients' rescale (train_llm.cpp:121-128) with the norm read on device.
__global__ void clip_scale_k(float* __restrict__ x, int64_t n, const float* __restrict__ sumsq,
                             float max_norm) {
  pdl_wait();     // the previous kernel's writes are visible (launched by launch_pdl)
  pdl_trigger();  // the next kernel, if launched as a programmatic dependent, may start
  const float norm = __fsqrt_rn(sumsq[0]);
  if (!(norm > max_norm && norm > 0.0f)) return;
  const float scale = __fdiv_rn(max_norm, norm);
  const int64_t n4 = n >> 2;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n4; i += stride) {
    float4 v = reinterpret_cast<float4*>(x)[i];
    v.x = __fmul_rn(v.x, scale); v.y = __fmul_rn(v.y, scale);
    v.z = __fmul_rn(v.z, scale); v.w = __fmul_rn(v.w, scale);
    reinterpret_cast<float4*>(x)[i] = v;
  }
  for (int64_t i = (n4 << 2) + blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += stride)
    x[i] = __fmul_rn(x[i], scale);
}

bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

constexpr int kSumsqCtas = 592;  // 4 x 148

}  // namespace
}  // namespace nsb

using namespace nsb;

extern "C" {

ns_status ns_gelu_fwd(const float* x, float* y, int64_t n, void* stream) {
  NS_REQUIRE(n >= 0, "ns_gelu_fwd: n < 0");
  NS_REQUIRE(al16(x) && al16(y), "ns_gelu_fwd: pointers must be 16-byte aligned");
  if (n == 0) return NS_OK;
  return launch_pdl(gelu_fwd_k, dim3(pointwise_grid(ceil_div64(n, 4))), dim3(256), 0,
                    as_stream(stream), "ns_gelu_fwd", x, y, n);
}

ns_status ns_gelu_fwd_lo(const float* x, float* y, float* y_lo, int64_t n, void* stream) {
  NS_REQUIRE(n >= 0, "ns_gelu_fwd_lo: n < 0");
  NS_REQUIRE(al16(x) && al16(y) && al16(y_lo), "ns_gelu_fwd_lo: pointers must be 16-byte aligned");
  if (n == 0) return NS_OK;
  return launch_pdl(gelu_fwd_lo_k, dim3(pointwise_grid(ceil_div64(n, 4))), dim3(256), 0,
                    as_stream(stream), "ns_gelu_fwd_lo", x, y, y_lo, n);
}

ns_status ns_gelu_bwd(const float* dout, const float* x, float* dx, int64_t n, void* stream) {
  NS_REQUIRE(n >= 0, "ns_gelu_bwd: n < 0");
  NS_REQUIRE(al16(x) && al16(dout) && al16(dx), "ns_gelu_bwd: pointers must be 16-byte aligned");
  if (n == 0) return NS_OK;
  return launch_pdl(gelu_bwd_k, dim3(pointwise_grid(ceil_div64(n, 4))), dim3(256), 0,
                    as_stream(stream), "ns_gelu_bwd", dout, x, dx, n);
}

ns_status ns_add(const float* a, const float* b, float* out, int64_t n, void* stream) {
  NS_REQUIRE(n >= 0, "ns_add: n < 0");
  NS_REQUIRE(al16(a) && al16(b) && al16(out), "ns_add: pointers must be 16-byte aligned");
  if (n == 0) return NS_OK;
  return launch_pdl(add_k, dim3(pointwise_grid(ceil_div64(n, 4))), dim3(256), 0, as_stream(stream),
                    "ns_add", a, b, out, n);
}

size_t ns_cross_entropy_workspace_size(int rows, int classes) {
  (void)classes;
  return rows > 0 ? (size_t)rows * sizeof(float) : 0;
}

ns_status ns_cross_entropy(const float* logits, const int32_t* targets, int rows, int classes,
                           float denom, float* loss_out, float* dlogits, int32_t* err_flag,
                           void* workspace, size_t workspace_bytes, void* stream) {
  NS_REQUIRE(rows > 0 && classes > 0, "ns_cross_entropy: rows and classes must be positive");
  NS_REQUIRE(denom > 0.0f, "ns_cross_entropy: denom must be positive");
  NS_REQUIRE(workspace && workspace_bytes >= ns_cross_entropy_workspace_size(rows, classes),
             "ns_cross_entropy: workspace too small");
  cudaStream_t s = as_stream(stream);
  float* row_loss = static_cast<float*>(workspace);
  const ns_status rc = launch_pdl(ce_rows_k, dim3(ceil_div(rows, 8)), dim3(256), 0, s,
                                  "ns_cross_entropy rows", logits, targets, rows, classes, denom,
                                  dlogits, row_loss, err_flag);
  if (rc != NS_OK) return rc;
  return launch_pdl(sum_finish_k, dim3(1), dim3(1024), 0, s, "ns_cross_entropy finish", row_loss,
                    rows, (float)rows, loss_out);
}

size_t ns_sumsq_workspace_size(int64_t n) {
  (void)n;
  return kSumsqCtas * sizeof(float);
}

ns_status ns_sumsq(const float* x, int64_t n, float* out, void* workspace, size_t workspace_bytes,
                   void* stream) {
  NS_REQUIRE(n >= 0, "ns_sumsq: n < 0");
  NS_REQUIRE(al16(x), "ns_sumsq: x must be 16-byte aligned");
  NS_REQUIRE(workspace && workspace_bytes >= ns_sumsq_workspace_size(n),
             "ns_sumsq: workspace too small");
  cudaStream_t s = as_stream(stream);
  float* part = static_cast<float*>(workspace);
  const ns_status rc = launch_pdl(sumsq_partial_k, dim3(kSumsqCtas), dim3(256), 0, s,
                                  "ns_sumsq partial", x, n, part);
  if (rc != NS_OK) return rc;
  return launch_pdl(sum_finish_k, dim3(1), dim3(1024), 0, s, "ns_sumsq finish", part, kSumsqCtas,
                    1.0f, out);
}

ns_status ns_clip_scale(float* x, int64_t n, const float* sumsq, float max_norm, void* stream) {
  NS_REQUIRE(n >= 0, "ns_clip_scale: n < 0");
  NS_REQUIRE(al16(x), "ns_clip_scale: x must be 16-byte aligned");
  if (n == 0) return NS_OK;
  return launch_pdl(clip_scale_k, dim3(pointwise_grid(ceil_div64(n, 4))), dim3(256), 0,
                    as_stream(stream), "ns_clip_scale", x, n, sumsq, max_norm);
}

}  // extern "C"

// ------------------------------------------------------------------------
// Allocation-free variant of ns_cross_entropy for callers that cannot call
// cudaMalloc at the point of the call (see ns_b200.h).  Its only scratch, one
// float of loss per row, is this file-scope device array.
namespace nsb {
namespace {

static __device__ __align__(256) float g_ce_noalloc_rows[NS_CE_NOALLOC_MAX_ROWS];

// Device address of g_ce_noalloc_rows for the current device, looked up with
// that device current on its first call and again whenever the device's
// context has changed since (cudaDeviceReset destroys the context the
// address belonged to; the next call runs in a new one).  Host code must not
// pass the symbol itself to a kernel: on the host it names a shadow variable,
// not device memory.
typedef CUresult (*CtxGetCurrentFn)(CUcontext*);

CtxGetCurrentFn ctx_get_current() {
  static const CtxGetCurrentFn fn = []() -> CtxGetCurrentFn {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      return reinterpret_cast<CtxGetCurrentFn>(p);
    return nullptr;
  }();
  return fn;
}

ns_status ce_noalloc_scratch(float** out) {
  static std::mutex mu;
  static float* addr[64] = {};
  static CUcontext ctx_of[64] = {};
  int dev = 0;
  NS_TRY_CUDA(cudaGetDevice(&dev), "ns_cross_entropy_noalloc: cudaGetDevice");
  if (dev < 0 || dev >= 64) return fail(NS_ERR_UNSUPPORTED, "ns_cross_entropy_noalloc: device index >= 64");
  CtxGetCurrentFn get = ctx_get_current();
  if (!get) return fail(NS_ERR_UNSUPPORTED, "ns_cross_entropy_noalloc: cuCtxGetCurrent unavailable");
  CUcontext ctx = nullptr;
  if (get(&ctx) != CUDA_SUCCESS)
    return fail(NS_ERR_CUDA, "ns_cross_entropy_noalloc: cuCtxGetCurrent failed");
  if (!ctx) {
    // No context on this thread yet (so no capture can be running either):
    // cudaFree(NULL) makes the device's primary context current, allocating
    // nothing.
    NS_TRY_CUDA(cudaFree(nullptr), "ns_cross_entropy_noalloc: context");
    if (get(&ctx) != CUDA_SUCCESS || !ctx)
      return fail(NS_ERR_CUDA, "ns_cross_entropy_noalloc: no current context");
  }
  std::lock_guard<std::mutex> lock(mu);
  if (!addr[dev] || ctx_of[dev] != ctx) {
    void* p = nullptr;
    NS_TRY_CUDA(cudaGetSymbolAddress(&p, g_ce_noalloc_rows),
                "ns_cross_entropy_noalloc: cudaGetSymbolAddress");
    addr[dev] = static_cast<float*>(p);
    ctx_of[dev] = ctx;
  }
  *out = addr[dev];
  return NS_OK;
}

}  // namespace
}  // namespace nsb

extern "C" ns_status ns_cross_entropy_noalloc(const float* logits, const int32_t* targets,
                                              int rows, int classes, float denom, float* loss_out,
                                              float* dlogits, int32_t* err_flag, void* stream) {
  NS_REQUIRE(rows > 0 && classes > 0, "ns_cross_entropy_noalloc: rows and classes must be positive");
  NS_REQUIRE(denom > 0.0f, "ns_cross_entropy_noalloc: denom must be positive");
  if (rows > NS_CE_NOALLOC_MAX_ROWS)
    return fail(NS_ERR_INVALID_ARGUMENT,
                "ns_cross_entropy_noalloc: rows = " + std::to_string(rows) +
                    " exceeds the static scratch of NS_CE_NOALLOC_MAX_ROWS = " +
                    std::to_string(NS_CE_NOALLOC_MAX_ROWS) +
                    " rows; use ns_cross_entropy with a caller workspace");
  float* row_loss = nullptr;
  ns_status rc = ce_noalloc_scratch(&row_loss);
  if (rc != NS_OK) return rc;
  cudaStream_t s = as_stream(stream);
  rc = launch_pdl(ce_rows_k, dim3(ceil_div(rows, 8)), dim3(256), 0, s,
                  "ns_cross_entropy_noalloc rows", logits, targets, rows, classes, denom, dlogits,
                  row_loss, err_flag);
  if (rc != NS_OK) return rc;
  return launch_pdl(sum_finish_k, dim3(1), dim3(1024), 0, s, "ns_cross_entropy_noalloc finish",
                    row_loss, rows, (float)rows, loss_out);
}
