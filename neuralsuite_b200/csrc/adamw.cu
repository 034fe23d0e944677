// K5: AdamW over every parameter tensor in one launch (AdamW::Step,
// include/optimizers.h:206-234).  Parameters, gradients and both moments are
// flat buffers in registration order; the segment table (tensor boundaries and
// each tensor's weight decay) travels by value in kernel parameter space.  The
// launch is one wave of CTAs, each given an equal share of the elements (its
// range may cross tensor boundaries), so no CTA starts late and none idles:
// the pass runs at the copy bandwidth.  28 bytes of HBM traffic per parameter.
#include <algorithm>
#include <vector>

#include "common.cuh"

namespace nsb {
namespace {

constexpr int kMaxSegs = 512;  // tensors per launch: 512 x 12 B of kernel parameters

struct AdamTable {
  int n;                       // segments in this launch
  int64_t per;                 // elements per CTA
  int64_t off[kMaxSegs + 1];   // segment t = [off[t], off[t + 1])
  float decay[kMaxSegs];
};

// The update, with every multiply/add rounded separately as in the reference.
__device__ __forceinline__ void adam_one(float& p, float g, float& m, float& v, float lr, float b1,
                                         float b2, float eps, float bc1, float bc2, float decay) {
  m = __fadd_rn(__fmul_rn(b1, m), __fmul_rn(__fsub_rn(1.0f, b1), g));
  v = __fadd_rn(__fmul_rn(b2, v), __fmul_rn(__fmul_rn(__fsub_rn(1.0f, b2), g), g));
  const float mh = __fdiv_rn(m, bc1);
  const float vh = __fdiv_rn(v, bc2);
  if (decay > 0.0f) p = __fsub_rn(p, __fmul_rn(__fmul_rn(lr, decay), p));
  p = __fsub_rn(p, __fdiv_rn(__fmul_rn(lr, mh), __fadd_rn(__fsqrt_rn(vh), eps)));
}

// Device-side hyper-parameters, so a captured step replays with the current
// step count and learning rate: [lr, b1, b2, eps, bc1, bc2, step(as float bits)].
struct AdamHyper {
  const float* dev;  // nullptr: use the by-value fields
  float lr, b1, b2, eps, bc1, bc2;
};

// One piece [s, s + n) of one tensor: scalar head up to a 16-byte boundary,
// float4 body, scalar tail.
__device__ __forceinline__ void adam_piece(int64_t s, int n, float decay, float* __restrict__ P,
                                           const float* __restrict__ G, float* __restrict__ M,
                                           float* __restrict__ V, float lr, float b1, float b2,
                                           float eps, float bc1, float bc2) {
  const int head = min(n, (int)((4 - (s & 3)) & 3));
  for (int i = threadIdx.x; i < head; i += blockDim.x) {
    float p = P[s + i], m = M[s + i], v = V[s + i];
    adam_one(p, G[s + i], m, v, lr, b1, b2, eps, bc1, bc2, decay);
    P[s + i] = p; M[s + i] = m; V[s + i] = v;
  }
  const int body4 = (n - head) >> 2;
  float4* P4 = reinterpret_cast<float4*>(P + s + head);
  const float4* G4 = reinterpret_cast<const float4*>(G + s + head);
  float4* M4 = reinterpret_cast<float4*>(M + s + head);
  float4* V4 = reinterpret_cast<float4*>(V + s + head);
  for (int i = threadIdx.x; i < body4; i += blockDim.x) {
    float4 p = P4[i], m = M4[i], v = V4[i];
    const float4 g = G4[i];
    adam_one(p.x, g.x, m.x, v.x, lr, b1, b2, eps, bc1, bc2, decay);
    adam_one(p.y, g.y, m.y, v.y, lr, b1, b2, eps, bc1, bc2, decay);
    adam_one(p.z, g.z, m.z, v.z, lr, b1, b2, eps, bc1, bc2, decay);
    adam_one(p.w, g.w, m.w, v.w, lr, b1, b2, eps, bc1, bc2, decay);
    P4[i] = p; M4[i] = m; V4[i] = v;
  }
  for (int i = head + body4 * 4 + threadIdx.x; i < n; i += blockDim.x) {
    float p = P[s + i], m = M[s + i], v = V[s + i];
    adam_one(p, G[s + i], m, v, lr, b1, b2, eps, bc1, bc2, decay);
    P[s + i] = p; M[s + i] = m; V[s + i] = v;
  }
}

__global__ void __launch_bounds__(256) adamw_k(const AdamTable tab, float* __restrict__ P,
                                               const float* __restrict__ G, float* __restrict__ M,
                                               float* __restrict__ V, AdamHyper hp) {
  pdl_wait();     // the previous kernel's writes are visible (launched by launch_pdl)
  pdl_trigger();  // the next kernel, if launched as a programmatic dependent, may start
  float lr = hp.lr, b1 = hp.b1, b2 = hp.b2, eps = hp.eps, bc1 = hp.bc1, bc2 = hp.bc2;
  if (hp.dev) {
    lr = hp.dev[0]; b1 = hp.dev[1]; b2 = hp.dev[2]; eps = hp.dev[3]; bc1 = hp.dev[4]; bc2 = hp.dev[5];
  }
  const int64_t end = tab.off[tab.n];
  const int64_t lo = tab.off[0] + tab.per * blockIdx.x;
  const int64_t hi = min(end, lo + tab.per);
  if (lo >= hi) return;
  // First segment that ends after lo (segments may be empty).
  int a = 0, b = tab.n - 1;
  while (a < b) {
    const int mid = (a + b) >> 1;
    if (tab.off[mid + 1] > lo) b = mid; else a = mid + 1;
  }
  for (int t = a; t < tab.n && tab.off[t] < hi; ++t) {
    const int64_t s = max(lo, tab.off[t]);
    const int64_t e = min(hi, tab.off[t + 1]);
    if (e > s) adam_piece(s, (int)(e - s), tab.decay[t], P, G, M, V, lr, b1, b2, eps, bc1, bc2);
  }
}

// Step counter + bias corrections on the device (AdamW::Step's first three
// lines, include/optimizers.h:208-210): step += 1; bc = 1 - pow(beta, step)
// evaluated in double and rounded to float, as std::pow(float, int) does.
__global__ void adamw_prep_k(float* hyper) {
  pdl_wait();     // the previous kernel's writes are visible (launched by launch_pdl)
  pdl_trigger();  // the next kernel, if launched as a programmatic dependent, may start
  int step = __float_as_int(hyper[6]) + 1;
  hyper[6] = __int_as_float(step);
  hyper[4] = (float)(1.0 - pow((double)hyper[1], (double)step));
  hyper[5] = (float)(1.0 - pow((double)hyper[2], (double)step));
}

ns_status adamw_run(float* params, const float* grads, float* m, float* v, int64_t n_total,
                    const int64_t* host_seg_offsets, const float* host_seg_decay, int n_seg,
                    AdamHyper hp, cudaStream_t s);

}  // namespace

// Prep + update with the hyper-parameters read on the device.
ns_status adamw_step_device(float* params, const float* grads, float* m, float* v,
                            int64_t n_total, const int64_t* host_seg_offsets,
                            const float* host_seg_decay, int n_seg, float* hyper,
                            cudaStream_t s) {
  {
    const ns_status rc = launch_pdl(adamw_prep_k, dim3(1), dim3(1), 0, s, "adamw prep", hyper);
    if (rc != NS_OK) return rc;
  }
  AdamHyper hp{hyper, 0.f, 0.f, 0.f, 0.f, 1.f, 1.f};
  return adamw_run(params, grads, m, v, n_total, host_seg_offsets, host_seg_decay, n_seg, hp, s);
}

namespace {
ns_status adamw_run(float* params, const float* grads, float* m, float* v, int64_t n_total,
                    const int64_t* host_seg_offsets, const float* host_seg_decay, int n_seg,
                    AdamHyper hp, cudaStream_t s) {
  NS_REQUIRE(n_seg >= 0 && host_seg_offsets && (n_seg == 0 || host_seg_decay),
             "ns_adamw_flat: bad segment table");
  NS_REQUIRE(((reinterpret_cast<uintptr_t>(params) | reinterpret_cast<uintptr_t>(grads) |
               reinterpret_cast<uintptr_t>(m) | reinterpret_cast<uintptr_t>(v)) & 15) == 0,
             "ns_adamw_flat: buffers must be 16-byte aligned");
  NS_REQUIRE(host_seg_offsets[0] >= 0 && host_seg_offsets[n_seg] <= n_total,
             "ns_adamw_flat: segments exceed the buffer");
  for (int t = 0; t < n_seg; ++t)
    NS_REQUIRE(host_seg_offsets[t + 1] >= host_seg_offsets[t],
               "ns_adamw_flat: segment offsets must be ascending");
  // One wave: as many CTAs as fit on the GPU at once, each with an equal
  // share (a multiple of 1024 elements) of the launch's range.
  // (CTAs per SM depend only on the kernel; the SM count is the current device's.)
  static const int per_sm = [] {
    int n = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, adamw_k, 256, 0) == cudaSuccess) return n;
    (void)cudaGetLastError();  // one CTA per SM then; the launch reports any real fault
    return 0;
  }();
  const int waves_cta = std::max(1, per_sm) * sm_count();
  AdamTable tab;
  for (int t0 = 0; t0 < n_seg; t0 += kMaxSegs) {
    const int n = std::min(kMaxSegs, n_seg - t0);
    tab.n = n;
    for (int t = 0; t <= n; ++t) tab.off[t] = host_seg_offsets[t0 + t];
    for (int t = 0; t < n; ++t) tab.decay[t] = host_seg_decay[t0 + t];
    const int64_t len = tab.off[n] - tab.off[0];
    if (len == 0) continue;
    const int64_t per = std::max<int64_t>(1024, (len + waves_cta - 1) / waves_cta + 1023) & ~int64_t(1023);
    tab.per = per;
    const int grid = (int)((len + per - 1) / per);
    ns_status rc = launch_pdl(adamw_k, dim3(grid), dim3(256), 0, s, "ns_adamw_flat", tab, params,
                              grads, m, v, hp);
    if (rc != NS_OK) return rc;
  }
  return NS_OK;
}
}  // namespace
}  // namespace nsb

using namespace nsb;

extern "C" ns_status ns_adamw_flat(float* params, const float* grads, float* m, float* v,
                                   int64_t n_total, const int64_t* host_seg_offsets,
                                   const float* host_seg_decay, int n_seg, float lr, float b1,
                                   float b2, float eps, float bc1, float bc2, void* stream) {
  AdamHyper hp{nullptr, lr, b1, b2, eps, bc1, bc2};
  return adamw_run(params, grads, m, v, n_total, host_seg_offsets, host_seg_decay, n_seg, hp,
                   as_stream(stream));
}

extern "C" ns_status ns_adamw_flat_device(float* params, const float* grads, float* m, float* v,
                                          int64_t n_total, const int64_t* host_seg_offsets,
                                          const float* host_seg_decay, int n_seg,
                                          float* dev_hyper, void* stream) {
  NS_REQUIRE(dev_hyper, "ns_adamw_flat_device: dev_hyper is NULL");
  return adamw_step_device(params, grads, m, v, n_total, host_seg_offsets, host_seg_decay, n_seg,
                           dev_hyper, as_stream(stream));
}
