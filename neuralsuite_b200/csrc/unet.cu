// The diffusion U-Net training step on the device (the reference has the
// layers but no U-Net; its wiring here is the one ref_harness.cpp builds from
// the reference's own classes):
//
//   e0 = LN0(Res0(conv_in(x)))                     base channels, S x S
//   e1 = LN1(Res1(down1(e0)))                      2*base, S/2 (stride 2)
//   m  = LN2(Res2(down2(e1)))                      4*base, S/4 (stride 2)
//   u1 = LN3(Res3(up1(Up(m)) + e1))                2*base, S/2
//   u0 = LN4(Res4(up0(Up(u1)) + e0))               base, S
//   y  = conv_out(u0);  loss = MSE(y, target)
//
// Res(a) = ReLU(conv(a) + a) (ResidualBlock, include/layers/residual.h:23-64,
// with a 3x3 Conv2D inside), LN normalises the last axis (LayerNormLayer,
// include/layers/layernorm.h), Up is nearest-neighbour 2x (not in the
// reference), MSE is MSELoss (include/losses.h:97-124).  Convolutions run
// as ns_conv2d_fwd/bwd do (im2col columns + tcgen05 3xTF32 GEMMs), each
// keeping its forward's columns for its backward (one column buffer per
// convolution, 4.6 GB at 32 images of 64 x 64, base 64); the
// element-wise steps are fused passes: residual add + ReLU, ReLU mask +
// skip add in the backward, upsample and its 2x2 sum, MSE with a two-stage
// ordered loss sum.  Parameters and gradients are flat buffers in
// registration order; AdamW is the same single-launch kernel as the GPT's.
#include <algorithm>
#include <memory>
#include <string>
#include <vector>

#include "comm.h"
#include "common.cuh"
#include "conv.h"

struct ns_unet {
  int in_ch = 3, base = 64, S = 64, max_batch = 1, B = 0;
  // conv i: 0 conv_in, 1 down1, 2 down2, 3 up1, 4 up0, 5 conv_out, 6..10 the
  // residual blocks' inner convolutions of levels 0..4.
  struct Conv {
    int ic, oc, stride, in_hw;
    int64_t w_off, b_off;
    float *cols = nullptr, *cols_lo = nullptr;  // the forward's columns, kept for the backward
  };
  std::vector<Conv> conv;
  int64_t ln_off[5][2];  // gamma, beta of LN0..LN4
  int lvl_c[5], lvl_hw[5];
  std::vector<int64_t> offsets;
  std::vector<int> ranks;
  std::vector<float> decay;
  float wd = 0.01f;
  int64_t n_params = 0;
  float *params = nullptr, *grads = nullptr, *m = nullptr, *v = nullptr, *hyper = nullptr;
  bool opt = false;
  float *x = nullptr, *out = nullptr, *dout = nullptr, *a[5] = {}, *r[5] = {}, *e[5] = {};
  float *mean[5] = {}, *rstd[5] = {};
  float *up_a = nullptr, *up_b = nullptr, *t0 = nullptr, *t1 = nullptr, *t2 = nullptr;
  float *g0 = nullptr, *g1 = nullptr;  // gradients of the two skip sums
  float* small = nullptr;  // [0] loss, [1..] partial sums
  void* conv_ws = nullptr;
  size_t conv_ws_bytes = 0;
  void* ln_ws = nullptr;
  size_t ln_ws_bytes = 0;
  float* loss_part = nullptr;
  ns_comm* comm = nullptr;
  int world = 1;
  std::vector<void*> allocs;
};

namespace nsb {
namespace unet {
namespace {

int grid_for(int64_t work) {
  return (int)std::max<int64_t>(1, std::min<int64_t>((work + 255) / 256, (int64_t)sm_count() * 8));
}

// y = ReLU(f + x) (ResidualBlock::Forward's sum then Activation(kRelu)).
__global__ void resid_relu_k(const float* __restrict__ f, const float* __restrict__ x, int64_t n,
                             float* __restrict__ y) {
  pdl_wait();     // the previous kernel's writes are visible (launched by launch_pdl)
  pdl_trigger();  // the next kernel, if launched as a programmatic dependent, may start
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const float s = __fadd_rn(f[i], x[i]);
    y[i] = s > 0.0f ? s : 0.0f;
  }
}

// dsum = y > 0 ? dy : 0 (ReluBackward on the pre-activation sum, whose sign
// is that of the output).  dsum may be dy.
__global__ void relu_mask_k(const float* dy, const float* __restrict__ y, int64_t n, float* dsum) {
  pdl_wait();     // the previous kernel's writes are visible (launched by launch_pdl)
  pdl_trigger();  // the next kernel, if launched as a programmatic dependent, may start
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    dsum[i] = y[i] > 0.0f ? dy[i] : 0.0f;
}

// y[bc][i][j] = x[bc][i/2][j/2]: one thread per input element writes its
// 2 x 2 block as two 8-byte stores (32-bit indexing: n < 2^31).
__global__ void up2_k(const float* __restrict__ x, int n, int W, float* __restrict__ y) {
  pdl_wait();     // the previous kernel's writes are visible (launched by launch_pdl)
  pdl_trigger();  // the next kernel, if launched as a programmatic dependent, may start
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    const int row = i / W, j = i - row * W;  // row = bc * H + r
    const float v = x[i];
    float* o = y + (size_t)row * 4 * W + 2 * j;  // output row 2r of plane bc
    *reinterpret_cast<float2*>(o) = make_float2(v, v);
    *reinterpret_cast<float2*>(o + 2 * W) = make_float2(v, v);
  }
}

// dx[bc][i][j] = dy[2i][2j] + dy[2i][2j+1] + dy[2i+1][2j] + dy[2i+1][2j+1], in that order.
__global__ void up2_bwd_k(const float* __restrict__ dy, int n, int W, float* __restrict__ dx) {
  pdl_wait();     // the previous kernel's writes are visible (launched by launch_pdl)
  pdl_trigger();  // the next kernel, if launched as a programmatic dependent, may start
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    const int row = i / W, j = i - row * W;
    const float* p = dy + (size_t)row * 4 * W + 2 * j;
    const float2 a = *reinterpret_cast<const float2*>(p);
    const float2 b = *reinterpret_cast<const float2*>(p + 2 * W);
    float s = 0.0f;
    s += a.x;
    s += a.y;
    s += b.x;
    s += b.y;
    dx[i] = s;
  }
}

// MSELoss forward + backward: d = 2 * (p - t) / denom, per-CTA sums of
// (p - t)^2 into part[blockIdx.x] (an ordered tree inside the CTA).
__global__ void mse_k(const float* __restrict__ p, const float* __restrict__ t, int64_t n,
                      float denom, float* __restrict__ d, float* __restrict__ part) {
  pdl_wait();     // the previous kernel's writes are visible (launched by launch_pdl)
  pdl_trigger();  // the next kernel, if launched as a programmatic dependent, may start
  __shared__ float red[256];
  float s = 0.0f;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const float diff = __fsub_rn(p[i], t[i]);
    s = __fadd_rn(s, __fmul_rn(diff, diff));
    d[i] = __fdiv_rn(__fmul_rn(2.0f, diff), denom);
  }
  red[threadIdx.x] = s;
  __syncthreads();
  for (int w = 128; w > 0; w >>= 1) {
    if ((int)threadIdx.x < w) red[threadIdx.x] += red[threadIdx.x + w];
    __syncthreads();
  }
  if (threadIdx.x == 0) part[blockIdx.x] = red[0];
}

// loss = (sum of the CTA partials in order) / n.
__global__ void mse_finish_k(const float* __restrict__ part, int nparts, float n,
                             float* __restrict__ loss) {
  pdl_wait();     // the previous kernel's writes are visible (launched by launch_pdl)
  pdl_trigger();  // the next kernel, if launched as a programmatic dependent, may start
  if (threadIdx.x == 0) {
    float s = 0.0f;
    for (int i = 0; i < nparts; ++i) s += part[i];
    loss[0] = s / n;
  }
}

constexpr int kMseBlocks = 296;

template <typename T>
ns_status dev_alloc(ns_unet* u, T** p, size_t count) {
  void* q = nullptr;
  NS_TRY_CUDA(cudaMalloc(&q, std::max<size_t>(count, 1) * sizeof(T)), "ns_unet_create");
  u->allocs.push_back(q);
  *p = static_cast<T*>(q);
  return NS_OK;
}

ns_status conv_fwd(ns_unet* u, int i, const float* in, float* out, int B, cudaStream_t s) {
  const auto& c = u->conv[i];
  return conv::forward_keep(in, B, c.ic, c.in_hw, c.in_hw, u->params + c.w_off,
                            u->params + c.b_off, c.oc, 3, c.stride, 1, out, c.cols, c.cols_lo,
                            u->conv_ws, u->conv_ws_bytes, s);
}

// The backward of conv i on the columns its forward kept (its input `in` is
// read again only by the direct paths of the 3-channel convolutions).
ns_status conv_bwd(ns_unet* u, int i, const float* in, const float* dy, float* dx, int B,
                   cudaStream_t s) {
  const auto& c = u->conv[i];
  return conv::backward_from_cols(in, c.cols, c.cols_lo, dy, B, c.ic, c.in_hw, c.in_hw,
                                  u->params + c.w_off, c.oc, 3, c.stride, 1, dx,
                                  u->grads + c.w_off, u->grads + c.b_off, u->conv_ws,
                                  u->conv_ws_bytes, s);
}

int64_t level_numel(const ns_unet* u, int l, int B) {
  return (int64_t)B * u->lvl_c[l] * u->lvl_hw[l] * u->lvl_hw[l];
}

// Res_l then LN_l on a[l] (the level's conv output): r[l] = ReLU(conv(a) + a), e[l] = LN(r).
ns_status res_ln_fwd(ns_unet* u, int l, int B, cudaStream_t s) {
  const int64_t n = level_numel(u, l, B);
  ns_status rc = conv_fwd(u, 6 + l, u->a[l], u->t0, B, s);
  if (rc != NS_OK) return rc;
  rc = launch_pdl(resid_relu_k, dim3(grid_for(n)), dim3(256), 0, s, "ns_unet residual", u->t0,
                  u->a[l], n, u->r[l]);
  if (rc != NS_OK) return rc;
  const int rows = (int)(n / u->lvl_hw[l]);
  return ns_layernorm_fwd(u->r[l], u->params + u->ln_off[l][0], u->params + u->ln_off[l][1],
                          u->e[l], u->mean[l], u->rstd[l], rows, u->lvl_hw[l], 1e-5f, s);
}

// Backward through LN_l and Res_l: de (the gradient at e[l]) -> da (at a[l]).
// Uses t1 (dr, then dsum) and t2 (the inner conv's dx).
ns_status res_ln_bwd(ns_unet* u, int l, const float* de, float* da, int B, cudaStream_t s) {
  const int64_t n = level_numel(u, l, B);
  const int rows = (int)(n / u->lvl_hw[l]);
  ns_status rc = ns_layernorm_bwd(de, u->r[l], u->params + u->ln_off[l][0], u->mean[l], u->rstd[l],
                                  nullptr, u->t1, u->grads + u->ln_off[l][0],
                                  u->grads + u->ln_off[l][1], rows, u->lvl_hw[l], u->ln_ws,
                                  u->ln_ws_bytes, s);
  if (rc != NS_OK) return rc;
  rc = launch_pdl(relu_mask_k, dim3(grid_for(n)), dim3(256), 0, s, "ns_unet relu backward", u->t1,
                  u->r[l], n, u->t1);
  if (rc != NS_OK) return rc;
  rc = conv_bwd(u, 6 + l, u->a[l], u->t1, u->t2, B, s);
  if (rc != NS_OK) return rc;
  return ns_add(u->t2, u->t1, da, n, s);  // dinput = dfx + dsum (residual.h:50-55)
}

void free_all(ns_unet* u) {
  for (void* p : u->allocs) cudaFree(p);
  u->allocs.clear();
}

}  // namespace
}  // namespace unet
}  // namespace nsb

using namespace nsb;
using namespace nsb::unet;

extern "C" {

ns_status ns_unet_create(const ns_unet_config* cfg, ns_unet** out) {
  NS_REQUIRE(cfg && out, "ns_unet_create: NULL argument");
  NS_REQUIRE(cfg->in_channels > 0 && cfg->base_channels > 0 && cfg->max_batch > 0,
             "ns_unet_create: sizes must be positive");
  NS_REQUIRE((int64_t)cfg->max_batch * 4 * cfg->base_channels * cfg->image_size * cfg->image_size <
                 (int64_t(1) << 31),
             "ns_unet_create: feature maps must stay below 2^31 floats");
  NS_REQUIRE(cfg->image_size >= 4 && cfg->image_size % 4 == 0,
             "ns_unet_create: image_size must be a positive multiple of 4");
  auto u = std::make_unique<ns_unet>();
  u->in_ch = cfg->in_channels;
  u->base = cfg->base_channels;
  u->S = cfg->image_size;
  u->max_batch = cfg->max_batch;
  const int b = u->base, S = u->S;
  const int c[5] = {b, 2 * b, 4 * b, 2 * b, b}, hw[5] = {S, S / 2, S / 4, S / 2, S};
  for (int l = 0; l < 5; ++l) u->lvl_c[l] = c[l], u->lvl_hw[l] = hw[l];
  // Parameters in registration order: conv_in, res0, ln0, down1, res1, ln1,
  // down2, res2, ln2, up1, res3, ln3, up0, res4, ln4, conv_out.
  const ns_unet::Conv lvl_conv[5] = {{u->in_ch, b, 1, S, 0, 0},   {b, 2 * b, 2, S, 0, 0},
                                     {2 * b, 4 * b, 2, S / 2, 0, 0}, {4 * b, 2 * b, 1, S / 2, 0, 0},
                                     {2 * b, b, 1, S, 0, 0}};
  u->conv.resize(11);
  int64_t off = 0;
  auto tensor = [&](int64_t n, int rank) {
    const int64_t o = off;
    u->offsets.push_back(off);
    u->ranks.push_back(rank);
    off += n;
    return o;
  };
  auto add_conv = [&](int idx, ns_unet::Conv cv) {
    cv.w_off = tensor((int64_t)cv.oc * cv.ic * 9, 4);
    cv.b_off = tensor(cv.oc, 1);
    u->conv[idx] = cv;
  };
  for (int l = 0; l < 5; ++l) {
    add_conv(l, lvl_conv[l]);
    add_conv(6 + l, {c[l], c[l], 1, hw[l], 0, 0});
    u->ln_off[l][0] = tensor(hw[l], 1);
    u->ln_off[l][1] = tensor(hw[l], 1);
  }
  add_conv(5, {b, u->in_ch, 1, S, 0, 0});
  u->offsets.push_back(off);
  u->n_params = off;
  const size_t Bm = (size_t)u->max_batch;
  size_t ws = 0;
  for (const auto& cv : u->conv)
    ws = std::max(ws, conv::keep_workspace_size((int)Bm, cv.ic, cv.in_hw, cv.in_hw, cv.oc, 3,
                                                cv.stride, 1));
  u->conv_ws_bytes = ws;
  size_t lnws = 0;
  for (int l = 0; l < 5; ++l)
    lnws = std::max(lnws, ns_layernorm_bwd_workspace_size((int)(Bm * c[l] * hw[l]), hw[l]));
  u->ln_ws_bytes = std::max<size_t>(lnws, 256);
  const size_t big = Bm * (size_t)std::max(4 * b * S * S / 4, b * S * S);  // largest feature map
  ns_status rc = NS_OK;
  auto A = [&](float** p, size_t n) {
    if (rc == NS_OK) rc = dev_alloc(u.get(), p, n);
  };
  A(&u->params, off);
  A(&u->grads, off);
  A(&u->m, off);
  A(&u->v, off);
  A(&u->hyper, 8);
  A(&u->x, Bm * u->in_ch * S * S);
  A(&u->out, Bm * u->in_ch * S * S);
  A(&u->dout, Bm * u->in_ch * S * S);
  for (int l = 0; l < 5; ++l) {
    const size_t n = Bm * c[l] * hw[l] * hw[l];
    A(&u->a[l], n);
    A(&u->r[l], n);
    A(&u->e[l], n);
    A(&u->mean[l], Bm * c[l] * hw[l]);
    A(&u->rstd[l], Bm * c[l] * hw[l]);
  }
  A(&u->up_a, Bm * 4 * b * (S / 2) * (S / 2));  // Up(m)
  A(&u->up_b, Bm * 2 * b * S * S);              // Up(u1)
  A(&u->t0, std::max(big, Bm * 2 * b * S * S));
  A(&u->t1, std::max(big, Bm * 2 * b * S * S));
  A(&u->t2, std::max(big, Bm * 2 * b * S * S));
  A(&u->g0, Bm * b * S * S);
  A(&u->g1, Bm * 2 * b * (S / 2) * (S / 2));
  A(&u->small, 64);
  A(&u->loss_part, kMseBlocks);
  for (auto& cv : u->conv) {
    const int64_t n = conv::cols_floats((int)Bm, cv.ic, cv.in_hw, cv.in_hw, cv.oc, 3, cv.stride, 1);
    A(&cv.cols, (size_t)n);
    A(&cv.cols_lo, (size_t)n);
  }
  if (rc == NS_OK) {
    void* p = nullptr;
    cudaError_t e = cudaMalloc(&p, ws);
    if (e != cudaSuccess) rc = cuda_fail(e, "ns_unet_create workspace");
    else u->allocs.push_back(p), u->conv_ws = p;
  }
  if (rc == NS_OK) {
    void* p = nullptr;
    cudaError_t e = cudaMalloc(&p, u->ln_ws_bytes);
    if (e != cudaSuccess) rc = cuda_fail(e, "ns_unet_create workspace");
    else u->allocs.push_back(p), u->ln_ws = p;
  }
  if (rc == NS_OK) {
    cudaError_t e = cudaMemset(u->grads, 0, off * sizeof(float));
    if (e == cudaSuccess) e = cudaMemset(u->small, 0, 64 * sizeof(float));
    if (e != cudaSuccess) rc = cuda_fail(e, "ns_unet_create");
  }
  if (rc != NS_OK) {
    free_all(u.get());
    return rc;
  }
  *out = u.release();
  return NS_OK;
}

ns_status ns_unet_destroy(ns_unet* u) {
  if (!u) return NS_OK;
  cudaDeviceSynchronize();
  free_all(u);
  delete u;
  return NS_OK;
}

int ns_unet_num_tensors(const ns_unet* u) { return u ? (int)u->ranks.size() : 0; }
int64_t ns_unet_tensor_numel(const ns_unet* u, int i) {
  return u && i >= 0 && i < (int)u->ranks.size() ? u->offsets[i + 1] - u->offsets[i] : 0;
}
int64_t ns_unet_num_params(const ns_unet* u) { return u ? u->n_params : 0; }
float* ns_unet_params(ns_unet* u) { return u ? u->params : nullptr; }
float* ns_unet_grads(ns_unet* u) { return u ? u->grads : nullptr; }
float* ns_unet_output(ns_unet* u) { return u ? u->out : nullptr; }
float* ns_unet_loss(ns_unet* u) { return u ? u->small : nullptr; }

ns_status ns_unet_forward(ns_unet* u, const float* x, int B, void* stream) {
  NS_REQUIRE(u && x, "ns_unet_forward: NULL argument");
  NS_REQUIRE(B >= 1 && B <= u->max_batch, "ns_unet_forward: B must be in [1, max_batch]");
  cudaStream_t s = as_stream(stream);
  u->B = B;
  const int S = u->S;
  NS_TRY_CUDA(cudaMemcpyAsync(u->x, x, (size_t)B * u->in_ch * S * S * sizeof(float),
                              cudaMemcpyDeviceToDevice, s),
              "ns_unet_forward input");
  ns_status rc = conv_fwd(u, 0, u->x, u->a[0], B, s);                    // conv_in
  if (rc == NS_OK) rc = res_ln_fwd(u, 0, B, s);                          // e0
  if (rc == NS_OK) rc = conv_fwd(u, 1, u->e[0], u->a[1], B, s);          // down1
  if (rc == NS_OK) rc = res_ln_fwd(u, 1, B, s);                          // e1
  if (rc == NS_OK) rc = conv_fwd(u, 2, u->e[1], u->a[2], B, s);          // down2
  if (rc == NS_OK) rc = res_ln_fwd(u, 2, B, s);                          // m
  if (rc != NS_OK) return rc;
  rc = launch_pdl(up2_k, dim3(grid_for(level_numel(u, 2, B))), dim3(256), 0, s, "ns_unet upsample",
                  u->e[2], (int)level_numel(u, 2, B), S / 4, u->up_a);
  if (rc == NS_OK) rc = conv_fwd(u, 3, u->up_a, u->t0, B, s);            // up1
  if (rc == NS_OK) rc = ns_add(u->t0, u->e[1], u->a[3], level_numel(u, 3, B), s);  // + e1
  if (rc == NS_OK) rc = res_ln_fwd(u, 3, B, s);                          // u1
  if (rc != NS_OK) return rc;
  rc = launch_pdl(up2_k, dim3(grid_for(level_numel(u, 3, B))), dim3(256), 0, s, "ns_unet upsample",
                  u->e[3], (int)level_numel(u, 3, B), S / 2, u->up_b);
  if (rc == NS_OK) rc = conv_fwd(u, 4, u->up_b, u->t0, B, s);            // up0
  if (rc == NS_OK) rc = ns_add(u->t0, u->e[0], u->a[4], level_numel(u, 4, B), s);  // + e0
  if (rc == NS_OK) rc = res_ln_fwd(u, 4, B, s);                          // u0
  if (rc == NS_OK) rc = conv_fwd(u, 5, u->e[4], u->out, B, s);           // conv_out
  return rc;
}

ns_status ns_unet_loss_backward(ns_unet* u, const float* target, void* stream) {
  NS_REQUIRE(u && target, "ns_unet_loss_backward: NULL argument");
  NS_REQUIRE(u->B > 0, "ns_unet_loss_backward: no forward pass yet");
  cudaStream_t s = as_stream(stream);
  const int64_t n = (int64_t)u->B * u->in_ch * u->S * u->S;
  ns_status rc = launch_pdl(mse_k, dim3(kMseBlocks), dim3(256), 0, s, "ns_unet mse", u->out,
                            target, n, (float)((double)n * u->world), u->dout, u->loss_part);
  if (rc != NS_OK) return rc;
  return launch_pdl(mse_finish_k, dim3(1), dim3(32), 0, s, "ns_unet mse finish", u->loss_part,
                    kMseBlocks, (float)n, u->small);
}

ns_status ns_unet_backward(ns_unet* u, void* stream) {
  NS_REQUIRE(u, "ns_unet_backward: NULL argument");
  NS_REQUIRE(u->B > 0, "ns_unet_backward: no forward pass yet");
  cudaStream_t s = as_stream(stream);
  const int B = u->B, S = u->S;
  // The skip sums' gradients live in g0 / g1 until the encoder side adds
  // them; the other gradients reuse the e[] slots of values the backward has
  // already consumed (u0 after conv_out, u1 and m after their upsamples).
  ns_status rc = conv_bwd(u, 5, u->e[4], u->dout, u->t0, B, s);                  // conv_out
  if (rc == NS_OK) rc = res_ln_bwd(u, 4, u->t0, u->g0, B, s);                    // ds0
  if (rc == NS_OK) rc = conv_bwd(u, 4, u->up_b, u->g0, u->t0, B, s);             // up0
  if (rc != NS_OK) return rc;
  rc = launch_pdl(up2_bwd_k, dim3(grid_for(level_numel(u, 3, B))), dim3(256), 0, s,
                  "ns_unet upsample backward", u->t0, (int)level_numel(u, 3, B), S / 2,
                  u->e[3]);  // du1
  if (rc == NS_OK) rc = res_ln_bwd(u, 3, u->e[3], u->g1, B, s);                  // ds1
  if (rc == NS_OK) rc = conv_bwd(u, 3, u->up_a, u->g1, u->t0, B, s);             // up1
  if (rc != NS_OK) return rc;
  rc = launch_pdl(up2_bwd_k, dim3(grid_for(level_numel(u, 2, B))), dim3(256), 0, s,
                  "ns_unet upsample backward", u->t0, (int)level_numel(u, 2, B), S / 4,
                  u->e[2]);  // dm
  if (rc == NS_OK) rc = res_ln_bwd(u, 2, u->e[2], u->t0, B, s);                  // d a2
  if (rc == NS_OK) rc = conv_bwd(u, 2, u->e[1], u->t0, u->t1, B, s);             // down2
  if (rc == NS_OK) rc = ns_add(u->t1, u->g1, u->e[3], level_numel(u, 1, B), s);    // de1
  if (rc == NS_OK) rc = res_ln_bwd(u, 1, u->e[3], u->t0, B, s);                  // d a1
  if (rc == NS_OK) rc = conv_bwd(u, 1, u->e[0], u->t0, u->t1, B, s);             // down1
  if (rc == NS_OK) rc = ns_add(u->t1, u->g0, u->e[4], level_numel(u, 0, B), s);    // de0
  if (rc == NS_OK) rc = res_ln_bwd(u, 0, u->e[4], u->t0, B, s);                  // d a0
  if (rc == NS_OK) rc = conv_bwd(u, 0, u->x, u->t0, nullptr, B, s);              // conv_in
  if (rc != NS_OK || !u->comm || u->world == 1) return rc;
  rc = comm::allreduce(u->comm, u->grads, u->n_params, s);
  if (rc == NS_OK) rc = comm::allreduce(u->comm, u->small, 1, s);
  return rc;
}

ns_status ns_unet_adamw_init(ns_unet* u, float lr, float b1, float b2, float eps, float wd) {
  NS_REQUIRE(u, "ns_unet_adamw_init: NULL argument");
  NS_TRY_CUDA(cudaMemset(u->m, 0, u->n_params * sizeof(float)), "ns_unet_adamw_init");
  NS_TRY_CUDA(cudaMemset(u->v, 0, u->n_params * sizeof(float)), "ns_unet_adamw_init");
  const float h[8] = {lr, b1, b2, eps, 1.0f, 1.0f, 0.0f, 0.0f};
  NS_TRY_CUDA(cudaMemcpy(u->hyper, h, sizeof(h), cudaMemcpyHostToDevice), "ns_unet_adamw_init");
  u->wd = wd;
  u->decay.clear();
  for (int r : u->ranks) u->decay.push_back(r >= 2 ? wd : 0.0f);
  u->opt = true;
  return NS_OK;
}

ns_status ns_unet_adamw_step(ns_unet* u, void* stream) {
  NS_REQUIRE(u && u->opt, "ns_unet_adamw_step: call ns_unet_adamw_init first");
  return ns_adamw_flat_device(u->params, u->grads, u->m, u->v, u->n_params, u->offsets.data(),
                              u->decay.data(), (int)u->decay.size(), u->hyper, stream);
}

ns_status ns_unet_train_step(ns_unet* u, const float* x, const float* target, int B,
                             float* host_loss, void* stream) {
  ns_status rc = ns_unet_forward(u, x, B, stream);
  if (rc == NS_OK) rc = ns_unet_loss_backward(u, target, stream);
  if (rc == NS_OK) rc = ns_unet_backward(u, stream);
  if (rc == NS_OK) rc = ns_unet_adamw_step(u, stream);
  if (rc != NS_OK || !host_loss) return rc;
  float l = 0.0f;
  NS_TRY_CUDA(cudaMemcpyAsync(&l, u->small, sizeof(float), cudaMemcpyDeviceToHost,
                              as_stream(stream)),
              "ns_unet loss");
  NS_TRY_CUDA(cudaStreamSynchronize(as_stream(stream)), "ns_unet loss");
  *host_loss = l / (float)u->world;
  return NS_OK;
}

ns_status ns_unet_set_comm(ns_unet* u, ns_comm* comm, int world_size) {
  NS_REQUIRE(u && world_size >= 1, "ns_unet_set_comm: bad arguments");
  u->comm = comm;
  u->world = comm ? world_size : 1;
  return NS_OK;
}

}  // extern "C"
