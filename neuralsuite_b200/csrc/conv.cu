// Conv2D forward and backward (include/layers/conv2d.h:192-414) on the
// tcgen05 GEMM.
//
// The reference lowers each image to columns [IC*k*k, OH*OW] (Im2Col,
// conv2d.h:348-375) and multiplies per image.  Here the whole batch is one
// product: the columns of all images sit side by side, cols[K, B*P] with
// K = IC*k*k and P = OH*OW (column b*P + p is window p of image b), so each
// convolution is one 3xTF32 tensor-core GEMM of B*P columns:
//   forward   Yc[OC, B*P]  = W[OC, K] . cols                (then to NCHW + bias)
//   backward  dW[OC, K]    = dYc[OC, B*P] . cols^T          (split-K, ordered)
//             dcols[K, B*P] = W^T . dYc                    (then col2im to dx)
//             db[oc]       = sum over images (in order) of sum over positions
// where Yc / dYc are the outputs / output gradients in [OC, B, P] order (a
// permute of NCHW).  The column pass writes the columns and their tf32 lo
// parts together (the GEMM's pre-split operand) with coalesced reads and
// writes along the positions.  col2im gathers: each input pixel sums its
// windows' contributions in the reference's (kh, kw) order (conv2d.h:378-403),
// so there are no atomics and the result is deterministic.
#include <algorithm>

#include "common.cuh"
#include "ns_b200.h"

namespace nsb {
namespace conv {
namespace {

struct Shape {
  int B, IC, H, W, OC, k, s, p, OH, OW;
  __host__ __device__ int64_t P() const { return (int64_t)OH * OW; }
  __host__ __device__ int64_t K() const { return (int64_t)IC * k * k; }
  __host__ __device__ int64_t N() const { return (int64_t)B * P(); }
};

__device__ __forceinline__ float lo_of(float x) {
  return x - __uint_as_float(__float_as_uint(x) & 0xFFFFE000u);
}

// cols[kk][b*P + oh*OW + ow] = x[b][ic][oh*s + kh - p][ow*s + kw - p] (0 in
// the padding), kk = (ic*k + kh)*k + kw, and its tf32 lo part.
__global__ void im2col_k(const float* __restrict__ x, Shape sh, float* __restrict__ cols,
                         float* __restrict__ cols_lo) {
  const int64_t N = sh.N(), total = sh.K() * N;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t kk = i / N, n = i % N;
    const int kw = (int)(kk % sh.k), kh = (int)((kk / sh.k) % sh.k), ic = (int)(kk / (sh.k * sh.k));
    const int b = (int)(n / sh.P());
    const int pp = (int)(n % sh.P());
    const int oh = pp / sh.OW, ow = pp % sh.OW;
    const int ih = oh * sh.s + kh - sh.p, iw = ow * sh.s + kw - sh.p;
    const float v = (ih >= 0 && ih < sh.H && iw >= 0 && iw < sh.W)
                        ? x[(((size_t)b * sh.IC + ic) * sh.H + ih) * sh.W + iw]
                        : 0.0f;
    cols[i] = v;
    if (cols_lo) cols_lo[i] = lo_of(v);
  }
}

// y[b][oc][p] = yc[oc][b*P + p] + bias[oc] (the reference adds the bias after
// the product, conv2d.h:255-263).
__global__ void cnhw_to_nchw_bias_k(const float* __restrict__ yc, const float* __restrict__ bias,
                                    Shape sh, float* __restrict__ y) {
  const int64_t P = sh.P(), total = (int64_t)sh.B * sh.OC * P;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t p = i % P;
    const int oc = (int)((i / P) % sh.OC), b = (int)(i / (P * sh.OC));
    const float v = yc[((size_t)oc * sh.B + b) * P + p];
    y[i] = bias ? __fadd_rn(v, bias[oc]) : v;
  }
}

// dyc[oc][b*P + p] = dy[b][oc][p], and its tf32 lo part.
__global__ void nchw_to_cnhw_k(const float* __restrict__ dy, Shape sh, float* __restrict__ dyc,
                               float* __restrict__ dyc_lo) {
  const int64_t P = sh.P(), total = (int64_t)sh.B * sh.OC * P;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t p = i % P;
    const int b = (int)((i / P) % sh.B), oc = (int)(i / (P * sh.B));
    const float v = dy[((size_t)b * sh.OC + oc) * P + p];
    dyc[i] = v;
    dyc_lo[i] = lo_of(v);
  }
}

// db[oc] = sum over images b in order of (sum over positions of dy[b][oc][:]):
// one CTA per output channel; each image's sum is a fixed-order tree.
__global__ void bias_grad_k(const float* __restrict__ dy, Shape sh, float* __restrict__ db) {
  __shared__ float red[256];
  const int oc = blockIdx.x;
  const int64_t P = sh.P();
  float total = 0.0f;
  for (int b = 0; b < sh.B; ++b) {
    const float* row = dy + ((size_t)b * sh.OC + oc) * P;
    float s = 0.0f;
    for (int64_t i = threadIdx.x; i < P; i += blockDim.x) s += row[i];
    red[threadIdx.x] = s;
    __syncthreads();
    for (int w = blockDim.x / 2; w > 0; w >>= 1) {
      if ((int)threadIdx.x < w) red[threadIdx.x] += red[threadIdx.x + w];
      __syncthreads();
    }
    if (threadIdx.x == 0) total += red[0];
    __syncthreads();
  }
  if (threadIdx.x == 0) db[oc] = total;
}

// dx[b][ic][ih][iw] = sum over (kh, kw), in that order, of the column entry
// of every window that covers the pixel: dcols[(ic*k + kh)*k + kw][b*P + oh*OW + ow]
// with oh*s + kh - p = ih and ow*s + kw - p = iw.
__global__ void col2im_k(const float* __restrict__ dcols, Shape sh, float* __restrict__ dx) {
  const int64_t total = (int64_t)sh.B * sh.IC * sh.H * sh.W;
  const int64_t N = sh.N(), P = sh.P();
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int iw = (int)(i % sh.W), ih = (int)((i / sh.W) % sh.H);
    const int ic = (int)((i / ((int64_t)sh.W * sh.H)) % sh.IC);
    const int b = (int)(i / ((int64_t)sh.W * sh.H * sh.IC));
    float acc = 0.0f;
    for (int kh = 0; kh < sh.k; ++kh) {
      const int th = ih + sh.p - kh;
      if (th < 0 || th % sh.s != 0) continue;
      const int oh = th / sh.s;
      if (oh >= sh.OH) continue;
      for (int kw = 0; kw < sh.k; ++kw) {
        const int tw = iw + sh.p - kw;
        if (tw < 0 || tw % sh.s != 0) continue;
        const int ow = tw / sh.s;
        if (ow >= sh.OW) continue;
        const int64_t kk = ((int64_t)ic * sh.k + kh) * sh.k + kw;
        acc += dcols[kk * N + (int64_t)b * P + (int64_t)oh * sh.OW + ow];
      }
    }
    dx[i] = acc;
  }
}

int grid_for(int64_t work) {
  return (int)std::max<int64_t>(1, std::min<int64_t>((work + 255) / 256, (int64_t)sm_count() * 8));
}

ns_status make_shape(int B, int IC, int H, int W, int OC, int k, int stride, int pad, Shape* sh) {
  if (B < 0 || IC <= 0 || H <= 0 || W <= 0 || OC <= 0 || k <= 0 || stride <= 0 || pad < 0)
    return fail(NS_ERR_INVALID_ARGUMENT, "ns_conv2d: bad convolution parameters");
  const int OH = (H + 2 * pad - k) / stride + 1, OW = (W + 2 * pad - k) / stride + 1;
  if (H + 2 * pad < k || W + 2 * pad < k || OH <= 0 || OW <= 0)
    return fail(NS_ERR_INVALID_ARGUMENT, "ns_conv2d: the kernel does not fit the input");
  *sh = Shape{B, IC, H, W, OC, k, stride, pad, OH, OW};
  if (sh->K() * sh->N() >= (int64_t(1) << 31) || (int64_t)OC * sh->N() >= (int64_t(1) << 31))
    return fail(NS_ERR_INVALID_ARGUMENT, "ns_conv2d: columns exceed 2^31 elements (split the batch)");
  return NS_OK;
}

// Workspace layout (floats, each piece 64-float aligned): cols, cols_lo,
// w_lo, yc | dyc, dyc_lo, dcols, then the GEMM workspace.
struct Ws {
  float *cols, *cols_lo, *w_lo, *yc, *dyc, *dyc_lo, *dcols;
  void* gemm;
  size_t gemm_bytes, total;
};
size_t al64(size_t n) { return (n + 63) & ~size_t(63); }

// A pre-split lo operand is usable when its stored rows are whole 16-byte
// units (`width` floats a multiple of 4); otherwise the GEMM splits the
// operand itself (or runs its SIMT path when TMA cannot read the rows).
const float* lo_if(const float* lo, int64_t width) { return width % 4 == 0 ? lo : nullptr; }
Ws layout(const Shape& sh, void* base) {
  const size_t KN = al64((size_t)(sh.K() * sh.N())), ON = al64((size_t)sh.OC * sh.N());
  const size_t WK = al64((size_t)sh.OC * sh.K());
  Ws w{};
  float* f = static_cast<float*>(base);
  size_t off = 0;
  auto take = [&](size_t n) {
    float* p = f ? f + off : nullptr;
    off += n;
    return p;
  };
  w.cols = take(KN);
  w.cols_lo = take(KN);
  w.w_lo = take(WK);
  w.yc = take(ON);
  w.dyc = take(ON);
  w.dyc_lo = take(ON);
  w.dcols = take(KN);
  const int M = sh.OC, N = (int)sh.N(), K = (int)sh.K();
  w.gemm_bytes = std::max({ns_gemm_workspace_size(M, N, K), ns_gemm_workspace_size(M, K, N),
                           ns_gemm_workspace_size(K, N, M)});
  w.gemm = f ? static_cast<void*>(f + off) : nullptr;
  w.total = off * sizeof(float) + w.gemm_bytes;
  return w;
}

}  // namespace
}  // namespace conv
}  // namespace nsb

using namespace nsb;
using namespace nsb::conv;

extern "C" {

size_t ns_conv2d_workspace_size(int B, int IC, int H, int W, int OC, int k, int stride, int pad) {
  Shape sh;
  if (make_shape(B, IC, H, W, OC, k, stride, pad, &sh) != NS_OK) return 0;
  return layout(sh, nullptr).total;
}

ns_status ns_conv2d_fwd(const float* x, int B, int IC, int H, int W, const float* weight,
                        const float* bias, int OC, int k, int stride, int pad, float* y,
                        void* workspace, size_t workspace_bytes, void* stream) {
  Shape sh;
  ns_status rc = make_shape(B, IC, H, W, OC, k, stride, pad, &sh);
  if (rc != NS_OK) return rc;
  if (B == 0) return NS_OK;
  NS_REQUIRE(x && weight && y, "ns_conv2d_fwd: NULL argument");
  NS_REQUIRE((reinterpret_cast<uintptr_t>(workspace) & 255) == 0,
             "ns_conv2d_fwd: workspace must be 256-byte aligned");
  Ws ws = layout(sh, workspace);
  NS_REQUIRE(workspace && workspace_bytes >= ws.total,
             "ns_conv2d_fwd: workspace smaller than ns_conv2d_workspace_size");
  cudaStream_t s = as_stream(stream);
  const int M = OC, N = (int)sh.N(), K = (int)sh.K();
  im2col_k<<<grid_for(sh.K() * sh.N()), 256, 0, s>>>(x, sh, ws.cols, ws.cols_lo);
  rc = check_launch("ns_conv2d_fwd im2col");
  if (rc != NS_OK) return rc;
  rc = ns_split_lo(weight, OC, K, K, ws.w_lo, stream);
  if (rc != NS_OK) return rc;
  // Yc[OC, B*P] = W[OC, K] . cols[K, B*P]
  rc = ns_gemm_lo(M, N, K, weight, K, 0, lo_if(ws.w_lo, K), ws.cols, N, 0, lo_if(ws.cols_lo, N),
                  ws.yc, N, 0.0f,
                  NS_EPI_STORE, nullptr, nullptr, nullptr, ws.gemm, ws.gemm_bytes, stream);
  if (rc != NS_OK) return rc;
  cnhw_to_nchw_bias_k<<<grid_for((int64_t)OC * N), 256, 0, s>>>(ws.yc, bias, sh, y);
  return check_launch("ns_conv2d_fwd layout");
}

ns_status ns_conv2d_bwd(const float* x, const float* dy, int B, int IC, int H, int W,
                        const float* weight, int OC, int k, int stride, int pad, float* dx,
                        float* dweight, float* dbias, void* workspace, size_t workspace_bytes,
                        void* stream) {
  Shape sh;
  ns_status rc = make_shape(B, IC, H, W, OC, k, stride, pad, &sh);
  if (rc != NS_OK) return rc;
  NS_REQUIRE(x && dy && weight && dweight && dbias, "ns_conv2d_bwd: NULL argument");
  NS_REQUIRE((reinterpret_cast<uintptr_t>(workspace) & 255) == 0,
             "ns_conv2d_bwd: workspace must be 256-byte aligned");
  Ws ws = layout(sh, workspace);
  NS_REQUIRE(workspace && workspace_bytes >= ws.total,
             "ns_conv2d_bwd: workspace smaller than ns_conv2d_workspace_size");
  cudaStream_t s = as_stream(stream);
  const int M = OC, N = (int)sh.N(), K = (int)sh.K();
  if (B == 0) {
    NS_TRY_CUDA(cudaMemsetAsync(dweight, 0, (size_t)OC * K * sizeof(float), s), "ns_conv2d_bwd");
    NS_TRY_CUDA(cudaMemsetAsync(dbias, 0, (size_t)OC * sizeof(float), s), "ns_conv2d_bwd");
    return NS_OK;
  }
  im2col_k<<<grid_for(sh.K() * sh.N()), 256, 0, s>>>(x, sh, ws.cols, ws.cols_lo);
  rc = check_launch("ns_conv2d_bwd im2col");
  if (rc != NS_OK) return rc;
  nchw_to_cnhw_k<<<grid_for((int64_t)OC * N), 256, 0, s>>>(dy, sh, ws.dyc, ws.dyc_lo);
  rc = check_launch("ns_conv2d_bwd layout");
  if (rc != NS_OK) return rc;
  bias_grad_k<<<OC, 256, 0, s>>>(dy, sh, dbias);
  rc = check_launch("ns_conv2d_bwd bias");
  if (rc != NS_OK) return rc;
  // dW[OC, K] = dYc[OC, B*P] . cols[K, B*P]^T (overwritten, as the reference zeroes it first)
  rc = ns_gemm_lo(M, K, N, ws.dyc, N, 0, lo_if(ws.dyc_lo, N), ws.cols, N, 1,
                  lo_if(ws.cols_lo, N), dweight, K, 0.0f,
                  NS_EPI_STORE, nullptr, nullptr, nullptr, ws.gemm, ws.gemm_bytes, stream);
  if (rc != NS_OK || !dx) return rc;
  rc = ns_split_lo(weight, OC, K, K, ws.w_lo, stream);
  if (rc != NS_OK) return rc;
  // dcols[K, B*P] = W[OC, K]^T . dYc[OC, B*P]
  rc = ns_gemm_lo(K, N, M, weight, K, 1, lo_if(ws.w_lo, K), ws.dyc, N, 0, lo_if(ws.dyc_lo, N),
                  ws.dcols, N, 0.0f,
                  NS_EPI_STORE, nullptr, nullptr, nullptr, ws.gemm, ws.gemm_bytes, stream);
  if (rc != NS_OK) return rc;
  col2im_k<<<grid_for((int64_t)B * IC * H * W), 256, 0, s>>>(ws.dcols, sh, dx);
  return check_launch("ns_conv2d_bwd col2im");
}

}  // extern "C"
