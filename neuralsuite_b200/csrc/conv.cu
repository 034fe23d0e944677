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
//
// Every data pass works on whole runs (the P positions of one image in one
// column row, channel or plane, contiguous on both sides), one CTA per run:
// 32-bit index arithmetic per element, 16-byte vectors where the sizes allow.
// A model can keep a forward's columns for its backward (conv.h) instead of
// rebuilding them.
#include <algorithm>
#include <string>

#include "common.cuh"
#include "conv.h"
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
// the padding), kk = (ic*k + kh)*k + kw, and its tf32 lo part.  A CTA fills
// whole column runs: run r = b*K + kk is the P entries of image b in row kk,
// contiguous in cols, so the index arithmetic per element is one add and the
// stores are coalesced (16-byte vectors when the rows allow).  Consecutive
// runs read the same input plane (the k*k taps of one channel).
__global__ void __launch_bounds__(256) im2col_k(const float* __restrict__ x, Shape sh,
                                                float* __restrict__ cols,
                                                float* __restrict__ cols_lo, int vec) {
  const int P = sh.OH * sh.OW, K = sh.IC * sh.k * sh.k, kk2 = sh.k * sh.k;
  const int64_t N = sh.N(), runs = (int64_t)K * sh.B;
  for (int64_t r = blockIdx.x; r < runs; r += gridDim.x) {
    const int b = (int)(r / K), kk = (int)(r - (int64_t)b * K);
    const int ic = kk / kk2, kr = kk - ic * kk2, kh = kr / sh.k, kw = kr - kh * sh.k;
    const float* xp = x + ((size_t)b * sh.IC + ic) * sh.H * sh.W;
    const int64_t o = (int64_t)kk * N + (int64_t)b * P;
    const int ih0 = kh - sh.p, iw0 = kw - sh.p;
    if (vec) {
      // P and OW multiples of 4: the 4 entries of a vector share a window row.
      for (int q = threadIdx.x * 4; q < P; q += blockDim.x * 4) {
        const int oh = q / sh.OW, ow = q - oh * sh.OW;
        const int ih = oh * sh.s + ih0;
        const bool row_in = ih >= 0 && ih < sh.H;
        const float* xr = xp + (size_t)ih * sh.W;
        float v[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int iw = (ow + j) * sh.s + iw0;
          v[j] = (row_in && iw >= 0 && iw < sh.W) ? __ldg(xr + iw) : 0.0f;
        }
        *reinterpret_cast<float4*>(cols + o + q) = make_float4(v[0], v[1], v[2], v[3]);
        if (cols_lo)
          *reinterpret_cast<float4*>(cols_lo + o + q) =
              make_float4(lo_of(v[0]), lo_of(v[1]), lo_of(v[2]), lo_of(v[3]));
      }
    } else {
      for (int q = threadIdx.x; q < P; q += blockDim.x) {
        const int oh = q / sh.OW, ow = q - oh * sh.OW;
        const int ih = oh * sh.s + ih0, iw = ow * sh.s + iw0;
        const float v = (ih >= 0 && ih < sh.H && iw >= 0 && iw < sh.W)
                            ? __ldg(xp + (size_t)ih * sh.W + iw)
                            : 0.0f;
        cols[o + q] = v;
        if (cols_lo) cols_lo[o + q] = lo_of(v);
      }
    }
  }
}

// y[b][oc][p] = yc[oc][b*P + p] + bias[oc] (the reference adds the bias after
// the product, conv2d.h:255-263).  Both sides of a (b, oc) pair are runs of P
// contiguous floats: one CTA per run.
__global__ void __launch_bounds__(256) cnhw_to_nchw_bias_k(const float* __restrict__ yc,
                                                           const float* __restrict__ bias,
                                                           Shape sh, float* __restrict__ y,
                                                           int vec) {
  const int P = sh.OH * sh.OW;
  const int64_t runs = (int64_t)sh.B * sh.OC;
  for (int64_t r = blockIdx.x; r < runs; r += gridDim.x) {
    const int b = (int)(r / sh.OC), oc = (int)(r - (int64_t)b * sh.OC);
    const float* src = yc + ((size_t)oc * sh.B + b) * P;
    float* dst = y + (size_t)r * P;
    const float bv = bias ? __ldg(bias + oc) : 0.0f;
    if (vec) {
      for (int q = threadIdx.x * 4; q < P; q += blockDim.x * 4) {
        float4 v = *reinterpret_cast<const float4*>(src + q);
        if (bias) v = make_float4(__fadd_rn(v.x, bv), __fadd_rn(v.y, bv), __fadd_rn(v.z, bv),
                                  __fadd_rn(v.w, bv));
        *reinterpret_cast<float4*>(dst + q) = v;
      }
    } else {
      for (int q = threadIdx.x; q < P; q += blockDim.x)
        dst[q] = bias ? __fadd_rn(src[q], bv) : src[q];
    }
  }
}

// dyc[oc][b*P + p] = dy[b][oc][p], and its tf32 lo part (one CTA per run).
__global__ void __launch_bounds__(256) nchw_to_cnhw_k(const float* __restrict__ dy, Shape sh,
                                                      float* __restrict__ dyc,
                                                      float* __restrict__ dyc_lo, int vec) {
  const int P = sh.OH * sh.OW;
  const int64_t runs = (int64_t)sh.B * sh.OC;
  for (int64_t r = blockIdx.x; r < runs; r += gridDim.x) {
    const int b = (int)(r / sh.OC), oc = (int)(r - (int64_t)b * sh.OC);
    const float* src = dy + (size_t)r * P;
    const size_t o = ((size_t)oc * sh.B + b) * P;
    if (vec) {
      for (int q = threadIdx.x * 4; q < P; q += blockDim.x * 4) {
        const float4 v = *reinterpret_cast<const float4*>(src + q);
        *reinterpret_cast<float4*>(dyc + o + q) = v;
        *reinterpret_cast<float4*>(dyc_lo + o + q) =
            make_float4(lo_of(v.x), lo_of(v.y), lo_of(v.z), lo_of(v.w));
      }
    } else {
      for (int q = threadIdx.x; q < P; q += blockDim.x) {
        const float v = src[q];
        dyc[o + q] = v;
        dyc_lo[o + q] = lo_of(v);
      }
    }
  }
}

// part[oc * B + b] = sum over positions of dy[b][oc][:], a fixed-order tree
// (one CTA per image and channel; blockDim 256).
__global__ void __launch_bounds__(256) bias_part_k(const float* __restrict__ dy, Shape sh,
                                                   float* __restrict__ part) {
  __shared__ float red[256];
  const int oc = blockIdx.x, b = blockIdx.y;
  const int64_t P = sh.P();
  const float* row = dy + ((size_t)b * sh.OC + oc) * P;
  float s = 0.0f;
  for (int64_t i = threadIdx.x; i < P; i += blockDim.x) s += row[i];
  red[threadIdx.x] = s;
  __syncthreads();
  for (int w = blockDim.x / 2; w > 0; w >>= 1) {
    if ((int)threadIdx.x < w) red[threadIdx.x] += red[threadIdx.x + w];
    __syncthreads();
  }
  if (threadIdx.x == 0) part[(size_t)oc * sh.B + b] = red[0];
}

// db[oc] = the per-image sums added in image order (conv2d.h:326-331).
__global__ void bias_finish_k(const float* __restrict__ part, int OC, int B,
                              float* __restrict__ db) {
  const int oc = blockIdx.x * blockDim.x + threadIdx.x;
  if (oc >= OC) return;
  float total = 0.0f;
  for (int b = 0; b < B; ++b) total += part[(size_t)oc * B + b];
  db[oc] = total;
}

// dx[b][ic][ih][iw] = sum over (kh, kw), in that order, of the column entry
// of every window that covers the pixel: dcols[(ic*k + kh)*k + kw][b*P + oh*OW + ow]
// with oh*s + kh - p = ih and ow*s + kw - p = iw.  One CTA per input plane
// (b, ic); neighbouring threads take neighbouring pixels, so each (kh, kw)
// term is a coalesced read of one column row.
__global__ void __launch_bounds__(256) col2im_k(const float* __restrict__ dcols, Shape sh,
                                                float* __restrict__ dx) {
  const int HW = sh.H * sh.W, P = sh.OH * sh.OW;
  const int64_t N = sh.N(), planes = (int64_t)sh.B * sh.IC;
  for (int64_t r = blockIdx.x; r < planes; r += gridDim.x) {
    const int b = (int)(r / sh.IC), ic = (int)(r - (int64_t)b * sh.IC);
    const float* base = dcols + (int64_t)ic * sh.k * sh.k * N + (int64_t)b * P;
    float* out = dx + (size_t)r * HW;
    for (int pix = threadIdx.x; pix < HW; pix += blockDim.x) {
      const int ih = pix / sh.W, iw = pix - ih * sh.W;
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
          acc += __ldg(base + (int64_t)(kh * sh.k + kw) * N + oh * sh.OW + ow);
        }
      }
      out[pix] = acc;
    }
  }
}

// CTAs for a pass over `runs` independent runs (a few waves of 256 threads).
// col2im_k for a k x k window at a fixed stride: every tap's load is issued
// before the sum (taps outside the output read 0.0f, which leaves a sum that
// starts at +0.0f unchanged), and the stride divisions are shifts.  Same sums
// in the same order as col2im_k.
template <int KS, int ST>
__global__ void __launch_bounds__(256) col2im_fixed_k(const float* __restrict__ dcols, Shape sh,
                                                      float* __restrict__ dx) {
  const int HW = sh.H * sh.W, P = sh.OH * sh.OW;
  const int64_t N = sh.N(), planes = (int64_t)sh.B * sh.IC;
  for (int64_t r = blockIdx.x; r < planes; r += gridDim.x) {
    const int b = (int)(r / sh.IC), ic = (int)(r - (int64_t)b * sh.IC);
    const float* base = dcols + (int64_t)ic * KS * KS * N + (int64_t)b * P;
    float* out = dx + (size_t)r * HW;
    for (int pix = threadIdx.x; pix < HW; pix += blockDim.x) {
      const int ih = pix / sh.W, iw = pix - ih * sh.W;
      float v[KS * KS];
#pragma unroll
      for (int kh = 0; kh < KS; ++kh) {
        const int th = ih + sh.p - kh;
        const int oh = th / ST;
        const bool hok = th >= 0 && th % ST == 0 && oh < sh.OH;
#pragma unroll
        for (int kw = 0; kw < KS; ++kw) {
          const int tw = iw + sh.p - kw;
          const int ow = tw / ST;
          const bool ok = hok && tw >= 0 && tw % ST == 0 && ow < sh.OW;
          v[kh * KS + kw] = ok ? __ldg(base + (int64_t)(kh * KS + kw) * N + oh * sh.OW + ow) : 0.0f;
        }
      }
      float acc = 0.0f;
#pragma unroll
      for (int t = 0; t < KS * KS; ++t) acc += v[t];
      out[pix] = acc;
    }
  }
}

int grid_runs(int64_t runs) {
  return (int)std::max<int64_t>(1, std::min<int64_t>(runs, (int64_t)sm_count() * 32));
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

ns_status make_shape(int B, int IC, int H, int W, int OC, int k, int stride, int pad, Shape* sh) {
  if (B < 0 || IC <= 0 || H <= 0 || W <= 0 || OC <= 0 || k <= 0 || stride <= 0 || pad < 0)
    return fail(NS_ERR_INVALID_ARGUMENT, "ns_conv2d: bad convolution parameters");
  const int OH = (H + 2 * pad - k) / stride + 1, OW = (W + 2 * pad - k) / stride + 1;
  if (H + 2 * pad < k || W + 2 * pad < k || OH <= 0 || OW <= 0)
    return fail(NS_ERR_INVALID_ARGUMENT, "ns_conv2d: the kernel does not fit the input");
  *sh = Shape{B, IC, H, W, OC, k, stride, pad, OH, OW};
  if (sh->K() * sh->N() >= (int64_t(1) << 31) || (int64_t)OC * sh->N() >= (int64_t(1) << 31) ||
      (int64_t)B * IC * H * W >= (int64_t(1) << 31) || B > 65535)
    return fail(NS_ERR_INVALID_ARGUMENT, "ns_conv2d: columns exceed 2^31 elements (split the batch)");
  return NS_OK;
}

// Workspace layout (floats, each piece 64-float aligned): [cols, cols_lo]
// (only when the columns live in the workspace), w_lo, yc | dyc, dyc_lo,
// dcols, the bias partials, then the GEMM workspace.
struct Ws {
  float *cols, *cols_lo, *w_lo, *yc, *dyc, *dyc_lo, *dcols, *bias_part;
  void* gemm;
  size_t gemm_bytes, total;
};
size_t al64(size_t n) { return (n + 63) & ~size_t(63); }

// A pre-split lo operand is usable when its stored rows are whole 16-byte
// units (`width` floats a multiple of 4); otherwise the GEMM splits the
// operand itself (or runs its SIMT path when TMA cannot read the rows).
const float* lo_if(const float* lo, int64_t width) { return width % 4 == 0 ? lo : nullptr; }
Ws layout(const Shape& sh, void* base, bool with_cols) {
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
  if (with_cols) {
    w.cols = take(KN);
    w.cols_lo = take(KN);
  }
  w.w_lo = take(WK);
  w.yc = take(ON);
  w.dyc = take(ON);
  w.dyc_lo = take(ON);
  w.dcols = take(KN);
  w.bias_part = take(al64((size_t)sh.OC * std::max(sh.B, 1)));
  const int M = sh.OC, N = (int)sh.N(), K = (int)sh.K();
  w.gemm_bytes = std::max({ns_gemm_workspace_size(M, N, K), ns_gemm_workspace_size(M, K, N),
                           ns_gemm_workspace_size(K, N, M)});
  w.gemm = f ? static_cast<void*>(f + off) : nullptr;
  w.total = off * sizeof(float) + w.gemm_bytes;
  return w;
}

ns_status check_ws(const Shape& sh, void* workspace, size_t workspace_bytes, bool with_cols,
                   const char* who, Ws* out) {
  if ((reinterpret_cast<uintptr_t>(workspace) & 255) != 0)
    return fail(NS_ERR_INVALID_ARGUMENT, std::string(who) + ": workspace must be 256-byte aligned");
  *out = layout(sh, workspace, with_cols);
  if (!workspace || workspace_bytes < out->total)
    return fail(NS_ERR_INVALID_ARGUMENT,
                std::string(who) + ": workspace smaller than the size its query returns");
  return NS_OK;
}

ns_status launch_im2col(const float* x, const Shape& sh, float* cols, float* cols_lo,
                        cudaStream_t s) {
  const int vec = (sh.P() % 4 == 0 && sh.OW % 4 == 0 && aligned16(cols) &&
                   (!cols_lo || aligned16(cols_lo))) ? 1 : 0;
  im2col_k<<<grid_runs(sh.K() * sh.B), 256, 0, s>>>(x, sh, cols, cols_lo, vec);
  return check_launch("ns_conv2d im2col");
}

// The forward once the columns are in place: Yc = W . cols, then NCHW + bias.
ns_status forward_body(const Shape& sh, const float* weight, const float* bias, float* y,
                       const float* cols, const float* cols_lo, const Ws& ws, cudaStream_t s) {
  const int M = sh.OC, N = (int)sh.N(), K = (int)sh.K();
  ns_status rc = ns_split_lo(weight, M, K, K, ws.w_lo, s);
  if (rc != NS_OK) return rc;
  // Yc[OC, B*P] = W[OC, K] . cols[K, B*P]
  rc = ns_gemm_lo(M, N, K, weight, K, 0, lo_if(ws.w_lo, K), cols, N, 0, lo_if(cols_lo, N), ws.yc,
                  N, 0.0f, NS_EPI_STORE, nullptr, nullptr, nullptr, ws.gemm, ws.gemm_bytes, s);
  if (rc != NS_OK) return rc;
  const int vec = (sh.P() % 4 == 0 && aligned16(ws.yc) && aligned16(y)) ? 1 : 0;
  cnhw_to_nchw_bias_k<<<grid_runs((int64_t)sh.B * sh.OC), 256, 0, s>>>(ws.yc, bias, sh, y, vec);
  return check_launch("ns_conv2d_fwd layout");
}

// The backward once the columns are in place.
ns_status backward_body(const Shape& sh, const float* cols, const float* cols_lo, const float* dy,
                        const float* weight, float* dx, float* dweight, float* dbias, const Ws& ws,
                        cudaStream_t s) {
  const int M = sh.OC, N = (int)sh.N(), K = (int)sh.K();
  const int vec = (sh.P() % 4 == 0 && aligned16(dy) && aligned16(ws.dyc) && aligned16(ws.dyc_lo))
                      ? 1 : 0;
  nchw_to_cnhw_k<<<grid_runs((int64_t)sh.B * sh.OC), 256, 0, s>>>(dy, sh, ws.dyc, ws.dyc_lo, vec);
  ns_status rc = check_launch("ns_conv2d_bwd layout");
  if (rc != NS_OK) return rc;
  bias_part_k<<<dim3(sh.OC, sh.B), 256, 0, s>>>(dy, sh, ws.bias_part);
  rc = check_launch("ns_conv2d_bwd bias");
  if (rc != NS_OK) return rc;
  bias_finish_k<<<ceil_div(sh.OC, 128), 128, 0, s>>>(ws.bias_part, sh.OC, sh.B, dbias);
  rc = check_launch("ns_conv2d_bwd bias");
  if (rc != NS_OK) return rc;
  // dW[OC, K] = dYc[OC, B*P] . cols[K, B*P]^T (overwritten, as the reference zeroes it first)
  rc = ns_gemm_lo(M, K, N, ws.dyc, N, 0, lo_if(ws.dyc_lo, N), cols, N, 1, lo_if(cols_lo, N),
                  dweight, K, 0.0f, NS_EPI_STORE, nullptr, nullptr, nullptr, ws.gemm,
                  ws.gemm_bytes, s);
  if (rc != NS_OK || !dx) return rc;
  rc = ns_split_lo(weight, M, K, K, ws.w_lo, s);
  if (rc != NS_OK) return rc;
  // dcols[K, B*P] = W[OC, K]^T . dYc[OC, B*P]
  rc = ns_gemm_lo(K, N, M, weight, K, 1, lo_if(ws.w_lo, K), ws.dyc, N, 0, lo_if(ws.dyc_lo, N),
                  ws.dcols, N, 0.0f, NS_EPI_STORE, nullptr, nullptr, nullptr, ws.gemm,
                  ws.gemm_bytes, s);
  if (rc != NS_OK) return rc;
  const int g = grid_runs((int64_t)sh.B * sh.IC);
  if (sh.k == 3 && sh.s == 1)
    col2im_fixed_k<3, 1><<<g, 256, 0, s>>>(ws.dcols, sh, dx);
  else if (sh.k == 3 && sh.s == 2)
    col2im_fixed_k<3, 2><<<g, 256, 0, s>>>(ws.dcols, sh, dx);
  else
    col2im_k<<<g, 256, 0, s>>>(ws.dcols, sh, dx);
  return check_launch("ns_conv2d_bwd col2im");
}

ns_status zero_grads(const Shape& sh, float* dweight, float* dbias, cudaStream_t s) {
  NS_TRY_CUDA(cudaMemsetAsync(dweight, 0, (size_t)sh.OC * sh.K() * sizeof(float), s),
              "ns_conv2d_bwd");
  NS_TRY_CUDA(cudaMemsetAsync(dbias, 0, (size_t)sh.OC * sizeof(float), s), "ns_conv2d_bwd");
  return NS_OK;
}

}  // namespace

int64_t cols_floats(int B, int IC, int H, int W, int OC, int k, int stride, int pad) {
  Shape sh;
  if (make_shape(B, IC, H, W, OC, k, stride, pad, &sh) != NS_OK) return 0;
  return sh.K() * sh.N();
}

size_t keep_workspace_size(int B, int IC, int H, int W, int OC, int k, int stride, int pad) {
  Shape sh;
  if (make_shape(B, IC, H, W, OC, k, stride, pad, &sh) != NS_OK) return 0;
  return layout(sh, nullptr, false).total;
}

ns_status forward_keep(const float* x, int B, int IC, int H, int W, const float* weight,
                       const float* bias, int OC, int k, int stride, int pad, float* y,
                       float* cols, float* cols_lo, void* workspace, size_t workspace_bytes,
                       cudaStream_t s) {
  Shape sh;
  ns_status rc = make_shape(B, IC, H, W, OC, k, stride, pad, &sh);
  if (rc != NS_OK || B == 0) return rc;
  NS_REQUIRE(x && weight && y && cols && cols_lo, "conv forward: NULL argument");
  Ws ws;
  rc = check_ws(sh, workspace, workspace_bytes, false, "conv forward", &ws);
  if (rc != NS_OK) return rc;
  rc = launch_im2col(x, sh, cols, cols_lo, s);
  if (rc != NS_OK) return rc;
  return forward_body(sh, weight, bias, y, cols, cols_lo, ws, s);
}

ns_status backward_from_cols(const float* cols, const float* cols_lo, const float* dy, int B,
                             int IC, int H, int W, const float* weight, int OC, int k, int stride,
                             int pad, float* dx, float* dweight, float* dbias, void* workspace,
                             size_t workspace_bytes, cudaStream_t s) {
  Shape sh;
  ns_status rc = make_shape(B, IC, H, W, OC, k, stride, pad, &sh);
  if (rc != NS_OK) return rc;
  NS_REQUIRE(cols && cols_lo && dy && weight && dweight && dbias, "conv backward: NULL argument");
  if (B == 0) return zero_grads(sh, dweight, dbias, s);
  Ws ws;
  rc = check_ws(sh, workspace, workspace_bytes, false, "conv backward", &ws);
  if (rc != NS_OK) return rc;
  return backward_body(sh, cols, cols_lo, dy, weight, dx, dweight, dbias, ws, s);
}

}  // namespace conv
}  // namespace nsb

using namespace nsb;
using namespace nsb::conv;

extern "C" {

size_t ns_conv2d_workspace_size(int B, int IC, int H, int W, int OC, int k, int stride, int pad) {
  Shape sh;
  if (make_shape(B, IC, H, W, OC, k, stride, pad, &sh) != NS_OK) return 0;
  return layout(sh, nullptr, true).total;
}

ns_status ns_conv2d_fwd(const float* x, int B, int IC, int H, int W, const float* weight,
                        const float* bias, int OC, int k, int stride, int pad, float* y,
                        void* workspace, size_t workspace_bytes, void* stream) {
  Shape sh;
  ns_status rc = make_shape(B, IC, H, W, OC, k, stride, pad, &sh);
  if (rc != NS_OK) return rc;
  if (B == 0) return NS_OK;
  NS_REQUIRE(x && weight && y, "ns_conv2d_fwd: NULL argument");
  Ws ws;
  rc = check_ws(sh, workspace, workspace_bytes, true, "ns_conv2d_fwd", &ws);
  if (rc != NS_OK) return rc;
  cudaStream_t s = as_stream(stream);
  rc = launch_im2col(x, sh, ws.cols, ws.cols_lo, s);
  if (rc != NS_OK) return rc;
  return forward_body(sh, weight, bias, y, ws.cols, ws.cols_lo, ws, s);
}

ns_status ns_conv2d_bwd(const float* x, const float* dy, int B, int IC, int H, int W,
                        const float* weight, int OC, int k, int stride, int pad, float* dx,
                        float* dweight, float* dbias, void* workspace, size_t workspace_bytes,
                        void* stream) {
  Shape sh;
  ns_status rc = make_shape(B, IC, H, W, OC, k, stride, pad, &sh);
  if (rc != NS_OK) return rc;
  NS_REQUIRE(x && dy && weight && dweight && dbias, "ns_conv2d_bwd: NULL argument");
  cudaStream_t s = as_stream(stream);
  if (B == 0) return zero_grads(sh, dweight, dbias, s);
  Ws ws;
  rc = check_ws(sh, workspace, workspace_bytes, true, "ns_conv2d_bwd", &ws);
  if (rc != NS_OK) return rc;
  rc = launch_im2col(x, sh, ws.cols, ws.cols_lo, s);
  if (rc != NS_OK) return rc;
  return backward_body(sh, ws.cols, ws.cols_lo, dy, weight, dx, dweight, dbias, ws, s);
}

}  // extern "C"
