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
  pdl_wait();     // the previous kernel's writes are visible (launched by launch_pdl)
  pdl_trigger();  // the next kernel, if launched as a programmatic dependent, may start
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
  pdl_wait();     // the previous kernel's writes are visible (launched by launch_pdl)
  pdl_trigger();  // the next kernel, if launched as a programmatic dependent, may start
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
  pdl_wait();     // the previous kernel's writes are visible (launched by launch_pdl)
  pdl_trigger();  // the next kernel, if launched as a programmatic dependent, may start
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
  pdl_wait();     // the previous kernel's writes are visible (launched by launch_pdl)
  pdl_trigger();  // the next kernel, if launched as a programmatic dependent, may start
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
  pdl_wait();     // the previous kernel's writes are visible (launched by launch_pdl)
  pdl_trigger();  // the next kernel, if launched as a programmatic dependent, may start
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
  pdl_wait();     // the previous kernel's writes are visible (launched by launch_pdl)
  pdl_trigger();  // the next kernel, if launched as a programmatic dependent, may start
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
  pdl_wait();     // the previous kernel's writes are visible (launched by launch_pdl)
  pdl_trigger();  // the next kernel, if launched as a programmatic dependent, may start
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

// ---------------------------------------------------------------- direct paths
//
// Convolutions with very few output channels (the U-Net's 3-channel head) or
// very few column rows (its 3-channel input layer) would fill a few percent
// of a tensor-core tile, so they run as direct CUDA-core loops on the input
// (no columns) in fp32, with the reference's order where it has one, and
// their operands staged in shared memory.
constexpr int kDirectMaxOC = 4;     // output channels per thread (forward, dx, dW groups)
constexpr int kDirectGroup = 8;     // input channels staged per round (forward)
constexpr int kDirectDxGroup = 16;  // input channels per CTA (dx)
constexpr int kDirectSmemFloats = 49152;  // 192 KB of staged planes at most

// The direct kernels work on kDirectPx consecutive pixels of one row per
// thread (rows a multiple of kDirectPx long), with the window (KS x KS, 1 or
// 3) and the channel count NOC (1..4) known at compile time and operands
// staged in shared memory with zero halos (no bounds tests in the inner
// loops).  The forward and dx keep the reference's operation order (separate
// multiplies and adds; a tap outside the image contributes an exact +0), the
// weight gradient uses FMA partial sums in a fixed order.
constexpr int kDirectPx = 4;
constexpr int kDirectThreads = 128;
constexpr int kDirectPixels = kDirectThreads * kDirectPx;  // pixels per CTA

// Rows per CTA: R * width = kDirectPixels (width divides it or R = 1).
__host__ __device__ inline int direct_rows(int width, int height) {
  const int r = kDirectPixels / width;
  return r < 1 ? 1 : (r > height ? height : r);
}

// y[b][oc][oh][ow] = (sum over k = (ic*k + kh)*k + kw ascending of
// W[oc][k] * x[b][ic][ih][iw]) + bias[oc] (the reference adds the bias after
// the product, conv2d.h:255-263).  A CTA computes R output rows of one image,
// staging kDirectGroup input channels' rows (with zero halos) per round and
// every weight once.
template <int KS, int NOC>
__global__ void __launch_bounds__(kDirectThreads) conv_direct_fwd_k(
    const float* __restrict__ x, Shape sh, const float* __restrict__ w,
    const float* __restrict__ bias, float* __restrict__ y) {
  pdl_wait();     // the previous kernel's writes are visible (launched by launch_pdl)
  pdl_trigger();  // the next kernel, if launched as a programmatic dependent, may start
  extern __shared__ __align__(16) float sm[];
  const int R = direct_rows(sh.OW, sh.OH), nrows = (R - 1) * sh.s + KS;
  const int pitch = sh.W + 2 * sh.p;          // staged row: p zeros | W values | p zeros
  const int K = sh.IC * KS * KS, P = sh.OH * sh.OW;
  float* xs = sm;                             // [group][nrows][pitch]
  float* ws = sm + kDirectGroup * nrows * pitch;  // [oc][K]
  const int tiles = (sh.OH + R - 1) / R;
  const int b = blockIdx.x / tiles, oh0 = (blockIdx.x - b * tiles) * R;
  const int ih0 = oh0 * sh.s - sh.p;
  const int rows = min(R, sh.OH - oh0);
  const int q0 = threadIdx.x * kDirectPx;     // this thread's first pixel of the tile
  const int r = q0 / sh.OW, ow0 = q0 - r * sh.OW;
  const bool active = r < rows;
  for (int i = threadIdx.x; i < NOC * K; i += blockDim.x) ws[i] = __ldg(w + i);
  float acc[kDirectPx][NOC];
#pragma unroll
  for (int j = 0; j < kDirectPx; ++j)
#pragma unroll
    for (int o = 0; o < NOC; ++o) acc[j][o] = 0.0f;
  constexpr int kSpan = (kDirectPx - 1) * 2 + KS;  // input values one row of taps reads (stride <= 2)
  for (int c0 = 0; c0 < sh.IC; c0 += kDirectGroup) {
    const int ng = min(kDirectGroup, sh.IC - c0);
    __syncthreads();  // the previous round's reads are done
    const int nrow_all = ng * nrows;
    for (int rr = threadIdx.x >> 5; rr < nrow_all; rr += blockDim.x >> 5) {
      const int g = rr / nrows, ih = ih0 + (rr - g * nrows);
      float* dst = xs + rr * pitch;
      const bool in = ih >= 0 && ih < sh.H;
      const float* src = x + (((size_t)b * sh.IC + c0 + g) * sh.H + (in ? ih : 0)) * sh.W;
      for (int c = threadIdx.x & 31; c < pitch; c += 32) {
        const int iw = c - sh.p;
        if (in && iw >= 0 && iw < sh.W) cp_async4(dst + c, src + iw);
        else dst[c] = 0.0f;
      }
    }
    cp_async_wait_all();
    __syncthreads();
    if (active) {
      for (int g = 0; g < ng; ++g) {
        const float* wg = ws + (c0 + g) * KS * KS;
#pragma unroll
        for (int kh = 0; kh < KS; ++kh) {
          const float* xr = xs + (g * nrows + r * sh.s + kh) * pitch + ow0 * sh.s;
          float xv[kSpan];
#pragma unroll
          for (int u = 0; u < kSpan; ++u)
            xv[u] = (u < (kDirectPx - 1) * sh.s + KS) ? xr[u] : 0.0f;
#pragma unroll
          for (int kw = 0; kw < KS; ++kw) {
            float wv[NOC];
#pragma unroll
            for (int o = 0; o < NOC; ++o) wv[o] = wg[o * K + kh * KS + kw];
#pragma unroll
            for (int j = 0; j < kDirectPx; ++j) {
              const float v = sh.s == 1 ? xv[j + kw] : xv[2 * j + kw];
#pragma unroll
              for (int o = 0; o < NOC; ++o) acc[j][o] = __fadd_rn(acc[j][o], __fmul_rn(wv[o], v));
            }
          }
        }
      }
    }
  }
  if (active) {
#pragma unroll
    for (int o = 0; o < NOC; ++o) {
      const float bv = bias ? __ldg(bias + o) : 0.0f;
#pragma unroll
      for (int j = 0; j < kDirectPx; ++j)
        y[((size_t)b * NOC + o) * P + (oh0 + r) * sh.OW + ow0 + j] =
            bias ? __fadd_rn(acc[j][o], bv) : acc[j][o];
    }
  }
}

// dx[b][ic][ih][iw] = sum over (kh, kw) in order of t(kh, kw), with
// t = sum over oc ascending of W[oc][ic][kh][kw] * dy[b][oc][ih + p - kh][iw + p - kw]
// (zero outside the output): the reference's dcols = W^T . dout (an
// oc-ascending MatMul sum) gathered by Col2Im in (kh, kw) order
// (conv2d.h:321-324, 378-403).  Stride 1.
// A CTA takes R input rows of one image for kDirectDxGroup channels: the dy
// rows they read (zero halos) and their weights in shared memory, each
// thread's dy values in registers across the channels.
template <int KS, int NOC>
__global__ void __launch_bounds__(kDirectThreads) conv_direct_dx_k(
    const float* __restrict__ dy, Shape sh, const float* __restrict__ w, float* __restrict__ dx) {
  pdl_wait();     // the previous kernel's writes are visible (launched by launch_pdl)
  pdl_trigger();  // the next kernel, if launched as a programmatic dependent, may start
  extern __shared__ __align__(16) float sm[];
  const int R = direct_rows(sh.W, sh.H), nrows = R + KS - 1;
  const int halo = KS - 1 - sh.p;  // zeros left of column 0 (dy column ow at halo + ow)
  const int pitch = sh.OW + 2 * (KS - 1);
  const int K = sh.IC * KS * KS, P = sh.OH * sh.OW;
  float* ds = sm;                                // [oc][nrows][pitch]
  float* ws = sm + NOC * nrows * pitch;          // [oc][K]
  const int tiles = (sh.H + R - 1) / R, groups = (sh.IC + kDirectDxGroup - 1) / kDirectDxGroup;
  int t = blockIdx.x;
  const int grp = t % groups;
  t /= groups;
  const int tile = t % tiles, b = t / tiles;
  const int ih0 = tile * R, c0 = grp * kDirectDxGroup, ng = min(kDirectDxGroup, sh.IC - c0);
  const int oh0 = ih0 + sh.p - (KS - 1);  // dy row held in smem row 0
  for (int i = threadIdx.x; i < NOC * K; i += blockDim.x) ws[i] = __ldg(w + i);
  for (int rr = threadIdx.x >> 5; rr < NOC * nrows; rr += blockDim.x >> 5) {
    const int o = rr / nrows, oh = oh0 + (rr - o * nrows);
    float* dst = ds + rr * pitch;
    const bool in = oh >= 0 && oh < sh.OH;
    const float* src = dy + ((size_t)b * NOC + o) * P + (size_t)(in ? oh : 0) * sh.OW;
    for (int c = threadIdx.x & 31; c < pitch; c += 32) {
      const int ow = c - halo;
      if (in && ow >= 0 && ow < sh.OW) cp_async4(dst + c, src + ow);
      else dst[c] = 0.0f;
    }
  }
  cp_async_wait_all();
  __syncthreads();
  const int rows = min(R, sh.H - ih0);
  const int q0 = threadIdx.x * kDirectPx;
  const int r = q0 / sh.W, iw0 = q0 - r * sh.W;
  if (r >= rows) return;
  const int ih = ih0 + r;
  // dy values of this thread's windows: row srow = r + KS - 1 - kh, columns
  // halo + iw0 + j + p - kw = iw0 + j + (KS - 1 - kw) in the staged row.
  constexpr int kSpan = kDirectPx + KS - 1;
  float dv[NOC][KS][kSpan];
#pragma unroll
  for (int o = 0; o < NOC; ++o)
#pragma unroll
    for (int kh = 0; kh < KS; ++kh) {
      const float* row = ds + (o * nrows + r + KS - 1 - kh) * pitch + iw0;
#pragma unroll
      for (int u = 0; u < kSpan; ++u) dv[o][kh][u] = row[u];
    }
  for (int g = 0; g < ng; ++g) {
    const float* wg = ws + (c0 + g) * KS * KS;
    float acc[kDirectPx];
#pragma unroll
    for (int j = 0; j < kDirectPx; ++j) acc[j] = 0.0f;
#pragma unroll
    for (int kh = 0; kh < KS; ++kh)
#pragma unroll
      for (int kw = 0; kw < KS; ++kw) {
        float wv[NOC];
#pragma unroll
        for (int o = 0; o < NOC; ++o) wv[o] = wg[o * K + kh * KS + kw];
#pragma unroll
        for (int j = 0; j < kDirectPx; ++j) {
          float tv = 0.0f;
#pragma unroll
          for (int o = 0; o < NOC; ++o)
            tv = __fadd_rn(tv, __fmul_rn(wv[o], dv[o][kh][j + KS - 1 - kw]));
          acc[j] += tv;
        }
      }
    float* out = dx + (((size_t)b * sh.IC + c0 + g) * sh.H + ih) * sh.W + iw0;
#pragma unroll
    for (int j = 0; j < kDirectPx; ++j) out[j] = acc[j];
  }
}

// part[(b * OC + oc) * K + (ic * k + kh) * k + kw] = sum over the positions
// of image b of dy[b][oc][p] * x[b][ic][oh*s + kh - p][ow*s + kw - p]: one CTA
// per (image, input channel, group of NOC output channels), with the input
// plane (zero halos) and the group's dy planes in shared memory; each thread
// sums kDirectPx consecutive positions of a row at a time over a strided
// share of the rows, the threads' sums meet in a fixed order (warp shuffles,
// then warps in order).
template <int KS, int NOC>
__global__ void __launch_bounds__(kDirectThreads) conv_direct_dw_k(
    const float* __restrict__ x, const float* __restrict__ dy, Shape sh,
    float* __restrict__ part) {
  pdl_wait();     // the previous kernel's writes are visible (launched by launch_pdl)
  pdl_trigger();  // the next kernel, if launched as a programmatic dependent, may start
  extern __shared__ __align__(16) float sm[];
  __shared__ float wred[kDirectThreads / 32][NOC * KS * KS];
  const int P = sh.OH * sh.OW, K = sh.IC * KS * KS;
  const int ph = sh.H + 2 * sh.p, pw = sh.W + 2 * sh.p;  // padded plane
  const int ogroups = sh.OC / NOC;
  int t = blockIdx.x;
  const int og = t % ogroups;
  t /= ogroups;
  const int ic = t % sh.IC, b = t / sh.IC;
  const int o0 = og * NOC;
  float* xs = sm;                          // [ph][pw]
  float* ds = sm + ((ph * pw + 3) & ~3);   // [NOC][P]
  const float* xp = x + ((size_t)b * sh.IC + ic) * sh.H * sh.W;
  for (int rr = threadIdx.x >> 5; rr < ph; rr += blockDim.x >> 5) {
    const int ih = rr - sh.p;
    const bool in = ih >= 0 && ih < sh.H;
    for (int c = threadIdx.x & 31; c < pw; c += 32) {
      const int iw = c - sh.p;
      if (in && iw >= 0 && iw < sh.W) cp_async4(xs + rr * pw + c, xp + (size_t)ih * sh.W + iw);
      else xs[rr * pw + c] = 0.0f;
    }
  }
  stage_async(ds, dy + ((size_t)b * sh.OC + o0) * P, NOC * P);
  cp_async_wait_all();
  __syncthreads();
  float acc[NOC][KS * KS];
#pragma unroll
  for (int o = 0; o < NOC; ++o)
#pragma unroll
    for (int tt = 0; tt < KS * KS; ++tt) acc[o][tt] = 0.0f;
  constexpr int kSpan = (kDirectPx - 1) * 2 + KS;
  for (int q0 = threadIdx.x * kDirectPx; q0 < P; q0 += blockDim.x * kDirectPx) {
    const int oh = q0 / sh.OW, ow0 = q0 - oh * sh.OW;
    float g[NOC][kDirectPx];
#pragma unroll
    for (int o = 0; o < NOC; ++o)
#pragma unroll
      for (int j = 0; j < kDirectPx; ++j) g[o][j] = ds[o * P + q0 + j];
#pragma unroll
    for (int kh = 0; kh < KS; ++kh) {
      const float* xr = xs + (oh * sh.s + kh) * pw + ow0 * sh.s;
      float xv[kSpan];
#pragma unroll
      for (int u = 0; u < kSpan; ++u) xv[u] = (u < (kDirectPx - 1) * sh.s + KS) ? xr[u] : 0.0f;
#pragma unroll
      for (int kw = 0; kw < KS; ++kw)
#pragma unroll
        for (int j = 0; j < kDirectPx; ++j) {
          const float v = sh.s == 1 ? xv[j + kw] : xv[2 * j + kw];
#pragma unroll
          for (int o = 0; o < NOC; ++o) acc[o][kh * KS + kw] = fmaf(g[o][j], v, acc[o][kh * KS + kw]);
        }
    }
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
#pragma unroll
  for (int o = 0; o < NOC; ++o)
#pragma unroll
    for (int tt = 0; tt < KS * KS; ++tt) {
      const float v = warp_sum(acc[o][tt]);
      if (lane == 0) wred[warp][o * KS * KS + tt] = v;
    }
  __syncthreads();
  for (int j = threadIdx.x; j < NOC * KS * KS; j += blockDim.x) {
    const int o = j / (KS * KS), tt = j - o * KS * KS;
    float sum = 0.0f;
    for (int wi = 0; wi < (int)(blockDim.x >> 5); ++wi) sum += wred[wi][j];
    part[((size_t)b * sh.OC + o0 + o) * K + ic * KS * KS + tt] = sum;
  }
}

// dw[oc][kk] = the per-image sums added in image order (conv2d.h:326-331).
__global__ void conv_direct_dw_finish_k(const float* __restrict__ part, int OC, int K, int B,
                                        float* __restrict__ dw) {
  pdl_wait();     // the previous kernel's writes are visible (launched by launch_pdl)
  pdl_trigger();  // the next kernel, if launched as a programmatic dependent, may start
  const int64_t n = (int64_t)OC * K;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    float total = 0.0f;
    for (int b = 0; b < B; ++b) total += part[(size_t)b * n + i];
    dw[i] = total;
  }
}

// Channels per thread of the direct weight gradient: the largest of 4..1
// that divides OC.
int direct_dw_noc(int OC) {
  for (int n = kDirectMaxOC; n > 1; --n)
    if (OC % n == 0) return n;
  return 1;
}

// Shared memory of the direct kernels (floats).
size_t direct_fwd_smem(const Shape& sh) {
  const int R = direct_rows(sh.OW, sh.OH);
  return (size_t)kDirectGroup * ((R - 1) * sh.s + sh.k) * (sh.W + 2 * sh.p) +
         (size_t)sh.OC * sh.IC * sh.k * sh.k;
}
size_t direct_dx_smem(const Shape& sh) {
  const int R = direct_rows(sh.W, sh.H);
  return (size_t)sh.OC * (R + sh.k - 1) * (sh.OW + 2 * (sh.k - 1)) +
         (size_t)sh.OC * sh.IC * sh.k * sh.k;
}
size_t direct_dw_smem(const Shape& sh) {
  return (size_t)(((sh.H + 2 * sh.p) * (sh.W + 2 * sh.p) + 3) & ~3) +
         (size_t)direct_dw_noc(sh.OC) * sh.OH * sh.OW;
}

int grid_runs(int64_t runs) {
  return (int)std::max<int64_t>(1, std::min<int64_t>(runs, (int64_t)sm_count() * 32));
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

// Which products run on the direct CUDA-core paths instead of the GEMM: few
// output channels (forward, dx, weight gradient) or few column rows (weight
// gradient), 1x1 or 3x3 windows, stride 1 or 2 (dx: 1), rows a multiple of
// kDirectPx long, and operands that fit the staging buffers.  A direct
// forward implies a direct weight gradient, so no columns are needed.
bool direct_window(const Shape& sh) { return (sh.k == 1 || sh.k == 3) && sh.s <= 2; }
bool direct_dw(const Shape& sh) {
  return (sh.OC <= kDirectMaxOC || sh.K() <= 32) && direct_window(sh) &&
         sh.OW % kDirectPx == 0 && direct_dw_smem(sh) <= (size_t)kDirectSmemFloats;
}
bool direct_fwd(const Shape& sh) {
  return sh.OC <= kDirectMaxOC && direct_dw(sh) && sh.OW <= kDirectPixels &&
         direct_fwd_smem(sh) <= (size_t)kDirectSmemFloats;
}
bool direct_dx(const Shape& sh) {
  return sh.OC <= kDirectMaxOC && direct_window(sh) && sh.s == 1 && sh.p <= sh.k - 1 &&
         sh.W % kDirectPx == 0 && sh.W <= kDirectPixels &&
         direct_dx_smem(sh) <= (size_t)kDirectSmemFloats;
}

// Launches a direct kernel instantiated for (KS, NOC).
template <template <int, int> class Launch, typename... Args>
ns_status direct_dispatch(int KS, int NOC, Args&&... args) {
  switch (KS * 8 + NOC) {
    case 1 * 8 + 1: return Launch<1, 1>::run(args...);
    case 1 * 8 + 2: return Launch<1, 2>::run(args...);
    case 1 * 8 + 3: return Launch<1, 3>::run(args...);
    case 1 * 8 + 4: return Launch<1, 4>::run(args...);
    case 3 * 8 + 1: return Launch<3, 1>::run(args...);
    case 3 * 8 + 2: return Launch<3, 2>::run(args...);
    case 3 * 8 + 3: return Launch<3, 3>::run(args...);
    case 3 * 8 + 4: return Launch<3, 4>::run(args...);
    default: return fail(NS_ERR_INVALID_ARGUMENT, "ns_conv2d: no direct kernel for this window");
  }
}

template <typename K>
ns_status set_smem(K kernel, size_t bytes, const char* what) {
  if (bytes > 48 * 1024)
    NS_TRY_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes),
                what);
  return NS_OK;
}

template <int KS, int NOC>
struct DirectFwd {
  static ns_status run(const float* x, const Shape& sh, const float* w, const float* bias,
                       float* y, cudaStream_t s) {
    const size_t smem = direct_fwd_smem(sh) * sizeof(float);
    ns_status rc = set_smem(conv_direct_fwd_k<KS, NOC>, smem, "ns_conv2d_fwd direct");
    if (rc != NS_OK) return rc;
    const int R = direct_rows(sh.OW, sh.OH);
    return launch_pdl(conv_direct_fwd_k<KS, NOC>, dim3(sh.B * ((sh.OH + R - 1) / R)),
                      dim3(kDirectThreads), smem, s, "ns_conv2d_fwd direct", x, sh, w, bias, y);
  }
};
template <int KS, int NOC>
struct DirectDx {
  static ns_status run(const float* dy, const Shape& sh, const float* w, float* dx,
                       cudaStream_t s) {
    const size_t smem = direct_dx_smem(sh) * sizeof(float);
    ns_status rc = set_smem(conv_direct_dx_k<KS, NOC>, smem, "ns_conv2d_bwd direct dx");
    if (rc != NS_OK) return rc;
    const int R = direct_rows(sh.W, sh.H);
    const int grid = sh.B * ((sh.H + R - 1) / R) * ((sh.IC + kDirectDxGroup - 1) / kDirectDxGroup);
    return launch_pdl(conv_direct_dx_k<KS, NOC>, dim3(grid), dim3(kDirectThreads), smem, s,
                      "ns_conv2d_bwd direct dx", dy, sh, w, dx);
  }
};
template <int KS, int NOC>
struct DirectDw {
  static ns_status run(const float* x, const float* dy, const Shape& sh, float* part,
                       cudaStream_t s) {
    const size_t smem = direct_dw_smem(sh) * sizeof(float);
    ns_status rc = set_smem(conv_direct_dw_k<KS, NOC>, smem, "ns_conv2d_bwd direct weight gradient");
    if (rc != NS_OK) return rc;
    return launch_pdl(conv_direct_dw_k<KS, NOC>, dim3(sh.B * sh.IC * (sh.OC / NOC)),
                      dim3(kDirectThreads), smem, s, "ns_conv2d_bwd direct weight gradient", x,
                      dy, sh, part);
  }
};

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
  float *cols, *cols_lo, *w_lo, *yc, *dyc, *dyc_lo, *dcols, *bias_part, *dw_part;
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
  w.dw_part = direct_dw(sh) ? take(al64((size_t)sh.OC * sh.K() * std::max(sh.B, 1))) : nullptr;
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
  return launch_pdl(im2col_k, dim3(grid_runs(sh.K() * sh.B)), dim3(256), 0, s, "ns_conv2d im2col",
                    x, sh, cols, cols_lo, vec);
}

ns_status launch_direct_fwd(const float* x, const Shape& sh, const float* weight,
                            const float* bias, float* y, cudaStream_t s) {
  return direct_dispatch<DirectFwd>(sh.k, sh.OC, x, sh, weight, bias, y, s);
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
  return launch_pdl(cnhw_to_nchw_bias_k, dim3(grid_runs((int64_t)sh.B * sh.OC)), dim3(256), 0, s,
                    "ns_conv2d_fwd layout", ws.yc, bias, sh, y, vec);
}

// The backward: x is read by the direct paths, the columns (of x) by the
// weight-gradient GEMM.
ns_status backward_body(const Shape& sh, const float* x, const float* cols, const float* cols_lo,
                        const float* dy, const float* weight, float* dx, float* dweight,
                        float* dbias, const Ws& ws, cudaStream_t s) {
  const int M = sh.OC, N = (int)sh.N(), K = (int)sh.K();
  ns_status rc = NS_OK;
  const bool gemm_dw = !direct_dw(sh), gemm_dx = dx && !direct_dx(sh);
  if (gemm_dw || gemm_dx) {
    const int vec = (sh.P() % 4 == 0 && aligned16(dy) && aligned16(ws.dyc) && aligned16(ws.dyc_lo))
                        ? 1 : 0;
    rc = launch_pdl(nchw_to_cnhw_k, dim3(grid_runs((int64_t)sh.B * sh.OC)), dim3(256), 0, s,
                    "ns_conv2d_bwd layout", dy, sh, ws.dyc, ws.dyc_lo, vec);
    if (rc != NS_OK) return rc;
  }
  rc = launch_pdl(bias_part_k, dim3(sh.OC, sh.B), dim3(256), 0, s, "ns_conv2d_bwd bias", dy, sh,
                  ws.bias_part);
  if (rc != NS_OK) return rc;
  rc = launch_pdl(bias_finish_k, dim3(ceil_div(sh.OC, 128)), dim3(128), 0, s, "ns_conv2d_bwd bias",
                  ws.bias_part, sh.OC, sh.B, dbias);
  if (rc != NS_OK) return rc;
  if (gemm_dw) {
    // dW[OC, K] = dYc[OC, B*P] . cols[K, B*P]^T (overwritten, as the reference zeroes it first)
    rc = ns_gemm_lo(M, K, N, ws.dyc, N, 0, lo_if(ws.dyc_lo, N), cols, N, 1, lo_if(cols_lo, N),
                    dweight, K, 0.0f, NS_EPI_STORE, nullptr, nullptr, nullptr, ws.gemm,
                    ws.gemm_bytes, s);
  } else {
    rc = direct_dispatch<DirectDw>(sh.k, direct_dw_noc(M), x, dy, sh, ws.dw_part, s);
    if (rc != NS_OK) return rc;
    rc = launch_pdl(conv_direct_dw_finish_k, dim3(grid_runs(ceil_div64((int64_t)M * K, 256))),
                    dim3(256), 0, s, "ns_conv2d_bwd direct weight gradient", ws.dw_part, M, K,
                    sh.B, dweight);
  }
  if (rc != NS_OK || !dx) return rc;
  if (!gemm_dx) {
    return direct_dispatch<DirectDx>(sh.k, sh.OC, dy, sh, weight, dx, s);
  }
  rc = ns_split_lo(weight, M, K, K, ws.w_lo, s);
  if (rc != NS_OK) return rc;
  // dcols[K, B*P] = W[OC, K]^T . dYc[OC, B*P]
  rc = ns_gemm_lo(K, N, M, weight, K, 1, lo_if(ws.w_lo, K), ws.dyc, N, 0, lo_if(ws.dyc_lo, N),
                  ws.dcols, N, 0.0f, NS_EPI_STORE, nullptr, nullptr, nullptr, ws.gemm,
                  ws.gemm_bytes, s);
  if (rc != NS_OK) return rc;
  const int g = grid_runs((int64_t)sh.B * sh.IC);
  if (sh.k == 3 && sh.s == 1)
    return launch_pdl(col2im_fixed_k<3, 1>, dim3(g), dim3(256), 0, s, "ns_conv2d_bwd col2im",
                      ws.dcols, sh, dx);
  if (sh.k == 3 && sh.s == 2)
    return launch_pdl(col2im_fixed_k<3, 2>, dim3(g), dim3(256), 0, s, "ns_conv2d_bwd col2im",
                      ws.dcols, sh, dx);
  return launch_pdl(col2im_k, dim3(g), dim3(256), 0, s, "ns_conv2d_bwd col2im", ws.dcols, sh,
                    dx);
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
  return direct_fwd(sh) && direct_dw(sh) ? 0 : sh.K() * sh.N();
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
  NS_REQUIRE(x && weight && y, "conv forward: NULL argument");
  if (direct_fwd(sh)) return launch_direct_fwd(x, sh, weight, bias, y, s);
  NS_REQUIRE(cols && cols_lo, "conv forward: NULL column buffer");
  Ws ws;
  rc = check_ws(sh, workspace, workspace_bytes, false, "conv forward", &ws);
  if (rc != NS_OK) return rc;
  rc = launch_im2col(x, sh, cols, cols_lo, s);
  if (rc != NS_OK) return rc;
  return forward_body(sh, weight, bias, y, cols, cols_lo, ws, s);
}

ns_status backward_from_cols(const float* x, const float* cols, const float* cols_lo,
                             const float* dy, int B, int IC, int H, int W, const float* weight,
                             int OC, int k, int stride, int pad, float* dx, float* dweight,
                             float* dbias, void* workspace, size_t workspace_bytes,
                             cudaStream_t s) {
  Shape sh;
  ns_status rc = make_shape(B, IC, H, W, OC, k, stride, pad, &sh);
  if (rc != NS_OK) return rc;
  NS_REQUIRE(x && dy && weight && dweight && dbias, "conv backward: NULL argument");
  NS_REQUIRE(direct_dw(sh) || (cols && cols_lo), "conv backward: NULL column buffer");
  if (B == 0) return zero_grads(sh, dweight, dbias, s);
  Ws ws;
  rc = check_ws(sh, workspace, workspace_bytes, false, "conv backward", &ws);
  if (rc != NS_OK) return rc;
  return backward_body(sh, x, cols, cols_lo, dy, weight, dx, dweight, dbias, ws, s);
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
  if (direct_fwd(sh)) return launch_direct_fwd(x, sh, weight, bias, y, s);
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
  if (!direct_dw(sh)) {
    rc = launch_im2col(x, sh, ws.cols, ws.cols_lo, s);
    if (rc != NS_OK) return rc;
  }
  return backward_body(sh, x, ws.cols, ws.cols_lo, dy, weight, dx, dweight, dbias, ws, s);
}

}  // extern "C"
