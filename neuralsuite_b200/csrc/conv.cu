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

// ---------------------------------------------------------------- direct paths
//
// Convolutions with very few output channels (the U-Net's 3-channel head) or
// very few column rows (its 3-channel input layer) would fill a few percent
// of a tensor-core tile, so they run as direct CUDA-core loops on the input
// (no columns) in fp32, with the reference's order where it has one, and
// their operands staged in shared memory.
constexpr int kDirectMaxOC = 4;     // output channels per thread (forward, dx, dW groups)
constexpr int kDirectMaxTaps = 9;   // k x k <= 9 for the direct weight gradient
constexpr int kDirectGroup = 16;    // input channels staged per round (forward)
constexpr int kDirectDxGroup = 16;  // input channels per CTA (dx)
constexpr int kDirectSmemFloats = 24576;  // 96 KB of staged planes (dW)

// Asynchronous global -> shared copies (cp.async): every copy of a staging
// round is in flight at once, then one wait.  16-byte copies where both
// addresses allow, 4-byte copies otherwise.
__device__ __forceinline__ uint32_t sm_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void cp_async16(float* dst, const float* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(sm_addr(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async4(float* dst, const float* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(sm_addr(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.wait_all;" ::: "memory");
}
// n floats from src to dst, shared by the CTA's threads (no wait).
__device__ __forceinline__ void stage(float* dst, const float* src, int n) {
  const bool vec = ((n & 3) == 0) && ((reinterpret_cast<uintptr_t>(src) & 15) == 0) &&
                   ((sm_addr(dst) & 15) == 0);
  if (vec) {
    for (int i = threadIdx.x * 4; i < n; i += blockDim.x * 4) cp_async16(dst + i, src + i);
  } else {
    for (int i = threadIdx.x; i < n; i += blockDim.x) cp_async4(dst + i, src + i);
  }
}

// Output rows per CTA of the direct forward (R * OW <= 256: one pixel per thread).
__host__ __device__ inline int direct_rows(int OW, int OH) {
  const int r = 256 / OW;
  return r < 1 ? 1 : (r > OH ? OH : r);
}
// Input rows per CTA of the direct dx (R * W <= 512).
__host__ __device__ inline int direct_dx_rows(int W, int H) {
  const int r = 512 / W;
  return r < 1 ? 1 : (r > H ? H : r);
}

// y[b][oc][oh][ow] = (sum over k = (ic*k + kh)*k + kw ascending of
// W[oc][k] * x[b][ic][ih][iw]) + bias[oc]: MatMul's k-ascending sum with
// separate multiplies and adds (src/tensor.cpp:236-257), then the bias
// (conv2d.h:255-263).  A CTA computes R output rows of one image for every
// channel, one pixel per thread, staging kDirectGroup input channels' rows
// at a time (rows outside the image as zeros).
__global__ void __launch_bounds__(256) conv_direct_fwd_k(const float* __restrict__ x, Shape sh,
                                                         const float* __restrict__ w,
                                                         const float* __restrict__ bias,
                                                         float* __restrict__ y) {
  extern __shared__ __align__(16) float sm[];
  const int R = direct_rows(sh.OW, sh.OH), nrows = (R - 1) * sh.s + sh.k;
  const int kk2 = sh.k * sh.k, K = sh.IC * kk2, P = sh.OH * sh.OW;
  const int rowlen = (sh.W + 3) & ~3;             // staged row pitch (16-byte rows)
  float* xs = sm;                                   // [group][nrows][rowlen]
  float* ws = sm + kDirectGroup * nrows * rowlen;   // [oc][K] (all weights)
  const int tiles = (sh.OH + R - 1) / R;
  const int b = blockIdx.x / tiles, oh0 = (blockIdx.x - b * tiles) * R;
  const int ih0 = oh0 * sh.s - sh.p;
  const int npix = min(R, sh.OH - oh0) * sh.OW;
  const int q = threadIdx.x, r = q / sh.OW, ow = q - r * sh.OW;
  stage(ws, w, sh.OC * K);
  float acc[kDirectMaxOC];
#pragma unroll
  for (int o = 0; o < kDirectMaxOC; ++o) acc[o] = 0.0f;
  for (int c0 = 0; c0 < sh.IC; c0 += kDirectGroup) {
    const int ng = min(kDirectGroup, sh.IC - c0);
    __syncthreads();  // the previous round's reads are done
    for (int g = 0; g < ng; ++g)
      for (int rr = threadIdx.x >> 5; rr < nrows; rr += blockDim.x >> 5) {
        const int ih = ih0 + rr;
        float* dst = xs + (g * nrows + rr) * rowlen;
        if (ih >= 0 && ih < sh.H) {
          const float* src = x + (((size_t)b * sh.IC + c0 + g) * sh.H + ih) * sh.W;
          for (int c = threadIdx.x & 31; c < sh.W; c += 32) cp_async4(dst + c, src + c);
        } else {
          for (int c = threadIdx.x & 31; c < sh.W; c += 32) dst[c] = 0.0f;
        }
      }
    cp_async_wait_all();
    __syncthreads();
    if (q < npix) {
      for (int g = 0; g < ng; ++g)
        for (int kh = 0; kh < sh.k; ++kh) {
          const float* xr = xs + (g * nrows + r * sh.s + kh) * rowlen;
          for (int kw = 0; kw < sh.k; ++kw) {
            const int iw = ow * sh.s + kw - sh.p;
            const float v = (iw >= 0 && iw < sh.W) ? xr[iw] : 0.0f;
            const float* wt = ws + (c0 + g) * kk2 + kh * sh.k + kw;
#pragma unroll
            for (int o = 0; o < kDirectMaxOC; ++o)
              if (o < sh.OC) acc[o] = __fadd_rn(acc[o], __fmul_rn(wt[o * K], v));
          }
        }
    }
  }
  if (q < npix) {
#pragma unroll
    for (int o = 0; o < kDirectMaxOC; ++o)
      if (o < sh.OC) {
        const float v = bias ? __fadd_rn(acc[o], __ldg(bias + o)) : acc[o];
        y[((size_t)b * sh.OC + o) * P + oh0 * sh.OW + q] = v;
      }
  }
}

// dx[b][ic][ih][iw] = sum over (kh, kw) in order of t(kh, kw), with
// t = sum over oc ascending of W[oc][ic][kh][kw] * dy[b][oc][oh][ow] for each
// window (oh, ow) = (ih + p - kh, iw + p - kw) inside the output: the
// reference's dcols = W^T . dout (an oc-ascending MatMul sum) gathered by
// Col2Im in (kh, kw) order (conv2d.h:321-324, 378-403).  Stride 1.  A CTA
// takes R input rows of one image for kDirectDxGroup channels, with the dy
// rows they read and their weights in shared memory.
__global__ void __launch_bounds__(256) conv_direct_dx_k(const float* __restrict__ dy, Shape sh,
                                                        const float* __restrict__ w,
                                                        float* __restrict__ dx) {
  extern __shared__ __align__(16) float sm[];
  const int R = direct_dx_rows(sh.W, sh.H), nrows = R + sh.k - 1;
  const int kk2 = sh.k * sh.k, K = sh.IC * kk2, P = sh.OH * sh.OW;
  float* ds = sm;                                // [oc][nrows][OW]
  float* ws = sm + sh.OC * nrows * sh.OW;        // [oc][K] (all weights)
  const int tiles = (sh.H + R - 1) / R, groups = (sh.IC + kDirectDxGroup - 1) / kDirectDxGroup;
  int t = blockIdx.x;
  const int grp = t % groups;
  t /= groups;
  const int tile = t % tiles, b = t / tiles;
  const int ih0 = tile * R, c0 = grp * kDirectDxGroup, ng = min(kDirectDxGroup, sh.IC - c0);
  const int oh0 = ih0 + sh.p - (sh.k - 1);  // dy row held in smem row 0
  stage(ws, w, sh.OC * K);
  for (int i = threadIdx.x >> 5; i < sh.OC * nrows; i += blockDim.x >> 5) {
    const int o = i / nrows, rr = i - o * nrows, oh = oh0 + rr;
    float* dst = ds + i * sh.OW;
    if (oh >= 0 && oh < sh.OH) {
      const float* src = dy + ((size_t)b * sh.OC + o) * P + (size_t)oh * sh.OW;
      for (int c = threadIdx.x & 31; c < sh.OW; c += 32) cp_async4(dst + c, src + c);
    } else {
      for (int c = threadIdx.x & 31; c < sh.OW; c += 32) dst[c] = 0.0f;
    }
  }
  cp_async_wait_all();
  __syncthreads();
  const int rows = min(R, sh.H - ih0), npix = rows * sh.W;
  for (int item = threadIdx.x; item < ng * npix; item += blockDim.x) {
    const int g = item / npix, q = item - g * npix;
    const int r = q / sh.W, iw = q - r * sh.W, ih = ih0 + r;
    float acc = 0.0f;
    for (int kh = 0; kh < sh.k; ++kh) {
      const int oh = ih + sh.p - kh;
      if (oh < 0 || oh >= sh.OH) continue;
      const int srow = oh - oh0;
      for (int kw = 0; kw < sh.k; ++kw) {
        const int ow = iw + sh.p - kw;
        if (ow < 0 || ow >= sh.OW) continue;
        const float* wt = ws + (c0 + g) * kk2 + kh * sh.k + kw;
        float tv = 0.0f;
#pragma unroll
        for (int o = 0; o < kDirectMaxOC; ++o)
          if (o < sh.OC)
            tv = __fadd_rn(tv, __fmul_rn(wt[o * K], ds[(o * nrows + srow) * sh.OW + ow]));
        acc += tv;
      }
    }
    dx[(((size_t)b * sh.IC + c0 + g) * sh.H + ih) * sh.W + iw] = acc;
  }
}

// part[(b * OC + oc) * K + (ic * k + kh) * k + kw] = sum over the positions
// of image b of dy[b][oc][p] * x[b][ic][oh*s + kh - p][ow*s + kw - p]: one CTA
// per (image, input channel, group of up to kDirectMaxOC output channels),
// with the input plane and the group's dy planes in shared memory; each
// thread sums a strided share of the positions, the threads' sums meet in a
// fixed order (warp shuffles, then warps in order).
__global__ void __launch_bounds__(256) conv_direct_dw_k(const float* __restrict__ x,
                                                        const float* __restrict__ dy, Shape sh,
                                                        float* __restrict__ part) {
  extern __shared__ __align__(16) float sm[];
  __shared__ float wred[8][kDirectMaxOC * kDirectMaxTaps];
  const int HW = sh.H * sh.W, P = sh.OH * sh.OW, kk2 = sh.k * sh.k, K = sh.IC * kk2;
  const int ogroups = (sh.OC + kDirectMaxOC - 1) / kDirectMaxOC;
  int t = blockIdx.x;
  const int og = t % ogroups;
  t /= ogroups;
  const int ic = t % sh.IC, b = t / sh.IC;
  const int o0 = og * kDirectMaxOC, no = min(kDirectMaxOC, sh.OC - o0);
  const int hw4 = (HW + 3) & ~3;
  float* xs = sm;         // [H*W]
  float* ds = sm + hw4;   // [no][P]
  stage(xs, x + ((size_t)b * sh.IC + ic) * HW, HW);
  stage(ds, dy + ((size_t)b * sh.OC + o0) * P, no * P);
  cp_async_wait_all();
  __syncthreads();
  // Tap offsets of the window, once.
  int tdh[kDirectMaxTaps], tdw[kDirectMaxTaps];
#pragma unroll
  for (int tt = 0; tt < kDirectMaxTaps; ++tt) {
    const int kh = tt / sh.k;
    tdh[tt] = kh - sh.p;
    tdw[tt] = tt - kh * sh.k - sh.p;
  }
  float acc[kDirectMaxOC * kDirectMaxTaps];
#pragma unroll
  for (int j = 0; j < kDirectMaxOC * kDirectMaxTaps; ++j) acc[j] = 0.0f;
  for (int q = threadIdx.x; q < P; q += blockDim.x) {
    const int oh = q / sh.OW, ow = q - oh * sh.OW;
    float g[kDirectMaxOC];
#pragma unroll
    for (int o = 0; o < kDirectMaxOC; ++o) g[o] = o < no ? ds[o * P + q] : 0.0f;
#pragma unroll
    for (int tt = 0; tt < kDirectMaxTaps; ++tt) {
      if (tt < kk2) {
        const int ih = oh * sh.s + tdh[tt], iw = ow * sh.s + tdw[tt];
        const float v = (ih >= 0 && ih < sh.H && iw >= 0 && iw < sh.W) ? xs[ih * sh.W + iw] : 0.0f;
#pragma unroll
        for (int o = 0; o < kDirectMaxOC; ++o) acc[o * kDirectMaxTaps + tt] = fmaf(g[o], v, acc[o * kDirectMaxTaps + tt]);
      }
    }
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
#pragma unroll
  for (int j = 0; j < kDirectMaxOC * kDirectMaxTaps; ++j) {
    const float v = warp_sum(acc[j]);
    if (lane == 0) wred[warp][j] = v;
  }
  __syncthreads();
  const int j = threadIdx.x;
  if (j < kDirectMaxOC * kDirectMaxTaps) {
    const int o = j / kDirectMaxTaps, tt = j - o * kDirectMaxTaps;
    if (o < no && tt < kk2) {
      float sum = 0.0f;
      for (int w = 0; w < (int)(blockDim.x >> 5); ++w) sum += wred[w][j];
      part[((size_t)b * sh.OC + o0 + o) * K + ic * kk2 + tt] = sum;
    }
  }
}

// dw[oc][kk] = the per-image sums added in image order (conv2d.h:326-331).
__global__ void conv_direct_dw_finish_k(const float* __restrict__ part, int OC, int K, int B,
                                        float* __restrict__ dw) {
  const int64_t n = (int64_t)OC * K;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    float total = 0.0f;
    for (int b = 0; b < B; ++b) total += part[(size_t)b * n + i];
    dw[i] = total;
  }
}

// Shared memory of the direct kernels (floats).
size_t direct_fwd_smem(const Shape& sh) {
  const int R = direct_rows(sh.OW, sh.OH);
  return (size_t)kDirectGroup * ((R - 1) * sh.s + sh.k) * ((sh.W + 3) & ~3) +
         (size_t)sh.OC * sh.IC * sh.k * sh.k;
}
size_t direct_dx_smem(const Shape& sh) {
  const int R = direct_dx_rows(sh.W, sh.H);
  return (size_t)sh.OC * (R + sh.k - 1) * sh.OW + (size_t)sh.OC * sh.IC * sh.k * sh.k;
}
size_t direct_dw_smem(const Shape& sh) {
  return (size_t)((sh.H * sh.W + 3) & ~3) + (size_t)kDirectMaxOC * sh.OH * sh.OW;
}

int grid_runs(int64_t runs) {
  return (int)std::max<int64_t>(1, std::min<int64_t>(runs, (int64_t)sm_count() * 32));
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

// Which products run on the direct CUDA-core paths instead of the GEMM: few
// output channels (forward, dx, weight gradient) or few column rows (weight
// gradient), small windows, and planes that fit the staging buffers.  A
// direct forward implies a direct weight gradient, so no columns are needed.
bool direct_dw(const Shape& sh) {
  return (sh.OC <= kDirectMaxOC || sh.K() <= 32) && sh.k * sh.k <= kDirectMaxTaps &&
         direct_dw_smem(sh) <= (size_t)kDirectSmemFloats;
}
bool direct_fwd(const Shape& sh) {
  return sh.OC <= kDirectMaxOC && sh.OW <= 256 && direct_dw(sh) &&
         direct_fwd_smem(sh) * sizeof(float) <= 48 * 1024;
}
bool direct_dx(const Shape& sh) {
  return sh.OC <= kDirectMaxOC && sh.s == 1 && sh.W <= 512 &&
         direct_dx_smem(sh) * sizeof(float) <= 48 * 1024;
}

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
  im2col_k<<<grid_runs(sh.K() * sh.B), 256, 0, s>>>(x, sh, cols, cols_lo, vec);
  return check_launch("ns_conv2d im2col");
}

ns_status launch_direct_fwd(const float* x, const Shape& sh, const float* weight,
                            const float* bias, float* y, cudaStream_t s) {
  const int R = direct_rows(sh.OW, sh.OH);
  const int grid = sh.B * ((sh.OH + R - 1) / R);
  conv_direct_fwd_k<<<grid, 256, direct_fwd_smem(sh) * sizeof(float), s>>>(x, sh, weight, bias, y);
  return check_launch("ns_conv2d_fwd direct");
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
    nchw_to_cnhw_k<<<grid_runs((int64_t)sh.B * sh.OC), 256, 0, s>>>(dy, sh, ws.dyc, ws.dyc_lo, vec);
    rc = check_launch("ns_conv2d_bwd layout");
    if (rc != NS_OK) return rc;
  }
  bias_part_k<<<dim3(sh.OC, sh.B), 256, 0, s>>>(dy, sh, ws.bias_part);
  rc = check_launch("ns_conv2d_bwd bias");
  if (rc != NS_OK) return rc;
  bias_finish_k<<<ceil_div(sh.OC, 128), 128, 0, s>>>(ws.bias_part, sh.OC, sh.B, dbias);
  rc = check_launch("ns_conv2d_bwd bias");
  if (rc != NS_OK) return rc;
  if (gemm_dw) {
    // dW[OC, K] = dYc[OC, B*P] . cols[K, B*P]^T (overwritten, as the reference zeroes it first)
    rc = ns_gemm_lo(M, K, N, ws.dyc, N, 0, lo_if(ws.dyc_lo, N), cols, N, 1, lo_if(cols_lo, N),
                    dweight, K, 0.0f, NS_EPI_STORE, nullptr, nullptr, nullptr, ws.gemm,
                    ws.gemm_bytes, s);
  } else {
    const size_t smem = direct_dw_smem(sh) * sizeof(float);
    if (smem > 48 * 1024)
      NS_TRY_CUDA(cudaFuncSetAttribute(conv_direct_dw_k, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)smem),
                  "ns_conv2d_bwd direct weight gradient");
    const int ogroups = (M + kDirectMaxOC - 1) / kDirectMaxOC;
    conv_direct_dw_k<<<sh.B * sh.IC * ogroups, 256, smem, s>>>(x, dy, sh, ws.dw_part);
    rc = check_launch("ns_conv2d_bwd direct weight gradient");
    if (rc != NS_OK) return rc;
    conv_direct_dw_finish_k<<<grid_runs(ceil_div64((int64_t)M * K, 256)), 256, 0, s>>>(
        ws.dw_part, M, K, sh.B, dweight);
    rc = check_launch("ns_conv2d_bwd direct weight gradient");
  }
  if (rc != NS_OK || !dx) return rc;
  if (!gemm_dx) {
    const int R = direct_dx_rows(sh.W, sh.H);
    const int grid = sh.B * ((sh.H + R - 1) / R) * ((sh.IC + kDirectDxGroup - 1) / kDirectDxGroup);
    conv_direct_dx_k<<<grid, 256, direct_dx_smem(sh) * sizeof(float), s>>>(dy, sh, weight, dx);
    return check_launch("ns_conv2d_bwd direct dx");
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
