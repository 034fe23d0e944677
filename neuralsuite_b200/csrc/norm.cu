// K3: LayerNorm forward / backward and the deterministic column sums used for
// dgamma, dbeta and the Linear bias gradient.  HBM-bound: one warp per row,
// float4 loads, warp-shuffle reductions; column sums are two-stage (per-CTA
// partials in caller workspace, then an ordered sum over CTAs) so every run
// gives the same bits.
#include <algorithm>
#include <type_traits>

#include "common.cuh"

namespace nsb {
namespace {

constexpr int kRowsWarps = 8;          // warps per CTA in the row kernels
constexpr int kMaxPartials = 296;      // 2 x 148 SMs: cap on stage-1 CTAs
constexpr int kMaxVec = 8;             // float4 per lane => dim <= 1024 on the fast path

// ----------------------------------------------------------- forward
// LayerNormForward (src/tensor.cpp:290-322): mean = sum/D, var = sum((x-m)^2)/D,
// rstd = 1/sqrt(var+eps), out = ((x-m)*rstd)*gamma + beta.
// RES: the row is first formed as x = resid + (raw + bias) (the residual add
// of a GEMM's bias epilogue, same rounding) and written to x_out.  LO: the
// output's tf32 lo part goes to out_lo as well (the next GEMM's operand split).
template <int NV, bool RES, bool LO>
__global__ void __launch_bounds__(256) ln_fwd_vec(const float* x,  // may alias x_out
                                                  const float* __restrict__ gamma,
                                                  const float* __restrict__ beta,
                                                  float* __restrict__ out, float* __restrict__ mean,
                                                  float* __restrict__ rstd, int rows, int dim,
                                                  float eps, const float* __restrict__ bias,
                                                  const float* __restrict__ resid, float* x_out,
                                                  float* __restrict__ out_lo) {
  pdl_wait();     // the previous kernel's writes are visible (launched by launch_pdl)
  pdl_trigger();  // the next kernel, if launched as a programmatic dependent, may start
  const int row = blockIdx.x * kRowsWarps + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const int nv = dim >> 2;
  const float4* xr = reinterpret_cast<const float4*>(x + (size_t)row * dim);
  float4 v[NV];
  float s = 0.0f;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int c = lane + i * 32;
    v[i] = c < nv ? xr[c] : make_float4(0.f, 0.f, 0.f, 0.f);
    if (RES && c < nv) {
      const float4 r = reinterpret_cast<const float4*>(resid + (size_t)row * dim)[c];
      const float4 b = reinterpret_cast<const float4*>(bias)[c];
      v[i].x = __fadd_rn(r.x, __fadd_rn(v[i].x, b.x));
      v[i].y = __fadd_rn(r.y, __fadd_rn(v[i].y, b.y));
      v[i].z = __fadd_rn(r.z, __fadd_rn(v[i].z, b.z));
      v[i].w = __fadd_rn(r.w, __fadd_rn(v[i].w, b.w));
      reinterpret_cast<float4*>(x_out + (size_t)row * dim)[c] = v[i];
    }
    s += (v[i].x + v[i].y) + (v[i].z + v[i].w);
  }
  s = warp_sum(s);
  const float m = __fdiv_rn(s, (float)dim);
  float q = 0.0f;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int c = lane + i * 32;
    if (c < nv) {
      const float a = v[i].x - m, b = v[i].y - m, cc = v[i].z - m, d = v[i].w - m;
      q += (a * a + b * b) + (cc * cc + d * d);
    }
  }
  q = warp_sum(q);
  const float var = __fdiv_rn(q, (float)dim);
  const float rs = __fdiv_rn(1.0f, __fsqrt_rn(var + eps));
  if (lane == 0) {
    mean[row] = m;
    rstd[row] = rs;
  }
  const float4* g4 = reinterpret_cast<const float4*>(gamma);
  const float4* b4 = reinterpret_cast<const float4*>(beta);
  float4* o4 = reinterpret_cast<float4*>(out + (size_t)row * dim);
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int c = lane + i * 32;
    if (c < nv) {
      const float4 g = g4[c], bb = b4[c];
      float4 r;
      r.x = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(v[i].x, m), rs), g.x), bb.x);
      r.y = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(v[i].y, m), rs), g.y), bb.y);
      r.z = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(v[i].z, m), rs), g.z), bb.z);
      r.w = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(v[i].w, m), rs), g.w), bb.w);
      o4[c] = r;
      if (LO) {
        auto lo = [](float a) { return a - __uint_as_float(__float_as_uint(a) & 0xFFFFE000u); };
        reinterpret_cast<float4*>(out_lo + (size_t)row * dim)[c] =
            make_float4(lo(r.x), lo(r.y), lo(r.z), lo(r.w));
      }
    }
  }
}

// x_out = resid + (raw + bias), element-wise (the fused LayerNorm's fallback
// for shapes without its vector path).  x_out may be raw (the model writes the
// sum over the GEMM product), so neither carries __restrict__.
__global__ void resid_bias_add_k(const float* raw, const float* __restrict__ bias,
                                 const float* __restrict__ resid, float* x_out,
                                 int64_t rows, int dim) {
  pdl_wait();     // the previous kernel's writes are visible (launched by launch_pdl)
  pdl_trigger();  // the next kernel, if launched as a programmatic dependent, may start
  const int64_t n = rows * dim;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    x_out[i] = __fadd_rn(resid[i], __fadd_rn(raw[i], bias[i % dim]));
}

// Any dim: strided scalar passes over the row (re-read from L1/L2).
__global__ void __launch_bounds__(256) ln_fwd_any(const float* __restrict__ x,
                                                  const float* __restrict__ gamma,
                                                  const float* __restrict__ beta,
                                                  float* __restrict__ out, float* __restrict__ mean,
                                                  float* __restrict__ rstd, int rows, int dim,
                                                  float eps) {
  pdl_wait();     // the previous kernel's writes are visible (launched by launch_pdl)
  pdl_trigger();  // the next kernel, if launched as a programmatic dependent, may start
  const int row = blockIdx.x * kRowsWarps + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const float* xr = x + (size_t)row * dim;
  float s = 0.0f;
  for (int c = lane; c < dim; c += 32) s += xr[c];
  s = warp_sum(s);
  const float m = __fdiv_rn(s, (float)dim);
  float q = 0.0f;
  for (int c = lane; c < dim; c += 32) {
    const float d = xr[c] - m;
    q += d * d;
  }
  q = warp_sum(q);
  const float rs = __fdiv_rn(1.0f, __fsqrt_rn(__fdiv_rn(q, (float)dim) + eps));
  if (lane == 0) {
    mean[row] = m;
    rstd[row] = rs;
  }
  for (int c = lane; c < dim; c += 32)
    out[(size_t)row * dim + c] =
        __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(xr[c], m), rs), gamma[c]), beta[c]);
}

// ----------------------------------------------------------- backward
// LayerNormBackward (src/tensor.cpp:324-359) per row:
//   xh = (x-m)*rs, dxh = dout*gamma, s1 = sum dxh, s2 = sum dxh*xh,
//   dx = (rs/D) * (D*dxh - s1 - xh*s2)   [+ dresid]
// and per-CTA partial column sums of dout*xh (dgamma) and dout (dbeta).
// Each warp takes R of its rows at a time and issues all of their loads
// (x, dout, dresid) before any arithmetic, so a row costs one memory latency
// rather than two (dresid read after the row's reductions was the second); one
// CTA per SM with the registers that takes.  Rows keep their order, so the
// dgamma/dbeta partials are summed in the same order as one row at a time.
template <int NV, int R>
__global__ void __launch_bounds__(256, 1) ln_bwd_vec(
    const float* __restrict__ dout, const float* __restrict__ x, const float* __restrict__ gamma,
    const float* __restrict__ mean, const float* __restrict__ rstd,
    const float* __restrict__ dresid, float* __restrict__ dx, float* __restrict__ part_g,
    float* __restrict__ part_b, int rows, int dim, int rows_per_cta) {
  pdl_wait();     // the previous kernel's writes are visible (launched by launch_pdl)
  pdl_trigger();  // the next kernel, if launched as a programmatic dependent, may start
  extern __shared__ float red[];  // [kRowsWarps][2][dim]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nv = dim >> 2;
  const int r0 = blockIdx.x * rows_per_cta;
  const int r1 = min(rows, r0 + rows_per_cta);
  float4 pg[NV], pb[NV];
#pragma unroll
  for (int i = 0; i < NV; ++i) pg[i] = pb[i] = make_float4(0.f, 0.f, 0.f, 0.f);
  const float4* g4 = reinterpret_cast<const float4*>(gamma);
  const float fdim = (float)dim;
  for (int row0 = r0 + warp; row0 < r1; row0 += R * kRowsWarps) {
    // Every load of the R rows first (x, dout, dresid), then the arithmetic.
    float4 xv[R][NV], dv[R][NV], rv[R][NV];
    float m[R], rs[R];
#pragma unroll
    for (int j = 0; j < R; ++j) {
      const int row = row0 + j * kRowsWarps;
      const bool in = row < r1;
      m[j] = in ? mean[row] : 0.f;
      rs[j] = in ? rstd[row] : 0.f;
      const float4* x4 = reinterpret_cast<const float4*>(x + (size_t)row * dim);
      const float4* d4 = reinterpret_cast<const float4*>(dout + (size_t)row * dim);
      const float4* r4 = reinterpret_cast<const float4*>(dresid + (size_t)row * dim);
#pragma unroll
      for (int i = 0; i < NV; ++i) {
        const int c = lane + i * 32;
        const bool ok = in && c < nv;
        xv[j][i] = ok ? x4[c] : make_float4(0.f, 0.f, 0.f, 0.f);
        dv[j][i] = ok ? d4[c] : make_float4(0.f, 0.f, 0.f, 0.f);
        rv[j][i] = (ok && dresid) ? r4[c] : make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
#pragma unroll
    for (int j = 0; j < R; ++j) {
      const int row = row0 + j * kRowsWarps;
      if (row >= r1) break;
      float s1 = 0.f, s2 = 0.f;
#pragma unroll
      for (int i = 0; i < NV; ++i) {
        const int c = lane + i * 32;
        if (c < nv) {
          const float4 g = g4[c];
          float4& xh = xv[j][i];
          float4& dh = dv[j][i];
          const float4 d = dh;
          xh.x = __fmul_rn(__fsub_rn(xh.x, m[j]), rs[j]);
          xh.y = __fmul_rn(__fsub_rn(xh.y, m[j]), rs[j]);
          xh.z = __fmul_rn(__fsub_rn(xh.z, m[j]), rs[j]);
          xh.w = __fmul_rn(__fsub_rn(xh.w, m[j]), rs[j]);
          pg[i].x += d.x * xh.x; pg[i].y += d.y * xh.y;
          pg[i].z += d.z * xh.z; pg[i].w += d.w * xh.w;
          pb[i].x += d.x; pb[i].y += d.y; pb[i].z += d.z; pb[i].w += d.w;
          dh.x = __fmul_rn(d.x, g.x); dh.y = __fmul_rn(d.y, g.y);
          dh.z = __fmul_rn(d.z, g.z); dh.w = __fmul_rn(d.w, g.w);
          s1 += (dh.x + dh.y) + (dh.z + dh.w);
          s2 += (dh.x * xh.x + dh.y * xh.y) + (dh.z * xh.z + dh.w * xh.w);
        }
      }
      s1 = warp_sum(s1);
      s2 = warp_sum(s2);
      const float scale = __fdiv_rn(rs[j], fdim);
      float4* o4 = reinterpret_cast<float4*>(dx + (size_t)row * dim);
#pragma unroll
      for (int i = 0; i < NV; ++i) {
        const int c = lane + i * 32;
        if (c < nv) {
          const float4 xh = xv[j][i], dh = dv[j][i];
          float4 o;
          o.x = __fmul_rn(scale, __fsub_rn(__fsub_rn(__fmul_rn(fdim, dh.x), s1), __fmul_rn(xh.x, s2)));
          o.y = __fmul_rn(scale, __fsub_rn(__fsub_rn(__fmul_rn(fdim, dh.y), s1), __fmul_rn(xh.y, s2)));
          o.z = __fmul_rn(scale, __fsub_rn(__fsub_rn(__fmul_rn(fdim, dh.z), s1), __fmul_rn(xh.z, s2)));
          o.w = __fmul_rn(scale, __fsub_rn(__fsub_rn(__fmul_rn(fdim, dh.w), s1), __fmul_rn(xh.w, s2)));
          if (dresid) {
            const float4 rr = rv[j][i];
            o.x = __fadd_rn(rr.x, o.x); o.y = __fadd_rn(rr.y, o.y);
            o.z = __fadd_rn(rr.z, o.z); o.w = __fadd_rn(rr.w, o.w);
          }
          o4[c] = o;
        }
      }
    }
  }
  // Fixed-order reduction of the 8 warps' column partials.
  float* rg = red + (size_t)warp * 2 * dim;
  float* rb = rg + dim;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int c = lane + i * 32;
    if (c < nv) {
      reinterpret_cast<float4*>(rg)[c] = pg[i];
      reinterpret_cast<float4*>(rb)[c] = pb[i];
    }
  }
  __syncthreads();
  for (int c = threadIdx.x; c < dim; c += blockDim.x) {
    float sg = 0.f, sb = 0.f;
    for (int w = 0; w < kRowsWarps; ++w) {
      sg += red[(size_t)w * 2 * dim + c];
      sb += red[(size_t)w * 2 * dim + dim + c];
    }
    part_g[(size_t)blockIdx.x * dim + c] = sg;
    part_b[(size_t)blockIdx.x * dim + c] = sb;
  }
}

__global__ void __launch_bounds__(256) ln_bwd_any(
    const float* __restrict__ dout, const float* __restrict__ x, const float* __restrict__ gamma,
    const float* __restrict__ mean, const float* __restrict__ rstd,
    const float* __restrict__ dresid, float* __restrict__ dx, float* __restrict__ part_g,
    float* __restrict__ part_b, int rows, int dim, int rows_per_cta) {
  pdl_wait();     // the previous kernel's writes are visible (launched by launch_pdl)
  pdl_trigger();  // the next kernel, if launched as a programmatic dependent, may start
  // One CTA walks its rows; each thread owns columns c = tid + k*256 for the
  // dgamma/dbeta partials (kept in the output workspace directly).
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r0 = blockIdx.x * rows_per_cta;
  const int r1 = min(rows, r0 + rows_per_cta);
  const float fdim = (float)dim;
  // Pass 1: dx per row, one warp per row.
  for (int row = r0 + warp; row < r1; row += kRowsWarps) {
    const float m = mean[row], rs = rstd[row];
    const float* xr = x + (size_t)row * dim;
    const float* dr = dout + (size_t)row * dim;
    float s1 = 0.f, s2 = 0.f;
    for (int c = lane; c < dim; c += 32) {
      const float xh = __fmul_rn(__fsub_rn(xr[c], m), rs);
      const float dh = __fmul_rn(dr[c], gamma[c]);
      s1 += dh;
      s2 += dh * xh;
    }
    s1 = warp_sum(s1);
    s2 = warp_sum(s2);
    const float scale = __fdiv_rn(rs, fdim);
    for (int c = lane; c < dim; c += 32) {
      const float xh = __fmul_rn(__fsub_rn(xr[c], m), rs);
      const float dh = __fmul_rn(dr[c], gamma[c]);
      float o = __fmul_rn(scale, __fsub_rn(__fsub_rn(__fmul_rn(fdim, dh), s1), __fmul_rn(xh, s2)));
      if (dresid) o = __fadd_rn(dresid[(size_t)row * dim + c], o);
      dx[(size_t)row * dim + c] = o;
    }
  }
  // Pass 2: column partials, rows in order.
  for (int c = threadIdx.x; c < dim; c += blockDim.x) {
    float sg = 0.f, sb = 0.f;
    for (int row = r0; row < r1; ++row) {
      const float d = dout[(size_t)row * dim + c];
      const float xh = __fmul_rn(__fsub_rn(x[(size_t)row * dim + c], mean[row]), rstd[row]);
      sg += d * xh;
      sb += d;
    }
    part_g[(size_t)blockIdx.x * dim + c] = sg;
    part_b[(size_t)blockIdx.x * dim + c] = sb;
  }
}

// Stage 2 of every column sum: out[n] = sum over p (ascending) of part[p][n].
// Column sums of part[n_part][N]: CTA = 32 columns, warp w sums partials
// w, w+8, w+16, ... in order, then the eight warp sums are added in warp order
// (a fixed order: deterministic).
// blockIdx.y == 1 sums part2 into out2 (two column sums of one shape in one
// launch: LayerNorm's dgamma and dbeta).  Four partials are loaded before
// they are added, in the same order.
__global__ void __launch_bounds__(256) colsum_finish(const float* __restrict__ part, int n_part,
                                                     int N, float* __restrict__ out,
                                                     const float* __restrict__ part2,
                                                     float* __restrict__ out2) {
  pdl_wait();     // the previous kernel's writes are visible (launched by launch_pdl)
  pdl_trigger();  // the next kernel, if launched as a programmatic dependent, may start
  __shared__ float red[kRowsWarps][32];
  if (blockIdx.y == 1) {
    part = part2;
    out = out2;
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n = blockIdx.x * 32 + lane;
  float s = 0.f;
  if (n < N) {
    int p = warp;
    for (; p + 3 * kRowsWarps < n_part; p += 4 * kRowsWarps) {
      const float a = part[(size_t)p * N + n];
      const float b = part[(size_t)(p + kRowsWarps) * N + n];
      const float c = part[(size_t)(p + 2 * kRowsWarps) * N + n];
      const float d = part[(size_t)(p + 3 * kRowsWarps) * N + n];
      s += a;
      s += b;
      s += c;
      s += d;
    }
    for (; p < n_part; p += kRowsWarps) s += part[(size_t)p * N + n];
  }
  red[warp][lane] = s;
  __syncthreads();
  if (warp == 0 && n < N) {
    float t = red[0][lane];
#pragma unroll
    for (int w = 1; w < kRowsWarps; ++w) t += red[w][lane];
    out[n] = t;
  }
}

// Stage 1 of the bias gradient: CTA (chunk) sums rows [r0, r1) of a
// 128-column slab (lane = 4 consecutive columns, warp = rows strided by 8).
// With LO, the same pass also writes lo = y - trunc_tf32(y) (the GEMM operand
// split of y, compact), so the bias gradient of dY costs no extra read.
// With GELU, y is first replaced in place by y * gelu'(pre) (GeluBackward on
// the way in: the column sums, the lo part and y itself are of the product).
// The last CTA of each 128-column block (counted in `done`, zeroed before
// the launch) then sums that block's partials into out, in colsum_finish's
// order (the same result as the two-launch form), instead of a second launch.
template <bool LO, bool GELU>
__global__ void __launch_bounds__(256) colsum_partial(float* __restrict__ y, int M, int N,
                                                      int rows_per_cta, float* __restrict__ part,
                                                      float* __restrict__ lo,
                                                      const float* __restrict__ pre,
                                                      int* __restrict__ done,
                                                      float* __restrict__ out) {
  pdl_wait();     // the previous kernel's writes are visible (launched by launch_pdl)
  pdl_trigger();  // the next kernel, if launched as a programmatic dependent, may start
  __shared__ float4 red[kRowsWarps][32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int col = (blockIdx.x * 32 + lane) * 4;
  const int r0 = blockIdx.y * rows_per_cta;
  const int r1 = min(M, r0 + rows_per_cta);
  float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
  const bool vec = (N & 3) == 0;
  auto take = [&](int r, float4 v) {
    if (GELU) {
      const float4 x = *reinterpret_cast<const float4*>(pre + (size_t)r * N + col);
      v.x = __fmul_rn(v.x, gelu_grad_f(x.x));
      v.y = __fmul_rn(v.y, gelu_grad_f(x.y));
      v.z = __fmul_rn(v.z, gelu_grad_f(x.z));
      v.w = __fmul_rn(v.w, gelu_grad_f(x.w));
      *reinterpret_cast<float4*>(y + (size_t)r * N + col) = v;
    }
    s.x += v.x; s.y += v.y; s.z += v.z; s.w += v.w;
    if (LO) {
      float4 l;
      l.x = v.x - __uint_as_float(__float_as_uint(v.x) & 0xFFFFE000u);
      l.y = v.y - __uint_as_float(__float_as_uint(v.y) & 0xFFFFE000u);
      l.z = v.z - __uint_as_float(__float_as_uint(v.z) & 0xFFFFE000u);
      l.w = v.w - __uint_as_float(__float_as_uint(v.w) & 0xFFFFE000u);
      *reinterpret_cast<float4*>(lo + (size_t)r * N + col) = l;
    }
  };
  if (col < N) {
    int r = r0 + warp;
    if (vec) {
      // Four rows' loads in flight before they are added (in row order).
      for (; r + 3 * kRowsWarps < r1; r += 4 * kRowsWarps) {
        const float4 v0 = *reinterpret_cast<const float4*>(y + (size_t)r * N + col);
        const float4 v1 = *reinterpret_cast<const float4*>(y + (size_t)(r + kRowsWarps) * N + col);
        const float4 v2 = *reinterpret_cast<const float4*>(y + (size_t)(r + 2 * kRowsWarps) * N + col);
        const float4 v3 = *reinterpret_cast<const float4*>(y + (size_t)(r + 3 * kRowsWarps) * N + col);
        take(r, v0);
        take(r + kRowsWarps, v1);
        take(r + 2 * kRowsWarps, v2);
        take(r + 3 * kRowsWarps, v3);
      }
    }
    for (; r < r1; r += kRowsWarps) {
      const float* p = y + (size_t)r * N + col;
      if (vec) {
        take(r, *reinterpret_cast<const float4*>(p));
      } else {
        s.x += p[0];
        if (col + 1 < N) s.y += p[1];
        if (col + 2 < N) s.z += p[2];
        if (col + 3 < N) s.w += p[3];
      }
    }
  }
  red[warp][lane] = s;
  __syncthreads();
  if (warp == 0 && col < N) {
    float4 t = red[0][lane];
    for (int w = 1; w < kRowsWarps; ++w) {
      const float4 u = red[w][lane];
      t.x += u.x; t.y += u.y; t.z += u.z; t.w += u.w;
    }
    float* o = part + (size_t)blockIdx.y * N + col;
    o[0] = t.x;
    if (col + 1 < N) o[1] = t.y;
    if (col + 2 < N) o[2] = t.z;
    if (col + 3 < N) o[3] = t.w;
  }
  __shared__ int last;
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) last = atomicAdd(done + blockIdx.x, 1) == (int)gridDim.y - 1;
  __syncthreads();
  if (!last) return;
  __threadfence();
  // Warp w sums partial rows w, w+8, ... (ascending), then the eight warp sums
  // are added in warp order: colsum_finish's order, per column.
  const int n_part = (int)gridDim.y;
  float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
  if (col < N) {
    for (int q = warp; q < n_part; q += kRowsWarps) {
      const float* r = part + (size_t)q * N + col;
      a.x += __ldcg(r);
      if (col + 1 < N) a.y += __ldcg(r + 1);
      if (col + 2 < N) a.z += __ldcg(r + 2);
      if (col + 3 < N) a.w += __ldcg(r + 3);
    }
  }
  red[warp][lane] = a;
  __syncthreads();
  if (warp == 0 && col < N) {
    float4 t = red[0][lane];
    for (int w = 1; w < kRowsWarps; ++w) {
      const float4 u = red[w][lane];
      t.x += u.x; t.y += u.y; t.z += u.z; t.w += u.w;
    }
    out[col] = t.x;
    if (col + 1 < N) out[col + 1] = t.y;
    if (col + 2 < N) out[col + 2] = t.z;
    if (col + 3 < N) out[col + 3] = t.w;
  }
}

int ln_bwd_ctas(int rows) { return std::max(1, std::min(ceil_div(rows, 4 * kRowsWarps), kMaxPartials)); }

// Row chunks of the bias-gradient column sums: about eight CTAs per SM (the
// pass is memory-latency bound; two per SM reached 40 % of HBM bandwidth,
// eight 75 %), at least 64 rows per chunk.
int bias_chunks(int M, int N) {
  const int col_blocks = ceil_div(N, 128);
  const int want = std::max(1, (8 * sm_count()) / std::max(1, col_blocks));
  return std::max(1, std::min(std::min(want, ceil_div(M, 64)), 128));
}

}  // namespace
}  // namespace nsb

using namespace nsb;

extern "C" {

ns_status ns_layernorm_fwd(const float* x, const float* gamma, const float* beta, float* out,
                           float* mean, float* rstd, int rows, int dim, float eps, void* stream) {
  return ns_layernorm_fwd_ex(x, nullptr, nullptr, nullptr, gamma, beta, out, nullptr, mean, rstd,
                             rows, dim, eps, stream);
}

ns_status ns_layernorm_fwd_ex(const float* x, const float* bias, const float* resid, float* x_out,
                              const float* gamma, const float* beta, float* out, float* out_lo,
                              float* mean, float* rstd, int rows, int dim, float eps, void* stream) {
  NS_REQUIRE(rows >= 0 && dim > 0, "ns_layernorm_fwd: rows must be >= 0 and dim > 0");
  NS_REQUIRE(!resid || (bias && x_out), "ns_layernorm_fwd_ex: resid needs bias and x_out");
  if (rows == 0) return NS_OK;
  const dim3 grid(ceil_div(rows, kRowsWarps)), block(32 * kRowsWarps);
  cudaStream_t s = as_stream(stream);
  const bool aligned = ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(out) |
                         reinterpret_cast<uintptr_t>(gamma) | reinterpret_cast<uintptr_t>(beta) |
                         reinterpret_cast<uintptr_t>(bias) | reinterpret_cast<uintptr_t>(resid) |
                         reinterpret_cast<uintptr_t>(x_out) | reinterpret_cast<uintptr_t>(out_lo)) &
                        15) == 0;
  if (dim % 4 == 0 && aligned && dim <= 128 * kMaxVec) {
    const int nv = dim / 4;
    auto launch = [&](auto kernel) {
      return launch_pdl(kernel, grid, block, 0, s, "ns_layernorm_fwd", x, gamma, beta, out, mean,
                        rstd, rows, dim, eps, bias, resid, x_out, out_lo);
    };
    auto go = [&](auto nvt) {
      constexpr int NV = decltype(nvt)::value;
      if (resid && out_lo) return launch(ln_fwd_vec<NV, true, true>);
      if (resid) return launch(ln_fwd_vec<NV, true, false>);
      if (out_lo) return launch(ln_fwd_vec<NV, false, true>);
      return launch(ln_fwd_vec<NV, false, false>);
    };
    if (nv <= 32) return go(std::integral_constant<int, 1>());
    if (nv <= 64) return go(std::integral_constant<int, 2>());
    if (nv <= 128) return go(std::integral_constant<int, 4>());
    return go(std::integral_constant<int, 8>());
  }
  const float* xin = x;
  if (resid) {
    const int64_t n = (int64_t)rows * dim;
    const ns_status rc = launch_pdl(
        resid_bias_add_k, dim3((unsigned)std::min<int64_t>(ceil_div64(n, 256), 148 * 8)),
        dim3(256), 0, s, "ns_layernorm_fwd residual", x, bias, resid, x_out, (int64_t)rows, dim);
    if (rc != NS_OK) return rc;
    xin = x_out;
  }
  const ns_status rc = launch_pdl(ln_fwd_any, grid, block, 0, s, "ns_layernorm_fwd", xin, gamma,
                                  beta, out, mean, rstd, rows, dim, eps);
  if (rc != NS_OK) return rc;
  if (out_lo) return ns_split_lo(out, rows, dim, dim, out_lo, stream);
  return NS_OK;
}

size_t ns_layernorm_bwd_workspace_size(int rows, int dim) {
  if (rows <= 0 || dim <= 0) return 0;
  return (size_t)2 * ln_bwd_ctas(rows) * dim * sizeof(float);
}

ns_status ns_layernorm_bwd(const float* dout, const float* x, const float* gamma,
                           const float* mean, const float* rstd, const float* dresid, float* dx,
                           float* dgamma, float* dbeta, int rows, int dim, void* workspace,
                           size_t workspace_bytes, void* stream) {
  NS_REQUIRE(rows >= 0 && dim > 0, "ns_layernorm_bwd: rows must be >= 0 and dim > 0");
  cudaStream_t s = as_stream(stream);
  if (rows == 0) {
    NS_TRY_CUDA(cudaMemsetAsync(dgamma, 0, sizeof(float) * dim, s), "ns_layernorm_bwd memset");
    NS_TRY_CUDA(cudaMemsetAsync(dbeta, 0, sizeof(float) * dim, s), "ns_layernorm_bwd memset");
    return NS_OK;
  }
  NS_REQUIRE(workspace_bytes >= ns_layernorm_bwd_workspace_size(rows, dim) && workspace,
             "ns_layernorm_bwd: workspace too small");
  const int ctas = ln_bwd_ctas(rows);
  const int rpc = ceil_div(rows, ctas);
  float* part_g = static_cast<float*>(workspace);
  float* part_b = part_g + (size_t)ctas * dim;
  const dim3 block(32 * kRowsWarps);
  const uintptr_t al = reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(dout) |
                       reinterpret_cast<uintptr_t>(dx) | reinterpret_cast<uintptr_t>(gamma) |
                       reinterpret_cast<uintptr_t>(dresid);
  // stage 1: dx and the per-CTA partial column sums; stage 2: the ordered sums
  auto stage1 = [&](auto kernel, size_t smem) {
    return launch_pdl(kernel, dim3(ctas), block, smem, s, "ns_layernorm_bwd stage 1", dout, x,
                      gamma, mean, rstd, dresid, dx, part_g, part_b, rows, dim, rpc);
  };
  auto stage1_big = [&](auto kernel, size_t smem) {
    NS_TRY_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)smem), "ns_layernorm_bwd attr");
    return stage1(kernel, smem);
  };
  ns_status rc;
  if (dim % 4 == 0 && (al & 15) == 0 && dim <= 128 * kMaxVec) {
    const int nv = dim / 4;
    const size_t smem = (size_t)kRowsWarps * 2 * dim * sizeof(float);
    if (nv <= 16)  // short rows (the U-Net's last-axis LayerNorms): more rows in flight
      rc = stage1(ln_bwd_vec<1, 8>, smem);
    else if (nv <= 32)
      rc = stage1(ln_bwd_vec<1, 2>, smem);
    else if (nv <= 64)
      rc = stage1(ln_bwd_vec<2, 2>, smem);
    else if (nv <= 96)
      rc = stage1(ln_bwd_vec<3, 2>, smem);
    else if (nv <= 128)
      rc = stage1_big(ln_bwd_vec<4, 2>, smem);
    else if (nv <= 192)  // dim <= 768: six float4 per lane, not eight (registers decide occupancy)
      rc = stage1_big(ln_bwd_vec<6, 2>, smem);
    else
      rc = stage1_big(ln_bwd_vec<8, 1>, smem);
  } else {
    rc = stage1(ln_bwd_any, 0);
  }
  if (rc != NS_OK) return rc;
  return launch_pdl(colsum_finish, dim3(ceil_div(dim, 32), 2), dim3(256), 0, s,
                    "ns_layernorm_bwd stage 2", part_g, ctas, dim, dgamma, part_b, dbeta);
}

size_t ns_bias_grad_workspace_size(int M, int N) {
  if (M <= 0 || N <= 0) return 0;
  // partials, then one completion counter per 128-column block
  const size_t part = ((size_t)bias_chunks(M, N) * N * sizeof(float) + 255) & ~(size_t)255;
  return part + (size_t)ceil_div(N, 128) * sizeof(int);
}

ns_status ns_bias_grad(const float* dY, int M, int N, float* db, void* workspace,
                       size_t workspace_bytes, void* stream) {
  NS_REQUIRE(M >= 0 && N > 0, "ns_bias_grad: bad shape");
  cudaStream_t s = as_stream(stream);
  if (M == 0) {
    NS_TRY_CUDA(cudaMemsetAsync(db, 0, sizeof(float) * N, s), "ns_bias_grad memset");
    return NS_OK;
  }
  NS_REQUIRE(workspace && workspace_bytes >= ns_bias_grad_workspace_size(M, N),
             "ns_bias_grad: workspace too small");
  NS_REQUIRE((reinterpret_cast<uintptr_t>(dY) & 15) == 0 || (N & 3) != 0,
             "ns_bias_grad: dY must be 16-byte aligned");
  const int chunks = bias_chunks(M, N);
  const int rpc = ceil_div(M, chunks);
  float* part = static_cast<float*>(workspace);
  int* done = reinterpret_cast<int*>(static_cast<char*>(workspace) +
                                     (((size_t)chunks * N * sizeof(float) + 255) & ~(size_t)255));
  NS_TRY_CUDA(cudaMemsetAsync(done, 0, (size_t)ceil_div(N, 128) * sizeof(int), s), "ns_bias_grad counters");
  return launch_pdl(colsum_partial<false, false>, dim3(ceil_div(N, 128), chunks), dim3(256),
                    0, s, "ns_bias_grad", const_cast<float*>(dY), M, N, rpc, part, nullptr, nullptr,
                    done, db);
}

ns_status ns_bias_grad_split(const float* dY, int M, int N, float* db, float* dy_lo,
                             void* workspace, size_t workspace_bytes, void* stream) {
  NS_REQUIRE(M > 0 && N > 0 && (N & 3) == 0, "ns_bias_grad_split: N must be a positive multiple of 4");
  NS_REQUIRE(((reinterpret_cast<uintptr_t>(dY) | reinterpret_cast<uintptr_t>(dy_lo)) & 15) == 0,
             "ns_bias_grad_split: dY and dy_lo must be 16-byte aligned");
  NS_REQUIRE(workspace && workspace_bytes >= ns_bias_grad_workspace_size(M, N),
             "ns_bias_grad_split: workspace too small");
  cudaStream_t s = as_stream(stream);
  const int chunks = bias_chunks(M, N);
  const int rpc = ceil_div(M, chunks);
  float* part = static_cast<float*>(workspace);
  int* done = reinterpret_cast<int*>(static_cast<char*>(workspace) +
                                     (((size_t)chunks * N * sizeof(float) + 255) & ~(size_t)255));
  NS_TRY_CUDA(cudaMemsetAsync(done, 0, (size_t)ceil_div(N, 128) * sizeof(int), s), "ns_bias_grad_split counters");
  return launch_pdl(colsum_partial<true, false>, dim3(ceil_div(N, 128), chunks), dim3(256), 0,
                    s, "ns_bias_grad_split", const_cast<float*>(dY), M, N, rpc, part, dy_lo,
                    nullptr, done, db);
}

ns_status ns_bias_grad_split_gelu(float* dY, const float* pre, int M, int N, float* db, float* dy_lo,
                                  void* workspace, size_t workspace_bytes, void* stream) {
  NS_REQUIRE(M > 0 && N > 0 && (N & 3) == 0,
             "ns_bias_grad_split_gelu: N must be a positive multiple of 4");
  NS_REQUIRE(((reinterpret_cast<uintptr_t>(dY) | reinterpret_cast<uintptr_t>(dy_lo) |
               reinterpret_cast<uintptr_t>(pre)) & 15) == 0,
             "ns_bias_grad_split_gelu: dY, pre and dy_lo must be 16-byte aligned");
  NS_REQUIRE(workspace && workspace_bytes >= ns_bias_grad_workspace_size(M, N),
             "ns_bias_grad_split_gelu: workspace too small");
  cudaStream_t s = as_stream(stream);
  const int chunks = bias_chunks(M, N);
  const int rpc = ceil_div(M, chunks);
  float* part = static_cast<float*>(workspace);
  int* done = reinterpret_cast<int*>(static_cast<char*>(workspace) +
                                     (((size_t)chunks * N * sizeof(float) + 255) & ~(size_t)255));
  NS_TRY_CUDA(cudaMemsetAsync(done, 0, (size_t)ceil_div(N, 128) * sizeof(int), s), "ns_bias_grad_split_gelu counters");
  return launch_pdl(colsum_partial<true, true>, dim3(ceil_div(N, 128), chunks), dim3(256), 0,
                    s, "ns_bias_grad_split_gelu", dY, M, N, rpc, part, dy_lo, pre, done, db);
}

}  // extern "C"
