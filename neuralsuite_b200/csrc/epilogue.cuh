// GEMM epilogues shared by the tcgen05 kernel, the SIMT kernel and the
// split-K reduction.  `acc` is the fp32 GEMM result of element (m, n).
#pragma once

#include "common.cuh"

namespace nsb {

struct EpiArgs {
  float* C;
  int ldc;
  int epi;
  float beta;
  const float* bias;
  const float* aux;
  float* aux_out;
  // Optional: the tf32 lo part (x - trunc_tf32(x)) of the epilogue's
  // activation output (aux_out for NS_EPI_BIAS_GELU, C otherwise), row
  // stride ldc: the next GEMM's operand split, written in the same pass.
  float* lo_out;
};

__device__ __forceinline__ float epi_lo(float x) {
  return x - __uint_as_float(__float_as_uint(x) & 0xFFFFE000u);
}

// Writes element (m, n); m < M and n < N are the caller's responsibility.
__device__ __forceinline__ void epi_store(const EpiArgs& e, int m, int n, float acc) {
  const size_t off = (size_t)m * e.ldc + n;
  float out;  // the activation output (lo_out's source)
  switch (e.epi) {
    case NS_EPI_STORE:
      out = (e.beta != 0.0f) ? __fadd_rn(e.C[off], acc) : acc;
      e.C[off] = out;
      break;
    case NS_EPI_BIAS:
      out = __fadd_rn(acc, e.bias[n]);
      e.C[off] = out;
      break;
    case NS_EPI_BIAS_GELU: {
      const float v = __fadd_rn(acc, e.bias[n]);
      e.C[off] = v;
      out = gelu_f(v);
      e.aux_out[off] = out;
      break;
    }
    case NS_EPI_BIAS_RESID:
      out = __fadd_rn(e.aux[off], __fadd_rn(acc, e.bias[n]));
      e.C[off] = out;
      break;
    case NS_EPI_GELU_BWD:
      out = __fmul_rn(acc, gelu_grad_f(e.aux[off]));
      e.C[off] = out;
      break;
    default:
      return;
  }
  if (e.lo_out) e.lo_out[off] = epi_lo(out);
}

// Four consecutive columns n..n+3 of row m (16-byte aligned, all in range).
__device__ __forceinline__ void epi_store4(const EpiArgs& e, int m, int n, float4 a) {
  const size_t off = (size_t)m * e.ldc + n;
  float4 r;
  switch (e.epi) {
    case NS_EPI_STORE:
      if (e.beta != 0.0f) {
        const float4 c = *reinterpret_cast<const float4*>(e.C + off);
        r = make_float4(__fadd_rn(c.x, a.x), __fadd_rn(c.y, a.y), __fadd_rn(c.z, a.z),
                        __fadd_rn(c.w, a.w));
      } else {
        r = a;
      }
      break;
    case NS_EPI_BIAS: {
      const float4 b = *reinterpret_cast<const float4*>(e.bias + n);
      r = make_float4(__fadd_rn(a.x, b.x), __fadd_rn(a.y, b.y), __fadd_rn(a.z, b.z),
                      __fadd_rn(a.w, b.w));
      break;
    }
    case NS_EPI_BIAS_GELU: {
      const float4 b = *reinterpret_cast<const float4*>(e.bias + n);
      r = make_float4(__fadd_rn(a.x, b.x), __fadd_rn(a.y, b.y), __fadd_rn(a.z, b.z),
                      __fadd_rn(a.w, b.w));
      const float4 g = make_float4(gelu_f(r.x), gelu_f(r.y), gelu_f(r.z), gelu_f(r.w));
      *reinterpret_cast<float4*>(e.aux_out + off) = g;
      if (e.lo_out)
        *reinterpret_cast<float4*>(e.lo_out + off) =
            make_float4(epi_lo(g.x), epi_lo(g.y), epi_lo(g.z), epi_lo(g.w));
      *reinterpret_cast<float4*>(e.C + off) = r;
      return;
    }
    case NS_EPI_BIAS_RESID: {
      const float4 b = *reinterpret_cast<const float4*>(e.bias + n);
      const float4 x = *reinterpret_cast<const float4*>(e.aux + off);
      r = make_float4(__fadd_rn(x.x, __fadd_rn(a.x, b.x)), __fadd_rn(x.y, __fadd_rn(a.y, b.y)),
                      __fadd_rn(x.z, __fadd_rn(a.z, b.z)), __fadd_rn(x.w, __fadd_rn(a.w, b.w)));
      break;
    }
    case NS_EPI_GELU_BWD: {
      const float4 x = *reinterpret_cast<const float4*>(e.aux + off);
      r = make_float4(__fmul_rn(a.x, gelu_grad_f(x.x)), __fmul_rn(a.y, gelu_grad_f(x.y)),
                      __fmul_rn(a.z, gelu_grad_f(x.z)), __fmul_rn(a.w, gelu_grad_f(x.w)));
      break;
    }
    default:
      return;
  }
  *reinterpret_cast<float4*>(e.C + off) = r;
  if (e.lo_out)
    *reinterpret_cast<float4*>(e.lo_out + off) =
        make_float4(epi_lo(r.x), epi_lo(r.y), epi_lo(r.z), epi_lo(r.w));
}

// Stores `count` (<= R) consecutive rows m0.. of column n, values v[0..count):
// the transposed GEMM epilogue.  The switch sits outside the loop, so each
// epilogue kind is one straight-line loop over registers.
template <int R>
__device__ __forceinline__ void epi_store_col(const EpiArgs& e, int m0, int n, int count,
                                              const float (&v)[R]) {
  float* c = e.C + (size_t)m0 * e.ldc + n;
  const size_t ld = (size_t)e.ldc;
  float* lo = e.lo_out ? e.lo_out + (size_t)m0 * e.ldc + n : nullptr;
  switch (e.epi) {
    case NS_EPI_STORE:
      if (e.beta != 0.0f) {
#pragma unroll
        for (int j = 0; j < R; ++j)
          if (j < count) {
            const float x = __fadd_rn(c[j * ld], v[j]);
            c[j * ld] = x;
            if (lo) lo[j * ld] = epi_lo(x);
          }
      } else {
#pragma unroll
        for (int j = 0; j < R; ++j)
          if (j < count) {
            c[j * ld] = v[j];
            if (lo) lo[j * ld] = epi_lo(v[j]);
          }
      }
      break;
    case NS_EPI_BIAS: {
      const float b = e.bias[n];
#pragma unroll
      for (int j = 0; j < R; ++j)
        if (j < count) {
          const float x = __fadd_rn(v[j], b);
          c[j * ld] = x;
          if (lo) lo[j * ld] = epi_lo(x);
        }
      break;
    }
    case NS_EPI_BIAS_GELU: {
      const float b = e.bias[n];
      float* g = e.aux_out + (size_t)m0 * e.ldc + n;
#pragma unroll
      for (int j = 0; j < R; ++j)
        if (j < count) {
          const float x = __fadd_rn(v[j], b);
          c[j * ld] = x;
          const float y = gelu_f(x);
          g[j * ld] = y;
          if (lo) lo[j * ld] = epi_lo(y);
        }
      break;
    }
    case NS_EPI_BIAS_RESID: {
      const float b = e.bias[n];
      const float* r = e.aux + (size_t)m0 * e.ldc + n;
#pragma unroll
      for (int j = 0; j < R; ++j)
        if (j < count) {
          const float x = __fadd_rn(r[j * ld], __fadd_rn(v[j], b));
          c[j * ld] = x;
          if (lo) lo[j * ld] = epi_lo(x);
        }
      break;
    }
    case NS_EPI_GELU_BWD: {
      const float* r = e.aux + (size_t)m0 * e.ldc + n;
#pragma unroll
      for (int j = 0; j < R; ++j)
        if (j < count) {
          const float x = __fmul_rn(v[j], gelu_grad_f(r[j * ld]));
          c[j * ld] = x;
          if (lo) lo[j * ld] = epi_lo(x);
        }
      break;
    }
    default:
      break;
  }
}

}  // namespace nsb
