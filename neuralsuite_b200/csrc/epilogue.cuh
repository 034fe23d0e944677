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
};

// Writes element (m, n); m < M and n < N are the caller's responsibility.
__device__ __forceinline__ void epi_store(const EpiArgs& e, int m, int n, float acc) {
  const size_t off = (size_t)m * e.ldc + n;
  switch (e.epi) {
    case NS_EPI_STORE:
      e.C[off] = (e.beta != 0.0f) ? __fadd_rn(e.C[off], acc) : acc;
      break;
    case NS_EPI_BIAS:
      e.C[off] = __fadd_rn(acc, e.bias[n]);
      break;
    case NS_EPI_BIAS_GELU: {
      const float v = __fadd_rn(acc, e.bias[n]);
      e.C[off] = v;
      e.aux_out[off] = gelu_f(v);
      break;
    }
    case NS_EPI_BIAS_RESID:
      e.C[off] = __fadd_rn(e.aux[off], __fadd_rn(acc, e.bias[n]));
      break;
    case NS_EPI_GELU_BWD:
      e.C[off] = __fmul_rn(acc, gelu_grad_f(e.aux[off]));
      break;
    default:
      break;
  }
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
      *reinterpret_cast<float4*>(e.aux_out + off) =
          make_float4(gelu_f(r.x), gelu_f(r.y), gelu_f(r.z), gelu_f(r.w));
      break;
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
}

// Stores `count` (<= R) consecutive rows m0.. of column n, values v[0..count):
// the transposed GEMM epilogue.  The switch sits outside the loop, so each
// epilogue kind is one straight-line loop over registers.
template <int R>
__device__ __forceinline__ void epi_store_col(const EpiArgs& e, int m0, int n, int count,
                                              const float (&v)[R]) {
  float* c = e.C + (size_t)m0 * e.ldc + n;
  const size_t ld = (size_t)e.ldc;
  switch (e.epi) {
    case NS_EPI_STORE:
      if (e.beta != 0.0f) {
#pragma unroll
        for (int j = 0; j < R; ++j)
          if (j < count) c[j * ld] = __fadd_rn(c[j * ld], v[j]);
      } else {
#pragma unroll
        for (int j = 0; j < R; ++j)
          if (j < count) c[j * ld] = v[j];
      }
      break;
    case NS_EPI_BIAS: {
      const float b = e.bias[n];
#pragma unroll
      for (int j = 0; j < R; ++j)
        if (j < count) c[j * ld] = __fadd_rn(v[j], b);
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
          g[j * ld] = gelu_f(x);
        }
      break;
    }
    case NS_EPI_BIAS_RESID: {
      const float b = e.bias[n];
      const float* r = e.aux + (size_t)m0 * e.ldc + n;
#pragma unroll
      for (int j = 0; j < R; ++j)
        if (j < count) c[j * ld] = __fadd_rn(r[j * ld], __fadd_rn(v[j], b));
      break;
    }
    case NS_EPI_GELU_BWD: {
      const float* r = e.aux + (size_t)m0 * e.ldc + n;
#pragma unroll
      for (int j = 0; j < R; ++j)
        if (j < count) c[j * ld] = __fmul_rn(v[j], gelu_grad_f(r[j * ld]));
      break;
    }
    default:
      break;
  }
}

}  // namespace nsb
