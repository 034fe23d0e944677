// K2: fused causal self-attention, forward and backward, on the interleaved
// c_attn output (no Extraer copies, no [B,H,T,T] probability cache).
//
// Forward (MultiHeadAttention::Forward, include/layers/attention.h:364-384):
// per (b, h, 64-query block), stream 64-key blocks 0..qb through shared
// memory, online softmax over the scaled scores S = (Q.K^T) * (1/sqrt(D)),
// O = P.V / l, and store lse = m + log(l) per query row.  Only causal tiles are
// visited (the reference computes the full square and zeroes the upper
// triangle, attention.h:316-322).
//
// Backward (attention.h:392-467): P is recomputed from lse; the reference's
// row sum  sum_j dP_ij P_ij  (computed there in double, attention.h:432-443)
// equals  Delta_i = dO_i . O_i, computed once per row here.  dK/dV are
// accumulated by a key-block kernel and dQ by a query-block kernel, so every
// output element has exactly one writer: deterministic, no atomics.
//
// fp32 SIMT: each thread owns a 4 x 4 tile of the 64 x 64 score block.
#include <algorithm>

#include "attention_tc.cuh"
#include "common.cuh"

namespace nsb {
namespace {

// 0 auto (tensor cores where supported, dK and dV from one kernel), 1 SIMT,
// 2 tensor cores with dK and dV from separate kernels (a cross-check).
thread_local int t_attn_engine = 0;

constexpr int kBr = 64;   // query rows per block
constexpr int kBc = 64;   // keys per block
constexpr int kThreads = 256;
constexpr int kPLD = kBc + 1;  // padded row of the P / dS tiles

template <int DP>
struct AttnTile {
  static constexpr int LD = DP + 1;
  static constexpr int KD = DP / 16;  // head-dim columns per thread
};

// Loads rows [r0, r0+64) of one head's D columns (column offset `col`) of a
// row-major matrix with row stride `ld` into smem [64][LD], zero-padded.
template <int DP>
__device__ __forceinline__ void load_tile(float* dst, const float* __restrict__ src, size_t ld,
                                          int col, int r0, int T, int D) {
  constexpr int LD = AttnTile<DP>::LD;
  for (int idx = threadIdx.x; idx < kBr * DP; idx += kThreads) {
    const int r = idx / DP, d = idx % DP;
    dst[r * LD + d] = (r0 + r < T && d < D) ? src[(size_t)(r0 + r) * ld + col + d] : 0.0f;
  }
}

template <int DP>
__global__ void __launch_bounds__(kThreads) attn_fwd_k(const float* __restrict__ qkv,
                                                       float* __restrict__ out,
                                                       float* __restrict__ lse, int T, int H,
                                                       int D, float scale) {
  constexpr int LD = AttnTile<DP>::LD, KD = AttnTile<DP>::KD;
  extern __shared__ float sm[];
  float* Qs = sm;
  float* Ks = Qs + kBr * LD;
  float* Vs = Ks + kBc * LD;
  float* Ps = Vs + kBc * LD;
  const int nqb = (T + kBr - 1) / kBr;
  const int qb = nqb - 1 - (int)blockIdx.x;  // longest rows first
  const int bh = blockIdx.y, b = bh / H, h = bh % H;
  const int C = H * D;
  const size_t ld = (size_t)3 * C;
  const float* base = qkv + (size_t)b * T * ld;
  const int q0 = qb * kBr;
  const int tid = threadIdx.x, ty = tid >> 4, tx = tid & 15;

  load_tile<DP>(Qs, base, ld, h * D, q0, T, D);
  float o[4][KD];
  float m_i[4], l_i[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    m_i[i] = -INFINITY;
    l_i[i] = 0.0f;
#pragma unroll
    for (int k = 0; k < KD; ++k) o[i][k] = 0.0f;
  }
  for (int kb = 0; kb <= qb; ++kb) {
    const int k0 = kb * kBc;
    __syncthreads();
    load_tile<DP>(Ks, base, ld, C + h * D, k0, T, D);
    load_tile<DP>(Vs, base, ld, 2 * C + h * D, k0, T, D);
    __syncthreads();
    float s[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) s[i][j] = 0.0f;
#pragma unroll 8
    for (int d = 0; d < DP; ++d) {
      float qv[4], kv[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) qv[i] = Qs[(ty * 4 + i) * LD + d];
#pragma unroll
      for (int j = 0; j < 4; ++j) kv[j] = Ks[(tx + 16 * j) * LD + d];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) s[i][j] = fmaf(qv[i], kv[j], s[i][j]);
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int r = q0 + ty * 4 + i;
      float mx = -INFINITY;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int c = k0 + tx + 16 * j;
        s[i][j] = (c <= r && c < T) ? s[i][j] * scale : -INFINITY;
        mx = fmaxf(mx, s[i][j]);
      }
#pragma unroll
      for (int off = 8; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
      const float m_new = fmaxf(m_i[i], mx);
      float rs = 0.0f;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float p = (s[i][j] == -INFINITY) ? 0.0f : expf(s[i][j] - m_new);
        Ps[(ty * 4 + i) * kPLD + tx + 16 * j] = p;
        rs += p;
      }
#pragma unroll
      for (int off = 8; off > 0; off >>= 1) rs += __shfl_xor_sync(0xffffffffu, rs, off);
      const float alpha = (m_i[i] == -INFINITY) ? 0.0f : expf(m_i[i] - m_new);
      l_i[i] = l_i[i] * alpha + rs;
      m_i[i] = m_new;
#pragma unroll
      for (int k = 0; k < KD; ++k) o[i][k] *= alpha;
    }
    __syncthreads();
#pragma unroll 4
    for (int c = 0; c < kBc; ++c) {
      float pv[4], vv[KD];
#pragma unroll
      for (int i = 0; i < 4; ++i) pv[i] = Ps[(ty * 4 + i) * kPLD + c];
#pragma unroll
      for (int k = 0; k < KD; ++k) vv[k] = Vs[c * LD + tx + 16 * k];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int k = 0; k < KD; ++k) o[i][k] = fmaf(pv[i], vv[k], o[i][k]);
    }
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int r = q0 + ty * 4 + i;
    if (r < T) {
      const float inv = 1.0f / l_i[i];
#pragma unroll
      for (int k = 0; k < KD; ++k) {
        const int d = tx + 16 * k;
        if (d < D) out[((size_t)b * T + r) * C + h * D + d] = o[i][k] * inv;
      }
      if (tx == 0) lse[(size_t)bh * T + r] = m_i[i] + logf(l_i[i]);
    }
  }
}

// Delta[bh, r] = sum_d dO[b, r, h*D + d] * O[b, r, h*D + d]: one warp per
// (b, r) row of all heads, lanes striding the C columns (coalesced), each
// head's D products summed by its lanes with shuffles.
// With dout_lo, the pass also writes dout's tf32 lo part (the tensor-core
// backward's operand split of dO) from the same loads.
__global__ void __launch_bounds__(256) attn_delta_k(const float* __restrict__ out,
                                                    const float* __restrict__ dout, int B, int T,
                                                    int H, int D, float* __restrict__ delta,
                                                    float* __restrict__ dout_lo) {
  pdl_wait();     // the previous kernel's writes are visible (launched by launch_pdl)
  pdl_trigger();  // the next kernel, if launched as a programmatic dependent, may start
  const int64_t row = blockIdx.x * 8 + (threadIdx.x >> 5);  // b * T + r
  const int lane = threadIdx.x & 31;
  if (row >= (int64_t)B * T) return;
  const int b = (int)(row / T), r = (int)(row % T);
  const int C = H * D;
  const float* o = out + row * C;
  const float* g = dout + row * C;
  if (D % 32 == 0) {
    // lanes cover 32 consecutive columns of one head per step
    for (int h = 0; h < H; ++h) {
      float s = 0.0f;
      for (int d = lane; d < D; d += 32) {
        const float gv = g[h * D + d];
        s = fmaf(gv, o[h * D + d], s);
        if (dout_lo) dout_lo[row * C + h * D + d] = gv - __uint_as_float(__float_as_uint(gv) & 0xFFFFE000u);
      }
      s = warp_sum(s);
      if (lane == 0) delta[((size_t)b * H + h) * T + r] = s;
    }
  } else {
    for (int h = lane; h < H; h += 32) {
      float s = 0.0f;
      for (int d = 0; d < D; ++d) {
        const float gv = g[h * D + d];
        s = fmaf(gv, o[h * D + d], s);
        if (dout_lo) dout_lo[row * C + h * D + d] = gv - __uint_as_float(__float_as_uint(gv) & 0xFFFFE000u);
      }
      delta[((size_t)b * H + h) * T + r] = s;
    }
  }
}

// Scores and dP of one (query block, key block) pair into P / dS smem tiles.
template <int DP>
__device__ __forceinline__ void scores_and_ds(const float* Qs, const float* dOs, const float* Ks,
                                              const float* Vs, const float* Ls, const float* Dl,
                                              float* Ps, float* dSs, int q0, int k0, int T,
                                              float scale) {
  constexpr int LD = AttnTile<DP>::LD;
  const int tid = threadIdx.x, ty = tid >> 4, tx = tid & 15;
  float s[4][4], dp[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) s[i][j] = dp[i][j] = 0.0f;
#pragma unroll 8
  for (int d = 0; d < DP; ++d) {
    float qv[4], gv[4], kv[4], vv[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      qv[i] = Qs[(ty * 4 + i) * LD + d];
      gv[i] = dOs[(ty * 4 + i) * LD + d];
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      kv[j] = Ks[(tx + 16 * j) * LD + d];
      vv[j] = Vs[(tx + 16 * j) * LD + d];
    }
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        s[i][j] = fmaf(qv[i], kv[j], s[i][j]);
        dp[i][j] = fmaf(gv[i], vv[j], dp[i][j]);
      }
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int rl = ty * 4 + i, r = q0 + rl;
    const float L = Ls[rl], Dv = Dl[rl];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int cl = tx + 16 * j, c = k0 + cl;
      const bool ok = c <= r && c < T && r < T;
      const float p = ok ? expf(s[i][j] * scale - L) : 0.0f;
      Ps[rl * kPLD + cl] = p;
      dSs[rl * kPLD + cl] = p * (dp[i][j] - Dv) * scale;
    }
  }
}

template <int DP>
__global__ void __launch_bounds__(kThreads) attn_bwd_dkdv_k(
    const float* __restrict__ qkv, const float* __restrict__ dout, const float* __restrict__ lse,
    const float* __restrict__ delta, float* __restrict__ dqkv, int T, int H, int D, float scale) {
  constexpr int LD = AttnTile<DP>::LD, KD = AttnTile<DP>::KD;
  extern __shared__ float sm[];
  float* Ks = sm;
  float* Vs = Ks + kBc * LD;
  float* Qs = Vs + kBc * LD;
  float* dOs = Qs + kBr * LD;
  float* Ps = dOs + kBr * LD;
  float* dSs = Ps + kBr * kPLD;
  float* Ls = dSs + kBr * kPLD;
  float* Dl = Ls + kBr;
  const int nkb = (T + kBc - 1) / kBc;
  const int kb = nkb - 1 - (int)blockIdx.x;  // fewest query blocks last
  const int bh = blockIdx.y, b = bh / H, h = bh % H;
  const int C = H * D;
  const size_t ld = (size_t)3 * C;
  const float* base = qkv + (size_t)b * T * ld;
  const float* gbase = dout + (size_t)b * T * C;
  const int k0 = kb * kBc;
  const int tid = threadIdx.x, ty = tid >> 4, tx = tid & 15;
  load_tile<DP>(Ks, base, ld, C + h * D, k0, T, D);
  load_tile<DP>(Vs, base, ld, 2 * C + h * D, k0, T, D);
  float dk[4][KD], dv[4][KD];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int k = 0; k < KD; ++k) dk[i][k] = dv[i][k] = 0.0f;
  const int nqb = (T + kBr - 1) / kBr;
  for (int qb = kb; qb < nqb; ++qb) {
    const int q0 = qb * kBr;
    __syncthreads();
    load_tile<DP>(Qs, base, ld, h * D, q0, T, D);
    load_tile<DP>(dOs, gbase, (size_t)C, h * D, q0, T, D);
    if (tid < kBr) {
      const int r = q0 + tid;
      Ls[tid] = r < T ? lse[(size_t)bh * T + r] : 0.0f;
      Dl[tid] = r < T ? delta[(size_t)bh * T + r] : 0.0f;
    }
    __syncthreads();
    scores_and_ds<DP>(Qs, dOs, Ks, Vs, Ls, Dl, Ps, dSs, q0, k0, T, scale);
    __syncthreads();
    // dV[c] += sum_r P[r][c] dO[r];  dK[c] += sum_r dS[r][c] Q[r]   (c = ty*4 + i)
#pragma unroll 4
    for (int r = 0; r < kBr; ++r) {
      float pr[4], sr[4], gv[KD], qv[KD];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        pr[i] = Ps[r * kPLD + ty * 4 + i];
        sr[i] = dSs[r * kPLD + ty * 4 + i];
      }
#pragma unroll
      for (int k = 0; k < KD; ++k) {
        gv[k] = dOs[r * LD + tx + 16 * k];
        qv[k] = Qs[r * LD + tx + 16 * k];
      }
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int k = 0; k < KD; ++k) {
          dv[i][k] = fmaf(pr[i], gv[k], dv[i][k]);
          dk[i][k] = fmaf(sr[i], qv[k], dk[i][k]);
        }
    }
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int c = k0 + ty * 4 + i;
    if (c < T) {
      float* row = dqkv + ((size_t)b * T + c) * ld;
#pragma unroll
      for (int k = 0; k < KD; ++k) {
        const int d = tx + 16 * k;
        if (d < D) {
          row[C + h * D + d] = dk[i][k];
          row[2 * C + h * D + d] = dv[i][k];
        }
      }
    }
  }
}

template <int DP>
__global__ void __launch_bounds__(kThreads) attn_bwd_dq_k(
    const float* __restrict__ qkv, const float* __restrict__ dout, const float* __restrict__ lse,
    const float* __restrict__ delta, float* __restrict__ dqkv, int T, int H, int D, float scale) {
  constexpr int LD = AttnTile<DP>::LD, KD = AttnTile<DP>::KD;
  extern __shared__ float sm[];
  float* Qs = sm;
  float* dOs = Qs + kBr * LD;
  float* Ks = dOs + kBr * LD;
  float* Vs = Ks + kBc * LD;
  float* Ps = Vs + kBc * LD;
  float* dSs = Ps + kBr * kPLD;
  float* Ls = dSs + kBr * kPLD;
  float* Dl = Ls + kBr;
  const int nqb = (T + kBr - 1) / kBr;
  const int qb = nqb - 1 - (int)blockIdx.x;
  const int bh = blockIdx.y, b = bh / H, h = bh % H;
  const int C = H * D;
  const size_t ld = (size_t)3 * C;
  const float* base = qkv + (size_t)b * T * ld;
  const float* gbase = dout + (size_t)b * T * C;
  const int q0 = qb * kBr;
  const int tid = threadIdx.x, ty = tid >> 4, tx = tid & 15;
  load_tile<DP>(Qs, base, ld, h * D, q0, T, D);
  load_tile<DP>(dOs, gbase, (size_t)C, h * D, q0, T, D);
  if (tid < kBr) {
    const int r = q0 + tid;
    Ls[tid] = r < T ? lse[(size_t)bh * T + r] : 0.0f;
    Dl[tid] = r < T ? delta[(size_t)bh * T + r] : 0.0f;
  }
  float dq[4][KD];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int k = 0; k < KD; ++k) dq[i][k] = 0.0f;
  for (int kb = 0; kb <= qb; ++kb) {
    const int k0 = kb * kBc;
    __syncthreads();
    load_tile<DP>(Ks, base, ld, C + h * D, k0, T, D);
    load_tile<DP>(Vs, base, ld, 2 * C + h * D, k0, T, D);
    __syncthreads();
    scores_and_ds<DP>(Qs, dOs, Ks, Vs, Ls, Dl, Ps, dSs, q0, k0, T, scale);
    __syncthreads();
    // dQ[r] += sum_c dS[r][c] K[c]   (r = ty*4 + i)
#pragma unroll 4
    for (int c = 0; c < kBc; ++c) {
      float sv[4], kv[KD];
#pragma unroll
      for (int i = 0; i < 4; ++i) sv[i] = dSs[(ty * 4 + i) * kPLD + c];
#pragma unroll
      for (int k = 0; k < KD; ++k) kv[k] = Ks[c * LD + tx + 16 * k];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int k = 0; k < KD; ++k) dq[i][k] = fmaf(sv[i], kv[k], dq[i][k]);
    }
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int r = q0 + ty * 4 + i;
    if (r < T) {
      float* row = dqkv + ((size_t)b * T + r) * ld;
#pragma unroll
      for (int k = 0; k < KD; ++k) {
        const int d = tx + 16 * k;
        if (d < D) row[h * D + d] = dq[i][k];
      }
    }
  }
}

template <int DP>
size_t fwd_smem() { return (size_t)(3 * 64 * AttnTile<DP>::LD + 64 * kPLD) * sizeof(float); }
template <int DP>
size_t bwd_smem() {
  return (size_t)(4 * 64 * AttnTile<DP>::LD + 2 * 64 * kPLD + 2 * 64) * sizeof(float);
}

template <int DP>
ns_status launch_fwd(const float* qkv, int B, int T, int H, int D, float* out, float* lse,
                     cudaStream_t s) {
  const size_t smem = fwd_smem<DP>();
  NS_TRY_CUDA(cudaFuncSetAttribute(attn_fwd_k<DP>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   (int)smem), "ns_attn_fwd attr");
  const dim3 grid((T + kBr - 1) / kBr, B * H);
  attn_fwd_k<DP><<<grid, kThreads, smem, s>>>(qkv, out, lse, T, H, D, 1.0f / sqrtf((float)D));
  return check_launch("ns_attn_fwd");
}

template <int DP>
ns_status launch_bwd(const float* qkv, const float* dout, const float* lse, const float* delta,
                     int B, int T, int H, int D, float* dqkv, cudaStream_t s) {
  const size_t smem = bwd_smem<DP>();
  NS_TRY_CUDA(cudaFuncSetAttribute(attn_bwd_dkdv_k<DP>,
                                   cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem),
              "ns_attn_bwd attr");
  NS_TRY_CUDA(cudaFuncSetAttribute(attn_bwd_dq_k<DP>,
                                   cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem),
              "ns_attn_bwd attr");
  const float scale = 1.0f / sqrtf((float)D);
  const dim3 grid((T + kBr - 1) / kBr, B * H);
  attn_bwd_dkdv_k<DP><<<grid, kThreads, smem, s>>>(qkv, dout, lse, delta, dqkv, T, H, D, scale);
  { ns_status _rc = check_launch("ns_attn_bwd dkdv"); if (_rc != NS_OK) return _rc; }
  attn_bwd_dq_k<DP><<<grid, kThreads, smem, s>>>(qkv, dout, lse, delta, dqkv, T, H, D, scale);
  return check_launch("ns_attn_bwd dq");
}

}  // namespace
}  // namespace nsb

using namespace nsb;

extern "C" {

size_t ns_attn_fwd_workspace_size(int B, int T, int H, int D) {
  if (B <= 0 || T <= 0 || H <= 0 || (D != 32 && D != 64)) return 0;
  return attn_tc::fwd_workspace_bytes(B, T, H, D);
}

ns_status ns_attn_set_engine(int engine) {
  NS_REQUIRE(engine >= 0 && engine <= 2, "ns_attn_set_engine: engine must be 0, 1 or 2");
  t_attn_engine = engine;
  return NS_OK;
}

ns_status ns_attn_fwd(const float* qkv, int B, int T, int H, int D, float* out, float* lse,
                      void* workspace, size_t workspace_bytes, void* stream) {
  return ns_attn_fwd_lo(qkv, nullptr, B, T, H, D, out, nullptr, lse, workspace, workspace_bytes,
                        stream);
}

ns_status ns_attn_fwd_lo(const float* qkv, const float* qkv_lo, int B, int T, int H, int D,
                         float* out, float* out_lo, float* lse, void* workspace,
                         size_t workspace_bytes, void* stream) {
  NS_REQUIRE(B >= 0 && T >= 0 && H > 0 && D > 0, "ns_attn_fwd: bad shape");
  NS_REQUIRE(D <= 128, "ns_attn_fwd: head_dim > 128 is not supported");
  NS_REQUIRE(!qkv_lo || (reinterpret_cast<uintptr_t>(qkv_lo) & 15) == 0,
             "ns_attn_fwd_lo: qkv_lo must be 16-byte aligned");
  NS_REQUIRE(!out_lo || ((reinterpret_cast<uintptr_t>(out_lo) & 15) == 0 && out_lo != out),
             "ns_attn_fwd_lo: out_lo must be 16-byte aligned and apart from out");
  if (B == 0 || T == 0) return NS_OK;
  // The K/V lo copy is needed only when the caller gives no qkv_lo.
  const size_t need = qkv_lo ? 0 : ns_attn_fwd_workspace_size(B, T, H, D);
  NS_REQUIRE(workspace_bytes >= need && (need == 0 || workspace),
             "ns_attn_fwd: workspace too small");
  cudaStream_t s = as_stream(stream);
  const bool ws_ok = qkv_lo ? true : (need > 0 && (reinterpret_cast<uintptr_t>(workspace) & 15) == 0);
  if (t_attn_engine != 1 && (D == 32 || D == 64) && ws_ok &&
      attn_tc::fwd_supported(qkv, out, B, T, H, D))
    return attn_tc::fwd(qkv, qkv_lo, B, T, H, D, out, out_lo, lse, static_cast<float*>(workspace), s);
  ns_status rc;
  if (D <= 16) rc = launch_fwd<16>(qkv, B, T, H, D, out, lse, s);
  else if (D <= 32) rc = launch_fwd<32>(qkv, B, T, H, D, out, lse, s);
  else if (D <= 64) rc = launch_fwd<64>(qkv, B, T, H, D, out, lse, s);
  else rc = launch_fwd<128>(qkv, B, T, H, D, out, lse, s);
  if (rc != NS_OK || !out_lo) return rc;
  return ns_split_lo(out, B * T, H * D, H * D, out_lo, stream);
}

size_t ns_attn_bwd_workspace_size(int B, int T, int H, int D) {
  if (B <= 0 || T <= 0 || H <= 0 || D <= 0) return 0;
  const size_t delta = ((size_t)B * H * T * sizeof(float) + 255) & ~(size_t)255;
  if (D != 32 && D != 64) return delta;
  return delta + attn_tc::bwd_lo_bytes(B, T, H, D);
}

ns_status ns_attn_bwd(const float* qkv, const float* out, const float* dout, const float* lse,
                      int B, int T, int H, int D, float* dqkv, void* workspace,
                      size_t workspace_bytes, void* stream) {
  return ns_attn_bwd_lo(qkv, nullptr, out, dout, lse, B, T, H, D, dqkv, workspace,
                        workspace_bytes, stream);
}

ns_status ns_attn_bwd_lo(const float* qkv, const float* qkv_lo, const float* out,
                         const float* dout, const float* lse, int B, int T, int H, int D,
                         float* dqkv, void* workspace, size_t workspace_bytes, void* stream) {
  NS_REQUIRE(B >= 0 && T >= 0 && H > 0 && D > 0, "ns_attn_bwd: bad shape");
  NS_REQUIRE(D <= 128, "ns_attn_bwd: head_dim > 128 is not supported");
  NS_REQUIRE(!qkv_lo || (reinterpret_cast<uintptr_t>(qkv_lo) & 15) == 0,
             "ns_attn_bwd_lo: qkv_lo must be 16-byte aligned");
  if (B == 0 || T == 0) return NS_OK;
  NS_REQUIRE(workspace && workspace_bytes >= ns_attn_bwd_workspace_size(B, T, H, D),
             "ns_attn_bwd: workspace too small");
  cudaStream_t s = as_stream(stream);
  float* delta = static_cast<float*>(workspace);
  const int64_t n = (int64_t)B * H * T;
  const size_t delta_bytes = ((size_t)n * sizeof(float) + 255) & ~(size_t)255;
  float* lo = reinterpret_cast<float*>(static_cast<char*>(workspace) + delta_bytes);
  const bool tc = t_attn_engine != 1 && (D == 32 || D == 64) &&
                  (reinterpret_cast<uintptr_t>(lo) & 15) == 0 &&
                  attn_tc::bwd_supported(qkv, dout, dqkv, B, T, H, D);
  // The tensor-core path takes dO's lo part from the Delta pass.
  float* dout_lo = tc ? attn_tc::bwd_dout_lo(lo, B, T, H, D) : nullptr;
  {
    const ns_status rc = launch_pdl(attn_delta_k, dim3((unsigned)ceil_div64((int64_t)B * T, 8)),
                                    dim3(256), 0, s, "ns_attn_bwd delta", out, dout, B, T, H, D,
                                    delta, dout_lo);
    if (rc != NS_OK) return rc;
  }
  if (tc)
    return attn_tc::bwd(qkv, qkv_lo, dout, lse, delta, B, T, H, D, dqkv, lo, t_attn_engine == 0, s);
  if (D <= 16) return launch_bwd<16>(qkv, dout, lse, delta, B, T, H, D, dqkv, s);
  if (D <= 32) return launch_bwd<32>(qkv, dout, lse, delta, B, T, H, D, dqkv, s);
  if (D <= 64) return launch_bwd<64>(qkv, dout, lse, delta, B, T, H, D, dqkv, s);
  return launch_bwd<128>(qkv, dout, lse, delta, B, T, H, D, dqkv, s);
}

}  // extern "C"
