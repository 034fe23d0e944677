// KV-cache decoding: GPTModel::ForwardWithKVCache (include/gpt.h:159-190),
// GPTBlock::ForwardWithKVCache (gpt.h:102-116) and
// MultiHeadAttention::ForwardWithKVCache (include/layers/attention.h:481-546)
// for B sequences that advance in lockstep, one token each per step.
//
// The reference decodes one token of one sequence with scalar loops and keeps
// its cache as vectors of per-position rows.  Here the cache lives in HBM as
// K and V arrays [layer][sequence][head][position][head_dim] (one head's keys
// are one contiguous block), and a step is bandwidth-bound: every weight is
// read once per step (344 MB for the 12-layer/768 model) plus the cached
// keys and values of every sequence.  So:
//  * the projections are split-K CUDA-core GEMVs (gemv_partial_k): each CTA
//    streams a [K-chunk x 128-column] slab of the weight with 16-byte loads
//    and applies it to all (up to 8) sequences at once; the partials are
//    summed in a fixed order (split by split) by whichever kernel comes next;
//  * attention is split over key chunks (dec_attn_partial_k: one CTA per
//    sequence, head and 64-position chunk, one position per lane for the
//    scores, one head dimension per lane for the output); the chunks are
//    merged in order, so results do not depend on timing;
//  * kernels are fused where one only fed the next: c_attn's partial sums are
//    finished together with the cache append (gemv_finish_append_k); the
//    attention merge and the GELU of mlp_fc run in the prologue of the GEMV
//    that reads them; each residual add runs with the following LayerNorm in
//    one CTA per sequence (row_finish_ln_k): seven launches per block;
//  * a prefill (ns_gpt_decoder_prefill) runs the batched training forward on
//    the prompt (tensor cores) and copies each layer's K and V columns into
//    the cache, which is what decoding the prompt token by token computes;
//  * a step's ~90 launches are one CUDA graph, captured once per (batch,
//    output buffers) on a private stream and replayed, each kernel launched
//    as a programmatic dependent of the one before (it starts while that one
//    finishes, prefetching the weights or cached rows it will read into L2,
//    and waits for it before reading its outputs): the position, the
//    cached length and the tokens reach it through a small device state that
//    one kernel fills before each replay, and the attention grid covers the
//    whole cache (chunks past the cached length do nothing), so the same graph
//    serves every step.
// The arithmetic of every fused piece is that of the separate pass it
// replaces (Linear::Forward, ElementwiseAdd, GeluForward, LayerNormForward
// order of operations); the LayerNorm's row sums are block reductions.
#include <algorithm>
#include <cmath>
#include <cstring>
#include <map>
#include <string>
#include <tuple>
#include <vector>

#include "common.cuh"
#include "gpt_handle.h"

using neuralsuite::cuda::GPTModel;

struct ns_gpt_decoder {
  ns_gpt* owner = nullptr;
  int max_batch = 0, cap = 0, L = 0, H = 0, D = 0, C = 0, V = 0;
  int B = 0, len = 0;  // sequences in the cache and cached positions per sequence
  float* kc = nullptr;  // [L][max_batch][H][cap][D]
  float* vc = nullptr;
  float *x = nullptr, *h = nullptr, *qkv = nullptr, *x1 = nullptr;
  float *xf = nullptr, *logits = nullptr, *mean = nullptr, *rstd = nullptr;
  float *part = nullptr, *part2 = nullptr;  // GEMV / attention partials, used in turn
  size_t part_floats = 0;
  int32_t* err = nullptr;
  int32_t* state = nullptr;  // device: [0] wpe position, [1] cached positions before the step
  int32_t* tok = nullptr;    // device: the step's tokens [max_batch]
  cudaStream_t capture = nullptr;
  // One instantiated step graph per (B, logits_out, err_flag).
  std::map<std::tuple<int, float*, int32_t*>, cudaGraphExec_t> graphs;
  std::vector<void*> allocs;
};

namespace nsb {
namespace decode {
namespace {

constexpr int kGvCols = 128;  // columns per CTA: 32 lanes x 4
constexpr int kGvWarps = 8;
constexpr int kGvRows = 8;    // sequences per CTA (more go to further grid.z slices)

// Where a GEMV's input rows come from.  kInRows: X [B, K] as stored.  The
// other two form the input in the GEMV's prologue from the previous step's
// partial results, so the kernel that would have produced it is not launched:
// kInAttention: the attention output, dec_attn_partial_k's chunks merged in
// chunk order (max over the chunks that saw a key, normaliser and output
// rescaled by e^(m - max), then output / normaliser; part [B*H][S][2 + D]);
// kInGelu: gelu(bias[k] + the sum over splits s in order of part[s][b][k])
// (part [S][B][K]).
enum GvInMode { kInRows = 0, kInAttention = 1, kInGelu = 2 };
struct GvIn {
  int mode = kInRows;
  const float* X = nullptr;
  const float* part = nullptr;
  int S = 0, H = 0, D = 0;
  const float* bias = nullptr;
};

// L2 prefetch of the 128-byte line holding p (a hint: no fault, no data).
__device__ __forceinline__ void prefetch_l2(const void* p) {
  asm volatile("prefetch.global.L2 [%0];" ::"l"(p));
}

// sum over s = 0 .. splits-1, in order, of p[s * stride]; the loads of eight
// splits are issued before their adds.
__device__ __forceinline__ float sum_splits(const float* __restrict__ p, int splits,
                                            size_t stride) {
  float sum = 0.0f;
  int s = 0;
  for (; s + 8 <= splits; s += 8) {
    float v[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = p[(size_t)(s + j) * stride];
#pragma unroll
    for (int j = 0; j < 8; ++j) sum += v[j];
  }
  for (; s < splits; ++s) sum += p[(size_t)s * stride];
  return sum;
}

// W[k][n..n+3] as a float4 (zeros past N).
__device__ __forceinline__ float4 load_w4(const float* __restrict__ wrow, int n, int N, int vec) {
  if (vec && n + 3 < N) return __ldg(reinterpret_cast<const float4*>(wrow + n));
  float4 w;
  w.x = n < N ? wrow[n] : 0.0f;
  w.y = n + 1 < N ? wrow[n + 1] : 0.0f;
  w.z = n + 2 < N ? wrow[n + 2] : 0.0f;
  w.w = n + 3 < N ? wrow[n + 3] : 0.0f;
  return w;
}

// part[s][b][n] = sum over k in split s of X[b][k] * W[k][n].  grid: x =
// column block, y = K split, z = group of 8 sequences.  Each warp takes every
// 8th row of the split; the eight warps' sums are added in warp order.
__global__ void __launch_bounds__(256) gemv_partial_k(GvIn in, int B, int K,
                                                      const float* __restrict__ W, int N, int kchunk,
                                                      int vec, float* __restrict__ part) {
  extern __shared__ float sm[];
  float* sx = sm;                          // [kGvRows][kchunk]
  float* red = sm + kGvRows * kchunk;      // [kGvWarps][kGvRows][kGvCols]
  float* stats = red + kGvWarps * kGvRows * kGvCols;  // attention: [kGvRows][heads][2]
  const int n0 = blockIdx.x * kGvCols, s = blockIdx.y, b0 = blockIdx.z * kGvRows;
  const int k0 = s * kchunk, kc = min(K, k0 + kchunk) - k0;
  const int nb = min(kGvRows, B - b0);
  // Launched while the previous kernel finishes (launch_pdl): the weight
  // slab does not depend on it, so it is brought toward L2 first.
  {
    const int n = n0 + (threadIdx.x & 31) * 4;
    if (n < N)
      for (int k = threadIdx.x >> 5; k < kc; k += kGvWarps) prefetch_l2(W + (size_t)(k0 + k) * N + n);
  }
  pdl_wait();
  pdl_trigger();
  if (in.mode == kInAttention) {
    // Per (row, head) of this split: the merged maximum and normaliser.
    const int h0 = k0 / in.D, nh = kc > 0 ? (k0 + kc - 1) / in.D - h0 + 1 : 0;
    const int stride = 2 + in.D;
    for (int i = threadIdx.x; i < nb * nh; i += blockDim.x) {
      const int b = i / nh, h = h0 + i % nh;
      const float* p = in.part + ((size_t)(b0 + b) * in.H + h) * in.S * stride;
      float M = -INFINITY;
      for (int c = 0; c < in.S; ++c)
        if (p[(size_t)c * stride + 1] > 0.0f) M = fmaxf(M, p[(size_t)c * stride]);
      float Lsum = 0.0f;
      for (int c = 0; c < in.S; ++c) {
        const float* pc = p + (size_t)c * stride;
        if (pc[1] > 0.0f) Lsum += pc[1] * expf(pc[0] - M);
      }
      stats[2 * i] = M;
      stats[2 * i + 1] = Lsum;
    }
    __syncthreads();
    for (int i = threadIdx.x; i < kGvRows * kchunk; i += blockDim.x) {
      const int b = i / kchunk, k = i % kchunk;
      float v = 0.0f;
      if (b < nb && k < kc) {
        const int kk = k0 + k, h = kk / in.D, d = kk - h * in.D;
        const float M = stats[2 * (b * nh + h - h0)], Lsum = stats[2 * (b * nh + h - h0) + 1];
        const float* p = in.part + ((size_t)(b0 + b) * in.H + h) * in.S * stride;
        float od = 0.0f;
        for (int c = 0; c < in.S; ++c) {
          const float* pc = p + (size_t)c * stride;
          if (pc[1] > 0.0f) od += pc[2 + d] * expf(pc[0] - M);
        }
        v = od / Lsum;
      }
      sx[i] = v;
    }
  } else {
    for (int i = threadIdx.x; i < kGvRows * kchunk; i += blockDim.x) {
      const int b = i / kchunk, k = i % kchunk;
      float v = 0.0f;
      if (b < nb && k < kc) {
        const int kk = k0 + k;
        if (in.mode == kInRows) {
          v = in.X[(size_t)(b0 + b) * K + kk];
        } else {
          const float sum = sum_splits(in.part + (size_t)(b0 + b) * K + kk, in.S, (size_t)B * K);
          v = gelu_f(__fadd_rn(sum, in.bias[kk]));
        }
      }
      sx[i] = v;
    }
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n = n0 + lane * 4;
  float acc[kGvRows][4];
#pragma unroll
  for (int b = 0; b < kGvRows; ++b) acc[b][0] = acc[b][1] = acc[b][2] = acc[b][3] = 0.0f;
  // Rows k = warp, warp + 8, ... in order; four rows' weights loaded first.
  int k = warp;
  for (; k + 3 * kGvWarps < kc; k += 4 * kGvWarps) {
    float4 w[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) w[u] = load_w4(W + (size_t)(k0 + k + u * kGvWarps) * N, n, N, vec);
#pragma unroll
    for (int u = 0; u < 4; ++u)
#pragma unroll
      for (int b = 0; b < kGvRows; ++b) {
        const float xv = sx[b * kchunk + k + u * kGvWarps];
        acc[b][0] = fmaf(xv, w[u].x, acc[b][0]);
        acc[b][1] = fmaf(xv, w[u].y, acc[b][1]);
        acc[b][2] = fmaf(xv, w[u].z, acc[b][2]);
        acc[b][3] = fmaf(xv, w[u].w, acc[b][3]);
      }
  }
  for (; k < kc; k += kGvWarps) {
    const float4 w = load_w4(W + (size_t)(k0 + k) * N, n, N, vec);
#pragma unroll
    for (int b = 0; b < kGvRows; ++b) {
      const float xv = sx[b * kchunk + k];
      acc[b][0] = fmaf(xv, w.x, acc[b][0]);
      acc[b][1] = fmaf(xv, w.y, acc[b][1]);
      acc[b][2] = fmaf(xv, w.z, acc[b][2]);
      acc[b][3] = fmaf(xv, w.w, acc[b][3]);
    }
  }
#pragma unroll
  for (int b = 0; b < kGvRows; ++b)
#pragma unroll
    for (int j = 0; j < 4; ++j) red[(warp * kGvRows + b) * kGvCols + lane * 4 + j] = acc[b][j];
  __syncthreads();
  for (int i = threadIdx.x; i < nb * kGvCols; i += blockDim.x) {
    const int b = i / kGvCols, c = i % kGvCols;
    if (n0 + c >= N) continue;
    float sum = 0.0f;
#pragma unroll
    for (int w = 0; w < kGvWarps; ++w) sum += red[(w * kGvRows + b) * kGvCols + c];
    part[((size_t)s * B + b0 + b) * N + n0 + c] = sum;
  }
}

// c_attn's finish: qkv[b][n] = (sum over splits in order of part) + bias[n],
// and the K and V columns also to the cache at position state[1].
__global__ void gemv_finish_append_k(const float* __restrict__ part, int splits, int B, int C,
                                     const float* __restrict__ bias, float* __restrict__ qkv,
                                     int H, int D, float* __restrict__ kc, float* __restrict__ vc,
                                     int cap, const int32_t* __restrict__ state) {
  pdl_wait();
  pdl_trigger();
  const int N = 3 * C, idx = state[1];
  const int64_t total = (int64_t)B * N;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const float sum = sum_splits(part + i, splits, (size_t)total);
    const int b = (int)(i / N), n = (int)(i - (int64_t)b * N);
    const float v = __fadd_rn(sum, bias[n]);
    qkv[i] = v;
    if (n >= C) {
      const int c = n >= 2 * C ? n - 2 * C : n - C;
      const int h = c / D, d = c - h * D;
      const size_t dst = (((size_t)b * H + h) * cap + idx) * D + d;
      (n >= 2 * C ? vc : kc)[dst] = v;
    }
  }
}

// One row per CTA (kFinishThreads threads): x_out[b] = resid[b] + ((sum over
// splits in order of part[s][b]) + bias) (Linear::Forward then
// ElementwiseAdd), then h[b] = LayerNorm(x_out[b]) * gamma + beta
// (src/tensor.cpp:290-315; the next layer's ln_1 or ln_2, or ln_f).  Dynamic
// shared memory: C floats.
constexpr int kFinishThreads = 1024;
__global__ void __launch_bounds__(kFinishThreads) row_finish_ln_k(
    const float* __restrict__ part, int splits, int B, int C, const float* __restrict__ bias,
    const float* __restrict__ resid, float* __restrict__ x_out, const float* __restrict__ gamma,
    const float* __restrict__ beta, float eps, float* __restrict__ h) {
  pdl_wait();
  pdl_trigger();
  extern __shared__ float row[];
  __shared__ float wsum[kFinishThreads / 32];
  const int b = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nw = blockDim.x >> 5;
  const int64_t total = (int64_t)B * C;
  float s1 = 0.0f;
  for (int c = threadIdx.x; c < C; c += blockDim.x) {
    const size_t i = (size_t)b * C + c;
    const float sum = sum_splits(part + i, splits, (size_t)total);
    const float v = __fadd_rn(resid[i], __fadd_rn(sum, bias[c]));
    x_out[i] = v;
    row[c] = v;
    s1 += v;
  }
  s1 = warp_sum(s1);
  if (lane == 0) wsum[warp] = s1;
  __syncthreads();
  float tot = 0.0f;
  for (int w = 0; w < nw; ++w) tot += wsum[w];
  const float m = __fdiv_rn(tot, (float)C);
  __syncthreads();
  float q = 0.0f;
  for (int c = threadIdx.x; c < C; c += blockDim.x) {
    const float d = row[c] - m;
    q += d * d;
  }
  q = warp_sum(q);
  if (lane == 0) wsum[warp] = q;
  __syncthreads();
  float qt = 0.0f;
  for (int w = 0; w < nw; ++w) qt += wsum[w];
  const float rs = __fdiv_rn(1.0f, __fsqrt_rn(__fdiv_rn(qt, (float)C) + eps));
  for (int c = threadIdx.x; c < C; c += blockDim.x)
    h[(size_t)b * C + c] =
        __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(row[c], m), rs), gamma[c]), beta[c]);
}

// x[b] = wte[tok[b]] + wpe[pos] (GPTModel::ForwardWithKVCache's embedding add).
__global__ void dec_embed_k(const int32_t* __restrict__ tok, int B, const float* __restrict__ wte,
                            int V, const float* __restrict__ wpe, const int32_t* __restrict__ state,
                            int C, float* __restrict__ x, int32_t* err) {
  pdl_wait();
  pdl_trigger();
  const int pos = state[0];
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < B * C; i += gridDim.x * blockDim.x) {
    const int b = i / C, c = i % C;
    int t = tok[b];
    if (t < 0 || t >= V) {
      if (err) atomicExch(err, 1);
      x[i] = 0.0f;
      continue;
    }
    x[i] = __fadd_rn(wte[(size_t)t * C + c], wpe[(size_t)pos * C + c]);
  }
}

// K and V of rows [row0, row0 + nrows) of each sequence's qkv ([rows, 3C],
// sequence b's row r at b * seq_stride + r) to cache positions [idx, idx + nrows),
// idx = state[1] when state is given.
__global__ void dec_append_k(const float* __restrict__ qkv, int B, int nrows, int seq_stride, int C,
                             int H, int D, float* __restrict__ kc, float* __restrict__ vc, int cap,
                             int idx, const int32_t* __restrict__ state) {
  if (state) idx = state[1];
  const int64_t total = (int64_t)B * nrows * C;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int c = (int)(i % C);
    const int r = (int)((i / C) % nrows);
    const int b = (int)(i / ((int64_t)C * nrows));
    const int h = c / D, d = c % D;
    const float* src = qkv + ((size_t)b * seq_stride + r) * 3 * C;
    const size_t dst = (((size_t)b * H + h) * cap + idx + r) * D + d;
    kc[dst] = src[C + c];
    vc[dst] = src[2 * C + c];
  }
}

// Partial attention of the query of sequence b, head h over cached keys
// [s*kch, min(n, (s+1)*kch)), n = state[1] + 1, kch = 32 * kAttWarps: each
// warp takes 32 positions, one per lane (score = q . k over the head
// dimension in order, the 32 scores' softmax by warp max and sum), then
// accumulates p . V with one output dimension per lane; the warps' (m, l, o)
// are merged in warp order.  part: [B*H][S][2 + D] with S = gridDim.y chunks
// covering the whole cache; a chunk past n writes l = 0, which the merge in
// the next GEMV skips.
constexpr int kAttWarps = 2;
constexpr int kAttThreads = 32 * kAttWarps;
__global__ void __launch_bounds__(kAttThreads) dec_attn_partial_k(
    const float* __restrict__ qkv, int C, int H, int D, const float* __restrict__ kc,
    const float* __restrict__ vc, int cap, const int32_t* __restrict__ state, int kch, float scale,
    float* __restrict__ part) {
  const int n = state[1] + 1;  // written before the step's graph was launched
  __shared__ float qs[128];
  __shared__ float wm[kAttWarps], wl[kAttWarps];
  __shared__ float wo[kAttWarps][128];
  const int bh = blockIdx.x, s = blockIdx.y, S = gridDim.y;
  const int b = bh / H, h = bh % H;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  {
    // Launched while the previous kernel finishes (launch_pdl): the cached
    // rows of this lane's position are brought toward L2 first (the newest
    // one is being written; L2 is where that write lands).
    const int tp = s * kch + warp * 32 + lane;
    if (tp < min(n, s * kch + kch)) {
      const size_t o = (((size_t)b * H + h) * cap + tp) * D;
      for (int d = 0; d < D; d += 32) {
        prefetch_l2(kc + o + d);
        prefetch_l2(vc + o + d);
      }
    }
  }
  pdl_wait();
  pdl_trigger();
  const float* q = qkv + (size_t)b * 3 * C + h * D;
  for (int d = threadIdx.x; d < D; d += blockDim.x) qs[d] = q[d];
  __syncthreads();
  const float* kb = kc + ((size_t)b * H + h) * cap * D;
  const float* vb = vc + ((size_t)b * H + h) * cap * D;
  const int t0 = s * kch + warp * 32, t1 = min(n, s * kch + kch);
  const int t = t0 + lane;
  float sc = -INFINITY;
  if (t < t1) {
    const float* kr = kb + (size_t)t * D;
    float dot = 0.0f;
    if ((D & 3) == 0) {
      for (int d = 0; d < D; d += 4) {
        const float4 kv = __ldg(reinterpret_cast<const float4*>(kr + d));
        dot = fmaf(qs[d], kv.x, dot);
        dot = fmaf(qs[d + 1], kv.y, dot);
        dot = fmaf(qs[d + 2], kv.z, dot);
        dot = fmaf(qs[d + 3], kv.w, dot);
      }
    } else {
      for (int d = 0; d < D; ++d) dot = fmaf(qs[d], __ldg(kr + d), dot);
    }
    sc = dot * scale;
  }
  const float m = warp_max(sc);
  const float p = (t < t1) ? expf(sc - m) : 0.0f;
  const float l = warp_sum(p);
  float o[4] = {0.0f, 0.0f, 0.0f, 0.0f};
  const int nv = min(32, max(0, t1 - t0));
  for (int j = 0; j < nv; ++j) {
    const float pj = __shfl_sync(0xffffffffu, p, j);
    const float* vr = vb + (size_t)(t0 + j) * D;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int d = lane + 32 * i;
      if (d < D) o[i] = fmaf(pj, __ldg(vr + d), o[i]);
    }
  }
  if (lane == 0) {
    wm[warp] = m;
    wl[warp] = l;
  }
#pragma unroll
  for (int i = 0; i < 4; ++i)
    if (lane + 32 * i < D) wo[warp][lane + 32 * i] = o[i];
  __syncthreads();
  float* dst = part + ((size_t)bh * S + s) * (2 + D);
  float M = -INFINITY;
  for (int w = 0; w < kAttWarps; ++w)
    if (wl[w] > 0.0f) M = fmaxf(M, wm[w]);
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float od = 0.0f;
    for (int w = 0; w < kAttWarps; ++w)
      if (wl[w] > 0.0f) od += wo[w][d] * expf(wm[w] - M);
    dst[2 + d] = od;
  }
  if (threadIdx.x == 0) {
    float Lsum = 0.0f;
    for (int w = 0; w < kAttWarps; ++w)
      if (wl[w] > 0.0f) Lsum += wl[w] * expf(wm[w] - M);
    dst[0] = M;
    dst[1] = Lsum;
  }
}

// logits[b][v] = sum_c xf[b][c] * wte[v][c]: one warp per vocabulary row
// (read once, 16-byte loads), up to 8 sequences from shared memory.
__global__ void __launch_bounds__(256) dec_logits_k(const float* __restrict__ xf, int B, int C,
                                                    const float* __restrict__ wte, int V, int vec,
                                                    float* __restrict__ logits) {
  extern __shared__ float sxf[];  // [8][C]
  const int b0 = blockIdx.y * 8, nb = min(8, B - b0);
  {
    const int v = blockIdx.x * 8 + (threadIdx.x >> 5);
    if (v < V)
      for (int c = (threadIdx.x & 31) * 32; c < C; c += 32 * 32) prefetch_l2(wte + (size_t)v * C + c);
  }
  pdl_wait();
  pdl_trigger();
  for (int i = threadIdx.x; i < 8 * C; i += blockDim.x) {
    const int b = i / C;
    sxf[i] = b < nb ? xf[(size_t)(b0 + b) * C + i % C] : 0.0f;
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int v = blockIdx.x * 8 + warp;
  if (v >= V) return;
  const float* row = wte + (size_t)v * C;
  float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  if (vec) {
    for (int c = lane * 4; c < C; c += 128) {
      const float4 w = __ldg(reinterpret_cast<const float4*>(row + c));
#pragma unroll
      for (int b = 0; b < 8; ++b) {
        const float* xb = sxf + b * C + c;
        acc[b] = fmaf(xb[0], w.x, fmaf(xb[1], w.y, fmaf(xb[2], w.z, fmaf(xb[3], w.w, acc[b]))));
      }
    }
  } else {
    for (int c = lane; c < C; c += 32) {
      const float w = row[c];
#pragma unroll
      for (int b = 0; b < 8; ++b) acc[b] = fmaf(sxf[b * C + c], w, acc[b]);
    }
  }
#pragma unroll
  for (int b = 0; b < 8; ++b) {
    const float t = warp_sum(acc[b]);
    if (lane == 0 && b < nb) logits[(size_t)(b0 + b) * V + v] = t;
  }
}

int grid_for(int64_t work, int threads) {
  return (int)std::max<int64_t>(1, std::min<int64_t>((work + threads - 1) / threads,
                                                     (int64_t)sm_count() * 8));
}

// Split of a [K x N] product: (column blocks, K splits, rows per split).
struct GvPlan {
  int cols, splits, kchunk;
};
GvPlan gv_plan(int K, int N) {
  GvPlan p;
  p.cols = (N + kGvCols - 1) / kGvCols;
  const int target = 2 * sm_count();
  int s = std::max(1, std::min((target + p.cols - 1) / p.cols, (K + kGvWarps - 1) / kGvWarps));
  p.kchunk = ((K + s - 1) / s + kGvWarps - 1) / kGvWarps * kGvWarps;
  p.splits = (K + p.kchunk - 1) / p.kchunk;
  return p;
}

size_t gv_part_floats(int B, int K, int N) {
  const GvPlan p = gv_plan(K, N);
  return (size_t)p.splits * B * N;
}

// Partials of one GEMV into `part`; its input rows as `in` says.
ns_status gemv_part(ns_gpt_decoder* d, const GvIn& in, int B, int K, const float* W, int N,
                    float* part, int* splits, cudaStream_t s) {
  const GvPlan p = gv_plan(K, N);
  if ((size_t)p.splits * B * N > d->part_floats) return fail(NS_ERR_INVALID_ARGUMENT, "decode: partial buffer too small");
  const int vec = (N % 4 == 0) && ((reinterpret_cast<uintptr_t>(W) & 15) == 0);
  const int heads = in.mode == kInAttention ? p.kchunk / in.D + 2 : 0;
  const size_t smem = (size_t)(kGvRows * p.kchunk + kGvWarps * kGvRows * kGvCols +
                               2 * kGvRows * heads) * sizeof(float);
  if (smem > 48 * 1024)
    NS_TRY_CUDA(cudaFuncSetAttribute(gemv_partial_k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem),
                "decode gemv attr");
  dim3 grid(p.cols, p.splits, (B + kGvRows - 1) / kGvRows);
  *splits = p.splits;
  return launch_pdl(gemv_partial_k, grid, dim3(256), smem, s, "decode gemv", in, B, K, W, N,
                    p.kchunk, vec, part);
}

// Attention partials of the B current queries (in d->qkv) over the
// state[1] + 1 cached positions per sequence of layer l, into `part`
// ([B*H][S][2 + D], S chunks covering the whole cache); the next GEMV merges
// them in its prologue.
ns_status attend(ns_gpt_decoder* d, int l, int B, float* part, int* chunks, cudaStream_t s) {
  const size_t per_layer = (size_t)d->max_batch * d->H * d->cap * d->D;
  const int kch = 32 * kAttWarps;
  const int S = (d->cap + kch - 1) / kch;
  if ((size_t)B * d->H * S * (2 + d->D) > d->part_floats)
    return fail(NS_ERR_INVALID_ARGUMENT, "decode: partial buffer too small for attention");
  dim3 grid(B * d->H, S);
  *chunks = S;
  return launch_pdl(dec_attn_partial_k, grid, dim3(kAttThreads), 0, s, "decode attention",
                    (const float*)d->qkv, d->C, d->H, d->D, (const float*)(d->kc + l * per_layer),
                    (const float*)(d->vc + l * per_layer), d->cap, (const int32_t*)d->state, kch,
                    1.0f / std::sqrt((float)d->D), part);
}

// x_out = resid + (partials + bias); h = LayerNorm(x_out) with gamma, beta.
ns_status row_finish_ln(ns_gpt_decoder* d, const float* part, int splits, int B,
                        const float* bias, const float* resid, float* x_out, const float* gamma,
                        const float* beta, float* h, cudaStream_t s) {
  const size_t smem = (size_t)d->C * sizeof(float);
  if (smem > 48 * 1024)
    NS_TRY_CUDA(cudaFuncSetAttribute(row_finish_ln_k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem),
                "decode finish attr");
  const int threads = std::min(kFinishThreads, (d->C + 31) / 32 * 32);
  return launch_pdl(row_finish_ln_k, dim3(B), dim3(threads), smem, s, "decode finish + LayerNorm",
                    part, splits, B, d->C, bias, resid, x_out, gamma, beta, 1e-5f, h);
}

// The step's inputs for the graph: its tokens and the state it reads.
__global__ void dec_state_k(const int32_t* __restrict__ tokens, int B, int pos, int len,
                            int32_t* __restrict__ state, int32_t* __restrict__ tok) {
  for (int i = threadIdx.x; i < B; i += blockDim.x) tok[i] = tokens[i];
  if (threadIdx.x == 0) {
    state[0] = pos;
    state[1] = len;
  }
}

// Every launch of one decode step (GPTModel::ForwardWithKVCache) on stream s,
// reading the tokens from d->tok and the position and cached length from
// d->state.
ns_status enqueue_step(ns_gpt_decoder* d, int B, float* lg, int32_t* err, cudaStream_t s) {
  GPTModel& m = *d->owner->model;
  const float* P = m.Values();
  const auto& off = m.Offsets();
  const int C = d->C, L = d->L;
  const size_t per_layer = (size_t)d->max_batch * d->H * d->cap * d->D;
  void* stream = s;
  auto prm = [&](int i) { return P + off[i]; };
  dec_embed_k<<<grid_for((int64_t)B * C, 256), 256, 0, s>>>(d->tok, B, prm(0), d->V, prm(1),
                                                           d->state, C, d->x, err);
  ns_status rc = check_launch("decode embedding");
  // ln_1 of the first block; every later LayerNorm runs inside the finish of
  // the GEMV before it.
  if (rc == NS_OK && L > 0)
    rc = ns_layernorm_fwd(d->x, prm(2), prm(3), d->h, d->mean, d->rstd, B, C, 1e-5f, stream);
  float *p1 = d->part, *p2 = d->part2;
  const int f = 2 + 12 * L;
  for (int l = 0; l < L && rc == NS_OK; ++l) {
    const int t = 2 + 12 * l;
    int splits = 0, chunks = 0;
    // x1 = x + c_proj(attention(c_attn(h))), h = ln_1(x)
    GvIn rows;
    rows.X = d->h;
    rc = gemv_part(d, rows, B, C, prm(t + 2), 3 * C, p1, &splits, s);
    if (rc == NS_OK) {
      rc = launch_pdl(gemv_finish_append_k, dim3(grid_for((int64_t)B * 3 * C, 256)), dim3(256), 0, s,
                      "decode qkv + cache append", p1, splits, B, C, prm(t + 3), d->qkv, d->H, d->D,
                      d->kc + l * per_layer, d->vc + l * per_layer, d->cap, d->state);
    }
    if (rc == NS_OK) rc = attend(d, l, B, p2, &chunks, s);
    if (rc == NS_OK) {
      GvIn att;
      att.mode = kInAttention;
      att.part = p2;
      att.S = chunks;
      att.H = d->H;
      att.D = d->D;
      rc = gemv_part(d, att, B, C, prm(t + 4), C, p1, &splits, s);
    }
    // x1 and h = ln_2(x1)
    if (rc == NS_OK)
      rc = row_finish_ln(d, p1, splits, B, prm(t + 5), d->x, d->x1, prm(t + 6), prm(t + 7), d->h, s);
    // x = x1 + mlp_proj(gelu(mlp_fc(h)))
    if (rc == NS_OK) rc = gemv_part(d, rows, B, C, prm(t + 8), 4 * C, p2, &splits, s);
    if (rc == NS_OK) {
      GvIn gel;
      gel.mode = kInGelu;
      gel.part = p2;
      gel.S = splits;
      gel.bias = prm(t + 9);
      rc = gemv_part(d, gel, B, 4 * C, prm(t + 10), C, p1, &splits, s);
    }
    // x and h = the next block's ln_1(x), or ln_f(x) after the last block
    const int g = l + 1 < L ? t + 12 : f;
    if (rc == NS_OK)
      rc = row_finish_ln(d, p1, splits, B, prm(t + 11), d->x1, d->x, prm(g), prm(g + 1),
                         l + 1 < L ? d->h : d->xf, s);
  }
  if (rc != NS_OK) return rc;
  if (L == 0) {
    rc = ns_layernorm_fwd(d->x, prm(f), prm(f + 1), d->xf, d->mean, d->rstd, B, C, 1e-5f, stream);
    if (rc != NS_OK) return rc;
  }
  const int vec = (C % 4 == 0) && ((reinterpret_cast<uintptr_t>(prm(0)) & 15) == 0);
  const size_t smem = (size_t)8 * C * sizeof(float);
  if (smem > 48 * 1024)
    NS_TRY_CUDA(cudaFuncSetAttribute(dec_logits_k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem),
                "decode logits attr");
  dim3 grid((d->V + 7) / 8, (B + 7) / 8);
  return launch_pdl(dec_logits_k, grid, dim3(256), smem, s, "decode logits", d->xf, B, C, prm(0),
                    d->V, vec, lg);
}

// The instantiated step graph for (B, lg, err), captured on first use on
// the decoder's own stream (the caller's may be the legacy default stream,
// which cannot be captured).
ns_status step_graph(ns_gpt_decoder* d, int B, float* lg, int32_t* err, cudaGraphExec_t* out) {
  const auto key = std::make_tuple(B, lg, err);
  auto it = d->graphs.find(key);
  if (it != d->graphs.end()) {
    *out = it->second;
    return NS_OK;
  }
  if (!d->capture)
    NS_TRY_CUDA(cudaStreamCreateWithFlags(&d->capture, cudaStreamNonBlocking), "decode graph stream");
  NS_TRY_CUDA(cudaStreamBeginCapture(d->capture, cudaStreamCaptureModeThreadLocal),
              "decode graph capture");
  ns_status rc = enqueue_step(d, B, lg, err, d->capture);
  cudaGraph_t g = nullptr;
  const cudaError_t e = cudaStreamEndCapture(d->capture, &g);
  if (rc != NS_OK) {
    if (g) cudaGraphDestroy(g);
    return rc;
  }
  if (e != cudaSuccess) return cuda_fail(e, "decode graph capture");
  cudaGraphExec_t exec = nullptr;
  const cudaError_t ei = cudaGraphInstantiate(&exec, g, 0);
  cudaGraphDestroy(g);
  if (ei != cudaSuccess) return cuda_fail(ei, "decode graph instantiate");
  d->graphs.emplace(key, exec);
  *out = exec;
  return NS_OK;
}

template <typename T>
ns_status dev_alloc(ns_gpt_decoder* d, T** p, size_t count) {
  void* q = nullptr;
  NS_TRY_CUDA(cudaMalloc(&q, std::max<size_t>(count, 1) * sizeof(T)), "ns_gpt_decoder_create");
  d->allocs.push_back(q);
  *p = static_cast<T*>(q);
  return NS_OK;
}

void free_all(ns_gpt_decoder* d) {
  for (auto& kv : d->graphs) cudaGraphExecDestroy(kv.second);
  d->graphs.clear();
  if (d->capture) cudaStreamDestroy(d->capture);
  d->capture = nullptr;
  for (void* p : d->allocs) cudaFree(p);
  d->allocs.clear();
}

}  // namespace
}  // namespace decode
}  // namespace nsb

using namespace nsb;
using namespace nsb::decode;

extern "C" {

ns_status ns_gpt_decoder_create(ns_gpt* model, int max_batch, ns_gpt_decoder** out) {
  NS_REQUIRE(model && out, "ns_gpt_decoder_create: NULL argument");
  NS_REQUIRE(max_batch >= 1 && max_batch <= 64, "ns_gpt_decoder_create: max_batch must be in [1, 64]");
  const auto& cfg = model->model->Config();
  NS_REQUIRE(cfg.n_head > 0 && cfg.n_embd % cfg.n_head == 0 && cfg.n_embd / cfg.n_head <= 128,
             "ns_gpt_decoder_create: head_dim must be at most 128");
  auto* d = new ns_gpt_decoder();
  d->owner = model;
  d->max_batch = max_batch;
  d->cap = cfg.block_size;
  d->L = cfg.n_layer;
  d->H = cfg.n_head;
  d->C = cfg.n_embd;
  d->D = cfg.n_embd / cfg.n_head;
  d->V = cfg.vocab_size;
  const size_t Bm = (size_t)max_batch, C = d->C;
  const size_t cache = (size_t)std::max(d->L, 1) * Bm * d->H * d->cap * d->D;
  size_t part = 0;
  for (auto kn : {std::make_pair(C, 3 * C), std::make_pair(C, C), std::make_pair(C, 4 * C),
                  std::make_pair(4 * C, C)})
    part = std::max(part, gv_part_floats((int)Bm, (int)kn.first, (int)kn.second));
  const int kch = 32 * kAttWarps;
  part = std::max(part, Bm * d->H * (size_t)((d->cap + kch - 1) / kch) * (2 + d->D));
  d->part_floats = part;
  ns_status rc = NS_OK;
  auto A = [&](float** p, size_t n) {
    if (rc == NS_OK) rc = dev_alloc(d, p, n);
  };
  A(&d->kc, cache);
  A(&d->vc, cache);
  A(&d->x, Bm * C);
  A(&d->h, Bm * C);
  A(&d->qkv, Bm * 3 * C);
  A(&d->x1, Bm * C);
  A(&d->xf, Bm * C);
  A(&d->logits, Bm * d->V);
  A(&d->mean, Bm);
  A(&d->rstd, Bm);
  A(&d->part, part);
  A(&d->part2, part);
  if (rc == NS_OK) rc = dev_alloc(d, &d->err, 1);
  if (rc == NS_OK) rc = dev_alloc(d, &d->state, 2);
  if (rc == NS_OK) rc = dev_alloc(d, &d->tok, Bm);
  if (rc == NS_OK) {
    cudaError_t e = cudaMemset(d->err, 0, sizeof(int32_t));
    if (e != cudaSuccess) rc = cuda_fail(e, "ns_gpt_decoder_create");
  }
  if (rc != NS_OK) {
    free_all(d);
    delete d;
    return rc;
  }
  *out = d;
  return NS_OK;
}

ns_status ns_gpt_decoder_destroy(ns_gpt_decoder* d) {
  if (!d) return NS_OK;
  cudaDeviceSynchronize();
  free_all(d);
  delete d;
  return NS_OK;
}

ns_status ns_gpt_decoder_clear(ns_gpt_decoder* d) {
  NS_REQUIRE(d, "ns_gpt_decoder_clear: NULL decoder");
  d->len = 0;
  d->B = 0;
  return NS_OK;
}

int ns_gpt_decoder_length(const ns_gpt_decoder* d) { return d ? d->len : 0; }

float* ns_gpt_decoder_logits(ns_gpt_decoder* d) { return d ? d->logits : nullptr; }

ns_status ns_gpt_decode_step(ns_gpt_decoder* d, const int32_t* tokens, int B, int pos,
                             float* logits_out, int32_t* err_flag, void* stream) {
  NS_REQUIRE(d && tokens, "ns_gpt_decode_step: NULL argument");
  NS_REQUIRE(B >= 1 && B <= d->max_batch, "ns_gpt_decode_step: B must be in [1, max_batch]");
  NS_REQUIRE(d->len == 0 || B == d->B,
             "ns_gpt_decode_step: B differs from the sequences in the cache (clear it first)");
  if (pos < 0 || pos >= d->cap)
    return fail(NS_ERR_OUT_OF_RANGE, "ns_gpt_decode_step: position outside [0, block_size)");
  if (d->len >= d->cap)
    return fail(NS_ERR_OUT_OF_RANGE, "ns_gpt_decode_step: the KV cache is full (block_size positions)");
  cudaStream_t s = as_stream(stream);
  float* lg = logits_out ? logits_out : d->logits;
  int32_t* err = err_flag ? err_flag : d->err;
  cudaGraphExec_t exec = nullptr;
  ns_status rc = step_graph(d, B, lg, err, &exec);
  if (rc != NS_OK) return rc;
  dec_state_k<<<1, 64, 0, s>>>(tokens, B, pos, d->len, d->state, d->tok);
  rc = check_launch("decode state");
  if (rc != NS_OK) return rc;
  NS_TRY_CUDA(cudaGraphLaunch(exec, s), "decode graph launch");
  d->B = B;
  d->len += 1;
  return NS_OK;
}

ns_status ns_gpt_decoder_prefill(ns_gpt_decoder* d, const int32_t* tokens, int B, int T,
                                 float* logits_out, void* stream) {
  NS_REQUIRE(d && tokens, "ns_gpt_decoder_prefill: NULL argument");
  NS_REQUIRE(d->len == 0, "ns_gpt_decoder_prefill: the cache is not empty (clear it first)");
  NS_REQUIRE(B >= 1 && B <= d->max_batch, "ns_gpt_decoder_prefill: B must be in [1, max_batch]");
  NS_REQUIRE(B <= d->owner->model->MaxBatch(), "ns_gpt_decoder_prefill: B exceeds the model's max_batch");
  if (T < 1 || T > d->cap)
    return fail(NS_ERR_OUT_OF_RANGE, "ns_gpt_decoder_prefill: T outside [1, block_size]");
  ns_status rc = ns_gpt_forward(d->owner, tokens, B, T, stream);
  if (rc != NS_OK) return rc;
  cudaStream_t s = as_stream(stream);
  GPTModel& m = *d->owner->model;
  const size_t per_layer = (size_t)d->max_batch * d->H * d->cap * d->D;
  for (int l = 0; l < d->L; ++l) {
    const float* qkv = m.Block(l).Attn().Qkv().Data();
    dec_append_k<<<grid_for((int64_t)B * T * d->C, 256), 256, 0, s>>>(
        qkv, B, T, T, d->C, d->H, d->D, d->kc + l * per_layer, d->vc + l * per_layer, d->cap, 0,
        nullptr);
    rc = check_launch("prefill cache fill");
    if (rc != NS_OK) return rc;
  }
  // The last position's logits of each sequence.
  float* lg = logits_out ? logits_out : d->logits;
  NS_TRY_CUDA(cudaMemcpy2DAsync(lg, (size_t)d->V * sizeof(float),
                                m.Logits().Data() + (size_t)(T - 1) * d->V,
                                (size_t)T * d->V * sizeof(float), (size_t)d->V * sizeof(float), B,
                                cudaMemcpyDeviceToDevice, s),
              "prefill logits");
  d->B = B;
  d->len = T;
  return NS_OK;
}

}  // extern "C"
