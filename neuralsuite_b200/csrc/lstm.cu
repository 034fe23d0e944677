// LSTM and BiLSTM forward / backward (include/layers/lstm.h:320-664).
//
// Layout as the reference: x [T, B, IN], output [T, B, H], gates in the
// order i, f, g, o over 4H columns, W_ih [4H, IN], W_hh [4H, H].
//
// The reference already splits the work into a batched part and a
// sequential part; here each runs where it belongs:
//  * pre = x . W_ih^T for all T steps is one tcgen05 3xTF32 GEMM, and so are
//    the backward's dW_ih = dpre^T . x, dW_hh = dpre^T . H_prev and
//    dx = dpre . W_ih; H_prev (the state entering each step) is the output
//    itself shifted by one step, so no stacked copy is made.
//  * The recurrence runs as one cooperative kernel over the whole sequence
//    (lstm_seq_fwd_k / lstm_seq_bwd_k: each CTA keeps its units' weight rows
//    in shared memory, a grid barrier between steps) when every CTA fits on
//    the GPU at once, else as one launch per step (each a programmatic
//    dependent of the one before).  Each CTA owns kUnits hidden
//    units: it forms their 4 gate pre-activations for every sequence from
//    h_{t-1} . W_hh^T (both streamed through shared memory in chunks) and
//    applies the cell update in the same launch, so a step needs no
//    grid-wide barrier.  The backward step kernel computes, for its units,
//    dh_next = dpre_{t+1} . W_hh (W_hh transposed once per call) and then the
//    step's dpre and the carried dc.
// Sums run in a fixed order (no atomics): results are deterministic.
#include <algorithm>
#include <cmath>

#include "common.cuh"
#include "gemm_tc.cuh"
#include "ns_b200.h"

namespace nsb {
namespace lstm {
namespace {

constexpr int kUnits = 8;             // hidden units per CTA (32 gate rows)
constexpr int kRows = 4 * kUnits;     // gate rows per CTA
constexpr int kChunk = 64;            // reduction chunk staged in shared memory
constexpr int kThreads = 256;
constexpr int kMaxB = 64;             // sequences per launch (8 per thread group)

__device__ __forceinline__ float sigmoid_f(float x) { return __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-x))); }

// Cache layout (floats): i, f, g, o, c, tanh_c, each [T, B, H].
struct Cache {
  float *i, *f, *g, *o, *c, *tc;
};
__host__ __device__ inline Cache cache_at(float* base, int64_t TBH) {
  return Cache{base, base + TBH, base + 2 * TBH, base + 3 * TBH, base + 4 * TBH, base + 5 * TBH};
}

// One forward step t.  pre [T*B, 4H] holds x . W_ih^T; h_prev = out[t-1]
// (ignored at t = 0), c_prev = c[t-1].
__global__ void __launch_bounds__(kThreads) lstm_step_fwd_k(
    const float* __restrict__ pre, const float* __restrict__ w_hh, const float* __restrict__ b_ih,
    const float* __restrict__ b_hh, int t, int B, int H, float* __restrict__ out, Cache cache) {
  __shared__ float sh[kMaxB][kChunk + 1];
  __shared__ float sw[kRows][kChunk + 1];
  __shared__ float gates[kMaxB][kRows];
  pdl_wait();  // launched as a programmatic dependent of the previous step
  pdl_trigger();
  const int k0 = blockIdx.x * kUnits;
  const int r = threadIdx.x % kRows, bq = threadIdx.x / kRows;  // 8 groups of sequences
  const int g = r / kUnits, u = r % kUnits;
  const int row = g * H + k0 + u;  // gate row of W_hh
  float acc[kMaxB / 8];
#pragma unroll
  for (int q = 0; q < kMaxB / 8; ++q) acc[q] = 0.0f;
  if (t > 0) {
    const float* hp = out + (size_t)(t - 1) * B * H;
    for (int j0 = 0; j0 < H; j0 += kChunk) {
      const int jn = min(kChunk, H - j0);
      for (int i = threadIdx.x; i < B * kChunk; i += kThreads) {
        const int b = i / kChunk, j = i % kChunk;
        sh[b][j] = j < jn ? hp[(size_t)b * H + j0 + j] : 0.0f;
      }
      for (int i = threadIdx.x; i < kRows * kChunk; i += kThreads) {
        const int rr = i / kChunk, j = i % kChunk;
        const int gg = rr / kUnits, uu = rr % kUnits;
        const bool in = j < jn && k0 + uu < H;
        sw[rr][j] = in ? w_hh[(size_t)(gg * H + k0 + uu) * H + j0 + j] : 0.0f;
      }
      __syncthreads();
#pragma unroll
      for (int q = 0; q < kMaxB / 8; ++q) {
        const int b = bq + 8 * q;
        if (b < B) {
          float a = acc[q];
          for (int j = 0; j < kChunk; ++j) a = fmaf(sh[b][j], sw[r][j], a);
          acc[q] = a;
        }
      }
      __syncthreads();
    }
  }
  // Gate pre-activations ((pre + b_ih) + b_hh) + h_prev . W_hh^T (lstm.h:380-386).
  if (k0 + u < H) {
#pragma unroll
    for (int q = 0; q < kMaxB / 8; ++q) {
      const int b = bq + 8 * q;
      if (b < B) {
        float v = __fadd_rn(__fadd_rn(pre[((size_t)t * B + b) * 4 * H + row], b_ih[row]), b_hh[row]);
        if (t > 0) v = __fadd_rn(v, acc[q]);
        gates[b][r] = v;
      }
    }
  }
  __syncthreads();
  // Cell update for (b, unit) pairs (lstm.h:389-407).
  for (int i = threadIdx.x; i < B * kUnits; i += kThreads) {
    const int b = i / kUnits, uu = i % kUnits, k = k0 + uu;
    if (k >= H) continue;
    const float ig = sigmoid_f(gates[b][0 * kUnits + uu]);
    const float fg = sigmoid_f(gates[b][1 * kUnits + uu]);
    const float gg = tanhf(gates[b][2 * kUnits + uu]);
    const float og = sigmoid_f(gates[b][3 * kUnits + uu]);
    const size_t s = ((size_t)t * B + b) * H + k;
    const float c_prev = t > 0 ? cache.c[s - (size_t)B * H] : 0.0f;
    const float c = __fadd_rn(__fmul_rn(fg, c_prev), __fmul_rn(ig, gg));
    const float tc = tanhf(c);
    cache.i[s] = ig;
    cache.f[s] = fg;
    cache.g[s] = gg;
    cache.o[s] = og;
    cache.c[s] = c;
    cache.tc[s] = tc;
    out[s] = __fmul_rn(og, tc);
  }
}

// ------------------------------------------------------------ whole sequences
//
// The recurrence in one cooperative launch (all CTAs resident at once): CTA c
// owns hidden units [c*kUnits, (c+1)*kUnits) for every step, keeps the weight
// rows those units need in shared memory for the whole sequence, and meets
// the other CTAs at a grid barrier after each step, since the next step reads
// every unit's output.  Each step does the same sums in the same order as the
// per-step kernels above, so the results are the same bits.  The barrier is
// a counter in the caller's workspace (zeroed before the launch); its wait is
// bounded (2 s of %globaltimer), after which the CTA raises g_timeout, which
// ns_kernel_health() reports, and returns.
__device__ int g_timeout;

__device__ __forceinline__ unsigned long long now_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ unsigned ld_acquire(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
// This CTA's writes of the step, then its arrival.
__device__ __forceinline__ void grid_arrive(unsigned* bar) {
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    atomicAdd(bar, 1u);
  }
}
// Until `target` arrivals (false after the time limit; every thread gets the answer).
__device__ __forceinline__ bool grid_wait(const unsigned* bar, unsigned target) {
  __shared__ int ok;
  if (threadIdx.x == 0) {
    const unsigned long long t0 = now_ns();
    int good = 1;
    while (ld_acquire(bar) < target) {
      if (now_ns() - t0 > 2000000000ull) {
        atomicExch(&g_timeout, 1);
        good = 0;
        break;
      }
      __nanosleep(64);
    }
    ok = good;
  }
  __syncthreads();
  return ok != 0;
}

// Dynamic shared memory of the whole-sequence kernels (bytes).
__host__ __device__ inline size_t seq_fwd_smem(int B, int H) {
  return ((((size_t)kRows * (H + 1) + 3) & ~(size_t)3) + (size_t)B * H) * sizeof(float);
}
__host__ __device__ inline size_t seq_bwd_smem(int B, int H) {
  return ((((size_t)kUnits * (4 * H + 1) + 3) & ~(size_t)3) + (size_t)B * 4 * H) * sizeof(float);
}

__global__ void __launch_bounds__(kThreads) lstm_seq_fwd_k(
    const float* __restrict__ pre, const float* __restrict__ w_hh, const float* __restrict__ b_ih,
    const float* __restrict__ b_hh, int T, int B, int H, float* __restrict__ out, Cache cache,
    unsigned* bar) {
  extern __shared__ __align__(16) float sm[];
  const int pitch = H + 1;          // odd row pitch: the 32 rows of a warp in different banks
  float* sw = sm;                   // [kRows][pitch]: W_hh row g*H + k0 + u at g*kUnits + u
  float* shp = sm + ((kRows * pitch + 3) & ~3);  // [B][H]: h_{t-1} (16-byte aligned)
  __shared__ float gates[kMaxB][kRows];
  const int k0 = blockIdx.x * kUnits;
  const int r = threadIdx.x % kRows, bq = threadIdx.x / kRows;
  const int g = r / kUnits, u = r % kUnits;
  const int row = g * H + k0 + u;
  for (int i = threadIdx.x; i < kRows * H; i += kThreads) {
    const int rr = i / H, j = i - rr * H;
    const int gg = rr / kUnits, uu = rr % kUnits;
    sw[rr * pitch + j] = k0 + uu < H ? w_hh[(size_t)(gg * H + k0 + uu) * H + j] : 0.0f;
  }
  for (int t = 0; t < T; ++t) {
    float acc[kMaxB / 8];
#pragma unroll
    for (int q = 0; q < kMaxB / 8; ++q) acc[q] = 0.0f;
    if (t > 0) {
      if (!grid_wait(bar, (unsigned)t * gridDim.x)) return;
      stage_async(shp, out + (size_t)(t - 1) * B * H, B * H);  // through L2: other SMs' writes
      cp_async_wait_all();
      __syncthreads();
      const float* wr = sw + r * pitch;
#pragma unroll
      for (int q = 0; q < kMaxB / 8; ++q) {
        const int b = bq + 8 * q;
        if (b < B) {
          const float* hb = shp + (size_t)b * H;
          float a = 0.0f;
          for (int j = 0; j < H; ++j) a = fmaf(hb[j], wr[j], a);
          acc[q] = a;
        }
      }
    } else {
      __syncthreads();  // the weight rows are in place
    }
    if (k0 + u < H) {
#pragma unroll
      for (int q = 0; q < kMaxB / 8; ++q) {
        const int b = bq + 8 * q;
        if (b < B) {
          float v = __fadd_rn(__fadd_rn(pre[((size_t)t * B + b) * 4 * H + row], b_ih[row]), b_hh[row]);
          if (t > 0) v = __fadd_rn(v, acc[q]);
          gates[b][r] = v;
        }
      }
    }
    __syncthreads();
    for (int i = threadIdx.x; i < B * kUnits; i += kThreads) {
      const int b = i / kUnits, uu = i % kUnits, k = k0 + uu;
      if (k >= H) continue;
      const float ig = sigmoid_f(gates[b][0 * kUnits + uu]);
      const float fg = sigmoid_f(gates[b][1 * kUnits + uu]);
      const float gg = tanhf(gates[b][2 * kUnits + uu]);
      const float og = sigmoid_f(gates[b][3 * kUnits + uu]);
      const size_t s = ((size_t)t * B + b) * H + k;
      const float c_prev = t > 0 ? cache.c[s - (size_t)B * H] : 0.0f;
      const float c = __fadd_rn(__fmul_rn(fg, c_prev), __fmul_rn(ig, gg));
      const float tc = tanhf(c);
      cache.i[s] = ig;
      cache.f[s] = fg;
      cache.g[s] = gg;
      cache.o[s] = og;
      cache.c[s] = c;
      cache.tc[s] = tc;
      out[s] = __fmul_rn(og, tc);
    }
    grid_arrive(bar);
  }
}

__global__ void __launch_bounds__(kThreads) lstm_seq_bwd_k(
    const float* __restrict__ dout, const float* __restrict__ w_t, int T, int B, int H,
    Cache cache, float* __restrict__ dc_next, float* __restrict__ dpre, unsigned* bar) {
  extern __shared__ __align__(16) float sm[];
  const int G = 4 * H, pitch = G + 1;
  float* sw = sm;                    // [kUnits][pitch]: rows k0 .. k0+kUnits-1 of W_hh^T
  float* sd = sm + ((kUnits * pitch + 3) & ~3);  // [B][G]: dpre_{t+1} (16-byte aligned)
  __shared__ float dhn[kMaxB][kUnits];
  const int k0 = blockIdx.x * kUnits;
  for (int i = threadIdx.x; i < kUnits * G; i += kThreads) {
    const int uu = i / G, j = i - uu * G;
    sw[uu * pitch + j] = k0 + uu < H ? w_t[(size_t)(k0 + uu) * G + j] : 0.0f;
  }
  __syncthreads();
  unsigned round = 0;
  for (int t = T - 1; t >= 0; --t, ++round) {
    if (t < T - 1) {
      if (!grid_wait(bar, round * gridDim.x)) return;
      stage_async(sd, dpre + (size_t)(t + 1) * B * G, B * G);  // through L2: other SMs' writes
      cp_async_wait_all();
      __syncthreads();
    }
    for (int base = 0; base < B * kUnits; base += kThreads) {
      const int o = base + threadIdx.x;
      if (o >= B * kUnits) break;
      const int b = o / kUnits, uu = o % kUnits;
      float a = 0.0f;
      if (t < T - 1) {
        const float* db = sd + (size_t)b * G;
        const float* wr = sw + uu * pitch;
        for (int j = 0; j < G; ++j) a = fmaf(db[j], wr[j], a);
      }
      dhn[b][uu] = a;
    }
    __syncthreads();
    for (int i = threadIdx.x; i < B * kUnits; i += kThreads) {
      const int b = i / kUnits, uu = i % kUnits, k = k0 + uu;
      if (k >= H) continue;
      const size_t s = ((size_t)t * B + b) * H + k;
      const float ig = cache.i[s], fg = cache.f[s], gg = cache.g[s], og = cache.o[s], tc = cache.tc[s];
      const float c_prev = t > 0 ? cache.c[s - (size_t)B * H] : 0.0f;
      const float dh = __fadd_rn(dout[s], dhn[b][uu]);
      const float do_g = __fmul_rn(dh, tc);
      const float dc = __fadd_rn(
          __fmul_rn(__fmul_rn(dh, og), __fsub_rn(1.0f, __fmul_rn(tc, tc))),
          dc_next[(size_t)b * H + k]);
      float* dr = dpre + ((size_t)t * B + b) * G;
      dr[k] = __fmul_rn(__fmul_rn(__fmul_rn(dc, gg), ig), __fsub_rn(1.0f, ig));
      dr[H + k] = __fmul_rn(__fmul_rn(__fmul_rn(dc, c_prev), fg), __fsub_rn(1.0f, fg));
      dr[2 * H + k] = __fmul_rn(__fmul_rn(dc, ig), __fsub_rn(1.0f, __fmul_rn(gg, gg)));
      dr[3 * H + k] = __fmul_rn(__fmul_rn(do_g, og), __fsub_rn(1.0f, og));
      dc_next[(size_t)b * H + k] = __fmul_rn(dc, fg);
    }
    grid_arrive(bar);
  }
}

// w_t[k][g] = w_hh[g][k]: W_hh^T [H, 4H], so the backward's dh_next reads rows.
__global__ void transpose_k(const float* __restrict__ w, int R, int C, float* __restrict__ wt) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < (int64_t)R * C;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int r = (int)(i / C), c = (int)(i % C);
    wt[(size_t)c * R + r] = w[i];
  }
}

// One backward step t (lstm.h:449-489): for this CTA's units, dh_next =
// dpre_{t+1} . W_hh (zero at t = T-1), then dh = dout + dh_next and the four
// gate gradients of step t; dc (carried in dc_next) for step t-1.
__global__ void __launch_bounds__(kThreads) lstm_step_bwd_k(
    const float* __restrict__ dout, const float* __restrict__ w_t, int t, int T, int B, int H,
    Cache cache, float* __restrict__ dc_next, float* __restrict__ dpre) {
  __shared__ float sd[kMaxB][kChunk + 1];
  __shared__ float sw[kUnits][kChunk + 1];
  __shared__ float dhn[kMaxB][kUnits];
  pdl_wait();  // launched as a programmatic dependent of the previous step
  pdl_trigger();
  const int k0 = blockIdx.x * kUnits;
  const int G = 4 * H;
  // dh_next for (b, unit): one output per thread (B * kUnits <= 512: two rounds).
  for (int base = 0; base < B * kUnits; base += kThreads) {
    const int o = base + threadIdx.x;
    const int b = o / kUnits, uu = o % kUnits;
    float a = 0.0f;
    if (t < T - 1) {
      const float* dp = dpre + (size_t)(t + 1) * B * G;
      for (int j0 = 0; j0 < G; j0 += kChunk) {
        for (int i = threadIdx.x; i < B * kChunk; i += kThreads) {
          const int bb = i / kChunk, j = i % kChunk;
          sd[bb][j] = j0 + j < G ? dp[(size_t)bb * G + j0 + j] : 0.0f;
        }
        for (int i = threadIdx.x; i < kUnits * kChunk; i += kThreads) {
          const int u2 = i / kChunk, j = i % kChunk;
          sw[u2][j] = (j0 + j < G && k0 + u2 < H) ? w_t[(size_t)(k0 + u2) * G + j0 + j] : 0.0f;
        }
        __syncthreads();
        if (o < B * kUnits)
          for (int j = 0; j < kChunk; ++j) a = fmaf(sd[b][j], sw[uu][j], a);
        __syncthreads();
      }
    }
    if (o < B * kUnits) dhn[b][uu] = a;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < B * kUnits; i += kThreads) {
    const int b = i / kUnits, uu = i % kUnits, k = k0 + uu;
    if (k >= H) continue;
    const size_t s = ((size_t)t * B + b) * H + k;
    const float ig = cache.i[s], fg = cache.f[s], gg = cache.g[s], og = cache.o[s], tc = cache.tc[s];
    const float c_prev = t > 0 ? cache.c[s - (size_t)B * H] : 0.0f;
    const float dh = __fadd_rn(dout[s], dhn[b][uu]);
    const float do_g = __fmul_rn(dh, tc);
    const float dc = __fadd_rn(
        __fmul_rn(__fmul_rn(dh, og), __fsub_rn(1.0f, __fmul_rn(tc, tc))),
        dc_next[(size_t)b * H + k]);
    float* dr = dpre + ((size_t)t * B + b) * G;
    dr[k] = __fmul_rn(__fmul_rn(__fmul_rn(dc, gg), ig), __fsub_rn(1.0f, ig));
    dr[H + k] = __fmul_rn(__fmul_rn(__fmul_rn(dc, c_prev), fg), __fsub_rn(1.0f, fg));
    dr[2 * H + k] = __fmul_rn(__fmul_rn(dc, ig), __fsub_rn(1.0f, __fmul_rn(gg, gg)));
    dr[3 * H + k] = __fmul_rn(__fmul_rn(do_g, og), __fsub_rn(1.0f, og));
    dc_next[(size_t)b * H + k] = __fmul_rn(dc, fg);
  }
}

// out[t] = in[T-1-t] for [T, rows, C] tensors (BiLSTM::ReverseTime, lstm.h:643-653).
__global__ void reverse_time_k(const float* __restrict__ in, int T, int64_t row, float* __restrict__ out) {
  const int64_t n = (int64_t)T * row;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int t = (int)(i / row);
    out[(int64_t)(T - 1 - t) * row + i % row] = in[i];
  }
}

// out[t][b] = [a[t][b] | r[T-1-t][b]] (BiLSTM::Forward's concatenation with the
// reverse cell's output turned back).
__global__ void concat_k(const float* __restrict__ a, const float* __restrict__ rr, int T, int B,
                         int H, float* __restrict__ out) {
  const int64_t n = (int64_t)T * B * 2 * H;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int k = (int)(i % (2 * H));
    const int64_t tb = i / (2 * H);
    const int t = (int)(tb / B), b = (int)(tb % B);
    out[i] = k < H ? a[tb * H + k] : rr[((int64_t)(T - 1 - t) * B + b) * H + k - H];
  }
}

// d_fwd[t][b] = dout[t][b][:H]; d_rev[T-1-t][b] = dout[t][b][H:].
__global__ void split_k(const float* __restrict__ dout, int T, int B, int H,
                        float* __restrict__ df, float* __restrict__ dr) {
  const int64_t n = (int64_t)T * B * 2 * H;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int k = (int)(i % (2 * H));
    const int64_t tb = i / (2 * H);
    const int t = (int)(tb / B), b = (int)(tb % B);
    if (k < H) df[tb * H + k] = dout[i];
    else dr[((int64_t)(T - 1 - t) * B + b) * H + k - H] = dout[i];
  }
}

// dx[t] = dxf[t] + dxr[T-1-t] (BiLSTM::Backward, lstm.h:628-634).
__global__ void add_reversed_k(const float* __restrict__ dxf, const float* __restrict__ dxr, int T,
                               int64_t row, float* __restrict__ dx) {
  const int64_t n = (int64_t)T * row;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int t = (int)(i / row);
    dx[i] = __fadd_rn(dxf[i], dxr[(int64_t)(T - 1 - t) * row + i % row]);
  }
}

int grid_for(int64_t work) {
  return (int)std::max<int64_t>(1, std::min<int64_t>((work + 255) / 256, (int64_t)sm_count() * 8));
}

size_t al64(size_t n) { return (n + 63) & ~size_t(63); }

// Workspace (floats): pre [T*B, 4H] | dpre [T*B, 4H] | W_hh^T [H, 4H] |
// dc [B, H] | GEMM workspace.
size_t gemm_ws(int T, int B, int IN, int H) {
  const int M = T * B, G = 4 * H;
  return std::max({ns_gemm_workspace_size(M, G, IN), ns_gemm_workspace_size(G, IN, M),
                   ns_gemm_workspace_size(G, H, M), ns_gemm_workspace_size(G, H, std::max(M - B, 1)),
                   ns_gemm_workspace_size(M, IN, G), ns_bias_grad_workspace_size(M, G)});
}
// Workspace (floats, 64-aligned pieces): pre | dpre | W_hh^T | dc | the
// grid-barrier counter of the whole-sequence kernels | the GEMM workspace.
size_t ws_floats(int T, int B, int IN, int H) {
  const size_t M = (size_t)T * B, G = 4 * (size_t)H;
  return 2 * al64(M * G) + al64((size_t)H * G) + al64((size_t)B * H) + 64 +
         (gemm_ws(T, B, IN, H) + 255) / sizeof(float);
}

// The whole-sequence kernel when the GPU can hold every CTA at once with its
// shared memory (a cooperative launch), else false: the caller then runs the
// per-step kernels.
thread_local int t_engine = 0;  // ns_lstm_set_engine

template <typename... Args>
bool launch_seq(void (*kernel)(Args...), int grid, size_t smem, cudaStream_t s, void** args,
                ns_status* rc) {
  *rc = NS_OK;
  if (t_engine == 1 || smem > 227 * 1024) return false;
  static thread_local int coop = -1;
  if (coop < 0) {
    int dev = 0, v = 0;
    coop = (cudaGetDevice(&dev) == cudaSuccess &&
            cudaDeviceGetAttribute(&v, cudaDevAttrCooperativeLaunch, dev) == cudaSuccess && v)
               ? 1 : 0;
  }
  if (!coop) return false;
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
      cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, kThreads, smem) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  if ((int64_t)per_sm * sm_count() < grid) return false;
  const cudaError_t e = cudaLaunchCooperativeKernel((const void*)kernel, dim3(grid), dim3(kThreads),
                                                    args, smem, s);
  if (e != cudaSuccess) {
    *rc = cuda_fail(e, "ns_lstm whole-sequence kernel");
    return true;
  }
  count_launch();
  return true;
}

ns_status check(int T, int B, int IN, int H) {
  if (T < 0 || B <= 0 || IN <= 0 || H <= 0)
    return fail(NS_ERR_INVALID_ARGUMENT, "ns_lstm: input_size and hidden_size must be positive");
  if (B > kMaxB) return fail(NS_ERR_INVALID_ARGUMENT, "ns_lstm: batch larger than 64");
  return NS_OK;
}

ns_status fwd_impl(const float* x, int T, int B, int IN, int H, const ns_lstm_weights& w,
                   float* out, float* cache, float* ws, cudaStream_t s) {
  const int M = T * B, G = 4 * H;
  float* pre = ws;
  float* gws = ws + 2 * al64((size_t)M * G) + al64((size_t)H * G) + al64((size_t)B * H) + 64;
  const size_t gbytes = gemm_ws(T, B, IN, H);
  // pre = x . W_ih^T  ([T*B, IN] x [IN, 4H]; W_ih stored [4H, IN])
  ns_status rc = ns_gemm(M, G, IN, x, IN, 0, w.w_ih, IN, 1, pre, G, 0.0f, NS_EPI_STORE, nullptr,
                         nullptr, nullptr, gws, gbytes, s);
  if (rc != NS_OK) return rc;
  Cache c = cache_at(cache, (int64_t)T * B * H);
  const int grid = (H + kUnits - 1) / kUnits;
  if (T > 1) {
    unsigned* bar = reinterpret_cast<unsigned*>(ws + 2 * al64((size_t)M * G) + al64((size_t)H * G) +
                                                al64((size_t)B * H));
    NS_TRY_CUDA(cudaMemsetAsync(bar, 0, sizeof(unsigned), s), "ns_lstm_fwd");
    const float* w_hh = w.w_hh;
    const float* b_ih = w.b_ih;
    const float* b_hh = w.b_hh;
    int T_ = T, B_ = B, H_ = H;
    void* args[] = {&pre, &w_hh, &b_ih, &b_hh, &T_, &B_, &H_, &out, &c, &bar};
    if (launch_seq(lstm_seq_fwd_k, grid, seq_fwd_smem(B, H), s, args, &rc)) return rc;
  }
  for (int t = 0; t < T; ++t) {
    rc = launch_pdl(lstm_step_fwd_k, dim3(grid), dim3(kThreads), 0, s, "ns_lstm_fwd step", pre,
                    w.w_hh, w.b_ih, w.b_hh, t, B, H, out, c);
    if (rc != NS_OK) return rc;
  }
  return NS_OK;
}

ns_status bwd_impl(const float* x, const float* out, const float* dout, int T, int B, int IN, int H,
                   const ns_lstm_weights& w, float* cache, float* dx, const ns_lstm_grads& g,
                   float* ws, cudaStream_t s) {
  const int M = T * B, G = 4 * H;
  float* dpre = ws + al64((size_t)M * G);
  float* w_t = dpre + al64((size_t)M * G);
  float* dc = w_t + al64((size_t)H * G);
  unsigned* bar = reinterpret_cast<unsigned*>(dc + al64((size_t)B * H));
  float* gws = dc + al64((size_t)B * H) + 64;
  const size_t gbytes = gemm_ws(T, B, IN, H);
  NS_TRY_CUDA(cudaMemsetAsync(dc, 0, (size_t)B * H * sizeof(float), s), "ns_lstm_bwd");
  transpose_k<<<grid_for((int64_t)G * H), 256, 0, s>>>(w.w_hh, G, H, w_t);
  ns_status rc = check_launch("ns_lstm_bwd transpose");
  Cache c = cache_at(cache, (int64_t)T * B * H);
  const int grid = (H + kUnits - 1) / kUnits;
  bool whole = false;
  if (rc == NS_OK && T > 1) {
    NS_TRY_CUDA(cudaMemsetAsync(bar, 0, sizeof(unsigned), s), "ns_lstm_bwd");
    int T_ = T, B_ = B, H_ = H;
    const float* w_tc = w_t;
    void* args[] = {&dout, &w_tc, &T_, &B_, &H_, &c, &dc, &dpre, &bar};
    whole = launch_seq(lstm_seq_bwd_k, grid, seq_bwd_smem(B, H), s, args, &rc);
  }
  for (int t = T - 1; !whole && t >= 0 && rc == NS_OK; --t) {
    rc = launch_pdl(lstm_step_bwd_k, dim3(grid), dim3(kThreads), 0, s, "ns_lstm_bwd step", dout,
                    w_t, t, T, B, H, c, dc, dpre);
  }
  if (rc != NS_OK) return rc;
  // The weight gradients sum over all T*B rows and their partial sums keep a
  // sign over long stretches of the sequence: 32-term accumulation chunks
  // halve the tensor core's round-toward-zero bias on them (gemm_tc.cuh).
  struct ChunkScope {
    int old = tc::set_accumulation_chunk(1);
    ~ChunkScope() { tc::set_accumulation_chunk(old); }
  } chunk_scope;
  // dW_ih = dpre^T . x, overwritten (lstm.h:497-500)
  rc = ns_gemm(G, IN, M, dpre, G, 1, x, IN, 0, g.w_ih, IN, 0.0f, NS_EPI_STORE, nullptr, nullptr,
               nullptr, gws, gbytes, s);
  // dW_hh = dpre^T . H_prev: H_prev's rows are out's rows shifted by one step
  // (zero for t = 0), so dW_hh = dpre[B:]^T . out[:(T-1)*B].
  if (rc == NS_OK) {
    if (T > 1)
      rc = ns_gemm(G, H, M - B, dpre + (size_t)B * G, G, 1, out, H, 0, g.w_hh, H, 0.0f,
                   NS_EPI_STORE, nullptr, nullptr, nullptr, gws, gbytes, s);
    else
      rc = cudaMemsetAsync(g.w_hh, 0, (size_t)G * H * sizeof(float), s) == cudaSuccess
               ? NS_OK
               : fail(NS_ERR_CUDA, "ns_lstm_bwd memset");
  }
  if (rc == NS_OK) {
    const size_t nb = ns_bias_grad_workspace_size(M, G);
    rc = nb <= gbytes ? ns_bias_grad(dpre, M, G, g.b_ih, gws, gbytes, s)
                      : fail(NS_ERR_INVALID_ARGUMENT, "ns_lstm_bwd: workspace for the bias sums");
  }
  if (rc == NS_OK)
    NS_TRY_CUDA(cudaMemcpyAsync(g.b_hh, g.b_ih, (size_t)G * sizeof(float), cudaMemcpyDeviceToDevice, s),
                "ns_lstm_bwd bias");
  if (rc == NS_OK && dx)
    rc = ns_gemm(M, IN, G, dpre, G, 0, w.w_ih, IN, 0, dx, IN, 0.0f, NS_EPI_STORE, nullptr, nullptr,
                 nullptr, gws, gbytes, s);
  return rc;
}

}  // namespace

// 1 if a whole-sequence kernel gave up its grid barrier since the last call
// (the flag is cleared), 0 if not, -(CUDA error) if the flag cannot be read.
int consume_timeout_flag() {
  int v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, g_timeout, sizeof(int));
  if (e != cudaSuccess) return -(int)e;
  if (v) {
    const int zero = 0;
    e = cudaMemcpyToSymbol(g_timeout, &zero, sizeof(int));
    if (e != cudaSuccess) return -(int)e;
  }
  return v ? 1 : 0;
}

}  // namespace lstm
}  // namespace nsb

using namespace nsb;
using namespace nsb::lstm;

extern "C" {

size_t ns_lstm_cache_floats(int T, int B, int H) { return (size_t)6 * T * B * H; }

size_t ns_lstm_workspace_size(int T, int B, int IN, int H) {
  if (check(T, B, IN, H) != NS_OK) return 0;
  return std::max<size_t>(ws_floats(T, B, IN, H) * sizeof(float), 256);
}

ns_status ns_lstm_set_engine(int engine) {
  NS_REQUIRE(engine == 0 || engine == 1, "ns_lstm_set_engine: engine must be 0 or 1");
  t_engine = engine;
  return NS_OK;
}

ns_status ns_lstm_fwd(const float* x, int T, int B, int IN, int H, ns_lstm_weights w, float* out,
                      float* cache, void* workspace, size_t workspace_bytes, void* stream) {
  ns_status rc = check(T, B, IN, H);
  if (rc != NS_OK || T == 0) return rc;
  NS_REQUIRE(x && w.w_ih && w.w_hh && w.b_ih && w.b_hh && out && cache, "ns_lstm_fwd: NULL argument");
  NS_REQUIRE(workspace && workspace_bytes >= ns_lstm_workspace_size(T, B, IN, H),
             "ns_lstm_fwd: workspace smaller than ns_lstm_workspace_size");
  return fwd_impl(x, T, B, IN, H, w, out, cache, static_cast<float*>(workspace), as_stream(stream));
}

ns_status ns_lstm_bwd(const float* x, const float* out, const float* dout, int T, int B, int IN,
                      int H, ns_lstm_weights w, float* cache, float* dx, ns_lstm_grads g,
                      void* workspace, size_t workspace_bytes, void* stream) {
  ns_status rc = check(T, B, IN, H);
  if (rc != NS_OK || T == 0) return rc;
  NS_REQUIRE(x && out && dout && w.w_ih && w.w_hh && cache && g.w_ih && g.w_hh && g.b_ih && g.b_hh,
             "ns_lstm_bwd: NULL argument");
  NS_REQUIRE(workspace && workspace_bytes >= ns_lstm_workspace_size(T, B, IN, H),
             "ns_lstm_bwd: workspace smaller than ns_lstm_workspace_size");
  return bwd_impl(x, out, dout, T, B, IN, H, w, cache, dx, g, static_cast<float*>(workspace),
                  as_stream(stream));
}

size_t ns_bilstm_workspace_size(int T, int B, int IN, int H) {
  const size_t one = ns_lstm_workspace_size(T, B, IN, H);
  if (!one) return 0;
  // + reversed x and (backward) the forward cell's dx, the reverse cell's dx,
  // and the two cells' output gradients
  return one + sizeof(float) * (3 * al64((size_t)T * B * IN) + 2 * al64((size_t)T * B * H) + 64);
}

size_t ns_bilstm_cache_floats(int T, int B, int H) { return 2 * ns_lstm_cache_floats(T, B, H) + 2 * (size_t)T * B * H; }

ns_status ns_bilstm_fwd(const float* x, int T, int B, int IN, int H, ns_lstm_weights wf,
                        ns_lstm_weights wr, float* out, float* cache, void* workspace,
                        size_t workspace_bytes, void* stream) {
  ns_status rc = check(T, B, IN, H);
  if (rc != NS_OK || T == 0) return rc;
  NS_REQUIRE(x && out && cache, "ns_bilstm_fwd: NULL argument");
  NS_REQUIRE(workspace && workspace_bytes >= ns_bilstm_workspace_size(T, B, IN, H),
             "ns_bilstm_fwd: workspace smaller than ns_bilstm_workspace_size");
  cudaStream_t s = as_stream(stream);
  const size_t one = ns_lstm_workspace_size(T, B, IN, H);
  float* ws = static_cast<float*>(workspace);
  float* xr = ws + one / sizeof(float);
  const int64_t TBH = (int64_t)T * B * H;
  // cache: forward cell | reverse cell | both cells' outputs [T, B, H]
  float* hf = cache + 2 * ns_lstm_cache_floats(T, B, H);
  float* hr = hf + TBH;
  reverse_time_k<<<grid_for((int64_t)T * B * IN), 256, 0, s>>>(x, T, (int64_t)B * IN, xr);
  rc = check_launch("ns_bilstm_fwd reverse");
  if (rc == NS_OK) rc = fwd_impl(x, T, B, IN, H, wf, hf, cache, ws, s);
  if (rc == NS_OK)
    rc = fwd_impl(xr, T, B, IN, H, wr, hr, cache + ns_lstm_cache_floats(T, B, H), ws, s);
  if (rc != NS_OK) return rc;
  concat_k<<<grid_for(2 * TBH), 256, 0, s>>>(hf, hr, T, B, H, out);
  return check_launch("ns_bilstm_fwd concat");
}

ns_status ns_bilstm_bwd(const float* x, const float* dout, int T, int B, int IN, int H,
                        ns_lstm_weights wf, ns_lstm_weights wr, float* cache, float* dx,
                        ns_lstm_grads gf, ns_lstm_grads gr, void* workspace,
                        size_t workspace_bytes, void* stream) {
  ns_status rc = check(T, B, IN, H);
  if (rc != NS_OK || T == 0) return rc;
  NS_REQUIRE(x && dout && cache, "ns_bilstm_bwd: NULL argument");
  NS_REQUIRE(workspace && workspace_bytes >= ns_bilstm_workspace_size(T, B, IN, H),
             "ns_bilstm_bwd: workspace smaller than ns_bilstm_workspace_size");
  cudaStream_t s = as_stream(stream);
  const size_t one = ns_lstm_workspace_size(T, B, IN, H);
  float* ws = static_cast<float*>(workspace);
  const int64_t TBH = (int64_t)T * B * H, TBI = (int64_t)T * B * IN;
  float* xr = ws + one / sizeof(float);
  float* dxf = xr + al64((size_t)TBI);
  float* dxr = dxf + al64((size_t)TBI);  // the reverse cell's dx, in its own time order
  float* df = dxr + al64((size_t)TBI);
  float* dr = df + al64((size_t)TBH);
  float* hf = cache + 2 * ns_lstm_cache_floats(T, B, H);
  float* hr = hf + TBH;
  reverse_time_k<<<grid_for(TBI), 256, 0, s>>>(x, T, (int64_t)B * IN, xr);
  rc = check_launch("ns_bilstm_bwd reverse");
  if (rc != NS_OK) return rc;
  split_k<<<grid_for(2 * TBH), 256, 0, s>>>(dout, T, B, H, df, dr);
  rc = check_launch("ns_bilstm_bwd split");
  if (rc == NS_OK) rc = bwd_impl(x, hf, df, T, B, IN, H, wf, cache, dx ? dxf : nullptr, gf, ws, s);
  if (rc == NS_OK)
    rc = bwd_impl(xr, hr, dr, T, B, IN, H, wr, cache + ns_lstm_cache_floats(T, B, H),
                  dx ? dxr : nullptr, gr, ws, s);
  if (rc != NS_OK || !dx) return rc;
  add_reversed_k<<<grid_for(TBI), 256, 0, s>>>(dxf, dxr, T, (int64_t)B * IN, dx);
  return check_launch("ns_bilstm_bwd add");
}

}  // extern "C"
