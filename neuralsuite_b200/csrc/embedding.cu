// K4: token + position embedding forward, and the deterministic backward that
// reproduces the reference's sequential scatter-add bit for bit.
//
// Backward of wte (include/layers/embedding.h:61-80, include/gpt.h:262-269):
// the reference zeroes dW and adds the rows of dx in (b, t) order, then adds
// the LM-head term.  One CTA per vocabulary entry v compacts, in ascending
// order, the rows whose token is v (a ballot + prefix scan over the token
// array, 4 KB of int32 per pass, L2-resident), then each thread sums its
// columns over that list sequentially starting from +0.0f.  Same operands,
// same order, IEEE adds => identical bits, with no atomics.
#include <algorithm>

#include "common.cuh"

namespace nsb {
namespace {

__global__ void __launch_bounds__(256) emb_fwd_k(const int32_t* __restrict__ tokens, int rows,
                                                 int T, const float* __restrict__ wte, int vocab,
                                                 const float* __restrict__ wpe, int dim,
                                                 float* __restrict__ out,
                                                 int32_t* __restrict__ err) {
  pdl_wait();     // the previous kernel's writes are visible (launched by launch_pdl)
  pdl_trigger();  // the next kernel, if launched as a programmatic dependent, may start
  // blockDim.x = 256: 8 warps, one row each; lanes stride the columns.
  const int row = blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const int tok = tokens[row];
  const int t = row % T;
  float* o = out + (size_t)row * dim;
  if (tok < 0 || tok >= vocab) {
    if (lane == 0 && err) atomicExch(err, 1);
    for (int c = lane; c < dim; c += 32) o[c] = 0.0f;
    return;
  }
  const float* a = wte + (size_t)tok * dim;
  const float* b = wpe + (size_t)t * dim;
  if ((dim & 3) == 0) {
    const int n4 = dim >> 2;
    for (int c = lane; c < n4; c += 32) {
      const float4 u = reinterpret_cast<const float4*>(a)[c];
      const float4 v = reinterpret_cast<const float4*>(b)[c];
      reinterpret_cast<float4*>(o)[c] = make_float4(__fadd_rn(u.x, v.x), __fadd_rn(u.y, v.y),
                                                    __fadd_rn(u.z, v.z), __fadd_rn(u.w, v.w));
    }
  } else {
    for (int c = lane; c < dim; c += 32) o[c] = __fadd_rn(a[c], b[c]);
  }
}

constexpr int kEmbThreads = 256;
constexpr int kListChunk = 4096;  // rows compacted per pass (16 KB of smem)
constexpr int kMaxColsPerThread = 16;  // dim <= 4096

// One CTA per vocabulary row v.
__global__ void __launch_bounds__(kEmbThreads) emb_bwd_wte_k(const int32_t* __restrict__ tokens,
                                                             int rows,
                                                             const float* __restrict__ dx,
                                                             int dim, float* __restrict__ dwte,
                                                             int accumulate) {
  pdl_wait();     // the previous kernel's writes are visible (launched by launch_pdl)
  pdl_trigger();  // the next kernel, if launched as a programmatic dependent, may start
  __shared__ int list[kListChunk];
  __shared__ int warp_cnt[kEmbThreads / 32];
  __shared__ int list_len;
  const int v = blockIdx.x;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  float acc[kMaxColsPerThread];
#pragma unroll
  for (int k = 0; k < kMaxColsPerThread; ++k) acc[k] = 0.0f;
  const int ncol = (dim + kEmbThreads - 1) / kEmbThreads;

  for (int base = 0; base < rows; base += kListChunk) {
    const int end = min(rows, base + kListChunk);
    if (tid == 0) list_len = 0;
    __syncthreads();
    // Ordered compaction of {r in [base, end) : tokens[r] == v}.
    for (int r0 = base; r0 < end; r0 += kEmbThreads) {
      const int r = r0 + tid;
      const bool hit = r < end && tokens[r] == v;
      const unsigned m = __ballot_sync(0xffffffffu, hit);
      if (lane == 0) warp_cnt[warp] = __popc(m);
      __syncthreads();
      int before = list_len;
      for (int w = 0; w < warp; ++w) before += warp_cnt[w];
      if (hit) list[before + __popc(m & ((1u << lane) - 1u))] = r;
      __syncthreads();
      if (tid == 0) {
        int tot = 0;
        for (int w = 0; w < kEmbThreads / 32; ++w) tot += warp_cnt[w];
        list_len += tot;
      }
      __syncthreads();
    }
    const int n = list_len;
    // Sequential sums over the list, ascending rows, per owned column.
#pragma unroll
    for (int k = 0; k < kMaxColsPerThread; ++k) {
      const int c = tid + k * kEmbThreads;
      if (k < ncol && c < dim) {
        float s = acc[k];
        for (int i = 0; i < n; ++i) s = __fadd_rn(s, dx[(size_t)list[i] * dim + c]);
        acc[k] = s;
      }
    }
    __syncthreads();
  }
#pragma unroll
  for (int k = 0; k < kMaxColsPerThread; ++k) {
    const int c = tid + k * kEmbThreads;
    if (k < ncol && c < dim) {
      float* o = dwte + (size_t)v * dim + c;
      *o = accumulate ? __fadd_rn(acc[k], *o) : acc[k];
    }
  }
}

// dwpe[t, c] = sum over b ascending of dx[b, t, c]; rows t >= T are zeroed.
__global__ void emb_bwd_wpe_k(const float* __restrict__ dx, int B, int T, int block, int dim,
                              float* __restrict__ dwpe) {
  pdl_wait();     // the previous kernel's writes are visible (launched by launch_pdl)
  pdl_trigger();  // the next kernel, if launched as a programmatic dependent, may start
  const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (i >= (int64_t)block * dim) return;
  const int t = (int)(i / dim), c = (int)(i % dim);
  float s = 0.0f;
  if (t < T)
    for (int b = 0; b < B; ++b) s = __fadd_rn(s, dx[((size_t)b * T + t) * dim + c]);
  dwpe[i] = s;
}

}  // namespace
}  // namespace nsb

using namespace nsb;

extern "C" {

ns_status ns_embedding_fwd(const int32_t* tokens, int B, int T, const float* wte, int vocab,
                           const float* wpe, int block, int dim, float* out, int32_t* err_flag,
                           void* stream) {
  NS_REQUIRE(B >= 0 && T >= 0 && vocab > 0 && dim > 0, "ns_embedding_fwd: bad shape");
  if (T > block)
    return fail(NS_ERR_OUT_OF_RANGE, "ns_embedding_fwd: sequence length exceeds block_size");
  const int rows = B * T;
  if (rows == 0) return NS_OK;
  NS_REQUIRE((dim & 3) != 0 || ((reinterpret_cast<uintptr_t>(wte) | reinterpret_cast<uintptr_t>(wpe) |
                                 reinterpret_cast<uintptr_t>(out)) & 15) == 0,
             "ns_embedding_fwd: buffers must be 16-byte aligned");
  return launch_pdl(emb_fwd_k, dim3(ceil_div(rows, 8)), dim3(256), 0, as_stream(stream),
                    "ns_embedding_fwd", tokens, rows, T, wte, vocab, wpe, dim, out, err_flag);
}

ns_status ns_embedding_bwd(const int32_t* tokens, int B, int T, const float* dx, int vocab,
                           int block, int dim, float* dwte, int accumulate_wte, float* dwpe,
                           void* stream) {
  NS_REQUIRE(B >= 0 && T >= 0 && vocab > 0 && dim > 0 && T <= block,
             "ns_embedding_bwd: bad shape");
  NS_REQUIRE(dim <= kEmbThreads * kMaxColsPerThread, "ns_embedding_bwd: dim > 4096");
  cudaStream_t s = as_stream(stream);
  const int rows = B * T;
  if (dwte) {
    {
      const ns_status rc = launch_pdl(emb_bwd_wte_k, dim3(vocab), dim3(kEmbThreads), 0, s,
                                      "ns_embedding_bwd wte", tokens, rows, dx, dim, dwte,
                                      accumulate_wte);
      if (rc != NS_OK) return rc;
    }
  }
  if (dwpe) {
    const int64_t n = (int64_t)block * dim;
    {
      const ns_status rc = launch_pdl(emb_bwd_wpe_k, dim3((unsigned)ceil_div64(n, 256)), dim3(256),
                                      0, s, "ns_embedding_bwd wpe", dx, B, T, block, dim, dwpe);
      if (rc != NS_OK) return rc;
    }
  }
  return NS_OK;
}

}  // extern "C"
