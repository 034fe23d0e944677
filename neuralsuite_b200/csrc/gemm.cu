// K1 dispatcher: ns_gemm routes to the tcgen05 3xTF32 kernel whenever the
// operands can be described to TMA (row pitches and base addresses 16-byte
// aligned), and to a plain fp32 SIMT kernel otherwise (ragged pitches such as
// the reference's odd test shapes).  Both run on the GPU; there is no host
// fallback.
#include <algorithm>

#include "epilogue.cuh"
#include "attention_tc.cuh"
#include "gemm_tc.cuh"

namespace nsb {
namespace lstm {
int consume_timeout_flag();  // lstm.cu
}  // namespace lstm
namespace {

// 0 auto, 1 SIMT, 2 tcgen05 with in-kernel operand split, 3 / 4: pre-split operands on
// 256 x 256 pair tiles / 128 x 256 tiles only, 5: 128 x 256 tiles storing rows (not C^T),
// 6 / 7: pair tiles 256 x 192 / 256 x 128 only
thread_local int t_engine = 0;

constexpr int kSB = 64, kSK = 16;

// SIMT fp32 GEMM: 64x64 tile, 256 threads, 4x4 outputs per thread, any
// transpose flags, any pitches.  C = op(A) op(B), epilogue applied per element.
template <bool AT, bool BT>
__global__ void __launch_bounds__(256) gemm_simt_k(int M, int N, int K, const float* __restrict__ A,
                                                   int lda, const float* __restrict__ B, int ldb,
                                                   const EpiArgs e_param) {
  const EpiArgs e = e_param;  // in registers, not re-read from parameter space
  __shared__ float As[kSK][kSB + 4];
  __shared__ float Bs[kSK][kSB + 4];
  const int tid = threadIdx.x, ty = tid >> 4, tx = tid & 15;
  const int m0 = blockIdx.y * kSB, n0 = blockIdx.x * kSB;
  float acc[4][4] = {};
  for (int k0 = 0; k0 < K; k0 += kSK) {
    for (int i = tid; i < kSB * kSK; i += 256) {
      int mm, kk;
      if (AT) { kk = i / kSB; mm = i % kSB; } else { mm = i / kSK; kk = i % kSK; }
      const int m = m0 + mm, k = k0 + kk;
      As[kk][mm] = (m < M && k < K) ? (AT ? A[(size_t)k * lda + m] : A[(size_t)m * lda + k]) : 0.f;
      int nn, kb;
      if (BT) { nn = i / kSK; kb = i % kSK; } else { kb = i / kSB; nn = i % kSB; }
      const int n = n0 + nn, k2 = k0 + kb;
      Bs[kb][nn] = (n < N && k2 < K) ? (BT ? B[(size_t)n * ldb + k2] : B[(size_t)k2 * ldb + n]) : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < kSK; ++kk) {
      float a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = As[kk][ty * 4 + i];
#pragma unroll
      for (int j = 0; j < 4; ++j) b[j] = Bs[kk][tx + 16 * j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int m = m0 + ty * 4 + i;
    if (m >= M) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int n = n0 + tx + 16 * j;
      if (n < N) epi_store(e, m, n, acc[i][j]);
    }
  }
}

ns_status gemm_simt(int M, int N, int K, const float* A, int lda, int at, const float* B, int ldb,
                    int bt, const EpiArgs& e, cudaStream_t s) {
  const dim3 grid(ceil_div(N, kSB), ceil_div(M, kSB)), block(256);
  if (!at && !bt) gemm_simt_k<false, false><<<grid, block, 0, s>>>(M, N, K, A, lda, B, ldb, e);
  else if (!at && bt) gemm_simt_k<false, true><<<grid, block, 0, s>>>(M, N, K, A, lda, B, ldb, e);
  else if (at && !bt) gemm_simt_k<true, false><<<grid, block, 0, s>>>(M, N, K, A, lda, B, ldb, e);
  else gemm_simt_k<true, true><<<grid, block, 0, s>>>(M, N, K, A, lda, B, ldb, e);
  return check_launch("ns_gemm simt");
}

bool tma_ok(const float* p, int ld) {
  return (reinterpret_cast<uintptr_t>(p) & 15) == 0 && ld % 4 == 0 && ld > 0;
}

bool use_tc(int M, int N, int K, const float* A, int lda, const float* B, int ldb) {
  if (t_engine == 1) return false;
  if (M <= 0 || N <= 0 || K <= 0) return false;
  if (!tma_ok(A, lda) || !tma_ok(B, ldb)) return false;
  static const int supported = ns_device_supported();  // thread-safe, once
  return supported == 1;
}

}  // namespace
}  // namespace nsb

using namespace nsb;

extern "C" {

size_t ns_gemm_workspace_size(int M, int N, int K) {
  if (M <= 0 || N <= 0 || K <= 0) return 0;
  // Enough for any plan ns_gemm may pick (every kernel, both store orientations).
  size_t part = 0;
  for (bool wide : {true, false})
    for (int force = -1; force <= 5; ++force)
      for (int trans = 0; trans <= 1; ++trans) {
        if (!wide && force > 0) continue;
        const tc::Plan p = tc::plan(M, N, K, true, wide, force, trans);
        part = std::max(part, (tc::split_workspace_bytes(p, M, N) + 255) & ~(size_t)255);
      }
  return part + tc::lo_workspace_bytes(M, N, K);
}

ns_status ns_gemm_set_engine(int engine) {
  NS_REQUIRE(engine >= 0 && engine <= 11, "ns_gemm_set_engine: engine must be 0..11");
  t_engine = engine;
  tc::set_pair_schedule(engine == 10 ? 0 : engine == 11 ? 1 : -1);
  return NS_OK;
}

}  // extern "C"

namespace {

ns_status gemm_impl(int M, int N, int K, const float* A, int lda, int a_trans, const float* B,
                    int ldb, int b_trans, float* C, int ldc, float beta, int epilogue,
                    const float* bias, const float* aux, float* aux_out, const float* a_lo_in,
                    const float* b_lo_in, float* out_lo, void* workspace, size_t workspace_bytes,
                    void* stream) {
  NS_REQUIRE(M >= 0 && N >= 0 && K >= 0, "ns_gemm: negative dimension");
  NS_REQUIRE(epilogue >= NS_EPI_STORE && epilogue <= NS_EPI_GELU_BWD, "ns_gemm: unknown epilogue");
  NS_REQUIRE(beta == 0.0f || beta == 1.0f, "ns_gemm: beta must be 0 or 1");
  NS_REQUIRE(beta == 0.0f || epilogue == NS_EPI_STORE, "ns_gemm: beta=1 needs NS_EPI_STORE");
  NS_REQUIRE(ldc >= N, "ns_gemm: ldc < N");
  NS_REQUIRE(lda >= (a_trans ? M : K) && ldb >= (b_trans ? K : N), "ns_gemm: leading dimension too small");
  const bool need_bias = epilogue == NS_EPI_BIAS || epilogue == NS_EPI_BIAS_GELU ||
                         epilogue == NS_EPI_BIAS_RESID;
  NS_REQUIRE(!need_bias || bias, "ns_gemm: epilogue needs bias");
  NS_REQUIRE(!(epilogue == NS_EPI_BIAS_RESID || epilogue == NS_EPI_GELU_BWD) || aux,
             "ns_gemm: epilogue needs aux");
  NS_REQUIRE(epilogue != NS_EPI_BIAS_GELU || aux_out, "ns_gemm: epilogue needs aux_out");
  const int a_cols = a_trans ? M : K, b_cols = b_trans ? K : N;  // lo copies need 16-byte rows
  NS_REQUIRE(!a_lo_in || (a_cols % 4 == 0 && (reinterpret_cast<uintptr_t>(a_lo_in) & 15) == 0),
             "ns_gemm_lo: a_lo needs 16-byte aligned rows (stored columns a multiple of 4)");
  NS_REQUIRE(!b_lo_in || (b_cols % 4 == 0 && (reinterpret_cast<uintptr_t>(b_lo_in) & 15) == 0),
             "ns_gemm_lo: b_lo needs 16-byte aligned rows (stored columns a multiple of 4)");
  NS_REQUIRE(!out_lo || out_lo != C, "ns_gemm_lo_out: out_lo must not alias C");
  if (M == 0 || N == 0) return NS_OK;
  EpiArgs e{C, ldc, epilogue, beta, bias, aux, aux_out, out_lo};
  cudaStream_t s = as_stream(stream);
  if (K == 0 || !use_tc(M, N, K, A, lda, B, ldb))
    return gemm_simt(M, N, K, A, lda, a_trans, B, ldb, b_trans, e, s);
  // Workspace: [split-K partials | lo(A) | lo(B)], each part used only if it fits
  // (lo parts the caller supplies take no room).  The pre-split path (lo parts
  // loaded by TMA) allows 128 x 256 tiles; otherwise the kernel splits in
  // shared memory.
  const bool ws_ok = workspace && (reinterpret_cast<uintptr_t>(workspace) & 255) == 0;
  const bool pre_ok = (t_engine == 0 || t_engine >= 3) && a_cols % 4 == 0 && b_cols % 4 == 0;
  const int force = t_engine == 3   ? 2
                    : (t_engine == 4 || t_engine == 5) ? 1
                    : t_engine == 6 ? 3
                    : t_engine == 7 ? 4
                    : t_engine == 8 ? 5
                                    : -1;
  // The wide kernels compute C^T (coalesced column stores); epilogues that
  // read the aux operand then run as a separate pass (tc::run).
  const int trans_mode = t_engine == 5 ? 0 : 1;
  const size_t lo_bytes = ((a_lo_in ? 0 : tc::lo_elems_a(M, K)) + (b_lo_in ? 0 : tc::lo_elems_a(N, K))) *
                          sizeof(float);
  tc::Plan pl{};
  size_t part = 0;
  float* lo = nullptr;
  bool chosen = false;
  const bool stream_k = t_engine != 9;
  for (int attempt = 0; attempt < 3 && !chosen; ++attempt) {
    // wide tiles with split-K / stream-K, wide tiles without, then 128 x 128 tiles
    const bool wide = attempt < 2;
    if (!pre_ok) break;
    if (force >= 0 && !wide) break;
    pl = tc::plan(M, N, K, ws_ok && attempt != 1, wide, force, trans_mode, stream_k);
    part = (tc::split_workspace_bytes(pl, M, N) + 255) & ~(size_t)255;
    if (lo_bytes == 0 && part == 0) {
      chosen = true;
    } else if (ws_ok && part + lo_bytes <= workspace_bytes) {
      if (lo_bytes) lo = reinterpret_cast<float*>(static_cast<char*>(workspace) + part);
      chosen = true;
    }
  }
  if (!chosen) {
    a_lo_in = b_lo_in = nullptr;
    pl = tc::plan(M, N, K, ws_ok, false);
    part = (tc::split_workspace_bytes(pl, M, N) + 255) & ~(size_t)255;
    if (!ws_ok || part > workspace_bytes) {
      pl = tc::plan(M, N, K, false, false);
      part = 0;
    }
  }
  return tc::run(pl, M, N, K, A, lda, a_trans, B, ldb, b_trans ? 0 : 1, e,
                 static_cast<float*>(workspace), lo, a_lo_in, b_lo_in, s);
}

}  // namespace

extern "C" {

ns_status ns_gemm(int M, int N, int K, const float* A, int lda, int a_trans, const float* B,
                  int ldb, int b_trans, float* C, int ldc, float beta, int epilogue,
                  const float* bias, const float* aux, float* aux_out, void* workspace,
                  size_t workspace_bytes, void* stream) {
  return gemm_impl(M, N, K, A, lda, a_trans, B, ldb, b_trans, C, ldc, beta, epilogue, bias, aux,
                   aux_out, nullptr, nullptr, nullptr, workspace, workspace_bytes, stream);
}

ns_status ns_gemm_lo(int M, int N, int K, const float* A, int lda, int a_trans, const float* a_lo,
                     const float* B, int ldb, int b_trans, const float* b_lo, float* C, int ldc,
                     float beta, int epilogue, const float* bias, const float* aux,
                     float* aux_out, void* workspace, size_t workspace_bytes, void* stream) {
  return gemm_impl(M, N, K, A, lda, a_trans, B, ldb, b_trans, C, ldc, beta, epilogue, bias, aux,
                   aux_out, a_lo, b_lo, nullptr, workspace, workspace_bytes, stream);
}

ns_status ns_gemm_lo_out(int M, int N, int K, const float* A, int lda, int a_trans, const float* a_lo,
                         const float* B, int ldb, int b_trans, const float* b_lo, float* C, int ldc,
                         float beta, int epilogue, const float* bias, const float* aux,
                         float* aux_out, float* out_lo, void* workspace, size_t workspace_bytes,
                         void* stream) {
  return gemm_impl(M, N, K, A, lda, a_trans, B, ldb, b_trans, C, ldc, beta, epilogue, bias, aux,
                   aux_out, a_lo, b_lo, out_lo, workspace, workspace_bytes, stream);
}

ns_status ns_split_lo(const float* x, int rows, int cols, int ld, float* lo, void* stream) {
  NS_REQUIRE(rows >= 0 && cols >= 0 && ld >= cols, "ns_split_lo: bad shape");
  if (rows == 0 || cols == 0) return NS_OK;
  return tc::split_operand(x, rows, cols, ld, lo, as_stream(stream));
}

ns_status ns_selftest_device_wait(int limit_us, void* stream) {
  NS_REQUIRE(limit_us > 0 && limit_us <= 1000000, "ns_selftest_device_wait: limit_us must be in (0, 1e6]");
  if (ns_device_supported() != 1) return fail(NS_ERR_UNSUPPORTED, "ns_selftest_device_wait: no sm_100 device");
  return tc::wait_probe(limit_us, as_stream(stream));
}

ns_status ns_kernel_health(void) {
  const int g = tc::consume_timeout_flag();
  const int a = attn_tc::consume_timeout_flag();
  const int l = lstm::consume_timeout_flag();
  if (g < 0) return cuda_fail((cudaError_t)(-g), "ns_kernel_health: reading the GEMM flag");
  if (a < 0) return cuda_fail((cudaError_t)(-a), "ns_kernel_health: reading the attention flag");
  if (l < 0) return cuda_fail((cudaError_t)(-l), "ns_kernel_health: reading the LSTM flag");
  if (g) return fail(NS_ERR_TIMEOUT, "a tcgen05 GEMM gave up a bounded wait (see ns_gemm)");
  if (a) return fail(NS_ERR_TIMEOUT, "a tcgen05 attention kernel gave up a bounded wait");
  if (l) return fail(NS_ERR_TIMEOUT, "an LSTM whole-sequence kernel gave up its grid barrier");
  return NS_OK;
}

}  // extern "C"
