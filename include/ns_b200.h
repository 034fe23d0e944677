/*
 * ns_b200.h -- C ABI of the B200 (sm_100a) backend for NeuralSuite's GPT
 * training step.
 *
 * The reference (NeuralSuite, a C++17 CPU library) has no plugin or FFI layer:
 * its boundary is the C++ API of Tensor / Layer::Forward / Layer::Backward /
 * Loss / Optimizer.  Each entry point below replaces one function or method of
 * that API; the reference symbol it stands in for is cited beside it
 * (paths inside the NeuralSuite project).  A C++ shim with the reference's
 * class names (neuralsuite_b200/csrc/gpt_device.h) sits on top of these calls,
 * and the model-level ns_gpt_* calls drive that shim for callers in other
 * languages.
 *
 * Conventions
 *  - Every buffer argument is a DEVICE pointer to fp32 row-major data unless
 *    its name says host_ / int32.  Token ids are int32 (the reference carries
 *    them as float and truncates, include/layers/embedding.h:43).
 *  - `stream` is a cudaStream_t passed as void* (NULL = legacy default stream).
 *  - Every call returns an ns_status; on failure ns_last_error() returns a
 *    thread-local message.  No C++ exception crosses this boundary; the C++
 *    shim rethrows std::invalid_argument / std::out_of_range like the
 *    reference.
 *  - Kernels are asynchronous on `stream`.  Entry points with a `workspace`
 *    argument take caller-owned device scratch of at least the size the
 *    matching *_workspace_size query returns; none of the kernel entry
 *    points allocates memory.
 */
#ifndef NS_B200_H_
#define NS_B200_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define NS_API __attribute__((visibility("default")))
#else
#define NS_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
  NS_OK = 0,
  NS_ERR_INVALID_ARGUMENT = 1, /* reference: std::invalid_argument */
  NS_ERR_OUT_OF_RANGE = 2,     /* reference: std::out_of_range (bad token id) */
  NS_ERR_CUDA = 3,             /* a CUDA runtime error */
  NS_ERR_UNSUPPORTED = 4,      /* e.g. no sm_100 device */
  NS_ERR_COMM = 5,             /* NCCL error or communicator aborted */
  NS_ERR_TIMEOUT = 6           /* a bounded host wait ran out */
} ns_status;

NS_API const char* ns_last_error(void);
NS_API int ns_version(void);
/* Kernels this library has launched in this process (a host-side counter,
 * for benchmarks that report how much of a step ran in this library). */
NS_API long long ns_launch_count(void);
/* 1 when the current device is an sm_100 part the tcgen05 kernels can run on. */
NS_API int ns_device_supported(void);

/* ------------------------------------------------------------------ K1 GEMM
 * C[M,N] = op(A) * op(B)  (+ epilogue), fp32 in / fp32 out, 3xTF32 on the
 * tcgen05 tensor cores (A = Ahi + Alo, B = Bhi + Blo, C ~ Ahi*Bhi + Ahi*Blo +
 * Alo*Bhi, accumulated in TMEM).
 *   a_trans = 0: A stored [M,K] (row stride lda);  1: A stored [K,M] (A^T).
 *   b_trans = 0: B stored [K,N] (row stride ldb);  1: B stored [N,K] (B^T).
 * Replaces MatMul (src/tensor.cpp:198-271) together with the Transpose copies
 * Linear / GPTModel make before the "T" products (src/tensor.cpp:275-288,
 * include/layers/linear.h:95-102, include/gpt.h:226-252).
 *
 * Epilogues (the element of the GEMM result is `acc`):
 *   NS_EPI_STORE      C = acc                       (MatMul; beta=1 adds into C)
 *   NS_EPI_BIAS       C = acc + bias[n]             (Linear::Forward, linear.h:69-76)
 *   NS_EPI_BIAS_GELU  C = acc + bias[n]; aux_out = gelu(C)
 *                     (Linear::Forward then GeluForward, src/tensor.cpp:428-443)
 *   NS_EPI_BIAS_RESID C = aux[m,n] + (acc + bias[n])
 *                     (Linear::Forward then ElementwiseAdd, include/gpt.h:70,77)
 *   NS_EPI_GELU_BWD   C = acc * gelu'(aux[m,n])     (Linear::Backward dX then
 *                     GeluBackward, src/tensor.cpp:445-461)
 * beta is 0 (overwrite, the reference's MatMul Resize+Zeros) or 1 (accumulate
 * into C, used for the weight-tied wte gradient, include/gpt.h:266-269); it is
 * only accepted with NS_EPI_STORE.  aux/aux_out rows use stride ldc.
 *
 * `workspace` (may be NULL) lets the kernel split K across CTAs when the
 * output has too few tiles to fill the GPU (the dW products), or run a
 * part-filled last wave of tiles as a stream-K tail (the leftover tiles'
 * k-blocks shared evenly by all CTA pairs); partial tiles are summed in a
 * fixed order, so results do not depend on timing.  With less than
 * ns_gemm_workspace_size bytes the call runs without either.
 *
 * Accuracy: the tensor core adds into its fp32 accumulator with
 * round-toward-zero; each 64-term run of K is accumulated in a fresh TMEM
 * buffer and folded into the result with round-to-nearest, so the error
 * stays at the level of a sequential fp32 loop (relative L2 ~1e-6 on random
 * operands, independent of K) except for a bias toward zero of up to about
 * 3e-6 x (sum of |64-term partial sums|), which shows where long runs of
 * terms share a sign.  The library's own long sequence reductions (the LSTM
 * weight gradients) use 32-term runs, which halves it.
 */
enum {
  NS_EPI_STORE = 0,
  NS_EPI_BIAS = 1,
  NS_EPI_BIAS_GELU = 2,
  NS_EPI_BIAS_RESID = 3,
  NS_EPI_GELU_BWD = 4
};
NS_API size_t ns_gemm_workspace_size(int M, int N, int K);
NS_API ns_status ns_gemm(int M, int N, int K, const float* A, int lda, int a_trans, const float* B,
                  int ldb, int b_trans, float* C, int ldc, float beta, int epilogue,
                  const float* bias, const float* aux, float* aux_out, void* workspace,
                  size_t workspace_bytes, void* stream);
/* lo = x - trunc_tf32(x) for a [rows, cols] matrix with row stride ld, written
 * compact (row stride cols): the low part of the 3xTF32 operand split that
 * ns_gemm otherwise computes into its workspace on every call.  Callers that
 * feed one operand to several products (an activation to its forward GEMM and
 * its weight-gradient GEMM; a weight to its forward and input-gradient GEMMs)
 * split it once and pass the copy to ns_gemm_lo.  cols must be a multiple of 4
 * and lo 16-byte aligned for ns_gemm_lo to use it.  No reference counterpart
 * (part of the MatMul implementation, src/tensor.cpp:198-271). */
NS_API ns_status ns_split_lo(const float* x, int rows, int cols, int ld, float* lo, void* stream);
/* ns_gemm with the operands' lo parts supplied: a_lo is ns_split_lo of A as
 * stored ([M,K], or [K,M] with a_trans), b_lo likewise of B ([K,N] or [N,K]).
 * Either may be NULL; a missing one is split into the workspace as ns_gemm
 * does.  Same results as ns_gemm, bit for bit. */
NS_API ns_status ns_gemm_lo(int M, int N, int K, const float* A, int lda, int a_trans,
                     const float* a_lo, const float* B, int ldb, int b_trans, const float* b_lo,
                     float* C, int ldc, float beta, int epilogue, const float* bias,
                     const float* aux, float* aux_out, void* workspace, size_t workspace_bytes,
                     void* stream);
/* ns_gemm_lo that also writes out_lo = the tf32 lo part (x - trunc_tf32(x))
 * of the epilogue's activation output (aux_out for NS_EPI_BIAS_GELU, C
 * otherwise; row stride ldc, not aliasing C): the next product's operand
 * split in the same pass as the store.  No reference counterpart. */
NS_API ns_status ns_gemm_lo_out(int M, int N, int K, const float* A, int lda, int a_trans,
                         const float* a_lo, const float* B, int ldb, int b_trans,
                         const float* b_lo, float* C, int ldc, float beta, int epilogue,
                         const float* bias, const float* aux, float* aux_out, float* out_lo,
                         void* workspace, size_t workspace_bytes, void* stream);
/* Selects the GEMM engine for subsequent calls on this thread: 0 = automatic
 * (tcgen05 wherever the operands allow TMA, SIMT fp32 otherwise), 1 = always
 * the SIMT fp32 kernel, 2 = tcgen05 with the operands' tf32 lo parts always
 * computed inside the kernel (never pre-split into the workspace), 3 / 4 =
 * pre-split operands on CTA-pair tiles (256 x 256, 192 or 128) / 128 x 256 tiles only
 * (where the workspace allows), 5 = as 4 but storing rows of C instead of
 * computing C^T, 6 / 7 / 8 = CTA-pair tiles 256 x 192 / 256 x 128 / 256 x 256 only,
 * 9 = as 0 but never running a part-filled last wave of CTA-pair tiles as a
 * stream-K tail (the leftover tiles' k-blocks shared by all pairs), 10 / 11
 * = as 0 but with the CTA-pair kernel's work always handed out in a fixed
 * order (cluster c takes tiles c, c + clusters, ...) / always from a
 * per-launch counter as the clusters become ready.  Under engine 0 GEMM calls
 * use the fixed order and ns_gpt_backward uses the counter when a
 * communicator with world_size > 1 is attached (the all-reduce beside the
 * backward holds SMs; clusters that start late then take fewer tiles).
 * Results are bit-identical either way.
 * TEST AND PROFILING ONLY: engines 1-11 exist so tests can cross-check the
 * kernels against one another and profiles can time one tile shape alone;
 * production callers leave the engine at 0, the only setting the planner's
 * shape choices are tuned for. */
NS_API ns_status ns_gemm_set_engine(int engine);
/* NS_ERR_TIMEOUT if any kernel of this library gave up a bounded wait on the
 * current device since the last call (the flag is cleared by the call);
 * NS_ERR_CUDA if the flag cannot be read (a sticky CUDA error on the device).
 * It synchronises with the device: do not call it while a stream is being
 * captured. */
NS_API ns_status ns_kernel_health(void);
/* No reference counterpart: a self-test of the bounded device waits above.
 * Launches one warp that waits, with the kernels' own wait routine but a limit
 * of limit_us microseconds (at most 1 s) instead of 2 s, on an mbarrier that
 * nothing arrives at; the wait runs out, raises the flag, and the kernel
 * returns, leaving the context usable.  The next ns_kernel_health() returns
 * NS_ERR_TIMEOUT. */
NS_API ns_status ns_selftest_device_wait(int limit_us, void* stream);

/* Column sums db[n] = sum_m dY[m,n]: the bias gradient of Linear::Backward
 * (include/layers/linear.h:104-111, overwritten).  Deterministic two-stage
 * reduction through `workspace`. */
NS_API size_t ns_bias_grad_workspace_size(int M, int N);
NS_API ns_status ns_bias_grad(const float* dY, int M, int N, float* db, void* workspace,
                       size_t workspace_bytes, void* stream);
/* ns_bias_grad that also writes dy_lo = ns_split_lo(dY) from the same pass
 * over dY (Linear::Backward needs both: db, and dY's tf32 lo part for the dX
 * and dW products through ns_gemm_lo).  N a multiple of 4, 16-byte aligned
 * pointers; same workspace as ns_bias_grad; db bit-identical to it.  No
 * reference counterpart (a fusion of linear.h:104-111 with the operand split). */
NS_API ns_status ns_bias_grad_split(const float* dY, int M, int N, float* db, float* dy_lo,
                             void* workspace, size_t workspace_bytes, void* stream);
/* GeluBackward fused on the way into ns_bias_grad_split: dY (the gradient at
 * the GELU output) is replaced in place by dY * gelu'(pre), and db and dy_lo
 * are those of the product (include/layers/activation.h GeluBackward followed
 * by linear.h:104-111's bias sum; one pass instead of three).  Same
 * requirements and workspace as ns_bias_grad_split; pre 16-byte aligned. */
NS_API ns_status ns_bias_grad_split_gelu(float* dY, const float* pre, int M, int N, float* db,
                                  float* dy_lo, void* workspace, size_t workspace_bytes,
                                  void* stream);

/* ------------------------------------------------------------ K2 attention
 * Fused causal self-attention on the interleaved c_attn output
 * qkv[B*T, 3*H*D] (Q of head h at columns h*D, K at C+h*D, V at 2C+h*D, the
 * layout of MultiHeadAttention::Extraer, include/layers/attention.h:563-575).
 * Forward writes out[B*T, H*D] (head h at columns h*D, attention.h:379-382)
 * and lse[B*H*T], the per-row log-sum-exp of the scaled scores, instead of the
 * reference's [B,H,T,T] probability cache (attention.h:361-378).
 * Replaces the per-(b,h) loop of MultiHeadAttention::Forward
 * (attention.h:364-384) and ::Backward (attention.h:405-461); backward writes
 * dqkv[B*T, 3C] in the same interleaved layout and needs `workspace` of
 * ns_attn_bwd_workspace_size bytes; forward needs ns_attn_fwd_workspace_size
 * bytes (16-byte aligned; 0 for head sizes without a tensor-core kernel).  Scale = 1/sqrt(D) applied after Q.K^T
 * (attention.h:362, 372-374). */
NS_API size_t ns_attn_fwd_workspace_size(int B, int T, int H, int D);
NS_API ns_status ns_attn_fwd(const float* qkv, int B, int T, int H, int D, float* out, float* lse,
                      void* workspace, size_t workspace_bytes, void* stream);
/* ns_attn_fwd with the 3xTF32 operand splits shared with the neighbouring
 * GEMMs: qkv_lo (optional) is the tf32 lo part of all of qkv (as written by
 * ns_gemm_lo_out for the c_attn product), so no K/V split runs and no
 * workspace is needed; out_lo (optional) receives the tf32 lo part of out
 * (the c_proj product's A operand split).  16-byte aligned; workspace as
 * ns_attn_fwd when qkv_lo is null.  No reference counterpart (a fusion of
 * include/layers/attention.h:364-384 with the operand splits). */
NS_API ns_status ns_attn_fwd_lo(const float* qkv, const float* qkv_lo, int B, int T, int H, int D,
                         float* out, float* out_lo, float* lse, void* workspace,
                         size_t workspace_bytes, void* stream);
/* 0 (default): head_dim 32 / 64 run on the tensor cores (3xTF32, tcgen05) in
 * both directions (the backward's dK and dV from one kernel), other sizes on
 * the SIMT kernels; 1: SIMT kernels for every size; 2: as 0 with dK and dV
 * from two separate kernels.  Per host thread.
 * No reference counterpart (engine selection for tests and profiling). */
NS_API ns_status ns_attn_set_engine(int engine);
NS_API size_t ns_attn_bwd_workspace_size(int B, int T, int H, int D);
NS_API ns_status ns_attn_bwd(const float* qkv, const float* out, const float* dout, const float* lse,
                      int B, int T, int H, int D, float* dqkv, void* workspace,
                      size_t workspace_bytes, void* stream);
/* ns_attn_bwd with qkv's tf32 lo part given (qkv_lo, optional, 16-byte
 * aligned; the forward's), so it is not split again.  Same workspace. */
NS_API ns_status ns_attn_bwd_lo(const float* qkv, const float* qkv_lo, const float* out,
                         const float* dout, const float* lse, int B, int T, int H, int D,
                         float* dqkv, void* workspace, size_t workspace_bytes, void* stream);

/* ------------------------------------------------------ K3 bandwidth kernels */
/* LayerNormForward, src/tensor.cpp:290-322 (last axis, biased variance). */
NS_API ns_status ns_layernorm_fwd(const float* x, const float* gamma, const float* beta, float* out,
                           float* mean, float* rstd, int rows, int dim, float eps, void* stream);
/* ns_layernorm_fwd with the neighbours' work fused in: with resid, the row is
 * first formed as x = resid + (x_raw + bias) (the residual add of the
 * producing GEMM's bias epilogue, same rounding; x_raw is that GEMM's plain
 * product) and written to x_out (which may be x_raw); with out_lo (optional),
 * out's tf32 lo part is written too (the next GEMM's operand split).  No
 * reference counterpart (ElementwiseAdd src/tensor.cpp:534-540 + LayerNorm
 * 290-322 + the split). */
NS_API ns_status ns_layernorm_fwd_ex(const float* x_raw, const float* bias, const float* resid,
                              float* x_out, const float* gamma, const float* beta, float* out,
                              float* out_lo, float* mean, float* rstd, int rows, int dim,
                              float eps, void* stream);
/* LayerNormBackward, src/tensor.cpp:324-359.  dgamma/dbeta are overwritten
 * (deterministic two-stage column sums through `workspace`).  If `dresid` is
 * non-NULL the result is dx = dresid + dx_ln: the ElementwiseAdd of the
 * residual gradient in GPTBlock::Backward (include/gpt.h:89-97). */
NS_API size_t ns_layernorm_bwd_workspace_size(int rows, int dim);
NS_API ns_status ns_layernorm_bwd(const float* dout, const float* x, const float* gamma,
                           const float* mean, const float* rstd, const float* dresid, float* dx,
                           float* dgamma, float* dbeta, int rows, int dim, void* workspace,
                           size_t workspace_bytes, void* stream);
/* GeluForward / GeluBackward, src/tensor.cpp:428-461. */
NS_API ns_status ns_gelu_fwd(const float* x, float* y, int64_t n, void* stream);
/* ns_gelu_fwd that also writes y_lo = y - trunc_tf32(y), the next product's
 * operand split (a pass that streams at memory speed, where the same work in
 * a GEMM epilogue holds up the GEMM).  16-byte aligned.  No reference
 * counterpart (GeluForward src/tensor.cpp:428-443 plus the split). */
NS_API ns_status ns_gelu_fwd_lo(const float* x, float* y, float* y_lo, int64_t n, void* stream);
NS_API ns_status ns_gelu_bwd(const float* dout, const float* x, float* dx, int64_t n, void* stream);
/* ElementwiseAdd, src/tensor.cpp:534-540. */
NS_API ns_status ns_add(const float* a, const float* b, float* out, int64_t n, void* stream);
/* CrossEntropyLoss::Forward + ::Backward fused (include/losses.h:34-86):
 * loss_out (one device float) = mean over rows of -log softmax(logits)[t];
 * dlogits = (softmax - onehot(t)) / denom, where denom = rows for the
 * reference's single-process step and rows*world_size under data parallel.
 * Targets out of [0, classes) are reported as NS_ERR_OUT_OF_RANGE after the
 * fact through *err_flag (device int, may be NULL). */
NS_API size_t ns_cross_entropy_workspace_size(int rows, int classes);
NS_API ns_status ns_cross_entropy(const float* logits, const int32_t* targets, int rows, int classes,
                           float denom, float* loss_out, float* dlogits, int32_t* err_flag,
                           void* workspace, size_t workspace_bytes, void* stream);
/* No counterpart in the reference: the same cross-entropy forward+backward
 * for callers that cannot allocate device memory when they call it -- code
 * recording a CUDA graph (cudaMalloc may not be called while a stream is
 * being captured), hosts whose device memory is fully owned by another
 * allocator, and loops that cannot afford cudaMalloc's implicit device
 * synchronisation.  The per-row loss scratch is a static device array inside
 * the library (NS_CE_NOALLOC_MAX_ROWS floats = 256 KiB, held by every GPU
 * that loads the library until the process exits), so nothing is allocated
 * and no workspace is passed.  rows > NS_CE_NOALLOC_MAX_ROWS is rejected with
 * NS_ERR_INVALID_ARGUMENT.  The first call on each device looks up the
 * array's device address (cudaGetSymbolAddress), and so does the first call
 * after the device's context has changed (cudaDeviceReset); make that first
 * call before any stream capture.  All calls share the one array, so calls that may
 * overlap on the GPU (different streams without ordering) race; each call
 * overwrites every scratch entry it reads, so no clearing is needed. */
#define NS_CE_NOALLOC_MAX_ROWS 65536
NS_API ns_status ns_cross_entropy_noalloc(const float* logits, const int32_t* targets, int rows,
                                   int classes, float denom, float* loss_out, float* dlogits,
                                   int32_t* err_flag, void* stream);

/* ------------------------------------------------------------ Conv2D
 * Conv2D::Forward / ::Backward (include/layers/conv2d.h:192-414), NCHW:
 * x [B, IC, H, W], weight [OC, IC, k, k], bias [OC] (may be NULL in the
 * forward), y [B, OC, OH, OW] with OH = (H + 2*pad - k)/stride + 1 (likewise
 * OW).  The batch's im2col columns [IC*k*k, B*OH*OW] go through one 3xTF32
 * tcgen05 GEMM per product.  Backward overwrites dweight [OC, IC, k, k] and
 * dbias [OC] (the reference zeroes them first) and writes dx (NULL: skipped,
 * for a first layer); the weight gradient is a deterministic split-K product
 * and dx a gather in the reference's window order (no atomics).  Both need
 * `workspace` of ns_conv2d_workspace_size bytes, 256-byte aligned.  Bad
 * parameters (non-positive sizes, a kernel larger than the padded input) are
 * NS_ERR_INVALID_ARGUMENT, the reference's std::invalid_argument. */
NS_API size_t ns_conv2d_workspace_size(int B, int IC, int H, int W, int OC, int k, int stride,
                                       int pad);
NS_API ns_status ns_conv2d_fwd(const float* x, int B, int IC, int H, int W, const float* weight,
                               const float* bias, int OC, int k, int stride, int pad, float* y,
                               void* workspace, size_t workspace_bytes, void* stream);
NS_API ns_status ns_conv2d_bwd(const float* x, const float* dy, int B, int IC, int H, int W,
                               const float* weight, int OC, int k, int stride, int pad, float* dx,
                               float* dweight, float* dbias, void* workspace,
                               size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------ LSTM / BiLSTM
 * LSTM::Forward / ::Backward (include/layers/lstm.h:320-529) and BiLSTM
 * (lstm.h:531-664): x [T, B, IN] -> out [T, B, H] (BiLSTM: [T, B, 2H], the
 * forward cell's state then the reverse cell's), gates i, f, g, o over 4H,
 * W_ih [4H, IN], W_hh [4H, H], b_ih / b_hh [4H].  The input projection and
 * the three weight/input-gradient products are tcgen05 GEMMs; the recurrence
 * is one cooperative kernel over the whole sequence (a grid barrier between
 * steps, bounded and reported by ns_kernel_health) where every CTA fits on
 * the GPU at once, else one launch per step; both give the same bits.
 * `cache` (ns_lstm_cache_floats / ns_bilstm_cache_floats
 * floats, device) carries the gates and cell states from the forward to the
 * backward; the backward overwrites every gradient (the reference's
 * MatMul/Zeros) and writes dx unless it is NULL.  B <= 64.
 * `workspace`: ns_lstm_workspace_size / ns_bilstm_workspace_size bytes. */
typedef struct {
  const float *w_ih, *w_hh, *b_ih, *b_hh;
} ns_lstm_weights;
typedef struct {
  float *w_ih, *w_hh, *b_ih, *b_hh;
} ns_lstm_grads;
NS_API size_t ns_lstm_cache_floats(int T, int B, int H);
NS_API size_t ns_lstm_workspace_size(int T, int B, int IN, int H);
NS_API ns_status ns_lstm_fwd(const float* x, int T, int B, int IN, int H, ns_lstm_weights w,
                             float* out, float* cache, void* workspace, size_t workspace_bytes,
                             void* stream);
/* out is the forward's output (it doubles as the stacked h_{t-1} of dW_hh). */
NS_API ns_status ns_lstm_bwd(const float* x, const float* out, const float* dout, int T, int B,
                             int IN, int H, ns_lstm_weights w, float* cache, float* dx,
                             ns_lstm_grads g, void* workspace, size_t workspace_bytes,
                             void* stream);
/* 0 (default): the whole-sequence recurrence where it fits, else one launch
 * per step; 1: always one launch per step.  Per host thread.  No reference
 * counterpart (engine selection for tests and profiling). */
NS_API ns_status ns_lstm_set_engine(int engine);
NS_API size_t ns_bilstm_cache_floats(int T, int B, int H);
NS_API size_t ns_bilstm_workspace_size(int T, int B, int IN, int H);
NS_API ns_status ns_bilstm_fwd(const float* x, int T, int B, int IN, int H, ns_lstm_weights fwd,
                               ns_lstm_weights rev, float* out, float* cache, void* workspace,
                               size_t workspace_bytes, void* stream);
NS_API ns_status ns_bilstm_bwd(const float* x, const float* dout, int T, int B, int IN, int H,
                               ns_lstm_weights fwd, ns_lstm_weights rev, float* cache, float* dx,
                               ns_lstm_grads gfwd, ns_lstm_grads grev, void* workspace,
                               size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------ K4 embedding
 * out[b,t,:] = wte[tok[b,t],:] + wpe[t,:]  (Embedding::Forward twice plus the
 * add of GPTModel::Forward, include/layers/embedding.h:34-59,
 * include/gpt.h:197-212).  A token outside [0, vocab) sets *err_flag (device
 * int) and its row is written as zeros; host callers validate first, which is
 * where the reference's std::out_of_range comes from (embedding.h:45-49). */
NS_API ns_status ns_embedding_fwd(const int32_t* tokens, int B, int T, const float* wte, int vocab,
                           const float* wpe, int block, int dim, float* out, int32_t* err_flag,
                           void* stream);
/* Embedding::Backward for wte and wpe (embedding.h:61-80) followed by the
 * weight-tying add of GPTModel::Backward (gpt.h:262-269):
 *   dwte[v,:] = (sum over rows r with tok[r]==v, ascending r, of dx[r,:]) + dwte[v,:]
 *   dwpe[t,:] =  sum over b ascending of dx[b,t,:]     (rows t >= T zeroed)
 * Sums run in the reference's order, so the result is bit-identical to it.
 * If accumulate_wte is 0 the incoming dwte is treated as zero. */
NS_API ns_status ns_embedding_bwd(const int32_t* tokens, int B, int T, const float* dx, int vocab,
                           int block, int dim, float* dwte, int accumulate_wte, float* dwpe,
                           void* stream);

/* -------------------------------------------------------------- K5 AdamW
 * One launch over every tensor of a flat parameter buffer (AdamW::Step,
 * include/optimizers.h:206-234): per element, in the reference's order,
 *   m = b1*m + (1-b1)*g;  v = b2*v + (1-b2)*g*g;
 *   p -= lr*wd_t*p (if wd_t > 0);  p -= lr*(m/bc1)/(sqrt(v/bc2)+eps)
 * Segment t covers [seg_offsets[t], seg_offsets[t+1]) with decay seg_decay[t]
 * (host arrays, n_seg entries; offsets has n_seg+1).  bc1 = 1 - b1^step and
 * bc2 = 1 - b2^step are computed by the caller in double and rounded to float,
 * as the reference does (optimizers.h:208-210). */
NS_API ns_status ns_adamw_flat(float* params, const float* grads, float* m, float* v, int64_t n_total,
                        const int64_t* host_seg_offsets, const float* host_seg_decay, int n_seg,
                        float lr, float b1, float b2, float eps, float bc1, float bc2,
                        void* stream);
/* The same update with its hyper-parameters in DEVICE memory, so that a step
 * captured in a CUDA graph replays correctly: dev_hyper = float[7]
 * {lr, b1, b2, eps, bc1, bc2, step}, step stored as int32 bits.  Each call
 * first increments step and recomputes bc1/bc2 on the device (double pow
 * rounded to float), then updates every segment. */
NS_API ns_status ns_adamw_flat_device(float* params, const float* grads, float* m, float* v,
                               int64_t n_total, const int64_t* host_seg_offsets,
                               const float* host_seg_decay, int n_seg, float* dev_hyper,
                               void* stream);
/* Sum of squares of a flat gradient buffer into one device float (the norm of
 * ClipGradients, train_llm.cpp:112-121), and the in-place scale by
 * min(1, max_norm / sqrt(sumsq)) of train_llm.cpp:122-128, read on the device. */
NS_API size_t ns_sumsq_workspace_size(int64_t n);
NS_API ns_status ns_sumsq(const float* x, int64_t n, float* out, void* workspace,
                   size_t workspace_bytes, void* stream);
NS_API ns_status ns_clip_scale(float* x, int64_t n, const float* sumsq, float max_norm, void* stream);

/* ------------------------------------------------- data-parallel comm (NCCL)
 * One communicator per process/GPU over NVLink.  NCCL is loaded at run time
 * (dlopen libnccl.so.2), so the library loads on machines without it.  The
 * reference has no distributed code; these exist for the data-parallel step. */
typedef struct ns_comm ns_comm;
NS_API ns_status ns_comm_unique_id(uint8_t host_id_out[128]);
/* Creates the communicator non-blocking and polls it until it is ready, with
 * a 300 s deadline: a rank that never joins makes the others return
 * NS_ERR_TIMEOUT (communicator aborted) instead of blocking inside NCCL.
 * Collectives that NCCL reports as still being enqueued, and the end-of-step
 * wait of ns_gpt_train_step, are polled with deadlines the same way, and an
 * asynchronous NCCL error aborts the communicator (NS_ERR_COMM). */
NS_API ns_status ns_comm_init(const uint8_t host_id[128], int world_size, int rank, ns_comm** out);
/* In-place sum over ranks of count floats on `stream`. */
NS_API ns_status ns_comm_allreduce_sum(ns_comm* comm, float* buf, int64_t count, void* stream);
/* Host poll of the communicator's asynchronous error state. */
NS_API ns_status ns_comm_check(ns_comm* comm);
NS_API ns_status ns_comm_abort(ns_comm* comm);
NS_API ns_status ns_comm_destroy(ns_comm* comm);
/* No reference counterpart: a self-test of the deadline and abort logic above
 * against a fake NCCL (no GPU and no NCCL needed).  The communicator's real
 * poll loop runs on a fake communicator whose behaviour the scenario sets:
 *   0  the awaited work finishes after a few polls        -> NS_OK
 *   1  it never finishes                                  -> NS_ERR_TIMEOUT
 *   2  NCCL reports an asynchronous (remote) error        -> NS_ERR_COMM
 *   3  a non-blocking creation that never completes       -> NS_ERR_TIMEOUT
 *   4  a non-blocking creation that completes             -> NS_OK
 * timeout_s is the deadline; *aborts (may be NULL) receives how many times the
 * loop aborted the communicator (1 in scenarios 1-3, 0 otherwise). */
NS_API ns_status ns_comm_selftest(int scenario, double timeout_s, int* aborts);

/* -------------------------------------------------- diffusion U-Net step
 * The denoising U-Net training step (no reference counterpart as a model:
 * the reference has its layers -- Conv2D, ResidualBlock
 * include/layers/residual.h:23-64, LayerNormLayer, MSELoss
 * include/losses.h:97-124 -- but no U-Net and no upsample).  NCHW, image
 * size S (a multiple of 4), base channels c:
 *   e0 = LN0(Res0(conv_in(x)))            c,  S
 *   e1 = LN1(Res1(down1(e0)))             2c, S/2  (3x3, stride 2, pad 1)
 *   m  = LN2(Res2(down2(e1)))             4c, S/4
 *   u1 = LN3(Res3(up1(Up(m)) + e1))       2c, S/2  (Up: nearest 2x)
 *   u0 = LN4(Res4(up0(Up(u1)) + e0))      c,  S
 *   y  = conv_out(u0); loss = MSELoss(y, target)
 * Res(a) = ReLU(Conv2D_3x3(a) + a); LN normalises the last axis (W), as the
 * reference's LayerNormLayer does on an NCHW tensor.  Parameters are a flat
 * buffer in registration order (conv_in, res0, ln0, down1, res1, ln1, down2,
 * res2, ln2, up1, res3, ln3, up0, res4, ln4, conv_out; each conv weight then
 * bias, each LN gamma then beta); AdamW decays rank >= 2 tensors (the conv
 * weights), as the reference's AdamW does.  With a communicator attached the
 * gradient and the loss are summed over ranks after the backward (the MSE
 * gradient is divided by the global element count). */
typedef struct ns_unet ns_unet;
typedef struct {
  int in_channels, base_channels, image_size, max_batch;
} ns_unet_config;
NS_API ns_status ns_unet_create(const ns_unet_config* cfg, ns_unet** out);
NS_API ns_status ns_unet_destroy(ns_unet* net);
NS_API int ns_unet_num_tensors(const ns_unet* net);
NS_API int64_t ns_unet_tensor_numel(const ns_unet* net, int i);
NS_API int64_t ns_unet_num_params(const ns_unet* net);
NS_API float* ns_unet_params(ns_unet* net);
NS_API float* ns_unet_grads(ns_unet* net);
NS_API float* ns_unet_output(ns_unet* net); /* device [B, in_channels, S, S] */
NS_API float* ns_unet_loss(ns_unet* net);   /* device, 1 float (summed over ranks) */
NS_API ns_status ns_unet_forward(ns_unet* net, const float* x, int B, void* stream);
NS_API ns_status ns_unet_loss_backward(ns_unet* net, const float* target, void* stream);
NS_API ns_status ns_unet_backward(ns_unet* net, void* stream);
NS_API ns_status ns_unet_adamw_init(ns_unet* net, float lr, float b1, float b2, float eps, float wd);
NS_API ns_status ns_unet_adamw_step(ns_unet* net, void* stream);
NS_API ns_status ns_unet_train_step(ns_unet* net, const float* x, const float* target, int B,
                                    float* host_loss, void* stream);
NS_API ns_status ns_unet_set_comm(ns_unet* net, ns_comm* comm, int world_size);

/* ------------------------------------------------------------ GPT model
 * The device GPTModel (include/gpt.h:136-327) + CrossEntropyLoss + AdamW, with
 * parameters, gradients, optimizer state and every activation resident in
 * HBM.  Parameters are one flat buffer in Module::Parameters() registration
 * order (include/module.h:44-52):
 *   wte, wpe, per block [ln_1 g b, c_attn W b, c_proj W b, ln_2 g b,
 *   mlp_fc W b, mlp_proj W b], ln_f g b
 * and gradients a second flat buffer with the same offsets. */
typedef struct ns_gpt ns_gpt;
typedef struct {
  int vocab_size, block_size, n_layer, n_head, n_embd; /* GPTConfig, gpt.h:33-39 */
  int max_batch;                                        /* sequences per step on this GPU */
} ns_gpt_config;

NS_API ns_status ns_gpt_create(const ns_gpt_config* cfg, ns_gpt** out);
NS_API ns_status ns_gpt_destroy(ns_gpt* model);
NS_API int ns_gpt_num_tensors(const ns_gpt* model);
NS_API int64_t ns_gpt_tensor_numel(const ns_gpt* model, int i);
NS_API int ns_gpt_tensor_rank(const ns_gpt* model, int i);
NS_API int64_t ns_gpt_tensor_offset(const ns_gpt* model, int i);
NS_API int64_t ns_gpt_num_params(const ns_gpt* model);
NS_API float* ns_gpt_params(ns_gpt* model); /* device, num_params floats */
NS_API float* ns_gpt_grads(ns_gpt* model);  /* device, num_params floats */
/* Device buffers of the last step: logits [B*T, V], dlogits, loss (1 float). */
NS_API float* ns_gpt_logits(ns_gpt* model);
NS_API float* ns_gpt_loss(ns_gpt* model);

/* GPTModel::Forward (gpt.h:192-232) on device int32 tokens [B,T]. */
NS_API ns_status ns_gpt_forward(ns_gpt* model, const int32_t* tokens, int B, int T, void* stream);
/* CrossEntropyLoss Forward/Backward on the last logits (losses.h:34-86);
 * dlogits are scaled by 1/(B*T*world_size). */
NS_API ns_status ns_gpt_loss_backward(ns_gpt* model, const int32_t* targets, void* stream);
/* GPTModel::Backward (gpt.h:234-272), gradients overwritten.  With a
 * communicator attached, gradient buckets are all-reduced over NCCL as their
 * blocks finish, overlapped with the rest of the backward. */
NS_API ns_status ns_gpt_backward(ns_gpt* model, void* stream);
/* AdamW (optimizers.h:148-162): configure, then Step (206-234). */
NS_API ns_status ns_gpt_adamw_init(ns_gpt* model, float lr, float b1, float b2, float eps, float wd);
NS_API ns_status ns_gpt_adamw_set_lr(ns_gpt* model, float lr);
NS_API ns_status ns_gpt_adamw_step(ns_gpt* model, void* stream);
/* ClipGradients(params, max_norm), train_llm.cpp:112-129, device-side. */
NS_API ns_status ns_gpt_clip_gradients(ns_gpt* model, float max_norm, void* stream);
/* One whole training step: forward, loss, backward (+ all-reduce), optional
 * clip (max_norm <= 0 disables), AdamW step.  host_loss may be NULL; if set,
 * the step synchronises the stream and returns the loss. */
NS_API ns_status ns_gpt_train_step(ns_gpt* model, const int32_t* tokens, const int32_t* targets, int B,
                            int T, float max_norm, float* host_loss, void* stream);
/* ------------------------------------------------------------ checkpoints
 * NSF weight files, byte for byte the format of the reference's
 * nsf::Save / nsf::Load (include/serialization.h:128-287): magic, version,
 * the architecture metadata of GPTModel::ArchitectureMetadata (gpt.h:309-316),
 * then every parameter with its NamedParameters() path ("wte.weight",
 * "blocks.0.attn.c_attn.weight", ...), shape and float32 data, and an FNV-1a
 * checksum.  Files written here load in the reference and the reference's
 * load here.  A load checks magic, version, every metadata value, tensor
 * count, names, shapes, byte counts and the checksum before anything is
 * copied to the model, so a rejected file (NS_ERR_INVALID_ARGUMENT, the
 * reason in ns_last_error) leaves the parameters unchanged.
 * GPTModel::SaveWeights / LoadWeights, include/gpt.h:293-306: */
NS_API ns_status ns_gpt_save_weights(ns_gpt* model, const char* path, void* stream);
NS_API ns_status ns_gpt_load_weights(ns_gpt* model, const char* path, void* stream);
/* The same file format for a flat host array of parameters in registration
 * order (no GPU needed): converting, inspecting or preparing checkpoints. */
NS_API ns_status ns_nsf_save_gpt(const ns_gpt_config* cfg, const float* host_params, const char* path);
NS_API ns_status ns_nsf_load_gpt(const ns_gpt_config* cfg, const char* path, float* host_params);
/* No reference counterpart (the reference saves weights only, so a run
 * cannot resume its optimizer): AdamW's first and second moments as tensors
 * "m.<name>" / "v.<name>" in an NSF file whose metadata add arch
 * "gpt-adamw", step, lr, beta1, beta2, eps and weight_decay.  Loading needs
 * ns_gpt_adamw_init first (with the file's weight decay); it restores the
 * moments, the step count and lr/betas/eps, so the next step continues the
 * saved run bit for bit. */
NS_API ns_status ns_gpt_save_optimizer(ns_gpt* model, const char* path, void* stream);
NS_API ns_status ns_gpt_load_optimizer(ns_gpt* model, const char* path, void* stream);

/* ------------------------------------------------------- KV-cache decoding
 * GPTModel::ForwardWithKVCache (include/gpt.h:159-190, with
 * MultiHeadAttention::ForwardWithKVCache, include/layers/attention.h:481-546)
 * for B sequences that advance together, one token each per step.  The
 * decoder owns a device KV cache of block_size positions for up to max_batch
 * sequences of `model` and reads the model's current parameters at every
 * step.  ns_gpt_decoder_clear is ClearKVCache (gpt.h:153-157).
 * ns_gpt_decode_step: tokens (device int32 [B]) at position `pos` (the wpe
 * row, as the reference's pos_idx; the token's K and V are appended to the
 * cache whatever pos is, as in the reference) -> logits [B, vocab] in
 * logits_out (device; NULL: the decoder's own buffer, ns_gpt_decoder_logits).
 * A token outside [0, vocab) sets *err_flag (device int; NULL: an internal
 * flag).  pos >= block_size or a full cache: NS_ERR_OUT_OF_RANGE.
 * ns_gpt_decoder_prefill: the prompt tokens [B, T] (device int32) through
 * the model's batched forward; the cache then holds what decoding the prompt
 * token by token at positions 0..T-1 leaves (ns_gpt_decoder_length = T), and
 * logits_out receives each sequence's last-position logits [B, vocab].  No
 * reference counterpart for the prefill (the reference decodes the prompt
 * one token at a time, generate_llm.cpp:146-149); B <= the model's
 * max_batch. */
typedef struct ns_gpt_decoder ns_gpt_decoder;
NS_API ns_status ns_gpt_decoder_create(ns_gpt* model, int max_batch, ns_gpt_decoder** out);
NS_API ns_status ns_gpt_decoder_destroy(ns_gpt_decoder* dec);
NS_API ns_status ns_gpt_decoder_clear(ns_gpt_decoder* dec);
NS_API int ns_gpt_decoder_length(const ns_gpt_decoder* dec);
NS_API float* ns_gpt_decoder_logits(ns_gpt_decoder* dec);
NS_API ns_status ns_gpt_decode_step(ns_gpt_decoder* dec, const int32_t* tokens, int B, int pos,
                                    float* logits_out, int32_t* err_flag, void* stream);
NS_API ns_status ns_gpt_decoder_prefill(ns_gpt_decoder* dec, const int32_t* tokens, int B, int T,
                                        float* logits_out, void* stream);

/* Data parallel: attach a communicator (NULL detaches).  bucket_floats caps a
 * gradient bucket (0 = one bucket per GPTBlock). */
NS_API ns_status ns_gpt_set_comm(ns_gpt* model, ns_comm* comm, int world_size, int64_t bucket_floats);
/* Data-parallel diagnostics (no reference counterpart).  With timing on, each
 * backward records three events: on the comm stream when the first bucket's
 * all-reduce may start and when the last (the loss sum) has finished, and on
 * the compute stream when its own backward work has been issued up to the
 * join.  ns_gpt_comm_times waits for the last backward's events and reports
 * exposed_ms, how long the compute stream waited for the all-reduces after
 * its backward (0 when they had finished), and span_ms, the time from the
 * first bucket's start to the last one's end.  Timing needs an attached
 * communicator with world_size > 1. */
NS_API ns_status ns_gpt_set_comm_timing(ns_gpt* model, int enable);
NS_API ns_status ns_gpt_comm_times(ns_gpt* model, float* exposed_ms, float* span_ms);
/* Gradient-bucket plan of the attached world (host-only; usable without a
 * GPU): writes up to max_buckets [begin, end) float ranges in launch order. */
NS_API int ns_gpt_plan_buckets(const ns_gpt_config* cfg, int64_t bucket_floats, int64_t* begin,
                        int64_t* end, int max_buckets);

#ifdef __cplusplus
}
#endif

#endif /* NS_B200_H_ */
