// Interface between the GEMM dispatcher and the tcgen05 kernel.
#pragma once

#include <cuda.h>

#include "common.cuh"
#include "epilogue.cuh"

namespace nsb {
namespace tc {

constexpr int kBM = 128;  // MMA M (one CTA, cta_group::1)
constexpr int kBK = 32;   // fp32 K per stage = one 128-byte swizzle row

struct Plan {
  int bn;          // 128 or 256
  int pair;        // 1: 256 x 256 tiles on a CTA pair (tiles_m counts 256-row tiles)
  int trans;       // 1: the kernel computes C^T (tiles_m over N, tiles_n over M)
  int stages;
  int tiles_m, tiles_n;
  int splits;      // K splits (>= 1), every split non-empty
  int kb_total;    // ceil(K / kBK)
  int kb_per;      // k-blocks per split
  int grid;        // persistent CTAs (CTA pairs for pair tiles)
  // CTA-pair plans with splits == 1 only: the last sk_tiles tiles run as a
  // stream-K tail, their k-blocks shared evenly by all `grid` pairs (0: none).
  int sk_tiles;
};

// allow_wide: 128 x 256 tiles may be chosen (they need pre-split operands).
// force_kind >= 0 restricts the choice to one kernel: 0 = 128 x 128,
// 1 = 128 x 256, 2 = CTA-pair tiles of any width, 3 / 4 = pair tiles
// 256 x 192 / 256 x 128 only, 5 = pair tiles 256 x 256 only (tests and profiling).
// trans_mode for the wide kernels: 1 = compute C^T (coalesced column stores),
// 0 = compute C (row stores).
// allow_split also allows the stream-K tail unless allow_stream_k is false.
Plan plan(int M, int N, int K, bool allow_split, bool allow_wide, int force_kind = -1,
          int trans_mode = 1, bool allow_stream_k = true);
size_t split_workspace_bytes(const Plan& p, int M, int N);

size_t lo_elems_a(int M, int K);
// Bytes for the compact lo copies of both operands (the pre-split path).
size_t lo_workspace_bytes(int M, int N, int K);

// Runs C = op(A) op(B) (+ epilogue) on the tcgen05 path.  `ws` holds the
// split-K partial tiles when plan.splits > 1.  With `lo_ws` (at least
// lo_workspace_bytes) the operands are split into hi/lo in global memory
// first and the kernel loads both parts by TMA; without it the kernel splits
// each tile in shared memory.
// a_lo_in / b_lo_in: the caller's compact lo copies (optional); the missing
// ones are split into lo_ws.
ns_status run(const Plan& pl, int M, int N, int K, const float* A, int lda, int a_mn,
              const float* B, int ldb, int b_mn, const EpiArgs& e, float* ws, float* lo_ws,
              const float* a_lo_in, const float* b_lo_in, cudaStream_t stream);

// lo = x - trunc_tf32(x) of a [rows, cols] matrix with row stride ld, compact.
ns_status split_operand(const float* x, int rows, int cols, int ld, float* lo, cudaStream_t s);

// 1 if a kernel hit a bounded-wait timeout since the last call (clears it);
// -(CUDA error) if the flag could not be read.
int consume_timeout_flag();

// The tensor core adds into its fp32 accumulator with round-toward-zero, so
// each TMEM chunk (kblocks x 32 terms) carries a bias toward zero of up to
// ~1 ulp of the chunk sum per MMA; chunks are folded with round-to-nearest.
// For reductions whose partial sums share a sign over many terms (a weight
// gradient summed over a long sequence) 1-k-block chunks halve that bias at
// about a quarter of the throughput.  Per host thread; returns the previous
// setting (2 = default).
int set_accumulation_chunk(int kblocks);

// CTA-pair kernel schedule, fixed (cluster c takes items c, c + clusters,
// ...) or dynamic (cluster c starts on item c, then takes its next item from
// a per-launch counter when it is ready for one).  Results are bit-identical.
// The dynamic order pays when another stream's kernel holds SMs while a GEMM
// starts (the all-reduce beside a data-parallel backward); alone on the GPU
// the fixed order measured the same or slightly faster.  So GEMM calls use
// the fixed order, and a backward whose gradient buckets are all-reduced
// beside it picks the dynamic one for its own GEMMs (PairScheduleScope).
// set_pair_schedule forces one for subsequent launches on this host thread
// (1 dynamic, 0 fixed, -1 none: the rule above) and returns the previous
// setting.
int set_pair_schedule(int mode);

// For the lifetime of the object, the GEMMs this host thread launches use the
// dynamic order if `dynamic` (unless set_pair_schedule forces one).
class PairScheduleScope {
 public:
  explicit PairScheduleScope(bool dynamic);
  ~PairScheduleScope();
  PairScheduleScope(const PairScheduleScope&) = delete;
  PairScheduleScope& operator=(const PairScheduleScope&) = delete;

 private:
  int saved_;
};

// Launches the bounded-wait self-test kernel (a wait that runs out after
// limit_us microseconds and raises the flag consume_timeout_flag reads).
ns_status wait_probe(int limit_us, cudaStream_t s);

}  // namespace tc
}  // namespace nsb
