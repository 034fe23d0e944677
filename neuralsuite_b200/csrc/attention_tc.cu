// K2 on the 5th-generation tensor cores: fused causal attention forward for
// head_dim 32 and 64, 3xTF32 (the attention.cu SIMT kernels serve every other
// head size).  Same contract as the SIMT forward: out[B*T, C] and lse[B*H*T]
// from the interleaved qkv[B*T, 3C] (MultiHeadAttention::Forward,
// include/layers/attention.h:364-384).
//
// Persistent: one CTA per SM (384 threads, warp-specialised) loops over work
// items (b, h, 128-query block):
//   warp 0      TMA producer: per 64-key block the K and V tiles of this head
//               and their tf32 lo parts (the caller's, or split beforehand into
//               the workspace) into a shared-memory ring.  K lands K-major
//               (16-byte chunk 128B swizzle), V MN-major (32-byte chunk 128B
//               swizzle).
//   warp 1      MMA issuer (converged warp, elected lane), A operands from TMEM:
//                 S_j  = Qhi.Khi + Qhi.Klo + Qlo.Khi      (M=128, N=64,  K=D)
//                 O_j  = Phi.Vhi + Phi.Vlo + Plo.Vhi      (M=128, N=D,   K=64)
//   warp 2      TMA producer of the next item's Q rows (into shared memory).
//   warps 4-11  two softmax warpgroups, both on every key block (column halves,
//               described above the forward kernel); one query row per thread
//               pair (TMEM lane = row).  Per block: read S_j, apply the causal
//               mask, exchange the row maxima, P = 2^(S*scale*log2e -
//               m*scale*log2e), write Phi (over S_j) and Plo to TMEM, and fold
//               the previous O into registers as acc = acc * alpha + O with
//               round-to-nearest (each O_j is a 64-term tensor-core sum; its
//               round-toward-zero accumulation stays at the 1e-7 level).
// TMEM (512 columns): Qhi [0,D), Qlo [D,2D); S/Phi at 128 + 64b, Plo at
// 256 + 64b, O at 384 + 64b, b = parity of the key block counted over all of
// the CTA's items (double buffers: S_{j+1} is computed while S_j turns into P_j).
// Every mbarrier wait is bounded (2 s); a timeout raises a device flag that
// ns_kernel_health() reports, and the CTA drains its copies and MMAs and exits.
#include <algorithm>

#include "attention_tc.cuh"
#include "tc_common.cuh"

namespace nsb {
namespace attn_tc {

__device__ int g_timeout;

namespace {

using namespace tcx;

constexpr int kBQ = 128;  // queries per CTA (MMA M)
constexpr int kBKV = 64;  // keys per block
constexpr int kThreads = 384;
constexpr int kWgThreads = 128;  // one softmax warpgroup

constexpr uint32_t kTS = 128, kTPlo = 256, kTO = 384, kTmemCols = 512;

template <int D>
struct FwdLayout {
  static constexpr int kStages = D == 64 ? 3 : 4;
  static constexpr uint32_t kTile = kBKV * D * 4;  // 64 keys x D fp32 (D/32 boxes of 8 KB)
  static constexpr uint32_t kStage = 4 * kTile;    // K raw | K lo | V raw | V lo
  // The next work item's Q rows (128 x D, D/32 boxes of 16 KB, 128B swizzle).
  static constexpr uint32_t kQ = kStages * kStage;
  static constexpr uint32_t kBars = kQ + kBQ * D * 4;
  static constexpr uint32_t kNumBars = 2 * kStages + 26;
  static constexpr uint32_t kBytes = kBars + kNumBars * 8 + 16;
  static constexpr uint32_t kDynSmem = kBytes + 1024;
  static_assert(kDynSmem <= 232448, "shared memory budget");
  static_assert(kDynSmem > 232448 / 2, "one CTA per SM (the CTA takes all 512 TMEM columns)");
};

struct FwdParams {
  const float* qkv;
  float* out;
  float* lse;
  int T, H, C;
  float scale;       // 1/sqrt(D)
  float scale_log2;  // scale * log2(e)
  int n_items;       // (128-query block, batch x head) pairs
  int nqb;           // query blocks per sequence
  int klo0, vlo0;    // columns of K's and V's lo parts in the lo tensor (head 0)
  float* out_lo;     // optional: tf32 lo part of out
};

// K tile (keys x D, K-major): 8-row groups 1024 B apart, 16-byte chunks;
// k-step kk (8 of D) is +32 B inside the 128-byte row, next 32 columns in the
// next 8 KB box.
__device__ __forceinline__ uint64_t k_desc(uint32_t base, int kk) {
  return smem_desc(base + (kk >> 2) * 8192 + (kk & 3) * 32, 16, 1024, 2u);
}
// V tile (keys x D, MN-major for O = P.V): boxes of 32 columns x 64 keys,
// 8 KB apart (LBO); 4-row groups 512 B apart; k-step kk (8 keys) is +1024 B.
__device__ __forceinline__ uint64_t v_desc(uint32_t base, int kk) {
  return smem_desc(base + kk * 1024, 8192, 512, 1u);
}

// Register split: the CTA launches with 384 x kLaunchRegs; warps 0-3 (TMA,
// MMA) give theirs down to kLowRegs (enough for their work-item and ring
// bookkeeping) so that the eight softmax / element-wise warps can hold a full
// S row and output row each.  4*32*kLowRegs + 8*32*kHighRegs must not exceed
// 384 * (registers per thread at launch): with 168 at launch it is exact, and
// the host checks it before launching.
constexpr int kLowRegs = 88, kHighRegs = 208;
constexpr int kMinLaunchRegs = (4 * 32 * kLowRegs + 8 * 32 * kHighRegs + kThreads - 1) / kThreads;

__device__ __forceinline__ void reg_dec() {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kLowRegs));
}

// Work item k of CTA c in a grid of G: the items (query block, batch x head)
// are ordered longest first (the last query block has the most keys) and
// dealt in a snake (c, then G-1-c, ...), which balances the CTAs' total
// lengths.  -1 when the CTA has no item k.
__device__ __forceinline__ int work_item(int c, int k, int G, int n_items) {
  const int w = k * G + ((k & 1) ? (G - 1 - c) : c);
  return w < n_items ? w : -1;
}

// Persistent: one CTA per SM loops over work items.  Per item the element-wise
// warps copy the item's Q rows (brought into shared memory by TMA while the
// previous item ran) into TMEM as soon as the previous item's last S MMA is
// done, and only then finish the previous item (last O fold, output), so the
// tensor core starts the next item's S blocks while the previous item's
// epilogue runs.
//
// Both softmax warpgroups work on every 64-key block, warpgroup w on keys
// [32w, 32w+32) of it and on output columns [D/2 w, D/2 w + D/2) (D=32: the
// output by warpgroup 0 alone): per block the two halves of a row exchange
// their maxima through a TMEM column of the block's O buffer (free until the
// block's O MMA) under an mbarrier of the two warps sharing the row's TMEM
// lanes; the row sums stay per half and meet at the end.  S/P, Plo and O are
// double-buffered in TMEM by block parity, so the tensor core computes
// S_{j+1} while both warpgroups turn S_j into P_j.
template <int D>
__global__ void __launch_bounds__(kThreads, 1)
    attn_fwd_tc_kernel(const __grid_constant__ CUtensorMap tmQ,
                       const __grid_constant__ CUtensorMap tmK,
                       const __grid_constant__ CUtensorMap tmKlo,
                       const __grid_constant__ CUtensorMap tmV,
                       const __grid_constant__ CUtensorMap tmVlo, const FwdParams p) {
  using L = FwdLayout<D>;
  constexpr int S = L::kStages;
  constexpr int kHalfD = 32;  // output columns one warpgroup folds (D=32: warpgroup 0 all)
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  const uint32_t sbase = smem_u32(smem);
  const uint32_t bar0 = sbase + L::kBars;
  auto kv_full = [&](int s) { return bar0 + 8u * s; };
  auto kv_empty = [&](int s) { return bar0 + 8u * (S + s); };
  const uint32_t q_full = bar0 + 8u * (2 * S), q_empty = q_full + 8u;
  const uint32_t q_ready = q_full + 16u, q_free = q_full + 24u;
  auto s_full = [&](int b) { return bar0 + 8u * (2 * S + 4 + b); };
  auto p_full = [&](int b) { return bar0 + 8u * (2 * S + 6 + b); };
  auto o_full = [&](int b) { return bar0 + 8u * (2 * S + 8 + b); };
  auto o_empty = [&](int b) { return bar0 + 8u * (2 * S + 10 + b); };
  const uint32_t drain = bar0 + 8u * (2 * S + 12);
  // row-quadrant e (warps 4+e and 8+e): block-max exchange per buffer, row-sum exchange
  auto mx_bar = [&](int e, int b) { return bar0 + 8u * (2 * S + 13 + 2 * e + b); };
  auto lx_bar = [&](int e) { return bar0 + 8u * (2 * S + 21 + e); };
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::kBars + L::kNumBars * 8);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int G = (int)gridDim.x, cta = (int)blockIdx.x;
  const int BH = p.n_items / p.nqb;
  // Item w: query block nqb-1-w/BH (longest first), batch x head w%BH.
  auto item_q0 = [&](int w) { return (p.nqb - 1 - w / BH) * kBQ; };
  auto item_bh = [&](int w) { return w % BH; };
  auto item_nkb = [&](int w) { return (min(item_q0(w) + kBQ, p.T) + kBKV - 1) / kBKV; };
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(kv_full(s), 1);
      mbar_init(kv_empty(s), 1);
    }
    mbar_init(q_full, 1);
    mbar_init(q_empty, 2 * kWgThreads);
    mbar_init(q_ready, 2 * kWgThreads);
    mbar_init(q_free, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(s_full(i), 1);
      mbar_init(p_full(i), 2 * kWgThreads);
      mbar_init(o_full(i), 1);
      mbar_init(o_empty(i), 2 * kWgThreads);
    }
    mbar_init(drain, 1);
    for (int e = 0; e < 4; ++e) {
      mbar_init(mx_bar(e, 0), 64);
      mbar_init(mx_bar(e, 1), 64);
      mbar_init(lx_bar(e), 64);
    }
    *abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  fence_before();
  __syncthreads();
  fence_after();
  // Launched as a programmatic dependent (launch_pdl): the set-up above ran
  // while the previous kernel finished; its outputs are read only from here.
  pdl_wait();
  pdl_trigger();
  const uint32_t tmem = *tmem_slot;

  if (warp < 4) {
    // setmaxnreg runs at one instruction for a whole warpgroup.
    reg_dec();
    if (warp == 0) {
      // ------------------------------------------------------------ K / V producer
      if (lane == 0) {
        int issued[S];
        uint32_t issued_ph[S];
        for (int s = 0; s < S; ++s) issued[s] = 0, issued_ph[s] = 0;
        bool ok = true;
        uint32_t g = 0;  // key blocks loaded so far (all items)
        for (int k = 0; ok; ++k) {
          const int w = work_item(cta, k, G, p.n_items);
          if (w < 0) break;
          const int bh = item_bh(w), b = bh / p.H, h = bh % p.H;
          const int n_kb = item_nkb(w);
          for (int j = 0; j < n_kb; ++j, ++g) {
            const int s = g % S;
            const uint32_t ph = (g / S) & 1u;
            if (!mbar_wait(kv_empty(s), ph ^ 1u, abort, &g_timeout)) {
              ok = false;
              break;
            }
            mbar_expect_tx(kv_full(s), L::kStage);
            issued[s] = 1;
            issued_ph[s] = ph;
            const uint32_t dst = sbase + s * L::kStage;
            const int row = b * p.T + j * kBKV;
#pragma unroll
            for (int c = 0; c < D / 32; ++c) {
              const int x = h * D + 32 * c;
              tma_load_2d(dst + c * 8192, &tmK, kv_full(s), p.C + x, row);
              tma_load_2d(dst + L::kTile + c * 8192, &tmKlo, kv_full(s), p.klo0 + x, row);
              tma_load_2d(dst + 2 * L::kTile + c * 8192, &tmV, kv_full(s), 2 * p.C + x, row);
              tma_load_2d(dst + 3 * L::kTile + c * 8192, &tmVlo, kv_full(s), p.vlo0 + x, row);
            }
          }
        }
        if (!ok)
          for (int s = 0; s < S; ++s)
            if (issued[s]) mbar_wait_drain(kv_full(s), issued_ph[s], &g_timeout);
      }
    } else if (warp == 2) {
      // ------------------------------------------------------------ Q producer
      if (lane == 0) {
        bool ok = true, pending = false;
        uint32_t pend_ph = 0;
        for (int k = 0;; ++k) {
          const int w = work_item(cta, k, G, p.n_items);
          if (w < 0) break;
          // The element-wise warps have copied the previous item's Q out.
          if (!mbar_wait(q_empty, ((uint32_t)k & 1u) ^ 1u, abort, &g_timeout)) {
            ok = false;
            break;
          }
          const int bh = item_bh(w), b = bh / p.H, h = bh % p.H;
          mbar_expect_tx(q_full, (uint32_t)(kBQ * D * 4));
          pending = true;
          pend_ph = (uint32_t)k & 1u;
#pragma unroll
          for (int c = 0; c < D / 32; ++c)
            tma_load_2d(sbase + L::kQ + c * 16384, &tmQ, q_full, h * D + 32 * c, b * p.T + item_q0(w));
        }
        if (!ok && pending) mbar_wait_drain(q_full, pend_ph, &g_timeout);
      }
    } else if (warp == 1) {
      // ------------------------------------------------------------ MMA issuer
      // The whole warp runs this loop converged; the elected lane issues.
      // Block G (counted over all items) uses S/P, Plo and O buffer G & 1.
      constexpr uint32_t id_s = instr_desc(kBKV, 0, 0);
      constexpr uint32_t id_o = instr_desc(D, 0, 1);
      uint32_t g = 0;  // key blocks of earlier items (ring position and block count)
      bool ok = true;
      auto emit_s = [&](uint32_t G) {
        const int s = G % S;
        const uint32_t d = tmem + kTS + (G & 1u) * kBKV;
        const uint32_t k_raw = sbase + s * L::kStage, k_lo = k_raw + L::kTile;
#pragma unroll
        for (int kk = 0; kk < D / 8; ++kk)
          mma_ts(d, tmem + kk * 8, k_desc(k_raw, kk), id_s, kk > 0 ? 1u : 0u);
#pragma unroll
        for (int kk = 0; kk < D / 8; ++kk) {
          mma_ts(d, tmem + kk * 8, k_desc(k_lo, kk), id_s, 1u);
          mma_ts(d, tmem + D + kk * 8, k_desc(k_raw, kk), id_s, 1u);
        }
        commit(s_full(G & 1u));
      };
      auto issue_s = [&](uint32_t G) -> bool {
        if (!warp_wait(kv_full(G % S), (G / S) & 1u, abort, &g_timeout)) return false;
        fence_after();
        if (elect_one()) emit_s(G);
        __syncwarp();
        return true;
      };
      // After the item's last S: Q's TMEM columns may take the next item's rows.
      auto release_q = [&]() {
        if (elect_one()) commit(q_free);
        __syncwarp();
      };
      for (int k = 0; ok; ++k) {
        const int w = work_item(cta, k, G, p.n_items);
        if (w < 0) break;
        const int n_kb = item_nkb(w);
        if (!warp_wait(q_ready, (uint32_t)k & 1u, abort, &g_timeout)) {
          ok = false;
          break;
        }
        fence_after();
        ok = issue_s(g);
        if (ok && n_kb > 1) ok = issue_s(g + 1);
        if (ok && n_kb <= 2) release_q();
        for (int j = 0; ok && j < n_kb; ++j) {
          const uint32_t Gj = g + (uint32_t)j;
          const uint32_t b = Gj & 1u, ph = (Gj >> 1) & 1u;
          // The K tile of S_{j+2} is nearly always there: tested while waiting
          // for P_j, so that O_j and S_{j+2} go out in one elected run (each
          // wait or re-convergence between MMAs idles the tensor core).
          const bool next_s = j + 2 < n_kb;
          bool k_ready = next_s && mbar_test(kv_full((Gj + 2) % S), ((Gj + 2) / S) & 1u);
          const bool pe = mbar_wait(p_full(b), ph, abort, &g_timeout) &&
                          mbar_wait(o_empty(b), ph ^ 1u, abort, &g_timeout);
          const uint32_t bits = __shfl_sync(0xffffffffu, (pe ? 1u : 0u) | (k_ready ? 2u : 0u), 0);
          if (!(bits & 1u)) {
            ok = false;
            break;
          }
          k_ready = (bits & 2u) != 0;
          fence_after();
          const int s = Gj % S;
          if (elect_one()) {
            const uint32_t v_raw = sbase + s * L::kStage + 2 * L::kTile, v_lo = v_raw + L::kTile;
            const uint32_t o = tmem + kTO + b * 64u;
            const uint32_t phi = tmem + kTS + b * kBKV, plo = tmem + kTPlo + b * kBKV;
#pragma unroll
            for (int kk = 0; kk < kBKV / 8; ++kk)
              mma_ts(o, phi + kk * 8, v_desc(v_raw, kk), id_o, kk > 0 ? 1u : 0u);
#pragma unroll
            for (int kk = 0; kk < kBKV / 8; ++kk) {
              mma_ts(o, phi + kk * 8, v_desc(v_lo, kk), id_o, 1u);
              mma_ts(o, plo + kk * 8, v_desc(v_raw, kk), id_o, 1u);
            }
            commit(o_full(b));
            commit(kv_empty(s));
            if (k_ready) emit_s(Gj + 2);
          }
          __syncwarp();
          // S_{j+2} reuses block j's S/P columns: issued after O_j, and the
          // tensor core runs one CTA's MMAs in issue order.
          if (next_s) {
            if (!k_ready) ok = issue_s(Gj + 2);
            if (ok && j + 2 == n_kb - 1) release_q();
          }
        }
        g += (uint32_t)n_kb;
      }
      if (!ok) {
        // Wait for every MMA already issued before TMEM is freed.
        if (elect_one()) commit(drain);
        __syncwarp();
        mbar_wait_drain(drain, 0, &g_timeout);
      }
    }
  } else {
    // ------------------------------------------------------------ softmax
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kHighRegs));
    const int wg = (warp - 4) >> 2;  // keys [32wg, 32wg+32) of every block
    const int ew = warp & 3;         // TMEM lanes 32*ew .. 32*ew+31
    const int row = ew * 32 + lane;
    const uint32_t lane_off = (uint32_t)(ew * 32) << 16;
    const float c = p.scale_log2;
    const bool folds = D == 64 || wg == 0;  // output columns [kHalfD*wg, kHalfD*wg + kHalfD)
    float acc[kHalfD];
    float m = -INFINITY, mc = 0.0f, l = 0.0f, alpha_prev = 0.0f;
    uint32_t T = 0;  // blocks so far (all items)
    int t = 0;       // ... of the current item
    int prev_w = -1, prev_k = -1;
    bool ok = true;
    // acc = acc * alpha + O of block Gb (buffer Gb & 1), then the O buffer is free.
    auto fold = [&](uint32_t Gb, float alpha) -> bool {
      if (!mbar_wait(o_full(Gb & 1u), (Gb >> 1) & 1u, abort, &g_timeout)) return false;
      fence_after();
      if (folds) {
        uint32_t v[32];
        tmem_ld32(tmem + lane_off + kTO + (Gb & 1u) * 64u + kHalfD * wg, v);
#pragma unroll
        for (int i = 0; i < kHalfD; ++i) acc[i] = fmaf(acc[i], alpha, __uint_as_float(v[i]));
      }
      fence_before();
      mbar_arrive(o_empty(Gb & 1u));
      return true;
    };
    // Last fold and output of item w (whose blocks are all turned into P).
    // The row sums of the two halves meet through a column of the last
    // block's O buffer, free after the fold.
    auto finish = [&](int w, uint32_t k_item) -> bool {
      if (!fold(T - 1, alpha_prev)) return false;
      const uint32_t xcol = tmem + lane_off + kTO + ((T - 1) & 1u) * 64u;
      tmem_st1(xcol + 32 * wg, l);
      tmem_wait_st();
      fence_before();
      mbar_arrive(lx_bar(ew));
      if (!mbar_wait(lx_bar(ew), k_item & 1u, abort, &g_timeout)) return false;
      fence_after();
      const float l_tot = l + tmem_ld1(xcol + 32 * (wg ^ 1));
      const float inv = 1.0f / l_tot;
      const int bh = item_bh(w), b = bh / p.H, h = bh % p.H;
      const int q = item_q0(w) + row;
      if (q < p.T && folds) {
        const size_t o = ((size_t)b * p.T + q) * p.C + (size_t)h * D + kHalfD * wg;
        float* dst = p.out + o;
#pragma unroll
        for (int d = 0; d < kHalfD; d += 4)
          *reinterpret_cast<float4*>(dst + d) =
              make_float4(acc[d] * inv, acc[d + 1] * inv, acc[d + 2] * inv, acc[d + 3] * inv);
        if (p.out_lo) {
          float* dlo = p.out_lo + o;
#pragma unroll
          for (int d = 0; d < kHalfD; d += 4)
            *reinterpret_cast<float4*>(dlo + d) =
                make_float4(tf32_lo(acc[d] * inv), tf32_lo(acc[d + 1] * inv),
                            tf32_lo(acc[d + 2] * inv), tf32_lo(acc[d + 3] * inv));
        }
        if (wg == 0) p.lse[(size_t)bh * p.T + q] = m * p.scale + logf(l_tot);
      }
      return true;
    };
    for (int k = 0; ok; ++k) {
      const int w = work_item(cta, k, G, p.n_items);
      if (w < 0) break;
      const int q0 = item_q0(w), q = q0 + row;
      const int n_kb = item_nkb(w);
      {
        // This item's Q rows: shared memory (128B swizzle: 16-byte chunk i of
        // row r sits at chunk i ^ (r & 7)) -> Qhi / Qlo columns, once the
        // previous item's last S MMA has read the old ones.
        if (!mbar_wait(q_full, (uint32_t)k & 1u, abort, &g_timeout) ||
            (k > 0 && !mbar_wait(q_free, (uint32_t)(k - 1) & 1u, abort, &g_timeout))) {
          ok = false;
          break;
        }
        fence_after();
        for (int cc = wg; cc < D / 32; cc += 2) {
          const uint8_t* qs = smem + L::kQ + cc * 16384 + row * 128;
          // hi, then lo (the previous item's accumulator is still live here)
#pragma unroll
          for (int part = 0; part < 2; ++part) {
            uint32_t v[32];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const float4 x = q < p.T ? *reinterpret_cast<const float4*>(qs + ((i ^ (row & 7)) << 4))
                                       : make_float4(0.f, 0.f, 0.f, 0.f);
              const float xs[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
              for (int e = 0; e < 4; ++e)
                v[4 * i + e] = __float_as_uint(part ? tf32_lo(xs[e]) : tf32_hi(xs[e]));
            }
            tmem_st32(tmem + lane_off + part * D + 32 * cc, v);
          }
        }
        mbar_arrive(q_empty);
        tmem_wait_st();
        fence_before();
        mbar_arrive(q_ready);
      }
      if (prev_w >= 0 && !finish(prev_w, (uint32_t)prev_k)) {
        ok = false;
        break;
      }
#pragma unroll
      for (int d = 0; d < kHalfD; ++d) acc[d] = 0.0f;
      m = -INFINITY;
      mc = 0.0f;
      l = 0.0f;
      alpha_prev = 0.0f;
      t = 0;
      for (int j = 0; j < n_kb; ++j, ++t, ++T) {
        const uint32_t b = T & 1u, ph = (T >> 1) & 1u;
        if (!mbar_wait(s_full(b), ph, abort, &g_timeout)) {
          ok = false;
          break;
        }
        fence_after();
        const uint32_t s_t = tmem + lane_off + kTS + b * kBKV + 32 * wg;
        const uint32_t pl_t = tmem + lane_off + kTPlo + b * kBKV + 32 * wg;
        const int k0 = j * kBKV + 32 * wg;  // key of this half's column 0
        uint32_t sv[32];
        tmem_ld32(s_t, sv);
        float x[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) x[i] = __uint_as_float(sv[i]);
        if (k0 + 31 > q) {
#pragma unroll
          for (int i = 0; i < 32; ++i)
            if (k0 + i > q) x[i] = -INFINITY;
        }
        float mx[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) mx[i] = x[i];
#pragma unroll
        for (int i = 8; i < 32; ++i) mx[i & 7] = fmaxf(mx[i & 7], x[i]);
        const float mh = fmaxf(fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])),
                               fmaxf(fmaxf(mx[4], mx[5]), fmaxf(mx[6], mx[7])));
        // The other half's maximum, through this block's O buffer (no MMA
        // writes it before P_j is complete).
        const uint32_t xcol = tmem + lane_off + kTO + b * 64u;
        tmem_st1(xcol + 32 * wg, mh);
        tmem_wait_st();
        fence_before();
        mbar_arrive(mx_bar(ew, b));
        if (!mbar_wait(mx_bar(ew, b), ph, abort, &g_timeout)) {
          ok = false;
          break;
        }
        fence_after();
        const float m_blk = fmaxf(mh, tmem_ld1(xcol + 32 * (wg ^ 1)));
        const float m_new = fmaxf(m, m_blk);
        // m_new = -inf: every key so far is masked (P = 0 below).
        const float mc_new = m_new == -INFINITY ? 0.0f : m_new * c;
        const float alpha = m == -INFINITY ? 0.0f : fast_exp2(mc - mc_new);
        float rs[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) rs[i] = 0.0f;
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          x[i] = fast_exp2(fmaf(x[i], c, -mc_new));
          rs[i & 7] += x[i];
        }
        l = l * alpha + (((rs[0] + rs[1]) + (rs[2] + rs[3])) + ((rs[4] + rs[5]) + (rs[6] + rs[7])));
        m = m_new;
        mc = mc_new;
#pragma unroll
        for (int i = 0; i < 32; ++i) sv[i] = __float_as_uint(tf32_hi(x[i]));
        tmem_st32(s_t, sv);
#pragma unroll
        for (int i = 0; i < 32; ++i) sv[i] = __float_as_uint(tf32_lo(x[i]));
        tmem_st32(pl_t, sv);
        tmem_wait_st();
        fence_before();
        mbar_arrive(p_full(b));
        // Now the previous block's O (its MMA ran while this block's softmax did).
        if (t > 0 && !fold(T - 1, alpha_prev)) {
          ok = false;
          break;
        }
        alpha_prev = alpha;
      }
      if (!ok) break;
      prev_w = w;
      prev_k = k;
    }
    if (ok && prev_w >= 0) ok = finish(prev_w, (uint32_t)prev_k);
  }

  fence_before();
  __syncthreads();
  if (warp == 1) {
    fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(kTmemCols)
                 : "memory");
  }
}

// lo[r, c] = tf32 lo part of qkv[r, C + c] for c in [0, 2C): the K and V
// columns, compact (row stride 2C).  2C is a multiple of 4.
__global__ void split_kv_lo_k(const float* __restrict__ qkv, int64_t rows, int C,
                              float* __restrict__ lo) {
  pdl_wait();     // the previous kernel's writes are visible (launched by launch_pdl)
  pdl_trigger();  // the next kernel, if launched as a programmatic dependent, may start
  const int c4 = (2 * C) >> 2;
  const int64_t total = rows * c4;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += stride) {
    const int64_t r = i / c4, c = (i % c4) * 4;
    const float4 v = *reinterpret_cast<const float4*>(qkv + r * 3 * C + C + c);
    *reinterpret_cast<float4*>(lo + r * 2 * C + c) =
        make_float4(tf32_lo(v.x), tf32_lo(v.y), tf32_lo(v.z), tf32_lo(v.w));
  }
}

// qkv_lo: the caller's tf32 lo part of all of qkv ([B*T, 3C]), or null: then
// K's and V's are split into `lo` ([B*T, 2C]) first.
template <int D>
ns_status launch_fwd(const float* qkv, const float* qkv_lo, int B, int T, int H, float* out,
                     float* out_lo, float* lse, float* lo, cudaStream_t s) {
  using L = FwdLayout<D>;
  const int C = H * D, rows = B * T;
  if (!qkv_lo) {
    const int64_t work = (int64_t)rows * (2 * C / 4);
    const int grid = (int)std::max<int64_t>(1, std::min<int64_t>(ceil_div64(work, 256), (int64_t)sm_count() * 8));
    ns_status rc = launch_pdl(split_kv_lo_k, dim3(grid), dim3(256), 0, s, "ns_attn_fwd kv split",
                              qkv, rows, C, lo);
    if (rc != NS_OK) return rc;
  }
  const float* lo_t = qkv_lo ? qkv_lo : lo;
  const int lo_w = qkv_lo ? 3 * C : 2 * C;
  CUtensorMap tq, tk, tklo, tv, tvlo;
  ns_status rc = make_map(&tq, qkv, 3 * C, rows, 3 * C, kBQ, false);
  if (rc == NS_OK) rc = make_map(&tk, qkv, 3 * C, rows, 3 * C, kBKV, false);
  if (rc == NS_OK) rc = make_map(&tklo, lo_t, lo_w, rows, lo_w, kBKV, false);
  if (rc == NS_OK) rc = make_map(&tv, qkv, 3 * C, rows, 3 * C, kBKV, true);
  if (rc == NS_OK) rc = make_map(&tvlo, lo_t, lo_w, rows, lo_w, kBKV, true);
  if (rc != NS_OK) return rc;
  const float scale = 1.0f / sqrtf((float)D);
  const int nqb = (T + kBQ - 1) / kBQ;
  const int n_items = nqb * B * H;
  FwdParams p{qkv, out, lse, T, H, C, scale, scale * 1.4426950408889634f, n_items, nqb,
              qkv_lo ? C : 0, qkv_lo ? 2 * C : C, out_lo};
  NS_TRY_CUDA(cudaFuncSetAttribute(attn_fwd_tc_kernel<D>,
                                   cudaFuncAttributeMaxDynamicSharedMemorySize, (int)L::kDynSmem),
              "ns_attn_fwd attr");
  {
    // setmaxnreg.inc would wait forever if the launch held fewer registers
    // than the split hands out.
    cudaFuncAttributes fa;
    NS_TRY_CUDA(cudaFuncGetAttributes(&fa, attn_fwd_tc_kernel<D>), "ns_attn_fwd attributes");
    if (fa.numRegs < kMinLaunchRegs)
      return fail(NS_ERR_UNSUPPORTED, "ns_attn_fwd: kernel compiled with too few registers for its split");
  }
  const int grid = std::min(n_items, sm_count());
  return launch_pdl(attn_fwd_tc_kernel<D>, dim3(grid), dim3(kThreads), L::kDynSmem, s,
                    "ns_attn_fwd tcgen05", tq, tk, tklo, tv, tvlo, p);
}

// ------------------------------------------------------------------ backward
//
// Three tensor-core kernels, one per gradient, on one skeleton: a 128-row
// "major" block whose A operands sit in TMEM (hi/lo), and a loop over 64-wide
// "minor" blocks whose B tiles (raw and lo) arrive by TMA:
//   kDV  rows = keys,    minor = queries:  S^T = K.Q^T -> P^T;           dV += P^T.dO
//   kDK  rows = keys,    minor = queries:  S^T, dP^T = V.dO^T -> dS^T;   dK += dS^T.Q
//   kDQ  rows = queries, minor = keys:     S = Q.K^T, dP = dO.V^T -> dS; dQ += dS.K
// with P = exp(scale*S - lse) and dS = P * (dP - Delta), Delta_i = dO_i . O_i
// (MultiHeadAttention::Backward, include/layers/attention.h:405-461).  A
// tensor that one kernel reads both K-major (for S or dP) and MN-major (for
// the gradient product) is loaded twice, once per swizzle, because the
// tensor core reads MN-major tf32 operands only from the 32-byte-atom swizzle
// and K-major ones only from the 16-byte-chunk one.
//
// Each B operand has its own TMA ring and producer warp (warp 0: the S
// operand, warp 2: the dP operand, warp 3: the product operand plus the
// block's lse / Delta vectors), because the three are consumed about one block
// apart.  With every A operand held as hi + lo, TMEM has room for one S, one
// dP, one product lo part and one product accumulator, so the order of work
// is what overlaps the tensor core with the eight element-wise warps:
//   tensor core:   ... product_j | dP_{j+1} | S_{j+2} | (wait E_{j+1}) product_{j+1} ...
//   element-wise:  S_{j+1} read (frees S) -> P_{j+1} = exp(..) while product_j and
//                  dP_{j+1} run -> fold product_j -> dS_{j+1} -> E_{j+1} hi/lo to TMEM
// S is freed as soon as it is read, so S_{j+2} is computed while the
// element-wise warps finish block j+1; the product's operand E (P^T or dS)
// goes over dP (unused by kDV) with its lo part apart.  Each block's product
// (a 64-term tensor-core sum) is folded into registers with round-to-nearest
// adds; the eight element-wise warps split each 64-column block in halves
// (once lse is known, no row reduction is needed).

enum BwdMode { kDV = 0, kDK = 1, kDQ = 2 };

constexpr float kLog2e = 1.4426950408889634f;
// TMEM columns of the backward kernels.
constexpr uint32_t kBA1 = 0, kBA2 = 128, kBS = 256, kBdP = 320, kBElo = 384, kBO = 448;

template <int MODE, int D>
struct BwdLayout {
  static constexpr bool kTwoA = MODE != kDV;
  static constexpr bool kKeyMajor = MODE != kDQ;
  static constexpr int kRing = D == 64 ? (kTwoA ? 2 : 3) : (kTwoA ? 4 : 6);  // slots per ring
  static constexpr uint32_t kTile = kBKV * D * 4;  // 64 x D fp32 (D/32 boxes of 8 KB)
  static constexpr uint32_t kSlot = 2 * kTile;     // raw | lo
  // Product-ring slots also carry lse*log2e [64] and Delta [64] of the block's
  // queries (key-major modes), padded to keep every tile 1024-byte aligned.
  static constexpr uint32_t kSlot2 = kSlot + (kKeyMajor ? 1024 : 0);
  static constexpr uint32_t kRing0 = 0;                                       // S operand
  static constexpr uint32_t kRing1 = kRing0 + kRing * kSlot;                  // dP operand
  static constexpr uint32_t kRing2 = kRing1 + (kTwoA ? kRing * kSlot : 0);    // product operand
  static constexpr uint32_t kBars = kRing2 + kRing * kSlot2;
  static constexpr uint32_t kNumBars = 6 * kRing + 8;
  static constexpr uint32_t kBytes = kBars + kNumBars * 8 + 16;
  static constexpr uint32_t kDynSmem = kBytes + 1024;
  static_assert(kDynSmem <= 232448, "shared memory budget");
  static_assert(kDynSmem > 232448 / 2, "one CTA per SM (the CTA takes all 512 TMEM columns)");
};

struct BwdParams {
  const float* qkv;
  const float* dout;
  const float* lse;
  const float* delta;
  float* dqkv;
  int T, H, C;
  float scale, scale_log2;
  int xb0, xb1, xb2;  // column of ring r's tensor for head 0 (head h adds h*D)
  int n_items;        // (128-row block, batch x head) pairs
  int nrb;            // 128-row blocks per sequence
};

// One work item: the 128 "major" rows [r0, r0+128) of head h of sequence b
// and their minor blocks blk0 .. blk0+n_blk-1.  Items are numbered longest
// first: key-major items start at the diagonal (the first key block has the
// most query blocks), query-major items end there (the last query block has
// the most key blocks).
struct BwdItem {
  int bh, b, h, r0, blk0, n_blk;
};
template <bool KEY_MAJOR>
__device__ __forceinline__ BwdItem bwd_item(int w, const BwdParams& p) {
  const int BH = p.n_items / p.nrb;
  BwdItem it;
  it.bh = w % BH;
  it.b = it.bh / p.H;
  it.h = it.bh % p.H;
  const int n_all = (p.T + kBKV - 1) / kBKV;
  if (KEY_MAJOR) {
    it.r0 = (w / BH) * kBQ;
    it.blk0 = it.r0 / kBKV;
    it.n_blk = n_all - it.blk0;
  } else {
    it.r0 = (p.nrb - 1 - w / BH) * kBQ;
    it.blk0 = 0;
    it.n_blk = (min(it.r0 + kBQ, p.T) + kBKV - 1) / kBKV;
  }
  return it;
}

// One producer warp: the ring of one B operand over all of the CTA's items
// (raw and lo tiles of each minor block; for the product ring of a key-major
// kernel also the block's lse / Delta vectors).  The copies already issued
// have landed when it returns.
template <int D, int R, bool VEC, bool KEY_MAJOR>
__device__ void produce_ring(uint32_t ring, uint32_t slot_bytes, uint32_t full0, uint32_t empty0,
                             const CUtensorMap* m, const CUtensorMap* mlo, int xb, uint8_t* smem_ring,
                             const BwdParams& p, volatile int* abort) {
  constexpr uint32_t kTile = kBKV * D * 4;
  const int lane = threadIdx.x & 31;
  bool issued[R];
  uint32_t issued_ph[R];
#pragma unroll
  for (int s = 0; s < R; ++s) issued[s] = false, issued_ph[s] = 0;
  bool ok = true;
  uint32_t g = 0;  // minor blocks loaded so far (all items)
  for (int k = 0; ok; ++k) {
    const int w = work_item((int)blockIdx.x, k, (int)gridDim.x, p.n_items);
    if (w < 0) break;
    const BwdItem it = bwd_item<KEY_MAJOR>(w, p);
    const int xcol = xb + it.h * D;
    for (int i = 0; i < it.n_blk; ++i, ++g) {
      const int s = g % R;
      const uint32_t ph = (g / R) & 1u;
      if (!warp_wait(empty0 + 8u * s, ph ^ 1u, abort, &g_timeout)) {
        ok = false;
        break;
      }
      issued[s] = true;
      issued_ph[s] = ph;
      const int blk = it.blk0 + i;
      const int row = it.b * p.T + blk * kBKV;
      const uint32_t dst = ring + s * slot_bytes;
      if (elect_one()) {
        mbar_expect_tx(full0 + 8u * s, 2 * kTile);
#pragma unroll
        for (int c = 0; c < D / 32; ++c) {
          tma_load_2d(dst + c * 8192, m, full0 + 8u * s, xcol + 32 * c, row);
          tma_load_2d(dst + kTile + c * 8192, mlo, full0 + 8u * s, xcol + 32 * c, row);
        }
      }
      __syncwarp();
      if (VEC) {
        float* vec = reinterpret_cast<float*>(smem_ring + s * slot_bytes + 2 * kTile);
        for (int c = lane; c < kBKV; c += 32) {
          const int q = blk * kBKV + c;
          const bool in = q < p.T;
          vec[c] = in ? p.lse[(size_t)it.bh * p.T + q] * kLog2e : 0.0f;
          vec[kBKV + c] = in ? p.delta[(size_t)it.bh * p.T + q] : 0.0f;
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(full0 + 8u * s);
        __syncwarp();
      }
    }
  }
  if (!ok && lane == 0)
    for (int s = 0; s < R; ++s)
      if (issued[s]) mbar_wait_drain(full0 + 8u * s, issued_ph[s], &g_timeout);
}

// Persistent: one CTA per SM loops over work items (dealt like the forward's).
// Per item the element-wise warps load the item's A rows into TMEM as soon as
// the previous item's last S / dP MMA is done, and only then fold the previous
// item's last product and store its gradient rows, so the tensor core starts
// the next item while the previous one's epilogue runs; the next item's A rows
// are prefetched into L2 meanwhile.
template <int MODE, int D>
__global__ void __launch_bounds__(kThreads, 1)
    attn_bwd_tc_kernel(const __grid_constant__ CUtensorMap tm0, const __grid_constant__ CUtensorMap tm0lo,
                       const __grid_constant__ CUtensorMap tm1, const __grid_constant__ CUtensorMap tm1lo,
                       const __grid_constant__ CUtensorMap tm2, const __grid_constant__ CUtensorMap tm2lo,
                       const BwdParams p) {
  using L = BwdLayout<MODE, D>;
  constexpr int R = L::kRing;
  constexpr bool kKeyMajor = L::kKeyMajor;
  constexpr bool kTwoA = L::kTwoA;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  const uint32_t sbase = smem_u32(smem);
  const uint32_t bar0 = sbase + L::kBars;
  const uint32_t full0 = bar0, empty0 = bar0 + 8u * R;
  const uint32_t full1 = bar0 + 16u * R, empty1 = bar0 + 24u * R;
  const uint32_t full2 = bar0 + 32u * R, empty2 = bar0 + 40u * R;
  const uint32_t a_ready = bar0 + 48u * R;
  const uint32_t s_full = a_ready + 8u, s_free = a_ready + 16u, dp_full = a_ready + 24u;
  const uint32_t ew_done = a_ready + 32u, out_full = a_ready + 40u, drain = a_ready + 48u;
  const uint32_t a_free = a_ready + 56u;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::kBars + L::kNumBars * 8);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int cta = (int)blockIdx.x, G = (int)gridDim.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < R; ++s) {
      mbar_init(full0 + 8u * s, 1);
      mbar_init(empty0 + 8u * s, 1);
      mbar_init(full1 + 8u * s, 1);
      mbar_init(empty1 + 8u * s, 1);
      mbar_init(full2 + 8u * s, kKeyMajor ? 2 : 1);
      mbar_init(empty2 + 8u * s, 1);
    }
    mbar_init(a_ready, 2 * kWgThreads);
    mbar_init(s_full, 1);
    mbar_init(s_free, 2 * kWgThreads);
    mbar_init(dp_full, 1);
    mbar_init(ew_done, 2 * kWgThreads);
    mbar_init(out_full, 1);
    mbar_init(drain, 1);
    mbar_init(a_free, 1);
    *abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  fence_before();
  __syncthreads();
  fence_after();
  // Launched as a programmatic dependent (launch_pdl): the set-up above ran
  // while the previous kernel finished; its outputs are read only from here.
  pdl_wait();
  pdl_trigger();
  const uint32_t tmem = *tmem_slot;

  if (warp < 4) {
    reg_dec();
    if (warp == 0) {
      // ---------------------------------------------------------- S operand
      produce_ring<D, R, false, kKeyMajor>(sbase + L::kRing0, L::kSlot, full0, empty0, &tm0, &tm0lo,
                                           p.xb0, smem + L::kRing0, p, abort);
    } else if (warp == 2) {
      // ---------------------------------------------------------- dP operand
      if (kTwoA)
        produce_ring<D, R, false, kKeyMajor>(sbase + L::kRing1, L::kSlot, full1, empty1, &tm1,
                                             &tm1lo, p.xb1, smem + L::kRing1, p, abort);
    } else if (warp == 3) {
      // ---------------------------------------------------------- product operand
      produce_ring<D, R, kKeyMajor, kKeyMajor>(sbase + L::kRing2, L::kSlot2, full2, empty2, &tm2,
                                               &tm2lo, p.xb2, smem + L::kRing2, p, abort);
    } else {
      // ---------------------------------------------------------- MMA issuer
      constexpr uint32_t id_s = instr_desc(kBKV, 0, 0);
      constexpr uint32_t id_o = instr_desc(D, 0, 1);
      // d = a.b over K = D with a (hi at a, lo at a + D) in TMEM and b's
      // K-major raw / lo tiles at t / t + kTile: hi.hi first, then the two
      // cross terms per k-step.
      auto issue_k = [&](uint32_t d, uint32_t a, uint32_t t) {
#pragma unroll
        for (int kk = 0; kk < D / 8; ++kk)
          mma_ts(d, a + kk * 8, k_desc(t, kk), id_s, kk > 0 ? 1u : 0u);
#pragma unroll
        for (int kk = 0; kk < D / 8; ++kk) {
          mma_ts(d, a + kk * 8, k_desc(t + L::kTile, kk), id_s, 1u);
          mma_ts(d, a + D + kk * 8, k_desc(t, kk), id_s, 1u);
        }
      };
      // MMAs and commits of one operation on minor block g (global index over
      // the CTA's items; the elected lane); the waits for its operands come before.
      auto emit_s = [&](uint32_t g) {
        const int s = g % R;
        issue_k(tmem + kBS, tmem + kBA1, sbase + L::kRing0 + s * L::kSlot);
        commit(empty0 + 8u * s);
        commit(s_full);
      };
      auto emit_dp = [&](uint32_t g) {
        const int s = g % R;
        issue_k(tmem + kBdP, tmem + kBA2, sbase + L::kRing1 + s * L::kSlot);
        commit(empty1 + 8u * s);
        commit(dp_full);
      };
      // Product of block g: A = E (hi over dP, lo apart), B = the MN-major tile.
      auto emit_out = [&](uint32_t g) {
        const int s = g % R;
        const uint32_t tb = sbase + L::kRing2 + s * L::kSlot2, tblo = tb + L::kTile;
#pragma unroll
        for (int kk = 0; kk < kBKV / 8; ++kk)
          mma_ts(tmem + kBO, tmem + kBdP + kk * 8, v_desc(tb, kk), id_o, kk > 0 ? 1u : 0u);
#pragma unroll
        for (int kk = 0; kk < kBKV / 8; ++kk) {
          mma_ts(tmem + kBO, tmem + kBdP + kk * 8, v_desc(tblo, kk), id_o, 1u);
          mma_ts(tmem + kBO, tmem + kBElo + kk * 8, v_desc(tb, kk), id_o, 1u);
        }
        commit(empty2 + 8u * s);
        commit(out_full);
      };
      // Tile barrier of ring r (0: S operand, 1: dP operand, 2: product operand) for block g.
      auto tile_full = [&](int r, uint32_t g) {
        return (r == 0 ? full0 : r == 1 ? full1 : full2) + 8u * (g % R);
      };
      auto tile_ph = [&](uint32_t g) { return (g / R) & 1u; };
      auto issue = [&](int r, uint32_t g) -> bool {
        if (!warp_wait(tile_full(r, g), tile_ph(g), abort, &g_timeout)) return false;
        fence_after();
        if (elect_one()) {
          if (r == 0)
            emit_s(g);
          else if (r == 1)
            emit_dp(g);
          else
            emit_out(g);
        }
        __syncwarp();
        return true;
      };
      // After the item's last S and dP: the A columns may take the next item's rows.
      auto release_a = [&]() {
        if (elect_one()) commit(a_free);
        __syncwarp();
      };
      bool ok = true;
      uint32_t g = 0;  // minor blocks of earlier items
      for (int k = 0; ok; ++k) {
        const int w = work_item(cta, k, G, p.n_items);
        if (w < 0) break;
        const int n_blk = bwd_item<kKeyMajor>(w, p).n_blk;
        ok = warp_wait(a_ready, (uint32_t)k & 1u, abort, &g_timeout);
        fence_after();
        if (ok) ok = issue(0, g);
        if (ok && kTwoA) ok = issue(1, g);
        if (ok && n_blk > 1) {
          ok = warp_wait(s_free, g & 1u, abort, &g_timeout);
          fence_after();
          if (ok) ok = issue(0, g + 1);
        }
        // The last S is S_{n-1}; with a dP operand the last dP (dP_{n-1}) comes later.
        if (ok && (n_blk == 1 || (!kTwoA && n_blk == 2))) release_a();
        // dP_{i+1} overwrites the columns product_i reads and S_{i+2} those S_{i+1}
        // was read from: each is issued after the MMAs or the reads it must
        // follow (one CTA's MMAs run in issue order).  The tensor core queues
        // almost no MMAs, so every wait or re-convergence between them idles it:
        // the tile barriers (nearly always complete) are tested while waiting
        // for the element-wise warps, and the MMAs that follow one such wait go
        // out in one elected run.
        for (int i = 0; ok && i < n_blk; ++i) {
          const uint32_t gi = g + (uint32_t)i;
          const bool dp_next = kTwoA && i + 1 < n_blk;
          {
            const bool r2 = mbar_test(tile_full(2, gi), tile_ph(gi));
            const bool r1 = dp_next ? mbar_test(tile_full(1, gi + 1), tile_ph(gi + 1)) : true;
            const bool e = mbar_wait(ew_done, gi & 1u, abort, &g_timeout);
            const uint32_t bits =
                __shfl_sync(0xffffffffu, (e ? 1u : 0u) | (r2 ? 2u : 0u) | (r1 ? 4u : 0u), 0);
            if (!(bits & 1u)) {
              ok = false;
              break;
            }
            fence_after();
            if ((bits & 6u) == 6u) {
              if (elect_one()) {
                emit_out(gi);
                if (dp_next) emit_dp(gi + 1);
              }
              __syncwarp();
            } else if (!issue(2, gi) || (dp_next && !issue(1, gi + 1))) {
              ok = false;
              break;
            }
            if (dp_next && i + 2 == n_blk) release_a();
          }
          if (i + 2 < n_blk) {
            const bool r0 = mbar_test(tile_full(0, gi + 2), tile_ph(gi + 2));
            const bool f = mbar_wait(s_free, (gi + 1) & 1u, abort, &g_timeout);
            const uint32_t bits = __shfl_sync(0xffffffffu, (f ? 1u : 0u) | (r0 ? 2u : 0u), 0);
            if (!(bits & 1u)) {
              ok = false;
              break;
            }
            fence_after();
            if (bits & 2u) {
              if (elect_one()) emit_s(gi + 2);
              __syncwarp();
            } else {
              ok = issue(0, gi + 2);
            }
            if (ok && !kTwoA && i + 3 == n_blk) release_a();
          }
        }
        g += (uint32_t)n_blk;
      }
      if (!ok) {
        if (elect_one()) commit(drain);
        __syncwarp();
        mbar_wait_drain(drain, 0, &g_timeout);
      }
    }
  } else {
    // ------------------------------------------------------------ element-wise
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kHighRegs));
    const int wg = (warp - 4) >> 2;  // columns [32*wg, 32*wg + 32) of every block
    const int ew = warp & 3;
    const int row = ew * 32 + lane;
    const uint32_t lane_off = (uint32_t)(ew * 32) << 16;
    const size_t ld = (size_t)3 * p.C;
    const bool folds = D == 64 || wg == 0;  // output columns [32*wg, 32*wg + 32)
    const float c2 = p.scale_log2;
    // A rows of an item: A1 = K (key-major kernels) or Q (dQ) from qkv, A2 =
    // V (dK) or dO (dQ); the dV kernel has A1 only.
    auto a_rows = [&](const BwdItem& it, const float*& a1, const float*& a2) -> bool {
      const int r = it.r0 + row;
      const bool r_in = r < p.T;
      const size_t grow = (size_t)it.b * p.T + (r_in ? r : 0);
      a1 = p.qkv + grow * ld + (kKeyMajor ? p.C : 0) + (size_t)it.h * D;
      a2 = MODE == kDK ? p.qkv + grow * ld + 2 * (size_t)p.C + (size_t)it.h * D
                       : p.dout + grow * (size_t)p.C + (size_t)it.h * D;
      return r_in;
    };
    float acc[32];
    bool ok = true;
    uint32_t g = 0;      // minor blocks of earlier items
    int prev_w = -1;
    uint32_t prev_last = 0;  // global index of the previous item's last block
    auto fold = [&](uint32_t gi) -> bool {
      if (!mbar_wait(out_full, gi & 1u, abort, &g_timeout)) return false;
      fence_after();
      if (folds) {
        uint32_t v[32];
        tmem_ld32(tmem + lane_off + kBO + 32 * wg, v);
#pragma unroll
        for (int c = 0; c < 32; ++c) acc[c] = __fadd_rn(acc[c], __uint_as_float(v[c]));
      }
      return true;
    };
    // Last fold and gradient rows of item w.
    auto finish = [&](int w) -> bool {
      if (!fold(prev_last)) return false;
      const BwdItem it = bwd_item<kKeyMajor>(w, p);
      const int r = it.r0 + row;
      if (r < p.T && folds) {
        const float f = MODE == kDV ? 1.0f : p.scale;
        const int col = (MODE == kDQ ? 0 : MODE == kDK ? p.C : 2 * p.C) + it.h * D + 32 * wg;
        float* dst = p.dqkv + ((size_t)it.b * p.T + r) * ld + col;
#pragma unroll
        for (int c = 0; c < 32; c += 4)
          *reinterpret_cast<float4*>(dst + c) =
              make_float4(acc[c] * f, acc[c + 1] * f, acc[c + 2] * f, acc[c + 3] * f);
      }
      return true;
    };
    for (int k = 0; ok; ++k) {
      const int w = work_item(cta, k, G, p.n_items);
      if (w < 0) break;
      const BwdItem it = bwd_item<kKeyMajor>(w, p);
      const int r = it.r0 + row;  // key (kDV, kDK) or query (kDQ) index
      {
        // A operands of this row -> TMEM (hi at base, lo at base + D), once the
        // previous item's last S / dP MMA has read the old ones.
        const float* a1;
        const float* a2;
        const bool r_in = a_rows(it, a1, a2);
        if (k > 0 && !mbar_wait(a_free, (uint32_t)(k - 1) & 1u, abort, &g_timeout)) {
          ok = false;
          break;
        }
        fence_after();
#pragma unroll
        for (int t = 0; t < (kTwoA ? 2 : 1); ++t) {
          const float* src = t ? a2 : a1;
          const uint32_t base = tmem + lane_off + (t ? kBA2 : kBA1);
          for (int cc = wg; cc < D / 32; cc += 2) {
            uint32_t hi[32], lo[32];
#pragma unroll
            for (int i = 0; i < 32; i += 4) {
              const float4 x = r_in ? *reinterpret_cast<const float4*>(src + 32 * cc + i)
                                    : make_float4(0.f, 0.f, 0.f, 0.f);
              const float xs[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                hi[i + e] = __float_as_uint(tf32_hi(xs[e]));
                lo[i + e] = __float_as_uint(tf32_lo(xs[e]));
              }
            }
            tmem_st32(base + 32 * cc, hi);
            tmem_st32(base + D + 32 * cc, lo);
          }
        }
        tmem_wait_st();
        fence_before();
        mbar_arrive(a_ready);
        // The next item's A rows -> L2 while this item runs.
        const int wn = work_item(cta, k + 1, G, p.n_items);
        if (wn >= 0) {
          const float* n1;
          const float* n2;
          if (a_rows(bwd_item<kKeyMajor>(wn, p), n1, n2)) {
            for (int cc = wg; cc < D / 32; cc += 2) {
              asm volatile("prefetch.L2 [%0];" ::"l"(n1 + 32 * cc));
              if (kTwoA) asm volatile("prefetch.L2 [%0];" ::"l"(n2 + 32 * cc));
            }
          }
        }
      }
      if (prev_w >= 0 && !finish(prev_w)) {
        ok = false;
        break;
      }
#pragma unroll
      for (int c = 0; c < 32; ++c) acc[c] = 0.0f;
      float lse2_row = 0.0f, delta_row = 0.0f;
      if (!kKeyMajor && r < p.T) {
        lse2_row = p.lse[(size_t)it.bh * p.T + r] * kLog2e;
        delta_row = p.delta[(size_t)it.bh * p.T + r];
      }
      for (int i = 0; i < it.n_blk; ++i) {
        const uint32_t gi = g + (uint32_t)i;
        const int s = gi % R;
        if (!mbar_wait(s_full, gi & 1u, abort, &g_timeout) ||
            (kKeyMajor && !mbar_wait(full2 + 8u * s, (gi / R) & 1u, abort, &g_timeout))) {
          ok = false;
          break;
        }
        fence_after();
        uint32_t sv[32];
        tmem_ld32(tmem + lane_off + kBS + 32 * wg, sv);
        fence_before();
        mbar_arrive(s_free);
        const float* vec =
            reinterpret_cast<const float*>(smem + L::kRing2 + s * L::kSlot2 + 2 * L::kTile) + 32 * wg;
        // Blocks clear of the diagonal (and of the sequence end) need no mask;
        // the test is uniform over the CTA.
        const int m0 = (it.blk0 + i) * kBKV + 32 * wg;  // minor index of column 0 of this half
        const int mb0 = (it.blk0 + i) * kBKV;
        const bool full = kKeyMajor ? (mb0 >= it.r0 + kBQ - 1 && mb0 + kBKV <= p.T)
                                    : (mb0 + kBKV - 1 <= it.r0);
        float e[32];
        if (full) {
#pragma unroll
          for (int c = 0; c < 32; ++c) {
            const float l2 = kKeyMajor ? vec[c] : lse2_row;
            e[c] = fast_exp2(fmaf(__uint_as_float(sv[c]), c2, -l2));
          }
        } else {
#pragma unroll
          for (int c = 0; c < 32; ++c) {
            const int m = m0 + c;
            const bool valid = kKeyMajor ? (m >= r && m < p.T) : (m <= r);
            const float l2 = kKeyMajor ? vec[c] : lse2_row;
            e[c] = valid ? fast_exp2(fmaf(__uint_as_float(sv[c]), c2, -l2)) : 0.0f;
          }
        }
        // dP_i done implies product_{i-1} done (issued before it).
        if (kTwoA && !mbar_wait(dp_full, gi & 1u, abort, &g_timeout)) {
          ok = false;
          break;
        }
        if (i > 0 && !fold(gi - 1)) {
          ok = false;
          break;
        }
        fence_after();
        uint32_t dv[32];
        if (kTwoA) {
          tmem_ld32(tmem + lane_off + kBdP + 32 * wg, dv);
#pragma unroll
          for (int c = 0; c < 32; ++c) {
            const float dl = kKeyMajor ? vec[kBKV + c] : delta_row;
            e[c] = e[c] * (__uint_as_float(dv[c]) - dl);
          }
        }
#pragma unroll
        for (int c = 0; c < 32; ++c) {
          sv[c] = __float_as_uint(tf32_hi(e[c]));
          dv[c] = __float_as_uint(tf32_lo(e[c]));
        }
        tmem_st32(tmem + lane_off + kBdP + 32 * wg, sv);
        tmem_st32(tmem + lane_off + kBElo + 32 * wg, dv);
        tmem_wait_st();
        fence_before();
        mbar_arrive(ew_done);
      }
      if (!ok) break;
      g += (uint32_t)it.n_blk;
      prev_w = w;
      prev_last = g - 1u;
    }
    if (ok && prev_w >= 0) ok = finish(prev_w);
  }

  fence_before();
  __syncthreads();
  if (warp == 1) {
    fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(kTmemCols)
                 : "memory");
  }
}

// ------------------------------------------------------- fused dK + dV
//
// One persistent kernel for both key-side gradients (rows = keys, minor
// blocks = 64 queries): per block j
//   S^T = K.Q^T -> P^T = exp(S^T*scale - lse);   dP^T = V.dO^T
//   dV += P^T.dO;   dS^T = P^T o (dP^T - Delta);   dK += dS^T.Q
// so S^T is computed once for both products (the two-kernel path computes it
// twice and streams Q and lse twice).  TMEM has the same map as the dK
// kernel's: K and V rows (hi / lo) as A operands, S (then P^T hi), dP (then
// dS^T hi), one lo column block shared in turn by P^T lo and dS^T lo, and one
// product accumulator shared in turn by the dV and dK products, which the
// element-wise warps fold into two register accumulators.  The tensor core
// runs, per block,
//   prodV_j | S_{j+1} | prodK_j | dP_{j+1} | prodV_{j+1} | ...
// and each MMA group waits only for the element-wise step it reads
// (ew_p: P^T written, ew_ds: dS^T written); the element-wise warps, per block:
//   read S_j -> P_j (registers) -> fold prodK_{j-1} -> write P^T hi/lo ->
//   fold prodV_j -> read dP_j -> dS_j -> write dS^T hi/lo.
// Rings: Q K-major (with the block's lse*log2e / Delta vectors, in a
// separate vector ring deep enough that a vector is never overwritten before
// its dS step), dO K-major, dO MN-major, Q MN-major.
template <int D>
struct KvLayout {
  static constexpr int kR0 = D == 64 ? 2 : 4;  // Q K-major / dO K-major slots
  static constexpr int kR2 = D == 64 ? 1 : 2;  // dO MN-major / Q MN-major slots
  static constexpr int kVec = 2 * kR0;         // vector slots (see the producer)
  static constexpr uint32_t kTile = kBKV * D * 4;
  static constexpr uint32_t kSlot = 2 * kTile;  // raw | lo
  static constexpr uint32_t kRing0 = 0;
  static constexpr uint32_t kRing1 = kRing0 + kR0 * kSlot;
  static constexpr uint32_t kRing2 = kRing1 + kR0 * kSlot;
  static constexpr uint32_t kRing3 = kRing2 + kR2 * kSlot;
  static constexpr uint32_t kVecs = kRing3 + kR2 * kSlot;  // [kVec][2][64] floats
  static constexpr uint32_t kBars = kVecs + kVec * 2 * kBKV * 4;
  static constexpr uint32_t kNumBars = 4 * kR0 + 4 * kR2 + kVec + 10;
  static constexpr uint32_t kBytes = kBars + kNumBars * 8 + 16;
  static constexpr uint32_t kDynSmem = kBytes + 1024;
  static_assert(kDynSmem <= 232448, "shared memory budget");
  static_assert(kDynSmem > 232448 / 2, "one CTA per SM (the CTA takes all 512 TMEM columns)");
  // The Q-ring producer runs at most kR0 + 1 blocks ahead of the element-wise
  // warps, so a vector slot is rewritten only after its block's dS step.
  static_assert(kVec >= kR0 + 2, "vector ring depth");
};

// Producer of one ring (raw and lo tiles of each block of every item of this
// CTA); with VEC > 0, also the block's lse*log2e and Delta into vector slot
// g % VEC, announced on that slot's barrier (vfull0 + 8 * slot).
template <int D, int R, int VEC>
__device__ void produce_kv(uint32_t ring, uint32_t full0, uint32_t empty0, const CUtensorMap* m,
                           const CUtensorMap* mlo, int xb, float* vecs, uint32_t vfull0,
                           const BwdParams& p, volatile int* abort) {
  constexpr uint32_t kTile = kBKV * D * 4, kSlot = 2 * kTile;
  const int lane = threadIdx.x & 31;
  bool issued[R];
  uint32_t issued_ph[R];
#pragma unroll
  for (int s = 0; s < R; ++s) issued[s] = false, issued_ph[s] = 0;
  bool ok = true;
  uint32_t g = 0;
  for (int k = 0; ok; ++k) {
    const int w = work_item((int)blockIdx.x, k, (int)gridDim.x, p.n_items);
    if (w < 0) break;
    const BwdItem it = bwd_item<true>(w, p);
    const int xcol = xb + it.h * D;
    for (int i = 0; i < it.n_blk; ++i, ++g) {
      const int s = g % R;
      const uint32_t ph = (g / R) & 1u;
      if (!warp_wait(empty0 + 8u * s, ph ^ 1u, abort, &g_timeout)) {
        ok = false;
        break;
      }
      issued[s] = true;
      issued_ph[s] = ph;
      const int blk = it.blk0 + i;
      const int row = it.b * p.T + blk * kBKV;
      const uint32_t dst = ring + s * kSlot;
      if (elect_one()) {
        mbar_expect_tx(full0 + 8u * s, 2 * kTile);
#pragma unroll
        for (int c = 0; c < D / 32; ++c) {
          tma_load_2d(dst + c * 8192, m, full0 + 8u * s, xcol + 32 * c, row);
          tma_load_2d(dst + kTile + c * 8192, mlo, full0 + 8u * s, xcol + 32 * c, row);
        }
      }
      __syncwarp();
      if constexpr (VEC > 0) {
        float* vec = vecs + (g % VEC) * 2 * kBKV;
        for (int c = lane; c < kBKV; c += 32) {
          const int q = blk * kBKV + c;
          const bool in = q < p.T;
          vec[c] = in ? p.lse[(size_t)it.bh * p.T + q] * kLog2e : 0.0f;
          vec[kBKV + c] = in ? p.delta[(size_t)it.bh * p.T + q] : 0.0f;
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(vfull0 + 8u * (g % VEC));
        __syncwarp();
      }
    }
  }
  if (!ok && lane == 0)
    for (int s = 0; s < R; ++s)
      if (issued[s]) mbar_wait_drain(full0 + 8u * s, issued_ph[s], &g_timeout);
}

// Producer of the two MN-major rings, block by block in consumption order
// (dO for prodV_j, then Q for prodK_j).
template <int D, int R>
__device__ void produce_kv_mn(uint32_t ring2, uint32_t full2, uint32_t empty2, uint32_t ring3,
                              uint32_t full3, uint32_t empty3, const CUtensorMap* mdo,
                              const CUtensorMap* mdolo, const CUtensorMap* mq,
                              const CUtensorMap* mqlo, const BwdParams& p, volatile int* abort) {
  constexpr uint32_t kTile = kBKV * D * 4, kSlot = 2 * kTile;
  const int lane = threadIdx.x & 31;
  bool issued[2][R];
  uint32_t issued_ph[2][R];
#pragma unroll
  for (int s = 0; s < R; ++s) issued[0][s] = issued[1][s] = false, issued_ph[0][s] = issued_ph[1][s] = 0;
  bool ok = true;
  uint32_t g = 0;
  for (int k = 0; ok; ++k) {
    const int w = work_item((int)blockIdx.x, k, (int)gridDim.x, p.n_items);
    if (w < 0) break;
    const BwdItem it = bwd_item<true>(w, p);
    for (int i = 0; i < it.n_blk && ok; ++i, ++g) {
      const int s = g % R;
      const uint32_t ph = (g / R) & 1u;
      const int row = it.b * p.T + (it.blk0 + i) * kBKV;
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        const uint32_t full = (r ? full3 : full2) + 8u * s, empty = (r ? empty3 : empty2) + 8u * s;
        if (!warp_wait(empty, ph ^ 1u, abort, &g_timeout)) {
          ok = false;
          break;
        }
        issued[r][s] = true;
        issued_ph[r][s] = ph;
        const uint32_t dst = (r ? ring3 : ring2) + s * kSlot;
        const CUtensorMap* m = r ? mq : mdo;
        const CUtensorMap* mlo = r ? mqlo : mdolo;
        const int xcol = it.h * D;  // Q's columns in qkv, dO's in dout
        if (elect_one()) {
          mbar_expect_tx(full, 2 * kTile);
#pragma unroll
          for (int c = 0; c < D / 32; ++c) {
            tma_load_2d(dst + c * 8192, m, full, xcol + 32 * c, row);
            tma_load_2d(dst + kTile + c * 8192, mlo, full, xcol + 32 * c, row);
          }
        }
        __syncwarp();
      }
    }
  }
  if (!ok && lane == 0)
    for (int r = 0; r < 2; ++r)
      for (int s = 0; s < R; ++s)
        if (issued[r][s]) mbar_wait_drain((r ? full3 : full2) + 8u * s, issued_ph[r][s], &g_timeout);
}

template <int D>
__global__ void __launch_bounds__(kThreads, 1)
    attn_bwd_kv_kernel(const __grid_constant__ CUtensorMap tmQk, const __grid_constant__ CUtensorMap tmQklo,
                       const __grid_constant__ CUtensorMap tmDk, const __grid_constant__ CUtensorMap tmDklo,
                       const __grid_constant__ CUtensorMap tmDmn, const __grid_constant__ CUtensorMap tmDmnlo,
                       const __grid_constant__ CUtensorMap tmQmn, const __grid_constant__ CUtensorMap tmQmnlo,
                       const BwdParams p) {
  using L = KvLayout<D>;
  constexpr int R0 = L::kR0, R2 = L::kR2;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  const uint32_t sbase = smem_u32(smem);
  const uint32_t bar0 = sbase + L::kBars;
  const uint32_t full0 = bar0, empty0 = bar0 + 8u * R0;
  const uint32_t full1 = bar0 + 16u * R0, empty1 = bar0 + 24u * R0;
  const uint32_t full2 = bar0 + 32u * R0, empty2 = full2 + 8u * R2;
  const uint32_t full3 = empty2 + 8u * R2, empty3 = full3 + 8u * R2;
  const uint32_t a_ready = empty3 + 8u * R2;
  const uint32_t a_free = a_ready + 8u, s_full = a_ready + 16u, dp_full = a_ready + 24u;
  const uint32_t ew_p = a_ready + 32u, ew_ds = a_ready + 40u, out_v = a_ready + 48u;
  const uint32_t out_k = a_ready + 56u, drain = a_ready + 64u, vfull = a_ready + 72u;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::kBars + L::kNumBars * 8);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* vecs = reinterpret_cast<float*>(smem + L::kVecs);

  const int cta = (int)blockIdx.x, G = (int)gridDim.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < R0; ++s) {
      mbar_init(full0 + 8u * s, 1);
      mbar_init(empty0 + 8u * s, 1);
      mbar_init(full1 + 8u * s, 1);
      mbar_init(empty1 + 8u * s, 1);
    }
    for (int s = 0; s < R2; ++s) {
      mbar_init(full2 + 8u * s, 1);
      mbar_init(empty2 + 8u * s, 1);
      mbar_init(full3 + 8u * s, 1);
      mbar_init(empty3 + 8u * s, 1);
    }
    mbar_init(a_ready, 2 * kWgThreads);
    mbar_init(a_free, 1);
    mbar_init(s_full, 1);
    mbar_init(dp_full, 1);
    mbar_init(ew_p, 2 * kWgThreads);
    mbar_init(ew_ds, 2 * kWgThreads);
    mbar_init(out_v, 1);
    mbar_init(out_k, 1);
    mbar_init(drain, 1);
    for (int v = 0; v < L::kVec; ++v) mbar_init(vfull + 8u * v, 1);
    *abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  fence_before();
  __syncthreads();
  fence_after();
  // Launched as a programmatic dependent (launch_pdl): the set-up above ran
  // while the previous kernel finished; its outputs are read only from here.
  pdl_wait();
  pdl_trigger();
  const uint32_t tmem = *tmem_slot;

  if (warp < 4) {
    reg_dec();
    if (warp == 0) {
      produce_kv<D, R0, L::kVec>(sbase + L::kRing0, full0, empty0, &tmQk, &tmQklo, 0, vecs, vfull,
                                 p, abort);
    } else if (warp == 2) {
      produce_kv<D, R0, 0>(sbase + L::kRing1, full1, empty1, &tmDk, &tmDklo, 0, nullptr, 0u, p,
                           abort);
    } else if (warp == 3) {
      produce_kv_mn<D, R2>(sbase + L::kRing2, full2, empty2, sbase + L::kRing3, full3, empty3,
                           &tmDmn, &tmDmnlo, &tmQmn, &tmQmnlo, p, abort);
    } else {
      // ---------------------------------------------------------- MMA issuer
      constexpr uint32_t id_s = instr_desc(kBKV, 0, 0);
      constexpr uint32_t id_o = instr_desc(D, 0, 1);
      auto issue_k = [&](uint32_t d, uint32_t a, uint32_t t) {
#pragma unroll
        for (int kk = 0; kk < D / 8; ++kk)
          mma_ts(d, a + kk * 8, k_desc(t, kk), id_s, kk > 0 ? 1u : 0u);
#pragma unroll
        for (int kk = 0; kk < D / 8; ++kk) {
          mma_ts(d, a + kk * 8, k_desc(t + L::kTile, kk), id_s, 1u);
          mma_ts(d, a + D + kk * 8, k_desc(t, kk), id_s, 1u);
        }
      };
      // Product into O: A hi at column a_hi, lo at kBElo; B the MN-major tile at tb.
      auto issue_prod = [&](uint32_t a_hi, uint32_t tb) {
        const uint32_t tblo = tb + L::kTile;
#pragma unroll
        for (int kk = 0; kk < kBKV / 8; ++kk)
          mma_ts(tmem + kBO, tmem + a_hi + kk * 8, v_desc(tb, kk), id_o, kk > 0 ? 1u : 0u);
#pragma unroll
        for (int kk = 0; kk < kBKV / 8; ++kk) {
          mma_ts(tmem + kBO, tmem + a_hi + kk * 8, v_desc(tblo, kk), id_o, 1u);
          mma_ts(tmem + kBO, tmem + kBElo + kk * 8, v_desc(tb, kk), id_o, 1u);
        }
      };
      // Each operation waits for its operand tile (and, for the products, the
      // element-wise step that wrote its A operand), then issues from one
      // elected lane of the converged warp and commits.
      auto op_s = [&](uint32_t g) -> bool {
        const int s = g % R0;
        if (!warp_wait(full0 + 8u * s, (g / R0) & 1u, abort, &g_timeout)) return false;
        fence_after();
        if (elect_one()) {
          issue_k(tmem + kBS, tmem + kBA1, sbase + L::kRing0 + s * L::kSlot);
          commit(empty0 + 8u * s);
          commit(s_full);
        }
        __syncwarp();
        return true;
      };
      auto op_dp = [&](uint32_t g) -> bool {
        const int s = g % R0;
        if (!warp_wait(full1 + 8u * s, (g / R0) & 1u, abort, &g_timeout)) return false;
        fence_after();
        if (elect_one()) {
          issue_k(tmem + kBdP, tmem + kBA2, sbase + L::kRing1 + s * L::kSlot);
          commit(empty1 + 8u * s);
          commit(dp_full);
        }
        __syncwarp();
        return true;
      };
      auto op_prod = [&](uint32_t g, bool dk) -> bool {
        const int s = g % R2;
        if (!warp_wait(dk ? ew_ds : ew_p, g & 1u, abort, &g_timeout)) return false;
        if (!warp_wait((dk ? full3 : full2) + 8u * s, (g / R2) & 1u, abort, &g_timeout)) return false;
        fence_after();
        if (elect_one()) {
          issue_prod(dk ? kBdP : kBS, sbase + (dk ? L::kRing3 : L::kRing2) + s * L::kSlot);
          commit((dk ? empty3 : empty2) + 8u * s);
          commit(dk ? out_k : out_v);
        }
        __syncwarp();
        return true;
      };
      auto release_a = [&]() {
        if (elect_one()) commit(a_free);
        __syncwarp();
      };
      bool ok = true;
      uint32_t g = 0;
      for (int k = 0; ok; ++k) {
        const int w = work_item(cta, k, G, p.n_items);
        if (w < 0) break;
        const int n_blk = bwd_item<true>(w, p).n_blk;
        ok = warp_wait(a_ready, (uint32_t)k & 1u, abort, &g_timeout);
        fence_after();
        if (ok) ok = op_s(g);
        if (ok) ok = op_dp(g);
        if (ok && n_blk == 1) release_a();
        // The tensor core queues almost no MMAs, so every wait between two
        // groups idles it: after each element-wise wait (the real dependency)
        // the tile barriers, nearly always complete, are only tested, and the
        // product and the next S (or dP) go out in one elected run.
        auto batch = [&](uint32_t gi, bool dk, bool next) -> bool {
          if (!warp_wait(dk ? ew_ds : ew_p, gi & 1u, abort, &g_timeout)) return false;
          const int s2 = gi % R2, s0 = (gi + 1) % R0;
          const uint32_t tfull = (dk ? full3 : full2) + 8u * s2;
          const uint32_t nfull = (dk ? full1 : full0) + 8u * s0;
          const bool r2 = mbar_test(tfull, (gi / R2) & 1u);
          const bool r0 = next ? mbar_test(nfull, ((gi + 1) / R0) & 1u) : true;
          const uint32_t bits = __shfl_sync(0xffffffffu, (r2 ? 1u : 0u) | (r0 ? 2u : 0u), 0);
          if (bits != 3u) {  // a tile is late: the plain waits
            if (!op_prod(gi, dk)) return false;
            return !next || (dk ? op_dp(gi + 1) : op_s(gi + 1));
          }
          fence_after();
          if (elect_one()) {
            issue_prod(dk ? kBdP : kBS, sbase + (dk ? L::kRing3 : L::kRing2) + s2 * L::kSlot);
            commit((dk ? empty3 : empty2) + 8u * s2);
            commit(dk ? out_k : out_v);
            if (next) {
              if (dk) {
                issue_k(tmem + kBdP, tmem + kBA2, sbase + L::kRing1 + s0 * L::kSlot);
                commit(empty1 + 8u * s0);
                commit(dp_full);
              } else {
                issue_k(tmem + kBS, tmem + kBA1, sbase + L::kRing0 + s0 * L::kSlot);
                commit(empty0 + 8u * s0);
                commit(s_full);
              }
            }
          }
          __syncwarp();
          return true;
        };
        for (int i = 0; ok && i < n_blk; ++i) {
          const uint32_t gi = g + (uint32_t)i;
          const bool next = i + 1 < n_blk;
          // prodV_i (after P_i), then S_{i+1} over P_i's columns (in issue order);
          // prodK_i (after dS_i), then dP_{i+1} over dS_i's columns.
          ok = batch(gi, false, next);
          if (ok) ok = batch(gi, true, next);
          if (ok && next && i + 2 == n_blk) release_a();  // the item's last S and dP are issued
        }
        g += (uint32_t)n_blk;
      }
      if (!ok) {
        if (elect_one()) commit(drain);
        __syncwarp();
        mbar_wait_drain(drain, 0, &g_timeout);
      }
    }
  } else {
    // ------------------------------------------------------------ element-wise
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kHighRegs));
    const int wg = (warp - 4) >> 2;
    const int ew = warp & 3;
    const int row = ew * 32 + lane;
    const uint32_t lane_off = (uint32_t)(ew * 32) << 16;
    const size_t ld = (size_t)3 * p.C;
    const bool folds = D == 64 || wg == 0;
    const float c2 = p.scale_log2;
    auto a_rows = [&](const BwdItem& it, const float*& a1, const float*& a2) -> bool {
      const int r = it.r0 + row;
      const bool r_in = r < p.T;
      const size_t grow = (size_t)it.b * p.T + (r_in ? r : 0);
      a1 = p.qkv + grow * ld + p.C + (size_t)it.h * D;
      a2 = p.qkv + grow * ld + 2 * (size_t)p.C + (size_t)it.h * D;
      return r_in;
    };
    float acc_v[32], acc_k[32];
    bool ok = true;
    uint32_t g = 0;
    int prev_w = -1;
    auto fold = [&](uint32_t bar, uint32_t gi, float (&acc)[32]) -> bool {
      if (!mbar_wait(bar, gi & 1u, abort, &g_timeout)) return false;
      fence_after();
      if (folds) {
        uint32_t v[32];
        tmem_ld32(tmem + lane_off + kBO + 32 * wg, v);
#pragma unroll
        for (int c = 0; c < 32; ++c) acc[c] = __fadd_rn(acc[c], __uint_as_float(v[c]));
      }
      return true;
    };
    // The previous item's last dK product, then its dK and dV rows.
    auto finish = [&](int w, uint32_t last) -> bool {
      if (!fold(out_k, last, acc_k)) return false;
      fence_before();  // the product's TMEM columns are read before the next prodV writes them
      const BwdItem it = bwd_item<true>(w, p);
      const int r = it.r0 + row;
      if (r < p.T && folds) {
        const size_t base = ((size_t)it.b * p.T + r) * ld + it.h * D + 32 * wg;
        float* dk = p.dqkv + base + p.C;
        float* dv = p.dqkv + base + 2 * (size_t)p.C;
        const float f = p.scale;
#pragma unroll
        for (int c = 0; c < 32; c += 4) {
          *reinterpret_cast<float4*>(dk + c) =
              make_float4(acc_k[c] * f, acc_k[c + 1] * f, acc_k[c + 2] * f, acc_k[c + 3] * f);
          *reinterpret_cast<float4*>(dv + c) =
              make_float4(acc_v[c], acc_v[c + 1], acc_v[c + 2], acc_v[c + 3]);
        }
      }
      return true;
    };
    uint32_t prev_last = 0;
    for (int k = 0; ok; ++k) {
      const int w = work_item(cta, k, G, p.n_items);
      if (w < 0) break;
      const BwdItem it = bwd_item<true>(w, p);
      const int r = it.r0 + row;  // key index
      {
        const float* a1;
        const float* a2;
        const bool r_in = a_rows(it, a1, a2);
        if (k > 0 && !mbar_wait(a_free, (uint32_t)(k - 1) & 1u, abort, &g_timeout)) {
          ok = false;
          break;
        }
        fence_after();
#pragma unroll
        for (int t = 0; t < 2; ++t) {
          const float* src = t ? a2 : a1;
          const uint32_t base = tmem + lane_off + (t ? kBA2 : kBA1);
          for (int cc = wg; cc < D / 32; cc += 2) {
            uint32_t hi[32], lo[32];
#pragma unroll
            for (int i = 0; i < 32; i += 4) {
              const float4 x = r_in ? *reinterpret_cast<const float4*>(src + 32 * cc + i)
                                    : make_float4(0.f, 0.f, 0.f, 0.f);
              const float xs[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                hi[i + e] = __float_as_uint(tf32_hi(xs[e]));
                lo[i + e] = __float_as_uint(tf32_lo(xs[e]));
              }
            }
            tmem_st32(base + 32 * cc, hi);
            tmem_st32(base + D + 32 * cc, lo);
          }
        }
        tmem_wait_st();
        fence_before();
        mbar_arrive(a_ready);
        const int wn = work_item(cta, k + 1, G, p.n_items);
        if (wn >= 0) {
          const float* n1;
          const float* n2;
          if (a_rows(bwd_item<true>(wn, p), n1, n2)) {
            for (int cc = wg; cc < D / 32; cc += 2) {
              asm volatile("prefetch.L2 [%0];" ::"l"(n1 + 32 * cc));
              asm volatile("prefetch.L2 [%0];" ::"l"(n2 + 32 * cc));
            }
          }
        }
      }
      if (prev_w >= 0 && !finish(prev_w, prev_last)) {
        ok = false;
        break;
      }
#pragma unroll
      for (int c = 0; c < 32; ++c) acc_v[c] = acc_k[c] = 0.0f;
      for (int i = 0; i < it.n_blk; ++i) {
        const uint32_t gi = g + (uint32_t)i;
        if (!mbar_wait(s_full, gi & 1u, abort, &g_timeout)) {
          ok = false;
          break;
        }
        fence_after();
        uint32_t sv[32];
        tmem_ld32(tmem + lane_off + kBS + 32 * wg, sv);
        // The vectors of block gi.
        if (!mbar_wait(vfull + 8u * (gi % L::kVec), (gi / L::kVec) & 1u, abort, &g_timeout)) {
          ok = false;
          break;
        }
        const float* vec = vecs + (gi % L::kVec) * 2 * kBKV + 32 * wg;
        const int m0 = (it.blk0 + i) * kBKV + 32 * wg;
        const int mb0 = (it.blk0 + i) * kBKV;
        const bool full = mb0 >= it.r0 + kBQ - 1 && mb0 + kBKV <= p.T;
        float e[32];
        if (full) {
#pragma unroll
          for (int c = 0; c < 32; ++c) e[c] = fast_exp2(fmaf(__uint_as_float(sv[c]), c2, -vec[c]));
        } else {
#pragma unroll
          for (int c = 0; c < 32; ++c) {
            const int m = m0 + c;
            const bool valid = m >= r && m < p.T;
            e[c] = valid ? fast_exp2(fmaf(__uint_as_float(sv[c]), c2, -vec[c])) : 0.0f;
          }
        }
        // prodK of the previous block of this item reads the lo columns and
        // writes O: fold it before P^T's lo part goes there.
        if (i > 0 && !fold(out_k, gi - 1, acc_k)) {
          ok = false;
          break;
        }
        {
          uint32_t hv[32], lv[32];
#pragma unroll
          for (int c = 0; c < 32; ++c) {
            hv[c] = __float_as_uint(tf32_hi(e[c]));
            lv[c] = __float_as_uint(tf32_lo(e[c]));
          }
          tmem_st32(tmem + lane_off + kBS + 32 * wg, hv);
          tmem_st32(tmem + lane_off + kBElo + 32 * wg, lv);
          tmem_wait_st();
          fence_before();
          mbar_arrive(ew_p);
        }
        // dV product of this block, then dS^T = P^T o (dP^T - Delta).
        if (!fold(out_v, gi, acc_v) || !mbar_wait(dp_full, gi & 1u, abort, &g_timeout)) {
          ok = false;
          break;
        }
        fence_after();
        uint32_t dv[32];
        tmem_ld32(tmem + lane_off + kBdP + 32 * wg, dv);
#pragma unroll
        for (int c = 0; c < 32; ++c) e[c] = e[c] * (__uint_as_float(dv[c]) - vec[kBKV + c]);
#pragma unroll
        for (int c = 0; c < 32; ++c) {
          sv[c] = __float_as_uint(tf32_hi(e[c]));
          dv[c] = __float_as_uint(tf32_lo(e[c]));
        }
        tmem_st32(tmem + lane_off + kBdP + 32 * wg, sv);
        tmem_st32(tmem + lane_off + kBElo + 32 * wg, dv);
        tmem_wait_st();
        fence_before();
        mbar_arrive(ew_ds);
      }
      if (!ok) break;
      g += (uint32_t)it.n_blk;
      prev_w = w;
      prev_last = g - 1u;
    }
    if (ok && prev_w >= 0) ok = finish(prev_w, prev_last);
  }

  fence_before();
  __syncthreads();
  if (warp == 1) {
    fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(kTmemCols)
                 : "memory");
  }
}

// lo[r, c] = tf32 lo part of x[r, c] for a [rows, cols] matrix with row
// stride ld, written compact (row stride cols).  cols and ld are multiples of 4.
__global__ void split_lo_rows_k(const float* __restrict__ x, int64_t rows, int cols, int64_t ld,
                                float* __restrict__ lo) {
  pdl_wait();     // the previous kernel's writes are visible (launched by launch_pdl)
  pdl_trigger();  // the next kernel, if launched as a programmatic dependent, may start
  const int c4 = cols >> 2;
  const int64_t total = rows * c4;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += stride) {
    const int64_t r = i / c4, c = (i % c4) * 4;
    const float4 v = *reinterpret_cast<const float4*>(x + r * ld + c);
    *reinterpret_cast<float4*>(lo + r * cols + c) =
        make_float4(tf32_lo(v.x), tf32_lo(v.y), tf32_lo(v.z), tf32_lo(v.w));
  }
}

ns_status split_rows(const float* x, int64_t rows, int cols, float* lo, cudaStream_t s) {
  const int64_t work = rows * (cols / 4);
  const int grid = (int)std::max<int64_t>(1, std::min<int64_t>(ceil_div64(work, 256), (int64_t)sm_count() * 8));
  return launch_pdl(split_lo_rows_k, dim3(grid), dim3(256), 0, s, "ns_attn_bwd operand split", x,
                    rows, cols, cols, lo);
}

template <int MODE, int D>
ns_status launch_bwd_mode(const CUtensorMap* maps, const BwdParams& p, int B, int T, int H,
                          cudaStream_t s) {
  using L = BwdLayout<MODE, D>;
  auto kern = attn_bwd_tc_kernel<MODE, D>;
  NS_TRY_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)L::kDynSmem),
              "ns_attn_bwd attr");
  cudaFuncAttributes fa;
  NS_TRY_CUDA(cudaFuncGetAttributes(&fa, kern), "ns_attn_bwd attributes");
  if (fa.numRegs < kMinLaunchRegs)
    return fail(NS_ERR_UNSUPPORTED, "ns_attn_bwd: kernel compiled with too few registers for its split");
  const int grid = std::min(p.n_items, sm_count());
  return launch_pdl(kern, dim3(grid), dim3(kThreads), L::kDynSmem, s,
                    MODE == kDV ? "ns_attn_bwd dV tcgen05"
                                : MODE == kDK ? "ns_attn_bwd dK tcgen05" : "ns_attn_bwd dQ tcgen05",
                    maps[0], maps[1], maps[2], maps[3], maps[4], maps[5], p);
}

template <int D>
ns_status launch_bwd_kv(const CUtensorMap* m, const BwdParams& p, cudaStream_t s) {
  using L = KvLayout<D>;
  auto kern = attn_bwd_kv_kernel<D>;
  NS_TRY_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)L::kDynSmem),
              "ns_attn_bwd attr");
  cudaFuncAttributes fa;
  NS_TRY_CUDA(cudaFuncGetAttributes(&fa, kern), "ns_attn_bwd attributes");
  if (fa.numRegs < kMinLaunchRegs)
    return fail(NS_ERR_UNSUPPORTED, "ns_attn_bwd: kernel compiled with too few registers for its split");
  const int grid = std::min(p.n_items, sm_count());
  return launch_pdl(kern, dim3(grid), dim3(kThreads), L::kDynSmem, s, "ns_attn_bwd dK+dV tcgen05",
                    m[0], m[1], m[2], m[3], m[4], m[5], m[6], m[7], p);
}

template <int D>
ns_status launch_bwd(const float* qkv, const float* qkv_lo_in, const float* dout, const float* lse,
                     const float* delta, int B, int T, int H, float* dqkv, float* qkv_lo_ws,
                     float* dout_lo, bool fused, cudaStream_t s) {
  const int C = H * D, rows = B * T;
  ns_status rc = NS_OK;
  if (!qkv_lo_in) rc = split_rows(qkv, rows, 3 * C, qkv_lo_ws, s);
  const float* qkv_lo = qkv_lo_in ? qkv_lo_in : qkv_lo_ws;

  if (rc != NS_OK) return rc;
  // qkv and dout (and their lo copies), each as a K-major and an MN-major map.
  CUtensorMap qk, qmn, qlk, qlmn, dk, dmn, dlk, dlmn;
  rc = make_map(&qk, qkv, 3 * C, rows, 3 * C, kBKV, false);
  if (rc == NS_OK) rc = make_map(&qmn, qkv, 3 * C, rows, 3 * C, kBKV, true);
  if (rc == NS_OK) rc = make_map(&qlk, qkv_lo, 3 * C, rows, 3 * C, kBKV, false);
  if (rc == NS_OK) rc = make_map(&qlmn, qkv_lo, 3 * C, rows, 3 * C, kBKV, true);
  if (rc == NS_OK) rc = make_map(&dk, dout, C, rows, C, kBKV, false);
  if (rc == NS_OK) rc = make_map(&dmn, dout, C, rows, C, kBKV, true);
  if (rc == NS_OK) rc = make_map(&dlk, dout_lo, C, rows, C, kBKV, false);
  if (rc == NS_OK) rc = make_map(&dlmn, dout_lo, C, rows, C, kBKV, true);
  if (rc != NS_OK) return rc;
  const float scale = 1.0f / sqrtf((float)D);
  const int nrb = (T + kBQ - 1) / kBQ;
  BwdParams p{qkv, dout, lse, delta, dqkv, T, H, C, scale, scale * kLog2e, 0, 0, 0, nrb * B * H, nrb};
  if (fused) {  // dK and dV: Q and dO, each K-major and MN-major
    const CUtensorMap m[8] = {qk, qlk, dk, dlk, dmn, dlmn, qmn, qlmn};
    rc = launch_bwd_kv<D>(m, p, s);
    if (rc != NS_OK) return rc;
  } else {
  {  // dV: Q (K-major), dO (MN-major)
    const CUtensorMap m[6] = {qk, qlk, dmn, dlmn, dmn, dlmn};
    p.xb0 = 0; p.xb1 = 0; p.xb2 = 0;
    rc = launch_bwd_mode<kDV, D>(m, p, B, T, H, s);
    if (rc != NS_OK) return rc;
  }
  {  // dK: Q (K-major), dO (K-major), Q (MN-major)
    const CUtensorMap m[6] = {qk, qlk, dk, dlk, qmn, qlmn};
    p.xb0 = 0; p.xb1 = 0; p.xb2 = 0;
    rc = launch_bwd_mode<kDK, D>(m, p, B, T, H, s);
    if (rc != NS_OK) return rc;
  }
  }
  {  // dQ: K (K-major), V (K-major), K (MN-major)
    const CUtensorMap m[6] = {qk, qlk, qk, qlk, qmn, qlmn};
    p.xb0 = C; p.xb1 = 2 * C; p.xb2 = C;
    rc = launch_bwd_mode<kDQ, D>(m, p, B, T, H, s);
  }
  return rc;
}

}  // namespace

bool fwd_supported(const float* qkv, const float* out, int B, int T, int H, int D) {
  if (D != 32 && D != 64) return false;
  if (((reinterpret_cast<uintptr_t>(qkv) | reinterpret_cast<uintptr_t>(out)) & 15) != 0) return false;
  if ((int64_t)B * T >= (1ll << 31) || (int64_t)3 * H * D >= (1ll << 31)) return false;
  static const int supported = ns_device_supported();  // thread-safe, once
  return supported == 1;
}

size_t fwd_workspace_bytes(int B, int T, int H, int D) {
  return (size_t)B * T * 2 * H * D * sizeof(float);
}

ns_status fwd(const float* qkv, const float* qkv_lo, int B, int T, int H, int D, float* out,
              float* out_lo, float* lse, float* lo, cudaStream_t s) {
  return D == 64 ? launch_fwd<64>(qkv, qkv_lo, B, T, H, out, out_lo, lse, lo, s)
                 : launch_fwd<32>(qkv, qkv_lo, B, T, H, out, out_lo, lse, lo, s);
}

bool bwd_supported(const float* qkv, const float* dout, const float* dqkv, int B, int T, int H,
                   int D) {
  if (((reinterpret_cast<uintptr_t>(dout) | reinterpret_cast<uintptr_t>(dqkv)) & 15) != 0) return false;
  return fwd_supported(qkv, qkv, B, T, H, D);
}

size_t bwd_lo_bytes(int B, int T, int H, int D) {
  return (size_t)B * T * 4 * H * D * sizeof(float);
}

float* bwd_dout_lo(float* lo, int B, int T, int H, int D) {
  return lo + (size_t)B * T * 3 * H * D;
}

ns_status bwd(const float* qkv, const float* qkv_lo, const float* dout, const float* lse,
              const float* delta, int B, int T, int H, int D, float* dqkv, float* lo, bool fused,
              cudaStream_t s) {
  float* qkv_lo_ws = lo;
  float* dout_lo = lo + (size_t)B * T * 3 * H * D;
  return D == 64 ? launch_bwd<64>(qkv, qkv_lo, dout, lse, delta, B, T, H, dqkv, qkv_lo_ws, dout_lo,
                                  fused, s)
                 : launch_bwd<32>(qkv, qkv_lo, dout, lse, delta, B, T, H, dqkv, qkv_lo_ws, dout_lo,
                                  fused, s);
}

// 1 if a kernel of this file raised the timeout flag since the last call
// (the flag is cleared), 0 if not, or -(CUDA error) if the flag could not be
// read or cleared (a sticky error, or a call during stream capture).
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

}  // namespace attn_tc
}  // namespace nsb
