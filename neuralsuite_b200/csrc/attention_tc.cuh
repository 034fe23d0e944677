// Interface between the attention entry points and the tcgen05 attention kernels.
#pragma once

#include "common.cuh"

namespace nsb {
namespace attn_tc {

// True when the tensor-core forward handles this shape on this device
// (head_dim 32 or 64, 16-byte aligned qkv and out, sm_100).
bool fwd_supported(const float* qkv, const float* out, int B, int T, int H, int D);

// Bytes of the K/V lo-part copy the tensor-core forward needs ([B*T, 2*H*D] fp32).
size_t fwd_workspace_bytes(int B, int T, int H, int D);

// out / lse from qkv; `lo` holds fwd_workspace_bytes, 16-byte aligned (unused
// when qkv_lo, the tf32 lo part of all of qkv, is given).  out_lo (optional)
// receives out's tf32 lo part.
ns_status fwd(const float* qkv, const float* qkv_lo, int B, int T, int H, int D, float* out,
              float* out_lo, float* lse, float* lo, cudaStream_t s);

// True when the tensor-core backward handles this shape (as forward, plus
// 16-byte aligned dout and dqkv).
bool bwd_supported(const float* qkv, const float* dout, const float* dqkv, int B, int T, int H,
                   int D);

// Bytes of the lo-part copies of qkv and dout the tensor-core backward needs.
size_t bwd_lo_bytes(int B, int T, int H, int D);

// Where in `lo` (bwd_lo_bytes) bwd expects dout's tf32 lo part, which the
// caller writes beforehand (with Delta).
float* bwd_dout_lo(float* lo, int B, int T, int H, int D);

// dqkv from qkv, dout, lse and delta (= rowsum(dout * out)); `lo` holds
// bwd_lo_bytes, 16-byte aligned, with dout's lo part already at
// bwd_dout_lo(lo).  qkv_lo (optional): the tf32 lo part of qkv, which is then
// not split again.  fused: dK and dV from one kernel (else one kernel each).
ns_status bwd(const float* qkv, const float* qkv_lo, const float* dout, const float* lse,
              const float* delta, int B, int T, int H, int D, float* dqkv, float* lo, bool fused,
              cudaStream_t s);

// 1 if an attention kernel hit a bounded-wait timeout since the last call (clears it).
int consume_timeout_flag();

}  // namespace attn_tc
}  // namespace nsb
