// Conv2D entry points shared inside the library (not part of the C ABI).
//
// forward_keep / backward_from_cols let a model that runs a convolution's
// forward and backward on the same input keep the batch's im2col columns
// (and their tf32 lo parts) from the forward instead of rebuilding them in
// the backward: the U-Net step holds one column buffer per convolution.
#pragma once

#include <stddef.h>
#include <stdint.h>

#include <cuda_runtime.h>

#include "ns_b200.h"

namespace nsb {
namespace conv {

// Floats of one column buffer (IC*k*k rows x B*OH*OW columns); 0 for bad
// parameters and for convolutions whose forward and weight gradient run on
// the direct paths (no columns).
int64_t cols_floats(int B, int IC, int H, int W, int OC, int k, int stride, int pad);

// Workspace bytes of forward_keep / backward_from_cols (no room for columns).
size_t keep_workspace_size(int B, int IC, int H, int W, int OC, int k, int stride, int pad);

// ns_conv2d_fwd that writes the columns and their lo parts to `cols` and
// `cols_lo` (cols_floats each, 16-byte aligned; unused when that is 0) and
// leaves them there.
ns_status forward_keep(const float* x, int B, int IC, int H, int W, const float* weight,
                       const float* bias, int OC, int k, int stride, int pad, float* y,
                       float* cols, float* cols_lo, void* workspace, size_t workspace_bytes,
                       cudaStream_t s);

// ns_conv2d_bwd on the columns forward_keep left for the same input x (x
// itself is read only by the direct paths of small convolutions).
ns_status backward_from_cols(const float* x, const float* cols, const float* cols_lo,
                             const float* dy, int B, int IC, int H, int W, const float* weight,
                             int OC, int k, int stride, int pad, float* dx, float* dweight,
                             float* dbias, void* workspace, size_t workspace_bytes,
                             cudaStream_t s);

}  // namespace conv
}  // namespace nsb
