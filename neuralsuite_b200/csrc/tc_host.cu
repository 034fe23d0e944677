// Host side of the tcgen05 kernels: TMA tensor-map encoding through the driver
// entry point (no link-time dependency on libcuda).
#include "tc_common.cuh"

namespace nsb {
namespace tcx {
namespace {

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  // Looked up once; the initialisation of a function-local static is thread-safe.
  static const EncodeTiledFn fn = []() -> EncodeTiledFn {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      return reinterpret_cast<EncodeTiledFn>(p);
    return nullptr;
  }();
  return fn;
}

}  // namespace

// 2-D fp32 map over a row-major [rows, inner] matrix with row stride ld,
// box {32, box_rows}, out-of-bounds elements read as zero.  K-major operands
// use the 16-byte-chunk 128B swizzle, MN-major operands the 32-byte-chunk one.
ns_status make_map(CUtensorMap* map, const float* ptr, int inner, int rows, int ld, int box_rows,
                   bool mn_major) {
  std::memset(map, 0, sizeof(*map));
  EncodeTiledFn enc = encode_fn();
  if (!enc) return fail(NS_ERR_UNSUPPORTED, "cuTensorMapEncodeTiled is not available");
  cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)ld * sizeof(float)};
  cuuint32_t box[2] = {32u, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1u, 1u};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(ptr), dims,
                   strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   mn_major ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B : CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(NS_ERR_INVALID_ARGUMENT, "cuTensorMapEncodeTiled failed");
  return NS_OK;
}

}  // namespace tcx
}  // namespace nsb
