// tma.cu — tensor-map encoding through cuTensorMapEncodeTiled.
#include "tma.h"

#include <mutex>

namespace nd {

namespace {
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn g_encode = nullptr;
std::once_flag g_encode_once;
cudaError_t g_encode_status = cudaSuccess;

void load_encode() {
  void* fn = nullptr;
  cudaDriverEntryPointQueryResult q;
  g_encode_status =
      cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &fn, 12000, cudaEnableDefault, &q);
  if (g_encode_status == cudaSuccess && q != cudaDriverEntryPointSuccess)
    g_encode_status = cudaErrorSymbolNotFound;
  if (g_encode_status == cudaSuccess) g_encode = reinterpret_cast<EncodeTiledFn>(fn);
}
using CtxGetCurrentFn = CUresult (*)(CUcontext*);
using CtxGetIdFn = CUresult (*)(CUcontext, unsigned long long*);
CtxGetCurrentFn g_ctx_current = nullptr;
CtxGetIdFn g_ctx_id = nullptr;
std::once_flag g_ctx_once;

void load_ctx() {
  void* fn = nullptr;
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPointByVersion("cuCtxGetCurrent", &fn, 12000, cudaEnableDefault, &q) ==
          cudaSuccess && q == cudaDriverEntryPointSuccess)
    g_ctx_current = reinterpret_cast<CtxGetCurrentFn>(fn);
  fn = nullptr;
  if (cudaGetDriverEntryPointByVersion("cuCtxGetId", &fn, 12000, cudaEnableDefault, &q) ==
          cudaSuccess && q == cudaDriverEntryPointSuccess)
    g_ctx_id = reinterpret_cast<CtxGetIdFn>(fn);
}
}  // namespace

unsigned long long current_context_id() {
  std::call_once(g_ctx_once, load_ctx);
  if (g_ctx_current == nullptr || g_ctx_id == nullptr) return 0;
  CUcontext ctx = nullptr;
  if (g_ctx_current(&ctx) != CUDA_SUCCESS || ctx == nullptr) return 0;
  unsigned long long id = 0;
  if (g_ctx_id(ctx, &id) != CUDA_SUCCESS) return 0;
  return id;
}

cudaError_t make_tmap_bf16_sw128(CUtensorMap* map, const void* base, int rank,
                                 const uint64_t* dims, const uint64_t* strides_bytes,
                                 const uint32_t* box, const char** err_msg) {
  return make_tmap_sw128(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, base, rank, dims, strides_bytes,
                         box, err_msg);
}

cudaError_t make_tmap_sw128(CUtensorMap* map, CUtensorMapDataType dtype, int elem_bytes,
                            const void* base, int rank, const uint64_t* dims,
                            const uint64_t* strides_bytes, const uint32_t* box,
                            const char** err_msg) {
  if (static_cast<uint64_t>(box[0]) * static_cast<uint64_t>(elem_bytes) != 128) {
    if (err_msg) *err_msg = "tensor-map box rows must be 128 bytes for the 128-byte swizzle";
    return cudaErrorInvalidValue;
  }
  std::call_once(g_encode_once, load_encode);
  if (g_encode == nullptr) {
    if (err_msg) *err_msg = "cuTensorMapEncodeTiled entry point unavailable";
    return g_encode_status != cudaSuccess ? g_encode_status : cudaErrorSymbolNotFound;
  }
  cuuint64_t gdim[5];
  cuuint64_t gstride[4];
  cuuint32_t bdim[5];
  cuuint32_t estride[5];
  for (int i = 0; i < rank; ++i) {
    gdim[i] = dims[i];
    bdim[i] = box[i];
    estride[i] = 1;
  }
  for (int i = 0; i + 1 < rank; ++i) gstride[i] = strides_bytes[i];
  CUresult r = g_encode(map, dtype, static_cast<cuuint32_t>(rank),
                        const_cast<void*>(base), gdim, gstride, bdim, estride,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    if (err_msg) *err_msg = "cuTensorMapEncodeTiled rejected the tensor geometry";
    return cudaErrorInvalidValue;
  }
  return cudaSuccess;
}

}  // namespace nd
