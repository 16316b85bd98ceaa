// tma.h — host-side TMA tensor-map construction (driver entry point fetched
// through the runtime, so the library needs no link-time libcuda).
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace nd {

// Encode a tiled bf16 tensor map with 128-byte swizzle.
//   rank 2 or 3; dims[0] is the contiguous dimension (elements);
//   strides_bytes[i] is the byte stride of dimension i+1;
//   box[i] the tile extent (box[0] * 2 bytes must equal 128 for SW128).
// Returns cudaSuccess or an error; writes a description into *err_msg on failure.
cudaError_t make_tmap_bf16_sw128(CUtensorMap* map, const void* base, int rank,
                                 const uint64_t* dims, const uint64_t* strides_bytes,
                                 const uint32_t* box, const char** err_msg);

// The same for another element type (CU_TENSOR_MAP_DATA_TYPE_*), 128-byte
// swizzle: box[0] * element size must be 128 bytes.
cudaError_t make_tmap_sw128(CUtensorMap* map, CUtensorMapDataType dtype, int elem_bytes,
                            const void* base, int rank, const uint64_t* dims,
                            const uint64_t* strides_bytes, const uint32_t* box,
                            const char** err_msg);

// Unique id of the calling thread's current CUDA context (cuCtxGetId through
// the driver entry point), or 0 when it cannot be read.  Device addresses of
// the library's __device__ variables are valid for one context only; callers
// that cache such an address compare this id to notice that the context was
// torn down and created again (cudaDeviceReset, primary-context release).
unsigned long long current_context_id();

}  // namespace nd
