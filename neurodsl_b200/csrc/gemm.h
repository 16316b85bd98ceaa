// gemm.h — launcher for the tcgen05 GEMM with bias / GELU / residual epilogue.
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "../../include/neurodsl_b200.h"

namespace nd {

// Y[M][N] = act(A[M][K] · W[N][K]ᵀ + bias[N]) + residual[M][N]
// A, W bf16 with K % 8 == 0 and 16-byte aligned bases; bias fp32 or null;
// residual bf16 / fp32 or null; Y bf16 or fp32.  act is an ND_ACT_* code.
cudaError_t launch_gemm(cudaStream_t stream, const __nv_bfloat16* A, const __nv_bfloat16* W,
                        const float* bias, const void* residual, bool residual_f32, void* Y,
                        bool out_f32, int M, int N, int K, int act, const char** err_msg);

}  // namespace nd
