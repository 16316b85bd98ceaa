// layernorm.h — launcher for the row LayerNorm kernel.
#pragma once
#include <cuda_runtime.h>

namespace nd {

// vec_ok: d % 8 == 0 and x, y, gamma, beta 16-byte aligned (vector path).
cudaError_t launch_layernorm(cudaStream_t stream, const void* x, bool x_bf16, const float* gamma,
                             const float* beta, void* y, bool y_bf16, float* mean, float* rstd,
                             int rows, int d, float eps, bool vec_ok);

}  // namespace nd
