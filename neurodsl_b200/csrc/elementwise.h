// elementwise.h — launchers of the unfused graph ops (:gelu, :scale_mask, :softmax).
#pragma once
#include <cuda_runtime.h>

#include "../../include/neurodsl_b200.h"

namespace nd {

// y[i] = GELU(x[i]) for n fp32 values; act is an ND_ACT_GELU_* form.
cudaError_t launch_gelu(cudaStream_t stream, const float* x, float* y, long long n, int act);

// y = x * scale with -Inf where column > row, for one [rows][cols] fp32 block.
cudaError_t launch_scale_mask(cudaStream_t stream, const float* x, float* y, int rows, int cols,
                              float scale);

// y = a + b over [rows][cols] fp32: b the same shape (mode 0), one value per
// column (mode 1) or one per row (mode 2).
cudaError_t launch_add(cudaStream_t stream, const float* a, const float* b, float* y, int rows,
                       int cols, int mode);

// Row softmax of [rows][cols] fp32 (rows of -Inf give zeros).
cudaError_t launch_softmax(cudaStream_t stream, const float* x, float* y, int rows, int cols);

}  // namespace nd
