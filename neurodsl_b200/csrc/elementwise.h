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

// out[i][:] = table[idx[i] - base][:] for i < n (d elements of elem_bytes 4
// or 2, row strides in elements); idx_kind 0: float indices, 1: int32,
// 2: int64.  Bad indices give zero rows and set *err_word.
cudaError_t launch_gather_rows(cudaStream_t stream, const void* table, int elem_bytes,
                               long long ld_table, int vocab, const void* idx, int idx_kind,
                               int base, int n, int d, void* out, long long ld_out, int* err_word);

// dst[b][r][c] = src[b][r][c], batch x rows x cols elements of elem_bytes (2
// or 4), row strides and batch strides in elements (batch <= 65535).
cudaError_t launch_copy_2d(cudaStream_t stream, const void* src, long long ld_src, void* dst,
                           long long ld_dst, int rows, int cols, int elem_bytes, int batch = 1,
                           long long bs_src = 0, long long bs_dst = 0);

// Row softmax of [rows][cols] fp32 (rows of -Inf give zeros).
cudaError_t launch_softmax(cudaStream_t stream, const float* x, float* y, int rows, int cols);

}  // namespace nd
