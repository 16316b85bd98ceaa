// elementwise.cu — the unfused graph ops (those rewrite rules fuse away, and
// the residual :add):
//   gelu_kernel        y = GELU(x) elementwise (the :gelu op; sigmoid, tanh or
//                      erf form, the same forms as the GEMM epilogue)
//   scale_mask_kernel  y = x / sqrt(d_head) + causal mask (the :scale_mask op,
//                      src/dispatch.jl:464-474 with scale_mask_fwd! and
//                      causal_mask, src/kernels.jl:425-430: -Inf above the
//                      diagonal of each [rows][cols] score block)
//   softmax_kernel     row softmax (the :softmax op, src/kernels.jl:269-287)
//   add_kernel         the :add op with its vector broadcasts
//                      (src/dispatch.jl:386-417)
// fp32 rows in and out (the graph's Float32 node values).  HBM-bound; a warp
// per row for the softmax with 16-byte loads where the row allows.
#include <cuda_bf16.h>
#include <math.h>
#include <stdint.h>

#include "elementwise.h"

namespace nd {
namespace {

__device__ __forceinline__ float gelu1(float z, int act) {
  if (act == ND_ACT_GELU_SIGMOID) return z / (1.f + expf(-1.702f * z));
  if (act == ND_ACT_GELU_TANH) {
    const float c0 = 0.7978845608028654f, c1 = 0.044715f;
    return 0.5f * z * (1.f + tanhf(c0 * (z + c1 * z * z * z)));
  }
  if (act == ND_ACT_GELU_ERF) return 0.5f * z * (1.f + erff(z * 0.7071067811865476f));
  return z;
}

__global__ void gelu_kernel(const float* __restrict__ x, float* __restrict__ y, long long n,
                            int act) {
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x)
    y[i] = gelu1(x[i], act);
}

__global__ void scale_mask_kernel(const float* __restrict__ x, float* __restrict__ y, int rows,
                                  int cols, float scale) {
  const long long n = static_cast<long long>(rows) * cols;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int r = static_cast<int>(i / cols), c = static_cast<int>(i - static_cast<long long>(r) * cols);
    y[i] = c > r ? -INFINITY : x[i] * scale;
  }
}

// y = a + b over [rows][cols] fp32; b is the same shape (mode 0), one value
// per column (mode 1), one per row (mode 2) or a single value (mode 3): the
// :add op with its bias broadcasts (src/dispatch.jl:386-417).
__global__ void add_kernel(const float* __restrict__ a, const float* __restrict__ b,
                           float* __restrict__ y, int rows, int cols, int mode) {
  const long long n = static_cast<long long>(rows) * cols;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long bi = mode == 0 ? i : mode == 1 ? i % cols : mode == 2 ? i / cols : 0;
    y[i] = a[i] + b[bi];
  }
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ float warp_add(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// A warp per row: max, then the sum of exp(x - max), then the normalised
// values.  A row of -Inf gives zeros (no NaN), like the reference's guarded
// division.
__global__ void __launch_bounds__(256)
    softmax_kernel(const float* __restrict__ x, float* __restrict__ y, int rows, int cols) {
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const float* xr = x + static_cast<size_t>(row) * cols;
  float* yr = y + static_cast<size_t>(row) * cols;
  float m = -INFINITY;
  for (int c = lane; c < cols; c += 32) m = fmaxf(m, xr[c]);
  m = warp_max(m);
  float s = 0.f;
  if (m != -INFINITY)
    for (int c = lane; c < cols; c += 32) s += expf(xr[c] - m);
  s = warp_add(s);
  const float inv = s > 0.f ? 1.f / s : 0.f;
  for (int c = lane; c < cols; c += 32) yr[c] = m == -INFINITY ? 0.f : expf(xr[c] - m) * inv;
}

int grid_for(long long n, int threads) {
  const long long b = (n + threads - 1) / threads;
  return static_cast<int>(b < 148 * 32 ? b : 148 * 32);
}

}  // namespace

cudaError_t launch_gelu(cudaStream_t stream, const float* x, float* y, long long n, int act) {
  if (n == 0) return cudaSuccess;
  gelu_kernel<<<grid_for(n, 256), 256, 0, stream>>>(x, y, n, act);
  return cudaGetLastError();
}

cudaError_t launch_scale_mask(cudaStream_t stream, const float* x, float* y, int rows, int cols,
                              float scale) {
  const long long n = static_cast<long long>(rows) * cols;
  if (n == 0) return cudaSuccess;
  scale_mask_kernel<<<grid_for(n, 256), 256, 0, stream>>>(x, y, rows, cols, scale);
  return cudaGetLastError();
}

cudaError_t launch_add(cudaStream_t stream, const float* a, const float* b, float* y, int rows,
                       int cols, int mode) {
  const long long n = static_cast<long long>(rows) * cols;
  if (n == 0) return cudaSuccess;
  add_kernel<<<grid_for(n, 256), 256, 0, stream>>>(a, b, y, rows, cols, mode);
  return cudaGetLastError();
}

cudaError_t launch_softmax(cudaStream_t stream, const float* x, float* y, int rows, int cols) {
  if (rows == 0 || cols == 0) return cudaSuccess;
  softmax_kernel<<<(rows + 7) / 8, 256, 0, stream>>>(x, y, rows, cols);
  return cudaGetLastError();
}

}  // namespace nd
