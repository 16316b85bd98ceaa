// layernorm.cu — row LayerNorm with fp32 statistics.
//
// y = (x - mean) * rstd * gamma + beta, mean/var over each row of x [rows][d],
// rstd = 1/sqrt(var + eps).  The reference has only RMSNorm
// (rmsnorm_fwd!, src/kernels.jl:48-64 and :104-131: one block per row, warp
// shuffles); this kernel keeps that per-row structure and adds the mean
// subtraction and beta of a true LayerNorm.  mean/rstd mirror the
// aux_data[:rms_inv] side output of :rmsnorm (src/dispatch.jl:426-438).
//
// HBM-bound: x is read once and y written once.  One warp owns a row and
// keeps it in registers (d <= 2048, d % 8 == 0 for 16-byte loads); other
// shapes use a block per row with the row staged in shared memory.
#include <cuda_bf16.h>
#include <stdint.h>

#include "launch.cuh"
#include "layernorm.h"

namespace nd {
namespace {

template <typename T>
struct Vec8;
template <>
struct Vec8<float> {
  static __device__ __forceinline__ void load(const float* p, float (&v)[8]) {
    const float4 a = reinterpret_cast<const float4*>(p)[0];
    const float4 b = reinterpret_cast<const float4*>(p)[1];
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  }
  static __device__ __forceinline__ void store(float* p, const float (&v)[8]) {
    reinterpret_cast<float4*>(p)[0] = make_float4(v[0], v[1], v[2], v[3]);
    reinterpret_cast<float4*>(p)[1] = make_float4(v[4], v[5], v[6], v[7]);
  }
};
template <>
struct Vec8<__nv_bfloat16> {
  static __device__ __forceinline__ void load(const __nv_bfloat16* p, float (&v)[8]) {
    const uint4 u = *reinterpret_cast<const uint4*>(p);
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      v[2 * i] = __uint_as_float(w[i] << 16);
      v[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
    }
  }
  static __device__ __forceinline__ void store(__nv_bfloat16* p, const float (&v)[8]) {
    uint32_t w[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      __nv_bfloat162 h = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
      w[i] = *reinterpret_cast<uint32_t*>(&h);
    }
    *reinterpret_cast<uint4*>(p) = make_uint4(w[0], w[1], w[2], w[3]);
  }
};

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

template <typename T>
__device__ __forceinline__ float to_f(T v);
template <>
__device__ __forceinline__ float to_f<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }

template <typename T>
__device__ __forceinline__ T from_f(float v);
template <>
__device__ __forceinline__ float from_f<float>(float v) { return v; }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }

// One warp per row; each lane holds up to kMaxVec groups of 8 elements.
template <typename TI, typename TO, int kMaxVec>
__global__ void __launch_bounds__(256)
    ln_warp_kernel(const TI* __restrict__ x, const float* __restrict__ gamma,
                   const float* __restrict__ beta, TO* __restrict__ y, float* __restrict__ mean_out,
                   float* __restrict__ rstd_out, int rows, int d, float eps) {
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  pdl_wait();  // x comes from the previous kernel
  pdl_trigger();
  if (row >= rows) return;
  const int nvec = d >> 3;
  const TI* xr = x + static_cast<size_t>(row) * d;
  float v[kMaxVec][8];
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < kMaxVec; ++i) {
    const int c = lane + i * 32;
    if (c < nvec) {
      Vec8<TI>::load(xr + c * 8, v[i]);
#pragma unroll
      for (int e = 0; e < 8; ++e) s += v[i][e];
    }
  }
  const float mu = warp_sum(s) / static_cast<float>(d);
  float q = 0.f;
#pragma unroll
  for (int i = 0; i < kMaxVec; ++i) {
    const int c = lane + i * 32;
    if (c < nvec) {
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float t = v[i][e] - mu;
        q += t * t;
      }
    }
  }
  const float rs = rsqrtf(warp_sum(q) / static_cast<float>(d) + eps);
  TO* yr = y + static_cast<size_t>(row) * d;
#pragma unroll
  for (int i = 0; i < kMaxVec; ++i) {
    const int c = lane + i * 32;
    if (c < nvec) {
      float g[8], b[8], o[8];
      if (gamma) Vec8<float>::load(gamma + c * 8, g);
      else {
#pragma unroll
        for (int e = 0; e < 8; ++e) g[e] = 1.f;
      }
      if (beta) Vec8<float>::load(beta + c * 8, b);
      else {
#pragma unroll
        for (int e = 0; e < 8; ++e) b[e] = 0.f;
      }
#pragma unroll
      for (int e = 0; e < 8; ++e) o[e] = (v[i][e] - mu) * rs * g[e] + b[e];
      Vec8<TO>::store(yr + c * 8, o);
    }
  }
  if (lane == 0) {
    if (mean_out) mean_out[row] = mu;
    if (rstd_out) rstd_out[row] = rs;
  }
}

// Generic path: one block per row, row staged in shared memory (fp32).
template <typename TI, typename TO>
__global__ void __launch_bounds__(256)
    ln_block_kernel(const TI* __restrict__ x, const float* __restrict__ gamma,
                    const float* __restrict__ beta, TO* __restrict__ y,
                    float* __restrict__ mean_out, float* __restrict__ rstd_out, int rows, int d,
                    float eps) {
  extern __shared__ float srow[];
  __shared__ float red[32];
  const int row = blockIdx.x;
  const TI* xr = x + static_cast<size_t>(row) * d;
  float s = 0.f;
  for (int j = threadIdx.x; j < d; j += blockDim.x) {
    const float t = to_f<TI>(xr[j]);
    srow[j] = t;
    s += t;
  }
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  s = warp_sum(s);
  if (lane == 0) red[w] = s;
  __syncthreads();
  s = (lane < nw) ? red[lane] : 0.f;
  if (w == 0) s = warp_sum(s);
  __syncthreads();
  if (threadIdx.x == 0) red[0] = s;
  __syncthreads();
  const float mu = red[0] / static_cast<float>(d);
  __syncthreads();
  float q = 0.f;
  for (int j = threadIdx.x; j < d; j += blockDim.x) {
    const float t = srow[j] - mu;
    q += t * t;
  }
  q = warp_sum(q);
  if (lane == 0) red[w] = q;
  __syncthreads();
  q = (lane < nw) ? red[lane] : 0.f;
  if (w == 0) q = warp_sum(q);
  __syncthreads();
  if (threadIdx.x == 0) red[0] = q;
  __syncthreads();
  const float rs = rsqrtf(red[0] / static_cast<float>(d) + eps);
  TO* yr = y + static_cast<size_t>(row) * d;
  for (int j = threadIdx.x; j < d; j += blockDim.x) {
    const float g = gamma ? gamma[j] : 1.f;
    const float b = beta ? beta[j] : 0.f;
    yr[j] = from_f<TO>((srow[j] - mu) * rs * g + b);
  }
  if (threadIdx.x == 0) {
    if (mean_out) mean_out[row] = mu;
    if (rstd_out) rstd_out[row] = rs;
  }
}

template <typename TI, typename TO>
cudaError_t launch_typed(cudaStream_t stream, const void* x, const float* gamma,
                         const float* beta, void* y, float* mean, float* rstd, int rows, int d,
                         float eps, bool vec_ok) {
  const TI* xi = static_cast<const TI*>(x);
  TO* yo = static_cast<TO*>(y);
  if (vec_ok && d <= 2048) {
    const int rows_per_block = 8;
    const int grid = (rows + rows_per_block - 1) / rows_per_block;
    const int nvec = d / 8;
    if (nvec <= 32)
      return launch_ex(ln_warp_kernel<TI, TO, 1>, grid, dim3(256), 0, stream, 1, true, xi, gamma, beta, yo, mean, rstd, rows, d, eps);
    else if (nvec <= 64)
      return launch_ex(ln_warp_kernel<TI, TO, 2>, grid, dim3(256), 0, stream, 1, true, xi, gamma, beta, yo, mean, rstd, rows, d, eps);
    else if (nvec <= 128)
      return launch_ex(ln_warp_kernel<TI, TO, 4>, grid, dim3(256), 0, stream, 1, true, xi, gamma, beta, yo, mean, rstd, rows, d, eps);
    else
      return launch_ex(ln_warp_kernel<TI, TO, 8>, grid, dim3(256), 0, stream, 1, true, xi, gamma, beta, yo, mean, rstd, rows, d, eps);
  } else {
    const size_t smem = static_cast<size_t>(d) * sizeof(float);
    if (smem > 48 * 1024) {
      cudaError_t e = cudaFuncSetAttribute(ln_block_kernel<TI, TO>,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           static_cast<int>(smem));
      if (e != cudaSuccess) return e;
    }
    ln_block_kernel<TI, TO><<<rows, 256, smem, stream>>>(xi, gamma, beta, yo, mean, rstd, rows, d, eps);
  }
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_layernorm(cudaStream_t stream, const void* x, bool x_bf16, const float* gamma,
                             const float* beta, void* y, bool y_bf16, float* mean, float* rstd,
                             int rows, int d, float eps, bool vec_ok) {
  if (rows == 0) return cudaSuccess;
  if (!x_bf16 && !y_bf16)
    return launch_typed<float, float>(stream, x, gamma, beta, y, mean, rstd, rows, d, eps, vec_ok);
  if (!x_bf16 && y_bf16)
    return launch_typed<float, __nv_bfloat16>(stream, x, gamma, beta, y, mean, rstd, rows, d, eps, vec_ok);
  if (x_bf16 && !y_bf16)
    return launch_typed<__nv_bfloat16, float>(stream, x, gamma, beta, y, mean, rstd, rows, d, eps, vec_ok);
  return launch_typed<__nv_bfloat16, __nv_bfloat16>(stream, x, gamma, beta, y, mean, rstd, rows, d, eps, vec_ok);
}

}  // namespace nd
