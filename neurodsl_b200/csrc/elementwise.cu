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
//   gather_rows_kernel the :embedding op (src/dispatch.jl:476-491): table
//                      rows picked by (1-based) indices, on the device
//   copy_2d_kernel     the :slice_cols, :hcat_heads and :identity copies
//                      (src/dispatch.jl:544-553, :349-361) between strided
//                      2-D views
// fp32 rows in and out (the graph's Float32 node values).  HBM-bound; a warp
// per row for the softmax with 16-byte loads where the row allows.
#include <cuda_bf16.h>
#include <math.h>
#include <stdint.h>

#include <type_traits>

#include "elementwise.h"
#include "model_ops.h"

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

// One block per output row: out[i] = table[idx[i] - base], element bits
// copied as T (uint32_t for fp32, uint16_t for bf16).  An index outside the
// table, or a Float32 index that is not an integer, gives a zero row and sets
// the device error word (the reference's Julia indexing would throw).
template <typename T, typename I>
__global__ void __launch_bounds__(128)
    gather_rows_kernel(const T* __restrict__ table, long long ld_table, int vocab,
                       const I* __restrict__ idx, int base, int n, int d, T* __restrict__ out,
                       long long ld_out, int* __restrict__ err_word) {
  const int i = blockIdx.x;
  if (i >= n) return;
  long long row = 0;
  bool ok;
  if constexpr (std::is_same<I, float>::value) {
    const float r = idx[i];
    ok = r == floorf(r) && r >= static_cast<float>(base) &&
         r < static_cast<float>(base) + static_cast<float>(vocab);
    if (ok) row = static_cast<long long>(r) - base;
  } else {
    row = static_cast<long long>(idx[i]) - base;
    ok = row >= 0 && row < vocab;
  }
  if (!ok) {
    row = 0;
    if (threadIdx.x == 0 && err_word != nullptr) atomicCAS(err_word, 0, kModelErrIndex);
  }
  const T* src = table + row * ld_table;
  T* dst = out + static_cast<long long>(i) * ld_out;
  for (int c = threadIdx.x; c < d; c += blockDim.x) dst[c] = ok ? src[c] : T(0);
}

// dst[b][r][c] = src[b][r][c] in units of U (16, 4 or 2 bytes), row and batch
// strides in units; batch b = blockIdx.y.
template <typename U>
__global__ void copy_2d_kernel(const U* __restrict__ src, long long ld_src, long long bs_src,
                               U* __restrict__ dst, long long ld_dst, long long bs_dst, int rows,
                               long long units) {
  const long long n = static_cast<long long>(rows) * units;
  src += blockIdx.y * bs_src;
  dst += blockIdx.y * bs_dst;
  for (long long k = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; k < n;
       k += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long r = k / units, c = k - r * units;
    dst[r * ld_dst + c] = src[r * ld_src + c];
  }
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

cudaError_t launch_gather_rows(cudaStream_t stream, const void* table, int elem_bytes,
                               long long ld_table, int vocab, const void* idx, int idx_kind,
                               int base, int n, int d, void* out, long long ld_out, int* err_word) {
  if (n == 0 || d == 0) return cudaSuccess;
#define ND_GATHER(T, I)                                                                         \
  gather_rows_kernel<T, I><<<n, 128, 0, stream>>>(static_cast<const T*>(table), ld_table, vocab, \
                                                  static_cast<const I*>(idx), base, n, d,        \
                                                  static_cast<T*>(out), ld_out, err_word)
  if (elem_bytes == 4) {
    if (idx_kind == 0) ND_GATHER(uint32_t, float);
    else if (idx_kind == 1) ND_GATHER(uint32_t, int32_t);
    else ND_GATHER(uint32_t, long long);
  } else {
    if (idx_kind == 0) ND_GATHER(uint16_t, float);
    else if (idx_kind == 1) ND_GATHER(uint16_t, int32_t);
    else ND_GATHER(uint16_t, long long);
  }
#undef ND_GATHER
  return cudaGetLastError();
}

cudaError_t launch_copy_2d(cudaStream_t stream, const void* src, long long ld_src, void* dst,
                           long long ld_dst, int rows, int cols, int elem_bytes, int batch,
                           long long bs_src, long long bs_dst) {
  const long long row_bytes = static_cast<long long>(cols) * elem_bytes;
  if (rows == 0 || row_bytes == 0 || batch == 0) return cudaSuccess;
  const long long sb = ld_src * elem_bytes, db = ld_dst * elem_bytes;
  const long long bsb = bs_src * elem_bytes, bdb = bs_dst * elem_bytes;
  const uintptr_t align = reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst) |
                          static_cast<uintptr_t>(sb) | static_cast<uintptr_t>(db) |
                          static_cast<uintptr_t>(bsb) | static_cast<uintptr_t>(bdb) |
                          static_cast<uintptr_t>(row_bytes);
  // the widest unit that divides both addresses, all strides and a row
  const int unit = (align % 16 == 0) ? 16 : (align % 4 == 0) ? 4 : 2;
  const long long units = row_bytes / unit;
  int gx = grid_for(static_cast<long long>(rows) * units, 256);
  const int cap = (148 * 32 + batch - 1) / batch;  // about the same CTAs in total
  if (gx > cap) gx = cap;
  const dim3 grid(gx, batch);
  if (unit == 16)
    copy_2d_kernel<uint4><<<grid, 256, 0, stream>>>(static_cast<const uint4*>(src), sb / 16, bsb / 16,
                                                   static_cast<uint4*>(dst), db / 16, bdb / 16, rows,
                                                   units);
  else if (unit == 4)
    copy_2d_kernel<uint32_t><<<grid, 256, 0, stream>>>(static_cast<const uint32_t*>(src), sb / 4,
                                                      bsb / 4, static_cast<uint32_t*>(dst), db / 4,
                                                      bdb / 4, rows, units);
  else
    copy_2d_kernel<uint16_t><<<grid, 256, 0, stream>>>(static_cast<const uint16_t*>(src), sb / 2,
                                                      bsb / 2, static_cast<uint16_t*>(dst), db / 2,
                                                      bdb / 2, rows, units);
  return cudaGetLastError();
}

cudaError_t launch_softmax(cudaStream_t stream, const float* x, float* y, int rows, int cols) {
  if (rows == 0 || cols == 0) return cudaSuccess;
  softmax_kernel<<<(rows + 7) / 8, 256, 0, stream>>>(x, y, rows, cols);
  return cudaGetLastError();
}

}  // namespace nd
