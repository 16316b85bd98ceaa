// model_ops.cu — the small device ops around the attention / GEMM kernels
// that a whole decoder needs on the GPU:
//
//   embed_kernel     y[t] = wte[ids[t]] + wpe[pos[t]]       (:embedding,
//                    src/dispatch.jl:476-491, plus the learned-position add)
//   argmax_kernel    greedy next token of each logits row    (the LM head's
//                    argmax; the first index of the maximum, like Julia's argmax)
//   kv_store_kernel  K/V rows of a prefill's QKV projection into the
//                    head-major decode caches [B][H][L_max][64]
//   add_ln_kernel    s = x + p (+ bias);  y = LayerNorm(s)   (the residual :add,
//                    dispatch.jl:386-417, fused with the next LayerNorm; used
//                    after a tensor-parallel all-reduce)
//
// All are HBM-bound and move 16-byte pieces where the layout allows.
#include <cuda_bf16.h>
#include <stdint.h>

#include "launch.cuh"
#include "model_ops.h"
#include "ptx.cuh"

namespace nd {
namespace {

__device__ __forceinline__ void bf16x8_to_f32(const uint4& u, float (&f)[8]) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(w[i] << 16);
    f[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
  }
}
__device__ __forceinline__ uint4 f32_to_bf16x8(const float (&f)[8]) {
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __nv_bfloat162 h = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
    w[i] = *reinterpret_cast<uint32_t*>(&h);
  }
  return make_uint4(w[0], w[1], w[2], w[3]);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// ---------------------------------------------------------------- embedding
// One warp per token; d % 8 == 0.  Ids or positions outside their tables
// raise the error word and produce a zero row (no out-of-range read).
__global__ void __launch_bounds__(256)
    embed_kernel(const int* __restrict__ ids, const int* __restrict__ pos,
                 const __nv_bfloat16* __restrict__ wte, const __nv_bfloat16* __restrict__ wpe,
                 __nv_bfloat16* __restrict__ y, int T, int d, int vocab, int n_pos,
                 int* __restrict__ err_word) {
  const int t = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  pdl_wait();  // the ids may come from the previous kernel (a greedy pick)
  pdl_trigger();
  if (t >= T) return;
  const int id = ids[t];
  const int p = pos ? pos[t] : -1;
  const bool id_ok = id >= 0 && id < vocab;
  const bool pos_ok = pos == nullptr || (p >= 0 && p < n_pos);
  if ((!id_ok || !pos_ok) && lane == 0 && err_word) atomicCAS(err_word, 0, kModelErrIndex);
  uint4* yr = reinterpret_cast<uint4*>(y + static_cast<size_t>(t) * d);
  const uint4* er = reinterpret_cast<const uint4*>(wte + static_cast<size_t>(id_ok ? id : 0) * d);
  const uint4* pr = (pos && pos_ok) ? reinterpret_cast<const uint4*>(wpe + static_cast<size_t>(p) * d)
                                    : nullptr;
  for (int c = lane; c < d / 8; c += 32) {
    float a[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    if (id_ok) bf16x8_to_f32(er[c], a);
    if (pr) {
      float b[8];
      bf16x8_to_f32(pr[c], b);
#pragma unroll
      for (int e = 0; e < 8; ++e) a[e] += b[e];
    }
    yr[c] = f32_to_bf16x8(a);
  }
}

// ------------------------------------------------------------------ argmax
// One block per row: the largest value and its first index.  NaN is never
// chosen over a number (a row of NaNs gives index 0).
template <typename T>
__device__ __forceinline__ float ld_f(const T* p);
template <>
__device__ __forceinline__ float ld_f<float>(const float* p) { return *p; }
template <>
__device__ __forceinline__ float ld_f<__nv_bfloat16>(const __nv_bfloat16* p) {
  return __bfloat162float(*p);
}

// (v2, i2) replaces (v, i) if larger, equal with a smaller index, or a
// number where v is NaN.
__device__ __forceinline__ void better(float& v, int& i, float v2, int i2) {
  if (v2 > v || (v2 == v && i2 < i) || (v != v && v2 == v2)) {
    v = v2;
    i = i2;
  }
}

constexpr int kArgmaxThreads = 512;
constexpr int kArgmaxUnroll = 8;    // independent loads in flight per thread
constexpr int kArgmaxCluster = 8;   // CTAs per row for long rows

// A cluster of CTAs per row (one CTA for short rows): CTA rank r scans a
// contiguous 1/cluster of the row, then rank 0 merges the CTAs' results from
// distributed shared memory.  The merge keeps the first index among equal
// maxima whatever the order, so the result is that of one sequential scan.
template <typename T>
__global__ void __launch_bounds__(kArgmaxThreads)
    argmax_kernel(const T* __restrict__ logits, long long ld, int V, int* __restrict__ idx,
                  float* __restrict__ val) {
  const int nc = static_cast<int>(cluster_nctarank());
  const int cr = static_cast<int>(cluster_ctarank());
  const int row = blockIdx.x / nc;
  const int per = (V + nc - 1) / nc;
  const int j_beg = cr * per;
  const int j_end = min(V, j_beg + per);
  pdl_wait();  // the logits come from the previous kernel
  pdl_trigger();
  const T* r = logits + static_cast<size_t>(row) * ld;
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  for (int j0 = j_beg + threadIdx.x; j0 < j_end; j0 += kArgmaxThreads * kArgmaxUnroll) {
    float v[kArgmaxUnroll];
#pragma unroll
    for (int u = 0; u < kArgmaxUnroll; ++u) {
      const int j = j0 + u * kArgmaxThreads;
      v[u] = j < j_end ? ld_f<T>(r + j) : -INFINITY;
    }
#pragma unroll
    for (int u = 0; u < kArgmaxUnroll; ++u)
      if (j0 + u * kArgmaxThreads < j_end) better(bv, bi, v[u], j0 + u * kArgmaxThreads);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float v2 = __shfl_xor_sync(0xffffffffu, bv, o);
    const int i2 = __shfl_xor_sync(0xffffffffu, bi, o);
    better(bv, bi, v2, i2);
  }
  __shared__ float sv[kArgmaxThreads / 32];
  __shared__ int si[kArgmaxThreads / 32];
  __shared__ float cv;
  __shared__ int ci;
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  if (lane == 0) {
    sv[w] = bv;
    si[w] = bi;
  }
  __syncthreads();
  if (w == 0) {
    bv = lane < nw ? sv[lane] : -INFINITY;
    bi = lane < nw ? si[lane] : 0x7fffffff;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float v2 = __shfl_xor_sync(0xffffffffu, bv, o);
      const int i2 = __shfl_xor_sync(0xffffffffu, bi, o);
      better(bv, bi, v2, i2);
    }
    if (lane == 0) {
      cv = bv;
      ci = bi;
    }
  }
  // every CTA of the cluster reaches both barriers (no early exit above)
  if (nc > 1) cluster_sync();
  if (cr == 0 && threadIdx.x == 0) {
    float v = cv;
    int i = ci;
    for (int q = 1; q < nc; ++q) {
      const float v2 = ld_dsmem_f32(&cv, static_cast<uint32_t>(q));
      const int i2 = __float_as_int(ld_dsmem_f32(&ci, static_cast<uint32_t>(q)));
      better(v, i, v2, i2);
    }
    idx[row] = i == 0x7fffffff ? 0 : i;
    if (val) val[row] = v;
  }
  if (nc > 1) cluster_sync();  // rank 0 has read every CTA's result
}

// ---------------------------------------------------------------- KV store
// Thread = 16 bytes of one (batch, position, head) row: the K and V rows of
// token (b, s) at columns k_col / v_col of a [B·S][ld] projection go to
// position pos0 + s of the caches [B][H][L_max][64].
__global__ void kv_store_kernel(const __nv_bfloat16* __restrict__ src, long long ld, int k_col,
                                int v_col, __nv_bfloat16* __restrict__ k_cache,
                                __nv_bfloat16* __restrict__ v_cache, int B, int S, int H,
                                int L_max, int pos0) {
  const long long n = static_cast<long long>(B) * S * H * 8;
  const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const int c = static_cast<int>(i & 7);
  const long long r = i >> 3;  // (b, s, h)
  const int h = static_cast<int>(r % H);
  const long long bs = r / H;
  const int s = static_cast<int>(bs % S);
  const int b = static_cast<int>(bs / S);
  const __nv_bfloat16* row = src + bs * ld;
  const size_t dst = ((static_cast<size_t>(b) * H + h) * L_max + pos0 + s) * 64;
  reinterpret_cast<uint4*>(k_cache + dst)[c] = reinterpret_cast<const uint4*>(row + k_col + h * 64)[c];
  reinterpret_cast<uint4*>(v_cache + dst)[c] = reinterpret_cast<const uint4*>(row + v_col + h * 64)[c];
}

// ------------------------------------------------------- residual + LayerNorm
// One warp per row, the row in registers (d <= 2048, d % 8 == 0).
// s = x + p (+ bias) is rounded to bf16 and written to s_out (which may be x
// itself: every thread reads its 16-byte pieces of x before writing them),
// and y = (s - mean) * rstd * gamma + beta over the stored s.  All of a row's
// x and p loads are issued before any arithmetic or store; with kVecParams
// (bias, gamma and beta 16-byte aligned) the parameters are read as float4.
template <bool kVecParams>
__device__ __forceinline__ void ld_param8(const float* __restrict__ v, int c, float dflt,
                                          float (&o)[8]) {
  if (v == nullptr) {
#pragma unroll
    for (int e = 0; e < 8; ++e) o[e] = dflt;
  } else if constexpr (kVecParams) {
    const float4 a = __ldg(reinterpret_cast<const float4*>(v) + 2 * c);
    const float4 b = __ldg(reinterpret_cast<const float4*>(v) + 2 * c + 1);
    o[0] = a.x; o[1] = a.y; o[2] = a.z; o[3] = a.w;
    o[4] = b.x; o[5] = b.y; o[6] = b.z; o[7] = b.w;
  } else {
#pragma unroll
    for (int e = 0; e < 8; ++e) o[e] = __ldg(v + c * 8 + e);
  }
}

template <typename TP, int kMaxVec, bool kVecParams>
__global__ void __launch_bounds__(256)
    add_ln_kernel(const __nv_bfloat16* x, const TP* __restrict__ p,
                  const float* __restrict__ bias, const float* __restrict__ gamma,
                  const float* __restrict__ beta, __nv_bfloat16* s_out,
                  __nv_bfloat16* __restrict__ y, int rows, int d, float eps) {
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  pdl_wait();  // x and p come from earlier kernels
  pdl_trigger();
  if (row >= rows) return;
  const int nvec = d >> 3;
  const size_t off = static_cast<size_t>(row) * d;
  constexpr int kPV = sizeof(TP) == 4 ? 2 : 1;   // 16-byte pieces of p per 8 values
  uint4 xr[kMaxVec], pr[kMaxVec][kPV];
#pragma unroll
  for (int i = 0; i < kMaxVec; ++i) {
    const int c = lane + i * 32;
    if (c < nvec) {
      xr[i] = reinterpret_cast<const uint4*>(x + off)[c];
#pragma unroll
      for (int k = 0; k < kPV; ++k) pr[i][k] = reinterpret_cast<const uint4*>(p + off)[kPV * c + k];
    }
  }
  float v[kMaxVec][8];
  float sum = 0.f;
#pragma unroll
  for (int i = 0; i < kMaxVec; ++i) {
    const int c = lane + i * 32;
    if (c < nvec) {
      bf16x8_to_f32(xr[i], v[i]);
      float q[8], bs[8];
      if constexpr (sizeof(TP) == 4) {
        const uint32_t w[8] = {pr[i][0].x, pr[i][0].y, pr[i][0].z, pr[i][0].w,
                               pr[i][1].x, pr[i][1].y, pr[i][1].z, pr[i][1].w};
#pragma unroll
        for (int e = 0; e < 8; ++e) q[e] = __uint_as_float(w[e]);
      } else {
        bf16x8_to_f32(pr[i][0], q);
      }
      ld_param8<kVecParams>(bias, c, 0.f, bs);
#pragma unroll
      for (int e = 0; e < 8; ++e) v[i][e] += q[e] + bs[e];
      const uint4 packed = f32_to_bf16x8(v[i]);
      bf16x8_to_f32(packed, v[i]);
      reinterpret_cast<uint4*>(s_out + off)[c] = packed;
#pragma unroll
      for (int e = 0; e < 8; ++e) sum += v[i][e];
    }
  }
  const float mu = warp_sum(sum) / static_cast<float>(d);
  float q2 = 0.f;
#pragma unroll
  for (int i = 0; i < kMaxVec; ++i) {
    if (lane + i * 32 < nvec) {
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float t = v[i][e] - mu;
        q2 += t * t;
      }
    }
  }
  const float rs = rsqrtf(warp_sum(q2) / static_cast<float>(d) + eps);
#pragma unroll
  for (int i = 0; i < kMaxVec; ++i) {
    const int c = lane + i * 32;
    if (c < nvec) {
      float g[8], b[8], o[8];
      ld_param8<kVecParams>(gamma, c, 1.f, g);
      ld_param8<kVecParams>(beta, c, 0.f, b);
#pragma unroll
      for (int e = 0; e < 8; ++e) o[e] = (v[i][e] - mu) * rs * g[e] + b[e];
      reinterpret_cast<uint4*>(y + off)[c] = f32_to_bf16x8(o);
    }
  }
}

template <typename TP, bool kVec>
cudaError_t launch_add_ln_vec(cudaStream_t stream, const __nv_bfloat16* x, const TP* pp,
                              const float* bias, const float* gamma, const float* beta,
                              __nv_bfloat16* s_out, __nv_bfloat16* y, int rows, int d, float eps) {
  const dim3 grid((rows + 7) / 8), block(256);
  if (d <= 256)
    return launch_ex(add_ln_kernel<TP, 1, kVec>, grid, block, 0, stream, 1, true, x, pp, bias, gamma, beta, s_out, y, rows, d, eps);
  if (d <= 512)
    return launch_ex(add_ln_kernel<TP, 2, kVec>, grid, block, 0, stream, 1, true, x, pp, bias, gamma, beta, s_out, y, rows, d, eps);
  if (d <= 1024)
    return launch_ex(add_ln_kernel<TP, 4, kVec>, grid, block, 0, stream, 1, true, x, pp, bias, gamma, beta, s_out, y, rows, d, eps);
  return launch_ex(add_ln_kernel<TP, 8, kVec>, grid, block, 0, stream, 1, true, x, pp, bias, gamma, beta, s_out, y, rows, d, eps);
}

template <typename TP>
cudaError_t launch_add_ln_typed(cudaStream_t stream, const __nv_bfloat16* x, const void* p,
                                const float* bias, const float* gamma, const float* beta,
                                __nv_bfloat16* s_out, __nv_bfloat16* y, int rows, int d,
                                float eps) {
  const TP* pp = static_cast<const TP*>(p);
  const bool vec = ((reinterpret_cast<uintptr_t>(bias) | reinterpret_cast<uintptr_t>(gamma) |
                     reinterpret_cast<uintptr_t>(beta)) & 15u) == 0;
  return vec ? launch_add_ln_vec<TP, true>(stream, x, pp, bias, gamma, beta, s_out, y, rows, d, eps)
             : launch_add_ln_vec<TP, false>(stream, x, pp, bias, gamma, beta, s_out, y, rows, d, eps);
}

}  // namespace

cudaError_t launch_embed(cudaStream_t stream, const int* ids, const int* pos,
                         const __nv_bfloat16* wte, const __nv_bfloat16* wpe, __nv_bfloat16* y,
                         int T, int d, int vocab, int n_pos, int* err_word) {
  if (T == 0) return cudaSuccess;
  return launch_ex(embed_kernel, dim3((T + 7) / 8), dim3(256), 0, stream, 1, true, ids, pos, wte,
                   wpe, y, T, d, vocab, n_pos, err_word);
}

cudaError_t launch_argmax(cudaStream_t stream, const void* logits, bool f32, long long ld,
                          int rows, int V, int* idx, float* val) {
  if (rows == 0) return cudaSuccess;
  // a few long rows (a decode batch's logits) spread over a cluster each
  const int nc = (V >= 2 * kArgmaxCluster * kArgmaxThreads && rows < 148) ? kArgmaxCluster : 1;
  const dim3 grid(static_cast<unsigned>(rows) * nc), block(kArgmaxThreads);
  if (f32)
    return launch_ex(argmax_kernel<float>, grid, block, 0, stream, nc, true,
                     static_cast<const float*>(logits), ld, V, idx, val);
  return launch_ex(argmax_kernel<__nv_bfloat16>, grid, block, 0, stream, nc, true,
                   static_cast<const __nv_bfloat16*>(logits), ld, V, idx, val);
}

cudaError_t launch_kv_store(cudaStream_t stream, const __nv_bfloat16* src, long long ld, int k_col,
                            int v_col, __nv_bfloat16* k_cache, __nv_bfloat16* v_cache, int B,
                            int S, int H, int L_max, int pos0) {
  const long long n = static_cast<long long>(B) * S * H * 8;
  if (n == 0) return cudaSuccess;
  kv_store_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, stream>>>(
      src, ld, k_col, v_col, k_cache, v_cache, B, S, H, L_max, pos0);
  return cudaGetLastError();
}

cudaError_t launch_add_layernorm(cudaStream_t stream, const __nv_bfloat16* x, const void* p,
                                 bool p_f32, const float* bias, const float* gamma,
                                 const float* beta, __nv_bfloat16* s_out, __nv_bfloat16* y,
                                 int rows, int d, float eps) {
  if (rows == 0) return cudaSuccess;
  return p_f32 ? launch_add_ln_typed<float>(stream, x, p, bias, gamma, beta, s_out, y, rows, d, eps)
               : launch_add_ln_typed<__nv_bfloat16>(stream, x, p, bias, gamma, beta, s_out, y, rows,
                                                    d, eps);
}

}  // namespace nd
