// skinny_core.cuh — the weight-streaming tile of the few-row linear layer
// (M <= 32 rows, decode steps), shared by the skinny GEMM (gemm.cu) and the
// tensor-parallel projection fused with its reduction (tp_comm.cu).
//
// A cluster of `ksplit` CTAs owns 8 rows of W; each CTA takes a contiguous
// 1/ksplit of the K range and its 8 warps split that.  Each lane reads 16
// bytes (8 k values) of one W row and of each A row per 32-wide k chunk and
// feeds two mma.m16n8k16 steps; the k values are assigned to fragment
// positions by the same permutation for A and W, which leaves every dot
// product intact.  The warps' 16x8 (or 32x8) partial tiles are summed through
// shared memory; the callers sum the cluster's tiles in rank order through
// distributed shared memory (so the result does not depend on timing).
#pragma once
#include <cuda_bf16.h>
#include <stdint.h>

#include "launch.cuh"
#include "ptx.cuh"

namespace nd {

// Tuning switch (compile-time): k chunks of 32 per warp whose loads are
// issued together; the split-K policy below sizes clusters so that one such
// batch covers a warp's share of K.
#ifndef ND_SKINNY_BATCH
#define ND_SKINNY_BATCH 4
#endif
constexpr int kSkinnyWarps = 8;
constexpr int kSkinnyBatch = ND_SKINNY_BATCH;  // k chunks whose loads are issued together
constexpr int kSkinnyMaxSplit = 8;

__device__ __forceinline__ void mma_bf16_16816(float (&c)[4], uint32_t a0, uint32_t a1,
                                               uint32_t a2, uint32_t a3, uint32_t b0,
                                               uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
      "{%8, %9}, {%0, %1, %2, %3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint4 ldg16_or_zero(const __nv_bfloat16* p, bool ok) {
  return ok ? __ldg(reinterpret_cast<const uint4*>(p)) : make_uint4(0, 0, 0, 0);
}

// K split across a cluster: enough CTAs that each warp's share of K is one
// batch of loads, at most kSkinnyMaxSplit, and no more than two CTAs per SM
// in total — two are resident per SM at the kernel's register use, and a
// second wave of CTAs costs more than a second batch of loads per warp (the
// 32-row 1024 x 4096 projection: 9.9 us in two waves of 512 CTAs, 6.9 us in
// one wave of 256).  The skinny GEMM and the fused tensor-parallel projection
// share the rule, so they split K alike and give the same bits.
inline int skinny_ksplit(int N, int K, int sms) {
  const int n_chunks = K / 32;
  const int nblk = (N + 7) / 8;
  int ks = (n_chunks + kSkinnyWarps * kSkinnyBatch - 1) / (kSkinnyWarps * kSkinnyBatch);
  if (ks > kSkinnyMaxSplit) ks = kSkinnyMaxSplit;
  if (nblk * ks > 2 * sms) ks = (2 * sms) / nblk;
  if (ks < 1) ks = 1;
  return ks;
}

// This CTA's share of the [kMB·16][8] tile A[M][K] · W[n0..n0+8)[K]ᵀ, the k
// chunks of cluster rank kr of ksplit, summed over the CTA's warps into
// part[] (row-major [kMB·16][8]; rows >= M are zero).  The first batch of W
// loads goes out before pdl_wait() (W is a constant operand), A after it;
// with trigger_early the dependent kernel is released right after the wait.
// Every thread of the CTA must call it (it contains a CTA barrier).
template <int kMB>
__device__ __forceinline__ void skinny_tile(const __nv_bfloat16* __restrict__ A,
                                            const __nv_bfloat16* __restrict__ W, int M, int N,
                                            int K, int n0, int ksplit, int kr,
                                            float (*red)[kMB * 16][8], float* part,
                                            bool trigger_early) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;  // fragment group (row / column) and slot
  const bool w_ok = n0 + g < N;
  const __nv_bfloat16* wrow = W + static_cast<size_t>(w_ok ? n0 + g : 0) * K + t * 8;
  const int n_chunks = K / 32;
  const int per = (n_chunks + ksplit - 1) / ksplit;
  const int cbeg = kr * per;
  const int cend = min(n_chunks, cbeg + per);
  constexpr int kStep = kSkinnyWarps * kSkinnyBatch;

  uint4 wv[kSkinnyBatch];
#pragma unroll
  for (int u = 0; u < kSkinnyBatch; ++u) {
    const int ch = cbeg + warp + u * kSkinnyWarps;
    wv[u] = ldg16_or_zero(wrow + ch * 32, ch < cend && w_ok);
  }
  pdl_wait();
  if (trigger_early) pdl_trigger();

  const __nv_bfloat16* arow[kMB][2];
  bool a_ok[kMB][2];
#pragma unroll
  for (int mb = 0; mb < kMB; ++mb)
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int m = mb * 16 + h * 8 + g;
      a_ok[mb][h] = m < M;
      arow[mb][h] = A + static_cast<size_t>(a_ok[mb][h] ? m : 0) * K + t * 8;
    }
  float c[kMB][4];
#pragma unroll
  for (int mb = 0; mb < kMB; ++mb)
#pragma unroll
    for (int i = 0; i < 4; ++i) c[mb][i] = 0.f;
  for (int c0 = cbeg + warp; c0 < cend; c0 += kStep) {
    uint4 av[kSkinnyBatch][kMB][2];
#pragma unroll
    for (int u = 0; u < kSkinnyBatch; ++u) {
      const int ch = c0 + u * kSkinnyWarps;
      const bool in = ch < cend;
      if (c0 != cbeg + warp) wv[u] = ldg16_or_zero(wrow + ch * 32, in && w_ok);
#pragma unroll
      for (int mb = 0; mb < kMB; ++mb)
#pragma unroll
        for (int h = 0; h < 2; ++h) av[u][mb][h] = ldg16_or_zero(arow[mb][h] + ch * 32, in && a_ok[mb][h]);
    }
#pragma unroll
    for (int u = 0; u < kSkinnyBatch; ++u) {
      const uint32_t w[4] = {wv[u].x, wv[u].y, wv[u].z, wv[u].w};
#pragma unroll
      for (int mb = 0; mb < kMB; ++mb) {
        const uint32_t lo[4] = {av[u][mb][0].x, av[u][mb][0].y, av[u][mb][0].z, av[u][mb][0].w};
        const uint32_t hi[4] = {av[u][mb][1].x, av[u][mb][1].y, av[u][mb][1].z, av[u][mb][1].w};
#pragma unroll
        for (int s = 0; s < 2; ++s)
          mma_bf16_16816(c[mb], lo[2 * s], hi[2 * s], lo[2 * s + 1], hi[2 * s + 1], w[2 * s],
                         w[2 * s + 1]);
      }
    }
  }
  // sum the warps' partial tiles: red[warp][m][n] for the 16·kMB x 8 tile
#pragma unroll
  for (int mb = 0; mb < kMB; ++mb) {
    red[warp][mb * 16 + g][2 * t] = c[mb][0];
    red[warp][mb * 16 + g][2 * t + 1] = c[mb][1];
    red[warp][mb * 16 + g + 8][2 * t] = c[mb][2];
    red[warp][mb * 16 + g + 8][2 * t + 1] = c[mb][3];
  }
  __syncthreads();
  for (int o = threadIdx.x; o < kMB * 16 * 8; o += blockDim.x) {
    float z = 0.f;
#pragma unroll
    for (int w = 0; w < kSkinnyWarps; ++w) z += red[w][o >> 3][o & 7];
    part[o] = z;
  }
}

}  // namespace nd
