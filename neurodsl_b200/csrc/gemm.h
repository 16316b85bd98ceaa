// gemm.h — launcher for the tcgen05 GEMM with bias / GELU / residual epilogue.
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "../../include/neurodsl_b200.h"

namespace nd {

// Optional second destination of a QKV projection's K and V columns: row m
// (token s = m % S of sequence b = m / S) of columns [dl, 2·dl) and
// [2·dl, 3·dl) also goes to position pos0 + s of the head-major caches
// k, v [B][H][L_max][64] (head = column / 64 within its block).  Written by
// the bf16 staged epilogue of the tensor-core path only: the caller checks
// that the launch takes it (bf16 Y, no residual, 16-byte aligned Y and bias,
// N % 8 == 0, dl % 64 == 0, more than 32 rows).
// With n_peers > 0 the heads are split over n_peers ranks of H heads each:
// head h goes to rank q = h / H, whose caches (k_peer[q], v_peer[q], peer
// memory mapped into this process; this rank's own among them) hold it as
// head h - q·H at sequence b0 + b; dl is then n_peers·H·64 and k, v only mark
// the cache-writing launch.
constexpr int kKvMaxPeers = 8;
struct KvOut {
  __nv_bfloat16* k = nullptr;
  __nv_bfloat16* v = nullptr;
  int S = 0, H = 0, L_max = 0, pos0 = 0, dl = 0;
  int n_peers = 0, b0 = 0;
  __nv_bfloat16* k_peer[kKvMaxPeers] = {};
  __nv_bfloat16* v_peer[kKvMaxPeers] = {};
};

// Y[M][N] = act(A[M][K] · W[N][K]ᵀ + bias[N]) + residual[M][N]
// A, W bf16 with K % 8 == 0 and 16-byte aligned bases; bias fp32 or null;
// residual bf16 / fp32 or null; Y bf16 or fp32.  act is an ND_ACT_* code.
cudaError_t launch_gemm(cudaStream_t stream, const __nv_bfloat16* A, const __nv_bfloat16* W,
                        const float* bias, const void* residual, bool residual_f32, void* Y,
                        bool out_f32, int M, int N, int K, int act, const char** err_msg,
                        const KvOut& kv = KvOut());

// Few-row linear layer with the residual add and LayerNorm in its prologue:
//   s = bf16(x + (p + p_bias));  Y = act(LayerNorm(s; gamma, beta, eps) · Wᵀ + bias)
// x, p, s_out [M][K] bf16 (p, p_bias, gamma, beta, s_out, bias may be null;
// s_out, when given, receives s and must not overlap x or p); W [N][K] bf16;
// Y [M][N] bf16 or fp32.  M <= kLnGemmMaxRows, K % 32 == 0, K <= kLnGemmMaxK.
constexpr int kLnGemmMaxRows = 32;
constexpr int kLnGemmMaxK = 1024;
cudaError_t launch_ln_gemm(cudaStream_t stream, const __nv_bfloat16* x, const __nv_bfloat16* p,
                           const float* p_bias, const float* gamma, const float* beta, float eps,
                           __nv_bfloat16* s_out, const __nv_bfloat16* W, const float* bias,
                           void* Y, bool out_f32, int M, int N, int K, int act);

}  // namespace nd
