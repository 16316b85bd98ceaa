// gemm.cu — Y = act(A·Wᵀ + bias) + residual on tcgen05 + TMEM + TMA.
//
// The :linear rule (src/dispatch.jl:363-384: mul!(out, X, W') then
// out .+= b'), :fused_matmul_add (:281-296), the notebook's fused_linear_gelu
// (notebook/compiler.ipynb cell 15: z·σ(1.702 z)) and the residual :add
// (:386-417) as one kernel: the bias, the GELU and the residual are applied
// in the epilogue while the fp32 accumulator is read out of tensor memory.
//
// A [M][K] and W [N][K] are bf16, K contiguous (W is the (out, in) weight of
// a Linear layer).  Per CTA: a 128 x BN output tile, K consumed in blocks of
// 64 through a kStages-deep TMA ring.  Warp roles (256 threads): warp 0 TMA
// producer, warp 1 TMEM allocator + UMMA issuer, warps 4..7 epilogue (thread
// t owns accumulator row t = TMEM lane t).
#include <cuda.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "gemm.h"
#include "ptx.cuh"
#include "tma.h"

namespace nd {
namespace {

constexpr int kBM = 128;
constexpr int kBK = 64;
constexpr int kThreads = 256;
constexpr uint32_t kATileBytes = kBM * kBK * 2;  // 16 KB

template <int BN>
struct GemmCfg {
  static constexpr int kStages = BN >= 256 ? 4 : 6;
  static constexpr uint32_t kBTileBytes = BN * kBK * 2;
  static constexpr uint32_t kStageBytes = kATileBytes + kBTileBytes;
  static constexpr uint32_t kOffBar = kStages * kStageBytes;
  static constexpr uint32_t kSmemBytes = kOffBar + 256 + 1024;
  static constexpr uint32_t kTmemCols = BN;  // power of two (128 or 256)
  static constexpr uint32_t kIdesc = idesc_bf16_f32(kBM, BN, false, false);
};

template <int kStages>
struct GemmBars {
  uint64_t full[kStages];
  uint64_t empty[kStages];
  uint64_t acc_full;
  uint32_t tmem_base;
  int abort_flag;
};

__device__ __forceinline__ float apply_act(float z, int act) {
  switch (act) {
    case ND_ACT_GELU_SIGMOID: return z / (1.f + __expf(-1.702f * z));
    case ND_ACT_GELU_TANH: {
      const float u = 0.7978845608028654f * (z + 0.044715f * z * z * z);
      return 0.5f * z * (1.f + tanhf(u));
    }
    case ND_ACT_GELU_ERF: return 0.5f * z * (1.f + erff(z * 0.7071067811865476f));
    default: return z;
  }
}

template <int BN, bool kOutF32>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_w,
                const float* __restrict__ bias, const void* __restrict__ residual,
                int residual_f32, void* __restrict__ Y, int M, int N, int K, int act,
                int* __restrict__ err_word) {
  using Cfg = GemmCfg<BN>;
  constexpr int kStages = Cfg::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  auto* bars = reinterpret_cast<GemmBars<kStages>*>(smem + Cfg::kOffBar);
  volatile int* abort_flag = &bars->abort_flag;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int n_blk = blockIdx.x;
  const int m_blk = blockIdx.y;
  const int n_k = (K + kBK - 1) / kBK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&bars->full[s], 1);
      mbar_init(&bars->empty[s], 1);
    }
    mbar_init(&bars->acc_full, 1);
    bars->abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(&bars->tmem_base, Cfg::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;

  if (warp == 0) {
    if (elect_one()) {
      tma_prefetch_desc(&tm_a);
      tma_prefetch_desc(&tm_w);
      int issued = 0;
      for (int kb = 0; kb < n_k; ++kb) {
        const int s = kb % kStages;
        if (kb >= kStages) {
          if (!mbar_wait(&bars->empty[s], ((kb / kStages) - 1) & 1, abort_flag)) {
            raise_abort(abort_flag, err_word, kDevErrTimeoutProducer);
            break;
          }
        }
        uint8_t* st = smem + s * Cfg::kStageBytes;
        mbar_arrive_expect_tx(&bars->full[s], Cfg::kStageBytes);
        tma_load_2d(&tm_a, &bars->full[s], st, kb * kBK, m_blk * kBM);
        tma_load_2d(&tm_w, &bars->full[s], st + kATileBytes, kb * kBK, n_blk * BN);
        ++issued;
      }
      for (int kb = (issued > kStages ? issued - kStages : 0); kb < issued; ++kb)
        (void)mbar_wait(&bars->full[kb % kStages], (kb / kStages) & 1, abort_flag);
    }
  } else if (warp == 1) {
    if (elect_one()) {
      bool ok = true;
      const uint32_t s0 = smem_u32(smem);
      for (int kb = 0; kb < n_k; ++kb) {
        const int s = kb % kStages;
        if (!mbar_wait(&bars->full[s], (kb / kStages) & 1, abort_flag)) { ok = false; break; }
        tc_fence_after();
        const uint32_t sa = s0 + s * Cfg::kStageBytes;
        const uint32_t sb = sa + kATileBytes;
#pragma unroll
        for (int kk = 0; kk < kBK / 16; ++kk) {
          umma_ss(tmem, sdesc_sw128(sa + kk * 32, 16, 1024), sdesc_sw128(sb + kk * 32, 16, 1024),
                  Cfg::kIdesc, (kb > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(&bars->empty[s]);
      }
      if (!ok) raise_abort(abort_flag, err_word, kDevErrTimeoutMma);
      umma_commit(&bars->acc_full);
      (void)mbar_wait(&bars->acc_full, 0, abort_flag);
    }
  } else if (warp >= 4) {
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const int m = m_blk * kBM + row;
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    if (!warp_wait(&bars->acc_full, 0, abort_flag)) {
      raise_abort(abort_flag, err_word, kDevErrTimeoutEpilogue);
    } else {
      tc_fence_after();
      const int n0 = n_blk * BN;
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        uint32_t r[32];
        tmem_ld32(tmem + lane_base + c * 32, r);
        tmem_ld_wait();
        if (m < M) {
          const int nc = n0 + c * 32;
          float v[32];
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            const int n = nc + e;
            float z = __uint_as_float(r[e]);
            if (bias != nullptr && n < N) z += bias[n];
            z = apply_act(z, act);
            if (residual != nullptr && n < N) {
              const size_t idx = static_cast<size_t>(m) * N + n;
              z += residual_f32 ? static_cast<const float*>(residual)[idx]
                                : __bfloat162float(static_cast<const __nv_bfloat16*>(residual)[idx]);
            }
            v[e] = z;
          }
          const size_t rowoff = static_cast<size_t>(m) * N;
          if (nc + 32 <= N && (N % 8) == 0) {
            if constexpr (kOutF32) {
              float4* dst = reinterpret_cast<float4*>(static_cast<float*>(Y) + rowoff + nc);
#pragma unroll
              for (int e = 0; e < 8; ++e)
                dst[e] = make_float4(v[4 * e], v[4 * e + 1], v[4 * e + 2], v[4 * e + 3]);
            } else {
              uint4* dst = reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(Y) + rowoff + nc);
#pragma unroll
              for (int e = 0; e < 4; ++e)
                dst[e] = make_uint4(pack_bf16x2(v[8 * e], v[8 * e + 1]),
                                    pack_bf16x2(v[8 * e + 2], v[8 * e + 3]),
                                    pack_bf16x2(v[8 * e + 4], v[8 * e + 5]),
                                    pack_bf16x2(v[8 * e + 6], v[8 * e + 7]));
            }
          } else {
#pragma unroll
            for (int e = 0; e < 32; ++e) {
              const int n = nc + e;
              if (n < N) {
                if constexpr (kOutF32) static_cast<float*>(Y)[rowoff + n] = v[e];
                else static_cast<__nv_bfloat16*>(Y)[rowoff + n] = __float2bfloat16_rn(v[e]);
              }
            }
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, Cfg::kTmemCols);
  }
}

template <int BN, bool kOutF32>
cudaError_t launch_typed(cudaStream_t stream, const CUtensorMap& ta, const CUtensorMap& tw,
                         const float* bias, const void* residual, bool residual_f32, void* Y,
                         int M, int N, int K, int act) {
  using Cfg = GemmCfg<BN>;
  auto kern = gemm_kernel<BN, kOutF32>;
  cudaError_t e =
      cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmemBytes);
  if (e != cudaSuccess) return e;
  dim3 grid((N + BN - 1) / BN, (M + kBM - 1) / kBM);
  kern<<<grid, kThreads, Cfg::kSmemBytes, stream>>>(ta, tw, bias, residual, residual_f32 ? 1 : 0,
                                                    Y, M, N, K, act, device_error_word());
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_gemm(cudaStream_t stream, const __nv_bfloat16* A, const __nv_bfloat16* W,
                        const float* bias, const void* residual, bool residual_f32, void* Y,
                        bool out_f32, int M, int N, int K, int act, const char** err_msg) {
  if (M == 0 || N == 0) return cudaSuccess;
  // Narrow problems (few row blocks) use 128-wide tiles for more CTAs.
  const int m_blocks = (M + kBM - 1) / kBM;
  const bool wide = (static_cast<long long>(m_blocks) * ((N + 255) / 256) >= 148);
  const int BN = wide ? 256 : 128;
  CUtensorMap ta, tw;
  {
    const uint64_t dims[2] = {static_cast<uint64_t>(K), static_cast<uint64_t>(M)};
    const uint64_t strides[1] = {static_cast<uint64_t>(K) * 2};
    const uint32_t box[2] = {kBK, kBM};
    cudaError_t e = make_tmap_bf16_sw128(&ta, A, 2, dims, strides, box, err_msg);
    if (e != cudaSuccess) return e;
  }
  {
    const uint64_t dims[2] = {static_cast<uint64_t>(K), static_cast<uint64_t>(N)};
    const uint64_t strides[1] = {static_cast<uint64_t>(K) * 2};
    const uint32_t box[2] = {kBK, static_cast<uint32_t>(BN)};
    cudaError_t e = make_tmap_bf16_sw128(&tw, W, 2, dims, strides, box, err_msg);
    if (e != cudaSuccess) return e;
  }
  if (K == 0) return cudaErrorInvalidValue;
  if (wide)
    return out_f32 ? launch_typed<256, true>(stream, ta, tw, bias, residual, residual_f32, Y, M, N, K, act)
                   : launch_typed<256, false>(stream, ta, tw, bias, residual, residual_f32, Y, M, N, K, act);
  return out_f32 ? launch_typed<128, true>(stream, ta, tw, bias, residual, residual_f32, Y, M, N, K, act)
                 : launch_typed<128, false>(stream, ta, tw, bias, residual, residual_f32, Y, M, N, K, act);
}

}  // namespace nd
