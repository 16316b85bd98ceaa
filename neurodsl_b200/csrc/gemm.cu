// gemm.cu — Y = act(A·Wᵀ + bias) + residual on tcgen05 + TMEM + TMA.
//
// The :linear rule (src/dispatch.jl:363-384: mul!(out, X, W') then
// out .+= b'), :fused_matmul_add (:281-296), the notebook's fused_linear_gelu
// (notebook/compiler.ipynb cell 15: z·σ(1.702 z)) and the residual :add
// (:386-417) as one kernel: the bias, the GELU and the residual are applied
// in the epilogue while the fp32 accumulator is read out of tensor memory.
//
// A [M][K] and W [N][K] are bf16, K contiguous (W is the (out, in) weight of
// a Linear layer).  Persistent CTAs walk 128 x BN output tiles; K is consumed
// in blocks of 64 through a TMA ring that runs on across tiles.  Warp roles
// (384 threads): warp 0 TMA producer, warp 1 TMEM allocator + UMMA issuer,
// warps 4..11 epilogue, two per TMEM lane quarter (thread = accumulator row
// = TMEM lane; the pair splits the tile's 32-column chunks).  Two
// TMEM accumulators alternate between tiles, so the epilogue of one tile
// overlaps the main loop of the next.  The epilogue transposes each 32x32
// chunk through padded shared memory so global stores (and residual loads)
// cover contiguous row segments instead of one row per lane; the activation
// is a template parameter, so the epilogue carries no per-element branches.
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
constexpr int kThreads = 384;
constexpr uint32_t kATileBytes = kBM * kBK * 2;  // 16 KB
constexpr int kStagePitch = 33;                  // words per staged row (32 + 1 pad)

template <int BN>
struct GemmCfg {
  // 4 x 48 KB (BN 256) or 6 x 32 KB (BN 128) stages + 33 KB staging + barriers
  // = 231,680 bytes, within the 232,448-byte per-block limit.
  static constexpr int kStages = BN >= 256 ? 4 : 6;
  static constexpr uint32_t kBTileBytes = BN * kBK * 2;
  static constexpr uint32_t kStageBytes = kATileBytes + kBTileBytes;
  static constexpr uint32_t kOffStage = kStages * kStageBytes;          // epilogue staging
  static constexpr uint32_t kStageAreaBytes = 8 * 32 * kStagePitch * 4; // 8 warps x 32x33 words
  static constexpr uint32_t kOffBar = kOffStage + kStageAreaBytes;
  static constexpr uint32_t kSmemBytes = kOffBar + 256 + 1024;
  static constexpr uint32_t kTmemCols = 2 * BN;   // two accumulators (power of two)
  static constexpr uint32_t kIdesc = idesc_bf16_f32(kBM, BN, false, false);
};

template <int kStages>
struct GemmBars {
  uint64_t full[kStages];
  uint64_t empty[kStages];
  uint64_t acc_full[2];    // accumulator b holds a finished tile (UMMA commit)
  uint64_t acc_empty[2];   // epilogue has read accumulator b (256 threads)
  uint64_t drained;
  uint32_t tmem_base;
  int abort_flag;
};

template <int kAct>
__device__ __forceinline__ float apply_act(float z) {
  if constexpr (kAct == ND_ACT_GELU_SIGMOID) {
    return __fdividef(z, 1.f + __expf(-1.702f * z));
  } else if constexpr (kAct == ND_ACT_GELU_TANH) {
    const float u = 0.7978845608028654f * (z + 0.044715f * z * z * z);
    float th;
    asm("tanh.approx.f32 %0, %1;" : "=f"(th) : "f"(u));  // hardware tanh
    return 0.5f * z * (1.f + th);
  } else if constexpr (kAct == ND_ACT_GELU_ERF) {
    return 0.5f * z * (1.f + erff(z * 0.7071067811865476f));
  } else {
    return z;
  }
}

// Tile t of the persistent walk: N fastest within groups of 8 row blocks, so
// CTAs running at the same time share A rows and W columns in L2.
__device__ __forceinline__ void tile_coords(int t, int m_tiles, int n_tiles, int& m_blk,
                                            int& n_blk) {
  constexpr int kGroup = 8;
  const int per_group = kGroup * n_tiles;
  const int g = t / per_group;
  const int first_m = g * kGroup;
  const int rows = min(kGroup, m_tiles - first_m);
  const int r = t - g * per_group;
  m_blk = first_m + r % rows;
  n_blk = r / rows;
}

template <int BN, bool kOutF32, int kAct>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_w,
                const float* __restrict__ bias, const void* __restrict__ residual,
                int residual_f32, void* __restrict__ Y, int M, int N, int K,
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
  const int m_tiles = (M + kBM - 1) / kBM;
  const int n_tiles = (N + BN - 1) / BN;
  const int n_tiles_total = m_tiles * n_tiles;
  const int n_k = (K + kBK - 1) / kBK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&bars->full[s], 1);
      mbar_init(&bars->empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&bars->acc_full[b], 1);
      mbar_init(&bars->acc_empty[b], 256);
    }
    mbar_init(&bars->drained, 1);
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
    // ------------------------------------------------------------ producer
    if (elect_one()) {
      tma_prefetch_desc(&tm_a);
      tma_prefetch_desc(&tm_w);
      int it = 0;  // k-blocks loaded so far (ring position)
      bool ok = true;
      for (int t = blockIdx.x; ok && t < n_tiles_total; t += gridDim.x) {
        int m_blk, n_blk;
        tile_coords(t, m_tiles, n_tiles, m_blk, n_blk);
        for (int kb = 0; kb < n_k; ++kb, ++it) {
          const int s = it % kStages;
          if (it >= kStages && !mbar_wait(&bars->empty[s], ((it / kStages) - 1) & 1, abort_flag)) {
            ok = false;
            break;
          }
          uint8_t* st = smem + s * Cfg::kStageBytes;
          mbar_arrive_expect_tx(&bars->full[s], Cfg::kStageBytes);
          tma_load_2d(&tm_a, &bars->full[s], st, kb * kBK, m_blk * kBM);
          tma_load_2d(&tm_w, &bars->full[s], st + kATileBytes, kb * kBK, n_blk * BN);
        }
      }
      if (!ok) raise_abort(abort_flag, err_word, kDevErrTimeoutProducer);
      for (int j = (it > kStages ? it - kStages : 0); j < it; ++j)
        (void)mbar_wait(&bars->full[j % kStages], (j / kStages) & 1, abort_flag);
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------- UMMA issuer
    if (elect_one()) {
      bool ok = true;
      const uint32_t s0 = smem_u32(smem);
      int it = 0, lt = 0;
      for (int t = blockIdx.x; ok && t < n_tiles_total; t += gridDim.x, ++lt) {
        const int b = lt & 1;
        // the epilogue must have drained accumulator b (tile lt - 2)
        if (lt >= 2 && !mbar_wait(&bars->acc_empty[b], ((lt >> 1) - 1) & 1, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t acc = tmem + b * BN;
        for (int kb = 0; kb < n_k; ++kb, ++it) {
          const int s = it % kStages;
          if (!mbar_wait(&bars->full[s], (it / kStages) & 1, abort_flag)) { ok = false; break; }
          tc_fence_after();
          const uint32_t sa = s0 + s * Cfg::kStageBytes;
          const uint32_t sb = sa + kATileBytes;
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk)
            umma_ss(acc, sdesc_sw128(sa + kk * 32, 16, 1024), sdesc_sw128(sb + kk * 32, 16, 1024),
                    Cfg::kIdesc, (kb > 0 || kk > 0) ? 1u : 0u);
          umma_commit(&bars->empty[s]);
        }
        if (ok) umma_commit(&bars->acc_full[b]);
      }
      if (!ok) raise_abort(abort_flag, err_word, kDevErrTimeoutMma);
      umma_commit(&bars->drained);
      (void)mbar_wait(&bars->drained, 0, abort_flag);
    }
  } else if (warp >= 4) {
    // ------------------------------------------------------------- epilogue
    // Per 32-column chunk: the raw fp32 accumulators are staged row-per-lane
    // in padded shared memory, then read back column-per-lane, where the
    // bias, the activation and the residual are applied and the output is
    // stored: every global access of a warp covers contiguous row segments.
    // The TMEM load of the next chunk is in flight during this column phase.
    // Two warps per TMEM lane quarter: warp 4+q takes the even chunks of rows
    // 32q..32q+31, warp 8+q the odd ones.
    const int quarter = warp & 3;
    const int half = (warp >> 2) - 1;
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    float* stage = reinterpret_cast<float*>(smem + Cfg::kOffStage) + (warp - 4) * 32 * kStagePitch;
    const int sub = lane >> 4;      // column phase: lanes 0..15 even rows, 16..31 odd rows
    const int cw = (lane & 15) * 2; // column pair within the chunk
    const bool pair_ok = (N % 2) == 0;
    bool ok = true;
    int lt = 0;
    for (int t = blockIdx.x; t < n_tiles_total; t += gridDim.x, ++lt) {
      int m_blk, n_blk;
      tile_coords(t, m_tiles, n_tiles, m_blk, n_blk);
      const int b = lt & 1;
      if (!warp_wait(&bars->acc_full[b], (lt >> 1) & 1, abort_flag)) { ok = false; break; }
      tc_fence_after();
      const int row0 = m_blk * kBM + quarter * 32;  // first row of this warp's 32
      const uint32_t acc = tmem + lane_base + b * BN;
      const int n_chunks = min(BN / 32, (N - n_blk * BN + 31) / 32);
      uint32_t r[2][32];
      if (half < n_chunks) tmem_ld32(acc + half * 32, r[0]);
#pragma unroll 1
      for (int c = half, k = 0; c < n_chunks; c += 2, ++k) {
        const int col0 = n_blk * BN + c * 32;
        tmem_ld_wait();
        // (k & 1) selects the register buffer; both branches are unrolled so
        // the buffers stay in registers
#define ND_STAGE_CHUNK(CUR, NXT)                                                  \
        {                                                                        \
          _Pragma("unroll") for (int e = 0; e < 32; ++e)                         \
            stage[lane * kStagePitch + e] = __uint_as_float(r[CUR][e]);          \
          if (c + 2 < n_chunks) tmem_ld32(acc + (c + 2) * 32, r[NXT]);           \
        }
        if (k & 1) ND_STAGE_CHUNK(1, 0) else ND_STAGE_CHUNK(0, 1)
#undef ND_STAGE_CHUNK
        __syncwarp();
        const int n = col0 + cw;
        float b0 = 0.f, b1 = 0.f;
        if (bias != nullptr) {
          if (n < N) b0 = __ldg(bias + n);
          if (n + 1 < N) b1 = __ldg(bias + n + 1);
        }
#pragma unroll 4
        for (int i = 0; i < 16; ++i) {
          const int rr = 2 * i + sub;
          const int m = row0 + rr;
          float z0 = apply_act<kAct>(stage[rr * kStagePitch + cw] + b0);
          float z1 = apply_act<kAct>(stage[rr * kStagePitch + cw + 1] + b1);
          if (m < M) {
            const size_t idx = static_cast<size_t>(m) * N + n;
            if (pair_ok && n + 1 < N) {
              if (residual != nullptr) {
                if (residual_f32) {
                  const float2 rv = *reinterpret_cast<const float2*>(static_cast<const float*>(residual) + idx);
                  z0 += rv.x;
                  z1 += rv.y;
                } else {
                  const __nv_bfloat162 rv =
                      *reinterpret_cast<const __nv_bfloat162*>(static_cast<const __nv_bfloat16*>(residual) + idx);
                  z0 += __low2float(rv);
                  z1 += __high2float(rv);
                }
              }
              if constexpr (kOutF32)
                *reinterpret_cast<float2*>(static_cast<float*>(Y) + idx) = make_float2(z0, z1);
              else
                *reinterpret_cast<uint32_t*>(static_cast<__nv_bfloat16*>(Y) + idx) = pack_bf16x2(z0, z1);
            } else {
              float zz[2] = {z0, z1};
#pragma unroll
              for (int q = 0; q < 2; ++q) {
                if (n + q < N) {
                  float zq = zz[q];
                  if (residual != nullptr)
                    zq += residual_f32 ? static_cast<const float*>(residual)[idx + q]
                                       : __bfloat162float(static_cast<const __nv_bfloat16*>(residual)[idx + q]);
                  if constexpr (kOutF32) static_cast<float*>(Y)[idx + q] = zq;
                  else static_cast<__nv_bfloat16*>(Y)[idx + q] = __float2bfloat16_rn(zq);
                }
              }
            }
          }
        }
        __syncwarp();
      }
      // accumulator b fully read: the MMA warp may reuse it
      tc_fence_before();
      mbar_arrive(&bars->acc_empty[b]);
    }
    if (!ok) raise_abort(abort_flag, err_word, kDevErrTimeoutEpilogue);
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, Cfg::kTmemCols);
  }
}

template <int BN, bool kOutF32, int kAct>
cudaError_t launch_typed(cudaStream_t stream, const CUtensorMap& ta, const CUtensorMap& tw,
                         const float* bias, const void* residual, bool residual_f32, void* Y,
                         int M, int N, int K, int sms) {
  using Cfg = GemmCfg<BN>;
  auto kern = gemm_kernel<BN, kOutF32, kAct>;
  cudaError_t e =
      cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmemBytes);
  if (e != cudaSuccess) return e;
  const int tiles = ((M + kBM - 1) / kBM) * ((N + BN - 1) / BN);
  dim3 grid(tiles < sms ? tiles : sms);
  kern<<<grid, kThreads, Cfg::kSmemBytes, stream>>>(ta, tw, bias, residual, residual_f32 ? 1 : 0,
                                                    Y, M, N, K, device_error_word());
  return cudaGetLastError();
}

template <int BN, bool kOutF32>
cudaError_t launch_act(int act, cudaStream_t stream, const CUtensorMap& ta, const CUtensorMap& tw,
                       const float* bias, const void* residual, bool residual_f32, void* Y, int M,
                       int N, int K, int sms) {
  switch (act) {
    case ND_ACT_GELU_SIGMOID:
      return launch_typed<BN, kOutF32, ND_ACT_GELU_SIGMOID>(stream, ta, tw, bias, residual, residual_f32, Y, M, N, K, sms);
    case ND_ACT_GELU_TANH:
      return launch_typed<BN, kOutF32, ND_ACT_GELU_TANH>(stream, ta, tw, bias, residual, residual_f32, Y, M, N, K, sms);
    case ND_ACT_GELU_ERF:
      return launch_typed<BN, kOutF32, ND_ACT_GELU_ERF>(stream, ta, tw, bias, residual, residual_f32, Y, M, N, K, sms);
    default:
      return launch_typed<BN, kOutF32, ND_ACT_NONE>(stream, ta, tw, bias, residual, residual_f32, Y, M, N, K, sms);
  }
}

template <bool kOutF32>
cudaError_t launch_bn(int BN, int act, cudaStream_t stream, const CUtensorMap& ta,
                      const CUtensorMap& tw, const float* bias, const void* residual,
                      bool residual_f32, void* Y, int M, int N, int K, int sms) {
  if (BN == 256)
    return launch_act<256, kOutF32>(act, stream, ta, tw, bias, residual, residual_f32, Y, M, N, K, sms);
  if (BN == 128)
    return launch_act<128, kOutF32>(act, stream, ta, tw, bias, residual, residual_f32, Y, M, N, K, sms);
  return launch_act<64, kOutF32>(act, stream, ta, tw, bias, residual, residual_f32, Y, M, N, K, sms);
}

}  // namespace

cudaError_t launch_gemm(cudaStream_t stream, const __nv_bfloat16* A, const __nv_bfloat16* W,
                        const float* bias, const void* residual, bool residual_f32, void* Y,
                        bool out_f32, int M, int N, int K, int act, const char** err_msg) {
  if (M == 0 || N == 0) return cudaSuccess;
  if (K == 0) return cudaErrorInvalidValue;
  int dev = 0, sms = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (e != cudaSuccess) return e;
  // Widest tile that still gives every SM at least one tile.
  const int m_tiles = (M + kBM - 1) / kBM;
  int BN = 256;
  while (BN > 64 && static_cast<long long>(m_tiles) * ((N + BN - 1) / BN) < sms) BN >>= 1;
  CUtensorMap ta, tw;
  {
    const uint64_t dims[2] = {static_cast<uint64_t>(K), static_cast<uint64_t>(M)};
    const uint64_t strides[1] = {static_cast<uint64_t>(K) * 2};
    const uint32_t box[2] = {kBK, kBM};
    e = make_tmap_bf16_sw128(&ta, A, 2, dims, strides, box, err_msg);
    if (e != cudaSuccess) return e;
  }
  {
    const uint64_t dims[2] = {static_cast<uint64_t>(K), static_cast<uint64_t>(N)};
    const uint64_t strides[1] = {static_cast<uint64_t>(K) * 2};
    const uint32_t box[2] = {kBK, static_cast<uint32_t>(BN)};
    e = make_tmap_bf16_sw128(&tw, W, 2, dims, strides, box, err_msg);
    if (e != cudaSuccess) return e;
  }
  return out_f32 ? launch_bn<true>(BN, act, stream, ta, tw, bias, residual, residual_f32, Y, M, N, K, sms)
                 : launch_bn<false>(BN, act, stream, ta, tw, bias, residual, residual_f32, Y, M, N, K, sms);
}

}  // namespace nd
