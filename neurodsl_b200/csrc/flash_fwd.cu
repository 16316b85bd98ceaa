// flash_fwd.cu — causal / non-causal attention prefill on tcgen05 + TMEM + TMA.
//
// Computes, for every (batch, head) of head-major [B][H][S][D] bf16 tensors,
//   O = softmax(Q·Kᵀ·scale [+ causal mask]) · V,  lse = log Σ exp(.),  m = rowmax
// which is flash_attn_fwd! / flash_attn_fwd_cpu_simple! of the reference
// (src/flash_attention.jl:49-69, :113-134) evaluated blockwise with an online
// softmax (the reference's tiled form, :9-46), never materialising S.
//
// Per CTA: 256 query rows of one head as two 128-row tiles that share one
// stream of K/V tiles (128 keys each).  Warp roles (320 threads):
//   warps 0..3   softmax of query tile 0 (thread t owns row t = TMEM lane t)
//   warps 4..7   softmax of query tile 1
//   warp 8       TMA producer: Q0/Q1 once, then K/V tiles (kStages-deep ring)
//   warp 9       TMEM allocator + single-thread UMMA issuer
// TMEM (512 columns): S0 [0,128), S1 [128,256), O0 [256,320), O1 [320,384).
// Softmax i reads S_i, writes P_i as packed bf16 over S_i's first 64
// columns, and O_i += P_i·V_j reads P_i straight from tensor memory (A
// operand in TMEM, V as an MN-major shared-memory operand).  While one
// tile's softmax runs, the tensor core works on the other tile.
// The running max is raised only when a row's max grows by more than 8
// (log2 units); O and l share the stale offset, so the final O/l is exact.
#include <cuda.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "flash_fwd.h"
#include "ptx.cuh"
#include "tma.h"

namespace nd {
namespace {

constexpr int kBM = 128;               // rows per query tile
constexpr int kTiles = 2;              // query tiles per CTA
constexpr int kRowsPerCta = kBM * kTiles;
constexpr int kBN = 128;               // keys per K/V tile
constexpr int kD = 64;
constexpr int kStages = 3;
constexpr int kSoftmaxThreads = 128 * kTiles;
constexpr int kThreads = kSoftmaxThreads + 64;   // + producer warp + MMA warp
constexpr int kWarpProducer = kSoftmaxThreads / 32;
constexpr int kWarpMma = kWarpProducer + 1;
constexpr uint32_t kTileBytes = kBM * kD * 2;    // 16 KB (one Q, K or V tile)
constexpr uint32_t kTmemCols = 512;
// TMEM columns: S_i at i*128, O_i at 256 + i*64
__host__ __device__ constexpr uint32_t col_s(int i) { return static_cast<uint32_t>(i) * 128u; }
__host__ __device__ constexpr uint32_t col_o(int i) { return 256u + static_cast<uint32_t>(i) * 64u; }
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;
constexpr float kRescaleThreshold = 8.0f;

// shared-memory map (offsets from a 1024-aligned base)
constexpr uint32_t kOffQ = 0;                                   // 2 x 16 KB
constexpr uint32_t kOffK = kOffQ + kTiles * kTileBytes;
constexpr uint32_t kOffV = kOffK + kStages * kTileBytes;
constexpr uint32_t kOffBar = kOffV + kStages * kTileBytes;
constexpr uint32_t kSmemBytes = kOffBar + 256 + 1024;           // + alignment slack

constexpr uint32_t kIdescS = idesc_bf16_f32(kBM, kBN, false, false);
constexpr uint32_t kIdescO = idesc_bf16_f32(kBM, kD, false, true);

struct Bars {
  uint64_t q_full;
  uint64_t kv_full[kStages];
  uint64_t kv_empty[kStages];
  uint64_t s_full[kTiles];
  uint64_t p_full[kTiles];
  uint64_t o_done[kTiles];
  uint64_t drained;
  uint32_t tmem_base;
  int abort_flag;
};

__host__ __device__ constexpr int ceil_div(int a, int b) { return (a + b - 1) / b; }

template <bool kCausal, bool kOutF32>
__global__ void __launch_bounds__(kThreads, 1)
    flash_fwd_kernel(const __grid_constant__ CUtensorMap tm_q,
                     const __grid_constant__ CUtensorMap tm_k,
                     const __grid_constant__ CUtensorMap tm_v, void* __restrict__ out,
                     float* __restrict__ lse_out, float* __restrict__ max_out, int BH, int Sq,
                     int Sk, float scale_log2, int* __restrict__ err_word) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  Bars* bars = reinterpret_cast<Bars*>(smem + kOffBar);
  volatile int* abort_flag = &bars->abort_flag;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  // Heavy blocks first: with a causal mask the last query rows see the most keys.
  const int n_blk = ceil_div(Sq, kRowsPerCta);
  const int blk = kCausal ? (n_blk - 1 - static_cast<int>(blockIdx.x) / BH)
                          : static_cast<int>(blockIdx.x) / BH;
  const int bh = static_cast<int>(blockIdx.x) % BH;
  const int n_k = ceil_div(Sk, kBN);
  // K/V tiles needed by query tile i (its index among 128-row tiles is 2*blk+i)
  int n_kv[kTiles];
#pragma unroll
  for (int i = 0; i < kTiles; ++i) {
    const int qt = blk * kTiles + i;
    n_kv[i] = kCausal ? min(qt + 1, n_k) : n_k;
  }
  const int n_total = n_kv[kTiles - 1];  // the last tile needs the most

  if (threadIdx.x == 0) {
    mbar_init(&bars->q_full, 1);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&bars->kv_full[s], 1);
      mbar_init(&bars->kv_empty[s], 1);
    }
    for (int i = 0; i < kTiles; ++i) {
      mbar_init(&bars->s_full[i], 1);
      mbar_init(&bars->p_full[i], kBM);
      mbar_init(&bars->o_done[i], 1);
    }
    mbar_init(&bars->drained, 1);
    bars->abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == kWarpMma) {
    tmem_alloc(&bars->tmem_base, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;

  if (warp == kWarpProducer) {
    // ------------------------------------------------------------ producer
    if (elect_one()) {
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
      mbar_arrive_expect_tx(&bars->q_full, kTiles * kTileBytes);
      for (int i = 0; i < kTiles; ++i)
        tma_load_3d(&tm_q, &bars->q_full, smem + kOffQ + i * kTileBytes, 0,
                    blk * kRowsPerCta + i * kBM, bh);
      int issued = 0;
      for (int j = 0; j < n_total; ++j) {
        const int s = j % kStages;
        if (j >= kStages) {
          if (!mbar_wait(&bars->kv_empty[s], ((j / kStages) - 1) & 1, abort_flag)) {
            raise_abort(abort_flag, err_word, kDevErrTimeoutProducer);
            break;
          }
        }
        mbar_arrive_expect_tx(&bars->kv_full[s], 2 * kTileBytes);
        tma_load_3d(&tm_k, &bars->kv_full[s], smem + kOffK + s * kTileBytes, 0, j * kBN, bh);
        tma_load_3d(&tm_v, &bars->kv_full[s], smem + kOffV + s * kTileBytes, 0, j * kBN, bh);
        ++issued;
      }
      // Drain: every issued copy lands before the CTA may exit.
      (void)mbar_wait(&bars->q_full, 0, abort_flag);
      for (int j = (issued > kStages ? issued - kStages : 0); j < issued; ++j)
        (void)mbar_wait(&bars->kv_full[j % kStages], (j / kStages) & 1, abort_flag);
    }
  } else if (warp == kWarpMma) {
    // ---------------------------------------------------------- UMMA issuer
    if (elect_one()) {
      const uint32_t sQ = smem_u32(smem + kOffQ);
      const uint32_t sK = smem_u32(smem + kOffK);
      const uint32_t sV = smem_u32(smem + kOffV);
      bool ok = mbar_wait(&bars->q_full, 0, abort_flag);
      int kv_ready = -1;  // highest K/V tile whose kv_full has been observed
      auto wait_kv = [&](int j) -> bool {
        if (j <= kv_ready) return true;
        if (!mbar_wait(&bars->kv_full[j % kStages], (j / kStages) & 1, abort_flag)) return false;
        kv_ready = j;
        return true;
      };
      auto issue_s = [&](int i, int j) {
        const int s = j % kStages;
        const uint32_t d = tmem + col_s(i);
#pragma unroll
        for (int kk = 0; kk < kD / 16; ++kk) {
          const uint64_t a = sdesc_sw128(sQ + i * kTileBytes + kk * 32, 16, 1024);
          const uint64_t b = sdesc_sw128(sK + s * kTileBytes + kk * 32, 16, 1024);
          umma_ss(d, a, b, kIdescS, kk > 0 ? 1u : 0u);
        }
        umma_commit(&bars->s_full[i]);
      };
      auto issue_pv = [&](int i, int j) {
        const int s = j % kStages;
#pragma unroll
        for (int kk = 0; kk < kBN / 16; ++kk) {
          const uint64_t b = sdesc_sw128(sV + s * kTileBytes + kk * 2048, 8192, 1024);
          // P_i: 128 lanes x 64 columns of packed bf16 pairs; 16 keys = 8 columns
          umma_ts(tmem + col_o(i), tmem + col_s(i) + kk * 8, b, kIdescO,
                  (j > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(&bars->o_done[i]);
      };
      if (ok && (ok = wait_kv(0))) {
        tc_fence_after();
        for (int i = 0; i < kTiles; ++i) issue_s(i, 0);
      }
      for (int j = 0; ok && j < n_total; ++j) {
        for (int i = 0; i < kTiles; ++i) {
          if (j >= n_kv[i]) continue;
          if (!mbar_wait(&bars->p_full[i], j & 1, abort_flag)) { ok = false; break; }
          tc_fence_after();
          issue_pv(i, j);
          if (i == kTiles - 1) umma_commit(&bars->kv_empty[j % kStages]);
          if (j + 1 < n_kv[i]) {
            if (!wait_kv(j + 1)) { ok = false; break; }
            tc_fence_after();
            issue_s(i, j + 1);
          }
        }
      }
      if (!ok) raise_abort(abort_flag, err_word, kDevErrTimeoutMma);
      // Every issued UMMA completes before teardown.
      umma_commit(&bars->drained);
      (void)mbar_wait(&bars->drained, 0, abort_flag);
    }
  } else {
    // -------------------------------------------------------------- softmax
    const int tile = warp >> 2;                     // 0 or 1
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;            // TMEM lane = row within the tile
    const int q_idx = blk * kRowsPerCta + tile * kBM + row;
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t s_addr = tmem + lane_base + col_s(tile);
    const uint32_t o_addr = tmem + lane_base + col_o(tile);
    const int nkv = n_kv[tile];
    float m_used = -INFINITY;  // offset used for exponentials (log2 units)
    float m_true = -INFINITY;  // true running row max (log2 units)
    float l = 0.f;
    bool ok = true;
    for (int j = 0; j < nkv; ++j) {
      if (!warp_wait(&bars->s_full[tile], j & 1, abort_flag)) { ok = false; break; }
      tc_fence_after();
      uint32_t sr[kBN];
#pragma unroll
      for (int c = 0; c < kBN / 32; ++c)
        tmem_ld32(s_addr + c * 32, *reinterpret_cast<uint32_t(*)[32]>(&sr[c * 32]));
      tmem_ld_wait();
      float* sv = reinterpret_cast<float*>(sr);
      if (j == nkv - 1) {
        const int k0 = j * kBN;
#pragma unroll
        for (int c = 0; c < kBN; ++c) {
          const int k_idx = k0 + c;
          if ((k_idx >= Sk) || (kCausal && k_idx > q_idx)) sv[c] = -INFINITY;
        }
      }
      float mx = -INFINITY;
#pragma unroll
      for (int c = 0; c < kBN; ++c) mx = fmaxf(mx, sv[c]);
      const float t_max = mx * scale_log2;
      m_true = fmaxf(m_true, t_max);
      float m_new = m_used;
      float alpha = 1.f;
      if (t_max > m_used + kRescaleThreshold) {
        m_new = t_max;
        alpha = (m_used == -INFINITY) ? 0.f : fast_exp2(m_used - m_new);
      }
      const float neg_m = -m_new;
      float rs = 0.f;
      uint32_t pk[kBN / 2];
#pragma unroll
      for (int c = 0; c < kBN; c += 2) {
        const float p0 = fast_exp2(fmaf(sv[c], scale_log2, neg_m));
        const float p1 = fast_exp2(fmaf(sv[c + 1], scale_log2, neg_m));
        rs += p0 + p1;
        pk[c >> 1] = pack_bf16x2(p0, p1);
      }
      l = l * alpha + rs;
      // P_i over the first 64 columns of S_i.  S_i(j) has been read in full,
      // and its commit followed P_i(j-1)·V in issue order, so that product has
      // finished reading the previous P_i and O_i is stable.
      tmem_st32(s_addr, *reinterpret_cast<const uint32_t(*)[32]>(&pk[0]));
      tmem_st32(s_addr + 32, *reinterpret_cast<const uint32_t(*)[32]>(&pk[32]));
      if (j > 0) {
        // already complete (see above); the wait is a cheap check
        if (!warp_wait(&bars->o_done[tile], (j - 1) & 1, abort_flag)) { ok = false; break; }
        tc_fence_after();
        if (__any_sync(0xffffffffu, alpha != 1.f)) {
          uint32_t orr[32];
#pragma unroll
          for (int c = 0; c < kD / 32; ++c) {
            tmem_ld32(o_addr + c * 32, orr);
            tmem_ld_wait();
#pragma unroll
            for (int e = 0; e < 32; ++e) orr[e] = __float_as_uint(__uint_as_float(orr[e]) * alpha);
            tmem_st32(o_addr + c * 32, orr);
          }
        }
      }
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(&bars->p_full[tile]);
      m_used = m_new;
    }
    // ------------------------------------------------------------ epilogue
    if (ok && nkv > 0) {
      if (!warp_wait(&bars->o_done[tile], (nkv - 1) & 1, abort_flag)) ok = false;
    }
    if (!ok) {
      raise_abort(abort_flag, err_word, kDevErrTimeoutSoftmax);
    } else {
      tc_fence_after();
      uint32_t orr[kD];
      tmem_ld32(o_addr, *reinterpret_cast<uint32_t(*)[32]>(&orr[0]));
      tmem_ld32(o_addr + 32, *reinterpret_cast<uint32_t(*)[32]>(&orr[32]));
      tmem_ld_wait();
      if (q_idx < Sq) {
        const float inv_l = 1.f / l;
        const size_t row_off = static_cast<size_t>(bh) * Sq + q_idx;
        if constexpr (kOutF32) {
          float4* dst = reinterpret_cast<float4*>(static_cast<float*>(out) + row_off * kD);
#pragma unroll
          for (int c = 0; c < kD / 4; ++c)
            dst[c] = make_float4(__uint_as_float(orr[4 * c]) * inv_l,
                                 __uint_as_float(orr[4 * c + 1]) * inv_l,
                                 __uint_as_float(orr[4 * c + 2]) * inv_l,
                                 __uint_as_float(orr[4 * c + 3]) * inv_l);
        } else {
          uint4* dst = reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(out) + row_off * kD);
#pragma unroll
          for (int c = 0; c < kD / 8; ++c)
            dst[c] = make_uint4(
                pack_bf16x2(__uint_as_float(orr[8 * c]) * inv_l, __uint_as_float(orr[8 * c + 1]) * inv_l),
                pack_bf16x2(__uint_as_float(orr[8 * c + 2]) * inv_l, __uint_as_float(orr[8 * c + 3]) * inv_l),
                pack_bf16x2(__uint_as_float(orr[8 * c + 4]) * inv_l, __uint_as_float(orr[8 * c + 5]) * inv_l),
                pack_bf16x2(__uint_as_float(orr[8 * c + 6]) * inv_l, __uint_as_float(orr[8 * c + 7]) * inv_l));
        }
        if (lse_out) lse_out[row_off] = (m_used + __log2f(l)) * kLn2;
        if (max_out) max_out[row_off] = m_true * kLn2;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kWarpMma) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

template <bool kCausal, bool kOutF32>
cudaError_t launch_typed(cudaStream_t stream, const CUtensorMap& tq, const CUtensorMap& tk,
                         const CUtensorMap& tv, void* out, float* lse, float* mx, int BH, int Sq,
                         int Sk, float scale_log2) {
  auto kern = flash_fwd_kernel<kCausal, kOutF32>;
  cudaError_t e =
      cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
  if (e != cudaSuccess) return e;
  dim3 grid(ceil_div(Sq, kRowsPerCta) * BH);
  kern<<<grid, kThreads, kSmemBytes, stream>>>(tq, tk, tv, out, lse, mx, BH, Sq, Sk, scale_log2,
                                               device_error_word());
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_flash_fwd(cudaStream_t stream, const __nv_bfloat16* Q, const __nv_bfloat16* K,
                             const __nv_bfloat16* V, void* O, bool out_f32, float* lse,
                             float* row_max, int B, int H, int Sq, int Sk, float scale,
                             bool causal, const char** err_msg) {
  const int BH = B * H;
  if (BH == 0 || Sq == 0) return cudaSuccess;
  CUtensorMap tq, tk, tv;
  const uint32_t box[3] = {kD, kBM, 1};
  {
    const uint64_t dims[3] = {kD, static_cast<uint64_t>(Sq), static_cast<uint64_t>(BH)};
    const uint64_t strides[2] = {kD * 2, static_cast<uint64_t>(Sq) * kD * 2};
    cudaError_t e = make_tmap_bf16_sw128(&tq, Q, 3, dims, strides, box, err_msg);
    if (e != cudaSuccess) return e;
  }
  {
    const uint64_t dims[3] = {kD, static_cast<uint64_t>(Sk), static_cast<uint64_t>(BH)};
    const uint64_t strides[2] = {kD * 2, static_cast<uint64_t>(Sk) * kD * 2};
    cudaError_t e = make_tmap_bf16_sw128(&tk, K, 3, dims, strides, box, err_msg);
    if (e != cudaSuccess) return e;
    e = make_tmap_bf16_sw128(&tv, V, 3, dims, strides, box, err_msg);
    if (e != cudaSuccess) return e;
  }
  const float sl2 = scale * kLog2e;
  if (causal) {
    return out_f32 ? launch_typed<true, true>(stream, tq, tk, tv, O, lse, row_max, BH, Sq, Sk, sl2)
                   : launch_typed<true, false>(stream, tq, tk, tv, O, lse, row_max, BH, Sq, Sk, sl2);
  }
  return out_f32 ? launch_typed<false, true>(stream, tq, tk, tv, O, lse, row_max, BH, Sq, Sk, sl2)
                 : launch_typed<false, false>(stream, tq, tk, tv, O, lse, row_max, BH, Sq, Sk, sl2);
}

}  // namespace nd
