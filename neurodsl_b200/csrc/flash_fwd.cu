// flash_fwd.cu — causal / non-causal attention prefill on tcgen05 + TMEM + TMA.
//
// Computes, for every (batch, head) of head-major [B][H][S][D] bf16 tensors,
//   O = softmax(Q·Kᵀ·scale [+ causal mask]) · V,  lse = log Σ exp(.) , m = rowmax
// which is flash_attn_fwd! / flash_attn_fwd_cpu_simple! of the reference
// (src/flash_attention.jl:49-69, :113-134) evaluated blockwise with an online
// softmax (the reference's tiled form, :9-46), never materialising S.
//
// Per CTA: one 128-query tile of one head.  Warp roles (256 threads):
//   warp 0      TMA producer: Q once, then K/V tiles of 128 keys (3 stages)
//   warp 1      TMEM allocator + single-thread UMMA issuer
//   warps 4..7  softmax: thread t owns query row t of the tile (TMEM lane t)
// TMEM (512 columns): S double buffer at columns [0,128) and [128,256),
// O accumulator (fp32, 64 columns) at [256,320).
// S_{j+1} = Q·K_{j+1}ᵀ runs on the tensor core while softmax reads S_j.
// P_j (bf16) goes to shared memory in the 128-byte-swizzled K-major layout
// and O += P_j·V_j reads it with V as an MN-major operand.
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

constexpr int kBM = 128;
constexpr int kBN = 128;
constexpr int kD = 64;
constexpr int kStages = 3;
constexpr int kThreads = 256;
constexpr uint32_t kTileBytes = kBM * kD * 2;  // 16 KB (Q, K or V tile)
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColS0 = 0, kColS1 = 128, kColO = 256;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;
constexpr float kRescaleThreshold = 8.0f;

// shared-memory map (offsets from a 1024-aligned base)
constexpr uint32_t kOffQ = 0;
constexpr uint32_t kOffK = kOffQ + kTileBytes;
constexpr uint32_t kOffV = kOffK + kStages * kTileBytes;
constexpr uint32_t kOffP = kOffV + kStages * kTileBytes;      // 2 x 16 KB (keys 0-63, 64-127)
constexpr uint32_t kOffBar = kOffP + 2 * kTileBytes;
constexpr uint32_t kSmemBytes = kOffBar + 256 + 1024;         // + alignment slack

constexpr uint32_t kIdescS = idesc_bf16_f32(kBM, kBN, false, false);
constexpr uint32_t kIdescO = idesc_bf16_f32(kBM, kD, false, true);

struct Bars {
  uint64_t q_full;
  uint64_t kv_full[kStages];
  uint64_t kv_empty[kStages];
  uint64_t s_full[2];
  uint64_t p_full;
  uint64_t o_done;
  uint64_t drained;
  uint32_t tmem_base;
  int abort_flag;
};

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

  // Heavy tiles first: with a causal mask the last query tiles see the most keys.
  const int n_qt = (Sq + kBM - 1) / kBM;
  const int qt = kCausal ? (n_qt - 1 - static_cast<int>(blockIdx.x) / BH)
                         : static_cast<int>(blockIdx.x) / BH;
  const int bh = static_cast<int>(blockIdx.x) % BH;
  const int n_kv = kCausal ? (qt + 1) : (Sk + kBN - 1) / kBN;

  if (threadIdx.x == 0) {
    mbar_init(&bars->q_full, 1);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&bars->kv_full[s], 1);
      mbar_init(&bars->kv_empty[s], 1);
    }
    mbar_init(&bars->s_full[0], 1);
    mbar_init(&bars->s_full[1], 1);
    mbar_init(&bars->p_full, kBM);
    mbar_init(&bars->o_done, 1);
    mbar_init(&bars->drained, 1);
    bars->abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(&bars->tmem_base, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (elect_one()) {
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
      mbar_arrive_expect_tx(&bars->q_full, kTileBytes);
      tma_load_3d(&tm_q, &bars->q_full, smem + kOffQ, 0, qt * kBM, bh);
      int issued = 0;
      for (int j = 0; j < n_kv; ++j) {
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
  } else if (warp == 1) {
    // ---------------------------------------------------------- UMMA issuer
    if (elect_one()) {
      const uint32_t sQ = smem_u32(smem + kOffQ);
      const uint32_t sK = smem_u32(smem + kOffK);
      const uint32_t sV = smem_u32(smem + kOffV);
      const uint32_t sP = smem_u32(smem + kOffP);
      bool ok = mbar_wait(&bars->q_full, 0, abort_flag);
      auto issue_s = [&](int j) -> bool {
        const int s = j % kStages;
        if (!mbar_wait(&bars->kv_full[s], (j / kStages) & 1, abort_flag)) return false;
        tc_fence_after();
        const uint32_t d = tmem + ((j & 1) ? kColS1 : kColS0);
#pragma unroll
        for (int kk = 0; kk < kD / 16; ++kk) {
          const uint64_t a = sdesc_sw128(sQ + kk * 32, 16, 1024);
          const uint64_t b = sdesc_sw128(sK + s * kTileBytes + kk * 32, 16, 1024);
          umma_ss(d, a, b, kIdescS, kk > 0 ? 1u : 0u);
        }
        umma_commit(&bars->s_full[j & 1]);
        return true;
      };
      if (ok) ok = issue_s(0);
      for (int j = 0; ok && j < n_kv; ++j) {
        if (j + 1 < n_kv) {
          if (!issue_s(j + 1)) { ok = false; break; }
        }
        if (!mbar_wait(&bars->p_full, j & 1, abort_flag)) { ok = false; break; }
        tc_fence_after();
        const int s = j % kStages;
#pragma unroll
        for (int kk = 0; kk < kBN / 16; ++kk) {
          const uint64_t a = sdesc_sw128(sP + (kk >> 2) * kTileBytes + (kk & 3) * 32, 16, 1024);
          const uint64_t b = sdesc_sw128(sV + s * kTileBytes + kk * 2048, 8192, 1024);
          umma_ss(tmem + kColO, a, b, kIdescO, (j > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(&bars->o_done);
        umma_commit(&bars->kv_empty[s]);
      }
      if (!ok) raise_abort(abort_flag, err_word, kDevErrTimeoutMma);
      // Wait until every issued UMMA has completed before teardown.
      umma_commit(&bars->drained);
      (void)mbar_wait(&bars->drained, 0, abort_flag);
    }
  } else if (warp >= 4) {
    // -------------------------------------------------------------- softmax
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;              // row within the tile = TMEM lane
    const int q_idx = qt * kBM + row;                 // query position
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t sP = smem_u32(smem + kOffP);
    float m_used = -INFINITY;  // offset used for exponentials (log2 units)
    float m_true = -INFINITY;  // true running row max (log2 units)
    float l = 0.f;
    bool ok = true;
    for (int j = 0; j < n_kv; ++j) {
      if (!warp_wait(&bars->s_full[j & 1], (j >> 1) & 1, abort_flag)) { ok = false; break; }
      tc_fence_after();
      const uint32_t s_addr = tmem + lane_base + ((j & 1) ? kColS1 : kColS0);
      uint32_t sr[kBN];
#pragma unroll
      for (int c = 0; c < kBN / 32; ++c)
        tmem_ld32(s_addr + c * 32, *reinterpret_cast<uint32_t(*)[32]>(&sr[c * 32]));
      tmem_ld_wait();
      float* sv = reinterpret_cast<float*>(sr);
      const bool last = (j == n_kv - 1);
      if (last) {
        const int k0 = j * kBN;
#pragma unroll
        for (int c = 0; c < kBN; ++c) {
          const int k_idx = k0 + c;
          const bool masked = (k_idx >= Sk) || (kCausal && k_idx > q_idx);
          if (masked) sv[c] = -INFINITY;
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
      // exponentials and row sum; m_new is finite because key 0 of the
      // first tile is never masked for a valid query row
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
      // P buffer and O are owned by the previous P·V until o_done fires.
      if (j > 0) {
        if (!warp_wait(&bars->o_done, (j - 1) & 1, abort_flag)) { ok = false; break; }
        tc_fence_after();
        // tcgen05.ld/st are warp-collective: the whole warp rescales when any
        // of its rows needs it (alpha = 1 for the others).
        if (__any_sync(0xffffffffu, alpha != 1.f)) {
          const uint32_t o_addr = tmem + lane_base + kColO;
          uint32_t orr[32];
#pragma unroll
          for (int c = 0; c < kD / 32; ++c) {
            tmem_ld32(o_addr + c * 32, orr);
            tmem_ld_wait();
#pragma unroll
            for (int e = 0; e < 32; ++e) orr[e] = __float_as_uint(__uint_as_float(orr[e]) * alpha);
            tmem_st32(o_addr + c * 32, orr);
          }
          tmem_st_wait();
        }
      }
      // write P row (bf16) in the 128B-swizzled K-major layout
      const uint32_t rsw = static_cast<uint32_t>(row & 7);
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const uint32_t rbase = sP + h * kTileBytes + row * 128;
#pragma unroll
        for (int ch = 0; ch < 8; ++ch) {
          const int w0 = h * 32 + ch * 4;
          st_shared_v4(rbase + ((ch ^ rsw) << 4), pk[w0], pk[w0 + 1], pk[w0 + 2], pk[w0 + 3]);
        }
      }
      fence_async_shared();
      tc_fence_before();
      mbar_arrive(&bars->p_full);
      m_used = m_new;
    }
    // ------------------------------------------------------------ epilogue
    if (ok && n_kv > 0) {
      if (!warp_wait(&bars->o_done, (n_kv - 1) & 1, abort_flag)) ok = false;
    }
    if (!ok) {
      raise_abort(abort_flag, err_word, kDevErrTimeoutSoftmax);
    } else {
      tc_fence_after();
      const uint32_t o_addr = tmem + lane_base + kColO;
      uint32_t orr[kD];
      tmem_ld32(o_addr, *reinterpret_cast<uint32_t(*)[32]>(&orr[0]));
      tmem_ld32(o_addr + 32, *reinterpret_cast<uint32_t(*)[32]>(&orr[32]));
      tmem_ld_wait();
      if (q_idx < Sq) {
        const float inv_l = 1.f / l;
        const size_t row_off = (static_cast<size_t>(bh) * Sq + q_idx);
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
  if (warp == 1) {
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
  const int n_qt = (Sq + kBM - 1) / kBM;
  dim3 grid(n_qt * BH);
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
