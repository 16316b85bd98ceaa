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
// overlaps the main loop of the next.  The epilogue keeps each row in
// registers: bias, activation and residual are applied two columns per
// instruction (f32x2); for bf16 outputs each warp then passes its 32 rows x 32
// columns through a small shared-memory staging buffer (80-byte pitch), so
// that every global store instruction writes whole 64-byte row segments
// rather than half sectors.  The activation is a template parameter, so
// there are no per-element branches.
#include <cuda.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include <mutex>
#include <vector>

#include "gemm.h"
#include "launch.cuh"
#include "ptx.cuh"
#include "skinny_core.cuh"
#include "tma.h"

namespace nd {
namespace {

constexpr int kBM = 128;
constexpr int kBK = 64;
constexpr int kThreads = 384;
constexpr uint32_t kATileBytes = kBM * kBK * 2;  // 16 KB

constexpr int kEpiWarps = 8;
constexpr uint32_t kStagePitch = 80;  // bytes per staged 32-column bf16 row (64 + 16 pad)
constexpr uint32_t kStageWarpBytes = 32 * kStagePitch;
constexpr uint32_t kBiasWarpBytes = 4 * 32 * 4;  // a warp's bias: up to 4 chunks of 32

template <int BN>
struct GemmCfg {
  // 4 x 48 KB (BN 256), 6 x 32 KB (BN 128) or 8 x 24 KB (BN 64) stages, then
  // barriers, the epilogue warps' store staging and their bias slices, within
  // the 232,448-byte per-block limit.
  static constexpr int kStages = BN >= 256 ? 4 : (BN >= 128 ? 6 : 8);
  static constexpr uint32_t kBTileBytes = BN * kBK * 2;
  static constexpr uint32_t kStageBytes = kATileBytes + kBTileBytes;
  static constexpr uint32_t kOffBar = kStages * kStageBytes;
  static constexpr uint32_t kOffStaging = kOffBar + 256;
  static constexpr uint32_t kOffBias = kOffStaging + kEpiWarps * kStageWarpBytes;
  static constexpr uint32_t kSmemBytes = kOffBias + kEpiWarps * kBiasWarpBytes + 1024;
  static_assert(kSmemBytes <= 232448, "dynamic shared memory per block");
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

// GELU constants: sqrt(2/pi) and sqrt(2/pi) * 0.044715 for the tanh form.
constexpr float kGeluC0 = 0.7978845608028654f;
constexpr float kGeluC1 = 0.7978845608028654f * 0.044715f;

// 1 / x on the special-function unit (relative error about 2^-23).
__device__ __forceinline__ float fast_rcp(float x) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// The activation of two pre-activation values, packed as f32x2.
//   sigmoid form  z·σ(1.702 z) = ½z + ½z·tanh(0.851 z), using the identity
//                 σ(a) = (1 + tanh(a/2)) / 2: one hardware tanh per value
//                 (relative error about 2^-11; this form is the throughput one);
//   tanh form     ½z (1 + tanh(u)), u = √(2/π) (z + 0.044715 z³), evaluated
//                 as z·σ(2u) = z / (1 + 2^(-2u·log2 e)) with the hardware
//                 exp2 and reciprocal (relative error about 1e-6), so the bf16
//                 activations round as the fp32 definition does — the
//                 decoders use this form, and a 2^-11 error in every layer's
//                 MLP activations shows up in 12-layer logits;
//   erf form      ½z (1 + erf(z / √2)) (CUDA's erff).
template <int kAct>
__device__ __forceinline__ uint64_t act2(uint64_t z) {
  if constexpr (kAct == ND_ACT_GELU_SIGMOID) {
    const uint64_t hz = f2_mul(z, f2_pack(0.5f, 0.5f));
    const uint64_t u = f2_mul(z, f2_pack(0.851f, 0.851f));
    float u0, u1;
    f2_unpack(u, u0, u1);
    return f2_fma(hz, f2_pack(tanh_approx(u0), tanh_approx(u1)), hz);
  } else if constexpr (kAct == ND_ACT_GELU_TANH) {
    constexpr float kM2Log2e = -2.0f * 1.4426950408889634f;
    const uint64_t c = f2_fma(f2_mul(z, z), f2_pack(kGeluC1 * kM2Log2e, kGeluC1 * kM2Log2e),
                              f2_pack(kGeluC0 * kM2Log2e, kGeluC0 * kM2Log2e));
    float t0, t1, z0, z1;
    f2_unpack(f2_mul(c, z), t0, t1);   // -2u·log2 e
    f2_unpack(z, z0, z1);
    return f2_pack(z0 * fast_rcp(1.f + fast_exp2(t0)), z1 * fast_rcp(1.f + fast_exp2(t1)));
  } else if constexpr (kAct == ND_ACT_GELU_ERF) {
    float z0, z1;
    f2_unpack(z, z0, z1);
    return f2_pack(0.5f * z0 * (1.f + erff(z0 * 0.7071067811865476f)),
                   0.5f * z1 * (1.f + erff(z1 * 0.7071067811865476f)));
  } else {
    return z;
  }
}
template <int kAct>
__device__ __forceinline__ float act1(float z) {
  float a, b;
  f2_unpack(act2<kAct>(f2_pack(z, 0.f)), a, b);
  return a;
}

// The residual segment of one output row for one 32-column chunk, as f32x2
// pairs; requested before the accumulators are read so the loads overlap.
// Only the 16-byte path (see store_chunk) uses it.
__device__ __forceinline__ void load_residual_chunk(uint64_t (&res)[16], const void* __restrict__ residual,
                                                    int residual_f32, int m, int M, int col0, int N,
                                                    int vec) {
  if (vec && col0 + 32 <= N && m < M) {
    const size_t idx = static_cast<size_t>(m) * N + col0;
    {
      if (residual_f32) {
        const float4* rp = reinterpret_cast<const float4*>(static_cast<const float*>(residual) + idx);
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          const float4 rv = rp[q];
          res[2 * q] = f2_pack(rv.x, rv.y);
          res[2 * q + 1] = f2_pack(rv.z, rv.w);
        }
      } else {
        // bf16 -> fp32 is exact: the 16 bits become the high half of the word
        const uint4* rp = reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(residual) + idx);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const uint4 rv = rp[q];
          const uint32_t w[4] = {rv.x, rv.y, rv.z, rv.w};
#pragma unroll
          for (int h = 0; h < 4; ++h)
            res[4 * q + h] = f2_pack(__uint_as_float(w[h] << 16), __uint_as_float(w[h] & 0xffff0000u));
        }
      }
    }
  }
}

// One 32-column chunk of one output row: y = act(acc + bias) + residual, the
// residual taken from `res` (load_residual_chunk) on the 16-byte path.
// `vec` says the row segments may be moved in 16-byte pieces (N % 8 == 0 and
// 16-byte aligned pointers); the ragged last chunk goes column by column.
template <bool kOutF32, int kAct, bool kRes>
__device__ __forceinline__ void store_chunk(const uint32_t (&r)[32], const uint64_t (&res)[16],
                                            const float* __restrict__ bias,
                                            const void* __restrict__ residual, int residual_f32,
                                            void* __restrict__ Y, int m, int M, int col0, int N,
                                            int vec) {
  if (vec && col0 + 32 <= N) {
    const size_t idx = static_cast<size_t>(m) * N + col0;
    uint64_t z[16];
#pragma unroll
    for (int q = 0; q < 16; ++q) z[q] = f2_pack(__uint_as_float(r[2 * q]), __uint_as_float(r[2 * q + 1]));
    if (bias != nullptr) {
      // every lane reads the same 128 bytes: a broadcast from L1
      const float4* b4 = reinterpret_cast<const float4*>(bias + col0);
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const float4 bb = __ldg(b4 + q);
        z[2 * q] = f2_add(z[2 * q], f2_pack(bb.x, bb.y));
        z[2 * q + 1] = f2_add(z[2 * q + 1], f2_pack(bb.z, bb.w));
      }
    }
#pragma unroll
    for (int q = 0; q < 16; ++q) z[q] = act2<kAct>(z[q]);
    if (m >= M) return;
    if constexpr (kRes) {
#pragma unroll
      for (int q = 0; q < 16; ++q) z[q] = f2_add(z[q], res[q]);
    }
    if constexpr (kOutF32) {
      float4* yp = reinterpret_cast<float4*>(static_cast<float*>(Y) + idx);
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        float a, b, c, d;
        f2_unpack(z[2 * q], a, b);
        f2_unpack(z[2 * q + 1], c, d);
        yp[q] = make_float4(a, b, c, d);
      }
    } else {
      uint4* yp = reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(Y) + idx);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        uint32_t w[4];
#pragma unroll
        for (int h = 0; h < 4; ++h) {
          float lo, hi;
          f2_unpack(z[4 * q + h], lo, hi);
          w[h] = pack_bf16x2(lo, hi);
        }
        yp[q] = make_uint4(w[0], w[1], w[2], w[3]);
      }
    }
  } else {
    if (m >= M) return;
    const size_t idx = static_cast<size_t>(m) * N + col0;
#pragma unroll
    for (int e = 0; e < 32; ++e) {
      const int n = col0 + e;
      if (n >= N) continue;
      float z = __uint_as_float(r[e]);
      if (bias != nullptr) z += __ldg(bias + n);
      z = act1<kAct>(z);
      if constexpr (kRes)
        z += residual_f32 ? static_cast<const float*>(residual)[idx + e]
                          : __bfloat162float(static_cast<const __nv_bfloat16*>(residual)[idx + e]);
      if constexpr (kOutF32) static_cast<float*>(Y)[idx + e] = z;
      else static_cast<__nv_bfloat16*>(Y)[idx + e] = __float2bfloat16_rn(z);
    }
  }
}

// One 32-column chunk of the bf16 output for a warp's 32 rows (thread = row),
// y = act(acc + bias): the bias comes from the tile's copy in shared memory
// (bias_s, a broadcast read) and the rows go out through the warp's staging
// buffer, so that each store instruction writes 8 whole 64-byte row segments
// (16 full sectors) instead of 32 half sectors.  Needs the 16-byte path
// (vec, col0 + 32 <= N).
template <int kAct, bool kKv>
__device__ __forceinline__ void store_chunk_staged(const uint32_t (&r)[32], uint32_t bias_s,
                                                   bool has_bias, uint32_t stg,
                                                   __nv_bfloat16* __restrict__ Y, int m_base,
                                                   int lane, int M, int col0, int N,
                                                   const KvOut& kv) {
  uint64_t z[16];
#pragma unroll
  for (int q = 0; q < 16; ++q) z[q] = f2_pack(__uint_as_float(r[2 * q]), __uint_as_float(r[2 * q + 1]));
  if (has_bias) {
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      float4 bb;
      asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
                   : "=f"(bb.x), "=f"(bb.y), "=f"(bb.z), "=f"(bb.w)
                   : "r"(bias_s + q * 16));
      z[2 * q] = f2_add(z[2 * q], f2_pack(bb.x, bb.y));
      z[2 * q + 1] = f2_add(z[2 * q + 1], f2_pack(bb.z, bb.w));
    }
  }
#pragma unroll
  for (int q = 0; q < 16; ++q) z[q] = act2<kAct>(z[q]);
  const uint32_t row_s = stg + static_cast<uint32_t>(lane) * kStagePitch;
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    uint32_t w[4];
#pragma unroll
    for (int h = 0; h < 4; ++h) {
      float lo, hi;
      f2_unpack(z[4 * q + h], lo, hi);
      w[h] = pack_bf16x2(lo, hi);
    }
    st_shared_v4(row_s + q * 16, w[0], w[1], w[2], w[3]);
  }
  __syncwarp();
  // read back 8 rows x 4 pieces per instruction, consecutive lanes along a
  // row, so each global store instruction writes 8 whole 64-byte segments.
  // (The 80-byte pitch makes the writes conflict-free and costs the reads
  // one 2-way conflict per quarter-warp; measured faster than a conflict-free
  // XOR swizzle and than reading 8 rows at one piece per quarter-warp.)
  const int piece = lane & 3;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int row = j * 8 + (lane >> 2);
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "r"(stg + row * kStagePitch + piece * 16));
    const int m = m_base + row;
    if (m < M) {
      *reinterpret_cast<uint4*>(Y + static_cast<size_t>(m) * N + col0 + piece * 8) = v;
      if (kKv && col0 >= kv.dl) {
        // a K or V column block: the same 16 bytes into the head-major cache
        // at token (b, s) = (m / S, m % S), head and dims of the column
        const int c = col0 - kv.dl;
        const int is_v = c >= kv.dl ? 1 : 0;
        const int hc = c - is_v * kv.dl;
        const int b = m / kv.S, s = m - b * kv.S;
        int head = hc >> 6, seq = b;
        __nv_bfloat16* base = is_v ? kv.v : kv.k;
        if (kv.n_peers > 0) {
          // the owning rank's cache (a select over the unrolled peer list,
          // so the pointer array stays in the parameter space)
          const int q = head / kv.H;
          head -= q * kv.H;
          seq += kv.b0;
#pragma unroll
          for (int j = 0; j < kKvMaxPeers; ++j)
            if (j == q) base = is_v ? kv.v_peer[j] : kv.k_peer[j];
        }
        const size_t idx =
            (static_cast<size_t>(seq * kv.H + head) * kv.L_max + kv.pos0 + s) * 64 + (hc & 63) +
            piece * 8;
        *reinterpret_cast<uint4*>(base + idx) = v;
      }
    }
  }
  __syncwarp();  // the buffer is rewritten by the next chunk
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

template <int BN, bool kOutF32, int kAct, bool kRes, bool kKv>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_w,
                const float* __restrict__ bias, const void* __restrict__ residual,
                int residual_f32, void* __restrict__ Y, int M, int N, int K, int vec,
                int* __restrict__ err_word, KvOut kv) {
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
    // Thread = accumulator row = TMEM lane.  Per 32-column chunk the row's
    // fp32 accumulators come out of tensor memory into registers
    // (tcgen05.ld 32x32b) and store_chunk finishes and writes them.  Two warps
    // per TMEM lane quarter: warp 4+q takes the even chunks of rows
    // 32q..32q+31, warp 8+q the odd ones; the next chunk's TMEM load is in
    // flight while one is processed.
    const int quarter = warp & 3;
    const int half = (warp >> 2) - 1;
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    bool ok = true;
    int lt = 0;
    auto prefetch_residual = [&](int t) {
      int pm, pn;
      tile_coords(t, m_tiles, n_tiles, pm, pn);
      const int row = pm * kBM + quarter * 32 + lane;
      const int chunks = min(BN / 32, (N - pn * BN + 31) / 32);
      if (row >= M) return;
      const size_t esz = residual_f32 ? 4 : 2;
      const char* base =
          static_cast<const char*>(residual) + (static_cast<size_t>(row) * N + pn * BN) * esz;
      for (int c = half; c < chunks; c += 2) prefetch_l2(base + c * 32 * esz);
    };
    if constexpr (kRes)
      if (static_cast<int>(blockIdx.x) < n_tiles_total) prefetch_residual(blockIdx.x);
    // bf16 path without residual: lane's float4 of the bias for tile t, chunk
    // half + 2 * (lane >> 3), columns (lane & 7) * 4 .. + 3 of that chunk
    auto load_bias4 = [&](int t) {
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      if (kRes || kOutF32 || bias == nullptr || !vec || t >= n_tiles_total) return v;
      int m2, n2;
      tile_coords(t, m_tiles, n_tiles, m2, n2);
      const int col = n2 * BN + (half + 2 * (lane >> 3)) * 32 + (lane & 7) * 4;
      if (col + 4 <= N && (half + 2 * (lane >> 3)) * 32 < BN)
        v = __ldg(reinterpret_cast<const float4*>(bias + col));
      return v;
    };
    float4 bias_cur = load_bias4(blockIdx.x);
    float4 bias_next = load_bias4(blockIdx.x + gridDim.x);
    for (int t = blockIdx.x; t < n_tiles_total; t += gridDim.x, ++lt) {
      int m_blk, n_blk;
      tile_coords(t, m_tiles, n_tiles, m_blk, n_blk);
      const int b = lt & 1;
      const int m = m_blk * kBM + quarter * 32 + lane;  // this thread's output row
      const int n_chunks = min(BN / 32, (N - n_blk * BN + 31) / 32);
      // The next tile's residual row segments go to L2 while this tile is
      // finished, so the epilogue's loads do not wait on DRAM.
      if constexpr (kRes)
        if (t + static_cast<int>(gridDim.x) < n_tiles_total) prefetch_residual(t + gridDim.x);
      if (!warp_wait(&bars->acc_full[b], (lt >> 1) & 1, abort_flag)) { ok = false; break; }
      tc_fence_after();
      const uint32_t acc = tmem + lane_base + b * BN;
      if constexpr (kRes) {
        // One TMEM buffer: the registers go to the residual segment instead,
        // whose global loads are the longer wait.
#pragma unroll 1
        for (int c = half; c < n_chunks; c += 2) {
          const int col0 = n_blk * BN + c * 32;
          uint32_t r[32];
          uint64_t res[16];
          tmem_ld32(acc + c * 32, r);
          load_residual_chunk(res, residual, residual_f32, m, M, col0, N, vec);
          tmem_ld_wait();
          store_chunk<kOutF32, kAct, true>(r, res, bias, residual, residual_f32, Y, m, M, col0, N, vec);
        }
      } else {
        const uint64_t no_res[16] = {};
        uint32_t r[2][32];
        if (half < n_chunks) tmem_ld32(acc + half * 32, r[0]);
        // bf16 output: this warp's bias for the tile (its chunks c = half + 2j,
        // 32 values each) into its own shared-memory slice, one float4 per
        // lane, the next tile's float4 already loaded; no other warp reads it
        const uint32_t wbias = smem_u32(smem + Cfg::kOffBias) + (warp - 4) * kBiasWarpBytes;
        if constexpr (!kOutF32) {
          st_shared_v4(wbias + lane * 16, __float_as_uint(bias_cur.x), __float_as_uint(bias_cur.y),
                       __float_as_uint(bias_cur.z), __float_as_uint(bias_cur.w));
          bias_cur = bias_next;
          bias_next = load_bias4(t + 2 * static_cast<int>(gridDim.x));
          __syncwarp();
        }
        const uint32_t stg = smem_u32(smem + Cfg::kOffStaging) + (warp - 4) * kStageWarpBytes;
        const int m_base = m_blk * kBM + quarter * 32;
#pragma unroll 1
        for (int c = half, k = 0; c < n_chunks; c += 2, ++k) {
          const int col0 = n_blk * BN + c * 32;
          tmem_ld_wait();
          // (k & 1) selects the register buffer; both branches are unrolled so
          // the buffers stay in registers
#define ND_EPILOGUE_CHUNK(CUR, NXT)                                                        \
          {                                                                               \
            if (c + 2 < n_chunks) tmem_ld32(acc + (c + 2) * 32, r[NXT]);                  \
            if (!kOutF32 && vec && col0 + 32 <= N)                                        \
              store_chunk_staged<kAct, kKv>(r[CUR], wbias + k * 128, bias != nullptr, stg, \
                                       static_cast<__nv_bfloat16*>(Y), m_base, lane, M,   \
                                       col0, N, kv);                                      \
            else                                                                          \
              store_chunk<kOutF32, kAct, false>(r[CUR], no_res, bias, residual, residual_f32, \
                                                Y, m, M, col0, N, vec);                   \
          }
          if (k & 1) ND_EPILOGUE_CHUNK(1, 0) else ND_EPILOGUE_CHUNK(0, 1)
#undef ND_EPILOGUE_CHUNK
        }
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

template <int BN, bool kOutF32, int kAct, bool kRes, bool kKv = false>
cudaError_t launch_typed(cudaStream_t stream, const CUtensorMap& ta, const CUtensorMap& tw,
                         const float* bias, const void* residual, bool residual_f32, void* Y,
                         int M, int N, int K, int sms, const KvOut& kv) {
  using Cfg = GemmCfg<BN>;
  auto kern = gemm_kernel<BN, kOutF32, kAct, kRes, kKv>;
  cudaError_t e =
      cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmemBytes);
  if (e != cudaSuccess) return e;
  const int tiles = ((M + kBM - 1) / kBM) * ((N + BN - 1) / BN);
  dim3 grid(tiles < sms ? tiles : sms);
  auto al16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  const int vec = (N % 8 == 0) && al16(Y) && al16(residual) && al16(bias) ? 1 : 0;
  kern<<<grid, kThreads, Cfg::kSmemBytes, stream>>>(ta, tw, bias, residual, residual_f32 ? 1 : 0,
                                                    Y, M, N, K, vec, device_error_word(), kv);
  return cudaGetLastError();
}

template <int BN, bool kOutF32>
cudaError_t launch_act(int act, cudaStream_t stream, const CUtensorMap& ta, const CUtensorMap& tw,
                       const float* bias, const void* residual, bool residual_f32, void* Y, int M,
                       int N, int K, int sms, const KvOut& kv) {
  switch (act) {
    case ND_ACT_GELU_SIGMOID:
      return residual != nullptr
                 ? launch_typed<BN, kOutF32, ND_ACT_GELU_SIGMOID, true>(stream, ta, tw, bias, residual, residual_f32, Y, M, N, K, sms, kv)
                 : launch_typed<BN, kOutF32, ND_ACT_GELU_SIGMOID, false>(stream, ta, tw, bias, residual, residual_f32, Y, M, N, K, sms, kv);
    case ND_ACT_GELU_TANH:
      return residual != nullptr
                 ? launch_typed<BN, kOutF32, ND_ACT_GELU_TANH, true>(stream, ta, tw, bias, residual, residual_f32, Y, M, N, K, sms, kv)
                 : launch_typed<BN, kOutF32, ND_ACT_GELU_TANH, false>(stream, ta, tw, bias, residual, residual_f32, Y, M, N, K, sms, kv);
    case ND_ACT_GELU_ERF:
      return residual != nullptr
                 ? launch_typed<BN, kOutF32, ND_ACT_GELU_ERF, true>(stream, ta, tw, bias, residual, residual_f32, Y, M, N, K, sms, kv)
                 : launch_typed<BN, kOutF32, ND_ACT_GELU_ERF, false>(stream, ta, tw, bias, residual, residual_f32, Y, M, N, K, sms, kv);
    default:
      if (residual != nullptr)
        return launch_typed<BN, kOutF32, ND_ACT_NONE, true>(stream, ta, tw, bias, residual, residual_f32, Y, M, N, K, sms, kv);
      if constexpr (!kOutF32)
        if (kv.k != nullptr)  // the QKV projection that also fills the caches
          return launch_typed<BN, false, ND_ACT_NONE, false, true>(stream, ta, tw, bias, residual, residual_f32, Y, M, N, K, sms, kv);
      return launch_typed<BN, kOutF32, ND_ACT_NONE, false>(stream, ta, tw, bias, residual, residual_f32, Y, M, N, K, sms, kv);
  }
}

template <bool kOutF32>
cudaError_t launch_bn(int BN, int act, cudaStream_t stream, const CUtensorMap& ta,
                      const CUtensorMap& tw, const float* bias, const void* residual,
                      bool residual_f32, void* Y, int M, int N, int K, int sms, const KvOut& kv) {
  if (BN == 256)
    return launch_act<256, kOutF32>(act, stream, ta, tw, bias, residual, residual_f32, Y, M, N, K, sms, kv);
  if (BN == 128)
    return launch_act<128, kOutF32>(act, stream, ta, tw, bias, residual, residual_f32, Y, M, N, K, sms, kv);
  return launch_act<64, kOutF32>(act, stream, ta, tw, bias, residual, residual_f32, Y, M, N, K, sms, kv);
}

// ---- skinny path: M <= 32 rows (decode-time activations) -------------------
// A 128-row tensor-core tile would compute mostly padding and leave N/BN
// CTAs streaming the weights; with M <= 32 the op is bound by reading W, and
// at decode sizes (a few MB of W) by the latency of that read.
// A cluster of `ksplit` CTAs owns 8 rows of W; each CTA takes a contiguous
// 1/ksplit of the K range and its 8 warps split that.  Each lane reads 16
// bytes (8 k values) of one W row and of each A row per 32-wide k chunk and
// feeds two mma.m16n8k16 steps; the k values are assigned to fragment
// positions by the same permutation for A and W, which leaves every dot
// product intact.  The warps' 16x8 (or 32x8) partial tiles are summed
// through shared memory, the cluster's tiles by CTA rank 0 through
// distributed shared memory (rank order, so the result does not depend on
// timing), and the epilogue adds bias, activation and residual like the main
// path.  ksplit is chosen so that a warp's loads for its whole share of K go
// out together (one round trip to memory).
// Under programmatic dependent launch the first batch of W loads is issued
// before pdl_wait(): W is a constant operand; A and the residual are read
// after it.
template <int kMB, bool kOutF32, int kAct, bool kRes>
__global__ void __launch_bounds__(kSkinnyWarps * 32)
    skinny_gemm_kernel(const __nv_bfloat16* __restrict__ A, const __nv_bfloat16* __restrict__ W,
                       const float* __restrict__ bias, const void* __restrict__ residual,
                       int residual_f32, void* __restrict__ Y, int M, int N, int K) {
  const int ksplit = static_cast<int>(cluster_nctarank());
  const int kr = static_cast<int>(cluster_ctarank());
  const int n0 = (blockIdx.x / ksplit) * 8;
  __shared__ float red[kSkinnyWarps][kMB * 16][8];
  __shared__ float part[kMB * 16 * 8];
  skinny_tile<kMB>(A, W, M, N, K, n0, ksplit, kr, red, part, true);
  // every CTA of the cluster reaches both barriers (no early exit above)
  if (ksplit > 1) cluster_sync();
  else __syncthreads();
  if (kr == 0) {
    for (int o = threadIdx.x; o < kMB * 16 * 8; o += blockDim.x) {
      const int m = o >> 3, n = n0 + (o & 7);
      float z = part[o];
      for (int r = 1; r < ksplit; ++r) z += ld_dsmem_f32(&part[o], static_cast<uint32_t>(r));
      if (m >= M || n >= N) continue;
      if (bias != nullptr) z += bias[n];
      z = act1<kAct>(z);
      const size_t idx = static_cast<size_t>(m) * N + n;
      if constexpr (kRes)
        z += residual_f32 ? static_cast<const float*>(residual)[idx]
                          : __bfloat162float(static_cast<const __nv_bfloat16*>(residual)[idx]);
      if constexpr (kOutF32) static_cast<float*>(Y)[idx] = z;
      else static_cast<__nv_bfloat16*>(Y)[idx] = __float2bfloat16_rn(z);
    }
  }
  // rank 0 has read every peer's tile before any CTA of the cluster exits
  if (ksplit > 1) cluster_sync();
}

template <int kMB, bool kOutF32, int kAct>
cudaError_t launch_skinny_act(cudaStream_t stream, const __nv_bfloat16* A, const __nv_bfloat16* W,
                              const float* bias, const void* residual, bool residual_f32, void* Y,
                              int M, int N, int K) {
  const int ks = skinny_ksplit(N, K, current_sm_count());
  const dim3 grid(((N + 7) / 8) * ks);
  if (residual != nullptr)
    return launch_ex(skinny_gemm_kernel<kMB, kOutF32, kAct, true>, grid, dim3(kSkinnyWarps * 32), 0,
                     stream, ks, true, A, W, bias, residual, residual_f32 ? 1 : 0, Y, M, N, K);
  return launch_ex(skinny_gemm_kernel<kMB, kOutF32, kAct, false>, grid, dim3(kSkinnyWarps * 32), 0,
                   stream, ks, true, A, W, bias, residual, 0, Y, M, N, K);
}

template <int kMB, bool kOutF32>
cudaError_t launch_skinny(int act, cudaStream_t stream, const __nv_bfloat16* A,
                          const __nv_bfloat16* W, const float* bias, const void* residual,
                          bool residual_f32, void* Y, int M, int N, int K) {
  switch (act) {
    case ND_ACT_GELU_SIGMOID:
      return launch_skinny_act<kMB, kOutF32, ND_ACT_GELU_SIGMOID>(stream, A, W, bias, residual, residual_f32, Y, M, N, K);
    case ND_ACT_GELU_TANH:
      return launch_skinny_act<kMB, kOutF32, ND_ACT_GELU_TANH>(stream, A, W, bias, residual, residual_f32, Y, M, N, K);
    case ND_ACT_GELU_ERF:
      return launch_skinny_act<kMB, kOutF32, ND_ACT_GELU_ERF>(stream, A, W, bias, residual, residual_f32, Y, M, N, K);
    default:
      return launch_skinny_act<kMB, kOutF32, ND_ACT_NONE>(stream, A, W, bias, residual, residual_f32, Y, M, N, K);
  }
}

// ---- LayerNorm-prologue linear for few rows (decode steps) ----------------
// Y = act(LN(x + p + p_bias) · Wᵀ + bias) for M <= 32 rows: the residual add,
// the LayerNorm and the linear layer after it in one kernel, so a decode step
// needs no separate residual + LayerNorm launch.  Persistent: each CTA
//   1. issues the W loads of its first 8-row tile and copies p_bias, gamma and
//      beta to shared memory (constant operands: before the previous kernel
//      has finished, under programmatic dependent launch),
//   2. forms s = x + (p + p_bias), rounded to bf16 as the residual stream
//      (CTA 0 stores it to s_out), and LayerNorm(s) in the arithmetic of the
//      separate residual + LayerNorm kernel (same per-lane order of the
//      sums), into shared memory as the bf16 A operand; a warp per row, the
//      row held in registers, all of its x / p loads in flight together (rows
//      padded by 64 bytes so the 16-byte fragment loads of a quarter-warp hit
//      distinct banks; rows >= M are zero),
//   3. loops over 8-row tiles of W: 8 warps split K, mma.m16n8k16 with the k
//      permutation of the skinny path, and the next tile's W loads issued
//      before this tile's reduction and epilogue, so the latency of the weight
//      stream overlaps them.
constexpr int kLnGemmWarps = 8;
constexpr int kLnGemmBatch = 4;   // k chunks of 32 per warp whose loads go out together
constexpr int kLnGemmVecs = 4;    // 16-byte pieces of a row per lane loaded together

__device__ __forceinline__ void bf16x8_to_f32_(const uint4& u, float (&f)[8]) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(w[i] << 16);
    f[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
  }
}

__device__ __forceinline__ float warp_allsum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ uint4 pack8_bf16(const float (&v)[8]) {
  uint4 r;
  r.x = pack_bf16x2(v[0], v[1]);
  r.y = pack_bf16x2(v[2], v[3]);
  r.z = pack_bf16x2(v[4], v[5]);
  r.w = pack_bf16x2(v[6], v[7]);
  return r;
}

// shared memory: A rows [kMB*16][K + 32] bf16 | params [3][K] f32 | red [8][kMB*16][8] f32
template <int kMB>
__host__ __device__ constexpr size_t ln_gemm_par_offset(int K) {
  return static_cast<size_t>(kMB) * 16 * (K + 32) * 2;
}
template <int kMB>
__host__ __device__ constexpr size_t ln_gemm_red_offset(int K) {
  return ln_gemm_par_offset<kMB>(K) + static_cast<size_t>(3) * K * 4;
}
template <int kMB>
__host__ __device__ constexpr size_t ln_gemm_smem_bytes(int K) {
  return ln_gemm_red_offset<kMB>(K) + static_cast<size_t>(kLnGemmWarps) * kMB * 16 * 8 * 4;
}

template <int kMB, bool kOutF32, int kAct>
__global__ void __launch_bounds__(kLnGemmWarps * 32)
    ln_gemm_kernel(const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ p,
                   const float* __restrict__ p_bias, const float* __restrict__ gamma,
                   const float* __restrict__ beta, float eps, __nv_bfloat16* __restrict__ s_out,
                   const __nv_bfloat16* __restrict__ W, const float* __restrict__ bias,
                   void* __restrict__ Y, int M, int N, int K) {
  extern __shared__ __align__(128) unsigned char ln_smem[];
  const int pitch = K + 32;  // bf16 elements per staged row
  __nv_bfloat16* As = reinterpret_cast<__nv_bfloat16*>(ln_smem);
  float* par = reinterpret_cast<float*>(ln_smem + ln_gemm_par_offset<kMB>(K));  // p_bias|gamma|beta
  float* red = reinterpret_cast<float*>(ln_smem + ln_gemm_red_offset<kMB>(K));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int nblk = (N + 7) / 8;
  const int n_chunks = K / 32;
  constexpr int kStep = kLnGemmWarps * kLnGemmBatch;

  auto load_w = [&](int tile, int c0, uint4 (&wv)[kLnGemmBatch]) {
    const int n = tile * 8 + g;
    const bool ok = n < N;
    const __nv_bfloat16* wrow = W + static_cast<size_t>(ok ? n : 0) * K + t * 8;
#pragma unroll
    for (int u = 0; u < kLnGemmBatch; ++u) {
      const int ch = c0 + u * kLnGemmWarps;
      wv[u] = (ok && ch < n_chunks) ? __ldg(reinterpret_cast<const uint4*>(wrow + ch * 32))
                                    : make_uint4(0, 0, 0, 0);
    }
  };

  int tile = blockIdx.x;
  uint4 wv[kLnGemmBatch];
  if (tile < nblk) load_w(tile, warp, wv);
  const int nvec = K >> 3;  // 16-byte pieces of a row (<= 32 * kLnGemmVecs)
  {
    // p_bias | gamma | beta to shared memory as par[(a * 8 + e) * nvec + c]
    // (array a, element e of piece c): a lane reading its piece's element e
    // and its neighbours' hits consecutive words.  All of a thread's float4
    // loads are issued before the first store (16-byte aligned bases).
    constexpr int kParLoads = (3 * kLnGemmMaxK / 4 + kLnGemmWarps * 32 - 1) / (kLnGemmWarps * 32);
    const int per = K / 4;
    float4 pv[kParLoads];
#pragma unroll
    for (int j = 0; j < kParLoads; ++j) {
      const int i = threadIdx.x + j * kLnGemmWarps * 32;
      const int a = i >= 2 * per ? 2 : (i >= per ? 1 : 0);
      const float* src = a == 0 ? p_bias : (a == 1 ? gamma : beta);
      const float dflt = a == 1 ? 1.f : 0.f;
      pv[j] = (i < 3 * per && src) ? __ldg(reinterpret_cast<const float4*>(src) + (i - a * per))
                                   : make_float4(dflt, dflt, dflt, dflt);
    }
#pragma unroll
    for (int j = 0; j < kParLoads; ++j) {
      const int i = threadIdx.x + j * kLnGemmWarps * 32;
      if (i < 3 * per) {
        const int a = i >= 2 * per ? 2 : (i >= per ? 1 : 0);
        const int k = (i - a * per) * 4;  // element index within the array
        const int c = k >> 3, e = k & 7;
        float* d = par + (a * 8 + e) * nvec + c;
        d[0] = pv[j].x;
        d[nvec] = pv[j].y;
        d[2 * nvec] = pv[j].z;
        d[3 * nvec] = pv[j].w;
      }
    }
  }
  pdl_wait();  // x and p come from earlier kernels
  pdl_trigger();
  __syncthreads();  // params staged

  // prologue: a warp per row, the row's pieces in registers through the
  // three passes (sum, centred sum of squares, normalise), all of its x / p
  // loads in flight together
  for (int m = warp; m < kMB * 16; m += kLnGemmWarps) {
    uint4* arow = reinterpret_cast<uint4*>(As + static_cast<size_t>(m) * pitch);
    if (m >= M) {  // warp-uniform
      for (int c = lane; c < nvec; c += 32) arow[c] = make_uint4(0, 0, 0, 0);
      continue;
    }
    const size_t off = static_cast<size_t>(m) * K;
    uint4 xv[kLnGemmVecs], qv[kLnGemmVecs];
#pragma unroll
    for (int i = 0; i < kLnGemmVecs; ++i) {
      const int c = lane + 32 * i;
      const bool ok = c < nvec;
      xv[i] = ok ? *reinterpret_cast<const uint4*>(x + off + c * 8) : make_uint4(0, 0, 0, 0);
      qv[i] = (ok && p) ? *reinterpret_cast<const uint4*>(p + off + c * 8) : make_uint4(0, 0, 0, 0);
    }
    float v[kLnGemmVecs][8];
    float sum = 0.f;
#pragma unroll
    for (int i = 0; i < kLnGemmVecs; ++i) {
      const int c = lane + 32 * i;
      if (c >= nvec) continue;
      float q[8];
      bf16x8_to_f32_(xv[i], v[i]);
      bf16x8_to_f32_(qv[i], q);
#pragma unroll
      for (int e = 0; e < 8; ++e) v[i][e] += q[e] + par[e * nvec + c];
      const uint4 packed = pack8_bf16(v[i]);
      if (s_out != nullptr && blockIdx.x == 0)
        reinterpret_cast<uint4*>(s_out + off)[c] = packed;
      bf16x8_to_f32_(packed, v[i]);
#pragma unroll
      for (int e = 0; e < 8; ++e) sum += v[i][e];
    }
    const float mu = warp_allsum(sum) / static_cast<float>(K);
    float q2 = 0.f;
#pragma unroll
    for (int i = 0; i < kLnGemmVecs; ++i) {
      if (lane + 32 * i >= nvec) continue;
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float d = v[i][e] - mu;
        q2 += d * d;
      }
    }
    const float rs = rsqrtf(warp_allsum(q2) / static_cast<float>(K) + eps);
#pragma unroll
    for (int i = 0; i < kLnGemmVecs; ++i) {
      const int c = lane + 32 * i;
      if (c >= nvec) continue;
      float o[8];
#pragma unroll
      for (int e = 0; e < 8; ++e)
        o[e] = (v[i][e] - mu) * rs * par[(8 + e) * nvec + c] + par[(16 + e) * nvec + c];
      arow[c] = pack8_bf16(o);
    }
  }
  __syncthreads();

  for (; tile < nblk; tile += gridDim.x) {
    const int n0 = tile * 8;
    // this thread's epilogue bias, fetched before the tile's math
    float bias_o[(kMB * 16 * 8 + kLnGemmWarps * 32 - 1) / (kLnGemmWarps * 32)];
#pragma unroll
    for (int j = 0; j < static_cast<int>(sizeof(bias_o) / sizeof(float)); ++j) {
      const int n = n0 + ((threadIdx.x + j * kLnGemmWarps * 32) & 7);
      bias_o[j] = (bias != nullptr && n < N) ? __ldg(bias + n) : 0.f;
    }
    float c[kMB][4];
#pragma unroll
    for (int mb = 0; mb < kMB; ++mb)
#pragma unroll
      for (int i = 0; i < 4; ++i) c[mb][i] = 0.f;
    for (int c0 = warp; c0 < n_chunks; c0 += kStep) {
      if (c0 != warp) load_w(tile, c0, wv);
#pragma unroll
      for (int u = 0; u < kLnGemmBatch; ++u) {
        const int ch = c0 + u * kLnGemmWarps;
        if (ch >= n_chunks) break;  // warp-uniform
        const uint32_t w[4] = {wv[u].x, wv[u].y, wv[u].z, wv[u].w};
#pragma unroll
        for (int mb = 0; mb < kMB; ++mb) {
          const __nv_bfloat16* a0 = As + static_cast<size_t>(mb * 16 + g) * pitch + ch * 32 + t * 8;
          const uint4 lo = *reinterpret_cast<const uint4*>(a0);
          const uint4 hi = *reinterpret_cast<const uint4*>(a0 + 8 * pitch);
          mma_bf16_16816(c[mb], lo.x, hi.x, lo.y, hi.y, w[0], w[1]);
          mma_bf16_16816(c[mb], lo.z, hi.z, lo.w, hi.w, w[2], w[3]);
        }
      }
    }
    // the next tile's first W loads overlap this tile's reduction and epilogue
    if (tile + static_cast<int>(gridDim.x) < nblk) load_w(tile + gridDim.x, warp, wv);
    float* rw = red + warp * (kMB * 16 * 8);
#pragma unroll
    for (int mb = 0; mb < kMB; ++mb) {
      rw[(mb * 16 + g) * 8 + 2 * t] = c[mb][0];
      rw[(mb * 16 + g) * 8 + 2 * t + 1] = c[mb][1];
      rw[(mb * 16 + g + 8) * 8 + 2 * t] = c[mb][2];
      rw[(mb * 16 + g + 8) * 8 + 2 * t + 1] = c[mb][3];
    }
    __syncthreads();
#pragma unroll
    for (int j = 0; j < static_cast<int>(sizeof(bias_o) / sizeof(float)); ++j) {
      const int o = threadIdx.x + j * kLnGemmWarps * 32;
      if (o >= kMB * 16 * 8) break;
      const int m = o >> 3, n = n0 + (o & 7);
      if (m >= M || n >= N) continue;
      float z = 0.f;
#pragma unroll
      for (int w = 0; w < kLnGemmWarps; ++w) z += red[w * (kMB * 16 * 8) + o];
      z += bias_o[j];
      z = act1<kAct>(z);
      const size_t idx = static_cast<size_t>(m) * N + n;
      if constexpr (kOutF32) static_cast<float*>(Y)[idx] = z;
      else static_cast<__nv_bfloat16*>(Y)[idx] = __float2bfloat16_rn(z);
    }
    __syncthreads();  // red is rewritten by the next tile
  }
}

template <int kMB, bool kOutF32, int kAct>
cudaError_t launch_ln_gemm_act(cudaStream_t stream, const __nv_bfloat16* x,
                               const __nv_bfloat16* p, const float* p_bias, const float* gamma,
                               const float* beta, float eps, __nv_bfloat16* s_out,
                               const __nv_bfloat16* W, const float* bias, void* Y, int M, int N,
                               int K) {
  auto kernel = ln_gemm_kernel<kMB, kOutF32, kAct>;
  const size_t smem = ln_gemm_smem_bytes<kMB>(K);
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  // per device: the kernel's shared-memory limit, SM count and occupancy at
  // this size (resident CTAs per SM bound the persistent grid)
  struct Entry {
    int dev;
    size_t smem;
    int grid_per_sm, sms;
  };
  static std::mutex mu;
  static std::vector<Entry> cache;
  int per_sm = 0, sms = 0;
  {
    std::lock_guard<std::mutex> lk(mu);
    for (const Entry& c : cache)
      if (c.dev == dev && c.smem == smem) {
        per_sm = c.grid_per_sm;
        sms = c.sms;
      }
    if (per_sm == 0) {
      e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               static_cast<int>(ln_gemm_smem_bytes<kMB>(kLnGemmMaxK)));
      if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
      if (e == cudaSuccess)
        e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, kLnGemmWarps * 32, smem);
      if (e != cudaSuccess) return e;
      if (per_sm < 1) return cudaErrorInvalidConfiguration;
      cache.push_back({dev, smem, per_sm, sms});
    }
  }
  const int nblk = (N + 7) / 8;
  const int grid = nblk < per_sm * sms ? nblk : per_sm * sms;
  return launch_ex(kernel, dim3(grid), dim3(kLnGemmWarps * 32), smem, stream, 1, true, x, p, p_bias,
                   gamma, beta, eps, s_out, W, bias, Y, M, N, K);
}

template <int kMB, bool kOutF32>
cudaError_t launch_ln_gemm_mb(int act, cudaStream_t stream, const __nv_bfloat16* x,
                              const __nv_bfloat16* p, const float* p_bias, const float* gamma,
                              const float* beta, float eps, __nv_bfloat16* s_out,
                              const __nv_bfloat16* W, const float* bias, void* Y, int M, int N,
                              int K) {
  switch (act) {
    case ND_ACT_GELU_SIGMOID:
      return launch_ln_gemm_act<kMB, kOutF32, ND_ACT_GELU_SIGMOID>(stream, x, p, p_bias, gamma, beta, eps, s_out, W, bias, Y, M, N, K);
    case ND_ACT_GELU_TANH:
      return launch_ln_gemm_act<kMB, kOutF32, ND_ACT_GELU_TANH>(stream, x, p, p_bias, gamma, beta, eps, s_out, W, bias, Y, M, N, K);
    case ND_ACT_GELU_ERF:
      return launch_ln_gemm_act<kMB, kOutF32, ND_ACT_GELU_ERF>(stream, x, p, p_bias, gamma, beta, eps, s_out, W, bias, Y, M, N, K);
    default:
      return launch_ln_gemm_act<kMB, kOutF32, ND_ACT_NONE>(stream, x, p, p_bias, gamma, beta, eps, s_out, W, bias, Y, M, N, K);
  }
}

}  // namespace

cudaError_t launch_gemm(cudaStream_t stream, const __nv_bfloat16* A, const __nv_bfloat16* W,
                        const float* bias, const void* residual, bool residual_f32, void* Y,
                        bool out_f32, int M, int N, int K, int act, const char** err_msg,
                        const KvOut& kv) {
  if (M == 0 || N == 0) return cudaSuccess;
  if (K == 0) return cudaErrorInvalidValue;
  if (M <= 32 && K % 32 == 0) {
    // few rows: the weight-streaming path (A and W rows are 16-byte aligned
    // because K % 32 == 0 and the bases are)
    if (M <= 16)
      return out_f32 ? launch_skinny<1, true>(act, stream, A, W, bias, residual, residual_f32, Y, M, N, K)
                     : launch_skinny<1, false>(act, stream, A, W, bias, residual, residual_f32, Y, M, N, K);
    return out_f32 ? launch_skinny<2, true>(act, stream, A, W, bias, residual, residual_f32, Y, M, N, K)
                   : launch_skinny<2, false>(act, stream, A, W, bias, residual, residual_f32, Y, M, N, K);
  }
  int dev = 0, sms = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (e != cudaSuccess) return e;
  sms = limited_sms(sms);
  // Tile width: fewest waves of tiles over the SMs, a wave of 128- or 64-wide
  // tiles counting half or a quarter of a 256-wide one, with a penalty for
  // the narrower tiles (each A tile is reused over fewer columns); ties keep
  // the wider tile.  M = 8192, N = 768 takes 128 (384 tiles in 3 waves of
  // half-width tiles instead of 192 tiles in 2 full-width waves).
  const int m_tiles = (M + kBM - 1) / kBM;
  int BN = 256;
  double best_cost = 0.0;
  for (int bn = 256; bn >= 64; bn >>= 1) {
    const long long tiles = static_cast<long long>(m_tiles) * ((N + bn - 1) / bn);
    const long long waves = (tiles + sms - 1) / sms;
    const double penalty = bn == 256 ? 1.0 : (bn == 128 ? 1.1 : 1.25);
    const double cost = static_cast<double>(waves) * (bn / 256.0) * penalty;
    if (bn == 256 || cost < best_cost * 0.999) {
      best_cost = cost;
      BN = bn;
    }
  }
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
  return out_f32 ? launch_bn<true>(BN, act, stream, ta, tw, bias, residual, residual_f32, Y, M, N, K, sms, kv)
                 : launch_bn<false>(BN, act, stream, ta, tw, bias, residual, residual_f32, Y, M, N, K, sms, kv);
}

cudaError_t launch_ln_gemm(cudaStream_t stream, const __nv_bfloat16* x, const __nv_bfloat16* p,
                           const float* p_bias, const float* gamma, const float* beta, float eps,
                           __nv_bfloat16* s_out, const __nv_bfloat16* W, const float* bias,
                           void* Y, bool out_f32, int M, int N, int K, int act) {
  if (M == 0 || N == 0) return cudaSuccess;
  if (M > kLnGemmMaxRows || K <= 0 || K % 32 != 0 || K > kLnGemmMaxK) return cudaErrorInvalidValue;
  if (M <= 16)
    return out_f32 ? launch_ln_gemm_mb<1, true>(act, stream, x, p, p_bias, gamma, beta, eps, s_out, W, bias, Y, M, N, K)
                   : launch_ln_gemm_mb<1, false>(act, stream, x, p, p_bias, gamma, beta, eps, s_out, W, bias, Y, M, N, K);
  return out_f32 ? launch_ln_gemm_mb<2, true>(act, stream, x, p, p_bias, gamma, beta, eps, s_out, W, bias, Y, M, N, K)
                 : launch_ln_gemm_mb<2, false>(act, stream, x, p, p_bias, gamma, beta, eps, s_out, W, bias, Y, M, N, K);
}

}  // namespace nd
