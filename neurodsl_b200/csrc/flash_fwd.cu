// flash_fwd.cu — causal / non-causal attention prefill on tcgen05 + TMEM + TMA.
//
// Computes, for every (batch, head) of head-major [B][H][S][D] bf16 tensors,
//   O = softmax(Q·Kᵀ·scale [+ causal mask]) · V,  lse = log Σ exp(.),  m = rowmax
// which is flash_attn_fwd! / flash_attn_fwd_cpu_simple! of the reference
// (src/flash_attention.jl:49-69, :113-134) evaluated blockwise with an online
// softmax (the reference's tiled form, :9-46), never materialising S.
//
// Persistent CTAs (one per SM) loop over work items of 256 query rows of one
// head, taken heaviest first in alternating-direction rounds.  An item is two
// 128-row query tiles sharing one stream of K/V tiles (128 keys each); Q is
// double-buffered and the K/V ring runs on across items, so the next item's
// loads overlap the current item's tail.  Warp roles (kHalves = 1, 384
// threads):
//   warps 0..3   softmax of query tile 0 (thread = row = TMEM lane)
//   warps 4..7   softmax of query tile 1
//   warp 8       TMA producer: Q0/Q1 per item, then K/V tiles (kStages ring)
//   warp 9       TMEM allocator + single-thread UMMA issuer
//   warps 10, 11 idle (they complete the control warpgroup)
// With kHalves = 2 every score row is split over two warpgroups that combine
// their row maxima through shared memory (more warps to hide latency); on
// B200 that loses to one warpgroup per tile because the exponential unit,
// not latency, bounds the softmax, so kHalves = 1 is the configuration built.
// TMEM (512 columns), per tile i at base 256·i: S_i [0,128) fp32 scores,
// P_i [128,192) packed bf16 probabilities, O_i [192,256) fp32 accumulator.
// Because P has its own columns, S_i(j+1) = Q_i·K_{j+1}ᵀ is issued as soon as
// softmax i has read S_i(j) (barrier s_free), so the tensor core computes the
// next scores while the softmax computes exponentials.  O_i += P_i·V_j reads
// P_i straight from tensor memory (A operand in TMEM, V an MN-major
// shared-memory operand).
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
constexpr int kHalves = 1;             // warpgroups sharing one score row (1 or 2)
constexpr int kHalfCols = kBN / kHalves;   // score columns per softmax thread
constexpr int kOutCols = kD / kHalves;     // output columns per softmax thread
constexpr int kSoftmaxThreads = 128 * kTiles * kHalves;
constexpr int kThreadsPerTile = 128 * kHalves;   // arrivals per softmax barrier
constexpr int kThreads = kSoftmaxThreads + 128;  // + one control warpgroup
constexpr int kWarpProducer = kSoftmaxThreads / 32;
constexpr int kWarpMma = kWarpProducer + 1;
// Register split.  One half (384 threads): launch gives 168 per thread
// (64512 total), control 72 + softmax 216: 128 x 72 + 256 x 216 = 64512.
// Two halves (640 threads): 96 per thread (61440), 128 x 32 + 512 x 112.
constexpr uint32_t kLaunchRegs = (65536 / kThreads) & ~7u;
constexpr uint32_t kRegsControl = kHalves == 1 ? 72 : 32;
constexpr uint32_t kRegsSoftmax = kHalves == 1 ? 216 : 112;
static_assert(128 * kRegsControl + kSoftmaxThreads * kRegsSoftmax <= kThreads * kLaunchRegs,
              "register split exceeds the launch budget");
constexpr uint32_t kTileBytes = kBM * kD * 2;    // 16 KB (one Q, K or V tile)
constexpr uint32_t kTmemCols = 512;
// TMEM columns of tile i
__host__ __device__ constexpr uint32_t col_s(int i) { return static_cast<uint32_t>(i) * 256u; }
__host__ __device__ constexpr uint32_t col_p(int i) { return col_s(i) + 128u; }
__host__ __device__ constexpr uint32_t col_o(int i) { return col_s(i) + 192u; }
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;
constexpr float kRescaleThreshold = 8.0f;

// shared-memory map (offsets from a 1024-aligned base)
constexpr uint32_t kOffQ = 0;                                   // 2 buffers x 2 x 16 KB
constexpr uint32_t kOffK = kOffQ + 2 * kTiles * kTileBytes;
constexpr uint32_t kOffV = kOffK + kStages * kTileBytes;
constexpr uint32_t kOffBar = kOffV + kStages * kTileBytes;
constexpr uint32_t kOffX = kOffBar + 256;                       // row-max / row-sum exchange
constexpr uint32_t kSmemBytes = kOffX + 8192 + 1024;            // + alignment slack

// Partner exchange between the two column halves of a score row: partial
// maxima (double-buffered by iteration parity) and the final row sums.
struct Exchange {
  float max_part[2][kTiles][kHalves][kBM];
  float sum_part[kTiles][kHalves][kBM];
};
static_assert(sizeof(Exchange) <= 8192, "exchange area");

constexpr uint32_t kIdescS = idesc_bf16_f32(kBM, kBN, false, false);
constexpr uint32_t kIdescO = idesc_bf16_f32(kBM, kD, false, true);

struct Bars {
  uint64_t q_full[2];        // Q tiles of item n land in buffer n & 1
  uint64_t q_empty[2];       // every S of that item has read the buffer
  uint64_t kv_full[kStages];
  uint64_t kv_empty[kStages];
  uint64_t s_full[kTiles];   // S_i(j) written (UMMA commit)
  uint64_t s_free[kTiles];   // S_i(j) read into registers (256 softmax threads)
  uint64_t p_full[kTiles];   // P_i(j) written and O_i rescaled (256 softmax threads)
  uint64_t o_done[kTiles];   // O_i += P_i(j)·V_j complete (UMMA commit)
  uint64_t drained;
  uint32_t tmem_base;
  int abort_flag;
};

__host__ __device__ constexpr int ceil_div(int a, int b) { return (a + b - 1) / b; }

// bf16x2 pack of two non-negative finite floats on the integer pipe: round to
// nearest (halfway cases up) by adding half an output ulp to the fp32 bits,
// then keep the high halves.  The conversion instruction would run on the
// same pipe as the exponentials; these three integer ops do not.
__device__ __forceinline__ uint32_t pack_bf16x2_int(float lo, float hi) {
  const uint32_t a = __float_as_uint(lo) + 0x8000u;
  const uint32_t b = __float_as_uint(hi) + 0x8000u;
  return __byte_perm(a, b, 0x7632);
}
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

// ---- exp2 on the FMA pipe ----------------------------------------------------
// 2^x for x in [-126, 8] by Cody-Waite range reduction and a polynomial:
// x = n + f with n = round(x) (the 1.5·2^23 magic-add rounding, exact for
// |x| < 2^22) and f in [-0.5, 0.5]; 2^f from a degree-3 minimax polynomial
// (coefficients computed for this kernel with the Remez exchange algorithm,
// minimising relative error on [-0.5, 0.5]: max 7.5e-5, far below the 2^-9
// rounding of the bf16 probabilities); 2^n is added into the exponent field.
constexpr float kExpC0 = 0.99992806f;
constexpr float kExpC1 = 0.69326097f;
constexpr float kExpC2 = 0.24261113f;
constexpr float kExpC3 = 0.05517167f;
constexpr float kRoundMagic = 12582912.0f;  // 1.5 * 2^23
// Pairs out of every 8 whose exponentials use the polynomial.  Measured on
// B200 at head_dim 64 the softmax is bound by instruction issue and latency,
// not by the exponential unit (which sustains 16/clk/SM), so moving work to
// the FMA pipe only adds instructions: 0 is the fastest setting.
constexpr int kPolyPairsPer8 = 0;

// Probabilities for 2·kHalfCols/2 scores: p = 2^(s·scale - m) packed to bf16
// in pk, row-sum partials accumulated in acc (four f32x2 chains).
template <int kPoly>
__device__ __forceinline__ void exp2_pairs(const float* sv, uint64_t scale2, uint64_t negm2,
                                           uint32_t* pk, uint64_t* acc) {
  const uint64_t magic2 = f2_pack(kRoundMagic, kRoundMagic);
  const uint64_t c0 = f2_pack(kExpC0, kExpC0), c1 = f2_pack(kExpC1, kExpC1);
  const uint64_t c2 = f2_pack(kExpC2, kExpC2), c3 = f2_pack(kExpC3, kExpC3);
#pragma unroll
  for (int c = 0; c < kHalfCols; c += 2) {
    const int q = c >> 1;
    float x0, x1, p0, p1;
    f2_unpack(f2_fma(f2_pack(sv[c], sv[c + 1]), scale2, negm2), x0, x1);
    if ((q & 7) < kPoly) {
      const uint64_t x2 = f2_pack(fmaxf(x0, -126.f), fmaxf(x1, -126.f));
      const uint64_t t2 = f2_add(x2, magic2);         // magic + round(x)
      const uint64_t f2 = f2_add(x2, f2_sub(magic2, t2));  // x - round(x)
      uint64_t pp = f2_fma(f2, c3, c2);
      pp = f2_fma(pp, f2, c1);
      pp = f2_fma(pp, f2, c0);
      float t0, t1;
      f2_unpack(t2, t0, t1);
      f2_unpack(pp, p0, p1);
      // low bits of t hold round(x); shifting by 23 drops the magic's bits
      p0 = __uint_as_float(__float_as_uint(p0) + (__float_as_uint(t0) << 23));
      p1 = __uint_as_float(__float_as_uint(p1) + (__float_as_uint(t1) << 23));
    } else {
      p0 = fast_exp2(x0);
      p1 = fast_exp2(x1);
    }
    acc[q & 3] = f2_add(acc[q & 3], f2_pack(p0, p1));
    pk[q] = pack_bf16x2_int(p0, p1);
  }
}

// One unit of work: 256 query rows (two tiles) of one (batch, head).
struct WorkItem {
  int blk;        // which 256-row block of the sequence
  int bh;         // batch * H + head
  int n_kv[kTiles];
  int n_total;    // K/V tiles streamed for the item (the last tile needs the most)
};

template <bool kCausal>
__device__ __forceinline__ WorkItem decode_item(int k, int BH, int n_blk, int n_k) {
  WorkItem w;
  // Heavy items first: with a causal mask the last query rows see the most keys.
  w.blk = kCausal ? (n_blk - 1 - k / BH) : k / BH;
  w.bh = k % BH;
#pragma unroll
  for (int i = 0; i < kTiles; ++i) {
    const int qt = w.blk * kTiles + i;
    w.n_kv[i] = kCausal ? min(qt + 1, n_k) : n_k;
  }
  w.n_total = w.n_kv[kTiles - 1];
  return w;
}

// Where one (batch, head)'s rows live.  Q, K and V are read through 4-D
// tensor maps whose dims are {64, S, H, B} (head-major) or {64, H, S, B}
// (token-major: rows of all heads interleaved, as a projection writes them);
// either way a box is 128 rows of 128 bytes, the same shared-memory tile.
struct FlashLayout {
  int H;                 // heads; bh = b * H + h
  int q_token_major;     // Q map dims {64, H, S, B}
  int kv_token_major;    // K and V maps dims {64, H, S, B}
  long long o_s, o_h, o_b;  // output element strides of a row, a head, a batch
};

// 128 rows starting at `row` of head h, batch b, into one shared tile.
__device__ __forceinline__ void load_rows(const CUtensorMap* map, uint64_t* bar, void* dst,
                                          int row, int h, int b, int token_major) {
  if (token_major)
    tma_load_4d(map, bar, dst, 0, h, row, b);
  else
    tma_load_4d(map, bar, dst, 0, row, h, b);
}

// The n-th item of CTA `cta` out of `grid` persistent CTAs: items are visited
// in rounds of `grid`, alternating direction so each CTA's heavy and light
// items pair up (the cost list is sorted heaviest first).
__device__ __forceinline__ int item_of(int n, int cta, int grid) {
  return n * grid + ((n & 1) ? (grid - 1 - cta) : cta);
}

// kStrided: Q/K/V through 4-D maps and O through FlashLayout strides; the
// contiguous head-major case keeps 3-D maps {64, S, B·H} and bh·S row offsets.
template <bool kCausal, bool kOutF32, bool kStrided>
__global__ void __launch_bounds__(kThreads, 1)
    flash_fwd_kernel(const __grid_constant__ CUtensorMap tm_q,
                     const __grid_constant__ CUtensorMap tm_k,
                     const __grid_constant__ CUtensorMap tm_v, void* __restrict__ out,
                     const FlashLayout lay,
                     float* __restrict__ lse_out, float* __restrict__ max_out, int BH, int Sq,
                     int Sk, float scale_log2, int* __restrict__ err_word) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  Bars* bars = reinterpret_cast<Bars*>(smem + kOffBar);
  volatile int* abort_flag = &bars->abort_flag;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int n_blk = ceil_div(Sq, kRowsPerCta);
  const int n_k = ceil_div(Sk, kBN);
  const int n_items = n_blk * BH;
  const int cta = static_cast<int>(blockIdx.x);
  const int grid = static_cast<int>(gridDim.x);

  if (threadIdx.x == 0) {
    for (int b = 0; b < 2; ++b) {
      mbar_init(&bars->q_full[b], 1);
      mbar_init(&bars->q_empty[b], 1);
    }
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&bars->kv_full[s], 1);
      mbar_init(&bars->kv_empty[s], 1);
    }
    for (int i = 0; i < kTiles; ++i) {
      mbar_init(&bars->s_full[i], 1);
      mbar_init(&bars->s_free[i], kThreadsPerTile);
      mbar_init(&bars->p_full[i], kThreadsPerTile);
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
    regs_decrease<kRegsControl>();
    if (elect_one()) {
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
      int kv_it = 0;  // K/V tiles loaded so far (ring position)
      int n = 0;
      bool ok = true;
      for (int k; ok && (k = item_of(n, cta, grid)) < n_items; ++n) {
        const WorkItem w = decode_item<kCausal>(k, BH, n_blk, n_k);
        const int qb = n & 1;
        if (n >= 2 && !mbar_wait(&bars->q_empty[qb], ((n >> 1) - 1) & 1, abort_flag)) {
          ok = false;
          break;
        }
        const int h = kStrided ? w.bh % lay.H : 0, b = kStrided ? w.bh / lay.H : 0;
        mbar_arrive_expect_tx(&bars->q_full[qb], kTiles * kTileBytes);
        for (int i = 0; i < kTiles; ++i) {
          void* dst = smem + kOffQ + (qb * kTiles + i) * kTileBytes;
          const int row = w.blk * kRowsPerCta + i * kBM;
          if constexpr (kStrided)
            load_rows(&tm_q, &bars->q_full[qb], dst, row, h, b, lay.q_token_major);
          else
            tma_load_3d(&tm_q, &bars->q_full[qb], dst, 0, row, w.bh);
        }
        for (int j = 0; j < w.n_total; ++j, ++kv_it) {
          const int s = kv_it % kStages;
          if (kv_it >= kStages &&
              !mbar_wait(&bars->kv_empty[s], ((kv_it / kStages) - 1) & 1, abort_flag)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&bars->kv_full[s], 2 * kTileBytes);
          if constexpr (kStrided) {
            load_rows(&tm_k, &bars->kv_full[s], smem + kOffK + s * kTileBytes, j * kBN, h, b,
                      lay.kv_token_major);
            load_rows(&tm_v, &bars->kv_full[s], smem + kOffV + s * kTileBytes, j * kBN, h, b,
                      lay.kv_token_major);
          } else {
            tma_load_3d(&tm_k, &bars->kv_full[s], smem + kOffK + s * kTileBytes, 0, j * kBN, w.bh);
            tma_load_3d(&tm_v, &bars->kv_full[s], smem + kOffV + s * kTileBytes, 0, j * kBN, w.bh);
          }
        }
      }
      if (!ok) raise_abort(abort_flag, err_word, kDevErrTimeoutProducer);
      // Drain: every issued copy lands before the CTA may exit.
      for (int m = (n > 2 ? n - 2 : 0); m < n; ++m)
        (void)mbar_wait(&bars->q_full[m & 1], (m >> 1) & 1, abort_flag);
      for (int j = (kv_it > kStages ? kv_it - kStages : 0); j < kv_it; ++j)
        (void)mbar_wait(&bars->kv_full[j % kStages], (j / kStages) & 1, abort_flag);
    }
  } else if (warp == kWarpMma) {
    // ---------------------------------------------------------- UMMA issuer
    regs_decrease<kRegsControl>();
    if (elect_one()) {
      const uint32_t sQ = smem_u32(smem + kOffQ);
      const uint32_t sK = smem_u32(smem + kOffK);
      const uint32_t sV = smem_u32(smem + kOffV);
      bool ok = true;
      int kv_base = 0;            // ring position of the item's first K/V tile
      int kv_ready = -1;          // highest ring position whose kv_full was observed
      int s_cnt[kTiles] = {0, 0};   // S_i products issued so far
      int pv_cnt[kTiles] = {0, 0};  // O_i products issued so far
      auto wait_kv = [&](int it) -> bool {
        if (it <= kv_ready) return true;
        if (!mbar_wait(&bars->kv_full[it % kStages], (it / kStages) & 1, abort_flag)) return false;
        kv_ready = it;
        return true;
      };
      // S_i = Q_i·K^T into TMEM once softmax i has read the previous S_i.
      auto issue_s = [&](int i, int qb, int it) -> bool {
        if (s_cnt[i] > 0 && !mbar_wait(&bars->s_free[i], (s_cnt[i] - 1) & 1, abort_flag))
          return false;
        if (!wait_kv(it)) return false;
        tc_fence_after();
        const int s = it % kStages;
#pragma unroll
        for (int kk = 0; kk < kD / 16; ++kk) {
          const uint64_t a = sdesc_sw128(sQ + (qb * kTiles + i) * kTileBytes + kk * 32, 16, 1024);
          const uint64_t b = sdesc_sw128(sK + s * kTileBytes + kk * 32, 16, 1024);
          umma_ss(tmem + col_s(i), a, b, kIdescS, kk > 0 ? 1u : 0u);
        }
        umma_commit(&bars->s_full[i]);
        ++s_cnt[i];
        return true;
      };
      // O_i (+)= P_i·V once softmax i has written P_i.
      auto issue_pv = [&](int i, int it, bool first) -> bool {
        if (!mbar_wait(&bars->p_full[i], pv_cnt[i] & 1, abort_flag)) return false;
        tc_fence_after();
        const int s = it % kStages;
#pragma unroll
        for (int kk = 0; kk < kBN / 16; ++kk) {
          const uint64_t b = sdesc_sw128(sV + s * kTileBytes + kk * 2048, 8192, 1024);
          // P_i: 128 lanes x 64 columns of packed bf16 pairs; 16 keys = 8 columns
          umma_ts(tmem + col_o(i), tmem + col_p(i) + kk * 8, b, kIdescO,
                  (!first || kk > 0) ? 1u : 0u);
        }
        umma_commit(&bars->o_done[i]);
        ++pv_cnt[i];
        return true;
      };
      for (int n = 0, k; ok && (k = item_of(n, cta, grid)) < n_items; ++n) {
        const WorkItem w = decode_item<kCausal>(k, BH, n_blk, n_k);
        const int qb = n & 1;
        if (!mbar_wait(&bars->q_full[qb], (n >> 1) & 1, abort_flag)) { ok = false; break; }
        for (int i = 0; ok && i < kTiles; ++i) ok = issue_s(i, qb, kv_base);
        for (int j = 0; ok && j < w.n_total; ++j) {
          // next scores as soon as each softmax has read the current ones
          for (int i = 0; ok && i < kTiles; ++i)
            if (j + 1 < w.n_kv[i]) ok = issue_s(i, qb, kv_base + j + 1);
          // then O_i += P_i·V_j as each P_i arrives
          for (int i = 0; ok && i < kTiles; ++i)
            if (j < w.n_kv[i]) ok = issue_pv(i, kv_base + j, j == 0);
          if (ok) umma_commit(&bars->kv_empty[(kv_base + j) % kStages]);
        }
        if (ok) umma_commit(&bars->q_empty[qb]);  // every S of this item has read Q
        kv_base += w.n_total;
      }
      if (!ok) raise_abort(abort_flag, err_word, kDevErrTimeoutMma);
      // Every issued UMMA completes before teardown.
      umma_commit(&bars->drained);
      (void)mbar_wait(&bars->drained, 0, abort_flag);
    }
  } else if (warp > kWarpMma) {
    regs_decrease<kRegsControl>();  // idle warps of the control warpgroup
  } else {
    // -------------------------------------------------------------- softmax
    // warp -> (tile, column half, TMEM lane quarter); thread = one score row,
    // half of its columns.  The two halves of a row meet through shared memory
    // at a 64-thread named barrier (ids 1..8, one per tile and lane quarter).
    regs_increase<kRegsSoftmax>();
    Exchange* xch = reinterpret_cast<Exchange*>(smem + kOffX);
    const int tile = warp / (4 * kHalves);
    const int half = (warp / 4) % kHalves;
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;            // TMEM lane = row within the tile
    const uint32_t pair_bar = 1 + tile * 4 + quarter;
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t s_addr = tmem + lane_base + col_s(tile) + half * kHalfCols;
    const uint32_t p_addr = tmem + lane_base + col_p(tile) + half * (kHalfCols / 2);
    const uint32_t o_addr = tmem + lane_base + col_o(tile) + half * kOutCols;
    const uint64_t scale2 = f2_pack(scale_log2, scale_log2);
    int it = 0;  // S_i tiles processed so far, across items
    bool ok = true;
    for (int n = 0, k; ok && (k = item_of(n, cta, grid)) < n_items; ++n) {
      const WorkItem w = decode_item<kCausal>(k, BH, n_blk, n_k);
      const int q_idx = w.blk * kRowsPerCta + tile * kBM + row;
      const int nkv = w.n_kv[tile];
      float m_used = -INFINITY;  // offset used for exponentials (log2 units)
      float m_true = -INFINITY;  // true running row max (log2 units)
      float l = 0.f;             // this half's share of the row sum
      for (int j = 0; j < nkv; ++j, ++it) {
        if (!warp_wait(&bars->s_full[tile], it & 1, abort_flag)) { ok = false; break; }
        tc_fence_after();
        uint32_t sr[kHalfCols];
#pragma unroll
        for (int c = 0; c < kHalfCols / 32; ++c)
          tmem_ld32(s_addr + c * 32, *reinterpret_cast<uint32_t(*)[32]>(&sr[c * 32]));
        tmem_ld_wait();
        // S_i now lives in registers: let the tensor core write the next one.
        tc_fence_before();
        mbar_arrive(&bars->s_free[tile]);
        float* sv = reinterpret_cast<float*>(sr);
        if (j == nkv - 1) {
          const int k0 = j * kBN + half * kHalfCols;
#pragma unroll
          for (int c = 0; c < kHalfCols; ++c) {
            const int k_idx = k0 + c;
            if ((k_idx >= Sk) || (kCausal && k_idx > q_idx)) sv[c] = -INFINITY;
          }
        }
        // partial row max over this half: 4 independent chains of 3-input max
        float mx0 = fmaxf(sv[0], sv[1]), mx1 = fmaxf(sv[2], sv[3]);
        float mx2 = fmaxf(sv[4], sv[5]), mx3 = fmaxf(sv[6], sv[7]);
        static_assert(kHalfCols % 8 == 0, "the max chains consume 8 scores per step");
#pragma unroll
        for (int c = 8; c < kHalfCols; c += 8) {
          mx0 = fmax3(mx0, sv[c], sv[c + 1]);
          mx1 = fmax3(mx1, sv[c + 2], sv[c + 3]);
          mx2 = fmax3(mx2, sv[c + 4], sv[c + 5]);
          mx3 = fmax3(mx3, sv[c + 6], sv[c + 7]);
        }
        float mx = fmaxf(fmaxf(mx0, mx1), fmaxf(mx2, mx3));
        if constexpr (kHalves > 1) {
          xch->max_part[it & 1][tile][half][row] = mx;
          named_bar_sync(pair_bar, 64);
          mx = fmaxf(mx, xch->max_part[it & 1][tile][half ^ 1][row]);
        }
        const float t_max = mx * scale_log2;
        m_true = fmaxf(m_true, t_max);
        float m_new = m_used;
        float alpha = 1.f;
        if (t_max > m_used + kRescaleThreshold) {
          m_new = t_max;
          alpha = (m_used == -INFINITY) ? 0.f : fast_exp2(m_used - m_new);
        }
        // p = 2^(s·scale_log2 - m_new), two at a time, four partial sums.  The
        // masked last tile uses the exponential unit for every element (masked
        // keys give exactly 0); other tiles send part of the pairs through the
        // FMA-pipe polynomial, which relieves the exponential unit.
        const uint64_t negm2 = f2_pack(-m_new, -m_new);
        uint64_t acc[4] = {0, 0, 0, 0};
        uint32_t pk[kHalfCols / 2];
        if (j == nkv - 1)
          exp2_pairs<0>(sv, scale2, negm2, pk, acc);
        else
          exp2_pairs<kPolyPairsPer8>(sv, scale2, negm2, pk, acc);
        float a0, a1;
        f2_unpack(f2_add(f2_add(acc[0], acc[1]), f2_add(acc[2], acc[3])), a0, a1);
        l = l * alpha + (a0 + a1);
        // P_i may be overwritten once the previous O_i += P_i·V has completed
        // (for j == 0 the previous item's epilogue already waited for it).
        if (j > 0) {
          if (!warp_wait(&bars->o_done[tile], (it - 1) & 1, abort_flag)) { ok = false; break; }
          tc_fence_after();
        }
#pragma unroll
        for (int c = 0; c < kHalfCols / 64; ++c)
          tmem_st32(p_addr + c * 32, *reinterpret_cast<const uint32_t(*)[32]>(&pk[c * 32]));
        // O_i is stable here; rescale this thread's output columns if the warp
        // has a row whose running max moved.
        if (j > 0 && __any_sync(0xffffffffu, alpha != 1.f)) {
#pragma unroll
          for (int c = 0; c < kOutCols / 32; ++c) {
            uint32_t orr[32];
            tmem_ld32(o_addr + c * 32, orr);
            tmem_ld_wait();
#pragma unroll
            for (int e = 0; e < 32; ++e) orr[e] = __float_as_uint(__uint_as_float(orr[e]) * alpha);
            tmem_st32(o_addr + c * 32, orr);
          }
        }
        tmem_st_wait();
        tc_fence_before();
        mbar_arrive(&bars->p_full[tile]);
        m_used = m_new;
      }
      if (!ok) break;
      // ---------------------------------------------------------- epilogue
      if (!warp_wait(&bars->o_done[tile], (it - 1) & 1, abort_flag)) { ok = false; break; }
      tc_fence_after();
      uint32_t orr[kOutCols];
#pragma unroll
      for (int c = 0; c < kOutCols / 32; ++c)
        tmem_ld32(o_addr + c * 32, *reinterpret_cast<uint32_t(*)[32]>(&orr[c * 32]));
      tmem_ld_wait();
      float l_row = l;
      if constexpr (kHalves > 1) {
        xch->sum_part[tile][half][row] = l;
        named_bar_sync(pair_bar, 64);
        l_row += xch->sum_part[tile][half ^ 1][row];
        // both halves have read the partner's sum before either reuses the slot
        named_bar_sync(pair_bar, 64);
      }
      if (q_idx < Sq) {
        const float inv_l = 1.f / l_row;
        const size_t row_off = static_cast<size_t>(w.bh) * Sq + q_idx;
        const long long o_off =
            kStrided ? (w.bh / lay.H) * lay.o_b + (w.bh % lay.H) * lay.o_h +
                           static_cast<long long>(q_idx) * lay.o_s
                     : static_cast<long long>(row_off) * kD;
        constexpr int kCols = kOutCols;
        if constexpr (kOutF32) {
          float4* dst = reinterpret_cast<float4*>(static_cast<float*>(out) + o_off +
                                                  half * kCols);
#pragma unroll
          for (int c = 0; c < kCols / 4; ++c)
            dst[c] = make_float4(__uint_as_float(orr[4 * c]) * inv_l,
                                 __uint_as_float(orr[4 * c + 1]) * inv_l,
                                 __uint_as_float(orr[4 * c + 2]) * inv_l,
                                 __uint_as_float(orr[4 * c + 3]) * inv_l);
        } else {
          uint4* dst = reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(out) + o_off +
                                                half * kCols);
#pragma unroll
          for (int c = 0; c < kCols / 8; ++c)
            dst[c] = make_uint4(
                pack_bf16x2(__uint_as_float(orr[8 * c]) * inv_l, __uint_as_float(orr[8 * c + 1]) * inv_l),
                pack_bf16x2(__uint_as_float(orr[8 * c + 2]) * inv_l, __uint_as_float(orr[8 * c + 3]) * inv_l),
                pack_bf16x2(__uint_as_float(orr[8 * c + 4]) * inv_l, __uint_as_float(orr[8 * c + 5]) * inv_l),
                pack_bf16x2(__uint_as_float(orr[8 * c + 6]) * inv_l, __uint_as_float(orr[8 * c + 7]) * inv_l));
        }
        if (half == 0) {
          if (lse_out) lse_out[row_off] = (m_used + __log2f(l_row)) * kLn2;
          if (max_out) max_out[row_off] = m_true * kLn2;
        }
      }
    }
    if (!ok) raise_abort(abort_flag, err_word, kDevErrTimeoutSoftmax);
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kWarpMma) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

template <bool kCausal, bool kOutF32, bool kStrided>
cudaError_t launch_typed(cudaStream_t stream, const CUtensorMap& tq, const CUtensorMap& tk,
                         const CUtensorMap& tv, void* out, const FlashLayout& lay, float* lse,
                         float* mx, int BH, int Sq, int Sk, float scale_log2) {
  auto kern = flash_fwd_kernel<kCausal, kOutF32, kStrided>;
  cudaError_t e =
      cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
  if (e != cudaSuccess) return e;
  // Persistent CTAs: one per SM (at most one fits, by shared memory and TMEM).
  int dev = 0, sms = 0;
  e = cudaGetDevice(&dev);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (e != cudaSuccess) return e;
  const int n_items = ceil_div(Sq, kRowsPerCta) * BH;
  dim3 grid(n_items < sms ? n_items : sms);
  kern<<<grid, kThreads, kSmemBytes, stream>>>(tq, tk, tv, out, lay, lse, mx, BH, Sq, Sk, scale_log2,
                                               device_error_word());
  return cudaGetLastError();
}

}  // namespace

FlashStrides flash_head_major_strides(int H, int Sq, int Sk) {
  FlashStrides st;
  const long long q[3] = {kD, static_cast<long long>(Sq) * kD, static_cast<long long>(H) * Sq * kD};
  const long long k[3] = {kD, static_cast<long long>(Sk) * kD, static_cast<long long>(H) * Sk * kD};
  for (int i = 0; i < 3; ++i) {
    st.q[i] = q[i];
    st.o[i] = q[i];
    st.k[i] = k[i];
    st.v[i] = k[i];
  }
  return st;
}

namespace {
// 4-D map over rows of S positions x H heads x B batches, 64 bf16 per row;
// the row and head dims are ordered by stride (a tensor map's dims go from
// the finest stride outwards).  Returns whether the head dim is the inner one.
cudaError_t make_rows_map(CUtensorMap* map, const void* base, int S, int H, int B,
                          const long long (&st)[3], int* token_major, const char** err_msg) {
  const bool tok = st[1] < st[0];
  const uint64_t s = static_cast<uint64_t>(S), h = static_cast<uint64_t>(H);
  const uint64_t dims[4] = {kD, tok ? h : s, tok ? s : h, static_cast<uint64_t>(B)};
  const uint64_t strides[3] = {static_cast<uint64_t>(tok ? st[1] : st[0]) * 2,
                               static_cast<uint64_t>(tok ? st[0] : st[1]) * 2,
                               static_cast<uint64_t>(st[2]) * 2};
  const uint32_t box[4] = {kD, tok ? 1u : static_cast<uint32_t>(kBM), tok ? static_cast<uint32_t>(kBM) : 1u, 1};
  *token_major = tok ? 1 : 0;
  return make_tmap_bf16_sw128(map, base, 4, dims, strides, box, err_msg);
}
}  // namespace

cudaError_t launch_flash_fwd(cudaStream_t stream, const __nv_bfloat16* Q, const __nv_bfloat16* K,
                             const __nv_bfloat16* V, void* O, bool out_f32, float* lse,
                             float* row_max, int B, int H, int Sq, int Sk, float scale,
                             bool causal, const FlashStrides& st, const char** err_msg) {
  const int BH = B * H;
  if (BH == 0 || Sq == 0) return cudaSuccess;
  CUtensorMap tq, tk, tv;
  FlashLayout lay;
  lay.H = H;
  lay.o_s = st.o[0];
  lay.o_h = st.o[1];
  lay.o_b = st.o[2];
  lay.q_token_major = lay.kv_token_major = 0;
  const FlashStrides hm = flash_head_major_strides(H, Sq, Sk);
  bool strided = false;
  for (int i = 0; i < 3; ++i)
    strided = strided || st.q[i] != hm.q[i] || st.k[i] != hm.k[i] || st.v[i] != hm.v[i] ||
              st.o[i] != hm.o[i];
  cudaError_t e = cudaSuccess;
  if (strided) {
    int k_tok = 0, v_tok = 0;
    e = make_rows_map(&tq, Q, Sq, H, B, st.q, &lay.q_token_major, err_msg);
    if (e == cudaSuccess) e = make_rows_map(&tk, K, Sk, H, B, st.k, &k_tok, err_msg);
    if (e == cudaSuccess) e = make_rows_map(&tv, V, Sk, H, B, st.v, &v_tok, err_msg);
    if (e != cudaSuccess) return e;
    if (k_tok != v_tok) {
      if (err_msg) *err_msg = "K and V must share one layout (both head-major or both token-major)";
      return cudaErrorInvalidValue;
    }
    lay.kv_token_major = k_tok;
  } else {
    // contiguous head-major: 3-D maps {64, S, B·H}, so a ragged S is
    // zero-filled per head, never read from the next head
    const uint32_t box[3] = {kD, kBM, 1};
    const uint64_t qdims[3] = {kD, static_cast<uint64_t>(Sq), static_cast<uint64_t>(BH)};
    const uint64_t qstr[2] = {kD * 2, static_cast<uint64_t>(Sq) * kD * 2};
    const uint64_t kdims[3] = {kD, static_cast<uint64_t>(Sk), static_cast<uint64_t>(BH)};
    const uint64_t kstr[2] = {kD * 2, static_cast<uint64_t>(Sk) * kD * 2};
    e = make_tmap_bf16_sw128(&tq, Q, 3, qdims, qstr, box, err_msg);
    if (e == cudaSuccess) e = make_tmap_bf16_sw128(&tk, K, 3, kdims, kstr, box, err_msg);
    if (e == cudaSuccess) e = make_tmap_bf16_sw128(&tv, V, 3, kdims, kstr, box, err_msg);
    if (e != cudaSuccess) return e;
  }
  const float sl2 = scale * kLog2e;
#define ND_FLASH_LAUNCH(C, F, S_)                                                              \
  launch_typed<C, F, S_>(stream, tq, tk, tv, O, lay, lse, row_max, BH, Sq, Sk, sl2)
  if (strided) {
    if (causal) return out_f32 ? ND_FLASH_LAUNCH(true, true, true) : ND_FLASH_LAUNCH(true, false, true);
    return out_f32 ? ND_FLASH_LAUNCH(false, true, true) : ND_FLASH_LAUNCH(false, false, true);
  }
  if (causal) return out_f32 ? ND_FLASH_LAUNCH(true, true, false) : ND_FLASH_LAUNCH(true, false, false);
  return out_f32 ? ND_FLASH_LAUNCH(false, true, false) : ND_FLASH_LAUNCH(false, false, false);
#undef ND_FLASH_LAUNCH
}

}  // namespace nd
