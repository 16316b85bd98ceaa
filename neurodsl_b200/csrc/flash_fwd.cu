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
// double-buffered and the K/V ring runs on across items.  Warp roles (384
// threads):
//   warps 0..3   softmax of query tile 0 (thread = row = TMEM lane)
//   warps 4..7   softmax of query tile 1
//   warp 8       TMA producer: K/V tiles (kStages ring); the next item's Q as
//                soon as its buffer is free
//   warp 9       TMEM allocator + UMMA issuer of tile 0 (one thread)
//   warp 10      UMMA issuer of tile 1 (one thread)
//   warp 11      idle (it completes the control warpgroup)
// TMEM (512 columns), per tile i at base 256·i: S_i [0,128) fp32 scores,
// P_i [128,192) packed bf16 probabilities, O_i [192,256) fp32 accumulator.
//
// Each tile has its own UMMA issuer thread, so the tiles proceed
// independently (each issuer blocks only on its own tile's barriers): S_i(k+1)
// = Q_i·K_{k+1}ᵀ is issued once softmax i has copied S_i(k) into registers,
// O_i (+)= P_i(k)·V_k once softmax i has written P_i(k), across item
// boundaries too, so a tile that finishes an item early starts the next one
// while the other tile finishes.  P_i is the A operand from tensor memory, V
// an MN-major shared-memory operand.
//
// Softmax (per row, per K/V tile, in two halves of 64 keys): the half's max
// is taken, the offset m (log2 units) raised if the max passed it by more
// than 8, then the half's exponentials are computed against m; the second
// half's max is independent of the first half's exponentials, so the two
// overlap.  Raising the offset (always at a row's first half, rarely after)
// multiplies l, O and the P already stored by 2^(old - new).  O and l share
// the offset, so the final O/l is exact; the reported m is the true row max.  A row's output (O/l, lse, m) is
// written during the first tile of its next item, before that item's first
// P·V overwrites O, so no warp waits for the last P·V of an item.
#include <cuda.h>
#include <cuda_bf16.h>
#include <limits.h>
#include <stdint.h>

#include "flash_fwd.h"
#include "launch.cuh"
#include "ptx.cuh"
#include "tma.h"

// Tuning switches (compile-time): how many of every 8 score pairs of an
// unmasked tile take the FMA-pipe polynomial exp2 instead of the exponential
// unit, and whether probabilities are packed to bf16 with the conversion
// instruction (1) or with integer rounding (0).
#ifndef ND_FLASH_POLY_PAIRS
#define ND_FLASH_POLY_PAIRS 0
#endif
#ifndef ND_FLASH_PACK_CVT
#define ND_FLASH_PACK_CVT 1
#endif
// K/V ring depth (stages of 32 KB).
#ifndef ND_FLASH_STAGES
#define ND_FLASH_STAGES 3
#endif

namespace nd {
namespace {

constexpr int kBM = 128;               // rows per query tile
constexpr int kTiles = 2;              // query tiles per CTA
constexpr int kRowsPerCta = kBM * kTiles;
constexpr int kBN = 128;               // keys per K/V tile
constexpr int kD = 64;
constexpr int kStages = ND_FLASH_STAGES;
constexpr int kSoftmaxThreads = 128 * kTiles;
constexpr int kThreads = kSoftmaxThreads + 128;  // + one control warpgroup
constexpr int kWarpProducer = kSoftmaxThreads / 32;
constexpr int kWarpMma = kWarpProducer + 1;
constexpr int kPolyPairs = ND_FLASH_POLY_PAIRS;
constexpr bool kPackCvt = ND_FLASH_PACK_CVT != 0;
static_assert(kPolyPairs >= 0 && kPolyPairs <= 8, "pairs out of 8");
// Register split: launch gives 168 per thread (64512 total); control 72 +
// softmax 216: 128 x 72 + 256 x 216 = 64512.
constexpr uint32_t kLaunchRegs = (65536 / kThreads) & ~7u;
constexpr uint32_t kRegsControl = 72;
constexpr uint32_t kRegsSoftmax = 216;
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
// per softmax warp, its 32 finished rows staged for a TMA tensor store
// (bf16: one 32 x 128 B box; fp32: two, one per 32 columns)
constexpr uint32_t kStageBytesWarp = 8192;
constexpr uint32_t kOffStage = kOffV + kStages * kTileBytes;
constexpr uint32_t kOffBar = kOffStage + (kSoftmaxThreads / 32) * kStageBytesWarp;
constexpr uint32_t kSmemBytes = kOffBar + 256 + 1024;           // + alignment slack

constexpr uint32_t kIdescS = idesc_bf16_f32(kBM, kBN, false, false);
constexpr uint32_t kIdescO = idesc_bf16_f32(kBM, kD, false, true);

struct Bars {
  uint64_t q_full[2];        // Q tiles of item n land in buffer n & 1
  uint64_t q_empty[2];       // every S of that item has read the buffer (both issuers)
  uint64_t kv_full[kStages];
  uint64_t kv_empty[kStages];  // both issuers are done with the stage
  uint64_t s_full[kTiles];   // S_i(k) written (UMMA commit)
  uint64_t s_free[kTiles];   // S_i(k) read into registers (128 softmax threads)
  uint64_t p_full[kTiles];   // P_i(k) written, O_i rescaled and read out (128 threads)
  uint64_t o_done[kTiles];   // O_i += P_i(k)·V_k complete (UMMA commit)
  uint64_t drained[kTiles];
  uint32_t tmem_base;
  int abort_flag;
};
static_assert(sizeof(Bars) <= 256, "barrier area");
static_assert(kSmemBytes <= 227 * 1024, "shared memory per CTA");

__host__ __device__ constexpr int ceil_div(int a, int b) { return (a + b - 1) / b; }

// bf16x2 pack of two non-negative finite floats: the conversion instruction
// (round to nearest even), or integer rounding on the ALU (halfway cases up:
// add half an output ulp to the fp32 bits, keep the high halves).
__device__ __forceinline__ uint32_t pack_p(float lo, float hi) {
  if constexpr (kPackCvt) {
    return pack_bf16x2(lo, hi);
  } else {
    const uint32_t a = __float_as_uint(lo) + 0x8000u;
    const uint32_t b = __float_as_uint(hi) + 0x8000u;
    return __byte_perm(a, b, 0x7632);
  }
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

__device__ __forceinline__ void poly_exp2_pair(float x0, float x1, float& p0, float& p1) {
  const uint64_t magic2 = f2_pack(kRoundMagic, kRoundMagic);
  const uint64_t x2 = f2_pack(fmaxf(x0, -126.f), fmaxf(x1, -126.f));
  const uint64_t t2 = f2_add(x2, magic2);                 // magic + round(x)
  const uint64_t fr = f2_sub(x2, f2_sub(t2, magic2));     // x - round(x)
  uint64_t pp = f2_fma(fr, f2_pack(kExpC3, kExpC3), f2_pack(kExpC2, kExpC2));
  pp = f2_fma(pp, fr, f2_pack(kExpC1, kExpC1));
  pp = f2_fma(pp, fr, f2_pack(kExpC0, kExpC0));
  float t0, t1;
  f2_unpack(t2, t0, t1);
  f2_unpack(pp, p0, p1);
  // the low bits of t hold round(x); shifting by 23 drops the magic's bits
  p0 = __uint_as_float(__float_as_uint(p0) + (__float_as_uint(t0) << 23));
  p1 = __uint_as_float(__float_as_uint(p1) + (__float_as_uint(t1) << 23));
}

// Probabilities of the score columns [C0, C1) of one row: p = 2^(s·scale - m)
// packed to bf16 pairs in pk[(c - C0) / 2], row-sum partials in acc (four
// f32x2 chains).  kPoly of every 8 pairs use the FMA-pipe polynomial.
template <int C0, int C1, int kPoly>
__device__ __forceinline__ void exp_span(const float* sv, uint64_t scale2, uint64_t negm2,
                                         uint32_t* pk, uint64_t* acc) {
#pragma unroll
  for (int c = C0; c < C1; c += 2) {
    const int q = c >> 1;
    float x0, x1, p0, p1;
    f2_unpack(f2_fma(f2_pack(sv[c], sv[c + 1]), scale2, negm2), x0, x1);
    if ((q & 7) < kPoly) {
      poly_exp2_pair(x0, x1, p0, p1);
    } else {
      p0 = fast_exp2(x0);
      p1 = fast_exp2(x1);
    }
    acc[q & 3] = f2_add(acc[q & 3], f2_pack(p0, p1));
    pk[(c - C0) >> 1] = pack_p(p0, p1);
  }
}

// The same with the polynomial switched off in a masked tile (masked keys
// must give exactly 0, which the exponential unit's 2^-inf does).
template <int C0, int C1>
__device__ __forceinline__ void exp_cols(bool masked_tile, const float* sv, uint64_t scale2,
                                         uint64_t negm2, uint32_t* pk, uint64_t* acc) {
  if constexpr (kPolyPairs == 0) {
    exp_span<C0, C1, 0>(sv, scale2, negm2, pk, acc);
  } else {
    if (masked_tile)
      exp_span<C0, C1, 0>(sv, scale2, negm2, pk, acc);
    else
      exp_span<C0, C1, kPolyPairs>(sv, scale2, negm2, pk, acc);
  }
}

// Max of the score columns [C0, C0 + 64) of one row (four 3-input chains).
template <int C0>
__device__ __forceinline__ float half_max(const float* sv) {
  float m0 = fmaxf(sv[C0], sv[C0 + 1]), m1 = fmaxf(sv[C0 + 2], sv[C0 + 3]);
  float m2 = fmaxf(sv[C0 + 4], sv[C0 + 5]), m3 = fmaxf(sv[C0 + 6], sv[C0 + 7]);
#pragma unroll
  for (int c = C0 + 8; c < C0 + 64; c += 8) {
    m0 = fmax3(m0, sv[c], sv[c + 1]);
    m1 = fmax3(m1, sv[c + 2], sv[c + 3]);
    m2 = fmax3(m2, sv[c + 4], sv[c + 5]);
    m3 = fmax3(m3, sv[c + 6], sv[c + 7]);
  }
  return fmaxf(fmaxf(m0, m1), fmaxf(m2, m3));
}

__device__ __forceinline__ float f2_sum4(const uint64_t* acc) {
  float a0, a1;
  f2_unpack(f2_add(f2_add(acc[0], acc[1]), f2_add(acc[2], acc[3])), a0, a1);
  return a0 + a1;
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
  int o_token_major;     // O map dims {64|32, H, S, B}
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

// Position of one tile's UMMA stream (S products or P·V products) in this
// CTA's item sequence: item n, K/V tile j of that item, ring position of the
// item's first K/V tile, and the item's tile counts (nkv = 0: no more items).
struct Cursor {
  int n, j, base, nkv, total;
};

// A row whose output is still to be written (the previous item's).
struct PendingRow {
  float l, m_used, m_true;
  int q_idx, bh;
  bool valid;
};

// kStrided: Q/K/V through 4-D maps and O through FlashLayout strides; the
// contiguous head-major case keeps 3-D maps {64, S, B·H} and bh·S row offsets.
template <bool kCausal, bool kOutF32, bool kStrided>
__global__ void __launch_bounds__(kThreads, 1)
    flash_fwd_kernel(const __grid_constant__ CUtensorMap tm_q,
                     const __grid_constant__ CUtensorMap tm_k,
                     const __grid_constant__ CUtensorMap tm_v,
                     const __grid_constant__ CUtensorMap tm_o, const FlashLayout lay,
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
      mbar_init(&bars->q_empty[b], kTiles);
    }
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&bars->kv_full[s], 1);
      mbar_init(&bars->kv_empty[s], kTiles);
    }
    for (int i = 0; i < kTiles; ++i) {
      mbar_init(&bars->s_full[i], 1);
      mbar_init(&bars->s_free[i], 128);
      mbar_init(&bars->p_full[i], 128);
      mbar_init(&bars->o_done[i], 1);
    }
    for (int i = 0; i < kTiles; ++i) mbar_init(&bars->drained[i], 1);
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
      int kv_it = 0;   // K/V tiles loaded so far (ring position)
      int n_q = 0;     // items whose Q tiles have been loaded
      bool ok = true;
      // Load item n_q's two Q tiles into buffer n_q & 1 once the item two
      // before it has released the buffer; without `block`, only if it has.
      auto load_q = [&](bool block) -> bool {
        const int k = item_of(n_q, cta, grid);
        if (k >= n_items) return true;
        const int qb = n_q & 1;
        if (n_q >= 2) {
          const uint32_t par = ((n_q >> 1) - 1) & 1;
          if (block) {
            if (!mbar_wait(&bars->q_empty[qb], par, abort_flag)) return false;
          } else if (!mbar_test(&bars->q_empty[qb], par)) {
            return true;
          }
        }
        const WorkItem w = decode_item<kCausal>(k, BH, n_blk, n_k);
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
        ++n_q;
        return true;
      };
      int n = 0;
      for (int k; ok && (k = item_of(n, cta, grid)) < n_items; ++n) {
        const WorkItem w = decode_item<kCausal>(k, BH, n_blk, n_k);
        while (ok && n_q <= n) ok = load_q(true);
        const int h = kStrided ? w.bh % lay.H : 0, b = kStrided ? w.bh / lay.H : 0;
        for (int j = 0; ok && j < w.n_total; ++j, ++kv_it) {
          // the next item's Q as soon as its buffer is free
          if (n_q == n + 1) ok = load_q(false);
          const int s = kv_it % kStages;
          if (ok && kv_it >= kStages &&
              !mbar_wait(&bars->kv_empty[s], ((kv_it / kStages) - 1) & 1, abort_flag))
            ok = false;
          if (!ok) break;
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
      for (int m = (n_q > 2 ? n_q - 2 : 0); m < n_q; ++m)
        (void)mbar_wait(&bars->q_full[m & 1], (m >> 1) & 1, abort_flag);
      for (int j = (kv_it > kStages ? kv_it - kStages : 0); j < kv_it; ++j)
        (void)mbar_wait(&bars->kv_full[j % kStages], (j / kStages) & 1, abort_flag);
    }
  } else if (warp == kWarpMma || warp == kWarpMma + 1) {
    // --------------------------------------------- UMMA issuers, one per tile
    regs_decrease<kRegsControl>();
    if (elect_one()) {
      const int i = warp - kWarpMma;   // query tile served by this thread
      const uint32_t sQ = smem_u32(smem + kOffQ);
      const uint32_t sK = smem_u32(smem + kOffK);
      const uint32_t sV = smem_u32(smem + kOffV);
      auto start = [&](Cursor& c, int n, int base) {
        c.n = n;
        c.j = 0;
        c.base = base;
        const int k = item_of(n, cta, grid);
        if (k < n_items) {
          const WorkItem w = decode_item<kCausal>(k, BH, n_blk, n_k);
          c.nkv = i == 0 ? w.n_kv[0] : w.n_kv[1];
          c.total = w.n_total;
        } else {
          c.nkv = 0;
          c.total = 0;
        }
      };
      auto advance = [&](Cursor& c) {
        if (++c.j == c.nkv) start(c, c.n + 1, c.base + c.total);
      };
      // This tile's products in the order S(0), S(1), P·V(0), S(2), P·V(1), ...
      // over all items, so each S is computed while the softmax works on the
      // previous one.  Every ring position and Q buffer is released by both
      // issuers (barrier counts 2).  A position this tile does not use (tile 0
      // skips the last K/V tile of an item) is released once a later
      // position has been seen landed — the producer loads in order, so the
      // stage's previous phase has completed and the arrival counts for this
      // position.  That is always true when the skip is recorded (the next
      // item's first S, one position later, was issued before this item's
      // last P·V), except after the CTA's last item, when nothing is loaded
      // any more.
      Cursor c, p;
      start(c, 0, 0);
      p = c;
      int s_cnt = 0, pv_cnt = 0;
      int skipped = -1;   // a position this tile skips, not yet released
      int landed = -1;    // highest ring position seen landed
      auto release_skipped = [&]() {
        if (skipped >= 0 && landed > skipped) {
          umma_commit(&bars->kv_empty[skipped % kStages]);
          skipped = -1;
        }
      };
      bool ok = true;
      while (ok && (c.nkv != 0 || p.nkv != 0)) {
        if (c.nkv != 0) {
          // S = Q·K^T into TMEM once the softmax has read the previous S
          const int pos = c.base + c.j;
          if (s_cnt > 0 && !mbar_wait(&bars->s_free[i], (s_cnt - 1) & 1, abort_flag)) { ok = false; break; }
          if (c.j == 0 && !mbar_wait(&bars->q_full[c.n & 1], (c.n >> 1) & 1, abort_flag)) { ok = false; break; }
          if (!mbar_wait(&bars->kv_full[pos % kStages], (pos / kStages) & 1, abort_flag)) { ok = false; break; }
          landed = pos > landed ? pos : landed;
          release_skipped();
          tc_fence_after();
          const int s = pos % kStages, qb = c.n & 1;
#pragma unroll
          for (int kk = 0; kk < kD / 16; ++kk) {
            const uint64_t a = sdesc_sw128(sQ + (qb * kTiles + i) * kTileBytes + kk * 32, 16, 1024);
            const uint64_t b = sdesc_sw128(sK + s * kTileBytes + kk * 32, 16, 1024);
            umma_ss(tmem + col_s(i), a, b, kIdescS, kk > 0 ? 1u : 0u);
          }
          umma_commit(&bars->s_full[i]);
          ++s_cnt;
          if (c.j + 1 == c.nkv) umma_commit(&bars->q_empty[qb]);  // every S of the item read Q
          advance(c);
        }
        if (p.nkv != 0 && (pv_cnt + 1 < s_cnt || c.nkv == 0)) {
          // O (+)= P·V once the softmax has written P
          if (!mbar_wait(&bars->p_full[i], pv_cnt & 1, abort_flag)) { ok = false; break; }
          tc_fence_after();
          const int pos = p.base + p.j;   // landed: its S product waited for it
          const int s = pos % kStages;
#pragma unroll
          for (int kk = 0; kk < kBN / 16; ++kk) {
            const uint64_t b = sdesc_sw128(sV + s * kTileBytes + kk * 2048, 8192, 1024);
            // P: 128 lanes x 64 columns of packed bf16 pairs; 16 keys = 8 columns
            umma_ts(tmem + col_o(i), tmem + col_p(i) + kk * 8, b, kIdescO,
                    (p.j > 0 || kk > 0) ? 1u : 0u);
          }
          umma_commit(&bars->o_done[i]);
          ++pv_cnt;
          umma_commit(&bars->kv_empty[s]);
          if (p.j + 1 == p.nkv && p.nkv < p.total) {
            skipped = p.base + p.nkv;
            release_skipped();
          }
          advance(p);
        }
      }
      if (!ok) raise_abort(abort_flag, err_word, kDevErrTimeoutMma);
      // Every issued UMMA completes before teardown.
      umma_commit(&bars->drained[i]);
      (void)mbar_wait(&bars->drained[i], 0, abort_flag);
    }
  } else if (warp > kWarpMma + 1) {
    regs_decrease<kRegsControl>();  // idle warp of the control warpgroup
  } else {
    // -------------------------------------------------------------- softmax
    // warp -> (tile, TMEM lane quarter); thread = one score row.
    regs_increase<kRegsSoftmax>();
    const int tile = warp / 4;
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;            // TMEM lane = row within the tile
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t s_addr = tmem + lane_base + col_s(tile);
    const uint32_t p_addr = tmem + lane_base + col_p(tile);
    const uint32_t o_addr = tmem + lane_base + col_o(tile);
    const uint64_t scale2 = f2_pack(scale_log2, scale_log2);

    // O/l, lse and m of a finished row (the previous item's), read from O_i
    // before the next P·V of this tile may overwrite it.  The warp's 32 rows
    // are staged in shared memory in the 128-byte-swizzled layout of a TMA
    // box and written by one tensor store (rows past Sq are clipped by it).
    uint8_t* stage = smem + kOffStage + warp * kStageBytesWarp;
    const uint32_t r7 = static_cast<uint32_t>(lane & 7);
    auto write_row = [&](const PendingRow& pr) {
      uint32_t orr[kD];
#pragma unroll
      for (int c = 0; c < kD / 32; ++c)
        tmem_ld32(o_addr + c * 32, *reinterpret_cast<uint32_t(*)[32]>(&orr[c * 32]));
      tmem_ld_wait();
      const float inv_l = 1.f / pr.l;
      // the previous store from this buffer has finished reading it
      if (lane == 0) bulk_wait_read_all();
      __syncwarp();
      const uint32_t row_s = smem_u32(stage) + static_cast<uint32_t>(lane) * 128u;
      if constexpr (kOutF32) {
#pragma unroll
        for (int c = 0; c < kD / 4; ++c)
          st_shared_v4(row_s + (c >> 3) * 4096u + (((c & 7) ^ r7) << 4),
                       __float_as_uint(__uint_as_float(orr[4 * c]) * inv_l),
                       __float_as_uint(__uint_as_float(orr[4 * c + 1]) * inv_l),
                       __float_as_uint(__uint_as_float(orr[4 * c + 2]) * inv_l),
                       __float_as_uint(__uint_as_float(orr[4 * c + 3]) * inv_l));
      } else {
#pragma unroll
        for (int c = 0; c < kD / 8; ++c)
          st_shared_v4(row_s + ((c ^ r7) << 4),
                       pack_bf16x2(__uint_as_float(orr[8 * c]) * inv_l, __uint_as_float(orr[8 * c + 1]) * inv_l),
                       pack_bf16x2(__uint_as_float(orr[8 * c + 2]) * inv_l, __uint_as_float(orr[8 * c + 3]) * inv_l),
                       pack_bf16x2(__uint_as_float(orr[8 * c + 4]) * inv_l, __uint_as_float(orr[8 * c + 5]) * inv_l),
                       pack_bf16x2(__uint_as_float(orr[8 * c + 6]) * inv_l, __uint_as_float(orr[8 * c + 7]) * inv_l));
      }
      fence_async_shared();  // the staged rows are visible to the tensor store
      __syncwarp();
      if (lane == 0) {
        // lane 0 holds the warp's first row
        constexpr int kBoxes = kOutF32 ? 2 : 1;
#pragma unroll
        for (int bx = 0; bx < kBoxes; ++bx) {
          const void* src = stage + bx * 4096;
          if constexpr (kStrided) {
            const int h = pr.bh % lay.H, b = pr.bh / lay.H;
            if (lay.o_token_major)
              tma_store_4d(&tm_o, src, bx * 32, h, pr.q_idx, b);
            else
              tma_store_4d(&tm_o, src, bx * 32, pr.q_idx, h, b);
          } else {
            tma_store_3d(&tm_o, src, bx * 32, pr.q_idx, pr.bh);
          }
        }
        bulk_commit_group();
      }
      if (pr.q_idx < Sq) {
        const size_t row_off = static_cast<size_t>(pr.bh) * Sq + pr.q_idx;
        if (lse_out) lse_out[row_off] = (pr.m_used + __log2f(pr.l)) * kLn2;
        if (max_out) max_out[row_off] = pr.m_true * kLn2;
      }
    };

    int it = 0;  // S_i tiles processed so far, across items
    bool ok = true;
    PendingRow pend;
    pend.valid = false;
    for (int n = 0, k; ok && (k = item_of(n, cta, grid)) < n_items; ++n) {
      const WorkItem w = decode_item<kCausal>(k, BH, n_blk, n_k);
      const int q_idx = w.blk * kRowsPerCta + tile * kBM + row;
      const int nkv = tile == 0 ? w.n_kv[0] : w.n_kv[1];
      float m_used = -INFINITY;  // offset of the exponentials (log2 units)
      float m_true = -INFINITY;  // true running row max (log2 units)
      float l = 0.f;             // row sum against m_used
      for (int j = 0; j < nkv; ++j, ++it) {
        if (!warp_wait(&bars->s_full[tile], it & 1, abort_flag)) { ok = false; break; }
        tc_fence_after();
        uint32_t sr[kBN];
#pragma unroll
        for (int c = 0; c < kBN / 32; ++c)
          tmem_ld32(s_addr + c * 32, *reinterpret_cast<uint32_t(*)[32]>(&sr[c * 32]));
        tmem_ld_wait();
        // S_i now lives in registers: let the tensor core write the next one.
        tc_fence_before();
        mbar_arrive(&bars->s_free[tile]);
        float* sv = reinterpret_cast<float*>(sr);
        const bool last = (j == nkv - 1);
        if (last) {
          const int k0 = j * kBN;
#pragma unroll
          for (int c = 0; c < kBN; ++c) {
            const int k_idx = k0 + c;
            if ((k_idx >= Sk) || (kCausal && k_idx > q_idx)) sv[c] = -INFINITY;
          }
        }
        // P_i may be overwritten, and O_i rescaled, once the previous
        // O_i += P_i·V has completed (for j == 0, the previous item's last).
        bool pv_done = (it == 0);
        auto wait_pv = [&]() -> bool {
          if (pv_done) return true;
          if (!warp_wait(&bars->o_done[tile], (it - 1) & 1, abort_flag)) return false;
          tc_fence_after();
          pv_done = true;
          return true;
        };
        // Raise the offset to t where a row's max passed it by more than the
        // threshold (always at the row's first tile, where it is -inf): l, O
        // (earlier tiles of this item) and the half of P_i already stored are
        // multiplied by 2^(old - new).  Rare after a row's first tile.
        auto raise_offset = [&](float t, bool half_stored) -> bool {
          const bool up = t > m_used + kRescaleThreshold;
          if (!__any_sync(0xffffffffu, up)) return true;
          const float m_new = up ? t : m_used;
          const float alpha = fast_exp2(m_used - m_new);   // 1 where the offset stays
          m_used = m_new;
          l *= alpha;
          if (j > 0 || half_stored) {
            if (!wait_pv()) return false;
            tmem_st_wait();
          }
          if (j > 0) {
#pragma unroll 1
            for (int c = 0; c < kD / 16; ++c) {
              uint32_t orr[16];
              tmem_ld16(o_addr + c * 16, orr);
              tmem_ld_wait();
#pragma unroll
              for (int e = 0; e < 16; ++e) orr[e] = __float_as_uint(__uint_as_float(orr[e]) * alpha);
              tmem_st16(o_addr + c * 16, orr);
            }
          }
          if (half_stored) {
#pragma unroll 1
            for (int c = 0; c < 2; ++c) {
              uint32_t prr[16];
              tmem_ld16(p_addr + c * 16, prr);
              tmem_ld_wait();
#pragma unroll
              for (int e = 0; e < 16; ++e)
                prr[e] = pack_bf16x2(__uint_as_float(prr[e] << 16) * alpha,
                                     __uint_as_float(prr[e] & 0xFFFF0000u) * alpha);
              tmem_st16(p_addr + c * 16, prr);
            }
          }
          return true;
        };
        uint32_t pk[kBN / 4];   // half a row of packed probabilities
        // ---- first half of the keys: its max, then its exponentials
        const float t_a = half_max<0>(sv) * scale_log2;
        m_true = fmaxf(m_true, t_a);
        if (!raise_offset(t_a, false)) { ok = false; break; }
        float sum_a;
        {
          uint64_t acc[4] = {0, 0, 0, 0};
          exp_cols<0, kBN / 2>(last, sv, scale2, f2_pack(-m_used, -m_used), pk, acc);
          sum_a = f2_sum4(acc);
        }
        // second half's max: independent of the exponentials above
        const float t_b = half_max<kBN / 2>(sv) * scale_log2;
        if (!wait_pv()) { ok = false; break; }
        tmem_st32(p_addr, *reinterpret_cast<const uint32_t(*)[32]>(pk));
        l += sum_a;
        // ---- second half
        m_true = fmaxf(m_true, t_b);
        if (!raise_offset(t_b, true)) { ok = false; break; }
        {
          uint64_t acc[4] = {0, 0, 0, 0};
          exp_cols<kBN / 2, kBN>(last, sv, scale2, f2_pack(-m_used, -m_used), pk, acc);
          l += f2_sum4(acc);
        }
        tmem_st32(p_addr + 32, *reinterpret_cast<const uint32_t(*)[32]>(pk));
        // the previous item's rows: O_i holds them until this P_i is released
        if (j == 0 && pend.valid) write_row(pend);
        tmem_st_wait();
        tc_fence_before();
        mbar_arrive(&bars->p_full[tile]);
      }
      if (!ok) break;
      pend.l = l;
      pend.m_used = m_used;
      pend.m_true = m_true;
      pend.q_idx = q_idx;
      pend.bh = w.bh;
      pend.valid = true;
    }
    // the last item's rows, once its last P·V has completed
    if (ok && pend.valid) {
      if (warp_wait(&bars->o_done[tile], (it - 1) & 1, abort_flag)) {
        tc_fence_after();
        write_row(pend);
      } else {
        ok = false;
      }
    }
    if (!ok) raise_abort(abort_flag, err_word, kDevErrTimeoutSoftmax);
    // the staged rows are read and written before the CTA's memory goes away
    if (lane == 0) bulk_wait_all();
    __syncwarp();
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
                         const CUtensorMap& tv, const CUtensorMap& to, const FlashLayout& lay,
                         float* lse, float* mx, int BH, int Sq, int Sk, float scale_log2) {
  auto kern = flash_fwd_kernel<kCausal, kOutF32, kStrided>;
  cudaError_t e =
      cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
  if (e != cudaSuccess) return e;
  // Persistent CTAs: one per SM (at most one fits, by shared memory and TMEM).
  int dev = 0, sms = 0;
  e = cudaGetDevice(&dev);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (e != cudaSuccess) return e;
  sms = limited_sms(sms);
  const int n_items = ceil_div(Sq, kRowsPerCta) * BH;
  dim3 grid(n_items < sms ? n_items : sms);
  kern<<<grid, kThreads, kSmemBytes, stream>>>(tq, tk, tv, to, lay, lse, mx, BH, Sq, Sk, scale_log2,
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
// 4-D map over rows of S positions x H heads x B batches, 64 values per row
// (bf16, or fp32 for an fp32 output); the row and head dims are ordered by
// stride (a tensor map's dims go from the finest stride outwards).  A box is
// `rows` rows of 128 bytes.  Returns whether the head dim is the inner one.
cudaError_t make_rows_map(CUtensorMap* map, const void* base, int S, int H, int B,
                          const long long (&st)[3], uint32_t rows, bool f32, int* token_major,
                          const char** err_msg) {
  const bool tok = st[1] < st[0];
  const uint64_t s = static_cast<uint64_t>(S), h = static_cast<uint64_t>(H);
  const uint64_t esz = f32 ? 4 : 2;
  const uint64_t dims[4] = {kD, tok ? h : s, tok ? s : h, static_cast<uint64_t>(B)};
  const uint64_t strides[3] = {static_cast<uint64_t>(tok ? st[1] : st[0]) * esz,
                               static_cast<uint64_t>(tok ? st[0] : st[1]) * esz,
                               static_cast<uint64_t>(st[2]) * esz};
  const uint32_t box[4] = {static_cast<uint32_t>(128 / esz), tok ? 1u : rows, tok ? rows : 1u, 1};
  *token_major = tok ? 1 : 0;
  return make_tmap_sw128(map, f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16,
                         static_cast<int>(esz), base, 4, dims, strides, box, err_msg);
}
}  // namespace

cudaError_t launch_flash_fwd(cudaStream_t stream, const __nv_bfloat16* Q, const __nv_bfloat16* K,
                             const __nv_bfloat16* V, void* O, bool out_f32, float* lse,
                             float* row_max, int B, int H, int Sq, int Sk, float scale,
                             bool causal, const FlashStrides& st, const char** err_msg) {
  const int BH = B * H;
  if (BH == 0 || Sq == 0) return cudaSuccess;
  CUtensorMap tq, tk, tv, to;
  FlashLayout lay;
  lay.H = H;
  lay.q_token_major = lay.kv_token_major = lay.o_token_major = 0;
  const FlashStrides hm = flash_head_major_strides(H, Sq, Sk);
  bool strided = false;
  for (int i = 0; i < 3; ++i)
    strided = strided || st.q[i] != hm.q[i] || st.k[i] != hm.k[i] || st.v[i] != hm.v[i] ||
              st.o[i] != hm.o[i];
  cudaError_t e = cudaSuccess;
  if (strided) {
    int k_tok = 0, v_tok = 0;
    e = make_rows_map(&tq, Q, Sq, H, B, st.q, kBM, false, &lay.q_token_major, err_msg);
    if (e == cudaSuccess) e = make_rows_map(&tk, K, Sk, H, B, st.k, kBM, false, &k_tok, err_msg);
    if (e == cudaSuccess) e = make_rows_map(&tv, V, Sk, H, B, st.v, kBM, false, &v_tok, err_msg);
    if (e == cudaSuccess)
      e = make_rows_map(&to, O, Sq, H, B, st.o, 32, out_f32, &lay.o_token_major, err_msg);
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
    // O: boxes of 32 rows x 128 bytes (64 bf16, or 32 of 64 fp32)
    const uint64_t esz = out_f32 ? 4 : 2;
    const uint32_t obox[3] = {static_cast<uint32_t>(128 / esz), 32, 1};
    const uint64_t ostr[2] = {kD * esz, static_cast<uint64_t>(Sq) * kD * esz};
    if (e == cudaSuccess)
      e = make_tmap_sw128(&to, out_f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16,
                          static_cast<int>(esz), O, 3, qdims, ostr, obox, err_msg);
    if (e != cudaSuccess) return e;
  }
  const float sl2 = scale * kLog2e;
#define ND_FLASH_LAUNCH(C, F, S_)                                                              \
  launch_typed<C, F, S_>(stream, tq, tk, tv, to, lay, lse, row_max, BH, Sq, Sk, sl2)
  if (strided) {
    if (causal) return out_f32 ? ND_FLASH_LAUNCH(true, true, true) : ND_FLASH_LAUNCH(true, false, true);
    return out_f32 ? ND_FLASH_LAUNCH(false, true, true) : ND_FLASH_LAUNCH(false, false, true);
  }
  if (causal) return out_f32 ? ND_FLASH_LAUNCH(true, true, false) : ND_FLASH_LAUNCH(true, false, false);
  return out_f32 ? ND_FLASH_LAUNCH(false, true, false) : ND_FLASH_LAUNCH(false, false, false);
#undef ND_FLASH_LAUNCH
}

}  // namespace nd
