// tp_comm.cu — one-shot all-reduce over NVLink peer memory, fused with the
// residual add, bias and LayerNorm that follow a tensor-parallel row-parallel
// projection (the out-projection and MLP-down of a Megatron block):
//
//   s = x + Σ_r p_r + bias   (p_r: rank r's partial sum),  y = LayerNorm(s)
//
// Every rank owns a "region" of device memory shared with the other ranks
// through CUDA IPC handles: a header of per-CTA sequence counters, two slots
// of rows_max x d bf16 for this rank's own partial sum (a caller's GEMM
// writes it there), and two receive areas of kCommMaxRanks blocks, one block
// per sending rank.  The exchange carries its own completion flags: every
// 8-byte word a rank pushes holds 4 bytes of data (two bf16) and, in its high
// half, the call's sequence number; an aligned 8-byte store is single-copy
// atomic, so a receiver that reads a word with the current sequence number
// has its data.  Per call, each CTA
//   1. pushes its rows of this rank's partial into this rank's block of every
//      peer's receive area, with plain 16-byte stores over NVLink (no
//      multicast, no fence, no separate flag);
//   2. reads its rows from local memory — its own partial, and every peer's
//      pushed words, polling (bounded) until their sequence numbers are the
//      current one — sums them in rank order (every rank computes the same
//      bits), adds x and the bias, and stores s and the LayerNorm of s.
// So a call costs one NVLink write latency and no rank waits on a remote
// read.  Slots and receive areas alternate between calls: a peer that pushes
// call n+2 has finished call n+1, which waited for this rank's call n+1 push,
// issued after this rank's call n had read everything, so a push never
// overwrites words still to be read; and the words of call n carry an older
// sequence number than those of call n+2.  Each CTA keeps its sequence
// counter in the local header, so captured CUDA graphs replay correctly.  A
// wait that passes the deadline sets the device error word and the CTA skips
// its rows (garbage out, no hang).
#include <cuda_bf16.h>
#include <stdint.h>

#include "launch.cuh"
#include "ptx.cuh"
#include "skinny_core.cuh"
#include "tp_comm.h"

namespace nd {
namespace {

// header: counters[kCommMaxCtas] (this rank's per-CTA sequence numbers of the
// reduction kernel), then one call counter of the fused projection kernel.
// The two kernels number their calls in disjoint ranges (bit 31 clear / set),
// so a word left by one never passes for a word of the other.
constexpr size_t kCountersOff = 0;
constexpr size_t kFusedCounterOff = sizeof(uint32_t) * kCommMaxCtas;
constexpr size_t kHeaderBytes = 256 * ((sizeof(uint32_t) * (kCommMaxCtas + 1) + 255) / 256);
constexpr uint32_t kSeqMask = 0x7fffffffu;
constexpr uint32_t kFusedSeqBit = 0x80000000u;

// two 8-byte words, each single-copy atomic, at system scope
__device__ __forceinline__ void st_words_sys(void* p, uint64_t a, uint64_t b) {
  asm volatile("st.relaxed.sys.global.v2.u64 [%0], {%1, %2};" ::"l"(p), "l"(a), "l"(b) : "memory");
}
__device__ __forceinline__ void ld_words_sys(const void* p, uint64_t& a, uint64_t& b) {
  asm volatile("ld.relaxed.sys.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}
// 16 bytes, cached in L2 only (the areas are rewritten every other call)
__device__ __forceinline__ uint4 ld_cg16(const void* p) {
  uint4 r;
  asm volatile("ld.global.cg.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

__device__ __forceinline__ void bf16x8_add(const uint4& u, float (&f)[8]) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] += __uint_as_float(w[i] << 16);
    f[2 * i + 1] += __uint_as_float(w[i] & 0xFFFF0000u);
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

// Vectors per polling round: kG vectors x kTP senders x four 8-byte words
// stay within 32 words (64 registers), 16 for the widest rows (whose
// vectors already hold most of the registers).
template <int kMaxVec, int kTP>
__host__ __device__ constexpr int poll_group() {
  return ((kMaxVec >= 8 ? 4 : 8) / kTP) < 1 ? 1
         : (((kMaxVec >= 8 ? 4 : 8) / kTP) > kMaxVec ? kMaxVec : ((kMaxVec >= 8 ? 4 : 8) / kTP));
}

// One row's sum over the senders for the kG vectors starting at i0: every
// sender's words of those vectors are loaded in one round (all loads in
// flight together, not one sender and vector after another), re-read until
// all carry `seq` (bounded by the deadline t0 + timeout; on expiry *ok is
// cleared and whatever was read is used), then added in rank order into v.
// `skip` (or -1) is a sender whose values the caller adds itself (the
// reduction kernel's own partial); its slot in the order is left to it.
template <int kMaxVec, int kTP, int kG>
__device__ __forceinline__ void poll_sum(const char* recv, size_t block, size_t off, int lane,
                                         int nvec, int i0, int skip, uint32_t seq, uint64_t t0,
                                         int* ok, float (&v)[kMaxVec][8], const uint4* own_vals) {
  uint64_t w[kG][kTP][4];
  uint32_t it = 0;
  for (;;) {
#pragma unroll
    for (int g = 0; g < kG; ++g) {
      const int c = lane + (i0 + g) * 32;
#pragma unroll
      for (int p = 0; p < kTP; ++p) {
        if (c < nvec && p != skip) {
          const char* src = recv + p * block + (off + c * 8) * 4;
          ld_words_sys(src, w[g][p][0], w[g][p][1]);
          ld_words_sys(src + 16, w[g][p][2], w[g][p][3]);
        }
      }
    }
    bool all = true;
#pragma unroll
    for (int g = 0; g < kG; ++g) {
      const int c = lane + (i0 + g) * 32;
#pragma unroll
      for (int p = 0; p < kTP; ++p)
        if (c < nvec && p != skip)
#pragma unroll
          for (int k = 0; k < 4; ++k) all &= static_cast<uint32_t>(w[g][p][k] >> 32) == seq;
    }
    if (all) break;
    if ((++it & 63u) == 0 && globaltimer() - t0 > ND_WAIT_TIMEOUT_NS) {
      *ok = 0;
      break;
    }
  }
#pragma unroll
  for (int g = 0; g < kG; ++g) {
    const int i = i0 + g, c = lane + i * 32;
    if (c >= nvec) continue;
#pragma unroll
    for (int e = 0; e < 8; ++e) v[i][e] = 0.f;
#pragma unroll
    for (int p = 0; p < kTP; ++p) {
      const uint4 u = p == skip ? own_vals[g]
                                : make_uint4(static_cast<uint32_t>(w[g][p][0]), static_cast<uint32_t>(w[g][p][1]),
                                             static_cast<uint32_t>(w[g][p][2]), static_cast<uint32_t>(w[g][p][3]));
      bf16x8_add(u, v[i]);
    }
  }
}

// s = x + Σ_p pv[p] + bias in rank order, rounded to bf16 and stored to
// s_out; then LayerNorm(s) stored to y — for the vectors of one row a lane
// holds (the same arithmetic and order in the reduction kernel and the fused
// projection kernel, so both give the same bits).
template <int kMaxVec>
__device__ __forceinline__ void add_ln_row(float (&v)[kMaxVec][8], int lane, int nvec, int d,
                                           size_t off, const float* __restrict__ gamma,
                                           const float* __restrict__ beta, __nv_bfloat16* s_out,
                                           __nv_bfloat16* __restrict__ y, float eps) {
  float sum = 0.f;
#pragma unroll
  for (int i = 0; i < kMaxVec; ++i) {
    const int c = lane + i * 32;
    if (c < nvec) {
      const uint4 packed = f32_to_bf16x8(v[i]);
      reinterpret_cast<uint4*>(s_out + off)[c] = packed;
#pragma unroll
      for (int e = 0; e < 8; ++e) v[i][e] = 0.f;
      bf16x8_add(packed, v[i]);  // normalise the stored (bf16) residual
#pragma unroll
      for (int e = 0; e < 8; ++e) sum += v[i][e];
    }
  }
  const float mu = warp_sum(sum) / static_cast<float>(d);
  float q = 0.f;
#pragma unroll
  for (int i = 0; i < kMaxVec; ++i) {
    if (lane + i * 32 < nvec) {
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float t = v[i][e] - mu;
        q += t * t;
      }
    }
  }
  const float rs = rsqrtf(warp_sum(q) / static_cast<float>(d) + eps);
#pragma unroll
  for (int i = 0; i < kMaxVec; ++i) {
    const int c = lane + i * 32;
    if (c < nvec) {
      float o[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float g = gamma ? __ldg(gamma + c * 8 + e) : 1.f;
        const float b = beta ? __ldg(beta + c * 8 + e) : 0.f;
        o[e] = (v[i][e] - mu) * rs * g + b;
      }
      reinterpret_cast<uint4*>(y + off)[c] = f32_to_bf16x8(o);
    }
  }
}

// kTP is the rank count (a compile-time count keeps the per-rank loops
// unrolled, every load of a row in flight together).  `own` is this rank's
// region (regs.r[rank]), passed on its own so that no dynamic index into the
// region array puts that array in local memory.  own_off: this rank's
// partial; recv_off: receive area of this call (block r at r * block).
template <int kMaxVec, int kTP>
__global__ void __launch_bounds__(256)
    allreduce_add_ln_kernel(CommRegions regs, char* own, int rank, size_t own_off, size_t recv_off,
                            size_t block, const __nv_bfloat16* x, const float* __restrict__ bias,
                            const float* __restrict__ gamma, const float* __restrict__ beta,
                            __nv_bfloat16* s_out, __nv_bfloat16* __restrict__ y, int rows, int d,
                            float eps, int* __restrict__ err_word) {
  const int warps = blockDim.x >> 5;
  const int lane = threadIdx.x & 31;
  const int nvec = d >> 3;
  const int row0 = blockIdx.x * warps + (threadIdx.x >> 5);
  const int row_step = gridDim.x * warps;
  // the bias is a constant operand: loaded before the previous kernel (the
  // GEMM writing this rank's partial) has finished, under programmatic
  // dependent launch
  float bs[kMaxVec][8];
#pragma unroll
  for (int i = 0; i < kMaxVec; ++i) {
    const int c = lane + i * 32;
    if (c < nvec) {
#pragma unroll
      for (int e = 0; e < 8; ++e) bs[i][e] = bias ? __ldg(bias + c * 8 + e) : 0.f;
    }
  }
  pdl_wait();  // x and this rank's partial come from earlier kernels
  pdl_trigger();
  __shared__ uint32_t s_seq;
  uint32_t* counters = reinterpret_cast<uint32_t*>(own + kCountersOff);
  if (threadIdx.x == 0) s_seq = (counters[blockIdx.x] + 1) & kSeqMask;
  __syncthreads();
  const uint32_t seq = s_seq;
  const uint64_t tag = static_cast<uint64_t>(seq) << 32;

  // 1. push this CTA's rows of the partial to every peer: 8 bf16 (16 bytes)
  //    become two 16-byte stores of {seq | 2 bf16} words
  const char* mine_p = own + own_off;
  if constexpr (kTP > 1) {
    for (int row = row0; row < rows; row += row_step) {
#pragma unroll
      for (int i = 0; i < kMaxVec; ++i) {
        const int c = lane + i * 32;
        if (c < nvec) {
          const uint4 v = ld_cg16(mine_p + (static_cast<size_t>(row) * d + c * 8) * 2);
          const size_t w = (static_cast<size_t>(row) * d + c * 8) * 4;   // 8 values -> 32 bytes
#pragma unroll
          for (int p = 0; p < kTP; ++p) {
            if (p == rank) continue;
            char* dst = static_cast<char*>(regs.r[p]) + recv_off + rank * block + w;
            st_words_sys(dst, tag | v.x, tag | v.y);
            st_words_sys(dst + 16, tag | v.z, tag | v.w);
          }
        }
      }
    }
  }
  if (threadIdx.x == 0) counters[blockIdx.x] = seq;
  int ok = 1;
  const uint64_t t0 = kTP > 1 ? globaltimer() : 0;

  // 3. sum in rank order from local memory (2. the peers' words of this
  //    call, polled a group of vectors at a time), residual, bias, LayerNorm
  constexpr int kG = poll_group<kMaxVec, kTP>();
  for (int row = row0; row < rows; row += row_step) {
    const size_t off = static_cast<size_t>(row) * d;
    float v[kMaxVec][8];
    uint4 xr[kMaxVec];
#pragma unroll
    for (int i = 0; i < kMaxVec; ++i) {
      const int c = lane + i * 32;
      if (c < nvec) xr[i] = reinterpret_cast<const uint4*>(x + off)[c];
    }
#pragma unroll
    for (int i0 = 0; i0 < kMaxVec; i0 += kG) {
      uint4 own_vals[kG];
#pragma unroll
      for (int g = 0; g < kG; ++g) {
        const int c = lane + (i0 + g) * 32;
        own_vals[g] = c < nvec ? ld_cg16(mine_p + (off + c * 8) * 2) : make_uint4(0, 0, 0, 0);
      }
      poll_sum<kMaxVec, kTP, kG>(own + recv_off, block, off, lane, nvec, i0, rank, seq, t0, &ok,
                                 v, own_vals);
    }
#pragma unroll
    for (int i = 0; i < kMaxVec; ++i) {
      const int c = lane + i * 32;
      if (c < nvec) {
        bf16x8_add(xr[i], v[i]);
#pragma unroll
        for (int e = 0; e < 8; ++e) v[i][e] += bs[i][e];
      }
    }
    add_ln_row<kMaxVec>(v, lane, nvec, d, off, gamma, beta, s_out, y, eps);
    if (!ok) break;
  }
  if (!ok && err_word) atomicCAS(err_word, 0, kDevErrTimeoutComm);
}

// The row-parallel projection of a decode step fused with its reduction:
//   s = x + Σ_r (A_r · W_rᵀ) + bias (bf16 partials, summed in rank order),
//   y = LayerNorm(s)
// where rank r holds A_r [M][K] (its heads' attention output or its MLP
// columns) and W_r [d][K] (the matching columns of the projection).  Each CTA
// computes an 8-column tile of this rank's partial for all M rows (the skinny
// path's weight-streaming tile, split-K over a cluster), rounds it to bf16 —
// as the separate GEMM stores it — and pushes it as {sequence | 2 bf16} words
// into this rank's block of the receive area of every rank, itself included.
// The first ceil(M/8) CTAs then each take 8 rows (a warp per row): they poll
// all ranks' words of their rows (local memory) and finish like the reduction
// kernel.  So the projection, the exchange and the LayerNorm are one launch,
// and the exchange is spread over every CTA of the projection.  Only the
// reducing CTAs wait, and every other CTA pushes and exits, so the grid needs
// no co-residency: CTAs not yet resident run on the SMs the finished ones
// free.  Each CTA releases the dependent kernel only after its push, so the
// dependent grid (which holds SMs while it waits) starts once every CTA of
// this grid has pushed.
template <int kMB, int kMaxVec, int kTP>
__global__ void __launch_bounds__(kSkinnyWarps * 32, 2)
    gemm_allreduce_ln_kernel(const __nv_bfloat16* __restrict__ A,
                             const __nv_bfloat16* __restrict__ W, int M, int d, int K,
                             CommRegions regs, char* own, int rank, size_t recv_off, size_t block,
                             const __nv_bfloat16* x, const float* __restrict__ bias,
                             const float* __restrict__ gamma, const float* __restrict__ beta,
                             __nv_bfloat16* s_out, __nv_bfloat16* __restrict__ y, float eps,
                             int* __restrict__ err_word) {
  const int ksplit = static_cast<int>(cluster_nctarank());
  const int kr = static_cast<int>(cluster_ctarank());
  const int n0 = (blockIdx.x / ksplit) * 8;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __shared__ float red[kSkinnyWarps][kMB * 16][8];
  __shared__ float part[kMB * 16 * 8];
  __shared__ uint32_t s_seq;
  skinny_tile<kMB>(A, W, M, d, K, n0, ksplit, kr, red, part, false);
  uint32_t* fused_counter = reinterpret_cast<uint32_t*>(own + kFusedCounterOff);
  if (threadIdx.x == 0) s_seq = ((*fused_counter + 1) & kSeqMask) | kFusedSeqBit;
  // every CTA of the cluster has its part[] before rank 0 reads them
  if (ksplit > 1) cluster_sync();
  else __syncthreads();
  const uint32_t seq = s_seq;
  const uint64_t tag = static_cast<uint64_t>(seq) << 32;
  if (kr == 0) {
    // this rank's tile, 4 columns per thread: two words to every rank
    for (int o = threadIdx.x; o < kMB * 16 * 2; o += blockDim.x) {
      const int m = o >> 1, q = (o & 1) * 4;
      if (m >= M || n0 + q >= d) continue;
      float z[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        z[j] = part[m * 8 + q + j];
        for (int r = 1; r < ksplit; ++r) z[j] += ld_dsmem_f32(&part[m * 8 + q + j], static_cast<uint32_t>(r));
      }
      const uint64_t w0 = tag | pack_bf16x2(z[0], z[1]);
      const uint64_t w1 = tag | pack_bf16x2(z[2], z[3]);
      const size_t v = static_cast<size_t>(m) * d + n0 + q;
#pragma unroll
      for (int p = 0; p < kTP; ++p) {
        char* base = p == rank ? own : static_cast<char*>(regs.r[p]);
        st_words_sys(base + recv_off + rank * block + v * 4, w0, w1);
      }
    }
  }
  // rank 0 has read every peer's part[] before any CTA of the cluster exits
  if (ksplit > 1) cluster_sync();
  pdl_trigger();   // every CTA of this grid is resident once all have pushed
  if (static_cast<int>(blockIdx.x) * kSkinnyWarps >= M) return;

  const int row = blockIdx.x * kSkinnyWarps + warp;
  if (row >= M) return;
  const int nvec = d >> 3;
  int ok = 1;
  const uint64_t t0 = globaltimer();
  const size_t off = static_cast<size_t>(row) * d;
  float v[kMaxVec][8];
  uint4 xr[kMaxVec];
#pragma unroll
  for (int i = 0; i < kMaxVec; ++i) {
    const int c = lane + i * 32;
    if (c < nvec) xr[i] = reinterpret_cast<const uint4*>(x + off)[c];
  }
  // every rank's words of this row, a group of vectors per polling round
  constexpr int kG = poll_group<kMaxVec, kTP>();
#pragma unroll
  for (int i0 = 0; i0 < kMaxVec; i0 += kG)
    poll_sum<kMaxVec, kTP, kG>(own + recv_off, block, off, lane, nvec, i0, -1, seq, t0, &ok, v,
                               nullptr);
#pragma unroll
  for (int i = 0; i < kMaxVec; ++i) {
    const int c = lane + i * 32;
    if (c < nvec) {
      bf16x8_add(xr[i], v[i]);
#pragma unroll
      for (int e = 0; e < 8; ++e) v[i][e] += bias ? __ldg(bias + c * 8 + e) : 0.f;
    }
  }
  add_ln_row<kMaxVec>(v, lane, nvec, d, off, gamma, beta, s_out, y, eps);
  // the call counter moves on once every rank's words of row 0 (pushed by
  // every CTA of every rank, after reading the counter) have arrived
  if (row == 0 && lane == 0) *fused_counter = seq & kSeqMask;
  if (!ok && lane == 0 && err_word) atomicCAS(err_word, 0, kDevErrTimeoutComm);
}

template <int kMaxVec, int kTP>
cudaError_t launch_one(dim3 grid, cudaStream_t stream, const CommRegions& regs, int rank,
                       const size_t (&so)[3], const __nv_bfloat16* x, const float* bias,
                       const float* gamma, const float* beta, __nv_bfloat16* s_out,
                       __nv_bfloat16* y, int rows, int d, float eps, int* err_word) {
  return launch_ex(allreduce_add_ln_kernel<kMaxVec, kTP>, grid, dim3(256), 0, stream, 1, true,
                   regs, static_cast<char*>(regs.r[rank]), rank, so[0], so[1], so[2], x, bias,
                   gamma, beta, s_out, y, rows, d, eps, err_word);
}

template <int kMaxVec>
cudaError_t launch_tp(int tp, dim3 grid, cudaStream_t stream, const CommRegions& regs, int rank,
                      const size_t (&so)[3], const __nv_bfloat16* x, const float* bias, const float* gamma,
                      const float* beta, __nv_bfloat16* s_out, __nv_bfloat16* y, int rows, int d,
                      float eps, int* err_word) {
  switch (tp) {
#define ND_TP_CASE(n) \
  case n:             \
    return launch_one<kMaxVec, n>(grid, stream, regs, rank, so, x, bias, gamma, beta, s_out, y, rows, d, eps, err_word);
    ND_TP_CASE(1) ND_TP_CASE(2) ND_TP_CASE(3) ND_TP_CASE(4)
    ND_TP_CASE(5) ND_TP_CASE(6) ND_TP_CASE(7) ND_TP_CASE(8)
#undef ND_TP_CASE
    default:
      return cudaErrorInvalidValue;
  }
}

template <int kMB, int kMaxVec, int kTP>
cudaError_t launch_fused_one(cudaStream_t stream, const __nv_bfloat16* A,
                             const __nv_bfloat16* W, int M, int d, int K, const CommRegions& regs,
                             int rank, size_t recv_off, size_t block, const __nv_bfloat16* x,
                             const float* bias, const float* gamma, const float* beta,
                             __nv_bfloat16* s_out, __nv_bfloat16* y, float eps, int* err_word) {
  auto kern = gemm_allreduce_ln_kernel<kMB, kMaxVec, kTP>;
  const int ks = skinny_ksplit(d, K, current_sm_count());
  const int grid = (d / 8) * ks;
  return launch_ex(kern, dim3(grid), dim3(kSkinnyWarps * 32), 0, stream, ks, true, A, W, M, d, K,
                   regs, static_cast<char*>(regs.r[rank]), rank, recv_off, block, x, bias, gamma,
                   beta, s_out, y, eps, err_word);
}

template <int kMB, int kMaxVec>
cudaError_t launch_fused_tp(int tp, cudaStream_t stream, const __nv_bfloat16* A,
                            const __nv_bfloat16* W, int M, int d, int K, const CommRegions& regs,
                            int rank, size_t recv_off, size_t block, const __nv_bfloat16* x,
                            const float* bias, const float* gamma, const float* beta,
                            __nv_bfloat16* s_out, __nv_bfloat16* y, float eps, int* err_word) {
#define ND_FUSED(n)                                                                            \
  launch_fused_one<kMB, kMaxVec, n>(stream, A, W, M, d, K, regs, rank, recv_off, block, x, \
                                    bias, gamma, beta, s_out, y, eps, err_word)
  switch (tp) {
    case 1: return ND_FUSED(1);
    case 2: return ND_FUSED(2);
    case 4: return ND_FUSED(4);
    case 8: return ND_FUSED(8);
    default: return cudaErrorInvalidValue;
  }
#undef ND_FUSED
}

template <int kMB>
cudaError_t launch_fused_d(int tp, cudaStream_t stream, const __nv_bfloat16* A,
                           const __nv_bfloat16* W, int M, int d, int K, const CommRegions& regs,
                           int rank, size_t recv_off, size_t block, const __nv_bfloat16* x,
                           const float* bias, const float* gamma, const float* beta,
                           __nv_bfloat16* s_out, __nv_bfloat16* y, float eps, int* err_word) {
  if (d <= 256)
    return launch_fused_tp<kMB, 1>(tp, stream, A, W, M, d, K, regs, rank, recv_off, block, x, bias, gamma, beta, s_out, y, eps, err_word);
  if (d <= 512)
    return launch_fused_tp<kMB, 2>(tp, stream, A, W, M, d, K, regs, rank, recv_off, block, x, bias, gamma, beta, s_out, y, eps, err_word);
  return launch_fused_tp<kMB, 4>(tp, stream, A, W, M, d, K, regs, rank, recv_off, block, x, bias, gamma, beta, s_out, y, eps, err_word);
}

}  // namespace

bool fused_projection_supported(int tp, int M, int d, int K) {
  return (tp == 1 || tp == 2 || tp == 4 || tp == 8) && M >= 1 && M <= 32 && d >= 8 &&
         d % 8 == 0 && d <= 1024 && K >= 32 && K % 32 == 0;
}

cudaError_t launch_gemm_allreduce_add_layernorm(cudaStream_t stream, const CommRegions& regs,
                                                int tp, int rank, int slot, int rows_max,
                                                const __nv_bfloat16* A, const __nv_bfloat16* W,
                                                int K, const __nv_bfloat16* x, const float* bias,
                                                const float* gamma, const float* beta,
                                                __nv_bfloat16* s_out, __nv_bfloat16* y, int M,
                                                int d, float eps, int* err_word) {
  if (!fused_projection_supported(tp, M, d, K) || rank < 0 || rank >= tp || M > rows_max)
    return cudaErrorInvalidValue;
  const size_t block = static_cast<size_t>(rows_max) * d * 4;
  const size_t recv_off = comm_slot_offset(2, rows_max, d) + static_cast<size_t>(slot) * kCommMaxRanks * block;
  if (M <= 16)
    return launch_fused_d<1>(tp, stream, A, W, M, d, K, regs, rank, recv_off, block, x, bias, gamma, beta, s_out, y, eps, err_word);
  return launch_fused_d<2>(tp, stream, A, W, M, d, K, regs, rank, recv_off, block, x, bias, gamma, beta, s_out, y, eps, err_word);
}

// [header][own slot 0][own slot 1][receive area 0: kCommMaxRanks blocks][receive area 1];
// a block holds rows_max x d values as {sequence | 2 bf16} 8-byte words
size_t comm_region_bytes(int rows_max, int d) {
  return comm_slot_offset(2, rows_max, d) +
         2 * static_cast<size_t>(kCommMaxRanks) * rows_max * d * 4;
}

size_t comm_slot_offset(int slot, int rows_max, int d) {
  const size_t header = kHeaderBytes;
  return header + static_cast<size_t>(slot) * rows_max * d * 2;
}

int comm_grid(int rows, int sms) {
  int g = (rows + 7) / 8;
  if (g > sms) g = sms;
  if (g > kCommMaxCtas) g = kCommMaxCtas;
  return g < 1 ? 1 : g;
}

cudaError_t launch_allreduce_add_layernorm(cudaStream_t stream, const CommRegions& regs, int tp,
                                           int rank, int slot, int rows_max,
                                           const __nv_bfloat16* x, const float* bias,
                                           const float* gamma, const float* beta,
                                           __nv_bfloat16* s_out, __nv_bfloat16* y, int rows,
                                           int d, float eps, int sms, int* err_word) {
  if (tp < 1 || tp > kCommMaxRanks || rank < 0 || rank >= tp) return cudaErrorInvalidValue;
  const dim3 grid(comm_grid(rows, sms));
  const size_t block = static_cast<size_t>(rows_max) * d * 4;
  const size_t so[3] = {comm_slot_offset(slot, rows_max, d),
                        comm_slot_offset(2, rows_max, d) + static_cast<size_t>(slot) * kCommMaxRanks * block,
                        block};
  if (d <= 256)
    return launch_tp<1>(tp, grid, stream, regs, rank, so, x, bias, gamma, beta, s_out, y, rows, d, eps, err_word);
  else if (d <= 512)
    return launch_tp<2>(tp, grid, stream, regs, rank, so, x, bias, gamma, beta, s_out, y, rows, d, eps, err_word);
  else if (d <= 1024)
    return launch_tp<4>(tp, grid, stream, regs, rank, so, x, bias, gamma, beta, s_out, y, rows, d, eps, err_word);
  return launch_tp<8>(tp, grid, stream, regs, rank, so, x, bias, gamma, beta, s_out, y, rows, d, eps, err_word);
}

}  // namespace nd
