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
#include "tp_comm.h"

namespace nd {
namespace {

// header: flags[kCommMaxRanks][kCommMaxCtas] (written by peers), then
// counters[kCommMaxCtas] (this rank's own sequence numbers)
constexpr size_t kFlagsBytes = sizeof(uint32_t) * kCommMaxRanks * kCommMaxCtas;
constexpr size_t kCountersOff = kFlagsBytes;

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
  // bias, gamma and beta are constant operands: loaded before the previous
  // kernel (the GEMM writing this rank's partial) has finished, under
  // programmatic dependent launch
  float bs[kMaxVec][8], gm[kMaxVec][8], bt[kMaxVec][8];
#pragma unroll
  for (int i = 0; i < kMaxVec; ++i) {
    const int c = lane + i * 32;
    if (c < nvec) {
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        bs[i][e] = bias ? __ldg(bias + c * 8 + e) : 0.f;
        gm[i][e] = gamma ? __ldg(gamma + c * 8 + e) : 1.f;
        bt[i][e] = beta ? __ldg(beta + c * 8 + e) : 0.f;
      }
    }
  }
  pdl_wait();  // x and this rank's partial come from earlier kernels
  pdl_trigger();
  __shared__ uint32_t s_seq;
  uint32_t* counters = reinterpret_cast<uint32_t*>(own + kCountersOff);
  if (threadIdx.x == 0) s_seq = counters[blockIdx.x] + 1;
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

  // 3. sum in rank order from local memory, residual, bias, LayerNorm
  for (int row = row0; row < rows; row += row_step) {
    const size_t off = static_cast<size_t>(row) * d;
    float v[kMaxVec][8];
    float sum = 0.f;
#pragma unroll
    for (int i = 0; i < kMaxVec; ++i) {
      const int c = lane + i * 32;
      if (c < nvec) {
        uint4 pv[kTP];
#pragma unroll
        for (int p = 0; p < kTP; ++p) {
          if (p == rank) {
            pv[p] = ld_cg16(mine_p + (off + c * 8) * 2);
            continue;
          }
          // 2. the peer's words of this call: poll until all four carry seq
          const char* src = own + recv_off + p * block + (off + c * 8) * 4;
          uint64_t w0, w1, w2, w3;
          uint32_t it = 0;
          for (;;) {
            ld_words_sys(src, w0, w1);
            ld_words_sys(src + 16, w2, w3);
            if (static_cast<uint32_t>(w0 >> 32) == seq && static_cast<uint32_t>(w1 >> 32) == seq &&
                static_cast<uint32_t>(w2 >> 32) == seq && static_cast<uint32_t>(w3 >> 32) == seq)
              break;
            if ((++it & 63u) == 0 && globaltimer() - t0 > ND_WAIT_TIMEOUT_NS) {
              ok = 0;
              break;
            }
          }
          pv[p] = make_uint4(static_cast<uint32_t>(w0), static_cast<uint32_t>(w1),
                             static_cast<uint32_t>(w2), static_cast<uint32_t>(w3));
        }
        const uint4 xr = reinterpret_cast<const uint4*>(x + off)[c];
#pragma unroll
        for (int e = 0; e < 8; ++e) v[i][e] = 0.f;
#pragma unroll
        for (int p = 0; p < kTP; ++p) bf16x8_add(pv[p], v[i]);
        bf16x8_add(xr, v[i]);
#pragma unroll
        for (int e = 0; e < 8; ++e) v[i][e] += bs[i][e];
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
        for (int e = 0; e < 8; ++e) o[e] = (v[i][e] - mu) * rs * gm[i][e] + bt[i][e];
        reinterpret_cast<uint4*>(y + off)[c] = f32_to_bf16x8(o);
      }
    }
    if (!ok) break;
  }
  if (!ok && err_word) atomicCAS(err_word, 0, kDevErrTimeoutComm);
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

}  // namespace

// [header][own slot 0][own slot 1][receive area 0: kCommMaxRanks blocks][receive area 1];
// a block holds rows_max x d values as {sequence | 2 bf16} 8-byte words
size_t comm_region_bytes(int rows_max, int d) {
  return comm_slot_offset(2, rows_max, d) +
         2 * static_cast<size_t>(kCommMaxRanks) * rows_max * d * 4;
}

size_t comm_slot_offset(int slot, int rows_max, int d) {
  const size_t header = (kFlagsBytes + sizeof(uint32_t) * kCommMaxCtas + 255) & ~static_cast<size_t>(255);
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
