// tp_comm.cu — one-shot all-reduce over NVLink peer memory, fused with the
// residual add, bias and LayerNorm that follow a tensor-parallel row-parallel
// projection (the out-projection and MLP-down of a Megatron block):
//
//   s = x + Σ_r p_r + bias   (p_r: rank r's partial sum),  y = LayerNorm(s)
//
// Every rank owns a "region" of device memory shared with the other ranks
// through CUDA IPC handles: a header of flags and counters, then two slots of
// rows_max x d bf16 partial sums.  A caller's GEMM writes its partial into
// its own region's slot; this kernel then
//   1. per CTA, publishes a sequence number into every peer's flag array
//      (release at system scope) and waits, bounded, for every peer's number
//      for the same CTA (acquire): a peer that has reached this point has
//      finished the GEMM that wrote its partial;
//   2. reads the rows of its share from all ranks' slots with plain loads over
//      NVLink (no multicast), sums them in rank order — every rank computes
//      the same bits — adds x and the bias, stores s and the LayerNorm of s.
// Slots alternate between calls: a peer that publishes call n+1 has finished
// every read of call n (its kernels run in stream order), so a rank's GEMM of
// call n+2 may overwrite the slot of call n.  Each CTA keeps its own sequence
// counter in the local header, so captured CUDA graphs replay correctly.
// A wait that passes the deadline sets the device error word and the CTA
// skips its rows (garbage out, no hang).
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

// Flags use the fence / relaxed-access form of release and acquire: one
// system-scope fence before the stores to every peer (a st.release per peer
// would wait for each earlier remote store to complete before the next), and
// relaxed polls followed by one fence once every peer's flag is seen.
__device__ __forceinline__ void st_relaxed_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_relaxed_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.relaxed.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
// 16 bytes, cached in L2 only (a slot is rewritten every other call)
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

// kTP is the rank count: a compile-time count lets every rank's slot load of
// a row issue before the first one is used (a runtime count leaves each load
// behind its own branch, so the NVLink reads of a row go out one at a time).
// `own` is this rank's region (regs.r[rank]), passed on its own so that no
// dynamic index into the region array puts that array in local memory.
template <int kMaxVec, int kTP>
__global__ void __launch_bounds__(256)
    allreduce_add_ln_kernel(CommRegions regs, char* own, int rank, size_t slot_off,
                            const __nv_bfloat16* x, const float* __restrict__ bias,
                            const float* __restrict__ gamma, const float* __restrict__ beta,
                            __nv_bfloat16* s_out, __nv_bfloat16* __restrict__ y, int rows, int d,
                            float eps, int* __restrict__ err_word) {
  __shared__ int s_ok;
  const int warps = blockDim.x >> 5;
  const int lane = threadIdx.x & 31;
  const int nvec = d >> 3;
  const int row0 = blockIdx.x * warps + (threadIdx.x >> 5);
  // This rank's inputs (x, bias, gamma, beta) come from earlier work on this
  // stream, so the first row's loads go out before the peers' flags are
  // awaited; only the partial sums in the slots wait for them.  bias, gamma
  // and beta (the same for every row) are constant operands and go out even
  // before the previous kernel has finished (programmatic dependent launch).
  uint4 xr[kMaxVec];
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
  if (row0 < rows) {
#pragma unroll
    for (int i = 0; i < kMaxVec; ++i) {
      const int c = lane + i * 32;
      if (c < nvec) xr[i] = reinterpret_cast<const uint4*>(x + static_cast<size_t>(row0) * d)[c];
    }
  }

  if (threadIdx.x == 0) {
    uint32_t* counters = reinterpret_cast<uint32_t*>(own + kCountersOff);
    const uint32_t seq = counters[blockIdx.x] + 1;
    __threadfence_system();  // release: this rank's slot before the flags
#pragma unroll
    for (int p = 0; p < kTP; ++p) {
      if (p == rank) continue;
      uint32_t* flags = reinterpret_cast<uint32_t*>(regs.r[p]);
      st_relaxed_sys(flags + rank * kCommMaxCtas + blockIdx.x, seq);
    }
    int ok = 1;
    const uint32_t* mine = reinterpret_cast<const uint32_t*>(own);
    const uint64_t t0 = globaltimer();
    for (int p = 0; p < kTP && ok; ++p) {
      if (p == rank) continue;
      const uint32_t* f = mine + p * kCommMaxCtas + blockIdx.x;
      uint32_t it = 0;
      while (static_cast<int32_t>(ld_relaxed_sys(f) - seq) < 0) {
        if ((++it & 63u) == 0 && globaltimer() - t0 > ND_WAIT_TIMEOUT_NS) {
          ok = 0;
          if (err_word) atomicCAS(err_word, 0, kDevErrTimeoutComm);
          break;
        }
      }
    }
    __threadfence_system();  // acquire: the peers' slots after their flags
    counters[blockIdx.x] = seq;
    s_ok = ok;
  }
  __syncthreads();
  if (!s_ok) return;

  for (int row = row0; row < rows; row += gridDim.x * warps) {
    const size_t off = static_cast<size_t>(row) * d;
    if (row != row0) {
#pragma unroll
      for (int i = 0; i < kMaxVec; ++i) {
        const int c = lane + i * 32;
        if (c < nvec) xr[i] = reinterpret_cast<const uint4*>(x + off)[c];
      }
    }
    float v[kMaxVec][8];
    float sum = 0.f;
#pragma unroll
    for (int i = 0; i < kMaxVec; ++i) {
      const int c = lane + i * 32;
      if (c < nvec) {
        // every rank's 16 bytes in flight together, then the partial sums in
        // rank order, the residual and the bias
        uint4 pv[kTP];
#pragma unroll
        for (int p = 0; p < kTP; ++p)
          pv[p] = ld_cg16(static_cast<const char*>(regs.r[p]) + slot_off + (off + c * 8) * 2);
#pragma unroll
        for (int e = 0; e < 8; ++e) v[i][e] = 0.f;
#pragma unroll
        for (int p = 0; p < kTP; ++p) bf16x8_add(pv[p], v[i]);
        bf16x8_add(xr[i], v[i]);
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
  }
}

template <int kMaxVec, int kTP>
cudaError_t launch_one(dim3 grid, cudaStream_t stream, const CommRegions& regs, int rank,
                       size_t so, const __nv_bfloat16* x, const float* bias, const float* gamma,
                       const float* beta, __nv_bfloat16* s_out, __nv_bfloat16* y, int rows, int d,
                       float eps, int* err_word) {
  return launch_ex(allreduce_add_ln_kernel<kMaxVec, kTP>, grid, dim3(256), 0, stream, 1, true,
                   regs, static_cast<char*>(regs.r[rank]), rank, so, x, bias, gamma, beta, s_out,
                   y, rows, d, eps, err_word);
}

template <int kMaxVec>
cudaError_t launch_tp(int tp, dim3 grid, cudaStream_t stream, const CommRegions& regs, int rank,
                      size_t so, const __nv_bfloat16* x, const float* bias, const float* gamma,
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

size_t comm_region_bytes(int rows_max, int d) {
  return comm_slot_offset(0, rows_max, d) + 2 * static_cast<size_t>(rows_max) * d * 2;
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
  const size_t so = comm_slot_offset(slot, rows_max, d);
  if (d <= 256)
    return launch_tp<1>(tp, grid, stream, regs, rank, so, x, bias, gamma, beta, s_out, y, rows, d, eps, err_word);
  else if (d <= 512)
    return launch_tp<2>(tp, grid, stream, regs, rank, so, x, bias, gamma, beta, s_out, y, rows, d, eps, err_word);
  else if (d <= 1024)
    return launch_tp<4>(tp, grid, stream, regs, rank, so, x, bias, gamma, beta, s_out, y, rows, d, eps, err_word);
  return launch_tp<8>(tp, grid, stream, regs, rank, so, x, bias, gamma, beta, s_out, y, rows, d, eps, err_word);
}

}  // namespace nd
