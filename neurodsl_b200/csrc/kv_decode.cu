// kv_decode.cu — single-token KV-cache decode attention (split-K over keys).
//
// Computes, per (batch, head), exact softmax attention of one query row over
// the first L cached keys:  out = softmax(q·Kᵀ·scale) · V.  This is the
// reference's simple CPU attention (src/flash_attention.jl:49-69) with one
// query row and causal=false.  Optionally the token at position L-1 is taken
// from k_new / v_new and written into the caches in the same pass (the
// append step of a decode loop).
//
// HBM-bound: every cached K/V byte is read exactly once with 128-bit loads.
// Grid = (chunks, B*H); a CTA of 128 threads owns a chunk of 128 keys.  Each
// lane group of 8 threads reads one 128-byte key row (8 bf16 per lane), so a
// warp load instruction touches 4 consecutive rows (512 contiguous bytes).
// Partial (max, sum, acc[64]) per chunk go to a workspace; the last CTA of a
// head (atomic ticket) merges them and resets the ticket to zero.
#include <cuda_bf16.h>
#include <stdint.h>

#include <mutex>

#include "kv_decode.h"
#include "launch.cuh"
#include "tma.h"

namespace nd {

namespace {

constexpr int kD = 64;             // head_dim
constexpr int kChunk = 128;        // keys per CTA
constexpr int kThreads = 128;      // 4 warps
constexpr int kKeysPerWarp = kChunk / (kThreads / 32);  // 32
constexpr int kIters = kKeysPerWarp / 4;                // 8 (4 keys per warp load)
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

__device__ __forceinline__ void bf16x8_to_f32(const uint4& u, float (&f)[8]) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(w[i] << 16);
    f[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
  }
}

__device__ __forceinline__ uint4 ld_stream(const uint4* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

// atomicAdd with acquire-release ordering at gpu scope; returns the old value.
__device__ __forceinline__ unsigned int atom_add_acq_rel_gpu(unsigned int* p, unsigned int v) {
  unsigned int old;
  asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}

template <bool kOutF32>
__device__ __forceinline__ void store_out(void* out, size_t idx, float v) {
  if constexpr (kOutF32) {
    static_cast<float*>(out)[idx] = v;
  } else {
    static_cast<__nv_bfloat16*>(out)[idx] = __float2bfloat16_rn(v);
  }
}

// Scratch record for one chunk: running max (log2 units), sum, unnormalised acc.
struct ChunkPartial {
  float m;
  float l;
  float pad[2];
  float acc[kD];
};

template <bool kOutF32>
__global__ void __launch_bounds__(kThreads)
    kv_decode_kernel(const __nv_bfloat16* __restrict__ q, const __nv_bfloat16* __restrict__ k_new,
                     const __nv_bfloat16* __restrict__ v_new, __nv_bfloat16* __restrict__ k_cache,
                     __nv_bfloat16* __restrict__ v_cache, void* __restrict__ out,
                     float* __restrict__ lse, int L, int L_max, float scale_log2,
                     ChunkPartial* __restrict__ partials, unsigned int* __restrict__ tickets,
                     int H, long long qkv_ld) {
  const int chunk = blockIdx.x;
  const int nchunks = gridDim.x;
  const int bh = blockIdx.y;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int grp = lane >> 3;   // which of the 4 keys of a warp load
  const int sub = lane & 7;    // which 8-dim slice of the key row

  const size_t head_off = static_cast<size_t>(bh) * L_max * kD;
  const uint4* kbase = reinterpret_cast<const uint4*>(k_cache + head_off);
  const uint4* vbase = reinterpret_cast<const uint4*>(v_cache + head_off);
  const int key0 = chunk * kChunk + warp * kKeysPerWarp + grp;

  // Issue every K/V load of keys below L-1 before any arithmetic.  Under
  // programmatic dependent launch they go out before the previous kernel (the
  // one producing q, k_new and v_new) has finished: keys below L-1 were
  // written by earlier, finished work.  The key at L-1 may be the one the
  // previous kernel is writing (a projection epilogue that fills the cache),
  // so it is read only after pdl_wait(), from k_new / v_new or the cache.
  uint4 kr[kIters], vr[kIters];
#pragma unroll
  for (int it = 0; it < kIters; ++it) {
    const int key = key0 + it * 4;
    if (key < L - 1) {
      kr[it] = ld_stream(kbase + static_cast<size_t>(key) * (kD / 8) + sub);
      vr[it] = ld_stream(vbase + static_cast<size_t>(key) * (kD / 8) + sub);
    } else {
      kr[it] = make_uint4(0, 0, 0, 0);
      vr[it] = make_uint4(0, 0, 0, 0);
    }
  }

  pdl_wait();
  pdl_trigger();

  // q, k_new and v_new rows: batch b at b * qkv_ld, head h at h * 64
  const size_t qoff = static_cast<size_t>(bh / H) * qkv_ld + static_cast<size_t>(bh % H) * kD;
  float qf[8];
  {
    const uint4 qr = *reinterpret_cast<const uint4*>(q + qoff + sub * 8);
    bf16x8_to_f32(qr, qf);
#pragma unroll
    for (int i = 0; i < 8; ++i) qf[i] *= scale_log2;
  }

  // The key at L-1: with k_new / v_new it comes from them and is written into
  // the caches by the CTA that owns that key (the fused append); without them
  // it is read from the caches (coherent loads: the previous kernel may have
  // written it).
#pragma unroll
  for (int it = 0; it < kIters; ++it) {
    if (key0 + it * 4 == L - 1) {
      uint4* kdst = reinterpret_cast<uint4*>(k_cache + head_off) + static_cast<size_t>(L - 1) * (kD / 8) + sub;
      uint4* vdst = reinterpret_cast<uint4*>(v_cache + head_off) + static_cast<size_t>(L - 1) * (kD / 8) + sub;
      if (k_new != nullptr) {
        const uint4 kn = *reinterpret_cast<const uint4*>(k_new + qoff + sub * 8);
        const uint4 vn = *reinterpret_cast<const uint4*>(v_new + qoff + sub * 8);
        kr[it] = kn;
        vr[it] = vn;
        *kdst = kn;
        *vdst = vn;
      } else {
        kr[it] = __ldcg(kdst);
        vr[it] = __ldcg(vdst);
      }
    }
  }

  // Scores (log2 domain) for this thread's keys; all 8 lanes of a group end
  // with the same value after the xor-reduction.
  float s[kIters];
  float mloc = -INFINITY;
#pragma unroll
  for (int it = 0; it < kIters; ++it) {
    float kf[8];
    bf16x8_to_f32(kr[it], kf);
    float d = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) d = fmaf(qf[i], kf[i], d);
    d += __shfl_xor_sync(0xffffffffu, d, 1);
    d += __shfl_xor_sync(0xffffffffu, d, 2);
    d += __shfl_xor_sync(0xffffffffu, d, 4);
    s[it] = (key0 + it * 4 < L) ? d : -INFINITY;
    mloc = fmaxf(mloc, s[it]);
  }
  // warp max over the 4 groups
  mloc = fmaxf(mloc, __shfl_xor_sync(0xffffffffu, mloc, 8));
  mloc = fmaxf(mloc, __shfl_xor_sync(0xffffffffu, mloc, 16));

  float lsum = 0.f;
  float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  if (mloc != -INFINITY) {
#pragma unroll
    for (int it = 0; it < kIters; ++it) {
      const float p = exp2f(s[it] - mloc);
      lsum += p;
      float vf[8];
      bf16x8_to_f32(vr[it], vf);
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] = fmaf(p, vf[i], acc[i]);
    }
  }
  // reduce over the 4 groups (same dim slice)
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    acc[i] += __shfl_xor_sync(0xffffffffu, acc[i], 8);
    acc[i] += __shfl_xor_sync(0xffffffffu, acc[i], 16);
  }
  lsum += __shfl_xor_sync(0xffffffffu, lsum, 8);
  lsum += __shfl_xor_sync(0xffffffffu, lsum, 16);

  // cross-warp merge in shared memory
  __shared__ float sm_m[4], sm_l[4];
  __shared__ float sm_acc[4][kD];
  if (lane < 8) {
#pragma unroll
    for (int i = 0; i < 8; ++i) sm_acc[warp][sub * 8 + i] = acc[i];
  }
  if (lane == 0) {
    sm_m[warp] = mloc;
    sm_l[warp] = lsum;
  }
  __syncthreads();

  // thread t < 64 owns output dim t
  float cm = -INFINITY;
#pragma unroll
  for (int w = 0; w < 4; ++w) cm = fmaxf(cm, sm_m[w]);
  float cl = 0.f, cacc = 0.f;
  const int dim = threadIdx.x;
  if (cm != -INFINITY) {
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      const float f = (sm_m[w] == -INFINITY) ? 0.f : exp2f(sm_m[w] - cm);
      cl += sm_l[w] * f;
      if (dim < kD) cacc += sm_acc[w][dim] * f;
    }
  }

  if (nchunks == 1) {
    if (dim < kD) store_out<kOutF32>(out, static_cast<size_t>(bh) * kD + dim, cacc / cl);
    if (dim == 0 && lse != nullptr) lse[bh] = (cm + log2f(cl)) * kLn2;
    return;
  }

  ChunkPartial* mine = partials + static_cast<size_t>(bh) * nchunks + chunk;
  if (dim < kD) mine->acc[dim] = cacc;
  if (dim == 0) {
    mine->m = cm;
    mine->l = cl;
  }
  // The barrier orders this CTA's partial writes before thread 0's ticket
  // increment, whose release (gpu scope, cumulative over what the barrier
  // ordered) publishes them; the CTA that draws the last ticket acquires
  // every earlier release, and its barrier orders the merge reads after it.
  // One fence-carrying atomic per CTA instead of a fence in every thread.
  __syncthreads();
  __shared__ unsigned int s_ticket;
  if (threadIdx.x == 0) s_ticket = atom_add_acq_rel_gpu(&tickets[bh], 1u);
  __syncthreads();
  if (s_ticket != static_cast<unsigned int>(nchunks - 1)) return;

  // Last CTA of this head: merge every chunk's partial.  The global max
  // first (thread t reads chunk t's max; a block reduction), then each output
  // dim sums its chunks in order, eight chunks' loads in flight at a time, so
  // the partials' L2 reads overlap instead of taking one round trip per chunk.
  const ChunkPartial* all = partials + static_cast<size_t>(bh) * nchunks;
  float tm = -INFINITY;
  for (int c = threadIdx.x; c < nchunks; c += kThreads) tm = fmaxf(tm, __ldcg(&all[c].m));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) tm = fmaxf(tm, __shfl_xor_sync(0xffffffffu, tm, o));
  __shared__ float s_gm[kThreads / 32];
  if (lane == 0) s_gm[warp] = tm;
  __syncthreads();
  float gm = s_gm[0];
#pragma unroll
  for (int w = 1; w < kThreads / 32; ++w) gm = fmaxf(gm, s_gm[w]);
  float gl = 0.f, gacc = 0.f;
  for (int c0 = 0; c0 < nchunks; c0 += 8) {
    float mc[8], lc[8], ac[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int c = c0 + u;
      const bool in = c < nchunks;
      mc[u] = in ? __ldcg(&all[c].m) : -INFINITY;
      lc[u] = in ? __ldcg(&all[c].l) : 0.f;
      ac[u] = (in && dim < kD) ? __ldcg(&all[c].acc[dim]) : 0.f;
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const float f = (mc[u] == -INFINITY) ? 0.f : exp2f(mc[u] - gm);
      gl += lc[u] * f;
      gacc += ac[u] * f;
    }
  }
  if (dim < kD) store_out<kOutF32>(out, static_cast<size_t>(bh) * kD + dim, gacc / gl);
  if (dim == 0) {
    if (lse != nullptr) lse[bh] = (gm + log2f(gl)) * kLn2;
    tickets[bh] = 0u;  // leave the ticket ready for the next call
  }
}

}  // namespace

// Workspace layout, identical for every shape so that one zero-filled buffer
// can serve calls of any (B, H, L): [tickets: kMaxHeads x u32][partials].
// The ticket words sit at fixed offsets and every call returns the ones it
// used to zero, so the ticket region stays zero between calls.
size_t kv_decode_workspace_bytes(int B, int H, int L) {
  const int nchunks = (L + kChunk - 1) / kChunk;
  if (nchunks <= 1) return 0;
  const size_t heads = static_cast<size_t>(B) * H;
  return kv_decode_partials_offset() + heads * nchunks * sizeof(ChunkPartial);
}

size_t kv_decode_partials_offset() {
  const size_t tick = static_cast<size_t>(kDecodeMaxHeads) * sizeof(unsigned int);
  return (tick + 255) & ~static_cast<size_t>(255);
}

// ---- scratch for the allocation-free decode entry point --------------------
// A fixed block of device memory, part of the library image: every GPU that
// loads the library holds these kDecodeStaticScratchBytes until the process
// exits, and no call ever allocates.  It has the same layout as a
// caller-provided workspace (ticket region, then per-chunk partials).  In host
// code the name g_decode_static_scratch is only a host-side stand-in, not a
// device address: kv_decode_static_scratch() obtains the real address of this
// device's copy with cudaGetSymbolAddress, once per device.
static __device__ __align__(256) unsigned char g_decode_static_scratch[kDecodeStaticScratchBytes];

namespace {
constexpr int kScratchMaxDevices = 64;
void* g_static_scratch_addr[kScratchMaxDevices] = {};
unsigned long long g_static_scratch_ctx[kScratchMaxDevices] = {};
std::mutex g_static_scratch_mu;
}  // namespace

cudaError_t kv_decode_static_scratch(int device, cudaStream_t stream, void** ptr) {
  if (device < 0 || device >= kScratchMaxDevices) return cudaErrorInvalidDevice;
  const unsigned long long ctx = current_context_id();
  std::lock_guard<std::mutex> lk(g_static_scratch_mu);
  if (g_static_scratch_addr[device] == nullptr || g_static_scratch_ctx[device] != ctx) {
    // Set-up, once per device (and again if the device's context was torn
    // down and recreated since, which reloads the array at a possibly new
    // address), with `device` current (the caller's current device): resolve
    // this device's copy of the array and clear its ticket region, which must
    // start at zero (every call then returns the tickets it used to zero).
    // The clear is ordered on the caller's stream before the first kernel
    // that reads the tickets.
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_decode_static_scratch);
    if (e != cudaSuccess) return e;
    e = cudaMemsetAsync(p, 0, kv_decode_partials_offset(), stream);
    if (e != cudaSuccess) return e;
    g_static_scratch_addr[device] = p;
    g_static_scratch_ctx[device] = ctx;
  }
  *ptr = g_static_scratch_addr[device];
  return cudaSuccess;
}

cudaError_t launch_kv_decode(cudaStream_t stream, const __nv_bfloat16* q,
                             const __nv_bfloat16* k_new, const __nv_bfloat16* v_new,
                             __nv_bfloat16* k_cache, __nv_bfloat16* v_cache, void* out,
                             bool out_f32, float* lse, int B, int H, int L, int L_max, float scale,
                             void* workspace, long long qkv_ld) {
  const int nchunks = (L + kChunk - 1) / kChunk;
  dim3 grid(nchunks, B * H);
  ChunkPartial* partials = nullptr;
  unsigned int* tickets = nullptr;
  if (nchunks > 1) {
    tickets = static_cast<unsigned int*>(workspace);
    partials = reinterpret_cast<ChunkPartial*>(static_cast<char*>(workspace) +
                                               kv_decode_partials_offset());
  }
  const float scale_log2 = scale * kLog2e;
  if (qkv_ld <= 0) qkv_ld = static_cast<long long>(H) * kD;
  if (out_f32)
    return launch_ex(kv_decode_kernel<true>, grid, dim3(kThreads), 0, stream, 1, true, q, k_new,
                     v_new, k_cache, v_cache, out, lse, L, L_max, scale_log2, partials, tickets, H,
                     qkv_ld);
  return launch_ex(kv_decode_kernel<false>, grid, dim3(kThreads), 0, stream, 1, true, q, k_new,
                   v_new, k_cache, v_cache, out, lse, L, L_max, scale_log2, partials, tickets, H,
                   qkv_ld);
}

// Append one token's K/V rows at position `pos` of every (batch, head).
__global__ void kv_append_kernel(const uint4* __restrict__ k_new, const uint4* __restrict__ v_new,
                                 uint4* __restrict__ k_cache, uint4* __restrict__ v_cache,
                                 int heads, int pos, int L_max, int vec_per_row) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= heads * vec_per_row) return;
  const int bh = i / vec_per_row;
  const int v = i - bh * vec_per_row;
  const size_t dst = (static_cast<size_t>(bh) * L_max + pos) * vec_per_row + v;
  k_cache[dst] = k_new[i];
  v_cache[dst] = v_new[i];
}

cudaError_t launch_kv_append(cudaStream_t stream, const __nv_bfloat16* k_new,
                             const __nv_bfloat16* v_new, __nv_bfloat16* k_cache,
                             __nv_bfloat16* v_cache, int B, int H, int pos, int L_max, int D) {
  const int heads = B * H;
  const int vpr = D / 8;
  const int n = heads * vpr;
  if (n == 0) return cudaSuccess;
  kv_append_kernel<<<(n + 255) / 256, 256, 0, stream>>>(
      reinterpret_cast<const uint4*>(k_new), reinterpret_cast<const uint4*>(v_new),
      reinterpret_cast<uint4*>(k_cache), reinterpret_cast<uint4*>(v_cache), heads, pos, L_max,
      vpr);
  return cudaGetLastError();
}

}  // namespace nd
