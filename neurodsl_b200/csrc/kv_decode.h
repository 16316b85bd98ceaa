// kv_decode.h — launchers for the decode-attention and KV-append kernels.
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stddef.h>

namespace nd {

// Most (batch, head) pairs one decode call may cover (grid.y limit).
constexpr int kDecodeMaxHeads = 65535;

// Scratch bytes for one decode call: a fixed ticket region of kDecodeMaxHeads
// words followed by the per-chunk partials.  The ticket region must be zero
// before the first call; every call leaves it at zero.
size_t kv_decode_workspace_bytes(int B, int H, int L);
size_t kv_decode_partials_offset();

// Size of the library's fixed decode scratch used by the allocation-free
// entry point: 8 MiB per GPU (256 KiB of tickets, the rest for partials).
constexpr size_t kDecodeStaticScratchBytes = static_cast<size_t>(8) << 20;

// Device address of that scratch on `device` (which must be current).  The
// first call on a device does the set-up: it resolves the address and clears
// the ticket region with cudaMemsetAsync on `stream`.  Allocates nothing.
cudaError_t kv_decode_static_scratch(int device, cudaStream_t stream, void** ptr);

// q, k_new and v_new hold one row of H*64 values per batch entry, rows
// qkv_ld elements apart (0: H*64, i.e. [B][H][64] contiguous).
cudaError_t launch_kv_decode(cudaStream_t stream, const __nv_bfloat16* q,
                             const __nv_bfloat16* k_new, const __nv_bfloat16* v_new,
                             __nv_bfloat16* k_cache, __nv_bfloat16* v_cache, void* out,
                             bool out_f32, float* lse, int B, int H, int L, int L_max, float scale,
                             void* workspace, long long qkv_ld = 0);

cudaError_t launch_kv_append(cudaStream_t stream, const __nv_bfloat16* k_new,
                             const __nv_bfloat16* v_new, __nv_bfloat16* k_cache,
                             __nv_bfloat16* v_cache, int B, int H, int pos, int L_max, int D);

}  // namespace nd
