// flash_fwd.h — launcher for the tcgen05 attention-prefill kernel.
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>

namespace nd {

// Element strides of Q, K, V and O as {row, head, batch}; the 64 head
// dimensions of a row are contiguous.  Head-major [B][H][S][64] is
// {64, S·64, H·S·64}; token-major [B][S][H][64] (the layout of an (S, H·64)
// projection output) is {H·64, 64, S·H·64}.
struct FlashStrides {
  long long q[3], k[3], v[3], o[3];
};

// Contiguous head-major strides for Q/O of length Sq and K/V of length Sk.
FlashStrides flash_head_major_strides(int H, int Sq, int Sk);

// Q [B][H][Sq][64], K/V [B][H][Sk][64] bf16 (16-byte aligned) at the given
// strides; O the same shape as Q in bf16 or fp32; lse / row_max [B][H][Sq]
// fp32 or null.  causal requires Sq == Sk (mask j > i, the reference's
// convention).
cudaError_t launch_flash_fwd(cudaStream_t stream, const __nv_bfloat16* Q, const __nv_bfloat16* K,
                             const __nv_bfloat16* V, void* O, bool out_f32, float* lse,
                             float* row_max, int B, int H, int Sq, int Sk, float scale,
                             bool causal, const FlashStrides& st, const char** err_msg);

}  // namespace nd
