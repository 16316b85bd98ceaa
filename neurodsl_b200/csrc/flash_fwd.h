// flash_fwd.h — launcher for the tcgen05 attention-prefill kernel.
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>

namespace nd {

// Q [B][H][Sq][64], K/V [B][H][Sk][64] bf16 (16-byte aligned); O the same
// shape as Q in bf16 or fp32; lse / row_max [B][H][Sq] fp32 or null.
// causal requires Sq == Sk (mask j > i, the reference's convention).
cudaError_t launch_flash_fwd(cudaStream_t stream, const __nv_bfloat16* Q, const __nv_bfloat16* K,
                             const __nv_bfloat16* V, void* O, bool out_f32, float* lse,
                             float* row_max, int B, int H, int Sq, int Sk, float scale,
                             bool causal, const char** err_msg);

}  // namespace nd
