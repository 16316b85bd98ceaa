// model_ops.h — launchers of the decoder's auxiliary device ops.
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>

namespace nd {

// Device error word code for an embedding id or position out of range.
constexpr int kModelErrIndex = 16;

// y [T][d] bf16 = wte[ids[t]] + wpe[pos[t]] (pos may be null: no position
// add).  d % 8 == 0.  Out-of-range ids/positions give zeros and set the
// error word (err_word may be null).
cudaError_t launch_embed(cudaStream_t stream, const int* ids, const int* pos,
                         const __nv_bfloat16* wte, const __nv_bfloat16* wpe, __nv_bfloat16* y,
                         int T, int d, int vocab, int n_pos, int* err_word);

// idx[r] = first index of the maximum of logits row r (rows x V, row stride
// ld elements, bf16 or fp32); val[r] that maximum (val may be null).
cudaError_t launch_argmax(cudaStream_t stream, const void* logits, bool f32, long long ld,
                          int rows, int V, int* idx, float* val);

// K/V rows of token (b, s) at columns k_col / v_col of src [B·S][ld] bf16
// into positions pos0 + s of k_cache / v_cache [B][H][L_max][64].
cudaError_t launch_kv_store(cudaStream_t stream, const __nv_bfloat16* src, long long ld, int k_col,
                            int v_col, __nv_bfloat16* k_cache, __nv_bfloat16* v_cache, int B,
                            int S, int H, int L_max, int pos0);

// s_out = x + p (+ bias) (bf16; may alias x), y = LayerNorm(s_out) · gamma +
// beta (bf16).  p bf16 or fp32; rows x d with d % 8 == 0 and d <= 2048.
cudaError_t launch_add_layernorm(cudaStream_t stream, const __nv_bfloat16* x, const void* p,
                                 bool p_f32, const float* bias, const float* gamma,
                                 const float* beta, __nv_bfloat16* s_out, __nv_bfloat16* y,
                                 int rows, int d, float eps);

}  // namespace nd
