// tp_comm.h — one-shot all-reduce over NVLink peer memory fused with the
// residual add, bias and LayerNorm (see tp_comm.cu for the protocol).
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stddef.h>

namespace nd {

constexpr int kCommMaxRanks = 8;
constexpr int kCommMaxCtas = 256;

// The regions of all ranks as device addresses valid in this process
// (this rank's own allocation and the IPC mappings of the others).
struct CommRegions {
  void* r[kCommMaxRanks];
};

// Bytes of one rank's region for partial sums of up to rows_max x d bf16.
size_t comm_region_bytes(int rows_max, int d);
// Offset of slot 0 or 1 inside a region.
size_t comm_slot_offset(int slot, int rows_max, int d);
// CTAs one call uses for `rows` rows on a GPU with `sms` SMs (<= kCommMaxCtas).
int comm_grid(int rows, int sms);

// s_out = x + Σ_r slot_r + bias (bf16), y = LayerNorm(s_out) · gamma + beta;
// slot_r is rank r's partial in slot `slot` of its region.  Every rank must
// make the same sequence of calls with the same rows (CTA counts match).
cudaError_t launch_allreduce_add_layernorm(cudaStream_t stream, const CommRegions& regs, int tp,
                                           int rank, int slot, int rows_max,
                                           const __nv_bfloat16* x, const float* bias,
                                           const float* gamma, const float* beta,
                                           __nv_bfloat16* s_out, __nv_bfloat16* y, int rows,
                                           int d, float eps, int sms, int* err_word);

// Whether the fused projection below supports the shape (tp in {1, 2, 4, 8},
// M <= 32 rows, d a multiple of 8 up to 1024, K a multiple of 32).
bool fused_projection_supported(int tp, int M, int d, int K);

// The row-parallel projection fused with the reduction:
//   s_out = x + Σ_r bf16(A_r [M][K] · W_r [d][K]ᵀ) + bias,  y = LayerNorm(s_out)
// through the receive areas `slot` of the ranks' regions (the same regions
// and slot alternation as launch_allreduce_add_layernorm; the own-partial
// slots are not used).  Every rank makes the same calls in the same order.
cudaError_t launch_gemm_allreduce_add_layernorm(cudaStream_t stream, const CommRegions& regs,
                                                int tp, int rank, int slot, int rows_max,
                                                const __nv_bfloat16* A, const __nv_bfloat16* W,
                                                int K, const __nv_bfloat16* x, const float* bias,
                                                const float* gamma, const float* beta,
                                                __nv_bfloat16* s_out, __nv_bfloat16* y, int M,
                                                int d, float eps, int* err_word);

}  // namespace nd
