/*
 * neurodsl_b200.h — C ABI of libneurodsl_b200.so, the B200 (sm_100a) kernels
 * behind NeuroDSL's transformer-inference operators.
 *
 * Every entry point takes plain device pointers, sizes and a CUDA stream
 * handle passed as void* (cudaStream_t; NULL = legacy default stream), is
 * asynchronous on that stream, and returns an int status (ND_OK = 0).  On a
 * non-zero status nd_last_error_string() describes the failure (thread-local).
 * Nothing here synchronises the device.
 *
 * Tensor layouts are C row-major.  Head-major attention tensors are
 * [B][H][S][D] (a Julia array of size (D, S, H, B) has the same bytes).  A
 * Julia column-major (rows, cols) Float32 matrix is converted to/from this
 * layout by nd_convert_2d.
 *
 * Reference interfaces replaced (paths inside the NeuroDSL project):
 *   nd_flash_attn_fwd   flash_attn_fwd!(::CUDADevice, out, Q, K, V, d_head; causal)
 *                       src/flash_attention.jl:116-134, reached from the
 *                       :flash_attn custom op _dispatch_flash_attn!
 *                       src/flash_attention.jl:175-200 (register_op! :203-208)
 *   nd_flash_attn_fwd_strided  the same, plus MultiHeadFlashAttention's
 *                       per-head :slice_cols / :hcat_heads copies
 *                       src/flash_attention.jl:225-256 (read and written
 *                       in place through strides)
 *   nd_kv_decode_attn   no reference counterpart (KV-cache decode is absent);
 *                       defined as flash_attn_fwd_cpu_simple!
 *                       (src/flash_attention.jl:49-69) with one query row
 *   nd_kv_decode_attn_qkv  nd_kv_decode_attn reading a fused QKV projection row
 *   nd_kv_append        no reference counterpart (cache append for decode)
 *   nd_set_pdl          no reference counterpart (launch mode of the decode steps)
 *   nd_gemm_qkv_cache_peers  no reference counterpart (prompt-sharded prefill
 *                       of a tensor-parallel model: K/V into the owners' caches)
 *   nd_set_sm_limit     no reference counterpart (SM share of the persistent
 *                       kernels, for compute overlapped with a collective)
 *   nd_gemm_bias_act    :linear src/dispatch.jl:363-384, :fused_matmul_add
 *                       :281-296, :matmul trans_b :213-243, residual :add
 *                       :386-417, fused_linear_gelu notebook/compiler.ipynb
 *                       cell 15 (rule name src/compiler_config.jl:154-158)
 *   nd_ln_gemm          residual :add src/dispatch.jl:386-417 + :layernorm +
 *                       :linear :363-384 for a decode step's few rows
 *   nd_add              :add with its vector broadcasts, src/dispatch.jl:386-417
 *   nd_gelu, nd_scale_mask, nd_softmax  the unfused :gelu (notebook/compiler.ipynb
 *                       cell 15 form), :scale_mask src/dispatch.jl:464-474 and
 *                       :softmax src/kernels.jl:269-287 ops
 *   nd_layernorm        the :layernorm rule symbol src/compiler_config.jl:168-172
 *                       (the reference ships only RMSNorm, rmsnorm_fwd!
 *                       src/kernels.jl:48-64,104-131, used by :rmsnorm
 *                       src/dispatch.jl:426-438)
 *   nd_convert_2d       Backend.to_device / Array() copies, src/backend.jl:20-26
 *   nd_convert_2d_padded  the same, writing an inner dimension padded with zeros
 *                       (the GEMMs' 16-byte rows; no reference counterpart)
 *   nd_gather_rows      :embedding src/dispatch.jl:476-491 (on the device)
 *   nd_copy_2d          :slice_cols src/dispatch.jl:544-553, :hcat_heads
 *                       :349-361 and :identity (device copies between views)
 *   nd_embed            :embedding src/dispatch.jl:476-491 (on the device) plus the
 *                       learned-position add of the GPT-2 graph
 *   nd_argmax           the greedy argmax over LM-head logits (:matmul trans_b
 *                       src/dispatch.jl:213-243 feeds it)
 *   nd_kv_store         no reference counterpart (prefill fills the decode cache)
 *   nd_gemm_qkv_cache   the QKV :linear (src/dispatch.jl:363-384) with that cache fill
 *   nd_add_layernorm    residual :add src/dispatch.jl:386-417 + :layernorm
 *   nd_comm_*, nd_allreduce_add_layernorm  no reference counterpart (multi-GPU
 *                       tensor-parallel reduction fused with :add + :layernorm)
 *   nd_gemm_allreduce_add_layernorm  the same, with the row-parallel :linear
 *                       before it in one launch
 */
#ifndef NEURODSL_B200_H
#define NEURODSL_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ----------------------------------------------------- */
#define ND_OK 0
#define ND_ERR_INVALID_ARG 1   /* null pointer where one is required, negative size */
#define ND_ERR_SHAPE 2         /* inconsistent or unsupported shape */
#define ND_ERR_ALIGNMENT 3     /* pointer not 16-byte aligned */
#define ND_ERR_UNSUPPORTED 4   /* dtype / head_dim / flag not supported */
#define ND_ERR_CUDA 5          /* CUDA runtime error (message has details) */
#define ND_ERR_DEVICE 6        /* current device is not an sm_100 GPU */
#define ND_ERR_WORKSPACE 7     /* workspace missing or too small */
#define ND_ERR_TIMEOUT 8       /* a kernel's bounded wait expired (nd_device_error) */

/* ---- element types ---------------------------------------------------- */
#define ND_F32 0
#define ND_BF16 1
#define ND_I32 2   /* index arrays only (nd_gather_rows) */
#define ND_I64 3   /* index arrays only (nd_gather_rows) */

/* ---- GEMM epilogue activation ------------------------------------------ */
#define ND_ACT_NONE 0
#define ND_ACT_GELU_SIGMOID 1  /* z * sigmoid(1.702 z): the reference's fused_linear_gelu */
#define ND_ACT_GELU_TANH 2     /* 0.5 z (1 + tanh(sqrt(2/pi) (z + 0.044715 z^3))) */
#define ND_ACT_GELU_ERF 3      /* 0.5 z (1 + erf(z / sqrt(2))) */

/* Library version (major*100 + minor). */
int nd_version(void);

/* Description of the last failure on the calling thread ("" if none). */
const char *nd_last_error_string(void);

/* 0 if `device` is an sm_100 GPU usable by this library, else ND_ERR_DEVICE. */
int nd_device_check(int device);

/* Read and clear the device-side error word (set when a kernel's bounded
 * wait expired; 0 = none).  Synchronises the current device. */
int nd_device_error(int *code);

/*
 * Attention prefill (flash attention forward).
 *   Q [B][H][Sq][D], K/V [B][H][Sk][D] bf16, 16-byte aligned; D must be 64.
 *   O [B][H][Sq][D] in o_dtype (ND_BF16 or ND_F32).
 *   lse, row_max: [B][H][Sq] fp32 or NULL — the reference's aux_data
 *   :flash_l (log-sum-exp) and :flash_m (row max of the scaled scores).
 *   scale: multiplies Q·Kᵀ (the reference uses 1/sqrt(d_head)).
 *   causal: key j is masked for query i when j > i; requires Sq == Sk.
 */
int nd_flash_attn_fwd(void *stream, const void *Q, const void *K, const void *V, void *O,
                      int o_dtype, float *lse, float *row_max, int B, int H, int Sq, int Sk,
                      int D, float scale, int causal);

/*
 * Attention prefill on strided tensors: the same computation as
 * nd_flash_attn_fwd, with each of Q, K, V and O given as element strides
 * {row, head, batch} (the D values of a row contiguous).  This reads an
 * (S, H·D) projection output directly (token-major: {H·D, D, S·H·D}) and
 * writes the (S, H·D) input of the output projection, replacing the per-head
 * :slice_cols and the :hcat_heads of MultiHeadFlashAttention
 * (src/flash_attention.jl:225-256, dispatch.jl:349-361,544-553).
 *   Strides: positive multiples of 8 elements; the batch stride the largest
 *   of a tensor's three; K and V both head-major (head stride > row stride)
 *   or both token-major.  lse, row_max stay [B][H][Sq] contiguous.
 */
int nd_flash_attn_fwd_strided(void *stream, const void *Q, const int64_t *q_strides,
                              const void *K, const int64_t *k_strides, const void *V,
                              const int64_t *v_strides, void *O, const int64_t *o_strides,
                              int o_dtype, float *lse, float *row_max, int B, int H, int Sq,
                              int Sk, int D, float scale, int causal);

/*
 * Scratch bytes needed by nd_kv_decode_attn for (B, H, L).  0 means the call
 * needs none.  A caller-provided workspace must be zero-filled once before
 * its first use; every call leaves it ready for the next.
 */
int nd_kv_decode_workspace_size(int B, int H, int L, int D, size_t *bytes);

/*
 * KV-cache single-token decode attention.
 *   q [B][H][D] bf16; k_cache, v_cache [B][H][L_max][D] bf16; attends over
 *   keys [0, L).  D must be 64.  If k_new and v_new (both [B][H][D] bf16) are
 *   given, they are the token at position L-1: they are written into the
 *   caches and used for that key (append fused into the attention pass).
 *   out [B][H][D] in o_dtype; lse [B][H] fp32 or NULL.
 *   workspace: nd_kv_decode_workspace_size bytes (zero-filled before first
 *   use), or NULL to use a buffer owned by the library for this device.
 */
int nd_kv_decode_attn(void *stream, const void *q, const void *k_new, const void *v_new,
                      void *k_cache, void *v_cache, void *out, int o_dtype, float *lse, int B,
                      int H, int L, int L_max, int D, float scale, void *workspace,
                      size_t workspace_bytes);

/*
 * KV-cache decode attention straight from a fused QKV projection.
 *   Row b of qkv (bf16, rows qkv_ld elements apart; qkv_ld >= 3*H*D and a
 *   multiple of 8) holds q [H][D], then k_new [H][D], then v_new [H][D]:
 *   the output of one linear layer whose weight stacks the query, key and
 *   value projections.  Same results as nd_kv_decode_attn with q, k_new and
 *   v_new taken from those column blocks (k_new / v_new are appended at
 *   position L-1); the other arguments are those of nd_kv_decode_attn.
 */
int nd_kv_decode_attn_qkv(void *stream, const void *qkv, int64_t qkv_ld, void *k_cache,
                          void *v_cache, void *out, int o_dtype, float *lse, int B, int H, int L,
                          int L_max, int D, float scale, void *workspace, size_t workspace_bytes);

/*
 * Programmatic dependent launch (PDL) for the calling host thread, off by
 * default; *previous (if not NULL) receives the earlier setting.  When on,
 * the decode-step kernels (nd_gemm_bias_act with M <= 32, nd_layernorm,
 * nd_add_layernorm, nd_allreduce_add_layernorm, nd_embed, nd_argmax and the
 * nd_kv_decode_attn family) are launched so that each may start while the
 * previous kernel on the stream is still running.  Before the previous
 * kernel finishes they read only operands the caller promises are not being
 * written: weights, biases and LayerNorm parameters, and in decode attention
 * the cached keys/values below position L-1.  Everything else (activations,
 * all writes) waits for the previous kernel.  Launches captured in a CUDA
 * graph keep the setting they were captured with.
 */
int nd_set_pdl(int enable, int *previous);

/*
 * Upper bound on the SMs the persistent kernels (nd_gemm_bias_act and its
 * fused forms with more than 32 rows, the nd_flash_attn_fwd family) occupy,
 * for launches from the calling host thread; 0 (the default) = all SMs.
 * *previous (if not NULL) receives the earlier setting.  The SMs left free
 * run kernels of other streams alongside, e.g. a collective that overlaps a
 * tensor-parallel prefill's compute.  Results do not depend on it.
 */
int nd_set_sm_limit(int sms, int *previous);

/*
 * Allocation-free KV-cache decode attention.  No counterpart in the
 * reference: it exists for callers that may not allocate device memory while
 * they run decode — a host runtime whose device memory all comes from its
 * own pool (a foreign cudaMalloc would escape the pool's accounting and its
 * limit), or a serving process that reserves its HBM at start-up and forbids
 * allocation and the device-wide synchronisation of cudaMalloc/cudaFree on
 * the token loop.  nd_kv_decode_attn either takes a caller workspace (which
 * someone must allocate) or grows a library-owned one with cudaMalloc; this
 * entry point does neither.
 *
 * Arguments and results are those of nd_kv_decode_attn without the
 * workspace.  Its scratch is a fixed 8 MiB block inside the library image
 * (held by every GPU that loads the library until the process exits);
 * shapes whose scratch exceeds it (256 KiB of tickets plus
 * B*H*ceil(L/128)*272 bytes of partials) are rejected with ND_ERR_WORKSPACE.
 * The first call on a device does a one-time set-up on `stream` (resolves the
 * block's device address, zero-fills its ticket words); make that first call
 * before any stream capture.  Every call shares the block and leaves the
 * tickets at zero for the next: calls that overlap on the GPU (concurrent
 * streams, or several host threads) race on it and must be serialised by the
 * caller.  It never calls cudaMalloc, cudaFree or an allocating routine.
 */
int nd_kv_decode_attn_noalloc(void *stream, const void *q, const void *k_new, const void *v_new,
                              void *k_cache, void *v_cache, void *out, int o_dtype, float *lse,
                              int B, int H, int L, int L_max, int D, float scale);

/* Write one token's K/V rows ([B][H][D] bf16) at position `pos` of the caches. */
int nd_kv_append(void *stream, const void *k_new, const void *v_new, void *k_cache, void *v_cache,
                 int B, int H, int pos, int L_max, int D);

/*
 * Fused linear layer: Y[M][N] = act(A[M][K] · W[N][K]ᵀ + bias[N]) + residual[M][N]
 *   A, W bf16 (K % 8 == 0, 16-byte aligned); bias fp32 [N] or NULL;
 *   residual [M][N] in residual_dtype or NULL; Y in y_dtype; act = ND_ACT_*.
 *   W is laid out like a Linear weight (out_features, in_features), i.e. the
 *   reference's :matmul with trans_b = true.
 */
int nd_gemm_bias_act(void *stream, const void *A, const void *W, const float *bias,
                     const void *residual, int residual_dtype, void *Y, int y_dtype, int M, int N,
                     int K, int act);

/*
 * The QKV projection of a prefill, filling the decode caches in the same
 * launch: Y[M][3*H*64] = A[M][K] · W[3*H*64][K]ᵀ + bias (bf16 Y, as
 * nd_gemm_bias_act), and the K and V column blocks of row m (token
 * s = m % S of sequence b = m / S, M = B*S) also go to position pos0 + s of
 * k_cache, v_cache [B][H][L_max][64] bf16 — what nd_kv_store would copy
 * afterwards, without reading the projection back.
 */
int nd_gemm_qkv_cache(void *stream, const void *A, const void *W, const float *bias, void *Y,
                      int M, int K, void *k_cache, void *v_cache, int B, int S, int H, int L_max,
                      int pos0);

/*
 * nd_gemm_qkv_cache over all tp·H heads of a model whose decode caches are
 * sharded by heads over tp ranks (no reference counterpart: the prefill of a
 * tensor-parallel model with the prompts sharded over the ranks).  This
 * rank's B prompts (sequences b0 .. b0+B-1 of the batch) are projected with
 * the full weights (W [3·tp·H·64][K], Y [M][3·tp·H·64]); the K and V columns
 * of head h are written straight into the caches of rank q = h / H as head
 * h - q·H, sequence b0 + b: k_caches[q], v_caches[q] [b0+B..][H][L_max][64]
 * bf16 are the ranks' caches mapped into this process (this rank's own
 * included; e.g. nd_comm_alloc regions), written with plain stores over
 * NVLink from the GEMM's epilogue.  The caller orders the ranks: no rank
 * reads a cache while another writes it, and a rank reads its caches only
 * after every writer's launch has finished (e.g. a collective on each
 * rank's stream before and after).  More than 32 rows (M = B·S), 16-byte
 * aligned bias; tp <= 8.
 */
int nd_gemm_qkv_cache_peers(void *stream, const void *A, const void *W, const float *bias,
                            void *Y, int M, int K, void *const *k_caches, void *const *v_caches,
                            int tp, int B, int b0, int S, int H, int L_max, int pos0);

/*
 * Few-row linear layer with the residual add and LayerNorm in its prologue
 * (the decode-step form of residual :add + :layernorm + :linear):
 *   s = bf16(x + (p + p_bias));  Y = act(LayerNorm(s) · Wᵀ + bias)
 *   x, p [M][K] bf16 (p NULL: s = x); p_bias, gamma, beta, bias fp32 or NULL
 *   (gamma NULL = 1, beta NULL = 0); LayerNorm over K with `eps`, computed
 *   like nd_add_layernorm.  s_out [M][K] bf16 receives s when not NULL and
 *   must not overlap x or p.  W [N][K] bf16; Y [M][N] in y_dtype.
 *   M <= 32, K % 32 == 0 and K <= 1024; every pointer 16-byte aligned.
 */
int nd_ln_gemm(void *stream, const void *x, const void *p, const float *p_bias,
               const float *gamma, const float *beta, float eps, void *s_out, const void *W,
               const float *bias, void *Y, int y_dtype, int M, int N, int K, int act);

/*
 * Unfused graph ops, fp32 in and out (the operator graph's Float32 values);
 * the compiler's rewrite rules replace them by the fused entry points, and
 * they run here when a graph is executed without rewriting.
 *   nd_gelu        y[i] = GELU(x[i]), i < n; act = ND_ACT_GELU_*   (:gelu)
 *   nd_scale_mask  y = x / sqrt(d_head), -Inf where col > row, for one
 *                  [rows][cols] score block  (:scale_mask with its causal mask)
 *   nd_softmax     row softmax of [rows][cols]; a row of -Inf gives zeros
 *                  (:softmax)
 */
int nd_gelu(void *stream, const float *x, float *y, int64_t n, int act);
int nd_scale_mask(void *stream, const float *x, float *y, int rows, int cols, int d_head);
int nd_softmax(void *stream, const float *x, float *y, int rows, int cols);

/*
 * The residual :add of the operator graph, fp32: y = a + b over
 * [rows][cols], with b the same shape (b_mode 0), one value per column
 * (b_mode 1, length cols), one per row (b_mode 2, length rows) or a single
 * value (b_mode 3) — the reference's matrix + vector broadcasts and the
 * general broadcast of its fallback branch for a (1, cols), (rows, 1) or
 * (1, 1) matrix b (src/dispatch.jl:386-417).
 */
int nd_add(void *stream, const float *a, const float *b, float *y, int rows, int cols, int b_mode);

/*
 * LayerNorm over the last dimension of x [rows][d]:
 *   y = (x - mean) / sqrt(var + eps) * gamma + beta
 *   x in x_dtype, y in y_dtype; gamma, beta fp32 [d] or NULL (1 / 0);
 *   mean, rstd fp32 [rows] or NULL.
 */
int nd_layernorm(void *stream, const void *x, int x_dtype, const float *gamma, const float *beta,
                 void *y, int y_dtype, float *mean, float *rstd, int rows, int d, float eps);

/*
 * Layout/dtype conversion of a 2-D matrix between a host-language array and
 * the row-major device layout used by this library.
 *   src_col_major = 1: src is column-major (rows, cols) (a Julia Matrix);
 *   dst is row-major [rows][cols].  src_col_major = 0: plain copy/convert.
 */
int nd_convert_2d(void *stream, const void *src, int src_dtype, int src_col_major, void *dst,
                  int dst_dtype, int rows, int cols);

/*
 * nd_convert_2d writing dst rows ld_dst elements apart (ld_dst >= cols), with
 * columns [cols, ld_dst) set to zero: an operand whose inner dimension is
 * not a multiple of 8 becomes a GEMM operand (16-byte rows) in one pass.
 */
int nd_convert_2d_padded(void *stream, const void *src, int src_dtype, int src_col_major,
                         void *dst, int dst_dtype, int rows, int cols, int ld_dst);

/*
 * The :embedding op on the device: out[i][:] = table[idx[i] - index_base][:]
 * for i < n.  table [vocab][d] and out [n][d] in dtype (ND_F32 or ND_BF16),
 * row strides ld_table / ld_out elements; idx holds n indices of idx_dtype:
 * ND_F32 (the reference's Float32 index arrays, 1-based with index_base 1),
 * ND_I32 or ND_I64.  An index outside [index_base, index_base + vocab), or a
 * Float32 index that is not an integer, gives a zero row and sets the device
 * error word to 16 (read and cleared by nd_device_error); the call itself
 * does not synchronise with the device.
 */
int nd_gather_rows(void *stream, const void *table, int dtype, long long ld_table, int vocab,
                   const void *idx, int idx_dtype, int index_base, int n, int d, void *out,
                   long long ld_out);

/*
 * dst[r][c] = src[r][c] for r < rows, c < cols, elements of elem_bytes (2 or
 * 4), row strides ld_src / ld_dst elements: the :slice_cols, :hcat_heads and
 * :identity copies between 2-D views (16-byte moves when the views allow).
 */
int nd_copy_2d(void *stream, const void *src, long long ld_src, void *dst, long long ld_dst,
               int rows, int cols, int elem_bytes);

/*
 * nd_copy_2d over `batch` (<= 65535) such views, the b-th at src + b·bs_src
 * and dst + b·bs_dst elements: dst[b][r][c] = src[b][r][c].  No reference
 * counterpart: packs each rank's key/value columns of a data-parallel
 * prefill for the all-to-all into the head-sharded decode caches.
 */
int nd_copy_2d_batched(void *stream, const void *src, long long ld_src, long long bs_src,
                       void *dst, long long ld_dst, long long bs_dst, int batch, int rows,
                       int cols, int elem_bytes);

/*
 * Token embedding with learned positions: y[t] = wte[ids[t]] + wpe[pos[t]].
 *   ids, pos int32 [T] (pos NULL: no position add); wte [vocab][d], wpe
 *   [n_pos][d], y [T][d] bf16; d % 8 == 0.  An id or position out of range
 *   gives a zero row and sets the device error word (nd_device_error).
 */
int nd_embed(void *stream, const int32_t *ids, const int32_t *pos, const void *wte,
             const void *wpe, void *y, int T, int d, int vocab, int n_pos);

/*
 * Greedy decoding: idx[r] = the first index of the largest value of logits
 * row r (rows x V, row stride ld elements, ND_BF16 or ND_F32), val[r] that
 * value (val may be NULL).  NaN never wins over a number.
 */
int nd_argmax(void *stream, const void *logits, int dtype, int64_t ld, int rows, int V,
              int32_t *idx, float *val);

/*
 * Prefill cache fill: the K and V rows of token (b, s) at columns k_col and
 * v_col of src [B·S][ld] bf16 (a QKV projection) are written to position
 * pos0 + s of k_cache, v_cache [B][H][L_max][D] bf16.  D must be 64; ld,
 * k_col and v_col multiples of 8; pos0 + S <= L_max.
 */
int nd_kv_store(void *stream, const void *src, int64_t ld, int k_col, int v_col, void *k_cache,
                void *v_cache, int B, int S, int H, int L_max, int pos0, int D);

/*
 * Residual add fused with the next LayerNorm (the residual :add
 * src/dispatch.jl:386-417 followed by :layernorm):
 *   s = x + p (+ bias),  y = (s - mean) / sqrt(var + eps) * gamma + beta
 *   x, s_out, y [rows][d] bf16 (s_out may be x); p [rows][d] in p_dtype
 *   (e.g. an all-reduced partial sum); bias, gamma, beta fp32 [d] or NULL.
 *   d % 8 == 0, d <= 2048.
 */
int nd_add_layernorm(void *stream, const void *x, const void *p, int p_dtype, const float *bias,
                     const float *gamma, const float *beta, void *s_out, void *y, int rows,
                     int d, float eps);

/*
 * Tensor-parallel reduction over NVLink peer memory, fused with the residual
 * add, bias and LayerNorm that follow a row-parallel projection (the
 * out-projection and MLP-down of a Megatron block).  No reference
 * counterpart: the reference runs on one device; this replaces an NCCL
 * all-reduce followed by nd_add_layernorm for small messages (decode).
 *
 * Every rank owns one "region" (nd_comm_region_bytes for rows_max x d),
 * allocated by nd_comm_alloc, whose 64-byte IPC handle the caller sends to
 * the other ranks; each opens the others' regions with nd_comm_open.  A
 * rank's partial sum [rows][d] bf16 is written by its GEMM into slot `slot`
 * of its own region (offset nd_comm_slot_offset(slot, rows_max, d)); then
 * every rank calls nd_allreduce_add_layernorm with the same arguments except
 * `rank` (regions[r] = rank r's region as mapped in this process) and gets
 *   s_out = x + Σ_r partial_r + bias (bf16),  y = LayerNorm(s_out)
 * computed with the same bits on every rank.  The call pushes the partial
 * into a receive area of every peer's region over NVLink and then reads only
 * local memory.  Calls must alternate slots
 * (0, 1, 0, ...), every rank makes the same calls in the same order, and a
 * peer that does not arrive within the library's wait limit (2 s) leaves
 * garbage in the outputs and sets the device error word (nd_device_error).
 */
int nd_comm_region_bytes(int rows_max, int d, size_t *bytes);
int nd_comm_slot_offset(int slot, int rows_max, int d, size_t *offset);
int nd_comm_alloc(size_t bytes, void **region, void *ipc_handle /* 64 bytes out */);
int nd_comm_open(const void *ipc_handle, void **peer_region);
int nd_comm_close(void *peer_region);
int nd_comm_free(void *region);
int nd_allreduce_add_layernorm(void *stream, void *const *regions, int tp, int rank,
                               size_t region_bytes, int rows_max, int slot, const void *x,
                               const float *bias, const float *gamma, const float *beta,
                               void *s_out, void *y, int rows, int d, float eps);

/*
 * The row-parallel projection of a decode step and the reduction after it in
 * one launch (no reference counterpart: the tensor-parallel out-projection /
 * MLP-down :linear, src/dispatch.jl:363-384, plus :add and :layernorm):
 *   s_out = x + Σ_r bf16(A_r [rows][K] · W_r [d][K]ᵀ) + bias,  y = LayerNorm(s_out)
 * where rank r passes its own A (bf16, its heads' attention output or its MLP
 * columns) and W (bf16, the matching columns of the projection).  The same
 * regions, rows_max and slot alternation as nd_allreduce_add_layernorm (the
 * two may be mixed, each call taking the next slot); the GEMM's tiles go
 * straight into every rank's receive area, so the own-partial slots are not
 * used.  Supported: tp 1, 2, 4 or 8, rows <= 32, d a multiple of 8 up to 1024,
 * K a multiple of 32 (ND_ERR_UNSUPPORTED otherwise).  The results are
 * bit-identical to nd_gemm_bias_act (no bias) into the own slot followed by
 * nd_allreduce_add_layernorm.
 */
int nd_gemm_allreduce_add_layernorm(void *stream, const void *A, const void *W, int K,
                                    void *const *regions, int tp, int rank, size_t region_bytes,
                                    int rows_max, int slot, const void *x, const float *bias,
                                    const float *gamma, const float *beta, void *s_out, void *y,
                                    int rows, int d, float eps);

#ifdef __cplusplus
}
#endif

#endif /* NEURODSL_B200_H */
