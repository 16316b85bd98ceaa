/*
 * neurodsl_oracle.c — CPU restatement of NeuroDSL's Float32 hot-path math.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity oracle for the CUDA
 * library in neurodsl_b200/csrc.  It is linked only by tests/, by
 * __graft_entry__.smoke() and by bench.py's CPU-baseline leg, always as the
 * checker or the timed CPU baseline, never as a product code path.
 *
 * Parity status: UNPINNED against reference outputs.  The reference is Julia
 * (no Julia toolchain is installed where this builds or runs) and its test suite holds no golden
 * vectors; its only equivalence test for this path compares its tiled and
 * simple CPU attention with each other (test/test_runtime_optimizations.jl:55-69).
 * The same equivalence is re-asserted against this restatement in
 * tests/test_oracle.py, together with a float64 NumPy cross-check and the
 * committed fixtures under tests/golden/.
 *
 * Layout convention: every matrix is C row-major.  A Julia column-major
 * (N, D) Float32 matrix holds the same bytes as a C row-major [D][N] array;
 * the restatement works on the logical (row, col) indices, so the arithmetic
 * is the reference's, only the storage order is C's.
 *
 * Arithmetic is fp32 with fp32 accumulation, as Julia's Float32 BLAS calls
 * (mul!, Q*K') do.  libm expf/logf/tanhf/erff are called for the
 * transcendental functions.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define ORACLE_EXPORT __attribute__((visibility("default")))

/* ------------------------------------------------------------------------ */
/* small fp32 GEMM helpers (the BLAS calls of the reference)                 */
/* ------------------------------------------------------------------------ */

/* C[M][N] = A[M][K] * B[N][K]^T   (A·Bᵀ, both operands K-contiguous).
 * The dot product keeps 8 interleaved fp32 partial sums (as blocked BLAS
 * kernels do), which lets the compiler use SIMD lanes without -ffast-math. */
static void gemm_abt(const float *A, int lda, const float *B, int ldb, float *C, int ldc,
                     int M, int N, int K) {
    const int K8 = K & ~7;
    for (int i = 0; i < M; ++i) {
        const float *a = A + (size_t)i * lda;
        for (int j = 0; j < N; ++j) {
            const float *b = B + (size_t)j * ldb;
            float part[8] = {0, 0, 0, 0, 0, 0, 0, 0};
            for (int k = 0; k < K8; k += 8)
                for (int u = 0; u < 8; ++u) part[u] += a[k + u] * b[k + u];
            float acc = ((part[0] + part[1]) + (part[2] + part[3])) +
                        ((part[4] + part[5]) + (part[6] + part[7]));
            for (int k = K8; k < K; ++k) acc += a[k] * b[k];
            C[(size_t)i * ldc + j] = acc;
        }
    }
}

/* C[M][N] = A[M][K] * B[K][N]   (A·B, B row-contiguous). */
static void gemm_ab(const float *A, int lda, const float *B, int ldb, float *C, int ldc,
                    int M, int N, int K) {
    for (int i = 0; i < M; ++i) {
        float *c = C + (size_t)i * ldc;
        for (int j = 0; j < N; ++j) c[j] = 0.0f;
        const float *a = A + (size_t)i * lda;
        for (int k = 0; k < K; ++k) {
            const float av = a[k];
            const float *b = B + (size_t)k * ldb;
            for (int j = 0; j < N; ++j) c[j] += av * b[j];
        }
    }
}

/* ------------------------------------------------------------------------ */
/* a1: flash_attn_fwd_cpu_simple!  (src/flash_attention.jl:49-69)            */
/* ------------------------------------------------------------------------ */
/*
 * One head: Q [N][D], K [Nk][D], V [Nk][D], O [N][D].
 *   S = Q·Kᵀ · (1/√d_head)                            (:56-57)
 *   causal: S[i][j] = -Inf for j > i                  (:58-62)
 *   m = rowmax(S); E = exp(S - m); l = rowsum(E)      (:63-65)
 *   P = E / max(l, 1e-38); O = P·V                    (:66-67)
 *   returns (O, log(l) + m, m)                        (:68)
 * The reference's causal loop runs j over i+1..N, i.e. it assumes Nk == N;
 * callers here pass Nk == N whenever causal is set.
 * work: caller-provided scratch of N*Nk floats (the materialised S matrix).
 */
ORACLE_EXPORT int oracle_attn_simple(const float *Q, const float *K, const float *V, float *O,
                                     float *lse, float *m_out, int N, int Nk, int D, int d_head,
                                     int causal, float *work) {
    if (N < 0 || Nk < 0 || D <= 0 || d_head <= 0) return 1;
    if (causal && Nk != N) return 2;
    if (N == 0) return 0;
    const float scale = 1.0f / sqrtf((float)d_head);
    float *S = work;
    gemm_abt(Q, D, K, D, S, Nk, N, Nk, D);
    for (size_t t = 0; t < (size_t)N * Nk; ++t) S[t] *= scale;
    if (causal)
        for (int i = 0; i < N; ++i)
            for (int j = i + 1; j < N; ++j) S[(size_t)i * Nk + j] = -INFINITY;
    for (int i = 0; i < N; ++i) {
        float *s = S + (size_t)i * Nk;
        float mv = -INFINITY;
        for (int j = 0; j < Nk; ++j) mv = s[j] > mv ? s[j] : mv;
        float l = 0.0f;
        for (int j = 0; j < Nk; ++j) {
            s[j] = expf(s[j] - mv);
            l += s[j];
        }
        const float denom = l > 1e-38f ? l : 1e-38f;
        for (int j = 0; j < Nk; ++j) s[j] /= denom;
        if (lse) lse[i] = logf(l) + mv;
        if (m_out) m_out[i] = mv;
    }
    gemm_ab(S, Nk, V, D, O, D, N, D, Nk);
    return 0;
}

/* ------------------------------------------------------------------------ */
/* a2: flash_attn_fwd_cpu!  tiled online softmax (src/flash_attention.jl:9-46) */
/* ------------------------------------------------------------------------ */
/*
 * Key blocks of `block` rows (FLASH_BLOCK = 64, :6).  For each block:
 *   S = Q·Kjᵀ·scale over all queries (:26); causal masks kj_abs > qi (:27-34)
 *   m_new = max(m, rowmax S); O *= exp(m - m_new); l *= exp(m - m_new)
 *   E = exp(S - m_new); O += E·Vj; l += rowsum E; m = m_new          (:35-43)
 * finally O /= max(l, 1e-38); returns (O, log(max(l,1e-38)) + m, m)  (:45-46)
 * work: caller-provided scratch of N*block floats.
 */
ORACLE_EXPORT int oracle_attn_tiled(const float *Q, const float *K, const float *V, float *O,
                                    float *lse, float *m_out, int N, int Nk, int D, int d_head,
                                    int causal, int block, float *work, float *lbuf,
                                    float *mbuf) {
    if (N < 0 || Nk < 0 || D <= 0 || d_head <= 0 || block <= 0) return 1;
    if (causal && Nk != N) return 2;
    if (N == 0) return 0;
    const float scale = 1.0f / sqrtf((float)d_head);
    float *l = lbuf, *m = mbuf;
    for (int i = 0; i < N; ++i) {
        l[i] = 0.0f;
        m[i] = -INFINITY;
    }
    memset(O, 0, sizeof(float) * (size_t)N * D);
    for (int js = 0; js < Nk; js += block) {
        const int je = js + block < Nk ? js + block : Nk;
        const int nb = je - js;
        float *S = work;
        gemm_abt(Q, D, K + (size_t)js * D, D, S, nb, N, nb, D);
        for (size_t t = 0; t < (size_t)N * nb; ++t) S[t] *= scale;
        if (causal)
            for (int qi = 0; qi < N; ++qi)
                for (int ki = 0; ki < nb; ++ki)
                    if (js + ki > qi) S[(size_t)qi * nb + ki] = -INFINITY;
        for (int qi = 0; qi < N; ++qi) {
            float *s = S + (size_t)qi * nb;
            float bm = -INFINITY;
            for (int ki = 0; ki < nb; ++ki) bm = s[ki] > bm ? s[ki] : bm;
            const float m_new = m[qi] > bm ? m[qi] : bm;
            /* exp(-Inf - -Inf) is NaN in IEEE arithmetic, as in Julia; a row
             * whose every key so far is masked keeps m = -Inf, l = 0, O = 0. */
            const float ed = expf(m[qi] - m_new);
            float *o = O + (size_t)qi * D;
            for (int d = 0; d < D; ++d) o[d] *= ed;
            l[qi] *= ed;
            float rs = 0.0f;
            for (int ki = 0; ki < nb; ++ki) {
                s[ki] = expf(s[ki] - m_new);
                rs += s[ki];
            }
            const float *vj = V + (size_t)js * D;
            for (int ki = 0; ki < nb; ++ki) {
                const float p = s[ki];
                const float *v = vj + (size_t)ki * D;
                for (int d = 0; d < D; ++d) o[d] += p * v[d];
            }
            l[qi] += rs;
            m[qi] = m_new;
        }
    }
    for (int qi = 0; qi < N; ++qi) {
        const float den = l[qi] > 1e-38f ? l[qi] : 1e-38f;
        float *o = O + (size_t)qi * D;
        for (int d = 0; d < D; ++d) o[d] /= den;
        if (lse) lse[qi] = logf(den) + m[qi];
        if (m_out) m_out[qi] = m[qi];
    }
    return 0;
}

/* ------------------------------------------------------------------------ */
/* Batched multi-head prefill: a1 over every (batch, head) of [B][H][S][D].  */
/* ------------------------------------------------------------------------ */
/*
 * The reference runs one :flash_attn rule per head on (S, D) slices
 * (src/flash_attention.jl:241-251); this loops a1 over the B·H heads of a
 * head-major [B][H][S][D] tensor, `nthreads` heads at a time.
 * lse/m_out are [B][H][S] (may be NULL).  Returns 0 or the first error.
 */
ORACLE_EXPORT int oracle_attn_simple_bhsd(const float *Q, const float *K, const float *V,
                                          float *O, float *lse, float *m_out, int B, int H,
                                          int S, int Sk, int D, int causal, int nthreads) {
    if (B < 0 || H < 0) return 1;
    const long long heads = (long long)B * H;
    int err = 0;
#ifdef _OPENMP
    if (nthreads <= 0) nthreads = omp_get_max_threads();
#pragma omp parallel num_threads(nthreads)
#endif
    {
        float *work = (float *)malloc(sizeof(float) * ((size_t)S * (size_t)(Sk > 0 ? Sk : 1)));
#ifdef _OPENMP
#pragma omp for schedule(dynamic, 1)
#endif
        for (long long bh = 0; bh < heads; ++bh) {
            int rc = work ? oracle_attn_simple(Q + (size_t)bh * S * D, K + (size_t)bh * Sk * D,
                                               V + (size_t)bh * Sk * D, O + (size_t)bh * S * D,
                                               lse ? lse + (size_t)bh * S : NULL,
                                               m_out ? m_out + (size_t)bh * S : NULL, S, Sk, D, D,
                                               causal, work)
                          : 3;
            if (rc) {
#ifdef _OPENMP
#pragma omp critical
#endif
                err = err ? err : rc;
            }
        }
        free(work);
    }
    return err;
}

/* ------------------------------------------------------------------------ */
/* a10: KV-cache single-token decode = a1 with one query row, causal=false.  */
/* ------------------------------------------------------------------------ */
/*
 * q [B][H][D]; k_cache, v_cache [B][H][L_max][D]; attends over keys 0..L-1.
 * With N = size(Q,1) = 1 the reference's simple path (src/flash_attention.jl:49-69)
 * is exact single-query softmax attention over the L cached keys.
 * out [B][H][D]; lse [B][H] (may be NULL).
 */
ORACLE_EXPORT int oracle_kv_decode(const float *q, const float *k_cache, const float *v_cache,
                                   float *out, float *lse, int B, int H, int L, int L_max, int D,
                                   int nthreads) {
    if (B < 0 || H < 0 || L <= 0 || L > L_max || D <= 0) return 1;
    const long long heads = (long long)B * H;
    int err = 0;
#ifdef _OPENMP
    if (nthreads <= 0) nthreads = omp_get_max_threads();
#pragma omp parallel num_threads(nthreads)
#endif
    {
        float *work = (float *)malloc(sizeof(float) * (size_t)L);
#ifdef _OPENMP
#pragma omp for schedule(static)
#endif
        for (long long bh = 0; bh < heads; ++bh) {
            int rc = work ? oracle_attn_simple(q + (size_t)bh * D, k_cache + (size_t)bh * L_max * D,
                                               v_cache + (size_t)bh * L_max * D,
                                               out + (size_t)bh * D, lse ? lse + bh : NULL, NULL,
                                               1, L, D, D, 0, work)
                          : 3;
            if (rc) {
#ifdef _OPENMP
#pragma omp critical
#endif
                err = err ? err : rc;
            }
        }
        free(work);
    }
    return err;
}

/* ------------------------------------------------------------------------ */
/* a6-a8, a11: :linear / :fused_matmul_add / fused_linear_gelu / :add        */
/* ------------------------------------------------------------------------ */

enum { ORACLE_ACT_NONE = 0, ORACLE_GELU_SIGMOID = 1, ORACLE_GELU_TANH = 2, ORACLE_GELU_ERF = 3 };

/*
 * GELU variants.  ORACLE_GELU_SIGMOID is the reference's only executable
 * definition, the notebook @defop fused_linear_gelu (notebook/compiler.ipynb
 * cell 15): out = z · 1/(1 + exp(-1.702 z)).  The tanh and erf forms are the
 * usual published GELU definitions (Hendrycks & Gimpel 2016).
 */
static float gelu_apply(float z, int act) {
    switch (act) {
    case ORACLE_GELU_SIGMOID: return z * (1.0f / (1.0f + expf(-1.702f * z)));
    case ORACLE_GELU_TANH: {
        const float c = 0.7978845608028654f; /* sqrt(2/pi) */
        return 0.5f * z * (1.0f + tanhf(c * (z + 0.044715f * z * z * z)));
    }
    case ORACLE_GELU_ERF: return 0.5f * z * (1.0f + erff(z * 0.7071067811865476f));
    default: return z;
    }
}

/*
 * Y[M][N] = act( A·op(W) + bias ) + residual
 *   trans_w = 1: W is [N][K] and op(W) = Wᵀ  (:linear, src/dispatch.jl:363-384;
 *                :matmul trans_b=true, :213-243)
 *   trans_w = 0: W is [K][N]                 (:matmul / :fused_matmul_add, :281-296)
 *   bias [N] or NULL  (:linear adds inputs[3]' , :377-379; :fused_matmul_add :292)
 *   act: ORACLE_ACT_NONE or one GELU variant
 *   residual [M][N] or NULL (:add, :386-417, applied after the activation)
 */
ORACLE_EXPORT int oracle_linear(const float *A, const float *W, const float *bias,
                                const float *residual, float *Y, int M, int N, int K, int trans_w,
                                int act, int nthreads) {
    if (M < 0 || N < 0 || K < 0) return 1;
#ifdef _OPENMP
    if (nthreads <= 0) nthreads = omp_get_max_threads();
#pragma omp parallel for num_threads(nthreads) schedule(static)
#endif
    for (int i = 0; i < M; ++i) {
        if (trans_w)
            gemm_abt(A + (size_t)i * K, K, W, K, Y + (size_t)i * N, N, 1, N, K);
        else
            gemm_ab(A + (size_t)i * K, K, W, N, Y + (size_t)i * N, N, 1, N, K);
        float *y = Y + (size_t)i * N;
        for (int j = 0; j < N; ++j) {
            float z = y[j] + (bias ? bias[j] : 0.0f);
            z = gelu_apply(z, act);
            if (residual) z += residual[(size_t)i * N + j];
            y[j] = z;
        }
    }
    return 0;
}

/* ------------------------------------------------------------------------ */
/* a9: LayerNorm (the reference has only RMSNorm, src/kernels.jl:48-64)      */
/* ------------------------------------------------------------------------ */
/*
 * Per row of x [rows][d]:  mu = mean(x); var = mean((x-mu)^2);
 * rstd = 1/sqrt(var + eps); y = (x-mu)·rstd·gamma + beta.
 * The loop structure follows rmsnorm_fwd! (per-row reduction, then a scaled
 * write), with the mean subtraction and beta of a true LayerNorm.
 * mean/rstd [rows] may be NULL (they mirror aux_data[:rms_inv] of :rmsnorm,
 * src/dispatch.jl:426-438).
 */
ORACLE_EXPORT int oracle_layernorm(const float *x, const float *gamma, const float *beta, float *y,
                                   float *mean, float *rstd, int rows, int d, float eps) {
    if (rows < 0 || d <= 0) return 1;
    for (int i = 0; i < rows; ++i) {
        const float *xr = x + (size_t)i * d;
        float s = 0.0f;
        for (int j = 0; j < d; ++j) s += xr[j];
        const float mu = s / (float)d;
        float v = 0.0f;
        for (int j = 0; j < d; ++j) {
            const float t = xr[j] - mu;
            v += t * t;
        }
        const float r = 1.0f / sqrtf(v / (float)d + eps);
        float *yr = y + (size_t)i * d;
        for (int j = 0; j < d; ++j)
            yr[j] = (xr[j] - mu) * r * (gamma ? gamma[j] : 1.0f) + (beta ? beta[j] : 0.0f);
        if (mean) mean[i] = mu;
        if (rstd) rstd[i] = r;
    }
    return 0;
}

/* RMSNorm, rmsnorm_fwd! (src/kernels.jl:48-64), kept as the norm template. */
ORACLE_EXPORT int oracle_rmsnorm(const float *x, const float *gamma, float *y, float *rms_inv,
                                 int rows, int d, float eps) {
    if (rows < 0 || d <= 0) return 1;
    for (int i = 0; i < rows; ++i) {
        const float *xr = x + (size_t)i * d;
        float s = 0.0f;
        for (int j = 0; j < d; ++j) s += xr[j] * xr[j];
        const float r = 1.0f / sqrtf(s / (float)d + eps);
        if (rms_inv) rms_inv[i] = r;
        for (int j = 0; j < d; ++j) y[(size_t)i * d + j] = xr[j] * r * gamma[j];
    }
    return 0;
}

/* ------------------------------------------------------------------------ */
/* a12: row softmax (src/kernels.jl:269-287) and :scale_mask (:427-430)      */
/* ------------------------------------------------------------------------ */
ORACLE_EXPORT int oracle_softmax(const float *x, float *out, int nr, int nc) {
    if (nr < 0 || nc <= 0) return 1;
    for (int i = 0; i < nr; ++i) {
        const float *xr = x + (size_t)i * nc;
        float *o = out + (size_t)i * nc;
        float mx = xr[0];
        for (int j = 1; j < nc; ++j) mx = xr[j] > mx ? xr[j] : mx;
        float s = 0.0f;
        for (int j = 0; j < nc; ++j) {
            o[j] = expf(xr[j] - mx);
            s += o[j];
        }
        const float inv = 1.0f / s;
        for (int j = 0; j < nc; ++j) o[j] *= inv;
    }
    return 0;
}

/* out = scores · (1/√d_head) + causal_mask (mask[i][j] = 0 for j<=i else -Inf). */
ORACLE_EXPORT int oracle_scale_mask(const float *scores, float *out, int n, int d_head) {
    if (n < 0 || d_head <= 0) return 1;
    const float sc = 1.0f / sqrtf((float)d_head);
    for (int i = 0; i < n; ++i)
        for (int j = 0; j < n; ++j)
            out[(size_t)i * n + j] = scores[(size_t)i * n + j] * sc + (j <= i ? 0.0f : -INFINITY);
    return 0;
}

ORACLE_EXPORT int oracle_version(void) { return 1; }
