/*
 * CPU oracle for the batched fp32 matmul path of torchlite-cpp.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the product links or calls this file;
 * only tests/, the smoke check and the CPU-baseline leg of bench.py load it,
 * and only as the checker.
 *
 * It restates, in plain C, the arithmetic of the reference's CPU path:
 *
 *  - gemm_blocked (src/ops.cpp:242-268), the kernel that every x86 matmul path
 *    ends in (gemm_tiled -> src/ops.cpp:383, gemm_packed -> src/ops.cpp:564).
 *    Its loop nest zeroes C and then, for each 64-wide k-slab in ascending
 *    order, does C[m,n] += A[m,k]*B[k,n] for k ascending.  Built with the
 *    reference's Release flags (-O3 -march=native, GNU fp-contract=fast) the
 *    multiply-add contracts to one fused multiply-add, so every output element
 *    is the chain  c = 0;  for k = 0..K-1: c = fmaf(a[m,k], b[k,n], c).
 *    orc_gemm_chain computes exactly that chain.
 *
 *  - sum over one dimension (src/ops.cpp:1181-1233): acc = 0.0f; acc += x[d]
 *    for d ascending.  orc_sum_dim computes exactly that order.
 *
 *  - element-wise add (src/ops.cpp:75-103), used by accumulate_grad
 *    (src/autograd.cpp:16-22): orc_add.
 *
 *  - softmax over the last dim (src/ops.cpp:985-1037): the row maximum
 *    (first element, then strict >), e_j = expf(x_j - max) with the C
 *    library's expf (what std::exp(float) calls), a sequential sum from 0.0f,
 *    and e_j / sum: orc_softmax.
 *
 *  - SoftmaxBackward (src/autograd.cpp:228-256): dot = sum_j g_j * y_j from
 *    0.0f in j order, then dx_i = y_i * (g_i - dot): orc_softmax_backward.
 *    How the Release build rounds the dot depends on its vectorisation: GCC
 *    vectorises the loop over blocks of `vec` elements (products rounded,
 *    then added in order: dot = dot + rn(g_j * y_j)) and leaves the last
 *    D mod vec elements to scalar code that it contracts to
 *    dot = fmaf(g_j, y_j, dot).  vec = 8 for the x86-64-v4 (AVX-512) build,
 *    4 for x86-64-v3; both measured against the compiled reference.
 *
 *  - flash_attention (src/ops.cpp:1040-1137) and FlashAttentionBackward
 *    (src/autograd.cpp:575-669): 64 x 64 query / key tiles, each score
 *    T = dot(q_i, k_j) * scale, the online softmax (m_new = max(m, max_j T),
 *    corr = expf(m - m_new), p = expf(T - m_new), l = fmaf(l, corr, sum p),
 *    O = O * corr then O = fmaf(p, v_j, O) per key), O = O * (1 / l),
 *    L = m + logf(l); the backward recomputes P = expf(T - L_i) and
 *    accumulates dV, dQ, dK per (i, j) pair in the reference's order:
 *    orc_flash_attention / orc_flash_attention_backward.  Each dot over d
 *    rounds the way the Release build's vectorisation does (the first
 *    d - d mod vec products rounded and added in order, the tail fused), as
 *    for SoftmaxBackward's dot.
 *
 * Operands are strided 2-D views (row and column strides in elements), so the
 * transposed views that MatmulBackward builds (src/autograd.cpp:370-371) are
 * read in place; Tensor::contiguous (src/tensor.cpp:174-193) only copies, it
 * does not change values, so reading through strides gives the same numbers.
 *
 * orc_gemm_f64 is not part of the reference: it is a double-precision product
 * used to measure error for the tensor-core modes.
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>

typedef struct {
    const float *A, *B;
    float *C;
    double *C64;
    int64_t sam, sak, sbk, sbn, ldc;
    int64_t M, N, K;
    int64_t m0, m1;
} orc_job;

static void *chain_rows(void *p) {
    const orc_job *j = (const orc_job *)p;
    for (int64_t m = j->m0; m < j->m1; ++m) {
        for (int64_t n = 0; n < j->N; ++n) {
            float c = 0.0f;
            const float *a = j->A + m * j->sam;
            const float *b = j->B + n * j->sbn;
            for (int64_t k = 0; k < j->K; ++k) c = fmaf(a[k * j->sak], b[k * j->sbk], c);
            j->C[m * j->ldc + n] = c;
        }
    }
    return NULL;
}

static void *f64_rows(void *p) {
    const orc_job *j = (const orc_job *)p;
    for (int64_t m = j->m0; m < j->m1; ++m) {
        for (int64_t n = 0; n < j->N; ++n) {
            double c = 0.0;
            const float *a = j->A + m * j->sam;
            const float *b = j->B + n * j->sbn;
            for (int64_t k = 0; k < j->K; ++k) c += (double)a[k * j->sak] * (double)b[k * j->sbk];
            j->C64[m * j->ldc + n] = c;
        }
    }
    return NULL;
}

static void run_rows(void *(*fn)(void *), orc_job base, int nthreads) {
    if (nthreads < 1) nthreads = 1;
    if (nthreads > 256) nthreads = 256;
    if (base.M < nthreads) nthreads = (int)(base.M > 0 ? base.M : 1);
    pthread_t th[256];
    orc_job jobs[256];
    int64_t per = (base.M + nthreads - 1) / nthreads;
    int started = 0;
    for (int t = 0; t < nthreads; ++t) {
        jobs[t] = base;
        jobs[t].m0 = (int64_t)t * per;
        jobs[t].m1 = jobs[t].m0 + per < base.M ? jobs[t].m0 + per : base.M;
        if (jobs[t].m0 >= base.M) break;
        if (nthreads == 1 || pthread_create(&th[t], NULL, fn, &jobs[t]) != 0) {
            fn(&jobs[t]);
            th[t] = 0;
        }
        started = t + 1;
    }
    for (int t = 0; t < started; ++t)
        if (th[t]) pthread_join(th[t], NULL);
}

/* C[m*ldc + n] = fmaf chain over k of A[m*sam + k*sak] * B[k*sbk + n*sbn]. */
void orc_gemm_chain(const float *A, int64_t sam, int64_t sak, const float *B, int64_t sbk,
                    int64_t sbn, float *C, int64_t ldc, int64_t M, int64_t N, int64_t K,
                    int nthreads) {
    orc_job j = {A, B, C, NULL, sam, sak, sbk, sbn, ldc, M, N, K, 0, M};
    run_rows(chain_rows, j, nthreads);
}

/* Same operands, double-precision accumulation (error measurement only). */
void orc_gemm_f64(const float *A, int64_t sam, int64_t sak, const float *B, int64_t sbk,
                  int64_t sbn, double *C, int64_t ldc, int64_t M, int64_t N, int64_t K,
                  int nthreads) {
    orc_job j = {A, B, NULL, C, sam, sak, sbk, sbn, ldc, M, N, K, 0, M};
    run_rows(f64_rows, j, nthreads);
}

/* out[o*inner + n] = sum over d ascending of in[o*D*inner + d*inner + n], from 0.0f. */
void orc_sum_dim(const float *in, float *out, int64_t outer, int64_t D, int64_t inner) {
    for (int64_t o = 0; o < outer; ++o)
        for (int64_t n = 0; n < inner; ++n) {
            float acc = 0.0f;
            for (int64_t d = 0; d < D; ++d) acc += in[o * D * inner + d * inner + n];
            out[o * inner + n] = acc;
        }
}

/* out[i] = a[i] + b[i] (same shape). */
void orc_add(const float *a, const float *b, float *out, int64_t n) {
    for (int64_t i = 0; i < n; ++i) out[i] = a[i] + b[i];
}

/* softmax of each row of D floats (src/ops.cpp:985-1037). */
void orc_softmax(const float *x, float *out, int64_t rows, int64_t D) {
    for (int64_t r = 0; r < rows; ++r) {
        const float *row = x + r * D;
        float *o = out + r * D;
        float mx = row[0];
        for (int64_t j = 1; j < D; ++j)
            if (row[j] > mx) mx = row[j];
        float sum = 0.0f;
        for (int64_t j = 0; j < D; ++j) {
            o[j] = expf(row[j] - mx);
            sum += o[j];
        }
        for (int64_t j = 0; j < D; ++j) o[j] /= sum;
    }
}

/* SoftmaxBackward of each row of D floats (src/autograd.cpp:228-256); the
 * first D - D mod vec products are rounded before they are added. */
void orc_softmax_backward(const float *g, const float *y, float *dx, int64_t rows, int64_t D,
                          int64_t vec) {
    const int64_t nv = D - D % vec;
    for (int64_t r = 0; r < rows; ++r) {
        const float *gr = g + r * D, *yr = y + r * D;
        float *o = dx + r * D;
        float dot = 0.0f;
        for (int64_t j = 0; j < nv; ++j) {
            const float p = gr[j] * yr[j];
            dot = dot + p;
        }
        for (int64_t j = nv; j < D; ++j) dot = fmaf(gr[j], yr[j], dot);
        for (int64_t i = 0; i < D; ++i) o[i] = yr[i] * (gr[i] - dot);
    }
}

/* dot over d in the Release build's rounding (see the header): the first
 * d - d mod vec products rounded and added in order, the tail fused; vec <= 0
 * means a plain fused chain. */
static float vdot(const float *a, const float *b, int64_t d, int64_t vec) {
    const int64_t nv = vec > 0 ? d - d % vec : 0;
    float dot = 0.0f;
    for (int64_t c = 0; c < nv; ++c) {
        const float p = a[c] * b[c];
        dot = dot + p;
    }
    for (int64_t c = nv; c < d; ++c) dot = fmaf(a[c], b[c], dot);
    return dot;
}

/* flash_attention (src/ops.cpp:1040-1137) on one head: q, k, v, o [S, d],
 * lse [S] (the reference's L_cache). */
void orc_flash_attention(const float *q, const float *k, const float *v, int64_t S, int64_t d,
                         float scale, float *o, float *lse, int64_t vec) {
    enum { B = 64 };
    float *T = malloc(sizeof(float) * B * B);
    float *m = malloc(sizeof(float) * B), *l = malloc(sizeof(float) * B);
    float *acc = malloc(sizeof(float) * B * (d > 0 ? d : 1));
    for (int64_t i0 = 0; i0 < S; i0 += B) {
        const int64_t qr = S - i0 < B ? S - i0 : B;
        for (int64_t i = 0; i < qr; ++i) {
            m[i] = -INFINITY;
            l[i] = 0.0f;
            for (int64_t c = 0; c < d; ++c) acc[i * d + c] = 0.0f;
        }
        for (int64_t j0 = 0; j0 < S; j0 += B) {
            const int64_t kr = S - j0 < B ? S - j0 : B;
            for (int64_t i = 0; i < qr; ++i)
                for (int64_t j = 0; j < kr; ++j)
                    T[i * B + j] = vdot(q + (i0 + i) * d, k + (j0 + j) * d, d, vec) * scale;
            for (int64_t i = 0; i < qr; ++i) {
                float mb = -INFINITY;
                for (int64_t j = 0; j < kr; ++j) mb = mb < T[i * B + j] ? T[i * B + j] : mb;  /* std::max(mb, t) */
                const float mn = m[i] < mb ? mb : m[i];  /* std::max(m, mb) */
                const float corr = expf(m[i] - mn);
                float rs = 0.0f;
                for (int64_t j = 0; j < kr; ++j) {
                    const float p = expf(T[i * B + j] - mn);
                    T[i * B + j] = p;
                    rs = rs + p;
                }
                l[i] = fmaf(l[i], corr, rs);
                float *a = acc + i * d;
                for (int64_t c = 0; c < d; ++c) a[c] = a[c] * corr;
                for (int64_t j = 0; j < kr; ++j) {
                    const float p = T[i * B + j];
                    const float *vr = v + (j0 + j) * d;
                    for (int64_t c = 0; c < d; ++c) a[c] = fmaf(p, vr[c], a[c]);
                }
                m[i] = mn;
            }
        }
        for (int64_t i = 0; i < qr; ++i) {
            const float inv = 1.0f / l[i];
            for (int64_t c = 0; c < d; ++c) o[(i0 + i) * d + c] = acc[i * d + c] * inv;
            lse[i0 + i] = m[i] + logf(l[i]);
        }
    }
    free(T);
    free(m);
    free(l);
    free(acc);
}

/* FlashAttentionBackward (src/autograd.cpp:575-669) on one head; dq, dk, dv
 * are overwritten (the reference starts them from zeros). */
void orc_flash_attention_backward(const float *dout, const float *q, const float *k,
                                  const float *v, const float *o, const float *lse, int64_t S,
                                  int64_t d, float scale, float *dq, float *dk, float *dv,
                                  int64_t vec) {
    enum { B = 64 };
    float *D = malloc(sizeof(float) * (S > 0 ? S : 1));
    float *P = malloc(sizeof(float) * B * B);
    for (int64_t i = 0; i < S * d; ++i) dq[i] = dk[i] = dv[i] = 0.0f;
    for (int64_t i = 0; i < S; ++i) D[i] = vdot(dout + i * d, o + i * d, d, vec);
    for (int64_t i0 = 0; i0 < S; i0 += B) {
        const int64_t qr = S - i0 < B ? S - i0 : B;
        for (int64_t j0 = 0; j0 < S; j0 += B) {
            const int64_t kr = S - j0 < B ? S - j0 : B;
            for (int64_t i = 0; i < qr; ++i)
                for (int64_t j = 0; j < kr; ++j) {
                    const float t = vdot(q + (i0 + i) * d, k + (j0 + j) * d, d, vec) * scale;
                    P[i * B + j] = expf(t - lse[i0 + i]);
                }
            for (int64_t i = 0; i < qr; ++i) {
                const float *doi = dout + (i0 + i) * d, *qi = q + (i0 + i) * d;
                float *dqi = dq + (i0 + i) * d;
                const float Di = D[i0 + i];
                for (int64_t j = 0; j < kr; ++j) {
                    const float p = P[i * B + j];
                    const float *vr = v + (j0 + j) * d, *kr_ = k + (j0 + j) * d;
                    float *dvj = dv + (j0 + j) * d, *dkj = dk + (j0 + j) * d;
                    const float dp = vdot(doi, vr, d, vec);
                    const float ds = p * (dp - Di);
                    const float sds = scale * ds;
                    for (int64_t c = 0; c < d; ++c) dvj[c] = fmaf(p, doi[c], dvj[c]);
                    for (int64_t c = 0; c < d; ++c) dqi[c] = fmaf(sds, kr_[c], dqi[c]);
                    for (int64_t c = 0; c < d; ++c) dkj[c] = fmaf(sds, qi[c], dkj[c]);
                }
            }
        }
    }
    free(D);
    free(P);
}
