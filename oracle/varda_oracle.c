/* CPU fp32 restatement of the reference's GraphTransformer kernels. TEST INFRASTRUCTURE ONLY:
 * see varda_oracle.h for who may call it. Built with -ffp-contract=off so that every multiply
 * and add is rounded separately, as in the reference's CPU build. */
#include "varda_oracle.h"

#include <math.h>
#include <omp.h>
#include <stdlib.h>
#include <string.h>

void vo_set_threads(int n) {
    if (n > 0) omp_set_num_threads(n);
}

/* graph.cpp:17-61. Count in-degrees, prefix-sum, then place every stored edge at the next free
 * slot of its destination in stored order (a stable counting sort). */
int vo_build_csr(const int64_t* ei, int64_t E, const float* ea, int A, int64_t n_src, int64_t n_dst,
                 int32_t* row_ptr, int32_t* src, int32_t* edge_id, float* attr_csr, int64_t* bad_edge) {
    const int64_t lim = 2147483647LL;
    if (E >= lim || n_src >= lim || n_dst >= lim) return -2;
    memset(row_ptr, 0, sizeof(int32_t) * (size_t)(n_dst + 1));
    for (int64_t e = 0; e < E; ++e) {
        const int64_t s = ei[e], d = ei[E + e];
        if (s < 0 || s >= n_src || d < 0 || d >= n_dst) {
            if (bad_edge) *bad_edge = e;
            return -1;
        }
        ++row_ptr[d + 1];
    }
    for (int64_t d = 0; d < n_dst; ++d) row_ptr[d + 1] += row_ptr[d];
    int32_t* fill = (int32_t*)malloc(sizeof(int32_t) * (size_t)(n_dst > 0 ? n_dst : 1));
    memcpy(fill, row_ptr, sizeof(int32_t) * (size_t)n_dst);
    for (int64_t e = 0; e < E; ++e) {
        const int32_t slot = fill[ei[E + e]]++;
        src[slot] = (int32_t)ei[e];
        edge_id[slot] = (int32_t)e;
        memcpy(attr_csr + (int64_t)slot * A, ea + e * A, sizeof(float) * (size_t)A);
    }
    free(fill);
    return 0;
}

/* Dot product with eight independent partial sums combined pairwise (the order the reference's
 * dot_q_ke uses, cpu/kernels.cpp:72-80). The Linear's own summation order inside OpenBLAS is not
 * specified; this order is one valid fp32 order, and the parity tolerance (1e-5) covers the
 * difference. */
static float dot8(const float* a, const float* b, int64_t n) {
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    int64_t c = 0;
    for (; c + 8 <= n; c += 8)
        for (int l = 0; l < 8; ++l) acc[l] += a[c + l] * b[c + l];
    float s = ((acc[0] + acc[1]) + (acc[2] + acc[3])) + ((acc[4] + acc[5]) + (acc[6] + acc[7]));
    for (; c < n; ++c) s += a[c] * b[c];
    return s;
}

/* cpu/kernels.cpp:13-24 and kernels.h:54-76. */
void vo_linear(const float* x, int64_t ldx, int64_t M, const float* w, const float* b, int64_t n_out,
               int64_t n_in, float* y, int64_t ldy) {
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < M; ++r) {
        const float* xr = x + r * ldx;
        float* yr = y + r * ldy;
        for (int64_t c = 0; c < n_out; ++c) {
            const float s = dot8(xr, w + c * n_in, n_in);
            yr[c] = b ? s + b[c] : s;
        }
    }
}

/* cpu/kernels.cpp:26-45. */
void vo_layer_norm(const float* x, int64_t ldx, int64_t M, int64_t n, const float* w, const float* b,
                   float eps, float* y, int64_t ldy) {
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < M; ++r) {
        const float* xr = x + r * ldx;
        float* yr = y + r * ldy;
        double sum = 0;
        for (int64_t c = 0; c < n; ++c) sum += xr[c];
        const double mean = sum / (double)n;
        double ss = 0;
        for (int64_t c = 0; c < n; ++c) {
            const double d = xr[c] - mean;
            ss += d * d;
        }
        const float mean_f = (float)mean;
        const float var_f = (float)(ss / (double)n); /* biased */
        const float rstd = 1.0f / sqrtf(var_f + eps);
        const float shift = -rstd * mean_f;
        for (int64_t c = 0; c < n; ++c) {
            float t = xr[c] * rstd + shift;
            t = t * w[c];
            yr[c] = b ? t + b[c] : t;
        }
    }
}

/* cpu/kernels.cpp:52-59. */
static float gelu1(float x, int tanh_approx) {
    if (!tanh_approx) return x * 0.5f * (1.0f + erff(x * (float)M_SQRT1_2));
    const float beta = (float)(M_SQRT2 * M_2_SQRTPI * 0.5);
    const float kappa = 0.044715f;
    const float cube = x * x * x;
    const float inner = beta * (x + kappa * cube);
    return 0.5f * x * (1.0f + tanhf(inner));
}

void vo_gelu(float* x, int64_t n, int tanh_approx) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; ++i) x[i] = gelu1(x[i], tanh_approx);
}

/* sum_c q[c] * (k[c] + e[c]) with 8 partial sums, cpu/kernels.cpp:72-80. */
static float dot_q_ke(const float* q, const float* k, const float* e, int64_t n) {
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    int64_t c = 0;
    for (; c + 8 <= n; c += 8)
        for (int l = 0; l < 8; ++l) acc[l] += q[c + l] * (k[c + l] + e[c + l]);
    float s = ((acc[0] + acc[1]) + (acc[2] + acc[3])) + ((acc[4] + acc[5]) + (acc[6] + acc[7]));
    for (; c < n; ++c) s += q[c] * (k[c] + e[c]);
    return s;
}

/* e = attr . W^T + b for one edge (attributes first, then the bias), cpu/kernels.cpp:83-94. */
static void edge_project(const float* wt, const float* b, int A, int64_t C, const float* attr, float* e) {
    for (int64_t c = 0; c < C; ++c) e[c] = attr[0] * wt[c];
    for (int a = 1; a < A; ++a) {
        const float aa = attr[a];
        const float* w = wt + (int64_t)a * C;
        for (int64_t c = 0; c < C; ++c) e[c] += aa * w[c];
    }
    if (b)
        for (int64_t c = 0; c < C; ++c) e[c] += b[c];
}

/* cpu/kernels.cpp:98-158: e materialised per edge, score / sqrt(d) (fp32 sqrt of the head
 * dimension), two-pass softmax with +1e-16, out = sum_j (v_j + e_j) a_j in CSR order. */
void vo_graph_attention(const int32_t* row_ptr, const int32_t* src, const float* attr, int A, int64_t d0,
                        int64_t nd, const float* q, int64_t ldq, const float* k, const float* v,
                        int64_t ldkv, const float* wt, const float* eb, int heads, int head_dim,
                        float* out, int64_t ldo) {
    const int64_t ct = (int64_t)heads * head_dim;
    int32_t max_deg = 0;
    for (int64_t i = 0; i < nd; ++i) {
        const int32_t dg = row_ptr[d0 + i + 1] - row_ptr[d0 + i];
        if (dg > max_deg) max_deg = dg;
    }
    const float scale_div = (float)sqrt((double)head_dim);
    const float softmax_eps = 1e-16f;
#pragma omp parallel
    {
        float* e = (float*)malloc(sizeof(float) * (size_t)(max_deg > 0 ? max_deg : 1) * (size_t)ct);
        float* s = (float*)malloc(sizeof(float) * (size_t)(max_deg > 0 ? max_deg : 1) * (size_t)heads);
#pragma omp for schedule(dynamic, 32)
        for (int64_t i = 0; i < nd; ++i) {
            const int64_t lo = row_ptr[d0 + i];
            const int64_t deg = row_ptr[d0 + i + 1] - lo;
            float* o = out + i * ldo;
            for (int64_t c = 0; c < ct; ++c) o[c] = 0.0f;
            if (deg == 0) continue;
            const float* qi = q + i * ldq;
            for (int64_t t = 0; t < deg; ++t) edge_project(wt, eb, A, ct, attr + (lo + t) * A, e + t * ct);
            for (int64_t t = 0; t < deg; ++t) {
                const float* kj = k + (int64_t)src[lo + t] * ldkv;
                const float* et = e + t * ct;
                for (int h = 0; h < heads; ++h) {
                    const int64_t off = (int64_t)h * head_dim;
                    s[t * heads + h] = dot_q_ke(qi + off, kj + off, et + off, head_dim) / scale_div;
                }
            }
            for (int h = 0; h < heads; ++h) {
                float m = s[h];
                for (int64_t t = 1; t < deg; ++t)
                    if (s[t * heads + h] > m) m = s[t * heads + h];
                float den = 0.0f;
                for (int64_t t = 0; t < deg; ++t) {
                    const float ex = expf(s[t * heads + h] - m);
                    s[t * heads + h] = ex;
                    den += ex;
                }
                den = den + softmax_eps;
                for (int64_t t = 0; t < deg; ++t) s[t * heads + h] = s[t * heads + h] / den;
            }
            for (int64_t t = 0; t < deg; ++t) {
                const float* vj = v + (int64_t)src[lo + t] * ldkv;
                const float* et = e + t * ct;
                for (int h = 0; h < heads; ++h) {
                    const float a = s[t * heads + h];
                    const int64_t off = (int64_t)h * head_dim;
                    for (int64_t c = off; c < off + head_dim; ++c) o[c] += (vj[c] + et[c]) * a;
                }
            }
        }
        free(e);
        free(s);
    }
}
