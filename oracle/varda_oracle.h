/* CPU fp32 restatement of the reference's GraphTransformer kernels (varda.cpp, src/varda/).
 *
 * TEST INFRASTRUCTURE ONLY. Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg
 * may load this library, and only as the checker. The product (libvarda_b200.so) never links or
 * calls it.
 *
 * Every function restates one reference function, cited by file:line of the reference project.
 * Pinned against the reference's own golden vectors (python/tests/synthetic.py models a-h) and
 * against the reference CPU backend compiled from its sources into oracle/_ref (tests/test_oracle.py).
 */
#ifndef VARDA_ORACLE_H
#define VARDA_ORACLE_H
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* build_csr_by_dst, src/varda/graph.cpp:17-61: stable counting sort of the stored edges by
 * destination. edge_index is [2, E] (row 0 source, row 1 destination), int64. Outputs:
 * row_ptr [n_dst + 1], src [E], edge_id [E], attr_csr [E, A]. Returns 0, or -1 (index out of
 * range, *bad_edge set) or -2 (graph too large for int32 indices). */
int vo_build_csr(const int64_t* edge_index, int64_t E, const float* edge_attr, int A, int64_t n_src,
                 int64_t n_dst, int32_t* row_ptr, int32_t* src, int32_t* edge_id, float* attr_csr,
                 int64_t* bad_edge);

/* Linear, src/varda/cpu/kernels.cpp:13-24 (linear_tile): y[r, c] = (sum_k x[r, k] w[c, k]) + b[c];
 * the sum is rounded before the bias is added (torch addmm). b may be NULL. Parallel over rows. */
void vo_linear(const float* x, int64_t ldx, int64_t M, const float* w, const float* b, int64_t n_out,
               int64_t n_in, float* y, int64_t ldy);

/* LayerNorm, src/varda/cpu/kernels.cpp:26-45: moments in double, then in fp32
 * rstd = 1/sqrt(var + eps), y = (x * rstd + (-rstd * mean)) * w (+ b). b may be NULL. */
void vo_layer_norm(const float* x, int64_t ldx, int64_t M, int64_t dim, const float* w, const float* b,
                   float eps, float* y, int64_t ldy);

/* GELU in place, src/varda/cpu/kernels.cpp:52-66: exact erf form, or the tanh form. */
void vo_gelu(float* x, int64_t n, int tanh_approx);

/* Graph attention, src/varda/cpu/kernels.cpp:98-158, for destinations [d0, d0 + nd) of a CSR
 * graph. q rows are local (ldq), k and v rows are global source ids (ldkv). edge_wt is the
 * transposed edge Linear weight [A, C], edge_b [C] or NULL. out [nd, C] (ldo): zero in-degree
 * destinations get zeros. */
void vo_graph_attention(const int32_t* row_ptr, const int32_t* src, const float* attr_csr, int A,
                        int64_t d0, int64_t nd, const float* q, int64_t ldq, const float* k,
                        const float* v, int64_t ldkv, const float* edge_wt, const float* edge_b,
                        int heads, int head_dim, float* out, int64_t ldo);

/* Threads used by the parallel loops (0 = OpenMP default). */
void vo_set_threads(int n);

#ifdef __cplusplus
}
#endif
#endif
