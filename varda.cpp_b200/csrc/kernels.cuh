// sm_100a kernels of libvarda_b200. Every launcher only enqueues on `s`: no allocation, no host
// synchronisation, so callers may capture them in a CUDA graph. Element type T of activations is
// float (fp32 mode) or __half (fp16 mode, the reference's autocast numerics). Row-major matrices
// take a leading dimension in elements.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "graph.h"

namespace vb::k {

// ------------------------------------------------------------------ input / output
// xn[i] = (x[i] * mul[v]) + add[v] with two separately rounded fp32 ops, v = i % V
// (reference cuda/kernels.h:16-19, CPU backend_cpu.cpp:470-477).
void normalise(const float* x, const float* mul, const float* add, float* xn, int64_t n, int V, cudaStream_t s);
// y[i] = (yn[i] - add[v]) / mul[v], IEEE subtraction and division.
void denormalise(const float* yn, const float* add, const float* mul, float* y, int64_t n, int V, cudaStream_t s);
// out[g, t V + v] = xn[t, g, v]; out[g, T V + a] = attr[g, a]; out[g, F..ld) = 0 for g < G, the input
// slots slot_rows rows apart (0: G; a row range of a larger input passes its full row count).
template <class T>
void assemble(const float* xn, const float* attr, int T_in, int64_t G, int V, int A, T* out, int64_t ld,
              cudaStream_t s, int64_t slot_rows = 0);
// dst[di(r), 0:cols] = src[si(r), 0:cols] for r < rows, di / si the index arrays or the identity
// when null; cols * sizeof(T) and both strides multiples of 16 bytes. Halo pack / unpack.
template <class T>
void copy_rows(T* dst, int64_t ldd, const int32_t* dst_idx, const T* src, int64_t lds, const int32_t* src_idx,
               int64_t rows, int64_t cols, cudaStream_t s);
// dst[r, 0:cols] = src[idx[r], 0:cols], fp32, any row width (rollout output exchange).
void gather_rows(float* dst, const float* src, const int32_t* idx, int64_t rows, int cols, cudaStream_t s);
// dst[r, c] = Tout(src[r, c]) for c < cols.
template <class Tin, class Tout>
void convert_2d(const Tin* src, int64_t ld_src, Tout* dst, int64_t ld_dst, int64_t rows, int64_t cols, cudaStream_t s);

struct BoundDev {
    int type = 0;  // 0 relu, 1 hardtanh, 2 fraction
    int n = 0, idx_off = 0, tot_off = 0, n_tot = 0;
    float lo = 0, hi = 0;
};
struct OutputArgs {
    const void* dec = nullptr;  // [G, ld_dec] T: decoder output, step t in columns [t V_out, (t+1) V_out)
    int64_t ld_dec = 0;
    const float* xn_step = nullptr;  // [G, V_in] normalised input of the residual step
    int V_in = 0, V_out = 0, T_out = 1;
    int64_t G = 0;
    const int* res_src = nullptr;  // [V_out]: input index added to output v, or -1
    const BoundDev* bounds = nullptr;
    int n_bounds = 0;
    const int* bidx = nullptr;
    float* pre_bound = nullptr;  // optional [T_out, G, V_out]
    float* y = nullptr;          // [T_out, G, V_out]
    int64_t y_slot = 0;          // rows between the output steps of y / pre_bound (0: G)
};
// Per output step: fp32 cast, prognostic residual, boundings in config order (reference
// backend_cpu.cpp:504-522, 111-136).
template <class T> void output_assemble(const OutputArgs& a, cudaStream_t s);

// Rollout state update of the reference (varda::StateUpdate::apply, rollout.cpp:70-92), on the
// window (T, rows, V_in) in place: every slot shifts down by one (slot t <- slot t+1), then the
// newest slot's channel c takes kind[c] = 1: the output y[row][src[c]] (prognostic), 2: the forcing
// f[row][src[c]] (dynamic forcing), 0: nothing (constant, kept in place), or 3: the oldest slot's
// old value (constant, inherited through the roll). y rows [0, n_own) come from y_own, rows
// [n_own, rows) from y_halo (the owners' outputs of this rank's halo rows, multi-GPU). Pure copies.
// slot_stride: elements between consecutive slots of the window (0: rows * V_in, a packed window).
void rollout_update(float* window, int T, int64_t rows, int V_in, const float* y_own, const float* y_halo,
                    int64_t n_own, int V_out, const float* f, int F, const int8_t* kind, const int* src, cudaStream_t s,
                    int64_t slot_stride = 0);
// Multi-slot rows (T slots of a (T, rows, V) window, `slot` elements apart): dst[i, t, :] =
// src[t slot + idx[i] V, +V) (pack), and dst[t slot + (row0 + i) V, +V) = src[i, t, :] (unpack).
void gather_slots(float* dst, const float* src, int T, int64_t slot, const int32_t* idx, int64_t n, int V,
                  cudaStream_t s);
void scatter_slots(float* dst, int T, int64_t slot, int64_t row0, const float* src, int64_t n, int V, cudaStream_t s);

// ------------------------------------------------------------------ LayerNorm (fp32 statistics)
// y = LN(x) * w + b over C channels per row (C a multiple of 128, <= 2048); b may be null; y may
// alias x. Output rounded to T once.
template <class T>
void layernorm(const T* x, int64_t ldx, const float* w, const float* b, T* y, int64_t ldy, int64_t rows, int C,
               float eps, cudaStream_t s);
// out1 = T(a + r) (rounded to T), then ln = LN(out1).
template <class T>
void add_layernorm(const T* a, const T* r, T* out1, const float* w, const float* b, T* ln, int64_t ld, int64_t rows,
                   int C, float eps, cudaStream_t s);
// LayerNorm folded into the next Linear (fp16 tensor-core path). For y = LN(x) W^T + b with LN's
// weight g and bias be: W'[n, k] = T(W[n, k] g[k]), colsum[n] = sum_k W'[n, k] (fp32),
// b'[n] = T(b[n] + sum_k be[k] W[n, k]); then y = rstd (x W'^T) - rstd mean colsum + b', rstd and mean
// of each x row coming from its segment records (dev.cuh). In place on W (ldw) and b (N, allocated);
// one warp per output row, fixed reduction order.
void fold_layernorm(__half* W, int64_t ldw, int64_t N, int K, const float* g, const float* be, __half* b,
                    float* colsum, cudaStream_t s);
// The segment records of rows [0, rows) of x (C columns, segments of segw; C a multiple of segw): the
// same values as the producing GEMM epilogue's (for rows that no GEMM produced: the processor block
// entry point, rows moved between ranks). st: [rows, C / segw] float2.
void row_seg_stats(const __half* x, int64_t ldx, int64_t rows, int C, int segw, float2* st, cudaStream_t s);

// ------------------------------------------------------------------ graph attention
template <class T> struct AttnArgs {
    const int32_t* row_ptr = nullptr;  // [n_dst + 1] of the whole graph
    const EdgeRec* edges = nullptr;    // [n_edges] CSR order
    int64_t dst_lo = 0, n_rows = 0;    // destinations [dst_lo, dst_lo + n_rows); q, xr, out rows are local
    const T* q = nullptr;
    int64_t ldq = 0;
    const T* k = nullptr;  // rows = source ids
    const T* v = nullptr;
    int64_t ldkv = 0;
    const T* xr = nullptr;
    int64_t ldxr = 0;
    T* out = nullptr;
    int64_t ldo = 0;
    const float* w_e = nullptr;  // [4, C]: edge Linear weight columns (zero padded to 3), then its bias
    int C = 0, heads = 0, head_dim = 0;
    // optional: the destinations as a list of graph rows (n_rows of them, each in
    // [dst_lo, dst_lo + rows of q/out)) instead of the range [dst_lo, dst_lo + n_rows)
    const int32_t* rows = nullptr;
};
// out[i] = T(T(att_i) + xr[i]); att_i = sum_j softmax_j(<q_i, k_j + e_ij> / sqrt(d)) (v_j + e_ij) per
// head with e_ij = W_e a_ij + b_e folded in; fp32 online softmax; zero in-degree -> att = 0.
// Semantics of the reference's cpu::graph_attention (cpu/kernels.cpp:98-158) plus the `+ x_r` of
// backend_cpu.cpp:333-340 and the fp16 roundings of the autocast reference.
template <class T> void attention(const AttnArgs<T>& a, cudaStream_t s);

// The same contract over a destination range [dst_lo, dst_lo + n_rows) (no row list), each row's edges
// cut into `splits` parts whose partial softmax results go to a static device scratch array and are
// then merged; allocates nothing (attention_split.cu). Calls must not overlap on the device: they share
// the one scratch array. Rows are processed in batches that fit it.
template <class T> void attention_split_noalloc(const AttnArgs<T>& a, int splits, cudaStream_t s);
size_t attention_split_scratch_bytes();

// The same contract for rows whose edges are cut into explicit parts (the engine's wide rows, scratch
// owned by the caller): part i = {graph row, first edge, end edge, -}; wide row w (graph row
// wide_rows[w]) merges parts [part0[w], part0[w + 1]). Parts [part_lo, part_lo + n_parts) and wide rows
// [wide_lo, wide_lo + n_wide) run; scratch holds one record of attention_parts_record(C, heads) floats
// per part, indexed by the part's global index.
struct PartsArgs {
    const int4* parts = nullptr;
    int64_t part_lo = 0, n_parts = 0;
    const int32_t* wide_rows = nullptr;
    const int32_t* part0 = nullptr;
    int64_t wide_lo = 0, n_wide = 0;
    float* scratch = nullptr;
};
template <class T> void attention_parts(const AttnArgs<T>& a, const PartsArgs& p, cudaStream_t s);
int attention_parts_record(int C, int heads);

// Shared-memory-staged attention (fp16) over destination tiles (graph.h TilePlan): same contract per
// destination row. Tiles [tile0, tile0 + ntiles) of the plan; q/x_r/out row of graph
// row d is d - dst_lo.
struct TileArgs {
    const int4* tiles = nullptr;    // per tile {row0, nrows, src0, nsrc}
    const int32_t* srcs = nullptr;  // distinct sources per tile
    const EdgeRec* edges = nullptr;  // CSR-order records, source = slot in the tile
    const int32_t* row_ptr = nullptr;
    int64_t dst_lo = 0;
    int tile0 = 0, ntiles = 0;
    const __half *q = nullptr, *k = nullptr, *v = nullptr, *xr = nullptr;
    __half* out = nullptr;
    int64_t ldq = 0, ldkv = 0, ldxr = 0, ldo = 0;
    const float* w_e = nullptr;
    int C = 0, heads = 0, head_dim = 0;
};
void attention_tiled(const TileArgs& a, float scale_log2, cudaStream_t s);
bool tiled_supported(int C, int head_dim);
int tiled_max_src();
int tiled_max_rows();
int tiled_max_edges();
// Synchronises; reads and clears the flag a timed-out wait of the tiled attention sets.
int take_attention_error();
// Tile-sparse tensor-core edge attention (fp16, head_dim 64; attention_tc.cu) over the tiles of a
// TcPlan (graph.h make_tc_tiles): same contract per destination row as attention(). Tiles
// [tile0, tile0 + ntiles) of the plan; the q / x_r / out row of graph row d is d - dst_lo (q has
// n_q_rows rows, k and v n_src rows). The plan's heavy rows are not covered (run them on attention()).
struct TcArgs {
    const TcTile* tiles = nullptr;
    const int32_t* srcs = nullptr;
    const uint8_t* blob = nullptr;
    int tile0 = 0, ntiles = 0;
    int64_t dst_lo = 0;
    const __half *q = nullptr, *k = nullptr, *v = nullptr, *xr = nullptr;
    __half* out = nullptr;
    int64_t ldq = 0, ldkv = 0, ldxr = 0, ldo = 0;
    int64_t n_q_rows = 0, n_src = 0;
    const float* w_e = nullptr;  // [4, C], fp16-representable values
    int C = 0, heads = 0, head_dim = 0;
    // dynamic tile order: two zeroed words the launch leaves zero (one counter per stream: launches that
    // share it must not run concurrently); null: static order (tile b + i x grid for CTA b)
    unsigned* sched = nullptr;
};
void attention_tc(const TcArgs& a, cudaStream_t s);
bool tc_attention_supported(int C, int heads, int head_dim);
int take_tc_error();  // reads and clears the kernel's timeout flag (no synchronise)

// ------------------------------------------------------------------ GEMM (Linear layers)
enum Epilogue : int {
    kEpiBias = 0,      // y = T(acc + b)
    kEpiGelu = 1,      // y = T(gelu(T(acc + b)))
    kEpiResidual = 2,  // y = T(T(acc + b) + r)
};
template <class T> struct GemmArgs {
    const T* A = nullptr;  // [M, K] lda
    int64_t lda = 0;
    const T* W = nullptr;  // [N, K] ldw (nn.Linear weight)
    int64_t ldw = 0;
    const T* bias = nullptr;  // [N] or null
    T* C = nullptr;           // [M, N] ldc
    int64_t ldc = 0;
    const T* R = nullptr;  // residual [M, N] ldr (kEpiResidual)
    int64_t ldr = 0;
    int64_t M = 0, N = 0, K = 0;
    int epi = kEpiBias;
    bool gelu_tanh = false;
    // LayerNorm fusion (fp16 tensor-core path, N a multiple of the segment width stats_segw(N)):
    float2* st_out = nullptr;        // write the output rows' segment records, [M, N / stats_segw(N)]
    const float2* st_in = nullptr;   // A's rows' segment records, [M, nseg_in]: y = LN(A) W^T + b, W and b
    const float* colsum = nullptr;   //   folded by fold_layernorm (bias, GELU epilogues)
    int nseg_in = 0, segw_in = 0;
    float eps = 0.0f;
};
// CUDA-core GEMM with fp32 accumulation (true fp32 FMA in fp32 mode).
template <class T> void gemm_simt(const GemmArgs<T>& a, cudaStream_t s);

}  // namespace vb::k
