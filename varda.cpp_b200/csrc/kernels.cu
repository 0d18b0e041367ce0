// Elementwise, LayerNorm and output kernels (see kernels.cuh).
#include <algorithm>
#include <string>

#include "common.h"
#include "dev.cuh"
#include "kernels.cuh"

namespace vb::k {

using namespace vb::d;

namespace {

unsigned grid_for(int64_t n, int per_block) {
    int64_t b = (n + per_block - 1) / per_block;
    // grid-stride loops cover the rest; 148 SMs x 16 resident blocks x 64 waves is plenty
    return unsigned(std::max<int64_t>(1, std::min<int64_t>(b, 148 * 16 * 64)));
}

// Element-wise kernels index with I: 32-bit where the launch's elements fit (the integer division of the
// row / column split is several times cheaper than in 64 bits), else 64-bit.
template <class I>
__global__ void normalise_kernel(const float* __restrict__ x, const float* __restrict__ mul,
                                 const float* __restrict__ add, float* __restrict__ xn, I n, int V) {
    for (I i = I(blockIdx.x) * I(blockDim.x) + I(threadIdx.x); i < n; i += I(gridDim.x) * I(blockDim.x)) {
        const int v = int(i % I(V));
        xn[i] = __fadd_rn(__fmul_rn(x[i], __ldg(mul + v)), __ldg(add + v));
    }
}

template <class I>
__global__ void denormalise_kernel(const float* __restrict__ yn, const float* __restrict__ add,
                                   const float* __restrict__ mul, float* __restrict__ y, I n, int V) {
    for (I i = I(blockIdx.x) * I(blockDim.x) + I(threadIdx.x); i < n; i += I(gridDim.x) * I(blockDim.x)) {
        const int v = int(i % I(V));
        y[i] = __fdiv_rn(__fsub_rn(yn[i], __ldg(add + v)), __ldg(mul + v));
    }
}

template <class T, class I>
__global__ void assemble_kernel(const float* __restrict__ xn, const float* __restrict__ attr, int T_in, int64_t G,
                                int V, int A, T* __restrict__ out, int64_t ld, int64_t slot_rows) {
    const I n = I(G * ld), ldi = I(ld);
    const int TV = T_in * V;
    for (I i = I(blockIdx.x) * I(blockDim.x) + I(threadIdx.x); i < n; i += I(gridDim.x) * I(blockDim.x)) {
        const int64_t g = int64_t(i / ldi);
        const int f = int(i - I(g) * ldi);
        float val = 0.0f;
        if (f < TV) {
            const int t = f / V, v = f - t * V;
            val = xn[(int64_t(t) * slot_rows + g) * V + v];
        } else if (f < TV + A) {
            val = attr[g * A + (f - TV)];
        }
        out[i] = from_f<T>(val);
    }
}

// The same, eight consecutive features of a row per thread and one 16-byte (fp16) or two (fp32) stores:
// for rows of ld a multiple of 8 with a 16-byte aligned base.
template <class T>
__global__ void assemble8_kernel(const float* __restrict__ xn, const float* __restrict__ attr, int T_in, int64_t G,
                                 int V, int A, T* __restrict__ out, int ld, int64_t slot_rows) {
    const int64_t n = G * (ld / 8);
    const int TV = T_in * V, l8 = ld / 8;
    for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x) {
        const int64_t g = i / l8;
        const int f0 = 8 * int(i - g * l8);
        float val[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const int f = f0 + k;
            float x = 0.0f;
            if (f < TV) {
                const int t = f / V, v = f - t * V;
                x = xn[(int64_t(t) * slot_rows + g) * V + v];
            } else if (f < TV + A) {
                x = attr[g * A + (f - TV)];
            }
            val[k] = x;
        }
        Vec<T, 8>::store(out + g * ld + f0, val);
    }
}

__global__ void rollout_update_kernel(float* __restrict__ w, int T, int64_t rows, int V, int64_t slot,
                                      const float* __restrict__ yo, const float* __restrict__ yh, int64_t n_own, int Vo,
                                      const float* __restrict__ f, int F, const int8_t* __restrict__ kind,
                                      const int* __restrict__ src) {
    const int64_t n = rows * V;
    for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x) {
        const int64_t row = i / V;
        const int c = int(i - row * V);
        const float oldest = w[i];
        for (int t = 0; t + 1 < T; ++t) w[t * slot + i] = w[(t + 1) * slot + i];
        float* newest = w + int64_t(T - 1) * slot + i;
        const int k = kind[c];
        if (k == 1) *newest = row < n_own ? yo[row * Vo + src[c]] : yh[(row - n_own) * Vo + src[c]];
        else if (k == 2) *newest = f[row * F + src[c]];
        else if (k == 3) *newest = oldest;
    }
}

__global__ void gather_slots_kernel(float* __restrict__ dst, const float* __restrict__ src, int T, int64_t slot,
                                    const int32_t* __restrict__ idx, int64_t n, int V) {
    const int64_t tot = n * T * V;
    for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < tot; i += int64_t(gridDim.x) * blockDim.x) {
        const int64_t r = i / (int64_t(T) * V);
        const int64_t rem = i - r * T * V;
        const int t = int(rem / V), c = int(rem - int64_t(t) * V);
        dst[i] = src[t * slot + int64_t(idx[r]) * V + c];
    }
}

__global__ void scatter_slots_kernel(float* __restrict__ dst, int T, int64_t slot, int64_t row0,
                                     const float* __restrict__ src, int64_t n, int V) {
    const int64_t tot = n * T * V;
    for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < tot; i += int64_t(gridDim.x) * blockDim.x) {
        const int64_t r = i / (int64_t(T) * V);
        const int64_t rem = i - r * T * V;
        const int t = int(rem / V), c = int(rem - int64_t(t) * V);
        dst[t * slot + (row0 + r) * V + c] = src[i];
    }
}

// One warp per row, 16-byte vectors.
__global__ void copy_rows_kernel(uint4* dst, int64_t ldd, const int32_t* __restrict__ di, const uint4* __restrict__ src,
                                 int64_t lds, const int32_t* __restrict__ si, int64_t rows, int64_t vecs) {
    const int64_t r = int64_t(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (r >= rows) return;
    const int lane = threadIdx.x & 31;
    const int64_t dr = di ? di[r] : r, sr = si ? si[r] : r;
    for (int64_t v = lane; v < vecs; v += 32) dst[dr * ldd + v] = src[sr * lds + v];
}

template <class Tin, class Tout>
__global__ void convert_kernel(const Tin* __restrict__ src, int64_t lds, Tout* __restrict__ dst, int64_t ldd,
                               int64_t rows, int64_t cols) {
    const int64_t n = rows * cols;
    for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x) {
        const int64_t r = i / cols, c = i - r * cols;
        dst[r * ldd + c] = from_f<Tout>(to_f<Tin>(src[r * lds + c]));
    }
}

// One warp per row; lane holds vectors of 4 channels at (lane + 32 i) * 4, i < NV (C = 128 NV).
// Two-pass fp32 statistics in registers, as torch's CUDA LayerNorm keeps fp32 statistics.
template <int NV>
__device__ __forceinline__ void ln_apply(float (&x)[NV][4], const float* __restrict__ w, const float* __restrict__ b,
                                         int lane, float eps) {
    constexpr int C = 128 * NV;
    float s = 0.0f;
#pragma unroll
    for (int i = 0; i < NV; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) s += x[i][j];
    const float mean = warp_sum(s) / float(C);
    float q = 0.0f;
#pragma unroll
    for (int i = 0; i < NV; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float dlt = x[i][j] - mean;
            q += dlt * dlt;
        }
    const float var = warp_sum(q) / float(C);
    const float rstd = 1.0f / sqrtf(var + eps);
#pragma unroll
    for (int i = 0; i < NV; ++i) {
        const int c0 = (lane + 32 * i) * 4;
        float wv[4], bv[4] = {0.f, 0.f, 0.f, 0.f};
        Vec<float, 4>::ldg(w + c0, wv);
        if (b) Vec<float, 4>::ldg(b + c0, bv);
#pragma unroll
        for (int j = 0; j < 4; ++j) x[i][j] = (x[i][j] - mean) * rstd * wv[j] + bv[j];
    }
}

template <class T, int NV>
__global__ void __launch_bounds__(256) layernorm_kernel(const T* x, int64_t ldx, const float* __restrict__ w,
                                                        const float* __restrict__ b, T* y, int64_t ldy, int64_t rows,
                                                        float eps) {
    const int lane = threadIdx.x & 31;
    const int64_t r = int64_t(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (r >= rows) return;
    float v[NV][4];
#pragma unroll
    for (int i = 0; i < NV; ++i) Vec<T, 4>::load(x + r * ldx + (lane + 32 * i) * 4, v[i]);
    ln_apply<NV>(v, w, b, lane, eps);
#pragma unroll
    for (int i = 0; i < NV; ++i) Vec<T, 4>::store(y + r * ldy + (lane + 32 * i) * 4, v[i]);
}

template <class T, int NV>
__global__ void __launch_bounds__(256) add_layernorm_kernel(const T* a, const T* r1, T* out1,
                                                            const float* __restrict__ w, const float* __restrict__ b,
                                                            T* ln, int64_t ld, int64_t rows, float eps) {
    const int lane = threadIdx.x & 31;
    const int64_t r = int64_t(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (r >= rows) return;
    float v[NV][4];
#pragma unroll
    for (int i = 0; i < NV; ++i) {
        const int64_t off = r * ld + (lane + 32 * i) * 4;
        float p[4], q[4];
        Vec<T, 4>::load(a + off, p);
        Vec<T, 4>::load(r1 + off, q);
#pragma unroll
        for (int j = 0; j < 4; ++j) v[i][j] = rnd<T>(p[j] + q[j]);
        Vec<T, 4>::store(out1 + off, v[i]);
    }
    ln_apply<NV>(v, w, b, lane, eps);
#pragma unroll
    for (int i = 0; i < NV; ++i) Vec<T, 4>::store(ln + r * ld + (lane + 32 * i) * 4, v[i]);
}

// One warp per output row n of W: b'[n] += sum_k be[k] W[n, k] (fp32, the original weights), then
// W[n, k] = T(W[n, k] g[k]) in place and colsum[n] = sum of the rounded values.
__global__ void __launch_bounds__(256) fold_ln_kernel(__half* W, int64_t ldw, int64_t N, int K, const float* __restrict__ g,
                                                      const float* __restrict__ be, __half* b, float* colsum) {
    const int lane = threadIdx.x & 31;
    const int64_t n = int64_t(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (n >= N) return;
    __half* w = W + n * ldw;
    float c = 0.0f, sw = 0.0f;
    for (int k = lane; k < K; k += 32) {
        const float wv = __half2float(w[k]);
        if (be) c = __fmaf_rn(be[k], wv, c);
        const __half wg = __float2half_rn(__fmul_rn(wv, g[k]));
        w[k] = wg;
        sw = __fadd_rn(sw, __half2float(wg));
    }
    c = warp_sum(c);
    sw = warp_sum(sw);
    if (lane == 0) {
        colsum[n] = sw;
        b[n] = __float2half_rn(__fadd_rn(__half2float(b[n]), c));
    }
}

// One thread per (row, segment), the segment's columns in the order the GEMM epilogue takes them.
__global__ void __launch_bounds__(256) row_seg_stats_kernel(const __half* x, int64_t ldx, int64_t rows, int nseg,
                                                            int segw, float2* st) {
    const int64_t t = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (t >= rows * nseg) return;
    const int64_t r = t / nseg;
    const int sg = int(t - r * nseg);
    const __half* p = x + r * ldx + int64_t(sg) * segw;
    const float k0 = __half2float(p[0]);
    float2 s1 = make_float2(0.0f, 0.0f), s2 = make_float2(0.0f, 0.0f);
    for (int j = 0; j < segw; j += 8) {
        const uint4 u = *reinterpret_cast<const uint4*>(p + j);
        const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
        for (int q = 0; q < 4; ++q) seg_add(s1, s2, k0, __half22float2(h[q]));
    }
    st[t] = seg_record(s1, s2, k0, float(segw));
}

// One warp per R consecutive output rows (step t, data nodes g0 .. g0 + R - 1), staged in shared
// memory: the R rows' loads of each column stripe are issued together; the boundings then run in config
// order with the lanes spread over each bounding's index list, row by row. Every element sees the same
// operations in the same order whatever R is.
template <class T, int R>
__global__ void __launch_bounds__(256) output_kernel(OutputArgs a) {
    extern __shared__ float sm[];
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    const int64_t g0 = (int64_t(blockIdx.x) * (blockDim.x >> 5) + wid) * R;
    if (g0 >= a.G) return;
    const int nr = int(a.G - g0 < R ? a.G - g0 : R);
    const int t = blockIdx.y, V = a.V_out;
    float* rows = sm + wid * R * V;
    const T* dec = static_cast<const T*>(a.dec) + g0 * a.ld_dec + int64_t(t) * V;
    const int64_t orow0 = int64_t(t) * (a.y_slot > 0 ? a.y_slot : a.G) + g0;
    for (int v = lane; v < V; v += 32) {
        const int rs = a.res_src[v];
        float val[R];
#pragma unroll
        for (int r = 0; r < R; ++r)
            if (r < nr) {
                val[r] = to_f<T>(dec[r * a.ld_dec + v]);
                if (rs >= 0) val[r] = __fadd_rn(val[r], a.xn_step[(g0 + r) * a.V_in + rs]);
            }
#pragma unroll
        for (int r = 0; r < R; ++r)
            if (r < nr) {
                rows[r * V + v] = val[r];
                if (a.pre_bound) a.pre_bound[(orow0 + r) * V + v] = val[r];
            }
    }
    __syncwarp();
    for (int bi = 0; bi < a.n_bounds; ++bi) {
        const BoundDev bd = a.bounds[bi];
        const int* idx = a.bidx + bd.idx_off;
        for (int j = lane; j < bd.n; j += 32) {
            const int iv = idx[j];
#pragma unroll
            for (int r = 0; r < R; ++r)
                if (r < nr) {
                    const float x = rows[r * V + iv];
                    if (bd.type == 0) {
                        rows[r * V + iv] = (x > 0.0f || x != x) ? x : 0.0f;  // relu, NaN propagates
                    } else {
                        // std::min(std::max(x, lo), hi) of the CPU reference, NaN propagating
                        const float m = (x < bd.lo) ? bd.lo : x;
                        rows[r * V + iv] = (bd.hi < m) ? bd.hi : m;
                    }
                }
        }
        __syncwarp();
        if (bd.type == 2) {
            // y[idx] *= y[total] (already bounded); index and total lists are disjoint (checked at load)
            const int* tot = a.bidx + bd.tot_off;
            for (int j = lane; j < bd.n; j += 32) {
                const int iv = idx[j], it = tot[bd.n_tot == 1 ? 0 : j];
#pragma unroll
                for (int r = 0; r < R; ++r)
                    if (r < nr) rows[r * V + iv] = __fmul_rn(rows[r * V + iv], rows[r * V + it]);
            }
            __syncwarp();
        }
    }
#pragma unroll
    for (int r = 0; r < R; ++r)
        if (r < nr) {
            float* y = a.y + (orow0 + r) * V;
            for (int v = lane; v < V; v += 32) y[v] = rows[r * V + v];
        }
}

[[noreturn]] void bad_c(int C, const char* what) {
    fail(kUnsupported, std::string(what) + ": num_channels " + std::to_string(C) +
                           " not supported (a multiple of 128 up to 2048)");
}

}  // namespace

// elements per launch that 32-bit indices cover (a grid-stride step stays below 2^31 too)
constexpr int64_t kIdx32 = (int64_t(1) << 31) - int64_t(148) * 16 * 64 * 256;

void normalise(const float* x, const float* mul, const float* add, float* xn, int64_t n, int V, cudaStream_t s) {
    if (n <= 0) return;
    if (n < kIdx32) normalise_kernel<int32_t><<<grid_for(n, 256), 256, 0, s>>>(x, mul, add, xn, int32_t(n), V);
    else normalise_kernel<int64_t><<<grid_for(n, 256), 256, 0, s>>>(x, mul, add, xn, n, V);
    VB_LAUNCH();
}

void denormalise(const float* yn, const float* add, const float* mul, float* y, int64_t n, int V, cudaStream_t s) {
    if (n <= 0) return;
    if (n < kIdx32) denormalise_kernel<int32_t><<<grid_for(n, 256), 256, 0, s>>>(yn, add, mul, y, int32_t(n), V);
    else denormalise_kernel<int64_t><<<grid_for(n, 256), 256, 0, s>>>(yn, add, mul, y, n, V);
    VB_LAUNCH();
}

template <class T>
void assemble(const float* xn, const float* attr, int T_in, int64_t G, int V, int A, T* out, int64_t ld,
              cudaStream_t s, int64_t slot_rows) {
    if (G <= 0) return;
    if (ld % 8 == 0 && ld < (int64_t(1) << 30) && (reinterpret_cast<uintptr_t>(out) & 15) == 0) {
        assemble8_kernel<T><<<grid_for(G * (ld / 8), 256), 256, 0, s>>>(xn, attr, T_in, G, V, A, out, int(ld),
                                                                       slot_rows > 0 ? slot_rows : G);
    } else if (G * ld < kIdx32)
        assemble_kernel<T, int32_t><<<grid_for(G * ld, 256), 256, 0, s>>>(xn, attr, T_in, G, V, A, out, ld,
                                                                         slot_rows > 0 ? slot_rows : G);
    else
        assemble_kernel<T, int64_t><<<grid_for(G * ld, 256), 256, 0, s>>>(xn, attr, T_in, G, V, A, out, ld,
                                                                         slot_rows > 0 ? slot_rows : G);
    VB_LAUNCH();
}

__global__ void gather_rows_kernel(float* __restrict__ dst, const float* __restrict__ src, const int32_t* __restrict__ idx,
                                   int64_t rows, int cols) {
    const int64_t n = rows * cols;
    for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x) {
        const int64_t r = i / cols;
        dst[i] = src[int64_t(idx[r]) * cols + (i - r * cols)];
    }
}

void gather_rows(float* dst, const float* src, const int32_t* idx, int64_t rows, int cols, cudaStream_t s) {
    if (rows <= 0 || cols <= 0) return;
    gather_rows_kernel<<<grid_for(rows * cols, 256), 256, 0, s>>>(dst, src, idx, rows, cols);
    VB_LAUNCH();
}

void rollout_update(float* window, int T, int64_t rows, int V_in, const float* y_own, const float* y_halo,
                    int64_t n_own, int V_out, const float* f, int F, const int8_t* kind, const int* src, cudaStream_t s,
                    int64_t slot_stride) {
    if (rows <= 0) return;
    const int64_t slot = slot_stride > 0 ? slot_stride : rows * V_in;
    rollout_update_kernel<<<grid_for(rows * V_in, 256), 256, 0, s>>>(window, T, rows, V_in, slot, y_own, y_halo, n_own,
                                                                     V_out, f, F, kind, src);
    VB_LAUNCH();
}

void gather_slots(float* dst, const float* src, int T, int64_t slot, const int32_t* idx, int64_t n, int V,
                  cudaStream_t s) {
    if (n <= 0) return;
    gather_slots_kernel<<<grid_for(n * T * V, 256), 256, 0, s>>>(dst, src, T, slot, idx, n, V);
    VB_LAUNCH();
}

void scatter_slots(float* dst, int T, int64_t slot, int64_t row0, const float* src, int64_t n, int V, cudaStream_t s) {
    if (n <= 0) return;
    scatter_slots_kernel<<<grid_for(n * T * V, 256), 256, 0, s>>>(dst, T, slot, row0, src, n, V);
    VB_LAUNCH();
}

template <class T>
void copy_rows(T* dst, int64_t ldd, const int32_t* di, const T* src, int64_t lds, const int32_t* si, int64_t rows,
               int64_t cols, cudaStream_t s) {
    if (rows <= 0 || cols <= 0) return;
    constexpr int64_t per = 16 / sizeof(T);
    if (cols % per || ldd % per || lds % per || (reinterpret_cast<uintptr_t>(dst) & 15) ||
        (reinterpret_cast<uintptr_t>(src) & 15))
        fail(kInvalidArgument, "copy_rows: rows must be 16-byte vectors");
    copy_rows_kernel<<<unsigned((rows + 7) / 8), 256, 0, s>>>(reinterpret_cast<uint4*>(dst), ldd / per, di,
                                                             reinterpret_cast<const uint4*>(src), lds / per, si, rows,
                                                             cols / per);
    VB_LAUNCH();
}
template void copy_rows<float>(float*, int64_t, const int32_t*, const float*, int64_t, const int32_t*, int64_t, int64_t,
                               cudaStream_t);
template void copy_rows<__half>(__half*, int64_t, const int32_t*, const __half*, int64_t, const int32_t*, int64_t,
                                int64_t, cudaStream_t);

template <class Tin, class Tout>
void convert_2d(const Tin* src, int64_t lds, Tout* dst, int64_t ldd, int64_t rows, int64_t cols, cudaStream_t s) {
    if (rows <= 0 || cols <= 0) return;
    convert_kernel<Tin, Tout><<<grid_for(rows * cols, 256), 256, 0, s>>>(src, lds, dst, ldd, rows, cols);
    VB_LAUNCH();
}

#define VB_NV_SWITCH(C, MACRO, what)                          \
    switch ((C) / 128) {                                      \
        case 1: MACRO(1); break;                              \
        case 2: MACRO(2); break;                              \
        case 3: MACRO(3); break;                              \
        case 4: MACRO(4); break;                              \
        case 5: MACRO(5); break;                              \
        case 6: MACRO(6); break;                              \
        case 7: MACRO(7); break;                              \
        case 8: MACRO(8); break;                              \
        case 10: MACRO(10); break;                            \
        case 12: MACRO(12); break;                            \
        case 14: MACRO(14); break;                            \
        case 16: MACRO(16); break;                            \
        default: bad_c(C, what);                              \
    }

template <class T>
void layernorm(const T* x, int64_t ldx, const float* w, const float* b, T* y, int64_t ldy, int64_t rows, int C,
               float eps, cudaStream_t s) {
    if (rows <= 0) return;
    if (C % 128) bad_c(C, "layernorm");
    const unsigned grid = unsigned((rows + 7) / 8);
#define VB_LN(NV) layernorm_kernel<T, NV><<<grid, 256, 0, s>>>(x, ldx, w, b, y, ldy, rows, eps)
    VB_NV_SWITCH(C, VB_LN, "layernorm")
#undef VB_LN
    VB_LAUNCH();
}

template <class T>
void add_layernorm(const T* a, const T* r, T* out1, const float* w, const float* b, T* ln, int64_t ld, int64_t rows,
                   int C, float eps, cudaStream_t s) {
    if (rows <= 0) return;
    if (C % 128) bad_c(C, "add_layernorm");
    const unsigned grid = unsigned((rows + 7) / 8);
#define VB_ALN(NV) add_layernorm_kernel<T, NV><<<grid, 256, 0, s>>>(a, r, out1, w, b, ln, ld, rows, eps)
    VB_NV_SWITCH(C, VB_ALN, "add_layernorm")
#undef VB_ALN
    VB_LAUNCH();
}

void fold_layernorm(__half* W, int64_t ldw, int64_t N, int K, const float* g, const float* be, __half* b,
                    float* colsum, cudaStream_t s) {
    if (N <= 0) return;
    fold_ln_kernel<<<unsigned((N + 7) / 8), 256, 0, s>>>(W, ldw, N, K, g, be, b, colsum);
    VB_LAUNCH();
}

void row_seg_stats(const __half* x, int64_t ldx, int64_t rows, int C, int segw, float2* st, cudaStream_t s) {
    if (rows <= 0) return;
    if (segw < 8 || segw % 8 || C % segw || ldx % 8 || (reinterpret_cast<uintptr_t>(x) & 15))
        fail(kInvalidArgument, "row_seg_stats: segments must be whole 16-byte runs");
    const int nseg = C / segw;
    row_seg_stats_kernel<<<unsigned((rows * nseg + 255) / 256), 256, 0, s>>>(x, ldx, rows, nseg, segw, st);
    VB_LAUNCH();
}

template <class T>
void output_assemble(const OutputArgs& a, cudaStream_t s) {
    if (a.G <= 0 || a.T_out <= 0) return;
    if (a.T_out > 65535) fail(kUnsupported, "output_assemble: T_out > 65535");
    // four rows per warp while their staging fits the default 48 KB of shared memory, else one
    const size_t smem4 = size_t(8) * 4 * a.V_out * sizeof(float), smem1 = size_t(8) * a.V_out * sizeof(float);
    if (smem1 > 48 * 1024) fail(kUnsupported, "output_assemble: too many output variables");
    if (smem4 <= 48 * 1024)
        output_kernel<T, 4><<<dim3(unsigned((a.G + 31) / 32), unsigned(a.T_out)), 256, smem4, s>>>(a);
    else
        output_kernel<T, 1><<<dim3(unsigned((a.G + 7) / 8), unsigned(a.T_out)), 256, smem1, s>>>(a);
    VB_LAUNCH();
}

template void assemble<float>(const float*, const float*, int, int64_t, int, int, float*, int64_t, cudaStream_t, int64_t);
template void assemble<__half>(const float*, const float*, int, int64_t, int, int, __half*, int64_t, cudaStream_t, int64_t);
template void convert_2d<float, float>(const float*, int64_t, float*, int64_t, int64_t, int64_t, cudaStream_t);
template void convert_2d<float, __half>(const float*, int64_t, __half*, int64_t, int64_t, int64_t, cudaStream_t);
template void convert_2d<__half, float>(const __half*, int64_t, float*, int64_t, int64_t, int64_t, cudaStream_t);
template void layernorm<float>(const float*, int64_t, const float*, const float*, float*, int64_t, int64_t, int, float,
                               cudaStream_t);
template void layernorm<__half>(const __half*, int64_t, const float*, const float*, __half*, int64_t, int64_t, int,
                                float, cudaStream_t);
template void add_layernorm<float>(const float*, const float*, float*, const float*, const float*, float*, int64_t,
                                   int64_t, int, float, cudaStream_t);
template void add_layernorm<__half>(const __half*, const __half*, __half*, const float*, const float*, __half*,
                                    int64_t, int64_t, int, float, cudaStream_t);
template void output_assemble<float>(const OutputArgs&, cudaStream_t);
template void output_assemble<__half>(const OutputArgs&, cudaStream_t);

}  // namespace vb::k
