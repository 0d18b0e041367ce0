// Graph attention over a destination-major CSR graph (see kernels.cuh for the contract).
//
// Layout: a destination's C channels are split over WPD = C / (32 CPL) warps; lane l of part p owns
// the CPL consecutive channels starting at p 32 CPL + l CPL (one 16-byte vector: 8 fp16 or 4 fp32).
// LPH = head_dim / CPL consecutive lanes share a head, so per-head dot products are a butterfly over
// LPH lanes. Each warp streams its destination's CSR row: edge records are fetched 32 at a time with
// one coalesced load (lane i holds record i) and broadcast with shuffles, and the K/V gathers of U
// edges are issued before any of them is consumed, so U x 2 x 16 bytes per lane are in flight.
//
// Numerics (the reference's semantics, cpu/kernels.cpp:98-158 and backend_cpu.cpp:333-340):
//   s_j  = (<q, k_j> + <W_e^T q, a_j> + <q, b_e>) / sqrt(d)    (edge projection folded, per head)
//   fp32 online softmax over the row: m, l, acc = sum p_j v_j, pa = sum p_j a_j
//   o    = acc / l + W_e (pa / l) + b_e                       (sum_j p_j / l = 1)
//   out  = T(T(o) + x_r);  zero in-degree: o = 0, so out = x_r exactly.
#include <cmath>
#include <string>

#include "common.h"
#include "dev.cuh"
#include "kernels.cuh"

namespace vb::k {

using namespace vb::d;

namespace {

// Raw 16-byte vectors of CPL channels, unpacked to fp32 when consumed.
template <class T, int CPL> struct Raw;
template <> struct Raw<__half, 8> {
    uint4 u;
    __device__ __forceinline__ void ldg(const __half* p) { u = __ldg(reinterpret_cast<const uint4*>(p)); }
    __device__ __forceinline__ void get(float* f) const { Vec<__half, 8>::unpack(u, f); }
};
template <> struct Raw<__half, 4> {
    uint2 u;
    __device__ __forceinline__ void ldg(const __half* p) { u = __ldg(reinterpret_cast<const uint2*>(p)); }
    __device__ __forceinline__ void get(float* f) const { Vec<__half, 4>::unpack(u, f); }
};
template <> struct Raw<float, 4> {
    float4 u;
    __device__ __forceinline__ void ldg(const float* p) { u = __ldg(reinterpret_cast<const float4*>(p)); }
    __device__ __forceinline__ void get(float* f) const { f[0] = u.x, f[1] = u.y, f[2] = u.z, f[3] = u.w; }
};
template <> struct Raw<float, 8> {
    float4 a, b;
    __device__ __forceinline__ void ldg(const float* p) {
        a = __ldg(reinterpret_cast<const float4*>(p));
        b = __ldg(reinterpret_cast<const float4*>(p) + 1);
    }
    __device__ __forceinline__ void get(float* f) const {
        f[0] = a.x, f[1] = a.y, f[2] = a.z, f[3] = a.w, f[4] = b.x, f[5] = b.y, f[6] = b.z, f[7] = b.w;
    }
};

template <int LPH>
__device__ __forceinline__ float head_sum(float x) {
#pragma unroll
    for (int o = 1; o < LPH; o <<= 1) x += __shfl_xor_sync(kFull, x, o);
    return x;
}

template <class T, int CPL, int LPH, int U>
__global__ void __launch_bounds__(256) attention_kernel(AttnArgs<T> a, float scale, int wpd) {
    const int lane = threadIdx.x & 31;
    const int64_t gw = int64_t(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int64_t r = gw / wpd;
    if (r >= a.n_rows) return;  // warp-uniform
    const int part = int(gw - r * wpd);
    const int ch = part * 32 * CPL + lane * CPL;
    const int64_t dst = a.dst_lo + r;
    const int beg = __ldg(a.row_ptr + dst), end = __ldg(a.row_ptr + dst + 1);
    const int C = a.C;

    float q[CPL];
    Vec<T, CPL>::ldg(a.q + r * a.ldq + ch, q);

    // W_e^T q and <q, b_e> per head (the folded edge projection).
    float qe0 = 0.f, qe1 = 0.f, qe2 = 0.f, qb = 0.f;
    {
        float w0[CPL], w1[CPL], w2[CPL], wb[CPL];
        Vec<float, CPL>::ldg(a.w_e + ch, w0);
        Vec<float, CPL>::ldg(a.w_e + C + ch, w1);
        Vec<float, CPL>::ldg(a.w_e + 2 * C + ch, w2);
        Vec<float, CPL>::ldg(a.w_e + 3 * C + ch, wb);
#pragma unroll
        for (int j = 0; j < CPL; ++j) {
            qe0 = fmaf(q[j], w0[j], qe0);
            qe1 = fmaf(q[j], w1[j], qe1);
            qe2 = fmaf(q[j], w2[j], qe2);
            qb = fmaf(q[j], wb[j], qb);
        }
        qe0 = head_sum<LPH>(qe0);
        qe1 = head_sum<LPH>(qe1);
        qe2 = head_sum<LPH>(qe2);
        qb = head_sum<LPH>(qb);
    }

    float m = -INFINITY, l = 0.f, pa0 = 0.f, pa1 = 0.f, pa2 = 0.f;
    float acc[CPL];
#pragma unroll
    for (int j = 0; j < CPL; ++j) acc[j] = 0.f;

    const T* K = a.k + ch;
    const T* V = a.v + ch;
    for (int e0 = beg; e0 < end; e0 += 32) {
        const int nb = min(32, end - e0);
        float4 rec = make_float4(0.f, 0.f, 0.f, 0.f);
        if (lane < nb) rec = __ldg(reinterpret_cast<const float4*>(a.edges + e0 + lane));
        for (int j = 0; j < nb; j += U) {
            float ax[U], ay[U], az[U];
            Raw<T, CPL> kr[U], vr[U];
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int src_lane = min(j + u, nb - 1);
                ax[u] = __shfl_sync(kFull, rec.x, src_lane);
                ay[u] = __shfl_sync(kFull, rec.y, src_lane);
                az[u] = __shfl_sync(kFull, rec.z, src_lane);
                const int sj = __float_as_int(__shfl_sync(kFull, rec.w, src_lane));
                if (j + u < nb) {
                    kr[u].ldg(K + int64_t(sj) * a.ldkv);
                    vr[u].ldg(V + int64_t(sj) * a.ldkv);
                }
            }
#pragma unroll
            for (int u = 0; u < U; ++u) {
                if (j + u < nb) {  // warp-uniform
                    float kf[CPL], vf[CPL];
                    kr[u].get(kf);
                    float dot = 0.f;
#pragma unroll
                    for (int c = 0; c < CPL; ++c) dot = fmaf(q[c], kf[c], dot);
                    dot = head_sum<LPH>(dot);
                    const float se = fmaf(qe2, az[u], fmaf(qe1, ay[u], qe0 * ax[u]));
                    const float s = ((dot + se) + qb) * scale;
                    const float mn = fmaxf(m, s);
                    const float corr = expf(m - mn);
                    const float p = expf(s - mn);
                    m = mn;
                    l = fmaf(l, corr, p);
                    vr[u].get(vf);
#pragma unroll
                    for (int c = 0; c < CPL; ++c) acc[c] = fmaf(p, vf[c], acc[c] * corr);
                    pa0 = fmaf(p, ax[u], pa0 * corr);
                    pa1 = fmaf(p, ay[u], pa1 * corr);
                    pa2 = fmaf(p, az[u], pa2 * corr);
                }
            }
        }
    }

    float xr[CPL], o[CPL];
    Vec<T, CPL>::ldg(a.xr + r * a.ldxr + ch, xr);
    if (end > beg) {
        const float inv = 1.0f / l;
        const float p0 = pa0 * inv, p1 = pa1 * inv, p2 = pa2 * inv;
        float w0[CPL], w1[CPL], w2[CPL], wb[CPL];
        Vec<float, CPL>::ldg(a.w_e + ch, w0);
        Vec<float, CPL>::ldg(a.w_e + C + ch, w1);
        Vec<float, CPL>::ldg(a.w_e + 2 * C + ch, w2);
        Vec<float, CPL>::ldg(a.w_e + 3 * C + ch, wb);
#pragma unroll
        for (int c = 0; c < CPL; ++c) {
            const float ev = fmaf(w2[c], p2, fmaf(w1[c], p1, w0[c] * p0)) + wb[c];
            o[c] = fmaf(acc[c], inv, ev);
        }
    } else {
#pragma unroll
        for (int c = 0; c < CPL; ++c) o[c] = 0.f;
    }
#pragma unroll
    for (int c = 0; c < CPL; ++c) o[c] = rnd<T>(rnd<T>(o[c]) + xr[c]);
    Vec<T, CPL>::store(a.out + r * a.ldo + ch, o);
}

}  // namespace

template <class T>
void attention(const AttnArgs<T>& a, cudaStream_t s) {
    if (a.n_rows <= 0) return;
    if (a.C != a.heads * a.head_dim) fail(kInvalidArgument, "attention: C != heads * head_dim");
    const int cpl = (a.C % 256 == 0 && a.head_dim % 8 == 0) ? 8 : 4;
    if (a.C % (32 * cpl) || a.head_dim % cpl)
        fail(kUnsupported, "attention: C must be a multiple of 128 and head_dim a multiple of 4 (got C=" +
                               std::to_string(a.C) + ", head_dim=" + std::to_string(a.head_dim) + ")");
    const int lph = a.head_dim / cpl;
    if (lph > 32 || (lph & (lph - 1)))
        fail(kUnsupported, "attention: head_dim / vector width must be a power of two <= 32");
    const int wpd = a.C / (32 * cpl);
    const float scale = 1.0f / std::sqrt(float(a.head_dim));
    const int64_t warps = a.n_rows * wpd;
    const unsigned grid = unsigned((warps + 7) / 8);
    constexpr int U = 4;
#define VB_ATT(CPL, LPH) attention_kernel<T, CPL, LPH, U><<<grid, 256, 0, s>>>(a, scale, wpd)
#define VB_ATT_L(CPL)                          \
    switch (lph) {                             \
        case 1: VB_ATT(CPL, 1); break;         \
        case 2: VB_ATT(CPL, 2); break;         \
        case 4: VB_ATT(CPL, 4); break;         \
        case 8: VB_ATT(CPL, 8); break;         \
        case 16: VB_ATT(CPL, 16); break;       \
        case 32: VB_ATT(CPL, 32); break;       \
    }
    if (cpl == 8) {
        VB_ATT_L(8)
    } else {
        VB_ATT_L(4)
    }
#undef VB_ATT_L
#undef VB_ATT
    VB_LAUNCH();
}

template void attention<float>(const AttnArgs<float>&, cudaStream_t);
template void attention<__half>(const AttnArgs<__half>&, cudaStream_t);

}  // namespace vb::k
