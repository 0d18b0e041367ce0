// Graph attention over a destination-major CSR graph (see kernels.cuh for the contract).
//
// Layout: a destination's C channels are split over WPD = C / (32 CPL) warps; lane l of part p owns
// the CPL consecutive channels starting at p 32 CPL + l CPL (16 fp16 channels = two 16-byte
// vectors at the Varda width, so a C = 1024 destination takes two warps). LPH = head_dim / CPL
// lanes share a head: per-head dot products are a butterfly over LPH lanes, and the per-edge
// softmax scalars are computed by those LPH lanes only. Each warp streams its destination's CSR row:
// edge records are fetched 32 at a time with one coalesced load (lane i holds record i) and
// broadcast with shuffles; the K/V gathers of the next U edges are issued before the current U are
// consumed (software pipeline, 2U x 2 x CPL channels in flight per lane).
//
// The kernel is bound by instruction issue, not memory (ncu on the C2 block: DRAM traffic at the
// compulsory bytes, L2 at 16% of its peak); the arithmetic is therefore packed fp32x2 FMAs
// (sm_100 FFMA2) for the dot products and the V accumulation, and the softmax runs in the log2
// domain on the hardware exp2.
//
// Numerics (the reference's semantics, cpu/kernels.cpp:98-158 and backend_cpu.cpp:333-340):
//   s_j  = (<q, k_j> + <W_e^T q, a_j> + <q, b_e>) / sqrt(d)    (edge projection folded, per head)
//   fp32 online softmax over the row: l = sum p_j, acc = sum p_j v_j, pa = sum p_j a_j with
//   p_j = 2^(s_j - m) relative to a reference maximum m that is raised (and the sums rescaled) only
//   when a score exceeds it by more than 2^8, so p_j <= 2^8 (exact in real arithmetic; only the
//   rounding of the sums differs from rescaling at every edge)
//   o    = acc / l + W_e (pa / l) + b_e                       (sum_j p_j / l = 1)
//   out  = T(T(o) + x_r);  zero in-degree: o = 0, so out = x_r exactly.
// Every destination's arithmetic depends only on its own row (not on the launch's row range), so a
// destination sub-range, and any partition of the destinations over GPUs, gives the same bits.
#include <cmath>
#include <cstdlib>
#include <string>

#include "common.h"
#include "dev.cuh"
#include "kernels.cuh"

namespace vb::k {

using namespace vb::d;

namespace {

// Raw CPL-channel vectors (16-byte loads), unpacked to fp32 pairs when consumed.
template <class T, int CPL> struct Raw;
template <> struct Raw<__half, 16> {
    uint4 u[2];
    __device__ __forceinline__ void ldg(const __half* p) {
        u[0] = __ldg(reinterpret_cast<const uint4*>(p));
        u[1] = __ldg(reinterpret_cast<const uint4*>(p) + 1);
    }
    __device__ __forceinline__ void get(float2* f) const {
        const __half2* h = reinterpret_cast<const __half2*>(u);
#pragma unroll
        for (int i = 0; i < 8; ++i) f[i] = __half22float2(h[i]);
    }
};
template <> struct Raw<__half, 8> {
    uint4 u;
    __device__ __forceinline__ void ldg(const __half* p) { u = __ldg(reinterpret_cast<const uint4*>(p)); }
    __device__ __forceinline__ void get(float2* f) const {
        const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
        for (int i = 0; i < 4; ++i) f[i] = __half22float2(h[i]);
    }
};
template <> struct Raw<__half, 4> {
    uint2 u;
    __device__ __forceinline__ void ldg(const __half* p) { u = __ldg(reinterpret_cast<const uint2*>(p)); }
    __device__ __forceinline__ void get(float2* f) const {
        const __half2* h = reinterpret_cast<const __half2*>(&u);
        f[0] = __half22float2(h[0]), f[1] = __half22float2(h[1]);
    }
};
template <> struct Raw<float, 4> {
    float4 u;
    __device__ __forceinline__ void ldg(const float* p) { u = __ldg(reinterpret_cast<const float4*>(p)); }
    __device__ __forceinline__ void get(float2* f) const { f[0] = make_float2(u.x, u.y), f[1] = make_float2(u.z, u.w); }
};
template <> struct Raw<float, 8> {
    float4 a, b;
    __device__ __forceinline__ void ldg(const float* p) {
        a = __ldg(reinterpret_cast<const float4*>(p));
        b = __ldg(reinterpret_cast<const float4*>(p) + 1);
    }
    __device__ __forceinline__ void get(float2* f) const {
        f[0] = make_float2(a.x, a.y), f[1] = make_float2(a.z, a.w), f[2] = make_float2(b.x, b.y);
        f[3] = make_float2(b.z, b.w);
    }
};

template <int LPH>
__device__ __forceinline__ float head_sum(float x) {
#pragma unroll
    for (int o = 1; o < LPH; o <<= 1) x += __shfl_xor_sync(kFull, x, o);
    return x;
}

__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// CPL channels of a row as CPL / 2 fp32 pairs
template <class T, int CPL>
__device__ __forceinline__ void load_pairs(const T* p, float2 (&f)[CPL / 2]) {
    Raw<T, CPL> r;
    r.ldg(p);
    r.get(f);
}
template <int CPL>
__device__ __forceinline__ void load_pairs_f32(const float* p, float2 (&f)[CPL / 2]) {
#pragma unroll
    for (int i = 0; i < CPL / 4; ++i) {
        const float4 v = __ldg(reinterpret_cast<const float4*>(p) + i);
        f[2 * i] = make_float2(v.x, v.y), f[2 * i + 1] = make_float2(v.z, v.w);
    }
}

constexpr float kSlack = 8.0f;  // log2 units of headroom of the softmax sums over their reference maximum

template <class T, int CPL, int LPH, int U, int MINB>
__global__ void __launch_bounds__(256, MINB) attention_kernel(AttnArgs<T> a, float scale_log2, int wpd) {
    constexpr int P = CPL / 2;  // fp32 pairs per lane
    const int lane = threadIdx.x & 31;
    const int64_t gw = int64_t(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int64_t ri = gw / wpd;
    if (ri >= a.n_rows) return;  // warp-uniform
    const int part = int(gw - ri * wpd);
    const int ch = part * 32 * CPL + lane * CPL;
    const int64_t dst = a.rows ? int64_t(__ldg(a.rows + ri)) : a.dst_lo + ri;
    const int64_t r = dst - a.dst_lo;  // local q / x_r / out row
    const int beg = __ldg(a.row_ptr + dst), end = __ldg(a.row_ptr + dst + 1);
    const int C = a.C;

    float2 q[P];
    load_pairs<T, CPL>(a.q + r * a.ldq + ch, q);

    // W_e^T q and <q, b_e> per head (the folded edge projection)
    float qe0, qe1, qe2, qb;
    {
        float2 w0[P], w1[P], w2[P], wb[P];
        load_pairs_f32<CPL>(a.w_e + ch, w0);
        load_pairs_f32<CPL>(a.w_e + C + ch, w1);
        load_pairs_f32<CPL>(a.w_e + 2 * C + ch, w2);
        load_pairs_f32<CPL>(a.w_e + 3 * C + ch, wb);
        float2 s0 = make_float2(0.f, 0.f), s1 = s0, s2 = s0, sb = s0;
#pragma unroll
        for (int j = 0; j < P; ++j) {
            s0 = __ffma2_rn(q[j], w0[j], s0);
            s1 = __ffma2_rn(q[j], w1[j], s1);
            s2 = __ffma2_rn(q[j], w2[j], s2);
            sb = __ffma2_rn(q[j], wb[j], sb);
        }
        qe0 = head_sum<LPH>(s0.x + s0.y);
        qe1 = head_sum<LPH>(s1.x + s1.y);
        qe2 = head_sum<LPH>(s2.x + s2.y);
        qb = head_sum<LPH>(sb.x + sb.y);
    }

    float m = -INFINITY, l = 0.f, pa0 = 0.f, pa1 = 0.f, pa2 = 0.f;
    float2 acc[P];
#pragma unroll
    for (int j = 0; j < P; ++j) acc[j] = make_float2(0.f, 0.f);

    const T* K = a.k + ch;
    const T* V = a.v + ch;
    for (int e0 = beg; e0 < end; e0 += 32) {
        const int nb = min(32, end - e0);
        float4 rec = make_float4(0.f, 0.f, 0.f, 0.f);
        if (lane < nb) rec = __ldg(reinterpret_cast<const float4*>(a.edges + e0 + lane));
        // software pipeline over this batch: gathers for edges [j + U, j + 2U) are in flight while
        // edges [j, j + U) are consumed
        // two register stages, indexed at compile time (stage 0 / stage 1 alternate in the loop body)
        Raw<T, CPL> kr0[U], vr0[U], kr1[U], vr1[U];
        float ax0[U], ay0[U], az0[U], ax1[U], ay1[U], az1[U];
        auto fetch = [&](Raw<T, CPL>(&kr)[U], Raw<T, CPL>(&vr)[U], float(&ax)[U], float(&ay)[U], float(&az)[U],
                         int j) {
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int sl = min(j + u, nb - 1);
                ax[u] = __shfl_sync(kFull, rec.x, sl);
                ay[u] = __shfl_sync(kFull, rec.y, sl);
                az[u] = __shfl_sync(kFull, rec.z, sl);
                const int sj = __float_as_int(__shfl_sync(kFull, rec.w, sl));
                if (j + u < nb) {
                    kr[u].ldg(K + int64_t(sj) * a.ldkv);
                    vr[u].ldg(V + int64_t(sj) * a.ldkv);
                }
            }
        };
        auto consume = [&](const Raw<T, CPL>(&kr)[U], const Raw<T, CPL>(&vr)[U], const float(&ax)[U],
                           const float(&ay)[U], const float(&az)[U], int j) {
#pragma unroll
            for (int u = 0; u < U; ++u) {
                if (j + u < nb) {  // warp-uniform
                    float2 kf[P], vf[P];
                    kr[u].get(kf);
                    float2 d2 = make_float2(0.f, 0.f);
#pragma unroll
                    for (int c = 0; c < P; ++c) d2 = __ffma2_rn(q[c], kf[c], d2);
                    const float dot = head_sum<LPH>(d2.x + d2.y);
                    const float se = fmaf(qe2, az[u], fmaf(qe1, ay[u], qe0 * ax[u]));
                    const float s = ((dot + se) + qb) * scale_log2;  // log2 domain
                    // the sums are kept relative to a reference maximum m that moves only when a score
                    // exceeds it by more than kSlack (any lane of the warp): p <= 2^kSlack, and most
                    // edges skip the rescale
                    if (__any_sync(kFull, s > m + kSlack)) {
                        const float mn = fmaxf(m, s);
                        const float corr = ex2(m - mn);
                        m = mn;
                        l *= corr, pa0 *= corr, pa1 *= corr, pa2 *= corr;
                        const float2 c2 = make_float2(corr, corr);
#pragma unroll
                        for (int c = 0; c < P; ++c) acc[c] = __fmul2_rn(acc[c], c2);
                    }
                    const float p = ex2(s - m);
                    l += p;
                    vr[u].get(vf);
                    const float2 p2 = make_float2(p, p);
#pragma unroll
                    for (int c = 0; c < P; ++c) acc[c] = __ffma2_rn(p2, vf[c], acc[c]);
                    pa0 = fmaf(p, ax[u], pa0);
                    pa1 = fmaf(p, ay[u], pa1);
                    pa2 = fmaf(p, az[u], pa2);
                }
            }
        };
        fetch(kr0, vr0, ax0, ay0, az0, 0);
        for (int j = 0; j < nb; j += 2 * U) {
            if (j + U < nb) fetch(kr1, vr1, ax1, ay1, az1, j + U);
            consume(kr0, vr0, ax0, ay0, az0, j);
            if (j + U >= nb) break;
            if (j + 2 * U < nb) fetch(kr0, vr0, ax0, ay0, az0, j + 2 * U);
            consume(kr1, vr1, ax1, ay1, az1, j + U);
        }
    }

    float xr[CPL], o[CPL];
    Vec<T, (CPL > 8 ? 8 : CPL)>::ldg(a.xr + r * a.ldxr + ch, xr);
    if (CPL > 8) Vec<T, 8>::ldg(a.xr + r * a.ldxr + ch + 8, xr + (CPL > 8 ? 8 : 0));
    if (end > beg) {
        const float inv = 1.0f / l;
        const float p0 = pa0 * inv, p1 = pa1 * inv, p2 = pa2 * inv;
        float2 w0[P], w1[P], w2[P], wb[P];
        load_pairs_f32<CPL>(a.w_e + ch, w0);
        load_pairs_f32<CPL>(a.w_e + C + ch, w1);
        load_pairs_f32<CPL>(a.w_e + 2 * C + ch, w2);
        load_pairs_f32<CPL>(a.w_e + 3 * C + ch, wb);
#pragma unroll
        for (int c = 0; c < P; ++c) {
            const float e_x = fmaf(w2[c].x, p2, fmaf(w1[c].x, p1, w0[c].x * p0)) + wb[c].x;
            const float e_y = fmaf(w2[c].y, p2, fmaf(w1[c].y, p1, w0[c].y * p0)) + wb[c].y;
            o[2 * c] = fmaf(acc[c].x, inv, e_x);
            o[2 * c + 1] = fmaf(acc[c].y, inv, e_y);
        }
    } else {
#pragma unroll
        for (int c = 0; c < CPL; ++c) o[c] = 0.f;
    }
#pragma unroll
    for (int c = 0; c < CPL; ++c) o[c] = rnd<T>(rnd<T>(o[c]) + xr[c]);
    T* out = a.out + r * a.ldo + ch;
    Vec<T, (CPL > 8 ? 8 : CPL)>::store(out, o);
    if (CPL > 8) Vec<T, 8>::store(out + 8, o + (CPL > 8 ? 8 : 0));
}

}  // namespace

template <class T>
void attention(const AttnArgs<T>& a, cudaStream_t s) {
    if (a.n_rows <= 0) return;
    if (a.C != a.heads * a.head_dim) fail(kInvalidArgument, "attention: C != heads * head_dim");
    // Launch shape: channels per lane (CPL), edges per pipeline stage (U) and resident blocks per SM
    // (MINB, the register budget). Measured on the C2 block (fp16, C = 1024, head_dim 64): 8 channels
    // per lane at 4 blocks per SM (32 warps) 1.65 ms, 16 channels at 2 blocks 1.97 ms, 8 at 3 blocks
    // 2.28 ms: the kernel is latency-bound and occupancy wins. VB_ATT_VARIANT picks an alternative:
    // 1 = (16, 1, 2), 2 = (8, 2, 3), 3 = (8, 1, 5), 4 = (4, 1, 4). (A variant with one broadcast record
    // load per edge instead of the 32-record batch and shuffles, and the q.k products on the sm_100
    // mixed-precision FMA, measured 1.70 ms against 1.57 ms.)
    const char* venv = std::getenv("VB_ATT_VARIANT");
    const int variant = venv && *venv ? std::atoi(venv) : 0;
    int cpl = 4;
    if (sizeof(T) == 2 && variant == 1 && a.C % 512 == 0 && a.head_dim % 16 == 0) cpl = 16;
    else if (variant != 4 && a.C % 256 == 0 && a.head_dim % 8 == 0) cpl = 8;
    if (a.C % (32 * cpl) || a.head_dim % cpl)
        fail(kUnsupported, "attention: C must be a multiple of 128 and head_dim a multiple of 4 (got C=" +
                               std::to_string(a.C) + ", head_dim=" + std::to_string(a.head_dim) + ")");
    const int lph = a.head_dim / cpl;
    if (lph > 32 || (lph & (lph - 1)))
        fail(kUnsupported, "attention: head_dim / vector width must be a power of two <= 32");
    const int wpd = a.C / (32 * cpl);
    const float scale_log2 = 1.4426950408889634f / std::sqrt(float(a.head_dim));
    const int64_t warps = a.n_rows * wpd;
    const unsigned grid = unsigned((warps + 7) / 8);
#define VB_ATT(CPL, LPH, U, MB) attention_kernel<T, CPL, LPH, U, MB><<<grid, 256, 0, s>>>(a, scale_log2, wpd)
#define VB_ATT_L(CPL, U, MB)                          \
    switch (lph) {                                    \
        case 1: VB_ATT(CPL, 1, U, MB); break;         \
        case 2: VB_ATT(CPL, 2, U, MB); break;         \
        case 4: VB_ATT(CPL, 4, U, MB); break;         \
        case 8: VB_ATT(CPL, 8, U, MB); break;         \
        case 16: VB_ATT(CPL, 16, U, MB); break;       \
        case 32: VB_ATT(CPL, 32, U, MB); break;       \
    }
    if constexpr (sizeof(T) == 2) {
        if (cpl == 16) {
            VB_ATT_L(16, 1, 2)
        } else if (cpl == 8 && variant == 2) {
            VB_ATT_L(8, 2, 3)
        } else if (cpl == 8 && variant == 3) {
            VB_ATT_L(8, 1, 5)
        } else if (cpl == 8) {
            VB_ATT_L(8, 1, 4)
        } else {
            VB_ATT_L(4, 1, 4)
        }
    } else {
        if (cpl == 8) {
            VB_ATT_L(8, 1, 2)
        } else {
            VB_ATT_L(4, 2, 2)
        }
    }
#undef VB_ATT_L
#undef VB_ATT
    VB_LAUNCH();
}

template void attention<float>(const AttnArgs<float>&, cudaStream_t);
template void attention<__half>(const AttnArgs<__half>&, cudaStream_t);

}  // namespace vb::k
