// Device-side helpers: typed vector loads/stores and fp16 rounding.
#pragma once

#include <cuda_fp16.h>

#include <cstdint>

namespace vb::d {

constexpr unsigned kFull = 0xffffffffu;

template <class T> __device__ __forceinline__ float to_f(T x);
template <> __device__ __forceinline__ float to_f<float>(float x) { return x; }
template <> __device__ __forceinline__ float to_f<__half>(__half x) { return __half2float(x); }
template <class T> __device__ __forceinline__ T from_f(float x);
template <> __device__ __forceinline__ float from_f<float>(float x) { return x; }
template <> __device__ __forceinline__ __half from_f<__half>(float x) { return __float2half_rn(x); }
// Round to the storage type and back (identity for fp32).
template <class T> __device__ __forceinline__ float rnd(float x) { return to_f<T>(from_f<T>(x)); }

// N consecutive elements (N = 4 or 8) through registers as fp32. fp16: 8 or 16 bytes, fp32: 16 or
// 32 bytes; pointers must be aligned to the vector size.
template <class T, int N> struct Vec;
template <> struct Vec<float, 4> {
    static __device__ __forceinline__ void load(const float* p, float* f) {
        const float4 v = *reinterpret_cast<const float4*>(p);
        f[0] = v.x, f[1] = v.y, f[2] = v.z, f[3] = v.w;
    }
    static __device__ __forceinline__ void ldg(const float* p, float* f) {
        const float4 v = __ldg(reinterpret_cast<const float4*>(p));
        f[0] = v.x, f[1] = v.y, f[2] = v.z, f[3] = v.w;
    }
    static __device__ __forceinline__ void store(float* p, const float* f) {
        *reinterpret_cast<float4*>(p) = make_float4(f[0], f[1], f[2], f[3]);
    }
};
template <> struct Vec<float, 8> {
    static __device__ __forceinline__ void load(const float* p, float* f) {
        Vec<float, 4>::load(p, f);
        Vec<float, 4>::load(p + 4, f + 4);
    }
    static __device__ __forceinline__ void ldg(const float* p, float* f) {
        Vec<float, 4>::ldg(p, f);
        Vec<float, 4>::ldg(p + 4, f + 4);
    }
    static __device__ __forceinline__ void store(float* p, const float* f) {
        Vec<float, 4>::store(p, f);
        Vec<float, 4>::store(p + 4, f + 4);
    }
};
template <> struct Vec<__half, 4> {
    static __device__ __forceinline__ void unpack(uint2 u, float* f) {
        const __half2* h = reinterpret_cast<const __half2*>(&u);
        float2 a = __half22float2(h[0]), b = __half22float2(h[1]);
        f[0] = a.x, f[1] = a.y, f[2] = b.x, f[3] = b.y;
    }
    static __device__ __forceinline__ void load(const __half* p, float* f) { unpack(*reinterpret_cast<const uint2*>(p), f); }
    static __device__ __forceinline__ void ldg(const __half* p, float* f) { unpack(__ldg(reinterpret_cast<const uint2*>(p)), f); }
    static __device__ __forceinline__ void store(__half* p, const float* f) {
        uint2 u;
        __half2* h = reinterpret_cast<__half2*>(&u);
        h[0] = __floats2half2_rn(f[0], f[1]);
        h[1] = __floats2half2_rn(f[2], f[3]);
        *reinterpret_cast<uint2*>(p) = u;
    }
};
template <> struct Vec<__half, 8> {
    static __device__ __forceinline__ void unpack(uint4 u, float* f) {
        const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float2 t = __half22float2(h[i]);
            f[2 * i] = t.x, f[2 * i + 1] = t.y;
        }
    }
    static __device__ __forceinline__ void load(const __half* p, float* f) { unpack(*reinterpret_cast<const uint4*>(p), f); }
    static __device__ __forceinline__ void ldg(const __half* p, float* f) { unpack(__ldg(reinterpret_cast<const uint4*>(p)), f); }
    static __device__ __forceinline__ void store(__half* p, const float* f) {
        uint4 u;
        __half2* h = reinterpret_cast<__half2*>(&u);
#pragma unroll
        for (int i = 0; i < 4; ++i) h[i] = __floats2half2_rn(f[2 * i], f[2 * i + 1]);
        *reinterpret_cast<uint4*>(p) = u;
    }
};

__device__ __forceinline__ float warp_sum(float x) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(kFull, x, o);
    return x;
}

// LayerNorm statistics of a row kept as segment records. A segment is a run of segw consecutive
// columns (the column half one GEMM epilogue warp writes); its record is {mean, M2} (M2 the sum of
// squared deviations from the segment mean) of the fp16 values stored there, accumulated in column
// order with the even and the odd columns in separate fp32 lanes, relative to the segment's first
// value k (no cancellation for rows with a large mean). The GEMM epilogue and row_seg_stats use these
// same functions in the same order, so a record does not depend on which kernel made it.
__device__ __forceinline__ void seg_add(float2& s1, float2& s2, float k, float2 v) {
    const float2 dv = __fadd2_rn(v, make_float2(-k, -k));
    s1 = __fadd2_rn(s1, dv);
    s2 = __ffma2_rn(dv, dv, s2);
}
__device__ __forceinline__ float2 seg_record(float2 s1, float2 s2, float k, float n) {
    const float a = __fadd_rn(s1.x, s1.y), q = __fadd_rn(s2.x, s2.y);
    const float m = __fdiv_rn(a, n);
    return make_float2(__fadd_rn(k, m), __fmaf_rn(-a, m, q));  // mean = k + a / n, M2 = q - a^2 / n
}
// A row's mean and 1 / sqrt(var + eps) from its nseg <= kMax records (segments of segw columns,
// C = nseg segw; record i at rec[i stride]), all loads issued first: the mean of the segment means, then
// M2 = sum of (M2_s + segw (mean_s - mean)^2) in segment order, var = M2 / C.
template <int kMax>
__device__ __forceinline__ float2 ln_from_records(const float2* rec, int stride, int nseg, float segw, float eps) {
    float2 r[kMax];
#pragma unroll
    for (int i = 0; i < kMax; ++i) r[i] = i < nseg ? __ldg(rec + i * stride) : make_float2(0.0f, 0.0f);
    float ms = 0.0f;
#pragma unroll
    for (int i = 0; i < kMax; ++i)
        if (i < nseg) ms = __fadd_rn(ms, r[i].x);
    const float mean = __fdiv_rn(ms, float(nseg));
    float m2 = 0.0f;
#pragma unroll
    for (int i = 0; i < kMax; ++i)
        if (i < nseg) {
            const float dm = __fadd_rn(r[i].x, -mean);
            m2 = __fadd_rn(m2, __fmaf_rn(__fmul_rn(segw, dm), dm, r[i].y));
        }
    const float var = __fdiv_rn(m2, __fmul_rn(segw, float(nseg)));
    return make_float2(mean, 1.0f / sqrtf(var + eps));
}

// GELU, torch's formulas in fp32: exact x/2 (1 + erf(x / sqrt 2)), or the tanh form.
__device__ __forceinline__ float gelu(float x, bool tanh_approx) {
    if (!tanh_approx) return x * 0.5f * (1.0f + erff(x * 0.70710678118654752440f));
    const float beta = 0.79788456080286535588f;  // sqrt(2 / pi)
    const float inner = beta * (x + 0.044715f * (x * x * x));
    return 0.5f * x * (1.0f + tanhf(inner));
}

}  // namespace vb::d
