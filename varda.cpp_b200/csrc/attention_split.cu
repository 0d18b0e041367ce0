// Split-row graph attention whose per-split partial results live in a fixed, statically allocated
// device array instead of memory allocated per call (vb_attention_split_noalloc in the C ABI).
//
// Who needs it: callers that cannot allocate device memory at call time. A serving process whose
// memory pool (PyTorch's caching allocator, a framework arena) already owns all free device memory
// gets cudaErrorMemoryAllocation from cudaMalloc; a latency-critical loop cannot take the implicit
// device-wide synchronisation of cudaMalloc / cudaFree. This entry point allocates nothing: its only
// device storage is g_split_scratch below, which the CUDA module owns for the life of the process.
//
// Each destination row's edges are cut into `splits` contiguous parts; one warp per (row, part,
// channel slab) runs an fp32 online softmax over its part and writes a partial record (per head: the
// running maximum m, the sum l and the softmax-weighted edge-attribute sums; per channel: the
// weighted value sum); a second kernel merges a row's partials (rescaled to the common maximum) into
// the same result as cuda::attention<T> (kernels.cuh): out = T(T(att) + x_r), zero in-degree -> att 0.
// Rows are processed in batches sized to the scratch, all on the caller's stream.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <mutex>
#include <string>
#include <type_traits>

#include "common.h"
#include "dev.cuh"
#include "kernels.cuh"

namespace vb::k {

using namespace vb::d;

namespace {

// 16 MiB of partial records. Every record the merge kernel reads is written in full by the partial
// kernel of the same batch first, so nothing here has to start at zero and nothing is cleared.
constexpr size_t kSplitScratchFloats = size_t(4) << 20;
static __device__ __align__(256) float g_split_scratch[kSplitScratchFloats];

constexpr int kMaxDevices = 64;

// Device address of g_split_scratch on the current device: looked up once per device (the first call
// on a device must run outside stream capture, since the lookup may load the module).
float* split_scratch() {
    static std::mutex mu;
    static float* addr[kMaxDevices] = {};
    int dev = 0;
    VB_CUDA(cudaGetDevice(&dev));
    if (dev < 0 || dev >= kMaxDevices) fail(kUnsupported, "attention_split: device index out of range");
    std::lock_guard<std::mutex> lock(mu);
    if (!addr[dev]) {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_split_scratch);
        if (e != cudaSuccess)
            fail(kCuda, std::string("attention_split: cudaGetSymbolAddress(scratch): ") + cudaGetErrorString(e));
        addr[dev] = static_cast<float*>(p);
    }
    return addr[dev];
}

struct SplitGeom {
    int splits, slabs, rec;  // rec: floats per partial record (C + 5 heads, rounded up to 4)
};

// Lanes of one head (LPH = head_dim / CPL, a power of two) reduce with xor shuffles.
__device__ __forceinline__ float head_sum(float x, int lph) {
    for (int o = 1; o < lph; o <<= 1) x += __shfl_xor_sync(kFull, x, o);
    return x;
}

template <class T, int CPL>
__device__ __forceinline__ void load_ch(const T* p, float (&f)[CPL]) {
#pragma unroll
    for (int i = 0; i < CPL; i += 4) Vec<T, 4>::ldg(p + i, f + i);
}

// The partial softmax of destination `row` (q / x_r / out row lr) over edges [b, e) for this lane's
// CPL channels starting at ch0, written as one partial record: per channel the weighted value sum,
// per head (by its first lane) the running maximum m, the sum l and the weighted attribute sums.
template <class T, int CPL>
__device__ __forceinline__ void partial_body(const AttnArgs<T>& a, int64_t lr, int32_t b, int32_t e, int ch0, int lane,
                                             float scale_log2, float* __restrict__ rec) {
    const int lph = a.head_dim / CPL;
    float q[CPL];
    load_ch<T, CPL>(a.q + lr * a.ldq + ch0, q);
    float qw0 = 0.f, qw1 = 0.f, qw2 = 0.f, qb = 0.f;
#pragma unroll
    for (int i = 0; i < CPL; ++i) {
        qw0 = fmaf(q[i], __ldg(a.w_e + ch0 + i), qw0);
        qw1 = fmaf(q[i], __ldg(a.w_e + a.C + ch0 + i), qw1);
        qw2 = fmaf(q[i], __ldg(a.w_e + 2 * a.C + ch0 + i), qw2);
        qb = fmaf(q[i], __ldg(a.w_e + 3 * a.C + ch0 + i), qb);
    }
    qw0 = head_sum(qw0, lph), qw1 = head_sum(qw1, lph);
    qw2 = head_sum(qw2, lph), qb = head_sum(qb, lph);

    float m = -INFINITY, l = 0.f, s0 = 0.f, s1 = 0.f, s2 = 0.f, acc[CPL];
#pragma unroll
    for (int i = 0; i < CPL; ++i) acc[i] = 0.f;
    for (int32_t j = b; j < e; ++j) {
        const EdgeRec er = a.edges[j];
        const int64_t src = er.src;
        float kv[CPL];
        load_ch<T, CPL>(a.k + src * a.ldkv + ch0, kv);
        float dot = 0.f;
#pragma unroll
        for (int i = 0; i < CPL; ++i) dot = fmaf(q[i], kv[i], dot);
        dot = head_sum(dot, lph);
        const float sc = (dot + er.a0 * qw0 + er.a1 * qw1 + er.a2 * qw2 + qb) * scale_log2;
        const float mn = fmaxf(m, sc);
        const float corr = exp2f(m - mn), p = exp2f(sc - mn);
        m = mn;
        l = fmaf(l, corr, p);
        s0 = fmaf(s0, corr, p * er.a0), s1 = fmaf(s1, corr, p * er.a1), s2 = fmaf(s2, corr, p * er.a2);
        load_ch<T, CPL>(a.v + src * a.ldkv + ch0, kv);
#pragma unroll
        for (int i = 0; i < CPL; ++i) acc[i] = fmaf(p, kv[i], acc[i] * corr);
    }
#pragma unroll
    for (int i = 0; i < CPL; i += 4) *reinterpret_cast<float4*>(rec + ch0 + i) = make_float4(acc[i], acc[i + 1], acc[i + 2], acc[i + 3]);
    if ((lane & (lph - 1)) == 0) {
        float* hrec = rec + a.C + (ch0 / a.head_dim) * 5;
        hrec[0] = m, hrec[1] = l, hrec[2] = s0, hrec[3] = s1, hrec[4] = s2;
    }
}

// Merges `nparts` partial records (rec0, stride `rec` floats) of the row with q / x_r / out row lr
// into out = T(T(att) + x_r); has_edges false gives att = 0.
template <class T, int CPL>
__device__ __forceinline__ void merge_body(const AttnArgs<T>& a, int64_t lr, bool has_edges, const float* __restrict__ rec0,
                                           int rec, int nparts, int ch0) {
    const int h = ch0 / a.head_dim;
    float att[CPL];
#pragma unroll
    for (int i = 0; i < CPL; ++i) att[i] = 0.f;
    if (has_edges) {
        float M = -INFINITY;
        for (int c = 0; c < nparts; ++c) M = fmaxf(M, rec0[c * int64_t(rec) + a.C + h * 5]);
        float L = 0.f, A0 = 0.f, A1 = 0.f, A2 = 0.f, acc[CPL];
#pragma unroll
        for (int i = 0; i < CPL; ++i) acc[i] = 0.f;
        for (int c = 0; c < nparts; ++c) {
            const float* r = rec0 + c * int64_t(rec);
            const float* hr = r + a.C + h * 5;
            if (hr[1] == 0.f) continue;  // an empty part (fewer edges than parts)
            const float wgt = exp2f(hr[0] - M);
            L = fmaf(hr[1], wgt, L);
            A0 = fmaf(hr[2], wgt, A0), A1 = fmaf(hr[3], wgt, A1), A2 = fmaf(hr[4], wgt, A2);
#pragma unroll
            for (int i = 0; i < CPL; i += 4) {
                const float4 v = *reinterpret_cast<const float4*>(r + ch0 + i);
                acc[i] = fmaf(v.x, wgt, acc[i]), acc[i + 1] = fmaf(v.y, wgt, acc[i + 1]);
                acc[i + 2] = fmaf(v.z, wgt, acc[i + 2]), acc[i + 3] = fmaf(v.w, wgt, acc[i + 3]);
            }
        }
        const float inv = 1.0f / L;
#pragma unroll
        for (int i = 0; i < CPL; ++i) {
            const int ch = ch0 + i;
            const float ev = __ldg(a.w_e + ch) * A0 + __ldg(a.w_e + a.C + ch) * A1 + __ldg(a.w_e + 2 * a.C + ch) * A2 +
                             __ldg(a.w_e + 3 * a.C + ch) * L;
            att[i] = (acc[i] + ev) * inv;
        }
    }
    float xr[CPL];
    load_ch<T, CPL>(a.xr + lr * a.ldxr + ch0, xr);
#pragma unroll
    for (int i = 0; i < CPL; ++i) att[i] = rnd<T>(rnd<T>(att[i]) + xr[i]);
    T* o = a.out + lr * a.ldo + ch0;
#pragma unroll
    for (int i = 0; i < CPL; i += 4) Vec<T, 4>::store(o + i, att + i);
}

// One warp per (batch row r, part c, slab s); lane covers channels [s 32 CPL + lane CPL, + CPL).
template <class T, int CPL>
__global__ void __launch_bounds__(256) split_partial_kernel(AttnArgs<T> a, int64_t r0, int64_t nr, SplitGeom g,
                                                            float* __restrict__ part, float scale_log2) {
    const int lane = threadIdx.x & 31;
    const int64_t w = int64_t(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (w >= nr * g.splits * g.slabs) return;
    const int s = int(w % g.slabs);
    const int64_t rc = w / g.slabs;
    const int c = int(rc % g.splits);
    const int64_t r = rc / g.splits;
    const int64_t row = a.dst_lo + r0 + r;
    const int32_t e_beg = a.row_ptr[row], e_end = a.row_ptr[row + 1];
    const int64_t deg = e_end - e_beg;
    const int32_t b = e_beg + int32_t(deg * c / g.splits), e = e_beg + int32_t(deg * (c + 1) / g.splits);
    partial_body<T, CPL>(a, r0 + r, b, e, s * 32 * CPL + lane * CPL, lane, scale_log2,
                         part + (r * g.splits + c) * int64_t(g.rec));
}

// One warp per (batch row r, slab s): merges the row's parts.
template <class T, int CPL>
__global__ void __launch_bounds__(256) split_merge_kernel(AttnArgs<T> a, int64_t r0, int64_t nr, SplitGeom g,
                                                          const float* __restrict__ part) {
    const int lane = threadIdx.x & 31;
    const int64_t w = int64_t(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (w >= nr * g.slabs) return;
    const int s = int(w % g.slabs);
    const int64_t r = w / g.slabs;
    const int64_t row = a.dst_lo + r0 + r;
    const bool has = a.row_ptr[row + 1] > a.row_ptr[row];
    merge_body<T, CPL>(a, r0 + r, has, part + r * g.splits * int64_t(g.rec), g.rec, g.splits,
                       s * 32 * CPL + lane * CPL);
}

// Explicit parts (the engine's wide rows): part i = {graph row, first edge, end edge}, its record at
// scratch + i rec; wide row w's parts are [part0[w], part0[w + 1]).
template <class T, int CPL>
__global__ void __launch_bounds__(256) parts_partial_kernel(AttnArgs<T> a, const int4* __restrict__ parts, int64_t p0,
                                                            int64_t np, int slabs, int rec, float* __restrict__ scratch,
                                                            float scale_log2) {
    const int lane = threadIdx.x & 31;
    const int64_t w = int64_t(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (w >= np * slabs) return;
    const int s = int(w % slabs);
    const int64_t i = p0 + w / slabs;
    const int4 pt = __ldg(parts + i);
    partial_body<T, CPL>(a, int64_t(pt.x) - a.dst_lo, pt.y, pt.z, s * 32 * CPL + lane * CPL, lane, scale_log2,
                         scratch + i * int64_t(rec));
}
template <class T, int CPL>
__global__ void __launch_bounds__(256) parts_merge_kernel(AttnArgs<T> a, const int32_t* __restrict__ rows,
                                                          const int32_t* __restrict__ part0, int64_t w0, int64_t nw,
                                                          int slabs, int rec, const float* __restrict__ scratch) {
    const int lane = threadIdx.x & 31;
    const int64_t w = int64_t(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (w >= nw * slabs) return;
    const int s = int(w % slabs);
    const int64_t r = w0 + w / slabs;
    const int32_t pb = __ldg(part0 + r), pe = __ldg(part0 + r + 1);
    merge_body<T, CPL>(a, int64_t(__ldg(rows + r)) - a.dst_lo, pe > pb, scratch + int64_t(pb) * rec, rec, pe - pb,
                       s * 32 * CPL + lane * CPL);
}

int pick_cpl(int C, int head_dim) {
    const int cpls[4] = {32, 16, 8, 4};
    for (int cpl : cpls) {
        const int lph = head_dim / cpl;
        if (C % (32 * cpl) || head_dim % cpl || lph < 1 || lph > 32 || (lph & (lph - 1))) continue;
        return cpl;
    }
    return 0;
}

template <class T, int CPL>
void run_split(const AttnArgs<T>& a, int splits, float* part, cudaStream_t s) {
    SplitGeom g;
    g.splits = splits;
    g.slabs = a.C / (32 * CPL);
    g.rec = int(align_up(size_t(a.C + 5 * a.heads), 4));
    const int64_t per_row = int64_t(splits) * g.rec;
    if (per_row > int64_t(kSplitScratchFloats))
        fail(kUnsupported, "attention_split: one row needs splits x (C + 5 heads) = " + std::to_string(per_row) +
                               " floats, more than the static scratch of " + std::to_string(kSplitScratchFloats));
    const int64_t batch = int64_t(kSplitScratchFloats) / per_row;
    const float scale_log2 = 1.4426950408889634f / std::sqrt(float(a.head_dim));
    for (int64_t r0 = 0; r0 < a.n_rows; r0 += batch) {
        const int64_t nr = std::min(batch, a.n_rows - r0);
        const int64_t wp = nr * splits * g.slabs, wm = nr * g.slabs;
        split_partial_kernel<T, CPL><<<unsigned((wp + 7) / 8), 256, 0, s>>>(a, r0, nr, g, part, scale_log2);
        VB_LAUNCH();
        split_merge_kernel<T, CPL><<<unsigned((wm + 7) / 8), 256, 0, s>>>(a, r0, nr, g, part);
        VB_LAUNCH();
    }
}

bool aligned(const void* p, size_t n) { return (reinterpret_cast<uintptr_t>(p) % n) == 0; }

}  // namespace

size_t attention_split_scratch_bytes() { return kSplitScratchFloats * sizeof(float); }

int attention_parts_record(int C, int heads) { return int(align_up(size_t(C + 5 * heads), 4)); }

template <class T>
void attention_parts(const AttnArgs<T>& a, const PartsArgs& p, cudaStream_t s) {
    if (p.n_parts <= 0 && p.n_wide <= 0) return;
    const int cpl = pick_cpl(a.C, a.head_dim);
    if (!cpl) fail(kUnsupported, "attention parts: unsupported layout");
    const int slabs = a.C / (32 * cpl), rec = attention_parts_record(a.C, a.heads);
    const float scale_log2 = 1.4426950408889634f / std::sqrt(float(a.head_dim));
    auto run = [&](auto cpl_tag) {
        constexpr int CPL = decltype(cpl_tag)::value;
        const int64_t wp = p.n_parts * slabs, wm = p.n_wide * slabs;
        if (wp > 0) {
            parts_partial_kernel<T, CPL><<<unsigned((wp + 7) / 8), 256, 0, s>>>(a, p.parts, p.part_lo, p.n_parts, slabs,
                                                                             rec, p.scratch, scale_log2);
            VB_LAUNCH();
        }
        if (wm > 0) {
            parts_merge_kernel<T, CPL><<<unsigned((wm + 7) / 8), 256, 0, s>>>(a, p.wide_rows, p.part0, p.wide_lo,
                                                                           p.n_wide, slabs, rec, p.scratch);
            VB_LAUNCH();
        }
    };
    switch (cpl) {
        case 32: run(std::integral_constant<int, 32>{}); break;
        case 16: run(std::integral_constant<int, 16>{}); break;
        case 8: run(std::integral_constant<int, 8>{}); break;
        default: run(std::integral_constant<int, 4>{}); break;
    }
}

template void attention_parts<float>(const AttnArgs<float>&, const PartsArgs&, cudaStream_t);
template void attention_parts<__half>(const AttnArgs<__half>&, const PartsArgs&, cudaStream_t);

template <class T>
void attention_split_noalloc(const AttnArgs<T>& a, int splits, cudaStream_t s) {
    float* part = split_scratch();  // before any early return: the per-device setup of the first call
    if (splits < 1 || splits > 64) fail(kInvalidArgument, "attention_split: splits must be in [1, 64]");
    if (a.rows) fail(kUnsupported, "attention_split: takes a destination range, not a row list");
    if (a.heads < 1 || a.C != a.heads * a.head_dim) fail(kInvalidArgument, "attention_split: C != heads x head_dim");
    if (a.n_rows < 0 || a.dst_lo < 0) fail(kInvalidArgument, "attention_split: bad destination range");
    if (a.n_rows == 0) return;
    if (!a.row_ptr || !a.edges || !a.q || !a.k || !a.v || !a.xr || !a.out || !a.w_e)
        fail(kInvalidArgument, "attention_split: row_ptr, edges, q, k, v, x_r, out and w_e must be non-null");
    if (a.ldq < a.C || a.ldkv < a.C || a.ldxr < a.C || a.ldo < a.C)
        fail(kInvalidArgument, "attention_split: leading dimensions must be at least C");
    const size_t vb = 4 * sizeof(T);  // the kernels move 4 channels at a time
    if (a.ldq % 4 || a.ldkv % 4 || a.ldxr % 4 || a.ldo % 4 || !aligned(a.q, vb) || !aligned(a.k, vb) ||
        !aligned(a.v, vb) || !aligned(a.xr, vb) || !aligned(a.out, vb) || !aligned(a.edges, 16))
        fail(kInvalidArgument, "attention_split: rows must be 4-element aligned (leading dimensions multiples of 4)");
    // channels per lane: the largest of 32/16/8/4 with whole warp slabs and whole heads per lane group
    switch (pick_cpl(a.C, a.head_dim)) {
        case 32: return run_split<T, 32>(a, splits, part, s);
        case 16: return run_split<T, 16>(a, splits, part, s);
        case 8: return run_split<T, 8>(a, splits, part, s);
        case 4: return run_split<T, 4>(a, splits, part, s);
        default: break;
    }
    fail(kUnsupported, "attention_split: needs C a multiple of 128 and head_dim a power-of-two multiple of the "
                       "channels per lane");
}

template void attention_split_noalloc<float>(const AttnArgs<float>&, int, cudaStream_t);
template void attention_split_noalloc<__half>(const AttnArgs<__half>&, int, cudaStream_t);

}  // namespace vb::k
