// Shared-memory-staged graph attention (fp16): one CTA per (destination tile, 256-channel head group).
//
// A tile is a run of consecutive destination rows with at most kMaxSrc distinct sources, kMaxRows rows
// and kMaxTileEdges edges (built at load time, graph.cpp make_tiles). The CTA first pulls, with TMA
// bulk copies completing on one mbarrier, the head group's 256-channel slices of K and V (512 bytes
// each) of every distinct source and the tile's packed edge records (contiguous in CSR order), so all
// of the tile's gathers are in flight at once and each source crosses L2 once per tile; meanwhile
// every warp fetches the q / x_r slices of its first row. Then every warp takes rows of the tile
// (prefetching its next row's q / x_r) and runs an fp32 online softmax over the row's edges from
// shared memory (lane = 8 channels = one 16-byte vector, LPH = head_dim / 8 lanes per head):
//   s_e = (<q, k_e> + <W_e^T q, a_e> + <q, b_e>) / sqrt(d)   (log2 domain, ex2),
//   acc = sum p_e v_e, l = sum p_e, pa = sum p_e a_e, p_e = 2^(s_e - m) relative to a reference
//   maximum m raised (and the sums rescaled) only when a score exceeds it by more than 2^8;
//   o = acc / l + W_e (pa / l) + b_e,  out = T(T(o) + x_r).
// Every row's arithmetic depends only on that row, so results do not depend on the tiling (hence not
// on the GPU partition either). Heavy rows go to the gather kernel (attention.cu).
#include <cmath>
#include <string>

#include "common.h"
#include "dev.cuh"
#include "kernels.cuh"

namespace vb::k {

using namespace vb::d;

namespace {

constexpr int kHG = 256;             // channels per head group (one CTA)
constexpr int kMaxSrc = 80;          // distinct sources per tile: 80 x 1 KB of K|V slices
constexpr int kMaxRows = 64;         // rows per tile
constexpr int kMaxTileEdges = 1024;  // edges per tile: 16 KB of packed records
constexpr size_t kSmemBytes = size_t(kMaxSrc) * kHG * 2 * 2 + size_t(kMaxTileEdges) * sizeof(EdgeRec);
constexpr unsigned long long kTimeoutNs = 4000000000ull;

__device__ int g_att_error = 0;

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return uint32_t(__cvta_generic_to_shared(p)); }
__device__ __forceinline__ uint64_t now_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
__device__ __forceinline__ bool mbar_test(uint64_t* b, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(ok)
        : "r"(smem_u32(b)), "r"(parity)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_u32(dst)),
                 "l"(src), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}
__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
template <int LPH>
__device__ __forceinline__ float head_sum(float x) {
#pragma unroll
    for (int o = 1; o < LPH; o <<= 1) x += __shfl_xor_sync(kFull, x, o);
    return x;
}
__device__ __forceinline__ void h8(const uint4& u, float2 (&f)[4]) {
    const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) f[i] = __half22float2(h[i]);
}
__device__ __forceinline__ void w8(const float* p, float2 (&f)[4]) {
    const float4 a = __ldg(reinterpret_cast<const float4*>(p)), b = __ldg(reinterpret_cast<const float4*>(p) + 1);
    f[0] = make_float2(a.x, a.y), f[1] = make_float2(a.z, a.w), f[2] = make_float2(b.x, b.y), f[3] = make_float2(b.z, b.w);
}

template <int LPH>
__global__ void __launch_bounds__(256, 2) attention_tiled_kernel(TileArgs a, float scale_log2) {
    extern __shared__ __align__(128) uint8_t sm[];
    __shared__ uint64_t bar;
    __shared__ int32_t rp[kMaxRows + 1];
    const int n_hg = a.C / kHG;
    const int t = a.tile0 + int(blockIdx.x) / n_hg, hg = int(blockIdx.x) % n_hg;
    const int4 tl = __ldg(a.tiles + t);  // row0, nrows, src0, nsrc
    const int ch0 = hg * kHG;
    __half* Ks = reinterpret_cast<__half*>(sm);
    __half* Vs = Ks + kMaxSrc * kHG;
    const EdgeRec* Es = reinterpret_cast<const EdgeRec*>(Vs + kMaxSrc * kHG);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int e0 = __ldg(a.row_ptr + tl.x), ne = __ldg(a.row_ptr + tl.x + tl.y) - e0;

    for (int i = threadIdx.x; i <= tl.y; i += blockDim.x) rp[i] = __ldg(a.row_ptr + tl.x + i) - e0;
    if (threadIdx.x == 0) {
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_u32(&bar)));
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    if (warp == 0) {
        if (lane == 0)
            asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(&bar)),
                         "r"(uint32_t(tl.w) * 2u * kHG * 2u + uint32_t(ne) * uint32_t(sizeof(EdgeRec)))
                         : "memory");
        __syncwarp();
        if (lane == 0 && ne > 0)
            bulk_g2s(const_cast<EdgeRec*>(Es), a.edges + e0, uint32_t(ne) * uint32_t(sizeof(EdgeRec)), &bar);
        for (int i = lane; i < tl.w; i += 32) {
            const int64_t s = __ldg(a.srcs + tl.z + i);
            bulk_g2s(Ks + i * kHG, a.k + s * a.ldkv + ch0, kHG * 2, &bar);
            bulk_g2s(Vs + i * kHG, a.v + s * a.ldkv + ch0, kHG * 2, &bar);
        }
    }
    // the first row's q / x_r slices and the edge weights of this lane's channels, while the copies fly
    const int C = a.C;
    const int ch = ch0 + lane * 8;
    int r = warp;
    uint4 qn = make_uint4(0, 0, 0, 0), xn = qn;
    if (r < tl.y) {
        const int64_t lr = int64_t(tl.x + r) - a.dst_lo;
        qn = __ldg(reinterpret_cast<const uint4*>(a.q + lr * a.ldq + ch));
        xn = __ldg(reinterpret_cast<const uint4*>(a.xr + lr * a.ldxr + ch));
    }
    float2 w0[4], w1[4], w2[4], wb[4];
    w8(a.w_e + ch, w0), w8(a.w_e + C + ch, w1), w8(a.w_e + 2 * C + ch, w2), w8(a.w_e + 3 * C + ch, wb);

    // bounded wait for the slices; on timeout flag the error and skip the compute (the CTA's copies
    // are then the only thing left in flight, and the next wait covers them)
    bool ok = mbar_test(&bar, 0);
    if (!ok) {
        const uint64_t t0 = now_ns();
        while (!(ok = mbar_test(&bar, 0)))
            if (now_ns() - t0 > kTimeoutNs) break;
    }
    if (!ok) {
        if (threadIdx.x == 0) atomicExch(&g_att_error, 1);
        return;
    }

    for (; r < tl.y; r += 8) {
        const int64_t lr = int64_t(tl.x + r) - a.dst_lo;  // local q / x_r / out row
        float2 q[4];
        h8(qn, q);
        const uint4 xu = xn;
        if (r + 8 < tl.y) {  // prefetch the next row's slices
            const int64_t ln = lr + 8;
            qn = __ldg(reinterpret_cast<const uint4*>(a.q + ln * a.ldq + ch));
            xn = __ldg(reinterpret_cast<const uint4*>(a.xr + ln * a.ldxr + ch));
        }
        float qe0, qe1, qe2, qb;
        {
            float2 s0 = make_float2(0.f, 0.f), s1 = s0, s2 = s0, sb = s0;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                s0 = __ffma2_rn(q[j], w0[j], s0), s1 = __ffma2_rn(q[j], w1[j], s1);
                s2 = __ffma2_rn(q[j], w2[j], s2), sb = __ffma2_rn(q[j], wb[j], sb);
            }
            qe0 = head_sum<LPH>(s0.x + s0.y), qe1 = head_sum<LPH>(s1.x + s1.y);
            qe2 = head_sum<LPH>(s2.x + s2.y), qb = head_sum<LPH>(sb.x + sb.y);
        }
        const int beg = rp[r], end = rp[r + 1];
        float m = -INFINITY, l = 0.f, pa0 = 0.f, pa1 = 0.f, pa2 = 0.f;
        float2 acc[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
#pragma unroll 2
        for (int e = beg; e < end; ++e) {
            const float4 rec = *reinterpret_cast<const float4*>(Es + e);
            const int slot = __float_as_int(rec.w);
            float2 kf[4], vf[4];
            h8(*reinterpret_cast<const uint4*>(Ks + slot * kHG + lane * 8), kf);
            h8(*reinterpret_cast<const uint4*>(Vs + slot * kHG + lane * 8), vf);
            float2 d2 = make_float2(0.f, 0.f);
#pragma unroll
            for (int c = 0; c < 4; ++c) d2 = __ffma2_rn(q[c], kf[c], d2);
            const float dot = head_sum<LPH>(d2.x + d2.y);
            const float se = fmaf(qe2, rec.z, fmaf(qe1, rec.y, qe0 * rec.x));
            const float s = ((dot + se) + qb) * scale_log2;
            // sums relative to a reference maximum raised only when a score exceeds it by 2^8
            if (__any_sync(kFull, s > m + 8.0f)) {
                const float mn = fmaxf(m, s);
                const float corr = ex2(m - mn);
                m = mn;
                l *= corr, pa0 *= corr, pa1 *= corr, pa2 *= corr;
                const float2 c2 = make_float2(corr, corr);
#pragma unroll
                for (int c = 0; c < 4; ++c) acc[c] = __fmul2_rn(acc[c], c2);
            }
            const float p = ex2(s - m);
            l += p;
            pa0 = fmaf(p, rec.x, pa0), pa1 = fmaf(p, rec.y, pa1), pa2 = fmaf(p, rec.z, pa2);
            const float2 p2 = make_float2(p, p);
#pragma unroll
            for (int c = 0; c < 4; ++c) acc[c] = __ffma2_rn(p2, vf[c], acc[c]);
        }
        float xr[8], o[8];
        {
            float2 xf[4];
            h8(xu, xf);
#pragma unroll
            for (int c = 0; c < 4; ++c) xr[2 * c] = xf[c].x, xr[2 * c + 1] = xf[c].y;
        }
        if (end > beg) {
            const float inv = 1.0f / l;
            const float p0 = pa0 * inv, p1 = pa1 * inv, p2 = pa2 * inv;
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                o[2 * c] = fmaf(acc[c].x, inv, fmaf(w2[c].x, p2, fmaf(w1[c].x, p1, w0[c].x * p0)) + wb[c].x);
                o[2 * c + 1] = fmaf(acc[c].y, inv, fmaf(w2[c].y, p2, fmaf(w1[c].y, p1, w0[c].y * p0)) + wb[c].y);
            }
        } else {
#pragma unroll
            for (int c = 0; c < 8; ++c) o[c] = 0.f;
        }
#pragma unroll
        for (int c = 0; c < 8; ++c) o[c] = rnd<__half>(rnd<__half>(o[c]) + xr[c]);
        Vec<__half, 8>::store(a.out + lr * a.ldo + ch, o);
    }
}

}  // namespace

int tiled_max_src() { return kMaxSrc; }
int tiled_max_rows() { return kMaxRows; }
int tiled_max_edges() { return kMaxTileEdges; }
bool tiled_supported(int C, int head_dim) {
    return C % kHG == 0 && head_dim % 8 == 0 && head_dim <= kHG && (head_dim / 8 & (head_dim / 8 - 1)) == 0;
}

void attention_tiled(const TileArgs& a, float scale_log2, cudaStream_t s) {
    if (a.ntiles <= 0) return;
    if (!tiled_supported(a.C, a.head_dim)) fail(kUnsupported, "tiled attention: unsupported layout");
    const int lph = a.head_dim / 8;
    const size_t smem = kSmemBytes;
    const unsigned grid = unsigned(a.ntiles * (a.C / kHG));
#define VB_TA(L)                                                                                               \
    do {                                                                                                       \
        static std::atomic<uint64_t> cfg{0};                                                                   \
        once_per_device(cfg, [&] {                                                                             \
            VB_CUDA(cudaFuncSetAttribute(attention_tiled_kernel<L>, cudaFuncAttributeMaxDynamicSharedMemorySize, \
                                         int(smem)));                                                          \
        });                                                                                                    \
        attention_tiled_kernel<L><<<grid, 256, smem, s>>>(a, scale_log2);                                      \
    } while (0)
    switch (lph) {
        case 1: VB_TA(1); break;
        case 2: VB_TA(2); break;
        case 4: VB_TA(4); break;
        case 8: VB_TA(8); break;
        case 16: VB_TA(16); break;
        case 32: VB_TA(32); break;
        default: fail(kUnsupported, "tiled attention: head_dim");
    }
#undef VB_TA
    VB_LAUNCH();
}

int take_attention_error() {
    VB_CUDA(cudaDeviceSynchronize());
    int e = 0, zero = 0;
    VB_CUDA(cudaMemcpyFromSymbol(&e, g_att_error, sizeof(int)));
    if (e) VB_CUDA(cudaMemcpyToSymbol(g_att_error, &zero, sizeof(int)));
    return e | take_tc_error();
}

}  // namespace vb::k
