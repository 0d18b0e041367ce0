// Tile-sparse tensor-core edge attention (fp16, head_dim 64): the processor graph's attention as small
// matrix products per tile of destination rows.
//
// A tile (graph.h, make_tc_tiles) is up to 64 consecutive destination rows whose edges reach at most
// 128 distinct sources, numbered by first appearance ("slots"). For each head h, with the tile's
// queries Q_h [64 x 64], its sources' K_h, V_h [128 x 64] and the edge attributes a_e:
//   S   = Q_h K_h^T                    (tensor cores, fp32 accumulation)   [64 x 128]
//   s_e = (S[r, slot_e] + <W_e^T q_r, a_e> + <q_r, b_e>) / sqrt(d)  for every edge e = (r, slot_e),
//         -inf where (r, slot) is not an edge; the log2 domain throughout (ex2)
//   p   = 2^(s - max_r s), rounded to fp16 (the operand of the next product); l_r = sum_e p_e
//   O   = P V_h + [pa | l] [W_e ; b_e]  (tensor cores; pa_r = sum_e p_e a_e carried as fp16 hi + lo)
//   out = T(T(O / l) + x_r)             (zero in-degree: O = 0, l = 0 -> out = x_r exactly)
// which is the reference's per-destination softmax over (k_j + e_ij) with values (v_j + e_ij),
// e_ij = W_e a_ij + b_e (cpu/kernels.cpp:98-158, backend_cpu.cpp:333-340), with fp32 arithmetic
// except that the attention weights enter the value sums as fp16 (relative rounding <= 2^-11, the
// normalisation uses the same rounded weights).
//
// The products run on the warp-level tensor-core instruction (mma.sync m16n8k16, fp16 in, fp32
// accumulate): the score matrix of a 16-row block is sparse (about 14 edges per row among the tile's
// 128 slots), and only the 8-column blocks that hold an edge of the row block are multiplied and
// exponentiated, which a 16-row granularity allows and the 128-row tiles of tcgen05 do not.
//
// Kernel layout: persistent CTAs of 4 consumer warps and 1 producer warp.
//   producer   per tile: the record block (row offsets, column-block masks, 8-byte edge records) by
//              one bulk copy; per head: K_h and V_h rows of the tile's sources by TMA row gathers
//              (cp.async.bulk.tensor tile::gather4, 4 rows of 128 bytes each) and Q_h by one 2-D TMA
//              tile copy, into a 3-deep ring of head stages (128-byte swizzle, full / empty mbarriers).
//   consumers  a tile of nb row blocks has nb x heads tasks (head-major); task i goes to warp i % 4, so
//              warps work on up to two heads at once. Per task (16 rows, one head):
//                qe = Q W_ext (the edge weights as 8 extra columns) -> per row <W_e^T q, a>, <q, b_e>;
//                pass 1 (two lanes per row, its edges): E[r][slot_e] = edge term, in a per-warp
//                  [16 x 136] fp32 buffer that otherwise holds -inf;
//                S for the active column blocks; s = S scale + E written back; row max; p (fp16);
//                pass 2 (per row, its edges): pa from the rounded weights, buffer entries back to -inf;
//                O = P V for the active 16-slot steps, plus the W_e / b_e terms; epilogue with x_r.
// Every mbarrier wait is bounded (4 s of %globaltimer): on timeout the CTA sets the device error flag
// (read by take_attention_error), stops, and the producer drains its own copies before returning.
#include <cuda.h>

#include <cmath>
#include <string>

#include "common.h"
#include "dev.cuh"
#include "gemm_tc.cuh"
#include "kernels.cuh"

namespace vb::k {

using namespace vb::d;

namespace {

constexpr int kHD = 64;                  // head_dim
constexpr int kNT = kTcMaxSrc / 8;       // 8-column blocks of the score matrix
constexpr int kStages = 3;               // head stages
constexpr int kConsumers = 4;
constexpr int kThreads = 32 * (kConsumers + 1);
constexpr int kEPad = kTcMaxSrc + 8;     // edge-term buffer row stride (floats)
constexpr int kKVBytes = kTcMaxSrc * kHD * 2;  // 16 KB
constexpr int kQBytes = kTcRows * kHD * 2;     // 8 KB
constexpr int kStageBytes = 2 * kKVBytes + kQBytes;
constexpr int kBlobMax = kTcEdgeOff + 8 * kTcMaxEdges;
constexpr int kMaxHeads = 32;
constexpr unsigned long long kTimeoutNs = 4000000000ull;

// shared memory layout (dynamic, 1024-byte aligned base)
constexpr int kOffStage = 0;
constexpr int kOffWext = kOffStage + kStages * kStageBytes;           // [heads][8 x 64] fp16, 1 KB each
constexpr int kOffBlob(int heads) { return kOffWext + heads * 1024; }  // 2 record blocks
constexpr int kOffE(int heads) { return kOffBlob(heads) + 2 * kBlobMax; }
constexpr int kOffBar(int heads) { return kOffE(heads) + kConsumers * 16 * kEPad * 4; }
constexpr int kSmemBytes(int heads) { return kOffBar(heads) + 128 + 1024; }  // + barriers + alignment slack

__device__ int g_tc_error = 0;

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return uint32_t(__cvta_generic_to_shared(p)); }
__device__ __forceinline__ uint64_t now_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
__device__ __forceinline__ void mbar_init(uint64_t* b, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(b)), "r"(count));
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* b, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(b)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* b) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(b)) : "memory");
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
// Bounded wait; false on timeout (flags raised) or when another warp of the CTA aborted.
__device__ __forceinline__ bool mbar_wait(uint64_t* b, uint32_t parity, volatile int* abort_flag) {
    if (mbar_test(b, parity)) return true;
    const uint64_t t0 = now_ns();
    for (;;) {
        if (mbar_test(b, parity)) return true;
        if (*abort_flag) return false;
        if (now_ns() - t0 > kTimeoutNs) {
            *abort_flag = 1;
            atomicExch(&g_tc_error, 1);
            return false;
        }
    }
}
// Wait used only to drain this CTA's own copies before it exits; bounded, ignores the abort flag.
__device__ __forceinline__ void mbar_drain(uint64_t* b, uint32_t parity) {
    const uint64_t t0 = now_ns();
    while (!mbar_test(b, parity))
        if (now_ns() - t0 > kTimeoutNs) {
            atomicExch(&g_tc_error, 2);
            return;
        }
}
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_u32(dst)),
                 "l"(src), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}
// 2-D TMA tile copy (box of the map) to shared memory
__device__ __forceinline__ void tma_tile(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
            "r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}
// TMA row gather: rows r0..r3 of the map (box one row high, x columns) to 4 consecutive smem rows
__device__ __forceinline__ void tma_gather4(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int4 r) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile::gather4.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, "
        "%4, %5, %6}], [%7];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(r.x), "r"(r.y), "r"(r.z), "r"(r.w), "r"(smem_u32(bar))
        : "memory");
}
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t (&r)[4]) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t (&r)[4]) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}
// D += A B, m16n8k16, fp16 operands, fp32 accumulators
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
__device__ __forceinline__ uint32_t pack_h2(float a, float b) {
    const __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&h);
}
__device__ __forceinline__ float2 unpack_h2(uint32_t u) {
    return __half22float2(*reinterpret_cast<const __half2*>(&u));
}
// byte offset of 16-byte chunk `c` of row `r` in a 128-byte-row tile with the 128-byte swizzle
__device__ __forceinline__ uint32_t swz(int r, int c) { return uint32_t(r * 128 + ((c ^ (r & 7)) << 4)); }

struct TcParams {
    const TcTile* tiles;
    const int32_t* srcs;
    const uint8_t* blob;
    int tile0, ntiles;
    int64_t dst_lo;
    const __half* xr;
    __half* out;
    int64_t ldxr, ldo;
    const float* w_e;  // [4, C] fp32 (fp16-representable values)
    int C, heads;
    int kcol, vcol;  // column offsets of K and V in their maps (0 when k / v have their own maps)
    float scale_log2;
};

__global__ void __launch_bounds__(kThreads, 1)
    attention_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                        const __grid_constant__ CUtensorMap tmV, const TcParams p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int heads = p.heads;
    uint8_t* wext = sm + kOffWext;
    uint8_t* blobs = sm + kOffBlob(heads);
    float* ebuf_all = reinterpret_cast<float*>(sm + kOffE(heads));
    uint64_t* bar = reinterpret_cast<uint64_t*>(sm + kOffBar(heads));
    uint64_t* full_h = bar;             // [kStages]
    uint64_t* empty_h = bar + kStages;  // [kStages]
    uint64_t* full_t = bar + 2 * kStages;
    uint64_t* empty_t = bar + 2 * kStages + 2;
    volatile int* abort_flag = reinterpret_cast<volatile int*>(bar + 2 * kStages + 4);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    // ---- set-up: barriers, -inf edge-term buffers, zeroed K/V slots, the edge weights as fp16 rows
    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) mbar_init(&full_h[s], 1), mbar_init(&empty_h[s], kConsumers);
        for (int s = 0; s < 2; ++s) mbar_init(&full_t[s], 1), mbar_init(&empty_t[s], kConsumers);
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    for (int i = threadIdx.x; i < kConsumers * 16 * kEPad; i += blockDim.x) ebuf_all[i] = -INFINITY;
    for (int i = threadIdx.x; i < kStages * kStageBytes / 16; i += blockDim.x)
        reinterpret_cast<uint4*>(sm + kOffStage)[i] = make_uint4(0, 0, 0, 0);
    // W_ext of head h: 8 rows of 64 fp16 = (W_e[:, 0], W_e[:, 1], W_e[:, 2], b_e) twice, swizzled
    for (int i = threadIdx.x; i < heads * 8 * 8; i += blockDim.x) {
        const int h = i / 64, row = (i / 8) % 8, ch = i % 8;  // 16-byte chunk ch of row `row`
        const float* w = p.w_e + size_t(row % 4) * p.C + h * kHD + ch * 8;
        uint4 u;
        u.x = pack_h2(w[0], w[1]), u.y = pack_h2(w[2], w[3]), u.z = pack_h2(w[4], w[5]), u.w = pack_h2(w[6], w[7]);
        *reinterpret_cast<uint4*>(wext + h * 1024 + swz(row, ch)) = u;
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    __syncthreads();

    if (warp == kConsumers) {
        // ================================================================ producer
        uint32_t hc = 0;  // head stages filled so far
        int tc = 0;       // tiles loaded so far
        int64_t last_round[kStages];
        for (int s = 0; s < kStages; ++s) last_round[s] = -1;
        int last_tile_round[2] = {-1, -1};
        bool ok = true;
        for (int ti = blockIdx.x; ti < p.ntiles && ok; ti += gridDim.x, ++tc) {
            const TcTile t = p.tiles[p.tile0 + ti];
            const int tb = tc & 1, tround = tc >> 1;
            ok = __all_sync(kFull, mbar_wait(&empty_t[tb], (tround & 1) ^ 1, abort_flag));
            if (!ok) break;
            if (lane == 0) {
                mbar_expect_tx(&full_t[tb], uint32_t(t.blob_bytes));
                bulk_g2s(blobs + tb * kBlobMax, p.blob + t.blob_off, uint32_t(t.blob_bytes), &full_t[tb]);
            }
            last_tile_round[tb] = tround;
            const int nsrc4 = (t.nsrc + 3) & ~3;
            int4 rows4 = make_int4(0, 0, 0, 0);
            const bool mine = 4 * lane < nsrc4;
            if (mine) rows4 = *reinterpret_cast<const int4*>(p.srcs + t.src_off + 4 * lane);
            const uint32_t bytes = uint32_t(kQBytes) + 2u * uint32_t(nsrc4) * 128u;
            const int qrow = int(t.row0 - p.dst_lo);
            for (int h = 0; h < heads; ++h, ++hc) {
                const int s = int(hc % kStages);
                const int64_t round = hc / kStages;
                ok = __all_sync(kFull, mbar_wait(&empty_h[s], uint32_t((round & 1) ^ 1), abort_flag));
                if (!ok) break;
                uint8_t* st = sm + kOffStage + s * kStageBytes;
                if (lane == 0) mbar_expect_tx(&full_h[s], bytes);
                __syncwarp();
                if (mine) {
                    tma_gather4(st + 4 * lane * 128, &tmK, &full_h[s], p.kcol + h * kHD, rows4);
                    tma_gather4(st + kKVBytes + 4 * lane * 128, &tmV, &full_h[s], p.vcol + h * kHD, rows4);
                }
                if (lane == 0) tma_tile(st + 2 * kKVBytes, &tmQ, &full_h[s], h * kHD, qrow);
                last_round[s] = round;
            }
        }
        // drain: every copy this warp issued has landed before the CTA may exit
        if (lane == 0) {
            for (int s = 0; s < kStages; ++s)
                if (last_round[s] >= 0) mbar_drain(&full_h[s], uint32_t(last_round[s] & 1));
            for (int s = 0; s < 2; ++s)
                if (last_tile_round[s] >= 0) mbar_drain(&full_t[s], uint32_t(last_tile_round[s] & 1));
        }
        return;
    }

    // ==================================================================== consumers
    const int g = lane >> 2, t4 = lane & 3;  // fragment coordinates: row group, column pair
    const int pr = lane >> 1, ph = lane & 1;  // edge passes: row of the block, parity of the edge index
    float* ebuf = ebuf_all + warp * 16 * kEPad;
    uint32_t hc = 0;
    int tc = 0;
    for (int ti = blockIdx.x; ti < p.ntiles; ti += gridDim.x, ++tc) {
        const TcTile t = p.tiles[p.tile0 + ti];
        const int tb = tc & 1;
        if (!__all_sync(kFull, mbar_wait(&full_t[tb], uint32_t((tc >> 1) & 1), abort_flag))) return;
        const uint8_t* bl = blobs + tb * kBlobMax;
        const uint16_t* roff = reinterpret_cast<const uint16_t*>(bl);
        const uint16_t* masks = reinterpret_cast<const uint16_t*>(bl + kTcMaskOff);
        const uint2* recs = reinterpret_cast<const uint2*>(bl + kTcEdgeOff);
        const int nb = (t.nrows + 15) >> 4;
        for (int h = 0; h < heads; ++h, ++hc) {
            const int s = int(hc % kStages);
            if (!__all_sync(kFull, mbar_wait(&full_h[s], uint32_t((hc / kStages) & 1), abort_flag))) return;
            const uint32_t kbase = smem_u32(sm + kOffStage + s * kStageBytes);
            const uint32_t vbase = kbase + kKVBytes, qbase = kbase + 2 * kKVBytes;
            const uint32_t wbase = smem_u32(wext + h * 1024);
            for (int rb = 0; rb < nb; ++rb) {
                if ((h * nb + rb) % kConsumers != warp) continue;
                const uint32_t nmask = masks[rb];
                // ---- Q fragments of rows [16 rb, 16 rb + 16)
                uint32_t qa[4][4];
                {
                    const int r = 16 * rb + (lane & 7) + ((lane >> 3) & 1) * 8;
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk) ldsm_x4(qbase + swz(r, 2 * kk + (lane >> 4)), qa[kk]);
                }
                // ---- qe = Q W_ext: (qe0, qe1 | qe2, qb) in lanes t4 = 0 | 1 (and again in 2 | 3)
                float ce[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
                for (int half = 0; half < 2; ++half) {
                    uint32_t b[4];
                    ldsm_x4(wbase + swz(lane & 7, 4 * half + (lane >> 3)), b);
                    mma16816(ce, qa[2 * half], b[0], b[1]);
                    mma16816(ce, qa[2 * half + 1], b[2], b[3]);
                }
                // ---- pass 1: edge terms of this lane's row (two lanes per row, alternate edges)
                const int grow = 16 * rb + pr;  // tile row of this lane in the edge passes
                const int e_beg = roff[grow], e_end = roff[grow + 1];
                {
                    const int la = (pr & 7) * 4;
                    const float a0 = __shfl_sync(kFull, ce[0], la), a2 = __shfl_sync(kFull, ce[2], la);
                    const float b0 = __shfl_sync(kFull, ce[1], la), b2 = __shfl_sync(kFull, ce[3], la);
                    const float c0 = __shfl_sync(kFull, ce[0], la + 1), c2 = __shfl_sync(kFull, ce[2], la + 1);
                    const float d0 = __shfl_sync(kFull, ce[1], la + 1), d2 = __shfl_sync(kFull, ce[3], la + 1);
                    const bool lo = pr < 8;
                    const float qe0 = (lo ? a0 : a2) * p.scale_log2, qe1 = (lo ? b0 : b2) * p.scale_log2;
                    const float qe2 = (lo ? c0 : c2) * p.scale_log2, qb = (lo ? d0 : d2) * p.scale_log2;
                    float* er = ebuf + pr * kEPad;
                    for (int e = e_beg + ph; e < e_end; e += 2) {
                        const uint2 rec = recs[e];
                        const float2 a01 = unpack_h2(rec.x >> 16 | (rec.y << 16));
                        const float a2v = __half2float(__ushort_as_half(uint16_t(rec.y >> 16)));
                        er[rec.x & 0xffff] = fmaf(qe0, a01.x, fmaf(qe1, a01.y, fmaf(qe2, a2v, qb)));
                    }
                }
                __syncwarp();
                // ---- S = Q K^T on the active column blocks; s = S scale + E; row maxima
                float sc[kNT][4];
                float mx0 = -INFINITY, mx1 = -INFINITY;
                const float* e_g = ebuf + g * kEPad + 2 * t4;
                const float* e_g8 = e_g + 8 * kEPad;
#pragma unroll
                for (int j = 0; j < kNT; ++j) {
                    if (!((nmask >> j) & 1)) continue;
                    sc[j][0] = sc[j][1] = sc[j][2] = sc[j][3] = 0.f;
#pragma unroll
                    for (int half = 0; half < 2; ++half) {
                        uint32_t b[4];
                        ldsm_x4(kbase + swz(8 * j + (lane & 7), 4 * half + (lane >> 3)), b);
                        mma16816(sc[j], qa[2 * half], b[0], b[1]);
                        mma16816(sc[j], qa[2 * half + 1], b[2], b[3]);
                    }
                    float2 ea = *reinterpret_cast<const float2*>(e_g + 8 * j);
                    float2 eb = *reinterpret_cast<const float2*>(e_g8 + 8 * j);
                    sc[j][0] = fmaf(sc[j][0], p.scale_log2, ea.x);
                    sc[j][1] = fmaf(sc[j][1], p.scale_log2, ea.y);
                    sc[j][2] = fmaf(sc[j][2], p.scale_log2, eb.x);
                    sc[j][3] = fmaf(sc[j][3], p.scale_log2, eb.y);
                    *reinterpret_cast<float2*>(ebuf + g * kEPad + 2 * t4 + 8 * j) = make_float2(sc[j][0], sc[j][1]);
                    *reinterpret_cast<float2*>(ebuf + (g + 8) * kEPad + 2 * t4 + 8 * j) =
                        make_float2(sc[j][2], sc[j][3]);
                    mx0 = fmaxf(mx0, fmaxf(sc[j][0], sc[j][1]));
                    mx1 = fmaxf(mx1, fmaxf(sc[j][2], sc[j][3]));
                }
                mx0 = fmaxf(mx0, __shfl_xor_sync(kFull, mx0, 1));
                mx0 = fmaxf(mx0, __shfl_xor_sync(kFull, mx0, 2));
                mx1 = fmaxf(mx1, __shfl_xor_sync(kFull, mx1, 1));
                mx1 = fmaxf(mx1, __shfl_xor_sync(kFull, mx1, 2));
                if (mx0 == -INFINITY) mx0 = 0.f;  // no edge in the row: every weight is 0
                if (mx1 == -INFINITY) mx1 = 0.f;
                // ---- weights p (fp16, the operand of O = P V) and l from the rounded weights
                uint32_t pf[kNT][2];
                float l0 = 0.f, l1 = 0.f;
#pragma unroll
                for (int j = 0; j < kNT; ++j) {
                    if (!((nmask >> j) & 1)) {
                        pf[j][0] = pf[j][1] = 0u;
                        continue;
                    }
                    pf[j][0] = pack_h2(ex2(sc[j][0] - mx0), ex2(sc[j][1] - mx0));
                    pf[j][1] = pack_h2(ex2(sc[j][2] - mx1), ex2(sc[j][3] - mx1));
                    const float2 u = unpack_h2(pf[j][0]), v = unpack_h2(pf[j][1]);
                    l0 += u.x + u.y;
                    l1 += v.x + v.y;
                }
                l0 += __shfl_xor_sync(kFull, l0, 1);
                l0 += __shfl_xor_sync(kFull, l0, 2);
                l1 += __shfl_xor_sync(kFull, l1, 1);
                l1 += __shfl_xor_sync(kFull, l1, 2);
                __syncwarp();
                // ---- pass 2: pa = sum of rounded weights x attributes per row; buffer back to -inf
                float pa0 = 0.f, pa1 = 0.f, pa2 = 0.f;
                {
                    const int la = (pr & 7) * 4;
                    const float m_lo = __shfl_sync(kFull, mx0, la), m_hi = __shfl_sync(kFull, mx1, la);
                    const float m = pr < 8 ? m_lo : m_hi;
                    float* er = ebuf + pr * kEPad;
                    for (int e = e_beg + ph; e < e_end; e += 2) {
                        const uint2 rec = recs[e];
                        const int sl = rec.x & 0xffff;
                        const float w = __half2float(__float2half_rn(ex2(er[sl] - m)));
                        const float2 a01 = unpack_h2(rec.x >> 16 | (rec.y << 16));
                        const float a2v = __half2float(__ushort_as_half(uint16_t(rec.y >> 16)));
                        pa0 = fmaf(w, a01.x, pa0), pa1 = fmaf(w, a01.y, pa1), pa2 = fmaf(w, a2v, pa2);
                        er[sl] = -INFINITY;
                    }
                    pa0 += __shfl_xor_sync(kFull, pa0, 1);
                    pa1 += __shfl_xor_sync(kFull, pa1, 1);
                    pa2 += __shfl_xor_sync(kFull, pa2, 1);
                }
                // ---- O = P V over the active 16-slot steps
                float o[8][4];
#pragma unroll
                for (int n = 0; n < 8; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
#pragma unroll
                for (int kk = 0; kk < kNT / 2; ++kk) {
                    if (!((nmask >> (2 * kk)) & 3)) continue;
                    const uint32_t a[4] = {pf[2 * kk][0], pf[2 * kk][1], pf[2 * kk + 1][0], pf[2 * kk + 1][1]};
                    const int vr = 16 * kk + (lane & 7) + ((lane >> 3) & 1) * 8;
#pragma unroll
                    for (int n = 0; n < 8; n += 2) {
                        uint32_t b[4];
                        ldsm_x4_t(vbase + swz(vr, n + (lane >> 4)), b);
                        mma16816(o[n], a, b[0], b[1]);
                        mma16816(o[n + 1], a, b[2], b[3]);
                    }
                }
                // ---- + [pa | l] [W_e ; b_e]: weights (pa0, pa1, pa2, l) as fp16 hi (columns 0-3) and lo
                // (columns 4-7) against W_ext rows (W_e[:, 0..2], b_e) twice
                {
                    const float x0 = __shfl_sync(kFull, pa0, 2 * g), x1 = __shfl_sync(kFull, pa1, 2 * g);
                    const float x2 = __shfl_sync(kFull, pa2, 2 * g);
                    const float y0 = __shfl_sync(kFull, pa0, 2 * g + 16), y1 = __shfl_sync(kFull, pa1, 2 * g + 16);
                    const float y2 = __shfl_sync(kFull, pa2, 2 * g + 16);
                    const bool odd = t4 & 1;
                    const float fa = odd ? x2 : x0, fb = odd ? l0 : x1;  // row g
                    const float ga = odd ? y2 : y0, gb = odd ? l1 : y1;  // row g + 8
                    uint32_t a[4];
                    if (t4 < 2) {
                        a[0] = pack_h2(fa, fb), a[1] = pack_h2(ga, gb);
                    } else {
                        const float2 hf = unpack_h2(pack_h2(fa, fb)), hg = unpack_h2(pack_h2(ga, gb));
                        a[0] = pack_h2(fa - hf.x, fb - hf.y), a[1] = pack_h2(ga - hg.x, gb - hg.y);
                    }
                    a[2] = a[3] = 0u;
#pragma unroll
                    for (int n = 0; n < 8; n += 2) {
                        uint32_t b[4];
                        ldsm_x4_t(wbase + swz(lane & 7, n + (lane >> 4)), b);
                        mma16816(o[n], a, b[0], b[1]);
                        mma16816(o[n + 1], a, b[2], b[3]);
                    }
                }
                // ---- out = T(T(O / l) + x_r), rows of this tile only
                const float i0 = l0 > 0.f ? 1.0f / l0 : 0.f, i1 = l1 > 0.f ? 1.0f / l1 : 0.f;
                const int r0 = 16 * rb + g, r1 = r0 + 8;
                const int64_t lr0 = int64_t(t.row0) + r0 - p.dst_lo, lr1 = lr0 + 8;
                const int c0 = h * kHD + 2 * t4;
#pragma unroll
                for (int n = 0; n < 8; ++n) {
                    const int c = c0 + 8 * n;
                    if (r0 < t.nrows) {
                        const float2 x = __half22float2(*reinterpret_cast<const __half2*>(p.xr + lr0 * p.ldxr + c));
                        const float u = rnd<__half>(rnd<__half>(o[n][0] * i0) + x.x);
                        const float v = rnd<__half>(rnd<__half>(o[n][1] * i0) + x.y);
                        *reinterpret_cast<__half2*>(p.out + lr0 * p.ldo + c) = __floats2half2_rn(u, v);
                    }
                    if (r1 < t.nrows) {
                        const float2 x = __half22float2(*reinterpret_cast<const __half2*>(p.xr + lr1 * p.ldxr + c));
                        const float u = rnd<__half>(rnd<__half>(o[n][2] * i1) + x.x);
                        const float v = rnd<__half>(rnd<__half>(o[n][3] * i1) + x.y);
                        *reinterpret_cast<__half2*>(p.out + lr1 * p.ldo + c) = __floats2half2_rn(u, v);
                    }
                }
                __syncwarp();
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty_h[s]);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty_t[tb]);
    }
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace

bool tc_attention_supported(int C, int heads, int head_dim) {
    return head_dim == kHD && heads >= 1 && heads <= kMaxHeads && C == heads * head_dim;
}

void attention_tc(const TcArgs& a, cudaStream_t s) {
    if (a.ntiles <= 0) return;
    if (!tc_attention_supported(a.C, a.heads, a.head_dim))
        fail(kUnsupported, "tensor-core attention: head_dim must be 64 and heads <= 32");
    if (!aligned16(a.q) || !aligned16(a.k) || !aligned16(a.v) || a.ldq % 8 || a.ldkv % 8)
        fail(kInvalidArgument, "tensor-core attention: q, k, v must be 16-byte aligned with ld a multiple of 8");
    if (reinterpret_cast<uintptr_t>(a.xr) & 3 || reinterpret_cast<uintptr_t>(a.out) & 3 || a.ldxr % 2 || a.ldo % 2)
        fail(kInvalidArgument, "tensor-core attention: x_r and out must be 4-byte aligned with even ld");
    if (a.ldq < a.C || a.ldkv < a.C || a.ldxr < a.C || a.ldo < a.C)
        fail(kInvalidArgument, "tensor-core attention: leading dimensions must be >= C");
    const CUtensorMap tq = tc::tensor_map_2d(a.q, a.n_q_rows, a.C, a.ldq, kTcRows, kHD, CU_TENSOR_MAP_SWIZZLE_128B);
    const CUtensorMap tk = tc::tensor_map_2d(a.k, a.n_src, a.C, a.ldkv, 1, kHD, CU_TENSOR_MAP_SWIZZLE_128B);
    const CUtensorMap tv = tc::tensor_map_2d(a.v, a.n_src, a.C, a.ldkv, 1, kHD, CU_TENSOR_MAP_SWIZZLE_128B);
    TcParams p{};
    p.tiles = a.tiles, p.srcs = a.srcs, p.blob = a.blob, p.tile0 = a.tile0, p.ntiles = a.ntiles, p.dst_lo = a.dst_lo;
    p.xr = a.xr, p.out = a.out, p.ldxr = a.ldxr, p.ldo = a.ldo, p.w_e = a.w_e, p.C = a.C, p.heads = a.heads;
    p.kcol = 0, p.vcol = 0;
    p.scale_log2 = 1.4426950408889634f / std::sqrt(float(a.head_dim));
    const int smem = kSmemBytes(a.heads);
    static std::atomic<uint64_t> configured{0};
    once_per_device(configured, [] {
        VB_CUDA(cudaFuncSetAttribute(attention_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     kSmemBytes(kMaxHeads)));
    });
    const int grid = std::min(a.ntiles, device_sm_count());
    attention_tc_kernel<<<grid, kThreads, smem, s>>>(tq, tk, tv, p);
    VB_LAUNCH();
}

int take_tc_error() {
    int e = 0, zero = 0;
    VB_CUDA(cudaMemcpyFromSymbol(&e, g_tc_error, sizeof(int)));
    if (e) VB_CUDA(cudaMemcpyToSymbol(g_tc_error, &zero, sizeof(int)));
    return e;
}

}  // namespace vb::k
