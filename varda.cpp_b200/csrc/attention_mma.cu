// Edge attention on the tensor cores (fp16, head_dim 64): persistent CTAs of 128 threads, two per SM,
// each taking destination tiles in turn.
//
// A tile (graph.cpp make_tiles) is a run of at most 128 consecutive destination rows with at most
// kMaxReal distinct sources ("slots", in source order) and kMaxEdges edges; each row's edge records
// are sorted by slot and carry the slot in place of the source. The tile's records are staged in shared
// memory once. Per head h (64 channels), with nr = the real slots rounded up to 16:
//   1. Q_h (the tile's rows), K_h and V_h (one 128-byte row per slot; missing rows zero) are gathered
//      into shared memory (cp.async) in the 128-byte-swizzled layout of the MMA descriptors; slots
//      nr .. nr + 3 of K_h and V_h hold the edge Linear's weight rows W_e[0..2] and bias b_e (fp16);
//   2. one thread issues S = Q_h K_h^T into TMEM (tcgen05.mma kind::f16, M = 128, N = nr + 16, K = 64),
//      which also yields <q, W_e[a]> and <q, b_e> in columns nr .. nr + 3; Q_h and K_h of the next head
//      start loading as soon as it completes;
//   3. thread r owns row r (TMEM lane r): it streams its row of S through registers, 16 columns at a
//      time, into a private shared-memory line and scores its own edges
//        s_e = (S[r][slot_e] + sum_a a_e[a] <q, W_e[a]> + <q, b_e>) / sqrt(64)   (log2 domain),
//      keeping them and their maximum m; then p_e = 2^(s_e - m) and
//        P[r][slot] = fp16(sum of p_e over the row's edges from that slot),   l = sum of those values,
//        P[r][nr + a] = fp16(sum_e p_e a_e[a]),   P[r][nr + 3] = fp16(l)
//      in a 128-byte-swizzled K-major tile;
//   4. one thread issues O = P V_h into TMEM (M = 128, N = 64, K = nr + 16; V_h read MN-major): the
//      softmax-weighted value sum plus the edge terms W_e (sum p a) + b_e l; V_h of the next head starts
//      loading as soon as it completes;
//   5. thread r: o = O[r] / l, out = T(T(o) + x_r) (zero in-degree: o = 0).
// The gather kernel's semantics (attention.cu) with the dot products and the value sums on the tensor
// cores (fp16 operands, fp32 accumulation): the softmax weights and their attribute sums are rounded to
// fp16 for the P V product, and W_e, b_e are taken in fp16 (the fp16 engine's edge weights are fp16
// values). Every wait is bounded (4 s of %globaltimer); on timeout the CTA sets its error flag (read
// with the other attention kernels' by take_attention_error), waits (bounded) once more for the MMAs
// it issued, frees its TMEM and returns.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <string>

#include "common.h"
#include "dev.cuh"
#include "kernels.cuh"

namespace vb::k {

using namespace vb::d;

namespace {

constexpr int kRows = 128;     // MMA M: tile rows (TMEM lanes), one thread each
constexpr int kMaxReal = 112;  // distinct sources per tile
constexpr int kSlots = 128;    // MMA N of S at most: real slots rounded up to 16, then 16 (4 edge-weight rows)
constexpr int kMaxEdges = 1024;
constexpr int kHD = 64;        // head_dim: one 128-byte swizzle atom
constexpr int kThreads = kRows;
constexpr int kStage = 20;     // floats per thread in the S staging lines (16 + 4: conflict-free v4 stores)
constexpr unsigned long long kTimeoutNs = 4000000000ull;
constexpr uint32_t kTmemCols = 256;  // S: kSlots columns, O: 64 columns at kOcol
constexpr uint32_t kOcol = kSlots;

// shared memory: Q, K, V (16 KB each), P (2 atoms), the S staging lines, the tile's edge records and
// scores, the per-slot source offsets, two mbarriers and the TMEM address: under half of an SM's
constexpr int kQ = kRows * 128, kKV = kSlots * 128, kP = kRows * 2 * kSlots;
constexpr int kSst = kThreads * kStage * 4, kE = kMaxEdges * 16, kSe = kMaxEdges * 4, kOff = kMaxReal * 8;
constexpr int kSmem = 1024 + kQ + 2 * kKV + kP + kSst + kE + kSe + kOff + 32;
static_assert(kQ % 1024 == 0 && kKV % 1024 == 0 && kP % 1024 == 0, "swizzle atoms must stay 1024-byte aligned");
static_assert(2 * (kSmem + 1024) <= 233472, "two CTAs per SM");

__device__ int g_mma_error = 0;

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return uint32_t(__cvta_generic_to_shared(p)); }
__device__ __forceinline__ uint64_t now_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
__device__ __forceinline__ bool mbar_test(uint32_t b, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(ok)
        : "r"(b), "r"(parity)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ bool mbar_wait(uint32_t b, uint32_t parity) {
    if (mbar_test(b, parity)) return true;
    const uint64_t t0 = now_ns();
    while (!mbar_test(b, parity))
        if (now_ns() - t0 > kTimeoutNs) return false;
    return true;
}
__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
// 16-byte global -> shared copy (zero fill when !valid: nothing is read)
__device__ __forceinline__ void cp16(uint32_t dst, const void* src, bool valid) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(valid ? 16 : 0) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// byte offset of 16-byte chunk c of row i in a 128-byte-swizzled [rows x 128 B] block
__device__ __forceinline__ uint32_t sw128(int i, int c) { return uint32_t(i * 128 + ((c ^ (i & 7)) << 4)); }

// Shared-memory matrix descriptor, 128-byte swizzle: K-major tiles (8-row groups 1024 bytes apart), and
// the MN-major V operand (one 64-element row per K index, 8-row groups 1024 bytes apart: the same
// physical layout, the major-ness is in the instruction descriptor).
__device__ __forceinline__ uint64_t sdesc(uint32_t saddr) {
    uint64_t d = 0;
    d |= uint64_t((saddr & 0x3FFFF) >> 4);
    d |= uint64_t(1) << 16;           // leading byte offset (unused: one swizzle atom across)
    d |= uint64_t(1024 >> 4) << 32;   // stride byte offset
    d |= uint64_t(1) << 46;           // descriptor version (sm_100)
    d |= uint64_t(2) << 61;           // SWIZZLE_128B
    return d;
}
// kind::f16 instruction descriptor: fp16 A and B, fp32 D, M = 128, N; B MN-major when b_mn
__device__ __forceinline__ uint32_t idesc(uint32_t n, bool b_mn) {
    return (1u << 4) | (b_mn ? (1u << 16) : 0u) | ((n >> 3) << 17) | (uint32_t(kRows >> 4) << 24);
}
__device__ __forceinline__ void mma(uint32_t d, uint64_t a, uint64_t b, uint32_t id, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d),
        "l"(a), "l"(b), "r"(id), "r"(acc));
}
__device__ __forceinline__ void mma_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
        "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    // the registers are in-out operands of the wait, so no use of them is scheduled before it
    asm volatile("tcgen05.wait::ld.sync.aligned;"
                 : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                   "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                   "+r"(r[15]), "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]),
                   "+r"(r[22]), "+r"(r[23]), "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]),
                   "+r"(r[29]), "+r"(r[30]), "+r"(r[31])
                 :
                 : "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;"
                 : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                   "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                   "+r"(r[15])
                 :
                 : "memory");
}

__global__ void __launch_bounds__(kThreads, 2) attention_mma_kernel(TileArgs a, float scale_log2) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* Qs = sm;
    uint8_t* Ks = Qs + kQ;
    uint8_t* Vs = Ks + kKV;
    uint8_t* Ps = Vs + kKV;
    float* Sst = reinterpret_cast<float*>(Ps + kP);
    float4* Es = reinterpret_cast<float4*>(Sst + kThreads * kStage);
    float* Se = reinterpret_cast<float*>(Es + kMaxEdges);
    int64_t* koff = reinterpret_cast<int64_t*>(Se + kMaxEdges);
    uint64_t* bars = reinterpret_cast<uint64_t*>(koff + kMaxReal);  // [0] S done, [1] O done
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2);

    const int tid = threadIdx.x, warp = tid >> 5, r = tid;
    const int heads = a.heads, C = a.C;
    if (tid == 0) {
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_u32(&bars[0])));
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_u32(&bars[1])));
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(kTmemCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    fence_before();
    __syncthreads();
    fence_after();
    const uint32_t tmem = *tmem_slot;
    const uint32_t lane_addr = uint32_t(warp * 32) << 16;  // this warp's TMEM lane quarter
    float* st = Sst + tid * kStage;

    bool ok = true;
    int pend = -1;  // the barrier a timed-out wait was on
    uint32_t pend_par = 0;
    uint32_t g = 0;  // heads done by this CTA: the barriers' phase
    for (int t = int(blockIdx.x); t < a.ntiles && ok; t += int(gridDim.x)) {
        const int4 tl = __ldg(a.tiles + a.tile0 + t);  // row0, nrows, src0, nsrc
        const int nsrc = tl.w, nr = (nsrc + 15) & ~15, nsp = nr + 16;
        const int e0 = __ldg(a.row_ptr + tl.x), ne = __ldg(a.row_ptr + tl.x + tl.y) - e0;
        const bool live = r < tl.y;
        const int64_t lr = int64_t(tl.x + r) - a.dst_lo;  // local q / x_r / out row
        int e_beg = 0, e_end = 0;
        if (live) e_beg = __ldg(a.row_ptr + tl.x + r) - e0, e_end = __ldg(a.row_ptr + tl.x + r + 1) - e0;

        // operand loads of head h: Q_h and K_h (with its edge-weight rows), or V_h (likewise)
        auto load_qk = [&](int h) {
            const int ch0 = h * kHD;
            for (int i = tid; i < kRows * 8; i += kThreads) {
                const int row = i >> 3, c = i & 7;
                const bool in = row < tl.y;
                const __half* src = a.q + (in ? (int64_t(tl.x + row) - a.dst_lo) * a.ldq : 0) + ch0 + c * 8;
                cp16(smem_u32(Qs + sw128(row, c)), src, in);
            }
            for (int i = tid; i < nr * 8; i += kThreads) {
                const int s = i >> 3, c = i & 7;
                const bool in = s < nsrc;
                cp16(smem_u32(Ks + sw128(s, c)), a.k + (in ? koff[s] : 0) + ch0 + c * 8, in);
            }
            cp_commit();
        };
        auto load_v = [&](int h) {
            const int ch0 = h * kHD;
            for (int i = tid; i < nr * 8; i += kThreads) {
                const int s = i >> 3, c = i & 7;
                const bool in = s < nsrc;
                cp16(smem_u32(Vs + sw128(s, c)), a.v + (in ? koff[s] : 0) + ch0 + c * 8, in);
            }
            cp_commit();
        };
        // rows nr .. nr + 15 of K_h or V_h: W_e[0..2], b_e (fp16), then zeros; one 16-byte chunk per thread
        auto edge_rows = [&](int h, uint8_t* dst) {
            const int row = tid >> 3, c = tid & 7;
            uint4 u = make_uint4(0, 0, 0, 0);
            if (row < 4) {
                const float4* w = reinterpret_cast<const float4*>(a.w_e + int64_t(row) * C + h * kHD + c * 8);
                const float4 x = __ldg(w), y = __ldg(w + 1);
                const __half2 h2[4] = {__floats2half2_rn(x.x, x.y), __floats2half2_rn(x.z, x.w),
                                       __floats2half2_rn(y.x, y.y), __floats2half2_rn(y.z, y.w)};
                u = *reinterpret_cast<const uint4*>(h2);
            }
            *reinterpret_cast<uint4*>(dst + sw128(nr + row, c)) = u;
        };

        // the tile's records and source offsets, then head 0's operands
        for (int i = tid; i < ne; i += kThreads) cp16(smem_u32(Es + i), a.edges + e0 + i, true);
        cp_commit();
        for (int i = tid; i < nsrc; i += kThreads) koff[i] = int64_t(__ldg(a.srcs + tl.z + i)) * a.ldkv;
        __syncthreads();
        load_qk(0);
        load_v(0);
        edge_rows(0, Ks);
        edge_rows(0, Vs);

        for (int h = 0; h < heads; ++h, ++g) {
            cp_wait_all();
            fence_async_smem();
            fence_before();
            __syncthreads();
            fence_after();
            if (tid == 0) {  // S = Q_h K_h^T
                const uint64_t da = sdesc(smem_u32(Qs)), db = sdesc(smem_u32(Ks));
                const uint32_t id = idesc(uint32_t(nsp), false);
#pragma unroll
                for (int k = 0; k < kHD / 16; ++k) mma(tmem, da + uint64_t(2 * k), db + uint64_t(2 * k), id, k ? 1u : 0u);
                mma_commit(smem_u32(&bars[0]));
            }
            // this row's x_r slice, consumed by the epilogue
            uint4 xr[8];
            if (live) {
                const uint4* xp = reinterpret_cast<const uint4*>(a.xr + lr * a.ldxr + h * kHD);
#pragma unroll
                for (int c = 0; c < 8; ++c) xr[c] = __ldg(xp + c);
            }
            bool w_ok = mbar_wait(smem_u32(&bars[0]), g & 1u);
            if (!w_ok && pend < 0) pend = 0, pend_par = g & 1u;
            ok = __syncthreads_and(w_ok) != 0;
            if (!ok) break;
            fence_after();
            if (h + 1 < heads) {  // Q and K are free again
                load_qk(h + 1);
                edge_rows(h + 1, Ks);
            }

            // pass 1: <q, W_e[a]>, <q, b_e> from the edge-weight columns, then the edges' scores
            float qe0, qe1, qe2, qb;
            {
                uint32_t v[16];
                __syncwarp();
                tmem_ld16(tmem + lane_addr + uint32_t(nr), v);
                qe0 = __uint_as_float(v[0]), qe1 = __uint_as_float(v[1]), qe2 = __uint_as_float(v[2]);
                qb = __uint_as_float(v[3]);
            }
            float m = -INFINITY;
            {
                int e = e_beg;
                for (int c0 = 0; c0 < nr; c0 += 16) {
                    uint32_t v[16];
                    __syncwarp();  // tcgen05.ld is warp-collective
                    tmem_ld16(tmem + lane_addr + uint32_t(c0), v);
#pragma unroll
                    for (int j = 0; j < 4; ++j)
                        *reinterpret_cast<uint4*>(st + 4 * j) = make_uint4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
                    for (; e < e_end; ++e) {
                        const float4 rec = Es[e];
                        const int slot = __float_as_int(rec.w);
                        if (slot >= c0 + 16) break;
                        const float se = fmaf(qe2, rec.z, fmaf(qe1, rec.y, qe0 * rec.x));
                        const float s = ((st[slot - c0] + se) + qb) * scale_log2;
                        Se[e] = s;
                        m = fmaxf(m, s);
                    }
                }
            }
            // pass 2: the P row (zeroed first), l, the attribute sums
            {
                for (int at = 0; at * 64 < nsp; ++at)
#pragma unroll
                    for (int c = 0; c < 8; ++c) *reinterpret_cast<uint4*>(Ps + at * (kRows * 128) + sw128(r, c)) = make_uint4(0, 0, 0, 0);
                auto put = [&](int slot, __half v) {
                    const int at = slot >> 6, k = slot & 63;
                    *reinterpret_cast<__half*>(Ps + at * (kRows * 128) + sw128(r, k >> 3) + (k & 7) * 2) = v;
                };
                float l = 0.f, pa0 = 0.f, pa1 = 0.f, pa2 = 0.f, run = 0.f;
                int run_slot = -1;
                for (int e = e_beg; e < e_end; ++e) {
                    const float4 rec = Es[e];
                    const int slot = __float_as_int(rec.w);
                    const float p = ex2(Se[e] - m);
                    pa0 = fmaf(p, rec.x, pa0), pa1 = fmaf(p, rec.y, pa1), pa2 = fmaf(p, rec.z, pa2);
                    if (slot != run_slot) {
                        if (run_slot >= 0) {
                            const __half hp = __float2half_rn(run);
                            l += __half2float(hp);
                            put(run_slot, hp);
                        }
                        run_slot = slot, run = 0.f;
                    }
                    run += p;
                }
                if (run_slot >= 0) {
                    const __half hp = __float2half_rn(run);
                    l += __half2float(hp);
                    put(run_slot, hp);
                }
                put(nr, __float2half_rn(pa0));
                put(nr + 1, __float2half_rn(pa1));
                put(nr + 2, __float2half_rn(pa2));
                put(nr + 3, __float2half_rn(l));
                st[16] = l;  // kept for the epilogue
            }
            fence_async_smem();
            fence_before();
            __syncthreads();
            fence_after();
            if (tid == 0) {  // O = P V_h
                const uint32_t id = idesc(uint32_t(kHD), true);
                const uint64_t dv = sdesc(smem_u32(Vs));
                for (int j = 0; j < nsp / 16; ++j) {
                    const uint64_t dp = sdesc(smem_u32(Ps + (j >> 2) * (kRows * 128))) + uint64_t(2 * (j & 3));
                    mma(tmem + kOcol, dp, dv + uint64_t(j * (2048 >> 4)), id, j ? 1u : 0u);
                }
                mma_commit(smem_u32(&bars[1]));
            }
            w_ok = mbar_wait(smem_u32(&bars[1]), g & 1u);
            if (!w_ok && pend < 0) pend = 1, pend_par = g & 1u;
            ok = __syncthreads_and(w_ok) != 0;
            if (!ok) break;
            fence_after();
            if (h + 1 < heads) {  // V is free again
                load_v(h + 1);
                edge_rows(h + 1, Vs);
            }
            {  // epilogue
                uint32_t o0[32], o1[32];
                __syncwarp();
                tmem_ld32(tmem + lane_addr + kOcol, o0);
                tmem_ld32(tmem + lane_addr + kOcol + 32, o1);
                if (live) {
                    const float l = st[16];
                    const float inv = e_end > e_beg ? 1.0f / l : 0.f;
                    uint4 outv[8];
#pragma unroll
                    for (int c = 0; c < 8; ++c) {
                        const __half2* hx = reinterpret_cast<const __half2*>(&xr[c]);
                        __half2 ho[4];
#pragma unroll
                        for (int j = 0; j < 4; ++j) {
                            const int ch = c * 8 + 2 * j;
                            const float ax = __uint_as_float(ch < 32 ? o0[ch] : o1[ch - 32]);
                            const float ay = __uint_as_float(ch + 1 < 32 ? o0[ch + 1] : o1[ch - 31]);
                            const float2 x = __half22float2(hx[j]);
                            ho[j] = __floats2half2_rn(rnd<__half>(rnd<__half>(ax * inv) + x.x),
                                                      rnd<__half>(rnd<__half>(ay * inv) + x.y));
                        }
                        outv[c] = *reinterpret_cast<const uint4*>(ho);
                    }
                    uint4* op = reinterpret_cast<uint4*>(a.out + lr * a.ldo + h * kHD);
#pragma unroll
                    for (int c = 0; c < 8; ++c) op[c] = outv[c];
                }
            }
            fence_before();
        }
        __syncthreads();  // the tile's records and offsets are no longer read
    }
    cp_wait_all();  // no copy may land after the CTA has left
    if (pend >= 0) mbar_wait(smem_u32(&bars[pend]), pend_par);  // the MMAs issued complete before the TMEM is freed
    if (!ok && tid == 0) atomicExch(&g_mma_error, 1);
    fence_before();
    __syncthreads();
    fence_after();
    if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
}

}  // namespace

int take_mma_error() {
    int e = 0, zero = 0;
    VB_CUDA(cudaMemcpyFromSymbol(&e, g_mma_error, sizeof(int)));
    if (e) VB_CUDA(cudaMemcpyToSymbol(g_mma_error, &zero, sizeof(int)));
    return e;
}

int mma_max_src() { return kMaxReal; }
int mma_max_edges() { return kMaxEdges; }
int mma_max_rows() { return kRows; }
bool mma_supported(int C, int head_dim) { return head_dim == kHD && C % kHD == 0; }

void attention_mma(const TileArgs& a, float scale_log2, cudaStream_t s) {
    if (a.ntiles <= 0) return;
    if (!mma_supported(a.C, a.head_dim)) fail(kUnsupported, "tensor-core attention: head_dim must be 64");
    auto al16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
    if (a.ldq % 8 || a.ldkv % 8 || a.ldxr % 8 || a.ldo % 8 || !al16(a.q) || !al16(a.k) || !al16(a.v) || !al16(a.xr) ||
        !al16(a.out) || !al16(a.w_e) || a.C % 4)
        fail(kUnsupported, "tensor-core attention: operands must be 16-byte aligned (leading dimensions multiples of 8)");
    static std::atomic<uint64_t> cfg{0};
    once_per_device(cfg, [] {
        VB_CUDA(cudaFuncSetAttribute(attention_mma_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem));
        VB_CUDA(cudaFuncSetAttribute(attention_mma_kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                                     int(cudaSharedmemCarveoutMaxShared)));
    });
    const int grid = std::min(a.ntiles, 2 * device_sm_count());  // persistent: two CTAs per SM
    attention_mma_kernel<<<unsigned(grid), kThreads, kSmem, s>>>(a, scale_log2);
    VB_LAUNCH();
}

}  // namespace vb::k
