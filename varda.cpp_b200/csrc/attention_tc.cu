// Tile-sparse tensor-core edge attention (fp16, head_dim 64): the processor graph's attention as small
// matrix products per tile of destination rows.
//
// A tile (graph.h, make_tc_tiles) is up to 64 consecutive destination rows whose edges reach at most
// 128 distinct sources, numbered by first appearance ("slots"). For each head h and 16-row block of
// the tile (a task), with the block's queries Q_h [16 x 64], the tile's K_h, V_h [128 x 64] and the
// edge attributes a_e:
//   S   = Q_h K_h^T over the 8-slot column blocks that hold edges of the block    (tensor cores)
//   s_e = (S[r, slot_e] + <W_e^T q_r, a_e> + <q_r, b_e>) / sqrt(d), for every edge e = (r, slot_e),
//         -inf at the other positions (the log2 domain throughout, ex2)
//   online over the column blocks, two at a time (one 16-slot step): p = 2^(s - m) relative to a
//   reference maximum m per row that is raised (and the sums rescaled) only when a score exceeds it
//   by more than 2^8; l = sum p, pa = sum p a_e (fp32), O += P V_h with P in fp16 (tensor cores)
//   O  += [pa | l] [W_e ; b_e]   (tensor cores; pa and l carried as fp16 hi + lo parts)
//   out = T(T(O / l) + x_r)      (zero in-degree: O = 0, l = 0 -> out = x_r exactly)
// which is the reference's per-destination softmax over (k_j + e_ij) with values (v_j + e_ij),
// e_ij = W_e a_ij + b_e (cpu/kernels.cpp:98-158, backend_cpu.cpp:333-340), in fp32 except that the
// attention weights enter the value sums as fp16 (relative rounding <= 2^-11).
//
// The products are warp-level tensor-core instructions (mma.sync m16n8k16, fp16 in, fp32 accumulate):
// the score matrix of a 16-row block is sparse (about 14 edges per row among the tile's 128 slots),
// and only the column blocks that hold an edge of the block are multiplied and exponentiated, which
// a 16-row granularity allows and the 128-row tiles of tcgen05 do not. The positions of the edges in
// a lane's fragments come from the tile's record block (per step and lane, each position's edge
// index in its row), so no lane searches for its edges.
//
// Kernel layout: persistent CTAs of 8 consumer warps and 4 producer warps.
//   producers  per tile: the record block by one bulk copy (cp.async.bulk); per head: K_h and V_h rows
//              of the tile's sources and the tile's Q_h rows by 16-byte asynchronous copies (cp.async:
//              on B200 four warps of them gather scattered 128-byte rows at about 22 bytes per clock per
//              SM, against 12 for TMA row gathers), completing on the stage's mbarrier, into a 5-deep
//              (more than 16 heads: 4-deep) ring of head stages laid out with the 128-byte swizzle
//              (full / empty mbarriers).
//   consumers  a tile of nb row blocks has nb x heads tasks (head-major); the warps take a stage's tasks
//              from its counter as they reach it, so they spread over the stages in the ring. Per task:
//              x_r read ahead; Q fragments; qe = Q W_ext (the edge weights as 8 extra columns: per row
//              <W_e^T q, a>, <q, b_e>); per 16-slot step the scores, the online weights and O += P V;
//              the W_e / b_e terms; out.
// Every mbarrier wait is bounded (4 s of %globaltimer): on timeout the CTA sets the device error flag
// (read by take_attention_error), stops, and the producers drain their own copies before returning.
#include <cmath>
#include <cstdlib>
#include <string>

#include "common.h"
#include "dev.cuh"
#include "kernels.cuh"

namespace vb::k {

using namespace vb::d;

namespace {

constexpr int kHD = 64;  // head_dim
// head stages in the ring: 5 where the shared memory holds them (heads <= 16: 200 KB of stages + the
// edge weights), else 4 (5 measured 1.067 against 1.107 ms on C2)
constexpr int kConsumers = 8, kProducers = 4;
constexpr int kThreads = 32 * (kConsumers + kProducers);
// per-thread registers after the split: the launch gives every thread 168 (65536 / 384, rounded down to
// a multiple of 8); one producer warpgroup at kProducerRegs and two consumer warpgroups at kConsumerRegs
// use exactly the CTA's 384 x 168
constexpr int kLaunchRegs = 168, kProducerRegs = 56, kConsumerRegs = 224;
static_assert(kConsumers == 8 && kProducers == 4, "the register split assumes 2 consumer and 1 producer warpgroups");
static_assert(32 * (kProducers * kProducerRegs + kConsumers * kConsumerRegs) <= kThreads * kLaunchRegs,
              "register split over the CTA's registers");
constexpr int kKVBytes = kTcMaxSrc * kHD * 2;  // 16 KB
constexpr int kQBytes = kTcRows * kHD * 2;     // 8 KB
constexpr int kStageBytes = 2 * kKVBytes + kQBytes;
constexpr int kBlobMax = kTcMaskOff + 32 * kTcMaxChunks;  // the part of a record block staged in shared memory
constexpr int kMaxHeads = 32;
constexpr unsigned long long kTimeoutNs = 4000000000ull;
constexpr float kSlack = 8.0f;  // log2 headroom of the weights over their reference maximum

// shared memory layout (dynamic, 1024-byte aligned base)
constexpr int kOffStage = 0;
constexpr int kSmemLimit = 232448;
constexpr int kOffWext(int st) { return kOffStage + st * kStageBytes; }                 // [heads][8 x 64] fp16, 1 KB each
constexpr int kOffBlob(int st, int heads) { return kOffWext(st) + heads * 1024; }  // 2 record blocks
constexpr int kOffBar(int st, int heads) { return kOffBlob(st, heads) + 2 * kBlobMax; }
constexpr int kSmemBytes(int st, int heads) { return kOffBar(st, heads) + 256 + 1024; }  // + barriers + slack
// the 256-byte barrier area: 2 st + 6 mbarriers, then the abort flag, 2 tile indices and st task counters
static_assert((2 * 5 + 6) * 8 + 4 * (1 + 2 + 5) <= 256, "barrier area");
static_assert(kSmemBytes(4, kMaxHeads) <= kSmemLimit && kSmemBytes(5, 16) <= kSmemLimit, "shared memory budget");
constexpr int stages_for(int heads) { return kSmemBytes(5, heads) <= kSmemLimit ? 5 : 4; }

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
// Bounded wait (limit_ns of %globaltimer); false on timeout (flags raised) or when another warp of the
// CTA aborted.
__device__ __forceinline__ bool mbar_wait(uint64_t* b, uint32_t parity, volatile int* abort_flag,
                                          unsigned long long limit_ns) {
    if (mbar_test(b, parity)) return true;
    const uint64_t t0 = now_ns();
    for (;;) {
        if (mbar_test(b, parity)) return true;
        if (*abort_flag) return false;
        if (now_ns() - t0 > limit_ns) {
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
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
// arrives on the barrier once this thread's cp.async copies so far have landed
__device__ __forceinline__ void cp_async_arrive(uint64_t* b) {
    asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(b)) : "memory");
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
    const __half *q, *k, *v, *xr;
    __half* out;
    int64_t ldq, ldkv, ldxr, ldo, n_q_rows;
    const float* w_e;  // [4, C] fp32 (fp16-representable values)
    int C, heads;
    float scale_log2;
    unsigned long long wait_ns;  // limit of every wait (kTimeoutNs; shorter in the failure-path test)
    int withhold;                // failure-path test only: CTA 0 leaves its first head stage unfilled
    unsigned* sched;             // dynamic tile order: [tiles handed out, CTAs done], zero between launches; or null
};

template <int kStages>
__global__ void __launch_bounds__(kThreads, 1) attention_tc_kernel(const TcParams p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int heads = p.heads;
    uint8_t* wext = sm + kOffWext(kStages);
    uint8_t* blobs = sm + kOffBlob(kStages, heads);
    uint64_t* bar = reinterpret_cast<uint64_t*>(sm + kOffBar(kStages, heads));
    uint64_t* full_h = bar;             // [kStages]
    uint64_t* empty_h = bar + kStages;  // [kStages]
    uint64_t* full_t = bar + 2 * kStages;
    uint64_t* empty_t = bar + 2 * kStages + 2;
    uint64_t* tready = bar + 2 * kStages + 4;  // the tile index of record-block buffer b is in tidx[b]
    volatile int* abort_flag = reinterpret_cast<volatile int*>(bar + 2 * kStages + 6);
    volatile int* tidx = abort_flag + 1;
    int* tgrab = const_cast<int*>(abort_flag) + 3;  // [kStages] task counters of the head stages
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    // ---- set-up: barriers, zeroed stages (every slot holds finite values), the edge weights as fp16 rows
    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) mbar_init(&full_h[s], 32 * kProducers), mbar_init(&empty_h[s], kConsumers);
        for (int s = 0; s < 2; ++s)
            mbar_init(&full_t[s], 1), mbar_init(&empty_t[s], kConsumers), mbar_init(&tready[s], 1);
        *abort_flag = 0;
        for (int s = 0; s < kStages; ++s) tgrab[s] = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
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

    if (warp >= kConsumers) {
        // ================================================================ producers
        // registers: the producer warpgroup gives back to the consumers' (kProducerRegs + 2 x
        // kConsumerRegs = 3 x the 168 of the launch: the split adds up to what the CTA holds)
        asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kProducerRegs));
        const int pl = threadIdx.x - 32 * kConsumers;  // 0 .. 32 kProducers - 1
        const int prow = pl >> 3, pch = pl & 7;        // 16 rows x 8 chunks of 16 bytes per round
        constexpr int kRows = 4 * kProducers;          // rows per round
        constexpr int kRounds = kTcMaxSrc / kRows;
        uint32_t hc = 0;
        int tc = 0;
        // per record-block buffer: the round of its barrier's last phase (a copy, or the end marker)
        int blob_round[2] = {-1, -1};
        bool ok = true;
        // Tile order: static (tile blockIdx.x + i gridDim.x), or dynamic (p.sched): the first tile is
        // blockIdx.x, each further one gridDim.x + the next index of the launch's counter, fetched by
        // producer thread 0 and published to the other producers (tready) and the consumers (full_t).
        for (tc = 0; ok; ++tc) {
            const int tb = tc & 1;
            ok = __all_sync(kFull, mbar_wait(&empty_t[tb], ((tc >> 1) & 1) ^ 1, abort_flag, p.wait_ns));
            if (!ok) break;
            if (pl == 0) {
                tidx[tb] = tc == 0 || !p.sched ? int(blockIdx.x + tc * gridDim.x)
                                                : int(gridDim.x + atomicAdd(p.sched, 1u));
                mbar_arrive(&tready[tb]);
            }
            ok = __all_sync(kFull, mbar_wait(&tready[tb], uint32_t((tc >> 1) & 1), abort_flag, p.wait_ns));
            if (!ok) break;
            const int ti = tidx[tb];
            blob_round[tb] = tc >> 1;  // the last phase of this buffer's barrier that anything completes
            if (ti >= p.ntiles) {  // no more tiles: the consumers read the index past the end and stop
                if (pl == 0) mbar_arrive(&full_t[tb]);
                break;
            }
            const TcTile t = p.tiles[p.tile0 + ti];
            if (pl == 0) {
                // the tile's block heads and position masks (its attributes stay in global memory)
                mbar_expect_tx(&full_t[tb], uint32_t(t.attr_off));
                bulk_g2s(blobs + tb * kBlobMax, p.blob + t.blob_off, uint32_t(t.attr_off), &full_t[tb]);
            }
            // this lane's source rows of the tile (rows prow + kRows i), -1 past the tile's sources
            int srow[kRounds];
#pragma unroll
            for (int i = 0; i < kRounds; ++i) {
                const int r = prow + kRows * i;
                srow[i] = r < t.nsrc ? __ldg(p.srcs + t.src_off + r) : -1;
            }
            const int nqr = (t.nrows + 15) & ~15;
            const int64_t qrow = int64_t(t.row0) - p.dst_lo;
            for (int h = 0; h < heads; ++h, ++hc) {
                const int s = int(hc % kStages);
                ok = __all_sync(kFull, mbar_wait(&empty_h[s], uint32_t(((hc / kStages) & 1) ^ 1), abort_flag, p.wait_ns));
                if (!ok) break;
                const uint32_t st = smem_u32(sm + kOffStage + s * kStageBytes);
                const int col = h * kHD + pch * 8;
                if (p.withhold && blockIdx.x == 0 && hc == 0) continue;  // no copies, no arrival: the wait runs out
#pragma unroll
                for (int i = 0; i < kRounds; ++i) {
                    if (srow[i] < 0) continue;
                    const int r = prow + kRows * i;
                    cp_async16(st + swz(r, pch), p.k + int64_t(srow[i]) * p.ldkv + col);
                    cp_async16(st + kKVBytes + swz(r, pch), p.v + int64_t(srow[i]) * p.ldkv + col);
                }
#pragma unroll
                for (int i = 0; i < kTcRows / kRows; ++i) {
                    const int r = prow + kRows * i;
                    if (r < nqr && qrow + r < p.n_q_rows)
                        cp_async16(st + 2 * kKVBytes + swz(r, pch), p.q + (qrow + r) * p.ldq + col);
                }
                cp_async_arrive(&full_h[s]);
            }
        }
        // drain: every copy of this thread has landed before the CTA may exit
        asm volatile("cp.async.wait_all;" ::: "memory");
        if (pl == 0) {
            for (int b = 0; b < 2; ++b)
                if (blob_round[b] >= 0) mbar_drain(&full_t[b], uint32_t(blob_round[b] & 1));
            if (p.sched) {  // the last CTA to finish zeroes the counter for the next launch
                __threadfence();
                if (atomicAdd(p.sched + 1, 1u) == gridDim.x - 1) {
                    atomicExch(p.sched, 0u);
                    atomicExch(p.sched + 1, 0u);
                }
            }
        }
        return;
    }

    // ==================================================================== consumers
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kConsumerRegs));
    const int g = lane >> 2, t4 = lane & 3;  // fragment coordinates: row group, column pair
    uint32_t hc = 0;
    int tc = 0;
    // The tasks of a head stage (its 16-row blocks) go to whichever consumer warps reach the stage first:
    // each grabs block indices from the stage's counter until one is past the tile's blocks. Every warp
    // makes exactly one failed grab per stage, so the counter of slot s advances by nb + kConsumers per
    // use and each warp tracks the slot's base itself (no reset).
    int gbase[kStages];
#pragma unroll
    for (int i = 0; i < kStages; ++i) gbase[i] = 0;
    for (;; ++tc) {
        const int tb = tc & 1;
        if (!__all_sync(kFull, mbar_wait(&full_t[tb], uint32_t((tc >> 1) & 1), abort_flag, p.wait_ns))) return;
        const int ti = tidx[tb];
        if (ti >= p.ntiles) return;
        const TcTile t = p.tiles[p.tile0 + ti];
        const uint8_t* bl = blobs + tb * kBlobMax;
        const uint8_t* attr = p.blob + t.blob_off + t.attr_off;  // per-position attributes (global)
        const int nb = (t.nrows + 15) >> 4;
        for (int h = 0; h < heads; ++h, ++hc) {
            const int s = int(hc % kStages);
            if (!__all_sync(kFull, mbar_wait(&full_h[s], uint32_t((hc / kStages) & 1), abort_flag, p.wait_ns))) return;
            const uint32_t kbase = smem_u32(sm + kOffStage + s * kStageBytes);
            const uint32_t vbase = kbase + kKVBytes, qbase = kbase + 2 * kKVBytes;
            const uint32_t wbase = smem_u32(wext + h * 1024);
            int base = 0;
#pragma unroll
            for (int i = 0; i < kStages; ++i) base = i == s ? gbase[i] : base;
            for (;;) {
                int rb = 0;
                if (lane == 0) rb = atomicAdd(&tgrab[s], 1);
                rb = __shfl_sync(kFull, rb, 0) - base;
                if (rb >= nb) break;
                const uint8_t* bh = bl + kTcBlockOff + 32 * rb;
                const int nch = bh[0], cbase = bh[1];
                // ---- x_r of this lane's output elements, read now so the loads overlap the products (the
                // compiler may not move loads of x_r past stores to out, which may alias)
                const int r0 = 16 * rb + g, r1 = r0 + 8;
                const int64_t lr0 = int64_t(t.row0) + r0 - p.dst_lo, lr1 = lr0 + 8;
                const int c0 = h * kHD + 2 * t4;
                uint32_t xv0[8], xv1[8];
#pragma unroll
                for (int n = 0; n < 8; ++n) {
                    xv0[n] = r0 < t.nrows ? __ldg(reinterpret_cast<const unsigned*>(p.xr + lr0 * p.ldxr + c0 + 8 * n)) : 0u;
                    xv1[n] = r1 < t.nrows ? __ldg(reinterpret_cast<const unsigned*>(p.xr + lr1 * p.ldxr + c0 + 8 * n)) : 0u;
                }
                // ---- Q fragments of rows [16 rb, 16 rb + 16)
                uint32_t qa[4][4];
                {
                    const int r = 16 * rb + (lane & 7) + ((lane >> 3) & 1) * 8;
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk) ldsm_x4(qbase + swz(r, 2 * kk + (lane >> 4)), qa[kk]);
                }
                // ---- qe = Q W_ext: columns (qe0, qe1 | qe2, qb) in lanes t4 = 0 | 1 of each quad
                float qv[2][4];  // per row (r0, r1): qe0, qe1, qe2, qb, scaled to the log2 domain
                {
                    float ce[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
                    for (int half = 0; half < 2; ++half) {
                        uint32_t b[4];
                        ldsm_x4(wbase + swz(lane & 7, 4 * half + (lane >> 3)), b);
                        mma16816(ce, qa[2 * half], b[0], b[1]);
                        mma16816(ce, qa[2 * half + 1], b[2], b[3]);
                    }
                    const int la = lane & ~3;
#pragma unroll
                    for (int rr = 0; rr < 2; ++rr) {
                        qv[rr][0] = __shfl_sync(kFull, ce[2 * rr], la) * p.scale_log2;
                        qv[rr][1] = __shfl_sync(kFull, ce[2 * rr + 1], la) * p.scale_log2;
                        qv[rr][2] = __shfl_sync(kFull, ce[2 * rr], la + 1) * p.scale_log2;
                        qv[rr][3] = __shfl_sync(kFull, ce[2 * rr + 1], la + 1) * p.scale_log2;
                    }
                }
                float m[2] = {-INFINITY, -INFINITY};
                // l and pa as two partial sums (even / odd slot column) updated by paired fp32 operations
                float2 l2[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
                float2 pa2[2][3];
#pragma unroll
                for (int rr = 0; rr < 2; ++rr) pa2[rr][0] = pa2[rr][1] = pa2[rr][2] = make_float2(0.f, 0.f);
                float2 qv2[2][4];
#pragma unroll
                for (int rr = 0; rr < 2; ++rr)
#pragma unroll
                    for (int k = 0; k < 4; ++k) qv2[rr][k] = make_float2(qv[rr][k], qv[rr][k]);
                const float2 scale2 = make_float2(p.scale_log2, p.scale_log2);
                float o[8][4];
#pragma unroll
                for (int n = 0; n < 8; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
                // ---- 16-slot steps: two column blocks (ja, jb) each. The products S, the position mask and
                // the attribute words of step c + 1 are issued before the weights of step c (software pipeline).
                auto scores = [&](int c, float (&sv)[8], uint4 (&at)[3], uint32_t& mk) {
                    const int ja = bh[2 + 2 * c], jb = bh[3 + 2 * c];
                    float sa[4] = {0.f, 0.f, 0.f, 0.f}, sb[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
                    for (int half = 0; half < 2; ++half) {
                        uint32_t b[4], d[4];
                        ldsm_x4(kbase + swz(8 * ja + (lane & 7), 4 * half + (lane >> 3)), b);
                        ldsm_x4(kbase + swz(8 * jb + (lane & 7), 4 * half + (lane >> 3)), d);
                        mma16816(sa, qa[2 * half], b[0], b[1]);
                        mma16816(sb, qa[2 * half], d[0], d[1]);
                        mma16816(sa, qa[2 * half + 1], b[2], b[3]);
                        mma16816(sb, qa[2 * half + 1], d[2], d[3]);
                    }
#pragma unroll
                    for (int i = 0; i < 4; ++i) sv[i] = sa[i], sv[4 + i] = sb[i];
                    const uint4* ap = reinterpret_cast<const uint4*>(attr + kTcChunkAttr * (cbase + c)) + 3 * lane;
                    at[0] = __ldg(ap), at[1] = __ldg(ap + 1), at[2] = __ldg(ap + 2);
                    mk = bl[kTcMaskOff + 32 * (cbase + c) + lane];
                };
                float svn[8];
                uint4 atn[3] = {make_uint4(0u, 0u, 0u, 0u), make_uint4(0u, 0u, 0u, 0u), make_uint4(0u, 0u, 0u, 0u)};
                uint32_t mkn = 0u;
                if (nch > 0) scores(0, svn, atn, mkn);
                for (int c = 0; c < nch; ++c) {
                    const int ja = bh[2 + 2 * c], jb = bh[3 + 2 * c];
                    // positions e = 4 k + 2 h + i: column block k (ja, jb), row r0 + 8 h, slot column 2 t4 + i;
                    // pair q = e / 2 = (block k, row h) holds columns 2 t4, 2 t4 + 1
                    float sv[8];
#pragma unroll
                    for (int i = 0; i < 8; ++i) sv[i] = svn[i];
                    float2 av[4][3], sp[4];
                    {
                        const uint32_t aw[12] = {atn[0].x, atn[0].y, atn[0].z, atn[0].w, atn[1].x, atn[1].y,
                                                 atn[1].z, atn[1].w, atn[2].x, atn[2].y, atn[2].z, atn[2].w};
#pragma unroll
                        for (int q = 0; q < 4; ++q)
#pragma unroll
                            for (int k = 0; k < 3; ++k) av[q][k] = unpack_h2(aw[3 * q + k]);
                    }
                    const uint32_t mk = mkn;
                    if (c + 1 < nch) scores(c + 1, svn, atn, mkn);
                    float cm[2] = {-INFINITY, -INFINITY};
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        const int rr = q & 1;
                        // s = S / sqrt(d) + <W_e^T q, a> + <q, b_e> in the log2 domain, in the reference's order
                        float2 tt = __ffma2_rn(qv2[rr][2], av[q][2], qv2[rr][3]);
                        tt = __ffma2_rn(qv2[rr][1], av[q][1], tt);
                        tt = __ffma2_rn(qv2[rr][0], av[q][0], tt);
                        float2 sc = __ffma2_rn(make_float2(sv[2 * q], sv[2 * q + 1]), scale2, tt);
                        sc.x = (mk >> (2 * q)) & 1u ? sc.x : -INFINITY;
                        sc.y = (mk >> (2 * q + 1)) & 1u ? sc.y : -INFINITY;
                        sp[q] = sc;
                        cm[rr] = fmaxf(cm[rr], fmaxf(sc.x, sc.y));
                    }
                    // the reference maxima m are the same in the four lanes of a row's quad; they move only
                    // when a lane's own score exceeds them by more than the slack (then over the quad)
                    if (__any_sync(kFull, cm[0] > m[0] + kSlack || cm[1] > m[1] + kSlack)) {
#pragma unroll
                        for (int rr = 0; rr < 2; ++rr) {
                            cm[rr] = fmaxf(cm[rr], __shfl_xor_sync(kFull, cm[rr], 1));
                            cm[rr] = fmaxf(cm[rr], __shfl_xor_sync(kFull, cm[rr], 2));
                            const float mn = fmaxf(m[rr], cm[rr]);
                            const float corr = mn == -INFINITY ? 1.f : ex2(m[rr] - mn);
                            m[rr] = mn;
                            const float2 c2 = make_float2(corr, corr);
                            l2[rr] = __fmul2_rn(l2[rr], c2);
                            pa2[rr][0] = __fmul2_rn(pa2[rr][0], c2), pa2[rr][1] = __fmul2_rn(pa2[rr][1], c2);
                            pa2[rr][2] = __fmul2_rn(pa2[rr][2], c2);
#pragma unroll
                            for (int n = 0; n < 8; ++n) o[n][2 * rr] *= corr, o[n][2 * rr + 1] *= corr;
                        }
                    }
                    const float mu[2] = {m[0] == -INFINITY ? 0.f : m[0], m[1] == -INFINITY ? 0.f : m[1]};
                    uint32_t a[4];
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        const int rr = q & 1;
                        const float2 d = __fadd2_rn(sp[q], make_float2(-mu[rr], -mu[rr]));
                        const float2 w = make_float2(ex2(d.x), ex2(d.y));
                        l2[rr] = __fadd2_rn(l2[rr], w);
#pragma unroll
                        for (int k = 0; k < 3; ++k) pa2[rr][k] = __ffma2_rn(w, av[q][k], pa2[rr][k]);
                        a[q] = pack_h2(w.x, w.y);
                    }
                    const int vr = 8 * (((lane >> 3) & 1) ? jb : ja) + (lane & 7);
#pragma unroll
                    for (int n = 0; n < 8; n += 2) {
                        uint32_t b[4];
                        ldsm_x4_t(vbase + swz(vr, n + (lane >> 4)), b);
                        mma16816(o[n], a, b[0], b[1]);
                        mma16816(o[n + 1], a, b[2], b[3]);
                    }
                }
                float l[2], pa[2][3];
#pragma unroll
                for (int rr = 0; rr < 2; ++rr) {
                    l[rr] = l2[rr].x + l2[rr].y;
#pragma unroll
                    for (int k = 0; k < 3; ++k) pa[rr][k] = pa2[rr][k].x + pa2[rr][k].y;
                }
#pragma unroll
                for (int rr = 0; rr < 2; ++rr) {
                    l[rr] += __shfl_xor_sync(kFull, l[rr], 1);
                    l[rr] += __shfl_xor_sync(kFull, l[rr], 2);
#pragma unroll
                    for (int k = 0; k < 3; ++k) {
                        pa[rr][k] += __shfl_xor_sync(kFull, pa[rr][k], 1);
                        pa[rr][k] += __shfl_xor_sync(kFull, pa[rr][k], 2);
                    }
                }
                // ---- + [pa | l] [W_e ; b_e]: (pa0, pa1, pa2, l) as fp16 hi (columns 0-3) and lo (columns
                // 4-7) against W_ext rows (W_e[:, 0..2], b_e) twice
                {
                    const bool odd = t4 & 1;
                    uint32_t a[4];
#pragma unroll
                    for (int rr = 0; rr < 2; ++rr) {
                        const float fa = odd ? pa[rr][2] : pa[rr][0], fb = odd ? l[rr] : pa[rr][1];
                        if (t4 < 2) {
                            a[rr] = pack_h2(fa, fb);
                        } else {
                            const float2 hi = unpack_h2(pack_h2(fa, fb));
                            a[rr] = pack_h2(fa - hi.x, fb - hi.y);
                        }
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
                const float i0 = l[0] > 0.f ? 1.0f / l[0] : 0.f, i1 = l[1] > 0.f ? 1.0f / l[1] : 0.f;
                // (T(T(o) + x_r) as one fp16 add of T(o) and x_r: the sum of two fp16 values is exact in
                // fp32 whenever it can round differently, so both give the same fp16)
#pragma unroll
                for (int n = 0; n < 8; ++n) {
                    const int cc = c0 + 8 * n;
                    if (r0 < t.nrows)
                        *reinterpret_cast<__half2*>(p.out + lr0 * p.ldo + cc) =
                            __hadd2(__floats2half2_rn(o[n][0] * i0, o[n][1] * i0), *reinterpret_cast<const __half2*>(&xv0[n]));
                    if (r1 < t.nrows)
                        *reinterpret_cast<__half2*>(p.out + lr1 * p.ldo + cc) =
                            __hadd2(__floats2half2_rn(o[n][2] * i1, o[n][3] * i1), *reinterpret_cast<const __half2*>(&xv1[n]));
                }
            }
#pragma unroll
            for (int i = 0; i < kStages; ++i) gbase[i] += i == s ? nb + kConsumers : 0;
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
    TcParams p{};
    p.tiles = a.tiles, p.srcs = a.srcs, p.blob = a.blob, p.tile0 = a.tile0, p.ntiles = a.ntiles, p.dst_lo = a.dst_lo;
    p.q = a.q, p.k = a.k, p.v = a.v, p.xr = a.xr, p.out = a.out;
    p.ldq = a.ldq, p.ldkv = a.ldkv, p.ldxr = a.ldxr, p.ldo = a.ldo, p.n_q_rows = a.n_q_rows;
    p.w_e = a.w_e, p.C = a.C, p.heads = a.heads;
    p.scale_log2 = 1.4426950408889634f / std::sqrt(float(a.head_dim));
    // failure-path test hooks (host-side, no fault): VB_DEBUG_WAIT_NS shortens every wait's limit and
    // VB_DEBUG_TC_WITHHOLD=1 makes CTA 0 skip its first stage's copies, so its consumers' wait runs out
    const char* wn = std::getenv("VB_DEBUG_WAIT_NS");
    const char* wh = std::getenv("VB_DEBUG_TC_WITHHOLD");
    p.wait_ns = wn && *wn ? std::strtoull(wn, nullptr, 10) : kTimeoutNs;
    p.withhold = wh && *wh && std::atoi(wh) != 0;
    p.sched = a.sched;
    static std::atomic<uint64_t> configured{0};
    once_per_device(configured, [] {
        VB_CUDA(cudaFuncSetAttribute(attention_tc_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     kSmemBytes(4, kMaxHeads)));
        VB_CUDA(cudaFuncSetAttribute(attention_tc_kernel<5>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     kSmemLimit));
    });
    const int grid = std::min(a.ntiles, device_sm_count());
    if (stages_for(a.heads) == 5) attention_tc_kernel<5><<<grid, kThreads, kSmemBytes(5, a.heads), s>>>(p);
    else attention_tc_kernel<4><<<grid, kThreads, kSmemBytes(4, a.heads), s>>>(p);
    VB_LAUNCH();
}

int take_tc_error() {
    int e = 0, zero = 0;
    VB_CUDA(cudaMemcpyFromSymbol(&e, g_tc_error, sizeof(int)));
    if (e) VB_CUDA(cudaMemcpyToSymbol(g_tc_error, &zero, sizeof(int)));
    return e;
}

}  // namespace vb::k
