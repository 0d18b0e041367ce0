// tcgen05 GEMM (see gemm_tc.cuh).
//
// Persistent kernel, one 320-thread CTA per SM (or one cluster of two CTAs per two SMs, below),
// warp-specialised:
//   warp 0 (one lane)   TMA producer: A [128 x 64] and W [BN x 64] fp16 tiles, 128-byte swizzle,
//                       into a STAGES-deep shared-memory ring (full/empty mbarriers).
//   warp 1 (one lane)   MMA issuer: 4 x tcgen05.mma (M=128, N=BN, K=16) per 64-wide k block into
//                       one of two TMEM accumulators; tcgen05.commit frees the smem stage, and a
//                       commit after the last k block hands the accumulator to the epilogue.
//   warps 2-9           epilogue: tcgen05.ld 32 columns at a time, the next chunk in flight (warp w
//                       reads TMEM lanes 32 (w % 4) .. + 31 = its 32 output rows; warps w and
//                       w + 4 split the columns in halves), bias / GELU / residual in fp32 with the
//                       fp16 operands added by mixed-precision adds (the residual row read into
//                       registers one chunk ahead), the 32 x 32 fp16 sub-tile staged in
//                       64-byte-swizzled shared memory and written by one TMA bulk tensor store;
//                       the accumulator goes back to the MMA warp once its last chunk is loaded.
// LayerNorm variants of the epilogue (template argument LN): kLnStats also accumulates, per row and per
// column half, the {mean, M2} record of the values it stores (the next LayerNorm's statistics); kLnFold
// applies a LayerNorm of A folded into W and the bias: y = rstd acc - rstd mean colsum + b', rstd and
// mean from A's row records (kernels.cuh fold_layernorm / row_seg_stats, dev.cuh for the arithmetic).
// Two accumulators (2 x BN TMEM columns) let the epilogue of tile i overlap the main loop of
// tile i + 1. With N > 128 the CTAs run in clusters of two (cta_group::2): the pair computes a
// 256-row tile with one MMA stream issued by the leader, each CTA loading its own 128 rows of A and
// half of the W tile (TMA loads without multicast, completing on the leader's barrier) and holding
// its 128 accumulator rows in its own TMEM; commits arrive on both CTAs' barriers, and both CTAs'
// epilogue warps release the leader's accumulator. Tiles are visited m-major (n fastest) so an A row
// block is reused from L2 by the CTAs working on its N tiles.
//
// Every mbarrier wait is bounded (kTimeoutNs of %globaltimer). On timeout a CTA sets the device
// error flag, stops issuing work, waits (bounded) for its own TMA loads and MMAs in flight,
// frees its TMEM and returns; the host reads the flag with take_error().
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstdint>
#include <cstdlib>
#include <map>
#include <mutex>
#include <string>
#include <thread>
#include <tuple>

#include "common.h"
#include "dev.cuh"
#include "gemm_tc.cuh"

namespace vb::tc {

namespace {

using vb::d::from_f;
using vb::d::gelu;
using vb::d::ln_from_records;
using vb::d::rnd;
using vb::d::seg_add;
using vb::d::seg_record;
using vb::d::to_f;

constexpr int BM = 128, BK = 64;
constexpr int kEpiWarps = 8, kThreads = 32 * (2 + kEpiWarps);
constexpr unsigned long long kTimeoutNs = 4000000000ull;  // 4 s
// Dynamic tile order: the tile indices a CTA (pair) takes from the launch's counter pass through a
// ring of kRing slots in shared memory, from the producer lane (the pair leader's) to every role.
constexpr int kRing = 8;

__device__ int g_error = 0;

struct Params {
    const __half* bias;
    __half* C;
    int64_t ldc;
    const __half* R;
    int64_t ldr;
    int M, N, K;
    int epi;
    int gelu_tanh;
    unsigned* sched;  // dynamic tile order: [tiles handed out, fetchers done], zero between launches; or null
    // LayerNorm fusion: the output rows' segment records (kLnStats), or A's records and the folded
    // weights' column sums (kLnFold)
    float2* st_out;
    int nseg_out;
    const float2* st_in;
    const float* colsum;
    int nseg_in;
    float segw_in, eps;
};
// LN template argument of the kernel: no LayerNorm work, write the output's segment records, or apply
// the LayerNorm of A folded into the weights.
constexpr int kLnNone = 0, kLnStats = 1, kLnFold = 2;
constexpr int kMaxSegs = 16;  // records per row a folded GEMM reads (C <= 2048)

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
// ... with acquire at cluster scope (for arrivals that carry another CTA's shared-memory writes)
__device__ __forceinline__ bool mbar_test_cl(uint64_t* b, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(ok)
        : "r"(smem_u32(b)), "r"(parity)
        : "memory");
    return ok != 0;
}
// Bounded wait for the phase of parity `parity`. Returns false on timeout (after raising the CTA's
// abort flag and the device error flag) or when another role already aborted.
template <bool CL = false>
__device__ __forceinline__ bool mbar_wait(uint64_t* b, uint32_t parity, volatile int* abort_flag) {
    auto test = [&] { return CL ? mbar_test_cl(b, parity) : mbar_test(b, parity); };
    if (test()) return true;
    const uint64_t t0 = now_ns();
    for (;;) {
        if (test()) return true;
        if (*abort_flag) return false;
        if (now_ns() - t0 > kTimeoutNs) {
            *abort_flag = 1;
            atomicExch(&g_error, 1);
            return false;
        }
    }
}
// Wait that ignores the abort flag (used only to drain work in flight), still bounded.
__device__ __forceinline__ void mbar_drain(uint64_t* b, uint32_t parity) {
    const uint64_t t0 = now_ns();
    while (!mbar_test(b, parity))
        if (now_ns() - t0 > kTimeoutNs) {
            atomicExch(&g_error, 2);
            return;
        }
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

// Shared-memory matrix descriptor: K-major tile, 128-byte swizzle, 8-row groups 1024 bytes apart.
__device__ __forceinline__ uint64_t smem_desc(uint32_t saddr) {
    uint64_t d = 0;
    d |= uint64_t((saddr & 0x3FFFF) >> 4);  // start address
    d |= uint64_t(1) << 16;                 // leading byte offset (unused for swizzled K-major)
    d |= uint64_t(1024 >> 4) << 32;         // stride byte offset
    d |= uint64_t(1) << 46;                 // descriptor version (sm_100)
    d |= uint64_t(2) << 61;                 // SWIZZLE_128B
    return d;
}

// Instruction descriptor, kind::f16: A = B = fp16, D = fp32, both K-major, M = MM (128, or 256 for a
// CTA pair), N = BN.
template <int BN, int MM = BM> constexpr uint32_t instr_desc() {
    return (1u << 4)                      // D format fp32
           | (0u << 7) | (0u << 10)       // A, B format fp16
           | (uint32_t(BN >> 3) << 17)    // N
           | (uint32_t(MM >> 4) << 24);   // M
}

__device__ __forceinline__ void mma_f16(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
        "l"(a), "l"(b), "r"(idesc), "r"(acc));
}
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}
// ---- CTA pairs (cta_group::2): the MMA of a cluster of two CTAs on SMs of one TPC computes a
// 256-row tile; each CTA holds its 128 rows of A and half of the BN rows of B in its own shared
// memory, and its 128 rows of the accumulator in its own TMEM.
__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
// shared::cluster address of the variable at shared::cta address `a` in the cluster's CTA `rank`
__device__ __forceinline__ uint32_t mapa(uint32_t a, uint32_t rank) {
    uint32_t d;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(rank));
    return d;
}
__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
__device__ __forceinline__ void st_cluster_u32(uint32_t cluster_addr, uint32_t v) {
    asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(cluster_addr), "r"(v) : "memory");
}
// TMA tile load into this CTA's shared memory whose bytes complete on the barrier at `bar_cluster`
// (the pair leader's); no multicast.
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const CUtensorMap* map, uint32_t bar_cluster, int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
        "[%4];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar_cluster)
        : "memory");
}
__device__ __forceinline__ void mma_f16_pair(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
        "l"(a), "l"(b), "r"(idesc), "r"(acc));
}
// completion of the pair's MMAs issued so far, arriving on the barrier at the same offset in both CTAs
__device__ __forceinline__ void mma_commit_pair(uint64_t* bar) {
    asm volatile(
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
            smem_u32(bar)),
        "h"(uint16_t(3))
        : "memory");
}
// ... and on this CTA's barrier only
__device__ __forceinline__ void mma_commit_pair_local(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// tcgen05.ld of 32 consecutive TMEM columns of this warp's 32 lanes, without waiting; tmem_wait32
// waits for every load of the thread and hands the registers on (they are in-out operands of the
// wait, so no use of them can be scheduled before it).
__device__ __forceinline__ void tmem_ld32_async(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
        "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait32(uint32_t (&r)[32]) {
    asm volatile("tcgen05.wait::ld.sync.aligned;"
                 : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                   "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                   "+r"(r[15]), "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]),
                   "+r"(r[22]), "+r"(r[23]), "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]),
                   "+r"(r[29]), "+r"(r[30]), "+r"(r[31])
                 :
                 : "memory");
}

// x + h (h an fp16 value, widened exactly): the sm_100 mixed-precision add, one instruction per element.
__device__ __forceinline__ float2 add_h2(uint32_t h2, float2 x) {
    float2 d;
    asm("{\n\t.reg .f16 lo, hi;\n\tmov.b32 {lo, hi}, %2;\n\t"
        "add.rn.f32.f16 %0, lo, %3;\n\tadd.rn.f32.f16 %1, hi, %4;\n\t}"
        : "=f"(d.x), "=f"(d.y)
        : "r"(h2), "f"(x.x), "f"(x.y));
    return d;
}
// Two fp32 values rounded to fp16 and packed (low half = x.x).
__device__ __forceinline__ uint32_t pack_h2(float2 x) {
    const __half2 h = __floats2half2_rn(x.x, x.y);
    return *reinterpret_cast<const uint32_t*>(&h);
}
__device__ __forceinline__ float2 unpack_h2(uint32_t u) { return __half22float2(*reinterpret_cast<const __half2*>(&u)); }
__device__ __forceinline__ float ex2f(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// Shared memory: the A/W stage ring, then per epilogue warp two 2 KB output staging buffers, then the
// mbarriers, the TMEM address and abort flag, and the ring of tile indices (dynamic tile order).
template <int BN, int STAGES, int EPI, bool PAIR> struct Layout {
    static constexpr int kA = BM * BK * 2;                   // bytes per A stage
    static constexpr int kB = (PAIR ? BN / 2 : BN) * BK * 2;  // this CTA's rows of W per stage
    static constexpr int kTiles = STAGES * (kA + kB);
    static constexpr int kSub = 32 * 32 * 2;  // one 32 x 32 fp16 sub-tile
    static constexpr int kOut = kEpiWarps * 2 * kSub;
    static constexpr int kBars = (2 * STAGES + 5 + 2 * kRing) * 8;
    static constexpr int kSmem = 1024 + kTiles + kOut + kBars + 16 + 4 * kRing;  // 1024: alignment slack
    static_assert(kSmem <= 232448, "shared memory over the 227 KB per-CTA limit");
};

// GELU for the fp16 path: x * Phi(x), Phi from the erf approximation of Abramowitz & Stegun,
// Handbook of Mathematical Functions, formula 7.1.26 (|error of erf| <= 1.5e-7), written as
// Phi(x) = 1 - q (x >= 0), q (x < 0) with q = P(t) exp(-z^2) / 2, z = |x| / sqrt(2), so the left tail
// has no cancellation. Checked against the erff-based GELU by the tests.
// Two values at a time with packed fp32 operations; q's factor 1/2 is folded into the polynomial's
// coefficients (exact: a power of two); exp(-z^2) = 2^(-z^2 log2 e) and the reciprocal on the SFU.
__device__ __forceinline__ float2 gelu_as2(float2 x) {
    const float2 z = __fmul2_rn(make_float2(fabsf(x.x), fabsf(x.y)), make_float2(0.70710678118654752f, 0.70710678118654752f));
    // t = 1 / (1 + p z) on the SFU. (A cubic first guess plus two Newton steps on the FMA pipe, which
    // frees the SFU, measured slower: 1159 against 1214 TFLOP/s on [189809 x 1024] x [1024 x 4096]; the
    // epilogue is bound by instruction issue, not by the SFU.)
    const float2 den = __ffma2_rn(make_float2(0.3275911f, 0.3275911f), z, make_float2(1.0f, 1.0f));
    float2 t;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(t.x) : "f"(den.x));
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(t.y) : "f"(den.y));
    float2 p = __ffma2_rn(t, make_float2(0.5307027145f, 0.5307027145f), make_float2(-0.7265760135f, -0.7265760135f));
    p = __ffma2_rn(t, p, make_float2(0.7107068705f, 0.7107068705f));
    p = __ffma2_rn(t, p, make_float2(-0.142248368f, -0.142248368f));
    p = __ffma2_rn(t, p, make_float2(0.127414796f, 0.127414796f));
    p = __fmul2_rn(t, p);
    // exp(-z^2) = 2^(-z^2 log2 e)
    const float2 a = __fmul2_rn(__fmul2_rn(z, z), make_float2(-1.4426950408889634f, -1.4426950408889634f));
    const float2 q = __fmul2_rn(p, make_float2(ex2f(a.x), ex2f(a.y)));
    const float2 one_q = __fadd2_rn(make_float2(1.0f, 1.0f), make_float2(-q.x, -q.y));
    return __fmul2_rn(x, make_float2(x.x >= 0.0f ? one_q.x : q.x, x.y >= 0.0f ? one_q.y : q.y));
}

__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, const void* src, int x, int y) {
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];" ::"l"(
                     reinterpret_cast<uint64_t>(map)),
                 "r"(x), "r"(y), "r"(smem_u32(src))
                 : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read1() { asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// Byte offset of 16-byte chunk j of row r in a 32 x 64-byte sub-tile with the 64-byte swizzle of the
// tensor map (chunk index XOR bits 1-2 of the row): conflict-free 16-byte accesses by 32 lanes.
__device__ __forceinline__ int sw64(int r, int j) { return r * 64 + ((j ^ ((r >> 1) & 3)) << 4); }

template <int BN, int STAGES, int EPI, bool PAIR, int LN>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ CUtensorMap tmC, Params p) {
    using L = Layout<BN, STAGES, EPI, PAIR>;
    constexpr int UM = PAIR ? 2 * BM : BM;  // rows of one output tile (one CTA, or the pair)
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sA = smem;
    uint8_t* sB = smem + STAGES * L::kA;
    uint8_t* sOut = smem + L::kTiles;
    uint64_t* bars = reinterpret_cast<uint64_t*>(sOut + L::kOut);
    uint64_t* full = bars;
    uint64_t* empty = bars + STAGES;
    uint64_t* tfull = bars + 2 * STAGES;
    uint64_t* tempty = bars + 2 * STAGES + 2;
    uint64_t* drain = bars + 2 * STAGES + 4;
    uint64_t* rfull = bars + 2 * STAGES + 5;  // tile ring: slot written
    uint64_t* rempty = rfull + kRing;         // tile ring: slot read by every role of the CTA (pair)
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(rempty + kRing);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    volatile int* ring = reinterpret_cast<volatile int*>(tmem_slot + 4);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = PAIR ? cluster_rank() : 0u;  // 0: the pair leader (issues the MMAs)
    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) mbar_init(&full[s], 1), mbar_init(&empty[s], 1);
        // the leader's accumulator is released by the epilogue warps of both CTAs
        for (int b = 0; b < 2; ++b) mbar_init(&tfull[b], 1), mbar_init(&tempty[b], PAIR ? 2 * kEpiWarps : kEpiWarps);
        mbar_init(drain, 1);
        // ring readers: the MMA lane and the epilogue warps (+ the peer's producer lane and epilogue warps)
        for (int r = 0; r < kRing; ++r)
            mbar_init(&rfull[r], 1), mbar_init(&rempty[r], PAIR ? 2 + 2 * kEpiWarps : 1 + kEpiWarps);
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        if (PAIR) {
            asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                         "r"(2 * BN));
            asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
        } else {
            asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                         "r"(2 * BN));
            asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
        }
    }
    fence_before();
    __syncthreads();
    if (PAIR) cluster_sync();  // both CTAs' barriers are initialised before either signals the other's
    fence_after();
    const uint32_t tmem = *tmem_slot;

    const int n_m = (p.M + UM - 1) / UM, n_n = (p.N + BN - 1) / BN;
    const int tiles = n_m * n_n, kblocks = (p.K + BK - 1) / BK;
    // tiles are handed out per CTA, or per pair (both CTAs of a pair walk the same sequence). Static
    // order: tile unit0 + i * units. Dynamic order (p.sched): the first tile is unit0, each further one
    // the next index of the launch's counter (+ units), fetched by the producer lane of the CTA (the
    // leader's, for a pair) and passed to the other roles (and the peer CTA) through the tile ring, so
    // the tiles in flight stay a contiguous window however the CTAs drift apart.
    const int unit0 = PAIR ? int(blockIdx.x >> 1) : int(blockIdx.x);
    const int units = PAIR ? int(gridDim.x >> 1) : int(gridDim.x);
    const bool dyn = p.sched != nullptr;
    // tile number `it` of the sequence, for the roles that read the ring (warp_wide: every lane waits
    // and reads, lane 0 releases the slot); -1 after an abort
    auto next_tile = [&](int it, bool warp_wide) -> int {
        if (!dyn) return unit0 + it * units;
        const int slot = it % kRing;
        if (!mbar_wait<true>(&rfull[slot], uint32_t(it / kRing) & 1u, abort_flag)) return -1;
        const int t = ring[slot];
        if (warp_wide) __syncwarp();
        if (!warp_wide || lane == 0) {
            if (PAIR && rank != 0) mbar_arrive_cluster(mapa(smem_u32(&rempty[slot]), 0));
            else mbar_arrive(&rempty[slot]);
        }
        return t;
    };
    // the fetching lane writes tile number `it` into the ring (and the peer's)
    auto publish = [&](int it, int t) -> bool {
        const int slot = it % kRing;
        if (!mbar_wait<true>(&rempty[slot], (uint32_t(it / kRing) & 1u) ^ 1u, abort_flag)) return false;
        ring[slot] = t;
        if (PAIR) {
            st_cluster_u32(mapa(smem_u32(const_cast<int*>(&ring[slot])), 1), uint32_t(t));
            mbar_arrive_cluster(mapa(smem_u32(&rfull[slot]), 1));
        }
        mbar_arrive(&rfull[slot]);
        return true;
    };

    if (warp == 0 && lane == 0) {
        // ---------------- TMA producer
        int stage = 0;
        uint32_t phase = 0;
        uint32_t issued = 0, last_parity = 0;  // per-stage bit masks for the drain
        const bool fetcher = !PAIR || rank == 0;
        int nxt = unit0;
        for (int it = 0; !*abort_flag; ++it) {
            int tile;
            if (!dyn) {
                tile = unit0 + it * units;
            } else if (fetcher) {
                tile = nxt;
                if (!publish(it, tile)) break;
                // the following index: the atomic's latency hides behind this tile's loads
                if (tile < tiles) nxt = units + int(atomicAdd(p.sched, 1u));
            } else {
                tile = next_tile(it, false);
            }
            if (tile < 0 || tile >= tiles) break;
            const int mb = tile / n_n, nb = tile - mb * n_n;
            for (int kb = 0; kb < kblocks; ++kb) {
                if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag)) break;
                if (PAIR) {
                    // both CTAs' tiles complete on the leader's barrier, which expects the pair's bytes
                    if (rank == 0) mbar_expect_tx(&full[stage], uint32_t(2 * (L::kA + L::kB)));
                    const uint32_t fb = mapa(smem_u32(&full[stage]), 0);
                    tma_load_2d_pair(sA + stage * L::kA, &tmA, fb, kb * BK, mb * UM + int(rank) * BM);
                    tma_load_2d_pair(sB + stage * L::kB, &tmB, fb, kb * BK, nb * BN + int(rank) * (BN / 2));
                } else {
                    mbar_expect_tx(&full[stage], uint32_t(L::kA + L::kB));
                    tma_load_2d(sA + stage * L::kA, &tmA, &full[stage], kb * BK, mb * BM);
                    tma_load_2d(sB + stage * L::kB, &tmB, &full[stage], kb * BK, nb * BN);
                }
                issued |= 1u << stage;
                last_parity = (last_parity & ~(1u << stage)) | (phase << stage);
                if (++stage == STAGES) stage = 0, phase ^= 1;
            }
        }
        if (dyn && fetcher) {  // the last fetcher to finish zeroes the counter for the next launch
            __threadfence();
            if (atomicAdd(p.sched + 1, 1u) == unsigned(units - 1)) {
                atomicExch(p.sched, 0u);
                atomicExch(p.sched + 1, 0u);
            }
        }
        if (*abort_flag) {  // let every load already issued land before the CTA exits
            if (!PAIR || rank == 0) {
                for (int s = 0; s < STAGES; ++s)
                    if (issued & (1u << s)) mbar_drain(&full[s], (last_parity >> s) & 1);
            } else {  // the peer's loads complete on the leader's barriers: give them time to land
                const uint64_t t0 = now_ns();
                while (now_ns() - t0 < 2000000ull) {
                }
            }
        }
    } else if (warp == 1 && lane == 0 && rank == 0) {
        // ---------------- MMA issuer (the pair's leader issues for both CTAs)
        constexpr uint32_t idesc = instr_desc<BN, UM>();
        int stage = 0;
        uint32_t phase = 0;
        int it = 0;
        bool any = false;
        for (;; ++it) {
            if (*abort_flag) break;
            const int tile = next_tile(it, false);
            if (tile < 0 || tile >= tiles) break;
            const int ab = it & 1;
            const uint32_t ap = (it >> 1) & 1;
            if (!mbar_wait(&tempty[ab], ap ^ 1, abort_flag)) break;
            fence_after();
            const uint32_t d = tmem + uint32_t(ab * BN);
            bool ok = true;
            for (int kb = 0; kb < kblocks; ++kb) {
                if (!mbar_wait(&full[stage], phase, abort_flag)) {
                    ok = false;
                    break;
                }
                fence_after();
                const uint64_t a0 = smem_desc(smem_u32(sA + stage * L::kA));
                const uint64_t b0 = smem_desc(smem_u32(sB + stage * L::kB));
#pragma unroll
                for (int j = 0; j < BK / 16; ++j) {
                    if (PAIR) mma_f16_pair(d, a0 + uint64_t(2 * j), b0 + uint64_t(2 * j), idesc, (kb | j) != 0 ? 1u : 0u);
                    else mma_f16(d, a0 + uint64_t(2 * j), b0 + uint64_t(2 * j), idesc, (kb | j) != 0 ? 1u : 0u);
                }
                if (PAIR) mma_commit_pair(&empty[stage]);
                else mma_commit(&empty[stage]);
                any = true;
                if (++stage == STAGES) stage = 0, phase ^= 1;
            }
            if (!ok) break;
            if (PAIR) mma_commit_pair(&tfull[ab]);
            else mma_commit(&tfull[ab]);
        }
        if (any) {  // every MMA issued by this thread completes before the TMEM is freed
            if (PAIR) mma_commit_pair_local(drain);
            else mma_commit(drain);
            mbar_drain(drain, 0);
        }
    } else if (warp >= 2) {
        // ---------------- epilogue: TMEM -> registers -> fused epilogue -> swizzled smem -> TMA store
        const int ew = warp - 2;
        const int lg = warp & 3;   // TMEM lane group this warp may access (rows 32 lg .. + 31)
        const int half = ew >> 2;  // which half of the BN columns
        constexpr int kChunks = BN / 64;  // 32-column chunks per half
        uint8_t* obuf = sOut + ew * 2 * L::kSub;
        uint32_t n_out = 0;  // output staging uses so far (buffer = count & 1)
        int it = 0;
        // this lane's row of the residual, 32 columns from col0, as fp16 pairs (zero out of bounds)
        auto load_res = [&](int row, int col0, uint32_t(&rr)[16]) {
            if (row < p.M && col0 + 32 <= p.N) {
                const uint4* src = reinterpret_cast<const uint4*>(p.R + int64_t(row) * p.ldr + col0);
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const uint4 u = __ldg(src + q);
                    rr[4 * q] = u.x, rr[4 * q + 1] = u.y, rr[4 * q + 2] = u.z, rr[4 * q + 3] = u.w;
                }
            } else {
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    const int c0 = col0 + 2 * i;
                    const __half* r = p.R + int64_t(row) * p.ldr;
                    const uint32_t lo = (row < p.M && c0 < p.N) ? __half_as_ushort(r[c0]) : 0u;
                    const uint32_t hi = (row < p.M && c0 + 1 < p.N) ? __half_as_ushort(r[c0 + 1]) : 0u;
                    rr[i] = lo | (hi << 16);
                }
            }
        };
        // 32 bias values from col0 as fp16 pairs (zero where absent), the same for every lane
        auto load_bias = [&](int col0, uint32_t(&bh)[16]) {
            if (p.bias && col0 + 32 <= p.N) {
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const uint4 u = __ldg(reinterpret_cast<const uint4*>(p.bias + col0) + q);
                    bh[4 * q] = u.x, bh[4 * q + 1] = u.y, bh[4 * q + 2] = u.z, bh[4 * q + 3] = u.w;
                }
            } else {
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    const int c0 = col0 + 2 * i;
                    const uint32_t lo = (p.bias && c0 < p.N) ? __half_as_ushort(p.bias[c0]) : 0u;
                    const uint32_t hi = (p.bias && c0 + 1 < p.N) ? __half_as_ushort(p.bias[c0 + 1]) : 0u;
                    bh[i] = lo | (hi << 16);
                }
            }
        };
        // 32 fp32 column sums of the folded weights from col0 (kLnFold; zero out of bounds)
        auto load_colsum = [&](int col0, float(&cs)[32]) {
            if (col0 + 32 <= p.N) {
#pragma unroll
                for (int q = 0; q < 8; ++q) {
                    const float4 u = __ldg(reinterpret_cast<const float4*>(p.colsum + col0) + q);
                    cs[4 * q] = u.x, cs[4 * q + 1] = u.y, cs[4 * q + 2] = u.z, cs[4 * q + 3] = u.w;
                }
            } else {
#pragma unroll
                for (int i = 0; i < 32; ++i) cs[i] = col0 + i < p.N ? p.colsum[col0 + i] : 0.0f;
            }
        };
        // the leader's tempty barriers, which both CTAs' epilogue warps release
        const uint32_t te0 = PAIR ? mapa(smem_u32(&tempty[0]), 0) : 0u, te1 = PAIR ? mapa(smem_u32(&tempty[1]), 0) : 0u;
        auto release = [&](int ab) {
            fence_before();
            __syncwarp();
            if (lane == 0) {
                if (PAIR) mbar_arrive_cluster(ab ? te1 : te0);
                else mbar_arrive(&tempty[ab]);
            }
        };
        for (;; ++it) {
            const int tile = next_tile(it, true);
            if (tile < 0 || tile >= tiles) break;
            const int ab = it & 1;
            const uint32_t ap = (it >> 1) & 1;
            const int mb = tile / n_n, nb = tile - mb * n_n;
            const int row0 = mb * UM + int(rank) * BM + lg * 32;
            const int colh = nb * BN + half * (BN / 2);
            // the first chunk's residual and bias loads fly while the accumulator is being computed
            uint32_t resa[16], resb[16], bia[16], bib[16];
            float cs[32];  // kLnFold: this chunk's column sums (the next chunk's loaded once o is formed)
            // kLnFold: y = rstd acc + (-rstd mean) colsum + b' for this lane's row (its records read
            // while the accumulator is being computed)
            float rstd = 0.0f, nm = 0.0f;
            if (LN == kLnFold && row0 + lane < p.M) {
                const float2 mr = ln_from_records<kMaxSegs>(p.st_in + int64_t(row0 + lane) * p.nseg_in, 1, p.nseg_in,
                                                            p.segw_in, p.eps);
                rstd = mr.y, nm = __fmul_rn(-mr.y, mr.x);
            }
            if (EPI == k::kEpiResidual) load_res(row0 + lane, colh, resa);
            load_bias(colh, bia);
            if (LN == kLnFold) load_colsum(colh, cs);
            // kLnStats: this half row's segment record, from its first stored value
            float2 s1 = make_float2(0.0f, 0.0f), s2 = make_float2(0.0f, 0.0f);
            float kshift = 0.0f;
            if (!mbar_wait(&tfull[ab], ap, abort_flag)) break;
            fence_after();
            const uint32_t taddr = tmem + (uint32_t(lg * 32) << 16) + uint32_t(ab * BN + half * (BN / 2));
            bool ok = true, released = false;
            // chunk c's 32 columns are in ra (c even) / rb (c odd); chunk c + 1's load is in flight
            // while chunk c is processed, and the accumulator goes back to the MMA warp as soon as
            // its last chunk has been read
            uint32_t ra[32], rb[32];
            tmem_ld32_async(taddr, ra);
            tmem_wait32(ra);
#pragma unroll
            for (int c = 0; c < kChunks; ++c) {
                uint32_t(&cur)[32] = (c & 1) ? rb : ra;
                uint32_t(&nxt)[32] = (c & 1) ? ra : rb;
                uint32_t(&rcur)[16] = (c & 1) ? resb : resa;
                uint32_t(&rnxt)[16] = (c & 1) ? resa : resb;
                if (c + 1 < kChunks) tmem_ld32_async(taddr + uint32_t((c + 1) * 32), nxt);
                const int col0 = colh + c * 32;
                if (EPI == k::kEpiResidual && c + 1 < kChunks) load_res(row0 + lane, col0 + 32, rnxt);
                // this chunk's bias; the next one's in flight (kLnFold: one buffer, reloaded with the column
                // sums once o is formed, for registers)
                uint32_t(&bh)[16] = (LN == kLnFold || !(c & 1)) ? bia : bib;
                if (LN != kLnFold && c + 1 < kChunks) load_bias(col0 + 32, (c & 1) ? bia : bib);
                uint32_t o[16];  // the output sub-row, fp16 pairs
                if (LN == kLnFold) {
#pragma unroll
                    for (int i = 0; i < 16; ++i) {
                        const float2 acc = make_float2(__uint_as_float(cur[2 * i]), __uint_as_float(cur[2 * i + 1]));
                        const float2 t = __ffma2_rn(acc, make_float2(rstd, rstd),
                                                    __fmul2_rn(make_float2(cs[2 * i], cs[2 * i + 1]), make_float2(nm, nm)));
                        o[i] = pack_h2(add_h2(bh[i], t));  // T(LN(x) W^T + b)
                    }
                    if (c + 1 < kChunks) load_colsum(col0 + 32, cs), load_bias(col0 + 32, bia);
                } else {
#pragma unroll
                    for (int i = 0; i < 16; ++i) {
                        const float2 x = add_h2(bh[i], make_float2(__uint_as_float(cur[2 * i]), __uint_as_float(cur[2 * i + 1])));
                        o[i] = pack_h2(x);  // T(acc + b)
                    }
                }
                if (EPI == k::kEpiGelu) {
                    if (p.gelu_tanh) {
#pragma unroll
                        for (int i = 0; i < 16; ++i) {
                            const float2 x = unpack_h2(o[i]);
                            o[i] = pack_h2(make_float2(gelu(x.x, true), gelu(x.y, true)));
                        }
                    } else {
#pragma unroll
                        for (int i = 0; i < 16; ++i) o[i] = pack_h2(gelu_as2(unpack_h2(o[i])));
                    }
                }
                if (EPI == k::kEpiResidual) {
#pragma unroll
                    for (int i = 0; i < 16; ++i) o[i] = pack_h2(add_h2(rcur[i], unpack_h2(o[i])));  // T(T(acc+b)+r)
                }
                if (LN == kLnStats) {  // over the stored (rounded) values
                    if (c == 0) kshift = unpack_h2(o[0]).x;
#pragma unroll
                    for (int i = 0; i < 16; ++i) seg_add(s1, s2, kshift, unpack_h2(o[i]));
                }
                if (c + 1 < kChunks) {
                    tmem_wait32(nxt);
                    if (c + 2 == kChunks) {  // every column of the accumulator is in registers
                        release(ab);
                        released = true;
                    }
                }
                // stage the fp16 sub-tile (row = lane) and store it with one TMA bulk copy
                const uint32_t obi = n_out & 1;
                if (n_out >= 2 && lane == 0) bulk_wait_read1();  // the store that used this buffer read it
                __syncwarp();
                uint8_t* ob = obuf + obi * L::kSub;
#pragma unroll
                for (int j = 0; j < 4; ++j)
                    *reinterpret_cast<uint4*>(ob + sw64(lane, j)) = make_uint4(o[4 * j], o[4 * j + 1], o[4 * j + 2], o[4 * j + 3]);
                fence_async_smem();
                __syncwarp();
                if (lane == 0) {
                    tma_store_2d(&tmC, ob, col0, row0);
                    bulk_commit();
                }
                ++n_out;
            }
            if (!released) release(ab);
            if (LN == kLnStats && row0 + lane < p.M && colh < p.N)  // (a half past N has no segment)
                p.st_out[int64_t(row0 + lane) * p.nseg_out + colh / (BN / 2)] = seg_record(s1, s2, kshift, float(BN / 2));
            if (!ok) break;
        }
        if (lane == 0) bulk_wait_all();  // every TMA store has finished before the CTA exits
        __syncwarp();
    }
    fence_before();
    __syncthreads();
    if (PAIR) cluster_sync();  // no CTA leaves while its peer may still read its shared memory or signal it
    if (warp == 1) {
        fence_after();
        if (PAIR) asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(2 * BN));
        else asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(2 * BN));
    }
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        cudaDriverEntryPointQueryResult q{};
        void* f = nullptr;
        VB_CUDA(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q));
        if (q != cudaDriverEntryPointSuccess || !f) fail(kCuda, "cuTensorMapEncodeTiled is not available");
        fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
    });
    return fn;
}

// 2-D fp16 tensor map over a row-major [rows, cols] matrix with leading dimension ld (elements),
// box [box_rows, box_cols], zero fill out of bounds (loads) / clipped (stores).
CUtensorMap make_map(const __half* base, int64_t rows, int64_t cols, int64_t ld, int box_rows, int box_cols = BK,
                     CUtensorMapSwizzle swz = CU_TENSOR_MAP_SWIZZLE_128B) {
    CUtensorMap m;
    const cuuint64_t dims[2] = {cuuint64_t(cols), cuuint64_t(rows)};
    const cuuint64_t strides[1] = {cuuint64_t(ld) * 2};
    const cuuint32_t box[2] = {cuuint32_t(box_cols), cuuint32_t(box_rows)};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<__half*>(base), dims, strides,
                                   box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) fail(kCuda, "cuTensorMapEncodeTiled failed (" + std::to_string(int(r)) + ")");
    return m;
}

// Per-stream tile counters for the dynamic tile order of launches that bring no counter of their own
// (the public vb_gemm with VB_GEMM_SCHED=1): g_sched, two words per (device, stream, thread): tiles
// handed out, fetchers done; each launch leaves them zero. Launches on one stream run one after
// another, so such a counter is shared only by launches that run concurrently on the same stream key,
// which a CUDA graph replayed on another stream (or twice at once) can do: the public entry point
// therefore uses the static order unless asked. Static order (nullptr) also when the slots are used up,
// or when the first launch on a device comes during stream capture (the symbol lookup may load the
// module).
constexpr int kSchedSlots = 1024, kMaxDevices = 64;
__device__ unsigned g_sched[2 * kSchedSlots];

unsigned* sched_counter(cudaStream_t s) {
    const char* e = std::getenv("VB_GEMM_SCHED");
    if (!(e && *e && std::atoi(e) != 0)) return nullptr;
    int dev = 0;
    VB_CUDA(cudaGetDevice(&dev));
    if (dev < 0 || dev >= kMaxDevices) return nullptr;
    static std::mutex mu;
    static unsigned* base[kMaxDevices] = {};
    static std::map<std::tuple<int, cudaStream_t, std::thread::id>, int> slot;
    static int used[kMaxDevices] = {};
    std::lock_guard<std::mutex> lock(mu);
    if (!base[dev]) {
        cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
        VB_CUDA(cudaStreamIsCapturing(s, &cs));
        if (cs != cudaStreamCaptureStatusNone) return nullptr;
        void* a = nullptr;
        VB_CUDA(cudaGetSymbolAddress(&a, g_sched));
        base[dev] = static_cast<unsigned*>(a);
    }
    const auto key = std::make_tuple(dev, s, s == cudaStreamPerThread ? std::this_thread::get_id() : std::thread::id());
    auto it = slot.find(key);
    if (it == slot.end()) {
        if (used[dev] == kSchedSlots) return nullptr;
        it = slot.emplace(key, used[dev]++).first;
    }
    return base[dev] + 2 * it->second;
}

int sm_count() { return device_sm_count(); }

template <int BN, int STAGES, int EPI, bool PAIR, int LN>
void launch(const k::GemmArgs<__half>& a, cudaStream_t s, unsigned* sched) {
    using L = Layout<BN, STAGES, EPI, PAIR>;
    static std::atomic<uint64_t> configured{0};  // per instantiation and device
    once_per_device(configured, [] {
        VB_CUDA(cudaFuncSetAttribute(gemm_tc_kernel<BN, STAGES, EPI, PAIR, LN>,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize, L::kSmem));
    });
    const CUtensorMap ta = make_map(a.A, a.M, a.K, a.lda, BM);
    const CUtensorMap tb = make_map(a.W, a.N, a.K, a.ldw, PAIR ? BN / 2 : BN);
    // 32 x 32 sub-tiles of the output, 64-byte swizzle: the epilogue's TMA stores
    const CUtensorMap tc = make_map(a.C, a.M, a.N, a.ldc, 32, 32, CU_TENSOR_MAP_SWIZZLE_64B);
    Params p{a.bias, a.C, a.ldc, a.R, a.ldr, int(a.M), int(a.N), int(a.K), a.epi, a.gelu_tanh ? 1 : 0, sched,
             a.st_out, int(a.N / (BN / 2)), a.st_in, a.colsum, a.nseg_in, float(a.segw_in), a.eps};
    constexpr int UM = PAIR ? 2 * BM : BM;
    const int64_t tiles = ((a.M + UM - 1) / UM) * ((a.N + BN - 1) / BN);
    if (!PAIR) {
        const int grid = int(std::min<int64_t>(tiles, sm_count()));
        gemm_tc_kernel<BN, STAGES, EPI, PAIR, LN><<<grid, kThreads, L::kSmem, s>>>(ta, tb, tc, p);
        VB_LAUNCH();
        return;
    }
    // clusters of two CTAs, one pair per two SMs
    const int pairs = int(std::min<int64_t>(tiles, sm_count() / 2));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(unsigned(2 * pairs));
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = size_t(L::kSmem);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2, attr[0].val.clusterDim.y = 1, attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr, cfg.numAttrs = 1;
    VB_CUDA(cudaLaunchKernelEx(&cfg, gemm_tc_kernel<BN, STAGES, EPI, PAIR, LN>, ta, tb, tc, p));
    ++launch_counter();
}

// the LayerNorm variant: records written by bias and residual epilogues, the fold applied by bias and
// GELU epilogues (supported() rejects the other combinations)
template <int BN, int STAGES, int EPI, bool PAIR>
void dispatch_ln(const k::GemmArgs<__half>& a, cudaStream_t s, unsigned* sched) {
    if constexpr (EPI != k::kEpiResidual) {
        if (a.st_in) return launch<BN, STAGES, EPI, PAIR, kLnFold>(a, s, sched);
    }
    if constexpr (EPI != k::kEpiGelu) {
        if (a.st_out) return launch<BN, STAGES, EPI, PAIR, kLnStats>(a, s, sched);
    }
    launch<BN, STAGES, EPI, PAIR, kLnNone>(a, s, sched);
}

// stage counts: as deep as the 227 KB of shared memory allows next to the epilogue staging
template <int BN, int EPI>
void dispatch_pair(const k::GemmArgs<__half>& a, cudaStream_t s, unsigned* sched) {
    if constexpr (BN == 256) {
        // CTA pairs (cta_group::2) for N > 128 unless VB_GEMM_PAIR=0: on C1's shapes 3-8% faster than
        // single CTAs (each SM loads half of W per tile: a third less L2-to-SM traffic)
        const char* pe = std::getenv("VB_GEMM_PAIR");
        if (!(pe && *pe && std::atoi(pe) == 0) && a.M >= 2 * BM) return dispatch_ln<BN, 6, EPI, true>(a, s, sched);
        return dispatch_ln<BN, 4, EPI, false>(a, s, sched);
    } else {
        return dispatch_ln<BN, 6, EPI, false>(a, s, sched);
    }
}

template <int BN>
void dispatch_epi(const k::GemmArgs<__half>& a, cudaStream_t s, unsigned* sched) {
    switch (a.epi) {
        case k::kEpiBias: dispatch_pair<BN, k::kEpiBias>(a, s, sched); break;
        case k::kEpiGelu: dispatch_pair<BN, k::kEpiGelu>(a, s, sched); break;
        case k::kEpiResidual: dispatch_pair<BN, k::kEpiResidual>(a, s, sched); break;
        default: fail(kInvalidArgument, "gemm: unknown epilogue");
    }
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace

bool supported(const k::GemmArgs<__half>& a) {
    if (a.M <= 0 || a.N <= 0 || a.K <= 0) return false;
    if (a.M > INT32_MAX / 2 || a.N > INT32_MAX / 2 || a.K > INT32_MAX / 2) return false;
    if (a.lda % 8 || a.ldw % 8 || a.ldc % 8) return false;
    if (!aligned16(a.A) || !aligned16(a.W) || !aligned16(a.C)) return false;
    if (a.bias && !aligned16(a.bias)) return false;
    if (a.epi == k::kEpiResidual && (!a.R || a.ldr % 8 || !aligned16(a.R))) return false;
    // LayerNorm fusion: records of whole segments, from bias / residual epilogues; the fold with its
    // column sums and bias, at most kMaxSegs records per row, in bias / GELU epilogues
    if (a.st_out && (a.epi == k::kEpiGelu || a.N % stats_segw(a.N) || !aligned16(a.st_out))) return false;
    if (a.st_in && (a.st_out || a.epi == k::kEpiResidual || !a.colsum || !a.bias || a.nseg_in < 1 ||
                    a.nseg_in > kMaxSegs || a.segw_in < 1 || !aligned16(a.colsum) ||
                    (reinterpret_cast<uintptr_t>(a.st_in) & 7)))
        return false;
    return true;
}

void gemm(const k::GemmArgs<__half>& a, cudaStream_t s) { gemm(a, s, sched_counter(s)); }

void gemm(const k::GemmArgs<__half>& a, cudaStream_t s, unsigned* sched) {
    if (!supported(a)) fail(kInvalidArgument, "tensor-core gemm: unsupported operand alignment");
    if (a.N <= 128) dispatch_epi<128>(a, s, sched);
    else dispatch_epi<256>(a, s, sched);
}

int take_error() {
    VB_CUDA(cudaDeviceSynchronize());
    int e = 0, zero = 0;
    VB_CUDA(cudaMemcpyFromSymbol(&e, g_error, sizeof(int)));
    if (e) VB_CUDA(cudaMemcpyToSymbol(g_error, &zero, sizeof(int)));
    return e;
}

CUtensorMap tensor_map_2d(const __half* base, int64_t rows, int64_t cols, int64_t ld, int box_rows, int box_cols,
                          CUtensorMapSwizzle swz) {
    return make_map(base, rows, cols, ld, box_rows, box_cols, swz);
}

}  // namespace vb::tc
