// Tensor-core GEMM for sm_100a (tcgen05 + TMEM + TMA): y[M, N] = A[M, K] W[N, K]^T with fp16
// operands, fp32 accumulation in tensor memory, and the fused epilogues of kernels.cuh
// (bias, GELU, residual; LayerNorm records written or a folded LayerNorm applied) applied when the
// accumulator is read back.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "kernels.cuh"

namespace vb::tc {

// True when the operands meet the tensor-memory-access rules: 16-byte aligned base pointers and
// row strides (multiples of 8 fp16 elements).
bool supported(const k::GemmArgs<__half>& a);
// Width of the LayerNorm segment records a GEMM with N output columns writes (st_out): one column
// half of its output tile, 64 for N <= 128, else 128.
inline int stats_segw(int64_t N) { return N <= 128 ? 64 : 128; }
// Enqueues the GEMM on s (no allocation, no synchronisation; capturable). Static tile order, or with
// VB_GEMM_SCHED=1 the dynamic order on a counter kept per (device, stream, thread).
void gemm(const k::GemmArgs<__half>& a, cudaStream_t s);
// The same with the dynamic tile order on the caller's counter: two unsigned words in device memory,
// zero before the first launch and left zero by each launch; launches that may run at the same time
// must not share one. nullptr: the static order. Both orders give the same bits.
void gemm(const k::GemmArgs<__half>& a, cudaStream_t s, unsigned* sched);
// Reads and clears the device-side error flag set when a bounded wait inside the kernel gave up
// (synchronises the device). Returns 0 when no wait timed out.
int take_error();

// 2-D fp16 tensor map over a row-major [rows, cols] matrix with leading dimension ld (elements):
// box [box_rows, box_cols] with the given shared-memory swizzle; out-of-bounds loads read zeros.
CUtensorMap tensor_map_2d(const __half* base, int64_t rows, int64_t cols, int64_t ld, int box_rows, int box_cols,
                          CUtensorMapSwizzle swz);

}  // namespace vb::tc
