// CUDA-core GEMM y[M, N] = A[M, K] W[N, K]^T (+ bias) with fp32 accumulation and the fused
// epilogues of kernels.cuh. Used for fp32 mode, where the reference requires true fp32 FMA
// (its cuBLASLt plan uses CUBLAS_COMPUTE_32F without TF32), and for shapes the tensor-core GEMM
// does not take. 128 x 128 x 16 tiles, 256 threads, 8 x 8 outputs per thread.
#include <algorithm>

#include "common.h"
#include "dev.cuh"
#include "kernels.cuh"

namespace vb::k {

using namespace vb::d;

namespace {

constexpr int BM = 128, BN = 128, BK = 16;

template <class T>
__device__ __forceinline__ float epilogue(float acc, const GemmArgs<T>& a, int64_t m, int64_t n) {
    float y = a.bias ? acc + to_f<T>(a.bias[n]) : acc;
    y = rnd<T>(y);
    if (a.epi == kEpiGelu) {
        y = rnd<T>(gelu(y, a.gelu_tanh));
    } else if (a.epi == kEpiResidual) {
        y = rnd<T>(y + to_f<T>(a.R[m * a.ldr + n]));
    }
    return y;
}

template <class T>
__global__ void __launch_bounds__(256) gemm_simt_kernel(GemmArgs<T> a) {
    __shared__ float As[BK][BM + 4];
    __shared__ float Bs[BK][BN + 4];
    const int t = threadIdx.x;
    const int tx = t & 15, ty = t >> 4;
    const int64_t m0 = int64_t(blockIdx.y) * BM, n0 = int64_t(blockIdx.x) * BN;
    float acc[8][8];
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = 0.f;

    const int lrow = t >> 1, lk = (t & 1) * 8;
    const int64_t am = m0 + lrow, bn = n0 + lrow;
    for (int64_t k0 = 0; k0 < a.K; k0 += BK) {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int64_t kk = k0 + lk + i;
            As[lk + i][lrow] = (am < a.M && kk < a.K) ? to_f<T>(a.A[am * a.lda + kk]) : 0.f;
            Bs[lk + i][lrow] = (bn < a.N && kk < a.K) ? to_f<T>(a.W[bn * a.ldw + kk]) : 0.f;
        }
        __syncthreads();
#pragma unroll
        for (int kk = 0; kk < BK; ++kk) {
            float av[8], bv[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) av[i] = As[kk][ty + 16 * i];
#pragma unroll
            for (int j = 0; j < 8; ++j) bv[j] = Bs[kk][tx + 16 * j];
#pragma unroll
            for (int i = 0; i < 8; ++i)
#pragma unroll
                for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int64_t m = m0 + ty + 16 * i;
        if (m >= a.M) continue;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int64_t n = n0 + tx + 16 * j;
            if (n < a.N) a.C[m * a.ldc + n] = from_f<T>(epilogue(acc[i][j], a, m, n));
        }
    }
}

}  // namespace

template <class T>
void gemm_simt(const GemmArgs<T>& a, cudaStream_t s) {
    if (a.M <= 0 || a.N <= 0) return;
    if (a.epi == kEpiResidual && !a.R) fail(kInvalidArgument, "gemm: residual epilogue without a residual");
    const int64_t gy = (a.M + BM - 1) / BM;
    if (gy > 65535 * 1024LL) fail(kUnsupported, "gemm: M too large");
    dim3 grid(unsigned((a.N + BN - 1) / BN), unsigned(gy));
    gemm_simt_kernel<T><<<grid, 256, 0, s>>>(a);
    VB_LAUNCH();
}

template void gemm_simt<float>(const GemmArgs<float>&, cudaStream_t);
template void gemm_simt<__half>(const GemmArgs<__half>&, cudaStream_t);

}  // namespace vb::k
