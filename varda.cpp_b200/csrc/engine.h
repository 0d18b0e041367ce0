// The B200 backend behind the C ABI: one Engine per loaded model (fp32 or fp16), holding every
// device weight, graph and activation buffer, allocated at load. Interface mirrors the reference's
// varda::Backend / varda::cuda::CudaBackend (src/varda/backend.h:12-17, cuda/cuda_backend.h:31-75).
#pragma once

#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>
#include <memory>
#include <string>

namespace vb {

using HookFn = void (*)(const char* key, const float* data, const int64_t* shape, int ndim, void* user);
// Rollout output of step `step`: this rank's rows (rows, V_out) physical, host, valid during the call.
using StepFn = void (*)(int step, const float* y, int64_t rows, void* user);

struct Options {
    int precision = 0;  // 0 fp32, 1 fp16
    int cuda_device = 0;
    bool cuda_graph = true;
    int gemm = 0;                // 0 auto (tensor cores for fp16), 1 CUDA cores only
    int64_t dec_chunk_rows = 0;  // 0: all data rows in one chunk when memory allows
    // multi-GPU (destination partition); world == 1 for a single GPU
    int rank = 0, world = 1;
    const void* nccl_id = nullptr;  // 128-byte ncclUniqueId, the same on every rank
};

class Model {
public:
    virtual ~Model() = default;
    // host pointers, physical units: x (1, T_in, G, V_in), y (1, T_out, 1, G, V_out)
    virtual void predict_step(const float* x, float* y, HookFn hook, void* user) = 0;
    virtual int64_t input_numel() const = 0;
    virtual int64_t output_numel() const = 0;
    virtual void normalise(const float* x, float* xn, cudaStream_t s) = 0;
    virtual void forward_normalised(const float* xn, float* yn, cudaStream_t s) = 0;
    virtual void denormalise(const float* yn, float* y, cudaStream_t s) = 0;
    virtual void predict_step_device(const float* x, float* y, cudaStream_t s) = 0;
    virtual void prepare() = 0;
    virtual void use_high_priority_stream() = 0;
    virtual float* device_input() = 0;
    virtual const float* device_output() const = 0;
    virtual cudaStream_t stream() const = 0;
    virtual void enqueue_predict() = 0;
    virtual int device() const = 0;
    virtual size_t weight_bytes() const = 0;
    virtual size_t activation_bytes() const = 0;
    virtual int64_t decoder_chunk_rows() const = 0;
    // sizes: T_in, G, V_in, T_out, V_out, H, C, n_proc
    virtual void sizes(int64_t out[8]) const = 0;
    // multi-GPU: this rank's data-node range [lo, hi)
    virtual void data_range(int64_t* lo, int64_t* hi) const = 0;
    // multi-GPU: this rank's hidden-node range [lo, hi) (the processor's destination rows)
    virtual void hidden_range(int64_t* lo, int64_t* hi) const = 0;
    // The isolated processor block: LN_dst then processor block `block`, `repeats` times on the same
    // input, this rank's hidden rows (sharded: the K|V halo exchange every run, a collective). z_in /
    // z_out host fp32 [own hidden rows, C] or null (keep the previous call's input / no read-back);
    // device_ms: device time of the runs. Synchronises.
    virtual void processor_block(int block, const float* z_in, float* z_out, int repeats, float* device_ms) = 0;
    // One eager forward_normalised on the internal buffers with a CUDA event pair around every
    // launch; returns a JSON array of {"name", "ms", "flop", "bytes"} records (algorithmic FLOPs
    // of the GEMMs, compulsory bytes of the bandwidth-bound kernels). Synchronises.
    virtual std::string profile_forward() = 0;
    // The same for one run of processor_block(block) on the current block input.
    virtual std::string profile_block(int block) = 0;
    // Device-resident autoregressive rollout with replayed forcings (include/varda_b200.h vb_rollout):
    // x0 (1, T_in, G, V_in) and forcings (n_steps - 1, G, F) full host arrays; y (n_steps, G, V_out)
    // receives this rank's rows when not null; cb gets each step's rows when not null; step_ms
    // [n_steps] the GPU time of each step when not null.
    virtual void rollout(const float* x0, int n_steps, const float* forcings, float* y, bool constants_oldest,
                         StepFn cb, void* user, float* step_ms) = 0;
};

std::unique_ptr<Model> load_model(const std::string& path, const Options& opts);

}  // namespace vb
