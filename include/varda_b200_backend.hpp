// varda.cpp's CUDA backend interface implemented over libvarda_b200 (include/varda_b200.h).
//
// For a varda.cpp build: compile the reference's core (config, format, graph, model, cpu backend)
// with VARDA_WITH_CUDA defined and WITHOUT its src/varda/cuda/*.cu, add one translation unit
//
//     #define VARDA_B200_IMPLEMENT
//     #include "varda_b200_backend.hpp"
//
// and link libvarda_b200.so. Model::load(path, {Device::CUDA, ...}) then returns this backend
// (make_cuda_backend, src/varda/backend.h:25-26), varda::cuda::as_cuda works
// (src/varda/cuda/cuda_backend.h:78), and every caller of varda::Backend / varda::cuda::CudaBackend
// (varda-run, varda-parity, varda-bench, the rollout) runs unchanged on the B200 kernels.
//
// Needs the reference's headers (varda/backend.h, varda/cuda/cuda_backend.h) on the include path.
#pragma once

#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

#include "varda/backend.h"
#include "varda/cuda/cuda_backend.h"
#include "varda_b200.h"

namespace varda {
namespace b200 {

inline void check(int rc, const char* what) {
    if (rc != VB_OK) throw std::runtime_error(std::string(what) + ": " + vb_last_error());
}

class Backend final : public cuda::CudaBackend {
public:
    // The library maps and reads `file` itself (by path); the caller's mapping is marked consumed so
    // Model::load's strict require_all_consumed() (model.cpp:76) holds exactly as for the
    // reference's own backend, whose strict checks the library performs on its own mapping.
    Backend(const Config&, SafeTensorsFile& file, const Options& opts) {
        vb_options o{opts.precision == Precision::FP16 ? VB_PRECISION_FP16 : VB_PRECISION_FP32, opts.cuda_device,
                     opts.cuda_graph ? 1 : 0, opts.num_threads};
        check(vb_load(file.path().c_str(), &o, &m_), "vb_load");
        for (const std::string& n : file.unconsumed()) file.take(n);
    }
    ~Backend() override { vb_free(m_); }
    Backend(const Backend&) = delete;
    Backend& operator=(const Backend&) = delete;

    void predict_step(const float* x, float* y, const ActivationHook* hook) override {
        if (hook && *hook) check(vb_predict_step(m_, x, y, &hook_trampoline, const_cast<ActivationHook*>(hook)),
                                 "vb_predict_step");
        else check(vb_predict_step(m_, x, y, nullptr, nullptr), "vb_predict_step");
    }
    int64_t input_numel() const override { return io(0); }
    int64_t output_numel() const override { return io(1); }
    void normalise(const float* x, float* xn, cudaStream_t s) override { check(vb_normalise(m_, x, xn, s), "vb_normalise"); }
    void forward_normalised(const float* xn, float* yn, cudaStream_t s) override {
        check(vb_forward_normalised(m_, xn, yn, s), "vb_forward_normalised");
    }
    void denormalise(const float* yn, float* y, cudaStream_t s) override {
        check(vb_denormalise(m_, yn, y, s), "vb_denormalise");
    }
    void predict_step_device(const float* x, float* y, cudaStream_t s) override {
        check(vb_predict_step_device(m_, x, y, s), "vb_predict_step_device");
    }
    void prepare() override { check(vb_prepare(m_), "vb_prepare"); }
    void use_high_priority_stream() override { check(vb_use_high_priority_stream(m_), "vb_use_high_priority_stream"); }
    float* device_input() override { return vb_device_input(m_); }
    const float* device_output() const override { return vb_device_output(m_); }
    cudaStream_t stream() const override { return static_cast<cudaStream_t>(vb_stream(m_)); }
    void enqueue_predict() override { check(vb_enqueue_predict(m_), "vb_enqueue_predict"); }
    int device() const override { return vb_device(m_); }
    size_t weight_bytes() const override { return vb_weight_bytes(m_); }
    size_t activation_bytes() const override { return vb_activation_bytes(m_); }
    int64_t decoder_chunk_rows() const override { return vb_decoder_chunk_rows(m_); }

private:
    static void hook_trampoline(const char* key, const float* data, const int64_t* shape, int ndim, void* user) {
        (*static_cast<const ActivationHook*>(user))(key, data, std::vector<int64_t>(shape, shape + ndim));
    }
    int64_t io(int which) const {
        int64_t in = 0, out = 0;
        check(vb_io_numel(m_, &in, &out), "vb_io_numel");
        return which ? out : in;
    }
    vb_model* m_ = nullptr;
};

}  // namespace b200

#ifdef VARDA_B200_IMPLEMENT
std::unique_ptr<Backend> make_cuda_backend(const Config& cfg, SafeTensorsFile& file, const Options& opts) {
    return std::make_unique<b200::Backend>(cfg, file, opts);
}
namespace cuda {
CudaBackend* as_cuda(Model& m) { return dynamic_cast<CudaBackend*>(&m.backend()); }
}  // namespace cuda
#endif

}  // namespace varda
