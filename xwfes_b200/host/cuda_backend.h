// cuda_backend.h -- ft::IBackend for one B200 over libftcuda.so (include/ftc.h).
//
// The drop-in for the reference's CpuBackend / VulkanBackend
// (ft/include/ft/cpu_backend.h, ft/include/ft/vulkan_backend.h): construct it
// where the engine builds its accelerator backend (ft/src/engine.cpp:
// 291-300); a construction failure throws std::runtime_error and the engine
// keeps its CPU backend, as it does for Vulkan.
#pragma once

#include <string>

#include "ft/backend.h"
#include "ft/gguf.h"

struct ftc_backend;

namespace ft {

class CudaBackend : public IBackend {
public:
    explicit CudaBackend(int device = 0);
    ~CudaBackend() override;
    CudaBackend(const CudaBackend&) = delete;
    CudaBackend& operator=(const CudaBackend&) = delete;

    std::string name() const override { return info_.name; }
    DeviceInfo info() const override { return info_; }
    bool ready() const override { return be_ != nullptr; }

    // y[m][n] = x_m . W_n for every m (per-row outputs, y is [M][N]).
    void matmul(const float* x, int64_t M, int64_t K, const HostTensor& W, float* y) override;
    // h = silu(x.gate) * (x.up); out += h . down (down rows = neurons).
    void run_expert_chunk(const ExpertChunkJob& job) override;
    // No staging buffers: windows resolve through the HBM weight cache, so
    // the streamer passes mmap pointers straight through.
    void* alloc_staging(size_t) override { return nullptr; }
    void sync() override;

    // Load a tensor's blocks into HBM once (call at Engine::load time).
    void upload(const HostTensor& t);
    // Every tensor of a model file, blocks unchanged (the engine's load step,
    // ft/src/engine.cpp:282-396): later matmuls and expert chunks on these
    // tensors find their device copies instead of copying per call.
    // Returns the bytes uploaded.
    size_t upload_all(const Gguf& model);

private:
    ftc_backend* be_ = nullptr;
    DeviceInfo info_;
};

}  // namespace ft
