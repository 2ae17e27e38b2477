// cuda_backend.h -- ft::IBackend for one B200 over libftcuda.so (include/ftc.h).
//
// The drop-in for the reference's CpuBackend / VulkanBackend
// (ft/include/ft/cpu_backend.h, ft/include/ft/vulkan_backend.h): construct it
// where the engine builds its accelerator backend (ft/src/engine.cpp:
// 291-300); a construction failure throws std::runtime_error and the engine
// keeps its CPU backend, as it does for Vulkan.
#pragma once

#include <string>
#include <vector>

#include "ft/backend.h"
#include "ft/gguf.h"

struct ftc_backend;

namespace ft {

// The two layouts an FFN down-projection weight comes in.  The reference's
// engine and test files store it neuron-major, n_ff rows of n_embd weights,
// and multiply with ft::matmul_down_axpy (ft/src/cpu_backend.cpp:60-75;
// ft/src/tests/test_core.cpp:164 writes ffn_down_exps with ne = (D, FF, E));
// standard GGUF files store it output-major, n_embd rows of n_ff weights,
// the layout every other projection has.
enum class DownLayout { NeuronRows, OutputRows };

// The layout of W by its shape: n_ff rows -> NeuronRows (also when W is
// square: the reference's convention); n_ff columns -> OutputRows.  Throws
// std::runtime_error when neither dimension is n_ff.
DownLayout down_layout(const HostTensor& W, int64_t n_ff);

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

    // ft::matmul_down_axpy on the GPU: y[m] += x_m . W over the first n_in
    // rows of W (W.cols() weights each; zero activations skipped); x host fp32
    // [M][n_in], y host fp32 [M][W.cols()] accumulated.  Replaces the free
    // function the engine calls beside the interface (ft/src/engine.cpp:256,
    // 275).  Throws when n_in exceeds W.rows().
    void matmul_down_axpy(const float* x, int64_t M, int64_t n_in, const HostTensor& W, float* y);

    // The engine's FFN down projection in either layout: y[m] += h_m . down,
    // h host fp32 [M][n_ff], y host fp32 [M][n_embd] accumulated.  NeuronRows
    // weights go through matmul_down_axpy, OutputRows weights through matmul
    // (the dequant GEMV / GEMM of every other projection).
    void down_project(const float* h, int64_t M, int64_t n_ff, const HostTensor& W, float* y);

    // The routed experts of the engine's moe_ffn (ft/src/engine.cpp:179-241)
    // after its router matmul, on the device (ftc_backend_moe_ffn): routing
    // with the router bias (empty: none), token grouping, the expert FFNs and
    // the weighted combine, added into tmpo [M][n_embd].  xn [M][n_embd] and
    // router [M][E] are the engine's host buffers; the expert tensors are the
    // model's gate_exps / up_exps / down_exps.  Returns false, touching
    // nothing, when moe_supported() says no (the engine then keeps its
    // ExpertStreamer loop, whose run_expert_chunk also runs here).
    bool moe_ffn(const float* xn, const float* router, const std::vector<float>& rbias, int64_t M,
                 int64_t n_expert_used, const HostTensor& gexps, const HostTensor& uexps,
                 const HostTensor& dexps, float* tmpo);
    // Q4_K expert planes with the down projection in the standard layout
    // (n_embd rows of n_ff weights per expert), 1..256 experts, n_embd and
    // n_ff multiples of 256, n_ff <= 49152.  moe_ffn also needs
    // 1 <= n_expert_used <= 8.
    static bool moe_supported(const HostTensor& gexps, const HostTensor& uexps,
                              const HostTensor& dexps);

    // The engine's KV cache in HBM (ft::KvCache::alloc, ft/include/ft/
    // kv_cache.h:12-20): n_layers x capacity rows of dim floats for K and V.
    void kv_alloc(int64_t n_layers, int64_t capacity, int64_t dim);
    // One layer of the engine's attention step (ft/src/engine.cpp:553-566):
    // with write_kv the block's k / v rows ([M][n_head_kv * head_dim], after
    // RoPE) are stored into the device cache at rows [base, base + M), then
    // Engine::Impl::attn's causal grouped-query attention of q ([M][n_head *
    // head_dim], after RoPE) over rows [0, base + M) writes attout.  Host
    // buffers, synchronous; head_dim 64, 128 or 256.
    void attention(int64_t layer, int64_t base, int64_t M, int64_t n_head, int64_t n_head_kv,
                   int64_t head_dim, const float* q, const float* k, const float* v,
                   bool write_kv, float* attout);
    // Rows [pos0, pos0 + n) of a layer of the device cache to / from host
    // [n][dim] buffers: the copies of the engine's prefix cache
    // (ft/src/engine.cpp:608-616 restore, 630-645 snapshot).
    void kv_read(int64_t layer, int64_t pos0, int64_t n, float* k, float* v);
    void kv_write(int64_t layer, int64_t pos0, int64_t n, const float* k, const float* v);

    // Load a tensor's blocks into HBM once (call at Engine::load time).  The
    // host blocks must stay mapped and unchanged until evict() or the
    // backend's destruction; tensors never uploaded are copied per call.
    void upload(const HostTensor& t);
    // Drop the HBM copy of an uploaded tensor (before its host memory goes).
    void evict(const HostTensor& t);
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
