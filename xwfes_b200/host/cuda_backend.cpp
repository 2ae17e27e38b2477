// cuda_backend.cpp -- ft::IBackend over the ftc_backend_* C ABI.
#include "cuda_backend.h"

#include <stdexcept>
#include <string>
#include <vector>

#include "ftc.h"

namespace ft {
namespace {

// The reference reports backend failures as std::runtime_error
// (e.g. ft/src/vulkan_backend.cpp:87-322); so does this adapter.
void check(int rc, const char* what) {
    if (rc != FTC_OK)
        throw std::runtime_error(std::string("cuda backend: ") + what + ": " + ftc_last_error());
}

}  // namespace

DownLayout down_layout(const HostTensor& W, int64_t n_ff) {
    if (W.rows() == n_ff) return DownLayout::NeuronRows;
    if (W.cols() == n_ff) return DownLayout::OutputRows;
    throw std::runtime_error("cuda backend: down weight " + W.name + " has no dimension of n_ff = " +
                             std::to_string(n_ff));
}

CudaBackend::CudaBackend(int device) {
    check(ftc_backend_create(device, &be_), "create");
    char name[256] = {0};
    uint64_t mem = 0;
    check(ftc_backend_info(be_, name, sizeof(name), &mem), "info");
    info_.name = name;
    info_.integrated = false;
    info_.uma = false;
    info_.mem_bytes = mem;
}

CudaBackend::~CudaBackend() { ftc_backend_destroy(be_); }

void CudaBackend::matmul(const float* x, int64_t M, int64_t K, const HostTensor& W, float* y) {
    if (K != W.cols()) throw std::runtime_error("cuda backend: matmul K != W.cols()");
    check(ftc_backend_matmul(be_, x, M, K, W.data, (int)W.dtype, W.rows(), y), "matmul");
}

void CudaBackend::run_expert_chunk(const ExpertChunkJob& job) {
    ftc_expert_chunk_job j;
    j.x = job.x;
    j.out = job.out;
    j.gate = job.gate;
    j.up = job.up;
    j.down = job.down;
    j.dtype = (int)job.dt;
    j.M = job.M;
    j.K = job.K;
    j.IC = job.IC;
    j.gate_up_row_stride = job.gate_up_row_stride;
    j.down_row_stride = job.down_row_stride;
    check(ftc_backend_run_expert_chunk(be_, &j), "run_expert_chunk");
}

void CudaBackend::sync() { check(ftc_backend_sync(be_), "sync"); }

void CudaBackend::matmul_down_axpy(const float* x, int64_t M, int64_t n_in, const HostTensor& W,
                                   float* y) {
    if (n_in > W.rows()) throw std::runtime_error("cuda backend: matmul_down_axpy n_in > W.rows()");
    check(ftc_backend_matmul_down_axpy(be_, x, M, n_in, W.data, (int)W.dtype, W.cols(), y),
          "matmul_down_axpy");
}

void CudaBackend::down_project(const float* h, int64_t M, int64_t n_ff, const HostTensor& W,
                               float* y) {
    if (down_layout(W, n_ff) == DownLayout::NeuronRows) {
        matmul_down_axpy(h, M, n_ff, W, y);
        return;
    }
    std::vector<float> t((size_t)(M * W.rows()));
    matmul(h, M, n_ff, W, t.data());
    for (size_t i = 0; i < t.size(); ++i) y[i] += t[i];
}

bool CudaBackend::moe_supported(const HostTensor& g, const HostTensor& u, const HostTensor& d) {
    const int64_t K = g.cols(), F = g.rows(), E = g.dim2();
    // type ids compared as GGML ids: the reference's own DType has no Q4_K
    // member until the K-quants are added to it
    const auto q4k = [](const HostTensor& t) { return (int)t.dtype == FTC_Q4_K; };
    // shapes the device MoE takes (ftc_moe_ffn): 1..256 experts, K and n_ff
    // whole super-blocks, n_ff <= 49152
    return q4k(g) && q4k(u) && q4k(d) && E >= 1 && E <= 256 && K % 256 == 0 && F % 256 == 0 &&
           F <= 49152 && u.cols() == K && u.rows() == F && u.dim2() == E && d.dim2() == E &&
           d.cols() == F && d.rows() == K && F != K;  // square: the reference's layout
}

bool CudaBackend::moe_ffn(const float* xn, const float* router, const std::vector<float>& rbias,
                          int64_t M, int64_t n_expert_used, const HostTensor& gexps,
                          const HostTensor& uexps, const HostTensor& dexps, float* tmpo) {
    if (!moe_supported(gexps, uexps, dexps) || n_expert_used < 1 || n_expert_used > 8)
        return false;
    const int64_t E = gexps.dim2();
    if (!rbias.empty() && (int64_t)rbias.size() != E)
        throw std::runtime_error("cuda backend: moe_ffn router bias size != n_experts");
    ftc_moe_desc d;
    d.dtype = FTC_Q4_K;
    d.n_experts = E;
    d.top_k = n_expert_used < E ? n_expert_used : E;  // std::min(n_expert_used, E), :183
    d.n_embd = gexps.cols();
    d.n_ff = gexps.rows();
    d.gate_exps = gexps.data;
    d.up_exps = uexps.data;
    d.down_exps = dexps.data;
    d.gu_row_stride = (int64_t)gexps.row_stride_bytes();
    d.gu_plane_stride = (int64_t)gexps.slice_bytes();
    d.dn_row_stride = (int64_t)dexps.row_stride_bytes();
    d.dn_plane_stride = (int64_t)dexps.slice_bytes();
    check(ftc_backend_moe_ffn(be_, &d, router, rbias.empty() ? nullptr : rbias.data(), xn, M, tmpo),
          "moe_ffn");
    return true;
}

void CudaBackend::kv_alloc(int64_t n_layers, int64_t capacity, int64_t dim) {
    check(ftc_backend_kv_alloc(be_, n_layers, capacity, dim), "kv_alloc");
}

void CudaBackend::attention(int64_t layer, int64_t base, int64_t M, int64_t n_head,
                            int64_t n_head_kv, int64_t head_dim, const float* q, const float* k,
                            const float* v, bool write_kv, float* attout) {
    check(ftc_backend_attention(be_, layer, base, M, n_head, n_head_kv, head_dim, q, k, v,
                                write_kv ? 1 : 0, attout),
          "attention");
}

void CudaBackend::kv_read(int64_t layer, int64_t pos0, int64_t n, float* k, float* v) {
    check(ftc_backend_kv_read(be_, layer, pos0, n, k, v), "kv_read");
}

void CudaBackend::kv_write(int64_t layer, int64_t pos0, int64_t n, const float* k,
                           const float* v) {
    check(ftc_backend_kv_write(be_, layer, pos0, n, k, v), "kv_write");
}

void CudaBackend::upload(const HostTensor& t) {
    const size_t n = t.nbytes ? t.nbytes
                              : t.slice_bytes() * (size_t)t.ne[2] * (size_t)t.ne[3];
    check(ftc_backend_upload(be_, t.data, n), "upload");
}

void CudaBackend::evict(const HostTensor& t) { check(ftc_backend_evict(be_, t.data), "evict"); }

size_t CudaBackend::upload_all(const Gguf& model) {
    size_t total = 0;
    for (const auto& kv : model.tensors()) {
        upload(kv.second);
        total += kv.second.nbytes;
    }
    return total;
}

}  // namespace ft
