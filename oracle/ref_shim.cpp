// ref_shim.cpp -- C entry points onto the reference's OWN CPU code, compiled
// from its sources (ft/src/cpu_backend.cpp + ft/include/ft/*.h) by
// oracle/Makefile into oracle/_ref/libftref.so.
//
// TEST INFRASTRUCTURE ONLY: used to pin the oracle (tests/, golden fixture
// generation) and as the timed "reference" CPU baseline in bench.py.
// Nothing here is reference source; it only calls it.
#include "ft/cpu_backend.h"
#include "ft/quant.h"

#include <cstdio>
#include <exception>

using namespace ft;

namespace {
HostTensor view(const void* data, uint32_t dtype, int64_t cols, int64_t rows) {
    HostTensor t;
    t.name = "ftref";
    t.ne[0] = cols;
    t.ne[1] = rows;
    t.n_dims = 2;
    t.dtype = (DType)dtype;
    t.data = (const uint8_t*)data;
    t.nbytes = dtype_row_bytes(t.dtype, cols) * (size_t)rows;
    return t;
}
}  // namespace

extern "C" {

float ftref_half_to_float(uint16_t h) { return half_to_float(h); }
uint16_t ftref_float_to_half(float f) { return float_to_half(f); }

// ft::dequant_row (ft/include/ft/quant.h:10-84); -1 if the reference throws.
int ftref_dequant_row(float* dst, const uint8_t* src, uint32_t dtype, int64_t n) {
    try { dequant_row(dst, src, (DType)dtype, n); return 0; }
    catch (const std::exception&) { return -1; }
}

// ft::dot_row_f32 (ft/include/ft/quant.h:86-103); -1 if the reference throws.
int ftref_dot_row_f32(const float* x, const uint8_t* w, uint32_t dtype, int64_t n, float* out) {
    try { *out = dot_row_f32(x, w, (DType)dtype, n); return 0; }
    catch (const std::exception&) { return -1; }
}

// ft::CpuBackend::matmul (ft/src/cpu_backend.cpp:90-104), unmodified: for
// M>1 it writes y[n] = sum_m dot(x_m, W_n) (the reference's batching).
int ftref_matmul(const float* x, int64_t M, int64_t K, const void* W, uint32_t dtype,
                 int64_t N, float* y, int threads) {
    try {
        CpuBackend cpu(threads);
        cpu.matmul(x, M, K, view(W, dtype, K, N), y);
        return 0;
    } catch (const std::exception&) { return -1; }
}

// ft::CpuBackend::run_expert_chunk (ft/src/cpu_backend.cpp:106-149).
int ftref_run_expert_chunk(const float* x, float* out, const void* gate, const void* up,
                           const void* down, uint32_t dtype, int64_t M, int64_t K, int64_t IC,
                           size_t gu_stride, size_t dn_stride, int threads) {
    try {
        CpuBackend cpu(threads);
        ExpertChunkJob job;
        job.x = x; job.out = out; job.gate = gate; job.up = up; job.down = down;
        job.dt = (DType)dtype; job.M = M; job.K = K; job.IC = IC;
        job.gate_up_row_stride = gu_stride; job.down_row_stride = dn_stride;
        cpu.run_expert_chunk(job);
        return 0;
    } catch (const std::exception&) { return -1; }
}

// ft::matmul_down_axpy (ft/src/cpu_backend.cpp:60-75): y[m] += x_m . W over
// n_in rows of N weights each.
int ftref_matmul_down_axpy(const float* x, int64_t M, int64_t n_in, const void* W, uint32_t dtype,
                           int64_t N, float* y) {
    try {
        matmul_down_axpy(x, M, n_in, view(W, dtype, N, n_in), y);
        return 0;
    } catch (const std::exception&) { return -1; }
}

}  // extern "C"
