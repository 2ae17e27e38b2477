// expert.cu -- the reference-layout expert chunk on the device.
//
// ft::CpuBackend::run_expert_chunk (ft/src/cpu_backend.cpp:106-149):
//   phase A  h[m][i]   = silu(x_m . gate_i) * (x_m . up_i)       (two GEMVs
//            from gemv.cu, then silu_mul below)
//   phase B  out[m][k] += sum_i h[m][i] * down_i[k]   down_i = row i of the
//            window, K weights long (the reference's neuron-major layout)
#include <algorithm>

#include "common.cuh"

namespace ftc {

int mul_mat_vec(int dtype, const void* w, int64_t N, int64_t K, int64_t row_stride,
                const float* x, int64_t M, float* y, cudaStream_t st);

namespace {

// silu(g) = g / (1 + exp(-g)), as ft/src/cpu_backend.cpp:127.
__global__ void silu_mul(const float* __restrict__ g, const float* __restrict__ u,
                         float* __restrict__ h, int64_t n) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
        const float gv = g[i];
        h[i] = (gv / (1.f + expf(-gv))) * u[i];
    }
}

// out[m][k] += sum_i h[m][i] * D_i[k]: one thread per column k, walking the
// IC rows in order (the reference's i loop) with its own fp32 sum, added to
// out at the end.
template <int MT>
__global__ void __launch_bounds__(256)
down_rows_axpy(int dtype, const uint8_t* __restrict__ D, int64_t stride, int64_t IC, int64_t K,
               const float* __restrict__ h, int64_t M, float* __restrict__ out) {
    const int64_t k = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int64_t m0 = (int64_t)blockIdx.y * MT;
    if (k >= K) return;
    float acc[MT];
#pragma unroll
    for (int t = 0; t < MT; ++t) acc[t] = 0.f;
    for (int64_t i = 0; i < IC; ++i) {
        const float w = decode_elem(dtype, D + i * stride, k);
#pragma unroll
        for (int t = 0; t < MT; ++t)
            if (m0 + t < M) acc[t] = fmaf(h[(m0 + t) * IC + i], w, acc[t]);
    }
#pragma unroll
    for (int t = 0; t < MT; ++t)
        if (m0 + t < M) out[(m0 + t) * K + k] += acc[t];
}

}  // namespace

// Device pointers throughout; gbuf/ubuf/hbuf hold M*IC floats each.
int expert_chunk_dev(int dtype, const float* x, float* out, const void* gate, const void* up,
                     const void* down, int64_t M, int64_t K, int64_t IC, int64_t gu_stride,
                     int64_t dn_stride, float* gbuf, float* ubuf, float* hbuf, cudaStream_t st) {
    for (int64_t m0 = 0; m0 < M; m0 += 8) {
        const int64_t mc = std::min<int64_t>(8, M - m0);
        int rc = mul_mat_vec(dtype, gate, IC, K, gu_stride, x + m0 * K, mc, gbuf + m0 * IC, st);
        if (rc) return rc;
        rc = mul_mat_vec(dtype, up, IC, K, gu_stride, x + m0 * K, mc, ubuf + m0 * IC, st);
        if (rc) return rc;
    }
    const int64_t n = M * IC;
    silu_mul<<<(unsigned)std::min<int64_t>((n + 255) / 256, 148 * 16), 256, 0, st>>>(gbuf, ubuf,
                                                                                   hbuf, n);
    constexpr int MT = 4;
    dim3 grid((unsigned)((K + 255) / 256), (unsigned)((M + MT - 1) / MT));
    down_rows_axpy<MT><<<grid, 256, 0, st>>>(dtype, static_cast<const uint8_t*>(down), dn_stride,
                                             IC, K, hbuf, M, out);
    FTC_CUDA(cudaGetLastError());
    return FTC_OK;
}

}  // namespace ftc
