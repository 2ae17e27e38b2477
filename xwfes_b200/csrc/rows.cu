// rows.cu -- activation-row helpers for chained dequant-matmuls on fp16
// tensor-core operands (the tensor-parallel block and other callers):
//
//   rows_to_f16   out[m] = fp16(x[m] * 2^-e[m]) with e[m] chosen so that
//                 max|x[m]| * 2^-e[m] lies in [2^14, 2^15): fp16 keeps 11
//                 significant bits for rows of any magnitude; the GEMM
//                 epilogue multiplies its output rows by 2^e[m] (exact).
//   silu_mul      h = silu(g) * u in fp32, g / (1 + exp(-g)) as the
//                 reference's expert FFN (ft/src/cpu_backend.cpp:127).
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>

#include "common.cuh"

namespace ftc {
namespace {

__device__ __forceinline__ float to_f(float v) { return v; }
__device__ __forceinline__ float to_f(__half v) { return __half2float(v); }
__device__ __forceinline__ float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }

template <typename TI>
__global__ void rows_to_f16_kernel(const TI* __restrict__ x, int64_t ld, int K,
                                   __half* __restrict__ out, int32_t* __restrict__ row_exp) {
    __shared__ float red[32];
    const TI* src = x + (int64_t)blockIdx.x * ld;
    float amax = 0.f;
    for (int k = threadIdx.x; k < K; k += blockDim.x) amax = fmaxf(amax, fabsf(to_f(src[k])));
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = amax;
    __syncthreads();
    float m = 0.f;
    for (int i = 0; i < (int)(blockDim.x >> 5); ++i) m = fmaxf(m, red[i]);
    int e = 0;
    if (m > 0.f && isfinite(m))
        e = max(-126, min(126, (int)((__float_as_uint(m) >> 23) & 0xFF) - 127 - 14));
    const float sc = __uint_as_float((uint32_t)(127 - e) << 23);
    __half2* dst = reinterpret_cast<__half2*>(out + (int64_t)blockIdx.x * K);
    for (int k = 2 * threadIdx.x; k < K; k += 2 * blockDim.x)
        dst[k >> 1] = __floats2half2_rn(to_f(src[k]) * sc, to_f(src[k + 1]) * sc);
    if (threadIdx.x == 0) row_exp[blockIdx.x] = e;
}

__global__ void silu_mul_kernel(const float* __restrict__ g, const float* __restrict__ u,
                                int64_t n, float* __restrict__ h) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
        const float gv = g[i];
        h[i] = gv / (1.f + expf(-gv)) * u[i];
    }
}

}  // namespace

int rows_to_f16(const void* x, int x_dtype, int64_t rows, int64_t K, int64_t ld, void* out,
                int32_t* row_exp, cudaStream_t st) {
    FTC_REQUIRE(x && out && row_exp, FTC_E_INVALID, "ftc_rows_to_f16: null pointer");
    FTC_REQUIRE(rows >= 0 && rows <= INT32_MAX && K > 0 && K % 2 == 0 && K <= INT32_MAX && ld >= K,
                FTC_E_INVALID, "ftc_rows_to_f16: bad shape (K even, ld >= K)");
    FTC_REQUIRE((uintptr_t)out % 4 == 0, FTC_E_INVALID, "ftc_rows_to_f16: out must be 4-byte aligned");
    if (rows == 0) return FTC_OK;
    const int r = (int)rows, k = (int)K;
    __half* o = static_cast<__half*>(out);
    if (x_dtype == FTC_F32)
        rows_to_f16_kernel<float><<<r, 256, 0, st>>>(static_cast<const float*>(x), ld, k, o, row_exp);
    else if (x_dtype == FTC_BF16)
        rows_to_f16_kernel<__nv_bfloat16><<<r, 256, 0, st>>>(static_cast<const __nv_bfloat16*>(x),
                                                             ld, k, o, row_exp);
    else if (x_dtype == FTC_F16)
        rows_to_f16_kernel<__half><<<r, 256, 0, st>>>(static_cast<const __half*>(x), ld, k, o,
                                                      row_exp);
    else
        return set_error(FTC_E_UNSUPPORTED, "ftc_rows_to_f16: x must be fp32, bf16 or fp16");
    FTC_CUDA(cudaGetLastError());
    return FTC_OK;
}

int silu_mul(const float* g, const float* u, int64_t n, float* h, cudaStream_t st) {
    FTC_REQUIRE(g && u && h && n >= 0, FTC_E_INVALID, "ftc_silu_mul: bad argument");
    if (n == 0) return FTC_OK;
    static int sms = 0;
    if (!sms) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, 0);
    const int grid = (int)std::max<int64_t>(1, std::min<int64_t>((n + 255) / 256, (int64_t)sms * 8));
    silu_mul_kernel<<<grid, 256, 0, st>>>(g, u, n, h);
    FTC_CUDA(cudaGetLastError());
    return FTC_OK;
}

}  // namespace ftc
