// rows.cu -- activation-row helpers for chained dequant-matmuls on fp16
// tensor-core operands (the tensor-parallel block and other callers):
//
//   rows_to_f16   out[m] = fp16(x[m] * 2^-e[m]) with e[m] chosen so that
//                 max|x[m]| * 2^-e[m] lies in [2^14, 2^15): fp16 keeps 11
//                 significant bits for rows of any magnitude; the GEMM
//                 epilogue multiplies its output rows by 2^e[m] (exact).
//   silu_mul      h = silu(g) * u in fp32, g / (1 + exp(-g)) as the
//                 reference's expert FFN (ft/src/cpu_backend.cpp:127).
//   silu_mul_rows the same on rows holding [gate | up] side by side (the
//                 output of one matmul over stacked gate and up weights),
//                 into fp32 rows, or straight into fp16 rows with their
//                 power-of-two scales (bit for bit rows_to_f16 of the fp32
//                 result).
//   copy_f32      a small float copy as a kernel, for the per-call host-buffer
//                 path: x from pinned host memory into device memory (reached
//                 through unified addressing), so that the launch behind it
//                 on the same stream can start early instead of waiting for a
//                 copy engine.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>

#include "common.cuh"
#include "sm100.cuh"

namespace ftc {
namespace {

// dst[i] = src[i]; 16-byte moves when both are 16-byte aligned.  The next
// grid on the stream may start at once (programmatic dependent launch); it
// reads dst only after its griddepcontrol.wait, i.e. after this grid ends.
__global__ void copy_f32_kernel(float* __restrict__ dst, const float* __restrict__ src, int64_t n,
                                int vec) {
    grid_launch_dependents();
    const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int64_t nth = (int64_t)gridDim.x * blockDim.x;
    if (vec) {
        const int64_t n4 = n / 4;
        for (int64_t i = tid; i < n4; i += nth)
            reinterpret_cast<float4*>(dst)[i] = reinterpret_cast<const float4*>(src)[i];
        for (int64_t i = 4 * n4 + tid; i < n; i += nth) dst[i] = src[i];
    } else {
        for (int64_t i = tid; i < n; i += nth) dst[i] = src[i];
    }
}

__device__ __forceinline__ float to_f(float v) { return v; }
__device__ __forceinline__ float to_f(__half v) { return __half2float(v); }
__device__ __forceinline__ float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }

template <typename TI>
__global__ void rows_to_f16_kernel(const TI* __restrict__ x, int64_t ld, int K,
                                   __half* __restrict__ out, int32_t* __restrict__ row_exp) {
    grid_launch_dependents();  // a following GEMM / GEMV may start its prologue
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
    grid_launch_dependents();  // a following GEMM / GEMV may start its prologue
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
        const float gv = g[i];
        h[i] = gv / (1.f + expf(-gv)) * u[i];
    }
}

// fp32 rows: h[m][k] = silu(gu[m][k]) * gu[m][n + k], grid-stride over all
// elements (decode-sized M has too few rows for one CTA per row).
__global__ void silu_mul_rows_f32(const float* __restrict__ gu, int64_t ld, int64_t rows, int n,
                                  float* __restrict__ h) {
    grid_launch_dependents();  // a following GEMM / GEMV may start its prologue
    const int64_t total = rows * n;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t m = i / n, k = i - m * n;
        const float* g = gu + m * ld;
        h[i] = silu_gate(g[k], g[n + k]);
    }
}

// fp16 rows scaled as rows_to_f16: one CTA per row; the row's silu values
// are kept in shared memory between the max and the scaling pass when they
// fit (cache = true), else recomputed (same arithmetic, same bits).
template <bool kCache>
__global__ void __launch_bounds__(1024)
silu_mul_rows_f16(const float* __restrict__ gu, int64_t ld, int n, __half* __restrict__ out16,
                  int32_t* __restrict__ row_exp) {
    grid_launch_dependents();  // a following GEMM / GEMV may start its prologue
    extern __shared__ float hs[];
    __shared__ float red[32];
    const float* g = gu + (int64_t)blockIdx.x * ld;
    const float* u = g + n;
    float amax = 0.f;
    for (int k = threadIdx.x; k < n; k += blockDim.x) {
        const float v = silu_gate(g[k], u[k]);
        if (kCache) hs[k] = v;
        amax = fmaxf(amax, fabsf(v));
    }
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = amax;
    __syncthreads();
    float m = 0.f;
    for (int i = 0; i < (int)(blockDim.x >> 5); ++i) m = fmaxf(m, red[i]);
    int e = 0;
    if (m > 0.f && isfinite(m))
        e = max(-126, min(126, (int)((__float_as_uint(m) >> 23) & 0xFF) - 127 - 14));
    const float sc = __uint_as_float((uint32_t)(127 - e) << 23);
    __half2* dst = reinterpret_cast<__half2*>(out16 + (int64_t)blockIdx.x * n);
    for (int k = 2 * threadIdx.x; k < n; k += 2 * blockDim.x) {
        const float a = kCache ? hs[k] : silu_gate(g[k], u[k]);
        const float b = kCache ? hs[k + 1] : silu_gate(g[k + 1], u[k + 1]);
        dst[k >> 1] = __floats2half2_rn(a * sc, b * sc);
    }
    if (threadIdx.x == 0) row_exp[blockIdx.x] = e;
}

constexpr int kSiluCacheMax = 48 * 1024;  // row values kept in shared memory (192 KB)

}  // namespace

int silu_mul_rows(const float* gu, int64_t rows, int64_t n, int64_t ld, float* h, void* out16,
                  int32_t* row_exp, cudaStream_t st) {
    FTC_REQUIRE(gu && (h || (out16 && row_exp)), FTC_E_INVALID, "ftc_silu_mul_rows: null pointer");
    FTC_REQUIRE(rows >= 0 && rows <= INT32_MAX && n > 0 && n <= INT32_MAX && ld >= 2 * n,
                FTC_E_INVALID, "ftc_silu_mul_rows: bad shape (ld >= 2n)");
    FTC_REQUIRE(h || (n % 2 == 0 && (uintptr_t)out16 % 4 == 0), FTC_E_INVALID,
                "ftc_silu_mul_rows: fp16 rows need an even n and 4-byte alignment");
    if (rows == 0) return FTC_OK;
    if (h) {
        const int sms = device_sms();
        const int64_t total = rows * n;
        const int grid = (int)std::max<int64_t>(1, std::min<int64_t>((total + 255) / 256, (int64_t)sms * 8));
        silu_mul_rows_f32<<<grid, 256, 0, st>>>(gu, ld, rows, (int)n, h);
    } else if (n <= kSiluCacheMax) {
        const int orc = opt_in_smem(reinterpret_cast<const void*>(silu_mul_rows_f16<true>),
                                    kSiluCacheMax * (int)sizeof(float),
                                    "cudaFuncSetAttribute(silu_mul_rows_f16)");
        if (orc) return orc;
        silu_mul_rows_f16<true><<<(int)rows, 1024, (size_t)n * sizeof(float), st>>>(
            gu, ld, (int)n, static_cast<__half*>(out16), row_exp);
    } else {
        silu_mul_rows_f16<false><<<(int)rows, 1024, 0, st>>>(gu, ld, (int)n,
                                                             static_cast<__half*>(out16), row_exp);
    }
    FTC_CUDA(cudaGetLastError());
    return FTC_OK;
}

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

int copy_f32(float* dst, const float* src, int64_t n, cudaStream_t st) {
    FTC_REQUIRE(dst && src && n >= 0, FTC_E_INVALID, "copy_f32: bad argument");
    if (n == 0) return FTC_OK;
    const int vec = ((uintptr_t)dst % 16 == 0 && (uintptr_t)src % 16 == 0) ? 1 : 0;
    // one 16-byte move per thread: every load of a pinned source is in
    // flight at once, so the copy costs about one PCIe round trip
    const int64_t per = vec ? 4 : 1;
    const int grid = (int)std::max<int64_t>(
        1, std::min<int64_t>((n + 256 * per - 1) / (256 * per), (int64_t)device_sms()));
    copy_f32_kernel<<<grid, 256, 0, st>>>(dst, src, n, vec);
    FTC_CUDA(cudaGetLastError());
    return FTC_OK;
}

int silu_mul(const float* g, const float* u, int64_t n, float* h, cudaStream_t st) {
    FTC_REQUIRE(g && u && h && n >= 0, FTC_E_INVALID, "ftc_silu_mul: bad argument");
    if (n == 0) return FTC_OK;
    const int sms = device_sms();
    const int grid = (int)std::max<int64_t>(1, std::min<int64_t>((n + 255) / 256, (int64_t)sms * 8));
    silu_mul_kernel<<<grid, 256, 0, st>>>(g, u, n, h);
    FTC_CUDA(cudaGetLastError());
    return FTC_OK;
}

}  // namespace ftc
