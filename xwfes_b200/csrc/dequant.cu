// dequant.cu -- element-wise dequantization of GGUF rows to fp32.
//
// The B200 form of ft::dequant_row (ft/include/ft/quant.h:10-84): one thread
// per weight, every weight written once.  It is the bit-exactness probe of
// the block decoders (tests compare it with the reference's own output) and
// the dequant stage of callers that want fp32 weights.
#include "common.cuh"

namespace ftc {
namespace {

__global__ void __launch_bounds__(256)
dequant_rows(int dtype, const uint8_t* __restrict__ W, int64_t stride, int64_t n_rows, int64_t K,
             float* __restrict__ out) {
    const int64_t total = n_rows * K;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = i / K, j = i - r * K;
        out[i] = decode_elem(dtype, W + r * stride, j);
    }
}

}  // namespace

int dequant(int dtype, const void* w, int64_t n_rows, int64_t k, int64_t row_stride, float* out,
            cudaStream_t st) {
    const Fmt f = fmt_of(dtype);
    FTC_REQUIRE(f.block_elems > 0, FTC_E_UNSUPPORTED, "ftc_dequant: unknown dtype");
    FTC_REQUIRE(w && out, FTC_E_INVALID, "ftc_dequant: null pointer");
    FTC_REQUIRE(n_rows >= 0 && k > 0 && k % f.block_elems == 0, FTC_E_INVALID,
                "ftc_dequant: k must be a positive whole number of blocks");
    FTC_REQUIRE(row_stride >= row_bytes(dtype, k), FTC_E_INVALID,
                "ftc_dequant: row_stride smaller than one row of blocks");
    if (inject_fail("ftc_dequant")) return set_error(FTC_E_INJECTED, "ftc_dequant: injected failure");
    if (n_rows == 0) return FTC_OK;
    const int64_t total = n_rows * k;
    const int64_t blocks = std::min<int64_t>((total + 255) / 256, 148 * 64);
    dequant_rows<<<(unsigned)blocks, 256, 0, st>>>(dtype, static_cast<const uint8_t*>(w),
                                                  row_stride, n_rows, k, out);
    FTC_CUDA(cudaGetLastError());
    return FTC_OK;
}

}  // namespace ftc
