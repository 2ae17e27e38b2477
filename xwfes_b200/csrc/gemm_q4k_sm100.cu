// gemm_q4k_sm100.cu -- prefill dequant-GEMM on the 5th-generation tensor cores:
//
//   Y[m][n] = sum_k X[m][k] * W[n][k]     X: [M][K] bf16 (or fp16), W: Q4_K
//                                         Y: [M][N] bf16 / fp16 / fp32
//
// The B200 form of the reference's batched matmul (ft/src/cpu_backend.cpp:
// 90-104 with per-row semantics; its M>1 path folds rows together, which this
// does not).  Weights stay in their GGUF blocks in HBM; every weight tile is
// dequantized on the SM into shared memory right before the tensor cores
// read it, so no dequantized copy of W ever exists in global memory.
//
// One persistent CTA per SM, warp-specialized (14 warps):
//   warp 0      TMA: raw Q4_K tile (128 rows x one 144-byte super-block) into a
//               2-slot ring; activation tiles (BN tokens x 64 k, 128-byte
//               swizzle) into the NS-slot A/B ring.  Also owns TMEM.
//   warp 1      one thread issues tcgen05.mma 128 x BN x 16 (A = weights,
//               B = tokens, both K-major from shared memory) into a TMEM
//               accumulator (two of them, so the epilogue of tile i overlaps
//               the MMAs of tile i+1).
//   warps 2-5   epilogue: tcgen05.ld 32 lanes x 32 columns, convert, store
//               Y[token][row] (a warp writes 32 consecutive n per token).
//   warps 6-13  dequant: thread (row r, half h) decodes 32 weights of one
//               64-wide k-step (codes of group g, both nibbles) with the
//               block's scale/min into the 16-bit operand type and writes
//               them in the 128-byte-swizzled K-major layout the MMA reads.
// Every pipeline wait is bounded in time (sm100.cuh); a kernel that gives up
// records a status and returns.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <mutex>
#include <type_traits>

#include "common.cuh"
#include "sm100.cuh"

namespace ftc {

FTC_DEVSTAT_READER(devstat_gemm_q4k)

namespace {

constexpr int BM = 128;       // weight rows per tile (MMA M)
constexpr int BK = 64;        // k per stage: one 128-byte swizzle row of 16-bit values
constexpr int kRawSlots = 2;  // raw super-block ring
constexpr int kRawBytes = BM * 144;
constexpr int kThreads = 14 * 32;
constexpr int kDequantWarps = 8;
constexpr int kEpiWarps = 4;

template <int BN>
struct Cfg {
    static constexpr int NS = BN == 256 ? 3 : 4;  // A/B stages
    static constexpr int A_BYTES = BM * BK * 2;   // 16 KB
    static constexpr int B_BYTES = BN * BK * 2;
    static constexpr int TMEM_COLS = 2 * BN;      // two accumulators
    // shared layout (all tiles 1024-byte aligned)
    static constexpr int OFF_A = 0;
    static constexpr int OFF_B = OFF_A + NS * A_BYTES;
    static constexpr int OFF_RAW = OFF_B + NS * B_BYTES;
    static constexpr int OFF_BAR = OFF_RAW + kRawSlots * kRawBytes;
    // barriers: a_full[NS] b_full[NS] ab_empty[NS] raw_full[2] raw_empty[2] acc_full[2] acc_empty[2]
    static constexpr int N_BARS = 3 * NS + 8;
    static constexpr int SMEM = OFF_BAR + N_BARS * 8 + 16 + 1024;  // +1024: base alignment slack
};

template <typename T>
__device__ __forceinline__ uint32_t pack2(float a, float b);
template <>
__device__ __forceinline__ uint32_t pack2<__half>(float a, float b) {
    const __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&h);
}
template <>
__device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float a, float b) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&h);
}

// y element store in the requested output type
__device__ __forceinline__ void store_out(void* y, int ytype, int64_t idx, float v) {
    if (ytype == FTC_F32) reinterpret_cast<float*>(y)[idx] = v;
    else if (ytype == FTC_BF16) reinterpret_cast<__nv_bfloat16*>(y)[idx] = __float2bfloat16_rn(v);
    else reinterpret_cast<__half*>(y)[idx] = __float2half_rn(v);
}

template <int BN, typename OP>
__global__ void __launch_bounds__(kThreads, 1)
gemm_q4k_tc(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_x,
            int M, int N, int K, void* __restrict__ y, int ytype) {
    using C = Cfg<BN>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sA = smem + C::OFF_A;
    uint8_t* sB = smem + C::OFF_B;
    uint8_t* sRaw = smem + C::OFF_RAW;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
    uint64_t* a_full = bars;
    uint64_t* b_full = bars + C::NS;
    uint64_t* ab_empty = bars + 2 * C::NS;
    uint64_t* raw_full = bars + 3 * C::NS;
    uint64_t* raw_empty = raw_full + 2;
    uint64_t* acc_full = raw_full + 4;
    uint64_t* acc_empty = raw_full + 6;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + C::N_BARS);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < C::NS; ++s) {
            mbar_init(&a_full[s], kDequantWarps);
            mbar_init(&b_full[s], 1);
            mbar_init(&ab_empty[s], 1);
        }
        for (int s = 0; s < 2; ++s) {
            mbar_init(&raw_full[s], 1);
            mbar_init(&raw_empty[s], kDequantWarps);
            mbar_init(&acc_full[s], 1);
            mbar_init(&acc_empty[s], kEpiWarps);
        }
        *abort_flag = 0;
        mbar_fence_init();
    }
    if (warp == 0) {
        tmem_alloc(tmem_slot, C::TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    const int n_tiles = (N + BM - 1) / BM;
    const int t_tiles = (M + BN - 1) / BN;
    const int tiles = n_tiles * t_tiles;
    const int nsb = K / 256;

    if (warp == 0) {
        // ---------------------------------------------------------- TMA
        if (lane == 0) {
            prefetch_tensormap(&tm_w);
            prefetch_tensormap(&tm_x);
            const uint64_t pol_w = policy_evict_last();  // weights are re-read per token tile
            const uint64_t pol_x = policy_evict_last();
            uint32_t kc = 0, rc = 0;
            for (int tile = blockIdx.x; tile < tiles && !*abort_flag; tile += gridDim.x) {
                const int nt = tile % n_tiles, tt = tile / n_tiles;
                for (int sb = 0; sb < nsb; ++sb) {
                    const int rs = rc % kRawSlots;
                    if (!mbar_wait(&raw_empty[rs], ((rc / kRawSlots) & 1) ^ 1)) { *abort_flag = 1; break; }
                    mbar_arrive_expect_tx(&raw_full[rs], kRawBytes);
                    tma_load_2d(sRaw + rs * kRawBytes, &tm_w, sb * 144, nt * BM, &raw_full[rs], pol_w);
                    ++rc;
                    for (int g = 0; g < 4; ++g) {
                        const int s = kc % C::NS;
                        if (!mbar_wait(&ab_empty[s], ((kc / C::NS) & 1) ^ 1)) { *abort_flag = 1; break; }
                        mbar_arrive_expect_tx(&b_full[s], C::B_BYTES);
                        tma_load_2d(sB + s * C::B_BYTES, &tm_x, (sb * 4 + g) * BK, tt * BN, &b_full[s],
                                    pol_x);
                        ++kc;
                    }
                    if (*abort_flag) break;
                }
            }
            if (*abort_flag) {  // let issued copies land before the CTA leaves
                for (uint32_t j = kc > (uint32_t)C::NS ? kc - C::NS : 0; j < kc; ++j)
                    mbar_wait(&b_full[j % C::NS], (j / C::NS) & 1);
                for (uint32_t j = rc > (uint32_t)kRawSlots ? rc - kRawSlots : 0; j < rc; ++j)
                    mbar_wait(&raw_full[j % kRawSlots], (j / kRawSlots) & 1);
            }
        }
    } else if (warp == 1) {
        // ---------------------------------------------------------- MMA
        if (lane == 0) {
            constexpr uint32_t fmt = std::is_same<OP, __half>::value ? 0u : 1u;
            constexpr uint32_t idesc = idesc_f16(fmt, BM, BN);
            uint32_t kc = 0;
            int i = 0;
            for (int tile = blockIdx.x; tile < tiles && !*abort_flag; tile += gridDim.x, ++i) {
                const int b = i & 1;
                if (!mbar_wait(&acc_empty[b], ((i >> 1) & 1) ^ 1)) { *abort_flag = 1; break; }
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + (uint32_t)(b * BN);
                for (int ks = 0; ks < nsb * 4; ++ks) {
                    const int s = kc % C::NS;
                    const uint32_t par = (kc / C::NS) & 1;
                    if (!mbar_wait(&a_full[s], par) || !mbar_wait(&b_full[s], par)) {
                        *abort_flag = 1;
                        break;
                    }
                    tc_fence_after();
                    const uint64_t da = smem_desc_k_sw128(sA + s * C::A_BYTES);
                    const uint64_t db = smem_desc_k_sw128(sB + s * C::B_BYTES);
#pragma unroll
                    for (int kk = 0; kk < BK / 16; ++kk)  // +32 bytes along k per MMA
                        umma_f16_ss(d_tmem, da + 2 * kk, db + 2 * kk, idesc, (ks | kk) != 0);
                    umma_commit(&ab_empty[s]);
                    ++kc;
                }
                if (*abort_flag) break;
                umma_commit(&acc_full[b]);
            }
            // wait for the last MMAs to retire before TMEM can be released
            if (kc > 0) mbar_wait(&ab_empty[(kc - 1) % C::NS], ((kc - 1) / C::NS) & 1);
        }
    } else if (warp < 2 + kEpiWarps) {
        // ---------------------------------------------------------- epilogue
        const int q = warp & 3;  // TMEM lane quadrant this warp may access
        int i = 0;
        for (int tile = blockIdx.x; tile < tiles; tile += gridDim.x, ++i) {
            const int b = i & 1;
            const int nt = tile % n_tiles, tt = tile / n_tiles;
            if (!mbar_wait_warp(&acc_full[b], (i >> 1) & 1)) { *abort_flag = 1; break; }
            tc_fence_after();
            const int n = nt * BM + 32 * q + lane;
            const uint32_t taddr = tmem_base + ((uint32_t)(32 * q) << 16) + (uint32_t)(b * BN);
#pragma unroll 1
            for (int c0 = 0; c0 < BN; c0 += 32) {
                uint32_t r[32];
                tmem_ld_32x32b_x32(taddr + c0, r);
                tmem_ld_wait();
                const int t0 = tt * BN + c0;
                if (n < N) {
#pragma unroll
                    for (int j = 0; j < 32; ++j)
                        if (t0 + j < M) store_out(y, ytype, (int64_t)(t0 + j) * N + n, __uint_as_float(r[j]));
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acc_empty[b]);
            if (*abort_flag) break;
        }
    } else {
        // ---------------------------------------------------------- dequant
        const int p = threadIdx.x - (2 + kEpiWarps) * 32;  // 0..255
        const int r = p >> 1, h = p & 1;                   // weight row in tile, half of group
        const int swz = r & 7;
        uint32_t kc = 0, rc = 0;
        for (int tile = blockIdx.x; tile < tiles; tile += gridDim.x) {
            for (int sb = 0; sb < nsb; ++sb) {
                const int rs = rc % kRawSlots;
                if (!mbar_wait_warp(&raw_full[rs], (rc / kRawSlots) & 1)) { *abort_flag = 1; break; }
                const uint8_t* blk = sRaw + rs * kRawBytes + r * 144;
                const uint4 hd = *reinterpret_cast<const uint4*>(blk);
                const float d = h2f(hd.x), dmin = h2f(hd.x >> 16);
                for (int g = 0; g < 4; ++g) {
                    const int s = kc % C::NS;
                    if (!mbar_wait_warp(&ab_empty[s], ((kc / C::NS) & 1) ^ 1)) { *abort_flag = 1; break; }
                    int sc0, mn0, sc1, mn1;
                    q4k_scale_min(hd.y, hd.z, hd.w, 2 * g, sc0, mn0);
                    q4k_scale_min(hd.y, hd.z, hd.w, 2 * g + 1, sc1, mn1);
                    const float dl = d * (float)sc0, ml = dmin * (float)mn0;
                    const float dh = d * (float)sc1, mh = dmin * (float)mn1;
                    const uint4 qv = *reinterpret_cast<const uint4*>(blk + 16 + 32 * g + 16 * h);
                    const uint32_t w[4] = {qv.x, qv.y, qv.z, qv.w};
                    uint32_t lo[8], hi[8];  // packed 16-bit pairs, k = 16h + 2i (+32 for hi)
#pragma unroll
                    for (int u = 0; u < 4; ++u) {
#pragma unroll
                        for (int e = 0; e < 2; ++e) {
                            const uint32_t b0 = (w[u] >> (16 * e)) & 0xFFu;
                            const uint32_t b1 = (w[u] >> (16 * e + 8)) & 0xFFu;
                            lo[2 * u + e] = pack2<OP>(fmaf(dl, (float)(b0 & 15u), -ml),
                                                      fmaf(dl, (float)(b1 & 15u), -ml));
                            hi[2 * u + e] = pack2<OP>(fmaf(dh, (float)(b0 >> 4), -mh),
                                                      fmaf(dh, (float)(b1 >> 4), -mh));
                        }
                    }
                    // 16-byte chunks c (8 values, k = 8c..8c+7) of row r, swizzled
                    uint8_t* arow = sA + s * C::A_BYTES + r * 128;
                    const int c_lo = 2 * h, c_hi = 4 + 2 * h;
                    *reinterpret_cast<uint4*>(arow + (((c_lo) ^ swz) << 4)) =
                        make_uint4(lo[0], lo[1], lo[2], lo[3]);
                    *reinterpret_cast<uint4*>(arow + (((c_lo + 1) ^ swz) << 4)) =
                        make_uint4(lo[4], lo[5], lo[6], lo[7]);
                    *reinterpret_cast<uint4*>(arow + (((c_hi) ^ swz) << 4)) =
                        make_uint4(hi[0], hi[1], hi[2], hi[3]);
                    *reinterpret_cast<uint4*>(arow + (((c_hi + 1) ^ swz) << 4)) =
                        make_uint4(hi[4], hi[5], hi[6], hi[7]);
                    fence_proxy_async_smem();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&a_full[s]);
                    ++kc;
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&raw_empty[rs]);
                ++rc;
                if (*abort_flag) break;
            }
            if (*abort_flag) break;
        }
    }

    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 0) tmem_dealloc(tmem_base, C::TMEM_COLS);
}

// ------------------------------------------------------------- host side

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

template <int BN, typename OP>
int launch(const CUtensorMap& tw, const CUtensorMap& tx, int M, int N, int K, void* y, int ytype,
           cudaStream_t st) {
    using C = Cfg<BN>;
    static bool configured = false;
    if (!configured) {
        cudaError_t e = cudaFuncSetAttribute(gemm_q4k_tc<BN, OP>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
        if (e != cudaSuccess) return cuda_error(e, "cudaFuncSetAttribute(gemm_q4k_tc)");
        configured = true;
    }
    static int sms = 0;
    if (!sms) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, 0);
    const int tiles = ((N + BM - 1) / BM) * ((M + BN - 1) / BN);
    const int grid = std::min(tiles, sms);
    gemm_q4k_tc<BN, OP><<<grid, kThreads, C::SMEM, st>>>(tw, tx, M, N, K, y, ytype);
    return FTC_OK;
}

}  // namespace

int gemm_q4k(const void* w, int64_t N, int64_t K, int64_t row_stride, const void* x, int x_dtype,
             int64_t M, void* y, int y_dtype, cudaStream_t st) {
    FTC_REQUIRE(w && x && y, FTC_E_INVALID, "ftc_gemm: null pointer");
    FTC_REQUIRE(M > 0 && N > 0 && K > 0, FTC_E_INVALID, "ftc_gemm: empty shape");
    FTC_REQUIRE(K % 256 == 0, FTC_E_INVALID, "ftc_gemm: K must be a multiple of 256 for Q4_K");
    FTC_REQUIRE(M <= INT32_MAX && N <= INT32_MAX && K <= INT32_MAX, FTC_E_INVALID,
                "ftc_gemm: shape too large");
    FTC_REQUIRE(x_dtype == FTC_BF16 || x_dtype == FTC_F16, FTC_E_UNSUPPORTED,
                "ftc_gemm: activations must be bf16 or fp16");
    FTC_REQUIRE(y_dtype == FTC_BF16 || y_dtype == FTC_F16 || y_dtype == FTC_F32, FTC_E_UNSUPPORTED,
                "ftc_gemm: output must be bf16, fp16 or fp32");
    FTC_REQUIRE(row_stride >= (K / 256) * 144 && row_stride % 16 == 0 && (uintptr_t)w % 16 == 0,
                FTC_E_INVALID, "ftc_gemm: weight rows must be 16-byte aligned");
    FTC_REQUIRE((uintptr_t)x % 16 == 0, FTC_E_INVALID, "ftc_gemm: activations must be 16-byte aligned");
    auto enc = encode_fn();
    FTC_REQUIRE(enc, FTC_E_CUDA, "ftc_gemm: cuTensorMapEncodeTiled unavailable");

    CUtensorMap tw, tx;
    {
        const cuuint64_t dims[2] = {(cuuint64_t)((K / 256) * 144), (cuuint64_t)N};
        const cuuint64_t strides[1] = {(cuuint64_t)row_stride};
        const cuuint32_t box[2] = {144, BM};
        const cuuint32_t es[2] = {1, 1};
        CUresult r = enc(&tw, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(w), dims, strides,
                         box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        FTC_REQUIRE(r == CUDA_SUCCESS, FTC_E_CUDA, "ftc_gemm: weight tensor map rejected");
    }
    const int BN = M <= 128 ? 128 : 256;
    {
        const cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)M};
        const cuuint64_t strides[1] = {(cuuint64_t)(K * 2)};
        const cuuint32_t box[2] = {BK, (cuuint32_t)BN};
        const cuuint32_t es[2] = {1, 1};
        CUresult r = enc(&tx,
                         x_dtype == FTC_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                             : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                         2, const_cast<void*>(x), dims, strides, box, es,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        FTC_REQUIRE(r == CUDA_SUCCESS, FTC_E_CUDA, "ftc_gemm: activation tensor map rejected");
    }
    if (inject_fail("ftc_gemm")) return set_error(FTC_E_INJECTED, "ftc_gemm: injected failure");
    int rc;
    const bool bf = x_dtype == FTC_BF16;
    if (BN == 128)
        rc = bf ? launch<128, __nv_bfloat16>(tw, tx, (int)M, (int)N, (int)K, y, y_dtype, st)
                : launch<128, __half>(tw, tx, (int)M, (int)N, (int)K, y, y_dtype, st);
    else
        rc = bf ? launch<256, __nv_bfloat16>(tw, tx, (int)M, (int)N, (int)K, y, y_dtype, st)
                : launch<256, __half>(tw, tx, (int)M, (int)N, (int)K, y, y_dtype, st);
    if (rc != FTC_OK) return rc;
    FTC_CUDA(cudaGetLastError());
    return FTC_OK;
}

}  // namespace ftc
