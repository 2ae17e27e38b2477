// gemv.cu -- decode GEMV / small-batch GEMM over GGUF blocks on CUDA cores.
//
//   y[m][n] = sum_k x[m][k] * W[n][k],  x fp32 [M][K], M <= 8, y fp32 [M][N]
//
// This is the B200 replacement of the reference's row loop
// (ft/src/cpu_backend.cpp:90-104 -> ft::dot_row_f32, ft/include/ft/quant.h:86-103):
// the same products summed in fp32, in a different order (per-lane partial
// sums, then a warp-shuffle tree).  HBM-bound: every weight byte is read
// once with 16-byte loads that bypass L1, while the activations (at most
// 8 x 57 KB) stay L1/L2-resident.
//
// Kernels:
//   gemv_q4k     Q4_K, 16-byte aligned rows, when the integer tensor-core
//                kernel (gemv_imma.cu, 2..8 rows) does not take the shape:
//                registers only.  An octet of 8
//                lanes covers one 144-byte super-block: every lane reads the
//                16-byte header and one 16-byte slice of the 128 code bytes
//                (32 weights: 16 of sub-block 2g, 16 of sub-block 2g+1).
//   gemv_staged  Q8_0 / Q6_K, 16-byte aligned rows: a warp copies groups of
//                blocks (16 x 34 B, 8 x 210 B: both multiples of 16 B) with
//                16-byte loads into its own shared-memory slot, then each
//                lane decodes a fixed slice from there.
//   gemv_generic any format, any alignment: element-wise decode.
#include <algorithm>

#include "common.cuh"
#include "gemv_batch.cuh"

namespace ftc {
namespace {

constexpr int kWarps = 8;  // warps per CTA for every GEMV kernel

template <int M, int R>
__device__ __forceinline__ void warp_sum(float (&acc)[R][M]) {
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
        for (int m = 0; m < M; ++m) {
            float v = acc[r][m];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
            acc[r][m] = v;
        }
}

// Reduce the per-warp row sums of the WG warps that share a row group and
// write y.  red: [kWarps][R][M] floats in shared memory.
template <int M, int R, int WG>
__device__ __forceinline__ void store_rows(float (&acc)[R][M], float* red, int warp, int lane,
                                           int row0, int N, float* __restrict__ y, int64_t ldy) {
    warp_sum<M, R>(acc);
    if constexpr (WG == 1) {
        if (lane < R * M) {
            const int r = lane / M, m = lane % M;
            float v = 0.f;
#pragma unroll
            for (int rr = 0; rr < R; ++rr)
#pragma unroll
                for (int mm = 0; mm < M; ++mm)
                    if (rr == r && mm == m) v = acc[rr][mm];
            if (row0 + r < N) y[(int64_t)m * ldy + row0 + r] = v;
        }
    } else {
        if (lane == 0) {
#pragma unroll
            for (int r = 0; r < R; ++r)
#pragma unroll
                for (int m = 0; m < M; ++m) red[(warp * R + r) * M + m] = acc[r][m];
        }
        __syncthreads();
        const int wg = warp % WG;
        if (wg == 0 && lane < R * M) {
            const int r = lane / M, m = lane % M;
            float v = 0.f;
#pragma unroll
            for (int w = 0; w < WG; ++w) v += red[((warp + w) * R + r) * M + m];
            if (row0 + r < N) y[(int64_t)m * ldy + row0 + r] = v;
        }
    }
}

__device__ __forceinline__ void ld_x16(const float* __restrict__ p, float (&v)[16]) {
    const float4* q = reinterpret_cast<const float4*>(p);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float4 t = __ldg(q + i);
        v[4 * i + 0] = t.x;
        v[4 * i + 1] = t.y;
        v[4 * i + 2] = t.z;
        v[4 * i + 3] = t.w;
    }
}

// ------------------------------------------------------------------ Q4_K

// Sum over 16 weights of q * x for the nibbles selected by `shift` (0: low,
// 4: high) of the four code words.
__device__ __forceinline__ float q4_dot16(const uint4 q, int shift, const float (&xv)[16]) {
    const uint32_t w[4] = {q.x, q.y, q.z, q.w};
    float s = 0.f;
#pragma unroll
    for (int u = 0; u < 4; ++u)
#pragma unroll
        for (int i = 0; i < 4; ++i)
            s = fmaf((float)((w[u] >> (8 * i + shift)) & 0xFu), xv[4 * u + i], s);
    return s;
}

template <int M, int R, int WG>
__global__ void __launch_bounds__(kWarps * 32)
gemv_q4k(const uint8_t* __restrict__ W, int64_t stride, int N, int nsb,
         const float* __restrict__ x, int64_t ldx, float* __restrict__ y, int64_t ldy) {
    constexpr int GROUPS = kWarps / WG;
    constexpr int NOCT = WG * 4;
    __shared__ float red[kWarps * R * M];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int rg = warp / WG, wg = warp % WG;
    const int row0 = (blockIdx.x * GROUPS + rg) * R;
    const int t = lane & 7;
    const int oct = wg * 4 + (lane >> 3);
    const int g = t >> 1;                       // sub-blocks 2g (low nibbles), 2g+1 (high)
    const int kin = 64 * g + 16 * (t & 1);      // first weight of the low-nibble run
    const uint8_t* rowp[R];
#pragma unroll
    for (int r = 0; r < R; ++r) rowp[r] = W + (int64_t)min(row0 + r, N - 1) * stride;

    float acc[R][M];
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
        for (int m = 0; m < M; ++m) acc[r][m] = 0.f;

    for (int sb = oct; sb < nsb; sb += NOCT) {
        uint4 hd[R], qv[R];
#pragma unroll
        for (int r = 0; r < R; ++r) {
            const uint8_t* b = rowp[r] + (int64_t)sb * 144;
            hd[r] = ld_stream16(b);
            qv[r] = ld_stream16(b + 16 + 16 * t);
        }
#pragma unroll
        for (int m = 0; m < M; ++m) {
            float xl[16], xh[16];
            const float* xp = x + (int64_t)m * ldx + (int64_t)sb * 256 + kin;
            ld_x16(xp, xl);
            ld_x16(xp + 32, xh);
            float sl = 0.f, sh = 0.f;
#pragma unroll
            for (int i = 0; i < 16; ++i) { sl += xl[i]; sh += xh[i]; }
#pragma unroll
            for (int r = 0; r < R; ++r) {
                int sc0, mn0, sc1, mn1;
                q4k_scale_min(hd[r].y, hd[r].z, hd[r].w, 2 * g, sc0, mn0);
                q4k_scale_min(hd[r].y, hd[r].z, hd[r].w, 2 * g + 1, sc1, mn1);
                const float d = h2f(hd[r].x), dmin = h2f(hd[r].x >> 16);
                const float dl = d * (float)sc0, ml = dmin * (float)mn0;
                const float dh = d * (float)sc1, mh = dmin * (float)mn1;
                const float ql = q4_dot16(qv[r], 0, xl);
                const float qh = q4_dot16(qv[r], 4, xh);
                float a = acc[r][m];
                a = fmaf(dl, ql, a);
                a = fmaf(-ml, sl, a);
                a = fmaf(dh, qh, a);
                a = fmaf(-mh, sh, a);
                acc[r][m] = a;
            }
        }
    }
    store_rows<M, R, WG>(acc, red, warp, lane, row0, N, y, ldy);
}

// ------------------------------------------------------------- staged

// 16 consecutive bytes starting at an arbitrary (2-byte aligned) shared
// memory offset, as four little-endian words.
__device__ __forceinline__ void lds16_unaligned(const uint8_t* base, int off, uint32_t (&w)[4]) {
    const int a = off & ~3, sh = (off & 3) * 8;
    const uint32_t* p = reinterpret_cast<const uint32_t*>(base + a);
    uint32_t v[5];
#pragma unroll
    for (int i = 0; i < 5; ++i) v[i] = p[i];
#pragma unroll
    for (int i = 0; i < 4; ++i) w[i] = __funnelshift_r(v[i], v[i + 1], sh);
}

__device__ __forceinline__ uint32_t lds_u16(const uint8_t* base, int off) {
    return *reinterpret_cast<const uint16_t*>(base + off);
}

// Q8_0: groups of 16 blocks (544 B = 34 x 16 B).  Lane l decodes half-block
// l&1 of block l>>1: 16 int8 codes and the block's fp16 scale.
struct StageQ8 {
    static constexpr int kBlocks = 16, kBB = 34, kElems = 32;
    static constexpr int kBytes = kBlocks * kBB;   // 544
    template <int M>
    __device__ static void dot(const uint8_t* s, int nblk, int lane, const float* __restrict__ x,
                               int64_t ldx, int64_t k0, float (&acc)[M]) {
        const int b = lane >> 1, h = lane & 1;
        if (b >= nblk) return;
        const float d = h2f(lds_u16(s, b * kBB));
        uint32_t w[4];
        lds16_unaligned(s, b * kBB + 2 + 16 * h, w);
        float q[16];
#pragma unroll
        for (int u = 0; u < 4; ++u)
#pragma unroll
            for (int i = 0; i < 4; ++i) q[4 * u + i] = (float)(int8_t)((w[u] >> (8 * i)) & 0xFF);
#pragma unroll
        for (int m = 0; m < M; ++m) {
            float xv[16];
            ld_x16(x + (int64_t)m * ldx + k0 + 32 * b + 16 * h, xv);
            float s2 = 0.f;
#pragma unroll
            for (int i = 0; i < 16; ++i) s2 = fmaf(q[i], xv[i], s2);
            acc[m] = fmaf(d, s2, acc[m]);
        }
    }
};

// Q6_K: groups of 8 super-blocks (1680 B = 105 x 16 B).  Lane l decodes
// block l>>2, half (l>>1)&1, rows l..l+15 of that half where
// l = 16*(l&1): 64 weights, 4 runs of 16 (one per 32-weight quad).
struct StageQ6 {
    static constexpr int kBlocks = 8, kBB = 210, kElems = 256;
    static constexpr int kBytes = kBlocks * kBB;   // 1680
    template <int M>
    __device__ static void dot(const uint8_t* s, int nblk, int lane, const float* __restrict__ x,
                               int64_t ldx, int64_t k0, float (&acc)[M]) {
        const int b = lane >> 2, half = (lane >> 1) & 1, lr = 16 * (lane & 1);
        if (b >= nblk) return;
        const int base = b * kBB;
        uint32_t qa[4], qb[4], hh[4];
        lds16_unaligned(s, base + 64 * half + lr, qa);        // ql[l]     l in run
        lds16_unaligned(s, base + 64 * half + 32 + lr, qb);   // ql[l+32]
        lds16_unaligned(s, base + 128 + 32 * half + lr, hh);  // qh[l]
        const float d = h2f(lds_u16(s, base + 208));
        // one int8 scale per 16 weights: quad q of this run uses byte
        // 8*half + (lr/16) + 2*q of the 16 scale bytes (byte reads: the
        // offset may be odd)
        const uint8_t* scb = s + base + 192 + 8 * half + (lr >> 4);
        const float sc[4] = {(float)(int8_t)scb[0], (float)(int8_t)scb[2], (float)(int8_t)scb[4],
                             (float)(int8_t)scb[6]};
#pragma unroll
        for (int m = 0; m < M; ++m) {
            float tot = 0.f;
#pragma unroll
            for (int quad = 0; quad < 4; ++quad) {
                float xv[16];
                ld_x16(x + (int64_t)m * ldx + k0 + (int64_t)b * 256 + 128 * half + 32 * quad + lr,
                       xv);
                float s2 = 0.f;
#pragma unroll
                for (int u = 0; u < 4; ++u)
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        const uint32_t lb = ((quad & 1) ? qb[u] : qa[u]) >> (8 * i);
                        const uint32_t lo = (quad & 2) ? ((lb >> 4) & 0xF) : (lb & 0xF);
                        const uint32_t hi = (hh[u] >> (8 * i + 2 * quad)) & 3;
                        s2 = fmaf((float)((int)(lo | (hi << 4)) - 32), xv[4 * u + i], s2);
                    }
                tot = fmaf(d * sc[quad], s2, tot);
            }
            acc[m] += tot;
        }
    }
};

template <class S, int M, int R>
__global__ void __launch_bounds__(kWarps * 32)
gemv_staged(const uint8_t* __restrict__ W, int64_t stride, int N, int nblk_row,
            const float* __restrict__ x, int64_t ldx, float* __restrict__ y, int64_t ldy) {
    // +16: the unaligned 16-byte reader fetches one word past its run
    __shared__ __align__(16) uint8_t stage[kWarps][R][S::kBytes + 16];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int row0 = (blockIdx.x * kWarps + warp) * R;
    constexpr int kChunks = S::kBytes / 16;
    float acc[R][M];
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
        for (int m = 0; m < M; ++m) acc[r][m] = 0.f;
    for (int b0 = 0; b0 < nblk_row; b0 += S::kBlocks) {
        const int nb = min(S::kBlocks, nblk_row - b0);
        const int nchunks = (nb * S::kBB) / 16;  // whole groups: multiple of 16 B
        uint4 v[R][(kChunks + 31) / 32];
#pragma unroll
        for (int r = 0; r < R; ++r) {
            const uint8_t* src = W + (int64_t)min(row0 + r, N - 1) * stride + (int64_t)b0 * S::kBB;
#pragma unroll
            for (int c = 0; c < (kChunks + 31) / 32; ++c) {
                const int ch = lane + 32 * c;
                if (ch < nchunks) v[r][c] = ld_stream16(src + 16 * ch);
            }
        }
        __syncwarp();
#pragma unroll
        for (int r = 0; r < R; ++r)
#pragma unroll
            for (int c = 0; c < (kChunks + 31) / 32; ++c) {
                const int ch = lane + 32 * c;
                if (ch < nchunks) reinterpret_cast<uint4*>(stage[warp][r])[ch] = v[r][c];
            }
        __syncwarp();
#pragma unroll
        for (int r = 0; r < R; ++r)
            S::template dot<M>(stage[warp][r], nb, lane, x, ldx, (int64_t)b0 * S::kElems, acc[r]);
    }
    store_rows<M, R, 1>(acc, nullptr, warp, lane, row0, N, y, ldy);
}

// ------------------------------------------------------------- generic

template <int M>
__global__ void __launch_bounds__(kWarps * 32)
gemv_generic(int dtype, const uint8_t* __restrict__ W, int64_t stride, int N, int64_t K,
             const float* __restrict__ x, int64_t ldx, float* __restrict__ y, int64_t ldy) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int row = blockIdx.x * kWarps + warp;
    if (row >= N) return;
    const uint8_t* rp = W + (int64_t)row * stride;
    float acc[1][M];
#pragma unroll
    for (int m = 0; m < M; ++m) acc[0][m] = 0.f;
    for (int64_t j = lane; j < K; j += 32) {
        const float w = decode_elem(dtype, rp, j);
#pragma unroll
        for (int m = 0; m < M; ++m) acc[0][m] = fmaf(x[(int64_t)m * ldx + j], w, acc[0][m]);
    }
    warp_sum<M, 1>(acc);
    if (lane == 0)
#pragma unroll
        for (int m = 0; m < M; ++m) y[(int64_t)m * ldy + row] = acc[0][m];
}

// ------------------------------------------------------------- dispatch

template <int M>
int launch_q4k(const uint8_t* W, int64_t stride, int N, int nsb, const float* x, int64_t K,
               float* y, cudaStream_t st) {
    // Row groups of R rows spread over WG warps: WG*4 octets walk the
    // super-blocks; pick WG so every octet gets the same count.
    constexpr int R = (M <= 2) ? 2 : 1;
    if (nsb % 16 == 0 && nsb <= 32) {
        const int rows_per_cta = R * (kWarps / 4);
        gemv_q4k<M, R, 4><<<(N + rows_per_cta - 1) / rows_per_cta, kWarps * 32, 0, st>>>(
            W, stride, N, nsb, x, K, y, N);
    } else if (nsb % 8 == 0) {
        const int rows_per_cta = R * (kWarps / 2);
        gemv_q4k<M, R, 2><<<(N + rows_per_cta - 1) / rows_per_cta, kWarps * 32, 0, st>>>(
            W, stride, N, nsb, x, K, y, N);
    } else {
        const int rows_per_cta = R * kWarps;
        gemv_q4k<M, R, 1><<<(N + rows_per_cta - 1) / rows_per_cta, kWarps * 32, 0, st>>>(
            W, stride, N, nsb, x, K, y, N);
    }
    return FTC_OK;
}

template <class S, int M>
int launch_staged(const uint8_t* W, int64_t stride, int N, int nblk, const float* x, int64_t K,
                  float* y, cudaStream_t st) {
    constexpr int R = (M <= 2) ? 2 : 1;
    const int rows_per_cta = R * kWarps;
    gemv_staged<S, M, R><<<(N + rows_per_cta - 1) / rows_per_cta, kWarps * 32, 0, st>>>(
        W, stride, N, nblk, x, K, y, N);
    return FTC_OK;
}

}  // namespace

int gemv_q4k_fast(const uint8_t* W, int64_t stride, int64_t N, int64_t K, const float* x,
                  float* y, cudaStream_t st);
int gemv_kq_fast(int wfmt, const uint8_t* W, int64_t stride, int64_t N, int64_t K, const float* x,
                 float* y, cudaStream_t st);
int gemv_q4k_fast_multi(int P, const uint8_t* const* W, const int64_t* N, float* const* y,
                        int64_t stride, int64_t K, const float* x, cudaStream_t st, int n_next,
                        const uint8_t* const* next_w, const int64_t* next_bytes);

int gemv_q4k_imma_batch(const GemvSpec& g, int64_t M, int64_t ldx, cudaStream_t st);

namespace {

// Q4_K with 2..8 tokens: the integer tensor-core kernel (gemv_imma.cu) for
// P matrices sharing x; FTC_E_UNSUPPORTED when it does not apply.
int imma_multi(int P, const uint8_t* const* W, const int64_t* N, float* const* y, int64_t stride,
               int64_t K, const float* x, int64_t M, cudaStream_t st) {
    GemvSpec g = {};
    g.P = P;
    g.K = K;
    g.stride = stride;
    g.x[0] = x;
    for (int i = 0; i < P; ++i) {
        g.W[i] = W[i];
        g.N[i] = N[i];
        g.y[i] = y[i];
    }
    return gemv_q4k_imma_batch(g, M, K, st);
}

template <int M>
int launch_m(int dtype, const uint8_t* W, int64_t stride, int N, int64_t K, const float* x,
             float* y, cudaStream_t st) {
    if (M == 1 && dtype == FTC_Q4_K) {
        const int rc = gemv_q4k_fast(W, stride, N, K, x, y, st);
        if (rc != FTC_E_UNSUPPORTED) return rc;
    }
    if (M == 1 && (dtype == FTC_Q6_K || dtype == FTC_Q8_0)) {
        const int rc = gemv_kq_fast(dtype == FTC_Q6_K ? kGemvQ6K : kGemvQ80, W, stride, N, K, x,
                                    y, st);
        if (rc != FTC_E_UNSUPPORTED) return rc;
    }
    if (M > 1 && dtype == FTC_Q4_K) {
        const int64_t n64 = N;
        const int rc = imma_multi(1, &W, &n64, &y, stride, K, x, M, st);
        if (rc != FTC_E_UNSUPPORTED) return rc;
    }
    const Fmt f = fmt_of(dtype);
    const int64_t nblk = K / f.block_elems;
    const bool aligned = ((uintptr_t)W % 16 == 0) && (stride % 16 == 0) && ((uintptr_t)x % 16 == 0);
    if (dtype == FTC_Q4_K && aligned) return launch_q4k<M>(W, stride, N, (int)nblk, x, K, y, st);
    if (dtype == FTC_Q8_0 && aligned && nblk % 8 == 0)
        return launch_staged<StageQ8, M>(W, stride, N, (int)nblk, x, K, y, st);
    if (dtype == FTC_Q6_K && aligned && nblk % 8 == 0)
        return launch_staged<StageQ6, M>(W, stride, N, (int)nblk, x, K, y, st);
    gemv_generic<M><<<(N + kWarps - 1) / kWarps, kWarps * 32, 0, st>>>(dtype, W, stride, N, K, x,
                                                                       K, y, N);
    return FTC_OK;
}

}  // namespace

int mul_mat_vec(int dtype, const void* w, int64_t N, int64_t K, int64_t row_stride,
                const float* x, int64_t M, float* y, cudaStream_t st) {
    const Fmt f = fmt_of(dtype);
    FTC_REQUIRE(f.block_elems > 0, FTC_E_UNSUPPORTED, "ftc_mul_mat_vec: unknown dtype");
    FTC_REQUIRE(w && x && y, FTC_E_INVALID, "ftc_mul_mat_vec: null pointer");
    FTC_REQUIRE(N > 0 && K > 0 && N <= INT32_MAX, FTC_E_INVALID, "ftc_mul_mat_vec: bad N/K");
    FTC_REQUIRE(M >= 1 && M <= 8, FTC_E_INVALID, "ftc_mul_mat_vec: M must be 1..8");
    FTC_REQUIRE(K % f.block_elems == 0, FTC_E_INVALID,
                "ftc_mul_mat_vec: K must be a whole number of blocks");
    FTC_REQUIRE(row_stride >= row_bytes(dtype, K), FTC_E_INVALID,
                "ftc_mul_mat_vec: row_stride smaller than one row of blocks");
    if (inject_fail("ftc_mul_mat_vec"))
        return set_error(FTC_E_INJECTED, "ftc_mul_mat_vec: injected failure");
    const uint8_t* W = static_cast<const uint8_t*>(w);
    const int n = (int)N;
    int rc;
    switch (M) {
        case 1: rc = launch_m<1>(dtype, W, row_stride, n, K, x, y, st); break;
        case 2: rc = launch_m<2>(dtype, W, row_stride, n, K, x, y, st); break;
        case 3: rc = launch_m<3>(dtype, W, row_stride, n, K, x, y, st); break;
        case 4: rc = launch_m<4>(dtype, W, row_stride, n, K, x, y, st); break;
        case 5: rc = launch_m<5>(dtype, W, row_stride, n, K, x, y, st); break;
        case 6: rc = launch_m<6>(dtype, W, row_stride, n, K, x, y, st); break;
        case 7: rc = launch_m<7>(dtype, W, row_stride, n, K, x, y, st); break;
        default: rc = launch_m<8>(dtype, W, row_stride, n, K, x, y, st); break;
    }
    if (rc != FTC_OK) return rc;
    FTC_CUDA(cudaGetLastError());
    return FTC_OK;
}

int mul_mat_vec_multi(int dtype, int P, const void* const* w, const int64_t* N, int64_t K,
                      int64_t row_stride, const float* x, int64_t M, float* const* y,
                      cudaStream_t st, int n_next, const void* const* next_w,
                      const int64_t* next_bytes) {
    FTC_REQUIRE(P >= 1 && P <= 8, FTC_E_INVALID, "ftc_mul_mat_vec_multi: n_mats must be 1..8");
    FTC_REQUIRE(w && N && y, FTC_E_INVALID, "ftc_mul_mat_vec_multi: null array");
    FTC_REQUIRE(n_next >= 0 && n_next <= 8 && (n_next == 0 || (next_w && next_bytes)),
                FTC_E_INVALID, "ftc_mul_mat_vec_multi: prefetch hint needs 0..8 regions");
    if (dtype == FTC_Q4_K && M == 1) {
        bool args_ok = row_stride >= row_bytes(dtype, K) && x != nullptr;
        for (int i = 0; i < P && args_ok; ++i) args_ok = w[i] && y[i] && N[i] > 0;
        if (args_ok) {
            if (inject_fail("ftc_mul_mat_vec"))
                return set_error(FTC_E_INJECTED, "ftc_mul_mat_vec_multi: injected failure");
            const int rc = gemv_q4k_fast_multi(P, reinterpret_cast<const uint8_t* const*>(w), N, y,
                                               row_stride, K, x, st, n_next,
                                               reinterpret_cast<const uint8_t* const*>(next_w),
                                               next_bytes);
            if (rc != FTC_E_UNSUPPORTED) return rc;
        }
    }
    if (dtype == FTC_Q4_K && M > 1 && M <= 8 && x && row_stride >= row_bytes(dtype, K)) {
        bool args_ok = true;
        for (int i = 0; i < P && args_ok; ++i) args_ok = w[i] && y[i] && N[i] > 0;
        if (args_ok) {
            if (inject_fail("ftc_mul_mat_vec"))
                return set_error(FTC_E_INJECTED, "ftc_mul_mat_vec_multi: injected failure");
            const int rc = imma_multi(P, reinterpret_cast<const uint8_t* const*>(w), N, y,
                                      row_stride, K, x, M, st);
            if (rc != FTC_E_UNSUPPORTED) return rc;
        }
    }
    for (int i = 0; i < P; ++i) {
        const int rc = mul_mat_vec(dtype, w[i], N[i], K, row_stride, x, M, y[i], st);
        if (rc) return rc;
    }
    return FTC_OK;
}

}  // namespace ftc
