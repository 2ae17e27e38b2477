// gemv_q4k.cu -- the decode GEMV for Q4_K weights, batch 1 and 2:
//
//   y[m][n] = sum_k x[m][k] * W[n][k]        W: Q4_K super-blocks of 256
//
// HBM-bound by design: every weight byte crosses HBM once, through a ring of
// bulk (TMA) copies into shared memory, and the SM spends about 1.8 issue
// slots per weight so that decoding stays well under the copy rate.
//
// Exact-integer activations.  At start-up each consumer lane turns its 64
// activations into 24-bit integers with one power-of-two scale per 256-block:
// x = s_b * x_int, |x_int| < 2^22, error <= s_b/2 <= 2^-22 * max|x_block|
// (zero for activations whose significant bits fit, e.g. one-hot vectors).
// x_int is held as three byte planes (hi signed, mid and lo unsigned), so
//   sum_l q_l * x_int_l = 65536*sum(q*hi) + 256*sum(q*mid) + sum(q*lo)
// comes from six dp4a per eight 4-bit codes, all in exact integer
// arithmetic; each sub-block's scale and min are applied once per row.
// Summation order differs from ft::dot_row_f32 (ft/include/ft/quant.h:86-103);
// the result agrees with the reference's fp32 sum to ~1e-6 relative.
//
// Work split.  A warp owns 8 super-blocks of K (4 lanes per super-block,
// lane t of a quartet takes code bytes [32t, 32t+32): sub-blocks 2t and
// 2t+1), keeps its 64 activations per m in registers for the whole kernel,
// and every row of a chunk passes through it.  WK = ceil(K/2048) warps cover
// a row; WR groups of WK warps share the rows of a chunk.  One more warp is
// the producer: it keeps S chunks of RC rows (contiguous bytes) in flight
// with cp.async.bulk, and after consumers release a stage it adds their
// per-row partial sums (fixed order: deterministic) and writes y.
#include <algorithm>

#include "common.cuh"
#include "sm100.cuh"

namespace ftc {

FTC_DEVSTAT_READER(devstat_gemv_q4k)

namespace {

constexpr int kStages = 4;

struct XParts {
    uint32_t h[16], m[16], l[16];  // byte planes of 64 x_int (4 per word)
    float sum_lo, sum_hi;          // sum of x_int over each 32-weight sub-block
    float scale;                   // s_b
};

// Load 64 activations (16 float4), derive the quartet's power-of-two scale
// and split into byte planes.  Lanes with !valid contribute zeros.
__device__ __forceinline__ void load_x_parts(const float* __restrict__ xp, bool valid,
                                             XParts& P) {
    float v[64];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
        float4 f = valid ? __ldg(reinterpret_cast<const float4*>(xp) + i)
                         : make_float4(0.f, 0.f, 0.f, 0.f);
        v[4 * i] = f.x;
        v[4 * i + 1] = f.y;
        v[4 * i + 2] = f.z;
        v[4 * i + 3] = f.w;
    }
    float amax = 0.f;
#pragma unroll
    for (int i = 0; i < 64; ++i) amax = fmaxf(amax, fabsf(v[i]));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
    // amax in [2^p, 2^(p+1)): s_b = 2^(p-21) keeps |x / s_b| < 2^22.
    int eb = (int)((__float_as_uint(amax) >> 23) & 0xFF);  // biased exponent
    int se = max(eb - 21, 1);
    const float s = __uint_as_float((uint32_t)se << 23);
    const float inv = __uint_as_float((uint32_t)(254 - se) << 23);
    int sl = 0, sh = 0;
#pragma unroll
    for (int u = 0; u < 16; ++u) {
        uint32_t h = 0, m = 0, l = 0;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            int q = __float2int_rn(v[4 * u + i] * inv);
            q = min(max(q, -(1 << 22)), (1 << 22) - 1);
            if (u < 8) sl += q; else sh += q;
            h |= ((uint32_t)(q >> 16) & 0xFFu) << (8 * i);
            m |= ((uint32_t)(q >> 8) & 0xFFu) << (8 * i);
            l |= ((uint32_t)q & 0xFFu) << (8 * i);
        }
        P.h[u] = h;
        P.m[u] = m;
        P.l[u] = l;
    }
    P.sum_lo = (float)sl;
    P.sum_hi = (float)sh;
    P.scale = s;
}

// One row: this lane's 64 weights (code bytes [32t, 32t+32) of the block)
// against its activations.  Returns s_b * (d * SQ - dmin * U).
__device__ __forceinline__ float q4k_row_partial(const uint8_t* blk, int t, bool hi_half,
                                                 int sh0, const XParts& P) {
    const uint4 hd = *reinterpret_cast<const uint4*>(blk);
    const uint4 qa = *reinterpret_cast<const uint4*>(blk + 16 + 32 * t);
    const uint4 qb = *reinterpret_cast<const uint4*>(blk + 32 + 32 * t);
    const uint32_t w[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
    int hl = 0, hh = 0;
    uint32_t ml = 0, mh = 0, ll = 0, lh = 0;
#pragma unroll
    for (int u = 0; u < 8; ++u) {
        const uint32_t lo = w[u] & 0x0F0F0F0Fu;         // sub-block 2t, weights 4u..4u+3
        const uint32_t hi = (w[u] >> 4) & 0x0F0F0F0Fu;  // sub-block 2t+1
        hl = __dp4a((int)lo, (int)P.h[u], hl);
        ml = __dp4a(lo, P.m[u], ml);
        ll = __dp4a(lo, P.l[u], ll);
        hh = __dp4a((int)hi, (int)P.h[8 + u], hh);
        mh = __dp4a(hi, P.m[8 + u], mh);
        lh = __dp4a(hi, P.l[8 + u], lh);
    }
    // scales / mins of sub-blocks 2t (byte i) and 2t+1 (byte i+1), i = sh0/8:
    //   sub-blocks 0-3: scale = s0.byte & 63, min = s1.byte & 63
    //   sub-blocks 4-7: scale = (s2.byte & 15) | (s0.byte >> 6) << 4,
    //                   min   = (s2.byte >> 4) | (s1.byte >> 6) << 4
    const uint32_t s0 = hd.y, s1 = hd.z, s2 = hd.w;
    uint32_t sc, mn;
    if (hi_half) {
        sc = ((s2 >> sh0) & 0x0F0Fu) | ((s0 >> (sh0 + 2)) & 0x3030u);
        mn = ((s2 >> (sh0 + 4)) & 0x0F0Fu) | ((s1 >> (sh0 + 2)) & 0x3030u);
    } else {
        sc = (s0 >> sh0) & 0x3F3Fu;
        mn = (s1 >> sh0) & 0x3F3Fu;
    }
    const int sc0 = (int)(sc & 0xFF), sc1 = (int)(sc >> 8);
    const int ph = sc0 * hl + sc1 * hh;                 // |.| < 2^23
    const int pm = (int)(sc0 * ml + sc1 * mh);          // < 2^24
    const int pl = (int)(sc0 * ll + sc1 * lh);
    const float sq = fmaf(65536.f, (float)ph, fmaf(256.f, (float)pm, (float)pl));
    const float u = fmaf((float)(mn >> 8), P.sum_hi, (float)(mn & 0xFF) * P.sum_lo);
    const float d = h2f(hd.x), dmin = h2f(hd.x >> 16);
    return P.scale * fmaf(-dmin, u, d * sq);
}

template <int RPW>
__global__ void __launch_bounds__(512, 1)
gemv_q4k_dp4a(const uint8_t* __restrict__ W, int64_t stride, int N, int nsb, int WK, int WR,
              const float* __restrict__ x, float* __restrict__ y) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int RC = RPW * WR;                   // rows per chunk
    const int NCW = WK * WR;                   // consumer warps
    const int stage_bytes = RC * (int)stride;  // multiple of 16
    uint8_t* stg = smem;
    float* red = reinterpret_cast<float*>(smem + kStages * stage_bytes);  // [S][WK][RC]
    uint64_t* full = reinterpret_cast<uint64_t*>(
        (reinterpret_cast<uintptr_t>(red + kStages * WK * RC) + 15) & ~uintptr_t(15));
    uint64_t* empty = full + kStages;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], NCW);
        }
        mbar_fence_init();
    }
    __syncthreads();
    const int nchunks = (N + RC - 1) / RC;

    if (warp == NCW) {
        // ------------------------------------------------ producer warp
        const uint64_t pol = policy_evict_first();
        bool ok = true;
        int it = 0;
        auto reduce = [&](int j) {  // partials of iteration j -> y
            const int s = j % kStages;
            const int c = blockIdx.x + j * gridDim.x;
            const int rows = min(RC, N - c * RC);
            if (lane < rows) {
                float v = 0.f;
                for (int wk = 0; wk < WK; ++wk) v += red[(s * WK + wk) * RC + lane];
                y[(int64_t)c * RC + lane] = v;
            }
        };
        for (int c = blockIdx.x; c < nchunks; c += gridDim.x, ++it) {
            const int s = it % kStages;
            if (it >= kStages) {
                ok = mbar_wait_warp(&empty[s], ((it / kStages) - 1) & 1);
                if (!ok) break;
                reduce(it - kStages);
            }
            __syncwarp();
            if (lane == 0) {
                const int rows = min(RC, N - c * RC);
                const uint32_t bytes = (uint32_t)(rows * stride);
                mbar_arrive_expect_tx(&full[s], bytes);
                bulk_g2s(stg + s * stage_bytes, W + (int64_t)c * RC * stride, bytes, &full[s], pol);
            }
        }
        if (ok) {
            for (int j = max(0, it - kStages); j < it; ++j) {
                if (!mbar_wait_warp(&empty[j % kStages], (j / kStages) & 1)) { ok = false; break; }
                reduce(j);
            }
        }
        if (!ok) {  // a consumer is stuck: let in-flight copies land, then leave
            for (int j = max(0, it - kStages); j < it; ++j)
                mbar_wait_warp(&full[j % kStages], (j / kStages) & 1);
        }
        return;
    }

    // ---------------------------------------------------- consumer warps
    const int wr = warp / WK, wk = warp % WK;
    const int qd = lane >> 2, t = lane & 3;
    const int sb = wk * 8 + qd;
    const bool valid = sb < nsb;
    const bool hi_half = t >= 2;             // sub-blocks 4..7 use the split encoding
    const int sh0 = 8 * ((2 * t) & 3);       // byte of sub-block 2t within its word
    XParts P;
    load_x_parts(x + (int64_t)sb * 256 + 64 * t, valid, P);

    int it = 0;
    for (int c = blockIdx.x; c < nchunks; c += gridDim.x, ++it) {
        const int s = it % kStages;
        if (!mbar_wait_warp(&full[s], (it / kStages) & 1)) break;
        const int rows = min(RC, N - c * RC);
        const uint8_t* base = stg + s * stage_bytes + sb * 144;
        float acc[RPW];
#pragma unroll
        for (int i = 0; i < RPW; ++i) {
            const int r = wr + WR * i;
            acc[i] = (valid && r < rows) ? q4k_row_partial(base + r * stride, t, hi_half, sh0, P)
                                         : 0.f;
        }
#pragma unroll
        for (int i = 0; i < RPW; ++i)
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) acc[i] += __shfl_xor_sync(0xffffffffu, acc[i], o);
        float mine = 0.f;
#pragma unroll
        for (int i = 0; i < RPW; ++i)
            if (lane == i) mine = acc[i];
        if (lane < RPW) red[(s * WK + wk) * RC + wr + WR * lane] = mine;
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
    }
}

struct Q4kPlan {
    int WK, WR, RPW, grid, threads;
    size_t smem;
};

bool plan_q4k(int64_t N, int64_t K, int64_t stride, Q4kPlan& p) {
    const int nsb = (int)(K / 256);
    p.WK = (nsb + 7) / 8;
    if (p.WK > 15) return false;
    p.WR = std::max(1, 14 / p.WK);  // ~14 consumer warps + 1 producer <= 512 threads
    static int sms = 0;
    if (!sms) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, 0);
    // rows per chunk: ~32 KB chunks, but small enough that every SM gets two
    int64_t rc = std::max<int64_t>(1, 32768 / stride);
    rc = std::min<int64_t>(rc, std::max<int64_t>(p.WR, N / (2 * (int64_t)sms)));
    const int64_t rpw = std::max<int64_t>(1, rc / p.WR);
    p.RPW = rpw >= 4 ? 4 : (rpw >= 2 ? 2 : 1);
    while (p.RPW > 1 && p.RPW * p.WR > 32) p.RPW /= 2;  // the producer reduces one row per lane
    if (p.RPW * p.WR > 32) return false;
    const int RC = p.RPW * p.WR;
    p.threads = (p.WK * p.WR + 1) * 32;
    p.smem = (size_t)kStages * RC * stride + (size_t)kStages * p.WK * RC * 4 + 16 +
             2 * kStages * 8;
    if (p.smem > 220 * 1024 || p.threads > 512) return false;
    const int64_t nchunks = (N + RC - 1) / RC;
    p.grid = (int)std::min<int64_t>(nchunks, sms);
    return true;
}

}  // namespace

// Fast path for Q4_K, M == 1.  Returns FTC_E_UNSUPPORTED when the shape or
// alignment does not fit (the caller then uses the general kernels).
int gemv_q4k_fast(const uint8_t* W, int64_t stride, int64_t N, int64_t K, const float* x,
                  float* y, cudaStream_t st) {
    if ((uintptr_t)W % 16 || stride % 16 || (uintptr_t)x % 16 || K % 256) return FTC_E_UNSUPPORTED;
    Q4kPlan p;
    if (!plan_q4k(N, K, stride, p)) return FTC_E_UNSUPPORTED;
    const int nsb = (int)(K / 256);
    // opt in to large dynamic shared memory once per instantiation
    static bool configured[3] = {false, false, false};
    auto launch = [&](auto kern, int idx) -> int {
        if (!configured[idx]) {
            cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 220 * 1024);
            if (e != cudaSuccess) return cuda_error(e, "cudaFuncSetAttribute(gemv_q4k_dp4a)");
            configured[idx] = true;
        }
        kern<<<p.grid, p.threads, p.smem, st>>>(W, stride, (int)N, nsb, p.WK, p.WR, x, y);
        return FTC_OK;
    };
    int rc = p.RPW == 4 ? launch(gemv_q4k_dp4a<4>, 2)
           : p.RPW == 2 ? launch(gemv_q4k_dp4a<2>, 1)
                        : launch(gemv_q4k_dp4a<1>, 0);
    if (rc != FTC_OK) return rc;
    FTC_CUDA(cudaGetLastError());
    return FTC_OK;
}

}  // namespace ftc
