// gemv_imma.cu -- small-batch decode GEMV for Q4_K on the integer tensor
// path of the SM (mma.sync m16n8k32, s8 x s8 -> s32):
//
//   y[m][n] = sum_k x[m][k] * W[n][k]     M = 1..8 tokens, fp32 in and out
//
// The batched form of the reference's row loop (ft/src/cpu_backend.cpp:
// 90-104 with per-row semantics; ft::dot_row_f32, ft/include/ft/quant.h:
// 86-103), for speculative verify and small decode batches.  HBM-bound: the
// weight streams once per launch for all M tokens.
//
// Exact-integer activations, as the batch-1 kernel (gemv_q4k.cu): every
// 256-block of a token's x becomes 24-bit integers with one power-of-two
// scale, x = s_b * x_int, held as three signed-digit byte planes
// x_int = 65536*D2 + 256*D1 + D0 (D0, D1 in [-128, 127]).  One MMA of 16
// weight rows x 32 k (one Q4_K sub-block: codes 0..15 as s8) against a
// column per (token, plane) gives per-row integer dot products; each is
// multiplied by its sub-block scale (6 bits) and summed over the super-block
// in int32 (|.| < 2^25), then
//   y += s_b * (d * (65536*H + 256*Mi + L) - dmin * sum_j m_j * xsum_j)
// where the min term is one more MMA per super-block: the 8 packed 6-bit mins
// of a row against the four signed-digit planes of the sub-block sums of
// x_int.  Nothing is rounded before the float conversion of these integer
// sums; the result agrees with the reference's fp32 sum to ~1e-6.
//
// Fragment mapping (m16n8k32, lane = 4*n + c).  The k order inside one MMA
// is free as long as A and B agree: lane c supplies positions 8c..8c+7 of
// the sub-block (A: 8 codes of rows n and n+8, i.e. code bytes 8c..8c+7 of
// the sub-block's 32-byte group, low nibbles for sub-block 2g and high for
// 2g+1; B: the same 8 positions of column n's digit plane).  Columns: for
// M <= 2 one block of (token, plane) pairs (3t + p); for M >= 3 one block
// per plane (column = token).
//
// Work split.  A unit is 128 rows x one super-block: the producer warp
// loads it with one tensor-map copy (a 144-byte x 128-row box) into a stage
// of the shared-memory ring, and the 8 warps of a consumer group each take 16
// of its rows; the producer adds the per-(row, token) partials of a unit to
// the running sums of its 128-row block.  CTAs specialise in one of KG
// k-groups (the activation digits of a k-group fit in shared memory) and
// take a contiguous range of that k-group's units (row block major), so
// every CTA streams the same number of bytes.  A row block whose super-blocks
// are spread over several CTAs is finished by the last of them (arrival
// counter): partials go to a fixed slot each and are summed in unit order,
// so the result does not depend on which CTA came last.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>

#include "common.cuh"
#include "gemv_batch.cuh"
#include "sm100.cuh"

namespace ftc {

FTC_DEVSTAT_READER(devstat_gemv_imma_raw)

namespace {

constexpr int kRB = 128;            // rows per row block (one tensor-map box)
constexpr int kWarpRows = 16;       // rows per consumer warp (MMA M)
constexpr int kGroupWarps = kRB / kWarpRows;
constexpr int kUnitBytes = kRB * 144;
constexpr int kMaxStages = 8;
constexpr int kMaxRB = 65536;       // row blocks per launch
constexpr int kMaxThreads = (2 * kGroupWarps + 1) * 32;
constexpr size_t kMaxSmem = 227 * 1024;
constexpr size_t kTableMax = 96 * 1024;  // activation digits per CTA
constexpr size_t kSlotFloats = (size_t)1 << 20;
constexpr int kFixCap = 30;  // row blocks a CTA finishes at its end

// Split-row-block fix-up: arrival counters per row block (zero between
// launches: the last arrival resets its counter) and partial slots.  Static
// device memory (4.25 MB per GPU), so no launch allocates; launches that
// overlap on the GPU (different streams) must not share it.
__device__ uint32_t g_imma_counters[kMaxRB];
__device__ float g_imma_slots[kSlotFloats];

struct ImmaMaps {
    CUtensorMap m[kGemvMaxMats];  // weight of matrix p: [N][nsb * 144] bytes, box 144 x 128
};

struct ImmaBatch {
    float* y[kGemvMaxMats];
    int N[kGemvMaxMats];
    int rb_first[kGemvMaxMats + 1];  // prefix sums of ceil(N / 128)
    int P;
    const float* x;
    int ldx;
    int nsb;   // super-blocks per row
    int KG;    // k-groups
    int nsbg;  // super-blocks per k-group (= units per row block and k-group)
    int R;     // row blocks
    int G;     // CTAs per k-group
    int S;     // stages
    int NGRP;  // consumer groups (units in flight together)
    int use_slots;
};

template <int M>
struct ImmaLay {
    static constexpr bool kCompact = M <= 2;
    static constexpr int NB = kCompact ? 1 : 3;   // main column blocks
    static constexpr int NBm = kCompact ? 1 : 4;  // min column blocks
};

__device__ __forceinline__ void mma_s8(int (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                       uint32_t b1) {
    asm("mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%10,%10,%10,%10};"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "r"(0));
}

// CTA i of a k-group with U units and G CTAs owns units [bnd(i), bnd(i+1)).
__device__ __host__ __forceinline__ int unit_bnd(int i, int U, int G) {
    return (int)((int64_t)i * U / G);
}
// The CTA whose range holds unit q.
__device__ __host__ __forceinline__ int unit_owner(int q, int U, int G) {
    return (int)((((int64_t)q + 1) * G + U - 1) / U - 1);
}

__device__ __forceinline__ int rb_matrix(const ImmaBatch& B, int rb) {
    int p = 0;
    while (p + 1 < B.P && rb >= B.rb_first[p + 1]) ++p;
    return p;
}

// Packed 6-bit scales / mins of sub-blocks 0-3 and 4-7 (one per byte).
__device__ __forceinline__ uint32_t sc_lo(const uint4& h) { return h.y & 0x3F3F3F3Fu; }
__device__ __forceinline__ uint32_t sc_hi(const uint4& h) {
    return (h.w & 0x0F0F0F0Fu) | ((h.y >> 2) & 0x30303030u);
}
__device__ __forceinline__ uint32_t mn_lo(const uint4& h) { return h.z & 0x3F3F3F3Fu; }
__device__ __forceinline__ uint32_t mn_hi(const uint4& h) {
    return ((h.w >> 4) & 0x0F0F0F0Fu) | ((h.z >> 2) & 0x30303030u);
}

// The consumer warps of a CTA: activation digits of the k-group into
// shared memory, then this CTA's units (group g takes units j = g mod NGRP).
template <int M>
__device__ __forceinline__ void consume_units(const ImmaBatch& B, const uint8_t* stg, uint8_t* T,
                                              uint8_t* XS, float* SX, float* red, uint64_t* full,
                                              uint64_t* empty, int kg, int u0, int nunits,
                                              int warp, int lane, int NCW) {
    using L = ImmaLay<M>;
    const int S = B.S, nsbg = B.nsbg;
    // activation digits of this CTA's k-group (x may be the preceding
    // kernel's output: read it after the dependency wait)
    grid_dependency_wait();
    for (int pr = warp; pr < M * nsbg; pr += NCW) {
        const int t = pr / nsbg, sbl = pr % nsbg;
        const float* xp = B.x + (int64_t)t * B.ldx + (int64_t)(kg * nsbg + sbl) * 256 + 8 * lane;
        const float4 xa = __ldg(reinterpret_cast<const float4*>(xp));
        const float4 xb = __ldg(reinterpret_cast<const float4*>(xp) + 1);
        const float v[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
        float amax = 0.f;
#pragma unroll
        for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(v[i]));
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
        // amax in [2^p, 2^(p+1)): s = 2^(p-21) keeps |x / s| < 2^22
        const int eb = (int)((__float_as_uint(amax) >> 23) & 0xFF);
        const int se = max(eb - 21, 1);
        const float inv = __uint_as_float((uint32_t)(254 - se) << 23);
        uint32_t pl[3][2] = {{0, 0}, {0, 0}, {0, 0}};
        int sum = 0;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            // round(x * inv) via the 1.5 * 2^23 magic constant (x * inv is exact)
            const int q = __float_as_int(fmaf(v[i], inv, 12582912.0f)) - 0x4B400000;
            sum += q;
            const int d0 = (int)(int8_t)(q & 0xFF);
            const int q1 = (q - d0) >> 8;
            const int d1 = (int)(int8_t)(q1 & 0xFF);
            const int d2 = (q1 - d1) >> 8;
            const int sh = 8 * (i & 3);
            pl[0][i >> 2] |= ((uint32_t)d0 & 0xFFu) << sh;
            pl[1][i >> 2] |= ((uint32_t)d1 & 0xFFu) << sh;
            pl[2][i >> 2] |= ((uint32_t)d2 & 0xFFu) << sh;
        }
        // lane covers positions 8*(lane&3) .. +7 of sub-block lane>>2
        const int sub = lane >> 2, pos = 8 * (lane & 3);
        uint8_t* dst = T + ((size_t)((sbl * 8 + sub) * M + t) * 3) * 32 + pos;
#pragma unroll
        for (int p = 0; p < 3; ++p)
            *reinterpret_cast<uint2*>(dst + p * 32) = make_uint2(pl[p][0], pl[p][1]);
        sum += __shfl_xor_sync(0xffffffffu, sum, 1);
        sum += __shfl_xor_sync(0xffffffffu, sum, 2);
        if ((lane & 3) == 0) {  // sub-block sum (|.| < 2^27) as four signed digits
            int r = sum;
            uint8_t* xs = XS + ((size_t)(sbl * M + t) * 4) * 8 + sub;
#pragma unroll
            for (int dgt = 0; dgt < 4; ++dgt) {
                const int e = (int)(int8_t)(r & 0xFF);
                xs[dgt * 8] = (uint8_t)(e & 0xFF);
                r = (r - e) >> 8;
            }
        }
        if (lane == 0) SX[sbl * M + t] = __uint_as_float((uint32_t)se << 23);
    }
    named_barrier(1, NCW * 32);

    const int grp = warp / kGroupWarps, wl = warp % kGroupWarps;
    const int n = lane >> 2, c = lane & 3;
    // this lane's B columns: byte offset of its digit row (-1: zero column),
    // and the (token, plane) of its accumulator columns
    int boff[L::NB], moff[L::NBm];
#pragma unroll
    for (int jb = 0; jb < L::NB; ++jb) {
        const int t = L::kCompact ? n / 3 : n;
        const int p = L::kCompact ? n % 3 : jb;
        boff[jb] = t < M ? (t * 3 + p) * 32 + 8 * c : -1;
    }
#pragma unroll
    for (int jb = 0; jb < L::NBm; ++jb) {
        const int t = L::kCompact ? n / 4 : n;
        const int dg = L::kCompact ? n % 4 : jb;
        moff[jb] = (t < M && c < 2) ? (t * 4 + dg) * 8 + 4 * c : -1;
    }
    // the (token, weight) of this lane's accumulator columns 2c + e: main
    // columns weigh 256^plane, min columns 256^digit; token -1 past M
    int ctm[2], ctn[2];
    float wm[2], wn[2];
#pragma unroll
    for (int e = 0; e < 2; ++e) {
        const int col = 2 * c + e;
        ctm[e] = L::kCompact ? (col / 3 < M ? col / 3 : -1) : (col < M ? col : -1);
        ctn[e] = L::kCompact ? (col / 4 < M ? col / 4 : -1) : ctm[e];
        wm[e] = __uint_as_float((uint32_t)(127 + 8 * (L::kCompact ? col % 3 : 0)) << 23);
        wn[e] = __uint_as_float((uint32_t)(127 + 8 * (L::kCompact ? col % 4 : 0)) << 23);
    }
    constexpr uint32_t kNib = 0x0F0F0F0Fu;

    for (int j = grp; j < nunits; j += B.NGRP) {
        const int s = j % S;
        if (!mbar_wait_warp(&full[s], (j / S) & 1)) break;
        const int sbl = (u0 + j) % nsbg;
        const uint8_t* r0 = stg + (size_t)s * kUnitBytes + (wl * kWarpRows + n) * 144;
        const uint8_t* r1 = r0 + 8 * 144;
        const uint4 h0 = *reinterpret_cast<const uint4*>(r0);
        const uint4 h1 = *reinterpret_cast<const uint4*>(r1);
        const uint32_t sc0[2] = {sc_lo(h0), sc_hi(h0)}, sc1[2] = {sc_lo(h1), sc_hi(h1)};
        const uint8_t* tb = T + (size_t)sbl * 8 * M * 96;
        int acc[L::NB][4];
#pragma unroll
        for (int jb = 0; jb < L::NB; ++jb)
#pragma unroll
            for (int e = 0; e < 4; ++e) acc[jb][e] = 0;
#pragma unroll
        for (int g = 0; g < 4; ++g) {
            const uint2 q0 = *reinterpret_cast<const uint2*>(r0 + 16 + 32 * g + 8 * c);
            const uint2 q1 = *reinterpret_cast<const uint2*>(r1 + 16 + 32 * g + 8 * c);
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int sub = 2 * g + h;
                uint32_t a[4];
                if (h == 0) {
                    a[0] = q0.x & kNib; a[1] = q1.x & kNib; a[2] = q0.y & kNib; a[3] = q1.y & kNib;
                } else {
                    a[0] = (q0.x >> 4) & kNib; a[1] = (q1.x >> 4) & kNib;
                    a[2] = (q0.y >> 4) & kNib; a[3] = (q1.y >> 4) & kNib;
                }
                const int s0 = (int)__byte_perm(sc0[sub >> 2], 0, 0x4440 | (sub & 3));
                const int s1 = (int)__byte_perm(sc1[sub >> 2], 0, 0x4440 | (sub & 3));
                const uint8_t* tbs = tb + (size_t)sub * M * 96;
#pragma unroll
                for (int jb = 0; jb < L::NB; ++jb) {
                    uint2 b = make_uint2(0u, 0u);
                    if (boff[jb] >= 0) b = *reinterpret_cast<const uint2*>(tbs + boff[jb]);
                    int d[4];
                    mma_s8(d, a, b.x, b.y);
                    acc[jb][0] += s0 * d[0];
                    acc[jb][1] += s0 * d[1];
                    acc[jb][2] += s1 * d[2];
                    acc[jb][3] += s1 * d[3];
                }
            }
        }
        // min term: the 8 mins of rows n, n+8 against the sub-block sums
        uint32_t am[4] = {0u, 0u, 0u, 0u};
        if (c == 0) { am[0] = mn_lo(h0); am[1] = mn_lo(h1); }
        if (c == 1) { am[0] = mn_hi(h0); am[1] = mn_hi(h1); }
        const uint8_t* xsb = XS + (size_t)sbl * M * 32;
        int um[L::NBm][4];
#pragma unroll
        for (int jb = 0; jb < L::NBm; ++jb) {
            uint32_t b = 0u;
            if (moff[jb] >= 0) b = *reinterpret_cast<const uint32_t*>(xsb + moff[jb]);
            mma_s8(um[jb], am, b, 0u);
        }
        // per (row, token): s_b * (d * sum_p 256^p * acc - dmin * sum_q 256^q * um)
        const float dr[2] = {h2f(h0.x), h2f(h1.x)};
        const float mr[2] = {h2f(h0.x >> 16), h2f(h1.x >> 16)};
        const float* sx = SX + sbl * M;
        float* rw = red + (size_t)s * (kRB * M) + (wl * kWarpRows) * M;
        if constexpr (L::kCompact) {
            // columns: main 3t + p, min 4t + q; a token's columns are spread
            // over the lanes of a quad, so sum over the quad
            float gv[2][2] = {{0.f, 0.f}, {0.f, 0.f}};
            const float sx0 = sx[0], sx1 = sx[M > 1 ? 1 : 0];
#pragma unroll
            for (int ri = 0; ri < 2; ++ri)
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                    const int ei = 2 * ri + e;
                    const float vm = (float)acc[0][ei] * wm[e] * dr[ri];
                    const float vn = (float)um[0][ei] * wn[e] * mr[ri];
                    gv[ri][0] += ctm[e] == 0 ? sx0 * vm : 0.f;
                    gv[ri][1] += ctm[e] == 1 ? sx1 * vm : 0.f;
                    gv[ri][0] -= ctn[e] == 0 ? sx0 * vn : 0.f;
                    gv[ri][1] -= ctn[e] == 1 ? sx1 * vn : 0.f;
                }
#pragma unroll
            for (int ri = 0; ri < 2; ++ri)
#pragma unroll
                for (int t = 0; t < 2; ++t) {
                    gv[ri][t] += __shfl_xor_sync(0xffffffffu, gv[ri][t], 1);
                    gv[ri][t] += __shfl_xor_sync(0xffffffffu, gv[ri][t], 2);
                }
            if (c == 0) {
#pragma unroll
                for (int t = 0; t < M; ++t) {
                    rw[n * M + t] = gv[0][t];
                    rw[(n + 8) * M + t] = gv[1][t];
                }
            }
        } else {
            // columns: token t in every block; block = plane (main) or digit (min)
#pragma unroll
            for (int ri = 0; ri < 2; ++ri)
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                    const int ei = 2 * ri + e;
                    const float sq = fmaf(65536.f, (float)acc[2][ei],
                                          fmaf(256.f, (float)acc[1][ei], (float)acc[0][ei]));
                    const float mq = fmaf(16777216.f, (float)um[3][ei],
                                          fmaf(65536.f, (float)um[2][ei],
                                               fmaf(256.f, (float)um[1][ei], (float)um[0][ei])));
                    if (ctm[e] >= 0)
                        rw[(n + 8 * ri) * M + ctm[e]] = sx[ctm[e]] * fmaf(-mr[ri], mq, dr[ri] * sq);
                }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
    }
}

// Sum the slots of row block rb in unit order (k-group by k-group, CTA by
// CTA) and store y; threads tid, tid + nth, ... take its (row, token)
// elements, each with up to 8 slot loads in flight.
template <int M>
__device__ __noinline__ void finish_row_block(const ImmaBatch& B, int rb, int U, int tid, int nth) {
    const int nsbg = B.nsbg;
    const int p = rb_matrix(B, rb);
    const int row0 = (rb - B.rb_first[p]) * kRB;
    const int Np = B.N[p];
    const int own0 = unit_owner(rb * nsbg, U, B.G);
    const int own1 = unit_owner(rb * nsbg + nsbg - 1, U, B.G);
    const int per_g = own1 - own0 + 1;
    const int ns = B.KG * per_g;
    for (int e = tid; e < kRB * M; e += nth) {
        const int row = e / M, t = e % M;
        float acc = 0.f;
        for (int i0 = 0; i0 < ns; i0 += 8) {
            float v[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const int idx = i0 + i;
                const int g = idx / per_g, own = own0 + idx % per_g;
                v[i] = idx < ns ? __ldcg(g_imma_slots +
                                         ((int64_t)g * (B.R + B.G) + rb + own) * (kRB * M) + e)
                                : 0.f;
            }
#pragma unroll
            for (int i = 0; i < 8; ++i)
                if (i0 + i < ns) acc += v[i];
        }
        if (row0 + row < Np) B.y[p][(int64_t)t * Np + row0 + row] = acc;
    }
}

template <int M>
__global__ void __launch_bounds__(kMaxThreads, 1)
gemv_q4k_imma(const __grid_constant__ ImmaMaps TM, const __grid_constant__ ImmaBatch B) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int S = B.S, nsbg = B.nsbg;
    const int NCW = B.NGRP * kGroupWarps;
    uint8_t* stg = smem;                                          // [S][128 rows][144]
    uint8_t* T = stg + (size_t)S * kUnitBytes;                    // [nsbg][8][M][3][32] digits
    uint8_t* XS = T + (size_t)nsbg * 8 * M * 96;                  // [nsbg][M][4][8] sum digits
    float* SX = reinterpret_cast<float*>(XS + (size_t)nsbg * M * 32);  // [nsbg][M] block scales
    float* red = SX + nsbg * M;                                   // [S][128 rows][M]
    uint64_t* full = reinterpret_cast<uint64_t*>(
        (reinterpret_cast<uintptr_t>(red + S * kRB * M) + 15) & ~uintptr_t(15));
    uint64_t* empty = full + S;
    int* fix = reinterpret_cast<int*>(empty + S);  // [0] count, [1..kFixCap] row blocks to finish

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kGroupWarps);
        }
        fix[0] = 0;
        mbar_fence_init();
    }
    __syncthreads();
    grid_launch_dependents();

    const int kg = (int)blockIdx.x / B.G, ci = (int)blockIdx.x % B.G;
    const int U = B.R * nsbg;
    const int u0 = unit_bnd(ci, U, B.G);
    const int nunits = unit_bnd(ci + 1, U, B.G) - u0;

    if (warp == NCW) {
        // ------------------------------------------------ producer / reducer
        const uint64_t pol = policy_evict_first();
        constexpr int kPairs = (kRB * M) / 32;
        float seg[kPairs];
        int seg_rb = -1, seg_parts = 0;
        if (lane == 0)
            for (int p = 0; p < B.P; ++p) prefetch_tensormap(&TM.m[p]);
        auto issue = [&](int j) {
            if (lane == 0) {
                const int s = j % S;
                const int u = u0 + j;
                const int rb = u / nsbg, sb = kg * nsbg + u % nsbg;
                const int p = rb_matrix(B, rb);
                mbar_arrive_expect_tx(&full[s], (uint32_t)kUnitBytes);
                tma_load_2d(stg + (size_t)s * kUnitBytes, &TM.m[p], sb * 144,
                            (rb - B.rb_first[p]) * kRB, &full[s], pol);
            }
            __syncwarp();
        };
        auto store_y = [&](int rb, const float (&v)[kPairs]) {
            const int p = rb_matrix(B, rb);
            const int row0 = (rb - B.rb_first[p]) * kRB;
            float* yp = B.y[p];
            const int Np = B.N[p];
#pragma unroll
            for (int i = 0; i < kPairs; ++i) {
                const int pr = lane + 32 * i;
                const int row = pr / M, t = pr % M;
                if (row0 + row < Np) yp[(int64_t)t * Np + row0 + row] = v[i];
            }
        };
        auto flush = [&]() {
            if (seg_rb < 0) return;
            const int Ptot = B.KG * nsbg;
            if (!B.use_slots || (B.KG == 1 && seg_parts == nsbg)) {
                store_y(seg_rb, seg);
                return;
            }
            float* slot = g_imma_slots + ((int64_t)kg * (B.R + B.G) + seg_rb + ci) * (kRB * M);
#pragma unroll
            for (int i = 0; i < kPairs; ++i) __stcg(slot + lane + 32 * i, seg[i]);
            __threadfence();
            __syncwarp();
            uint32_t old = 0;
            if (lane == 0) old = atomicAdd(&g_imma_counters[seg_rb], (uint32_t)seg_parts);
            old = __shfl_sync(0xffffffffu, old, 0);
            if ((int)old + seg_parts != Ptot) return;
            // last arrival: every part of the row block is in its slot; the
            // whole CTA sums them once its own units are done (or this warp
            // now, when the list is full)
            __threadfence();
            if (lane == 0) g_imma_counters[seg_rb] = 0;  // ready for the next launch
            const int k = fix[0];
            __syncwarp();
            if (k < kFixCap) {
                if (lane == 0) {
                    fix[1 + k] = seg_rb;
                    fix[0] = k + 1;
                }
                __syncwarp();
            } else {
                finish_row_block<M>(B, seg_rb, U, lane, 32);
            }
        };
        auto reduce = [&](int j) {
            const int rb = (u0 + j) / nsbg;
            if (rb != seg_rb) {
                flush();
                seg_rb = rb;
                seg_parts = 0;
#pragma unroll
                for (int i = 0; i < kPairs; ++i) seg[i] = 0.f;
            }
            const float* r = red + (size_t)(j % S) * (kRB * M);
#pragma unroll
            for (int i = 0; i < kPairs; ++i) seg[i] += r[lane + 32 * i];
            ++seg_parts;
        };
        bool ok = true;
        int j = 0;
        for (; j < nunits; ++j) {
            const int s = j % S;
            if (j >= S) {
                // the stage's previous unit is done: fold its partials, then refill
                ok = mbar_wait_warp(&empty[s], ((j / S) - 1) & 1);
                if (!ok) break;
                reduce(j - S);
            }
            issue(j);
        }
        if (ok) {
            for (int k = max(0, nunits - S); k < nunits; ++k) {
                if (!mbar_wait_warp(&empty[k % S], (k / S) & 1)) { ok = false; break; }
                reduce(k);
            }
            if (ok) flush();
        }
        if (!ok) {  // a consumer is stuck: let in-flight copies land, then leave
            for (int k = max(0, j - S); k < j; ++k) mbar_wait_warp(&full[k % S], (k / S) & 1);
        }
    } else {
        consume_units<M>(B, stg, T, XS, SX, red, full, empty, kg, u0, nunits, warp, lane, NCW);
    }
    // every warp: finish the row blocks whose last part arrived here
    named_barrier(2, blockDim.x);
    for (int f = 0; f < fix[0]; ++f)
        finish_row_block<M>(B, fix[1 + f], U, threadIdx.x, blockDim.x);
}

struct ImmaPlan {
    int KG, nsbg, G, S, NGRP, grid, threads, use_slots;
    size_t smem;
};

bool plan_imma(int M, int nsb, int R, int sms, ImmaPlan& p) {
    // k-groups: the fewest whose activation digits fit
    p.KG = 0;
    for (int kg = 1; kg <= std::min(nsb, 8); ++kg) {
        if (nsb % kg) continue;
        if ((size_t)(nsb / kg) * M * (768 + 32 + 4) <= kTableMax) {
            p.KG = kg;
            break;
        }
    }
    if (!p.KG) return false;
    p.nsbg = nsb / p.KG;
    const int64_t U = (int64_t)R * p.nsbg;
    if (U > (1 << 26)) return false;
    p.G = (int)std::max<int64_t>(1, std::min<int64_t>(sms / p.KG, U));
    p.grid = p.KG * p.G;
    // does any CTA boundary cut a row block?
    p.use_slots = p.KG > 1;
    for (int i = 1; i < p.G && !p.use_slots; ++i)
        if (unit_bnd(i, (int)U, p.G) % p.nsbg) p.use_slots = 1;
    if (p.use_slots && (size_t)p.KG * (R + p.G) * kRB * M > kSlotFloats) return false;
    const size_t table = (size_t)p.nsbg * M * (768 + 32 + 4);
    const size_t per_stage = (size_t)kUnitBytes + (size_t)kRB * M * 4;
    const size_t fixed = table + 2 * kMaxStages * 8 + (kFixCap + 1) * 4 + 16 + 128;
    if (fixed >= kMaxSmem) return false;
    int S = (int)std::min<size_t>(kMaxStages, (kMaxSmem - fixed) / per_stage);
    if (S >= 4) S &= ~1;  // two consumer groups take alternate stages
    if (S < 2) return false;
    p.NGRP = S >= 4 ? 2 : 1;
    p.S = S;
    p.threads = (p.NGRP * kGroupWarps + 1) * 32;
    p.smem = (size_t)S * per_stage + table + 16 + 2 * S * 8 + (kFixCap + 1) * 4 + 16;
    return p.threads <= kMaxThreads && p.smem <= kMaxSmem;
}

PFN_cuTensorMapEncodeTiled_v12000 tmap_encode() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* q = nullptr;
        cudaDriverEntryPointQueryResult r;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &q, cudaEnableDefault, &r) ==
                cudaSuccess &&
            r == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(q);
    });
    return fn;
}

// W: N rows of nsb super-blocks (row_stride bytes apart), as 144-byte x
// 128-row boxes.
int unit_map(CUtensorMap* m, const void* w, int64_t N, int nsb, int64_t row_stride) {
    auto enc = tmap_encode();
    if (!enc) return FTC_E_UNSUPPORTED;
    const cuuint64_t dims[2] = {(cuuint64_t)nsb * 144, (cuuint64_t)N};
    const cuuint64_t strides[1] = {(cuuint64_t)row_stride};
    const cuuint32_t box[2] = {144, kRB};
    const cuuint32_t es[2] = {1, 1};
    const CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(w), dims, strides,
                           box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? FTC_OK : FTC_E_UNSUPPORTED;
}

template <int M>
int launch_imma(const ImmaMaps& TM, const ImmaBatch& B, const ImmaPlan& p, cudaStream_t st) {
    auto kern = gemv_q4k_imma<M>;
    const int orc = opt_in_smem(reinterpret_cast<const void*>(kern), (int)kMaxSmem,
                                "cudaFuncSetAttribute(gemv_q4k_imma)");
    if (orc) return orc;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(p.grid);
    cfg.blockDim = dim3(p.threads);
    cfg.dynamicSmemBytes = p.smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, TM, B);
    if (e != cudaSuccess) return cuda_error(e, "launch gemv_q4k_imma");
    return FTC_OK;
}

}  // namespace

// Status reader: clearing a recorded timeout also zeroes the fix-up
// counters, which a launch that gave up part way may have left uneven.
int devstat_gemv_imma(int clear) {
    const int v = devstat_gemv_imma_raw(clear);
    if (v > 0 && clear) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_imma_counters) != cudaSuccess) return -1;
        if (cudaMemset(p, 0, sizeof(uint32_t) * kMaxRB) != cudaSuccess) return -1;
    }
    return v;
}

// Q4_K, M = 1..8 tokens sharing x (x[m] at x + m * ldx), up to
// kGemvMaxMats matrices with the same K and row pitch.  FTC_E_UNSUPPORTED
// when the shape or alignment does not fit (the caller then uses another
// kernel).
int gemv_q4k_imma_batch(const GemvSpec& g, int64_t M, int64_t ldx, cudaStream_t st) {
    if (M < 1 || M > 8 || g.P < 1 || g.P > kGemvMaxMats) return FTC_E_UNSUPPORTED;
    if (g.per_matrix_x || g.sel || g.peer || g.x_up) return FTC_E_UNSUPPORTED;
    if (g.stride % 16 || g.K % 256 || g.K / 256 > 4096) return FTC_E_UNSUPPORTED;
    if ((uintptr_t)g.x[0] % 16 || ldx % 4 || ldx < g.K || ldx > INT32_MAX) return FTC_E_UNSUPPORTED;
    const int nsb = (int)(g.K / 256);
    ImmaBatch B = {};
    ImmaMaps TM;
    B.P = g.P;
    B.rb_first[0] = 0;
    for (int i = 0; i < g.P; ++i) {
        if ((uintptr_t)g.W[i] % 16 || g.N[i] <= 0 || g.N[i] > (1 << 24)) return FTC_E_UNSUPPORTED;
        if (unit_map(&TM.m[i], g.W[i], g.N[i], nsb, g.stride) != FTC_OK) return FTC_E_UNSUPPORTED;
        B.y[i] = g.y[i];
        B.N[i] = (int)g.N[i];
        B.rb_first[i + 1] = B.rb_first[i] + (int)((g.N[i] + kRB - 1) / kRB);
    }
    B.R = B.rb_first[g.P];
    if (B.R > kMaxRB) return FTC_E_UNSUPPORTED;
    B.x = g.x[0];
    B.ldx = (int)ldx;
    B.nsb = nsb;
    ImmaPlan p;
    if (!plan_imma((int)M, nsb, B.R, device_sms(), p)) return FTC_E_UNSUPPORTED;
    B.KG = p.KG;
    B.nsbg = p.nsbg;
    B.G = p.G;
    B.S = p.S;
    B.NGRP = p.NGRP;
    B.use_slots = p.use_slots;
    int rc;
    switch (M) {
        case 1: rc = launch_imma<1>(TM, B, p, st); break;
        case 2: rc = launch_imma<2>(TM, B, p, st); break;
        case 3: rc = launch_imma<3>(TM, B, p, st); break;
        case 4: rc = launch_imma<4>(TM, B, p, st); break;
        case 5: rc = launch_imma<5>(TM, B, p, st); break;
        case 6: rc = launch_imma<6>(TM, B, p, st); break;
        case 7: rc = launch_imma<7>(TM, B, p, st); break;
        default: rc = launch_imma<8>(TM, B, p, st); break;
    }
    if (rc != FTC_OK) return rc;
    FTC_CUDA(cudaGetLastError());
    return FTC_OK;
}

}  // namespace ftc
