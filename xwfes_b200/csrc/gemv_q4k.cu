// gemv_q4k.cu -- the decode GEMV for Q4_K weights, batch 1:
//
//   y[n] = sum_k x[k] * W[n][k]        W: Q4_K super-blocks of 256 weights
//
// HBM-bound by design: every weight byte crosses HBM once, through a ring of
// bulk (TMA) copies into shared memory, and the SM spends ~1.7 issue slots
// per weight, so decoding keeps up with the copy rate.
//
// Exact-integer activations.  At start-up the CTA turns x into 24-bit
// integers with one power-of-two scale per 256-block: x = s_b * x_int,
// |x_int| < 2^22, error <= s_b/2 <= 2^-22 * max|x_block| (zero for
// activations whose bits fit, e.g. one-hot vectors).  x_int is kept as three
// byte planes (hi signed, mid and lo unsigned) in shared memory, so
//   sum_l q_l * x_int_l = 65536*sum(q*hi) + 256*sum(q*mid) + sum(q*lo)
// comes from six dp4a per eight 4-bit codes in exact integer arithmetic; each
// sub-block's scale and min are applied once per row.  The summation order
// differs from ft::dot_row_f32 (ft/include/ft/quant.h:86-103); the result
// agrees with the reference's fp32 sum to ~1e-6 relative.
//
// Work split.  A consumer warp owns 8 super-blocks of K (4 lanes per
// super-block: lane t of a quartet takes code bytes [32t, 32t+32), i.e.
// sub-blocks 2t (low nibbles) and 2t+1 (high nibbles)), keeps the matching
// 64 activations as plane words in registers, and every row of a chunk
// passes through it.  WK = ceil(K/2048) warps cover a row; WR groups of WK
// warps share the rows of a chunk.  One more warp is the producer: it keeps
// kStages chunks of RC rows (contiguous bytes) in flight with
// cp.async.bulk and, once consumers release a stage, refills it first and
// then adds their per-row partials in a fixed order (deterministic) into y.
//
// Launched with programmatic dependent launch: weight copies start before
// griddepcontrol.wait, activations are read after it, so back-to-back GEMVs
// overlap one kernel's tail with the next one's weight prefetch.
#include <algorithm>

#include "common.cuh"
#include "gemv_batch.cuh"
#include "sm100.cuh"

namespace ftc {

FTC_DEVSTAT_READER(devstat_gemv_q4k)

namespace {

constexpr int kStages = 4;
// Activation words per (super-block, quartet lane): 3 planes x 16 words,
// padded to 52 so that the 128-bit loads of 8 consecutive lanes (stride 52
// words = 20 banks mod 32) fall on 8 different bank quads; at 48 words they
// would collide 4-way and the 18 consumer warps' start-up loads would take
// ~2 us of shared-memory time per launch.
constexpr int kPlaneWords = 52;
constexpr int kMaxThreads = 608; // 18 consumer warps + 1 producer at <= 107 registers
constexpr size_t kMaxSmem = 227 * 1024;  // dynamic shared memory per CTA (the sm_100 limit)

}  // namespace

// Up to kGemvMaxMats weight matrices with the same K in one launch.
//  * shared activations (q/k/v, gate/up): every CTA walks all row chunks of
//    all matrices with x[0];
//  * per-matrix activations (per_matrix_x): CTAs [cta_first[p],
//    cta_first[p+1]) serve matrix p only, with x[p] (MoE experts, each with
//    its own token or hidden vector).
// Device-side expert selection: when sel is set, matrix p with
// sel_slot[p] >= 0 starts at W[p] + sel[sel_slot[p]] * sel_stride (the id
// clamped to [0, sel_max]); sel is read after the preceding kernel finishes.
struct GemvBatch {
    const uint8_t* W[kGemvMaxMats];
    float* y[kGemvMaxMats];
    const float* x[kGemvMaxMats];
    int N[kGemvMaxMats];
    int first_chunk[kGemvMaxMats + 1];  // prefix sums of ceil(N / RC)
    int cta_first[kGemvMaxMats + 1];    // per-matrix activations: CTA ranges
    int P;
    int per_matrix_x;
    const int32_t* sel;
    int64_t sel_stride;
    int sel_max;
    int sel_slot[kGemvMaxMats];
    // prefetch hint (see GemvSpec): regions of the next launch, window bytes
    int pf_n;
    const uint8_t* pf_ptr[kGemvMaxMats];
    int64_t pf_len[kGemvMaxMats];
    int64_t pf_total;
    // fused allreduce (one matrix): y = sum over the group's ranks of their
    // partial products, exchanged through peer memory (see peer_ar.cu)
    int fused;
    PeerView peer;
    int64_t x_up;  // see GemvSpec::x_up
};

namespace {

// d = a (unsigned bytes) . b (signed bytes) + c
__device__ __forceinline__ int dp4a_us(uint32_t a, uint32_t b, int c) {
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

// One 256-block of x (lane j holds elements 8j..8j+7): block scale, three
// byte planes and the sub-block sums.
__device__ __forceinline__ void plane_block(const float (&v)[8], int sb, int lane, uint32_t* planes,
                                            float* sums, float* scales) {
    float amax = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(v[i]));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    // amax in [2^p, 2^(p+1)): s_b = 2^(p-21) keeps |x / s_b| < 2^22
    const int eb = (int)((__float_as_uint(amax) >> 23) & 0xFF);
    const int se = max(eb - 21, 1);
    const float inv = __uint_as_float((uint32_t)(254 - se) << 23);
    uint32_t h[2] = {0, 0}, m[2] = {0, 0}, l[2] = {0, 0};
    int sum = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        // round(x * inv) via the 1.5 * 2^23 magic constant (x * inv is exact)
        const int q = __float_as_int(fmaf(v[i], inv, 12582912.0f)) - 0x4B400000;
        sum += q;
        h[i >> 2] |= ((uint32_t)(q >> 16) & 0xFFu) << (8 * (i & 3));
        m[i >> 2] |= ((uint32_t)(q >> 8) & 0xFFu) << (8 * (i & 3));
        l[i >> 2] |= ((uint32_t)q & 0xFFu) << (8 * (i & 3));
    }
    const int t = lane >> 3, u = 2 * (lane & 7);
    uint32_t* dst = planes + (sb * 4 + t) * kPlaneWords;
    *reinterpret_cast<uint2*>(dst + u) = make_uint2(h[0], h[1]);
    *reinterpret_cast<uint2*>(dst + 16 + u) = make_uint2(m[0], m[1]);
    *reinterpret_cast<uint2*>(dst + 32 + u) = make_uint2(l[0], l[1]);
    // sub-block sums: lanes 8t..8t+3 hold sub-block 2t, 8t+4..8t+7 sub-block 2t+1
    sum += __shfl_xor_sync(0xffffffffu, sum, 1);
    sum += __shfl_xor_sync(0xffffffffu, sum, 2);
    if ((lane & 3) == 0) sums[(sb * 4 + t) * 2 + ((lane >> 2) & 1)] = (float)sum;
    if (lane == 0) scales[sb] = __uint_as_float((uint32_t)se << 23);
}

// Per-CTA activation prologue: consumer warp w converts super-blocks w,
// w + NCW, ... (lane j: elements 8j..8j+7 of the block) into plane words,
// sub-block sums and the block scale, laid out for the consumers:
//   planes[(sb*4 + t)*kPlaneWords + plane*16 + u]   u = word within the lane's 64
//   sums[(sb*4 + t)*2 + {0: low sub-block, 1: high}],  scales[sb]
// kSilu: x is a [gate | up] row (up at x + x_up) and the activation is
// silu_gate(gate, up).
template <bool kSilu>
__device__ __forceinline__ void build_planes(const float* __restrict__ x, int64_t x_up, int nsb,
                                             int cw, int ncw, int lane, uint32_t* planes,
                                             float* sums, float* scales) {
    // the warp's blocks go four at a time: all loads of a batch are in
    // flight together, so a long x costs one L2 round trip per batch
    constexpr int kBatch = 4;
    for (int sb0 = cw; sb0 < nsb; sb0 += kBatch * ncw) {
        float4 a[kBatch], b[kBatch], ua[kBatch], ub[kBatch];
#pragma unroll
        for (int i = 0; i < kBatch; ++i) {
            const int sb = sb0 + i * ncw;
            if (sb < nsb) {
                const float4* xp = reinterpret_cast<const float4*>(x + (int64_t)sb * 256 + 8 * lane);
                a[i] = __ldg(xp);
                b[i] = __ldg(xp + 1);
                if (kSilu) {
                    const float4* up = reinterpret_cast<const float4*>(x + x_up + (int64_t)sb * 256 +
                                                                       8 * lane);
                    ua[i] = __ldg(up);
                    ub[i] = __ldg(up + 1);
                }
            }
        }
#pragma unroll
        for (int i = 0; i < kBatch; ++i) {
            const int sb = sb0 + i * ncw;
            if (sb >= nsb) break;
            float v[8] = {a[i].x, a[i].y, a[i].z, a[i].w, b[i].x, b[i].y, b[i].z, b[i].w};
            if (kSilu) {
                const float u[8] = {ua[i].x, ua[i].y, ua[i].z, ua[i].w,
                                    ub[i].x, ub[i].y, ub[i].z, ub[i].w};
#pragma unroll
                for (int j = 0; j < 8; ++j) v[j] = silu_gate(v[j], u[j]);
            }
            plane_block(v, sb, lane, planes, sums, scales);
        }
    }
}

struct LaneX {
    uint32_t h[16], m[16], l[16];
    float sum_lo, sum_hi, scale;
};

// One row: this lane's 64 weights against its activations.
// Returns s_b * (d * SQ - dmin * U), SQ = sum q*x_int, U = sum m*x_int.
__device__ __forceinline__ float q4k_row_partial(const uint8_t* blk, int t, uint32_t use_s2,
                                                 int sh0, uint32_t mask_a, uint32_t mask_b,
                                                 const LaneX& X) {
    const uint4 hd = *reinterpret_cast<const uint4*>(blk);
    const uint4 qa = *reinterpret_cast<const uint4*>(blk + 16 + 32 * t);
    const uint4 qb = *reinterpret_cast<const uint4*>(blk + 32 + 32 * t);
    const uint32_t w[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
    int hl = 0, hh = 0;
    uint32_t ml = 0, mh = 0, ll = 0, lh = 0;
#pragma unroll
    for (int u = 0; u < 8; ++u) {
        const uint32_t lo = w[u] & 0x0F0F0F0Fu;  // q of sub-block 2t, weights 4u..4u+3
        const uint32_t hi = w[u] & 0xF0F0F0F0u;  // 16 * q of sub-block 2t+1
        hl = __dp4a((int)lo, (int)X.h[u], hl);
        ml = __dp4a(lo, X.m[u], ml);
        ll = __dp4a(lo, X.l[u], ll);
        hh = dp4a_us(hi, X.h[8 + u], hh);
        mh = __dp4a(hi, X.m[8 + u], mh);
        lh = __dp4a(hi, X.l[8 + u], lh);
    }
    // scales / mins of sub-blocks 2t (byte i) and 2t+1 (byte i+1), i = sh0/8:
    //   sub-blocks 0-3: scale = s0.byte & 63, min = s1.byte & 63
    //   sub-blocks 4-7: scale = (s2.byte & 15) | (s0.byte >> 6) << 4,
    //                   min   = (s2.byte >> 4) | (s1.byte >> 6) << 4
    // branch-free: mask_a = 0x3F3F / 0x0F0F, mask_b = 0 / 0x3030 per lane
    const uint32_t s0 = hd.y, s1 = hd.z, s2 = hd.w;
    const uint32_t sa = use_s2 ? s2 : s0;
    const uint32_t ma = use_s2 ? (s2 >> 4) : s1;
    const uint32_t sc = ((sa >> sh0) & mask_a) | ((s0 >> (sh0 + 2)) & mask_b);
    const uint32_t mn = ((ma >> sh0) & mask_a) | ((s1 >> (sh0 + 2)) & mask_b);
    const int sc0 = (int)(sc & 0xFF), sc1 = (int)(sc >> 8);
    // high-nibble sums carry a factor 16 (exact: every term is a multiple of 16)
    const int ph = sc0 * hl + sc1 * (hh >> 4);                            // |.| < 2^23
    const int pm = (int)(sc0 * ml + sc1 * (mh >> 4));                     // < 2^24
    const int pl = (int)(sc0 * ll + sc1 * (lh >> 4));
    const float sq = fmaf(65536.f, (float)ph, fmaf(256.f, (float)pm, (float)pl));
    const float um = fmaf((float)(mn >> 8), X.sum_hi, (float)(mn & 0xFF) * X.sum_lo);
    const float d = h2f(hd.x), dmin = h2f(hd.x >> 16);
    return X.scale * fmaf(-dmin, um, d * sq);
}

// d = a (signed bytes) . b (unsigned bytes) + c
__device__ __forceinline__ int dp4a_su(uint32_t a, uint32_t b, int c) {
    int d;
    asm("dp4a.s32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

// N words of the bytes at p, which is only 2-byte aligned (Q6_K super-blocks
// are 210 bytes): N + 1 aligned shared-memory words and a funnel shift.
template <int N>
__device__ __forceinline__ void lds_words_a2(const uint8_t* p, uint32_t (&w)[N]) {
    const uint32_t* a =
        reinterpret_cast<const uint32_t*>(reinterpret_cast<uintptr_t>(p) & ~uintptr_t(3));
    const uint32_t sh = (uint32_t)(reinterpret_cast<uintptr_t>(p) & 3) * 8;
    uint32_t prev = a[0];
#pragma unroll
    for (int i = 0; i < N; ++i) {
        const uint32_t nx = a[i + 1];
        w[i] = __funnelshift_r(prev, nx, sh);
        prev = nx;
    }
}

// One Q6_K row: this lane's 64 weights [64t, 64t + 64) of the super-block
// against its activations (the same x range as a Q4_K lane).  Q6_K keeps
// 256 weights as two halves of 128 (ql 64 bytes, qh 32, then 16 int8 scales
// and d): in half h, weight 32q + l (quad q, l < 32) is
//   q6 = (ql[l + 32 (q & 1)] nibble q >> 1) | (qh[l] bits 2q, 2q + 1) << 4,
// value d * scale[8h + 2q + l / 16] * (q6 - 32).  Lane t takes half t >> 1,
// quads 2 (t & 1) and 2 (t & 1) + 1.  q6 - 32 is formed per byte as a signed
// byte: (q6 ^ 32) read as a 6-bit two's complement number, sign-extended
// (+ 0xC0 where bit 5 is set; no carry leaves a byte), so three dp4a per
// four weights give exact integer sums per activation digit plane; each
// 16-weight group's sums are multiplied by its scale in int32 (|.| < 2^27).
__device__ __forceinline__ float q6k_row_partial(const uint8_t* blk, int t, const LaneX& X) {
    const int h = t >> 1, qq = t & 1;
    uint32_t ql[16], qh[8], scw[1];
    lds_words_a2<16>(blk + 64 * h, ql);
    lds_words_a2<8>(blk + 128 + 32 * h, qh);
    lds_words_a2<1>(blk + 192 + 8 * h + 4 * qq, scw);
    const float d = h2f(*reinterpret_cast<const uint16_t*>(blk + 208));
    const int sh_lo = 4 * qq;
    int ph = 0, pm = 0, pl = 0;
#pragma unroll
    for (int j = 0; j < 2; ++j) {      // quad 2qq + j: ql bytes 32j.., qh bits 4qq + 2j
#pragma unroll
        for (int g = 0; g < 2; ++g) {  // 16-weight group: scale byte 2j + g of the lane's 4
            int sh = 0, sm = 0, sl = 0;
#pragma unroll
            for (int uu = 0; uu < 4; ++uu) {
                const int u = 4 * g + uu;  // weights 4u .. 4u + 3 of the quad
                const uint32_t lo = (ql[8 * j + u] >> sh_lo) & 0x0F0F0F0Fu;
                const uint32_t hx = ((qh[u] >> (sh_lo + 2 * j)) & 0x03030303u) ^ 0x02020202u;
                const uint32_t s6 = lo + hx * 16u;                  // q6 ^ 32
                const uint32_t q = s6 + (s6 & 0x20202020u) * 6u;   // q6 - 32, signed bytes
                sh = __dp4a((int)q, (int)X.h[8 * j + u], sh);
                sm = dp4a_su(q, X.m[8 * j + u], sm);
                sl = dp4a_su(q, X.l[8 * j + u], sl);
            }
            const int sc = (int)(int8_t)(uint8_t)(scw[0] >> (8 * (2 * j + g)));
            ph += sc * sh;
            pm += sc * sm;
            pl += sc * sl;
        }
    }
    const float sq = fmaf(65536.f, (float)ph, fmaf(256.f, (float)pm, (float)pl));
    return X.scale * (d * sq);
}

// One Q8_0 row stretch of 256 weights (8 blocks of 34 bytes: fp16 d, 32
// int8 codes): lane t takes blocks 2t and 2t + 1, weights [64t, 64t + 64)
// (the same x range as a Q4_K lane).  The codes are signed bytes already:
// three dp4a per four weights, exact per block; d applied per block.
__device__ __forceinline__ float q80_row_partial(const uint8_t* unit, int t, const LaneX& X) {
    float acc = 0.f;
#pragma unroll
    for (int j = 0; j < 2; ++j) {
        const uint8_t* blk = unit + 34 * (2 * t + j);
        uint32_t q[8];
        lds_words_a2<8>(blk + 2, q);
        const float d = h2f(*reinterpret_cast<const uint16_t*>(blk));
        int sh = 0, sm = 0, sl = 0;
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            sh = __dp4a((int)q[u], (int)X.h[8 * j + u], sh);
            sm = dp4a_su(q[u], X.m[8 * j + u], sm);
            sl = dp4a_su(q[u], X.l[8 * j + u], sl);
        }
        acc = fmaf(d, fmaf(65536.f, (float)sh, fmaf(256.f, (float)sm, (float)sl)), acc);
    }
    return X.scale * acc;
}

// Sum each of R per-lane values over the warp.  Halving steps exchange half
// of the values with the partner lane (xor 1, 2, ...), so after log2(R)
// steps each lane holds one row; the remaining steps are a plain butterfly.
// Lane l ends with the total of row lane_row<R>(l) (every lane of a group of
// R consecutive lanes holds a different row).
template <int R>
__device__ __forceinline__ float warp_rows_sum(float (&v)[R], int lane) {
    if constexpr (R == 1) {
        float a = v[0];
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
        return a;
    } else if constexpr (R == 2) {
        const bool b = lane & 1;
        float a = (b ? v[1] : v[0]) + __shfl_xor_sync(0xffffffffu, b ? v[0] : v[1], 1);
#pragma unroll
        for (int o = 2; o < 32; o <<= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
        return a;
    } else {  // R == 4
        const bool b0 = lane & 1, b1 = lane & 2;
        // step 1: keep rows {2*b0, 2*b0+1}
        const float k0 = (b0 ? v[2] : v[0]) + __shfl_xor_sync(0xffffffffu, b0 ? v[0] : v[2], 1);
        const float k1 = (b0 ? v[3] : v[1]) + __shfl_xor_sync(0xffffffffu, b0 ? v[1] : v[3], 1);
        // step 2: keep row 2*b0 + b1
        float a = (b1 ? k1 : k0) + __shfl_xor_sync(0xffffffffu, b1 ? k0 : k1, 2);
#pragma unroll
        for (int o = 4; o < 32; o <<= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
        return a;
    }
}

template <int R>
__device__ __forceinline__ int lane_row(int lane) {
    if constexpr (R == 4) return 2 * (lane & 1) + ((lane >> 1) & 1);
    else if constexpr (R == 2) return lane & 1;
    else return 0;
}

// matrix holding chunk c, its first row and its row count in the chunk
__device__ __forceinline__ int chunk_matrix(const GemvBatch& B, int c) {
    int p = 0;
    while (p + 1 < B.P && c >= B.first_chunk[p + 1]) ++p;
    return p;
}

// This CTA's chunks: c0, c0 + step, ... < cend (global chunk indices), and
// the activation vector they use.
struct ChunkWalk {
    int c0, step, cend;
    const float* x;
};

__device__ __forceinline__ ChunkWalk chunk_walk(const GemvBatch& B) {
    ChunkWalk w;
    if (!B.per_matrix_x) {
        w.c0 = blockIdx.x;
        w.step = gridDim.x;
        w.cend = B.first_chunk[B.P];
        w.x = B.x[0];
    } else {
        int p = 0;
        while (p + 1 < B.P && (int)blockIdx.x >= B.cta_first[p + 1]) ++p;
        w.c0 = B.first_chunk[p] + ((int)blockIdx.x - B.cta_first[p]);
        w.step = B.cta_first[p + 1] - B.cta_first[p];
        w.cend = B.first_chunk[p + 1];
        w.x = B.x[p];
    }
    return w;
}

__device__ __forceinline__ const uint8_t* matrix_base(const GemvBatch& B, int p) {
    const uint8_t* w = B.W[p];
    if (B.sel && B.sel_slot[p] >= 0) {
        const int e = min(max(B.sel[B.sel_slot[p]], 0), B.sel_max);
        w += (int64_t)e * B.sel_stride;
    }
    return w;
}

__device__ __forceinline__ void st_word(uint64_t* p, uint64_t v) {
    asm volatile("st.volatile.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ uint64_t ld_word(const uint64_t* p) {
    uint64_t v;
    asm volatile("ld.volatile.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

// Fused allreduce, after the producer has pushed this CTA's rows to every
// rank: every thread takes rows of this CTA's chunks, waits (bounded) until
// each rank's word for the row carries this launch's epoch, and writes the
// sum in rank order.  Every rank's CTA b owns the same rows (the ranks run
// the same plan), so a CTA only waits for its counterparts.
__device__ __noinline__ void fused_allreduce_tail(const GemvBatch& B, const ChunkWalk& cw, int RC) {
    named_barrier(2, blockDim.x);  // this CTA's pushes are done
    const PeerView& P = B.peer;
    grid_dependency_wait();        // (returns at once: the pushes came after it)
    const uint32_t epoch = P.ctr[0] + 1u;
    const int world = P.world;
    const uint64_t* d = P.data[P.rank] + (int64_t)(epoch & 1u) * (world + 1) * P.max_elems;
    const int64_t N = B.N[0];
    const int nck = (cw.cend - cw.c0 + cw.step - 1) / cw.step;
    uint64_t t0 = 0;
    bool ok = true;
    for (int idx = threadIdx.x; idx < nck * RC && ok; idx += blockDim.x) {
        const int ci = idx / RC;
        const int64_t row = (int64_t)(cw.c0 + ci * cw.step) * RC + (idx - ci * RC);
        if (row >= N) continue;
        uint64_t w[kPeerMaxRanks];
        uint32_t pending = (1u << world) - 1u;
        while (pending) {
#pragma unroll
            for (int s = 0; s < kPeerMaxRanks; ++s)
                if ((pending >> s) & 1u) w[s] = ld_word(d + s * P.max_elems + row);
#pragma unroll
            for (int s = 0; s < kPeerMaxRanks; ++s)
                if (((pending >> s) & 1u) && (uint32_t)(w[s] >> 32) == epoch) pending &= ~(1u << s);
            if (pending) {
                const uint64_t now = global_ns();
                if (t0 == 0) {
                    t0 = now;
                } else if (now - t0 > kWaitLimitNs) {
                    record_timeout();
                    ok = false;
                    break;
                }
            }
        }
        if (!ok) break;
        float a = __uint_as_float((uint32_t)w[0]);
#pragma unroll
        for (int s = 1; s < kPeerMaxRanks; ++s)
            if (s < world) a += __uint_as_float((uint32_t)w[s]);
        B.y[0][row] = a;
    }
    named_barrier(2, blockDim.x);
    if (threadIdx.x == 0) peer_call_done(P.ctr, epoch);
}

template <int RPW, bool kSilu, int kFmt = 0>
__global__ void __launch_bounds__(kMaxThreads, 1)
gemv_q4k_dp4a(const __grid_constant__ GemvBatch B, int64_t stride, int nsb, int WK, int WR,
              int RC) {
    extern __shared__ __align__(128) uint8_t smem[];
    // RC rows per chunk (<= RPW * WR, chosen by the host to balance CTAs);
    // stages and partial slots are sized for RPW * WR rows
    const int RM = RPW * WR;
    const int NCW = WK * WR;                   // consumer warps
    const int stage_bytes = RM * (int)stride;  // multiple of 16
    uint8_t* stg = smem;
    uint32_t* planes = reinterpret_cast<uint32_t*>(smem + kStages * stage_bytes);
    float* sums = reinterpret_cast<float*>(planes + nsb * 4 * kPlaneWords);
    float* scales = sums + nsb * 8;
    float* red = scales + nsb;  // [2 rounds][kStages][WK][RM]
    uint64_t* full = reinterpret_cast<uint64_t*>(
        (reinterpret_cast<uintptr_t>(red + 2 * kStages * WK * RM) + 15) & ~uintptr_t(15));
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
    grid_launch_dependents();
    const ChunkWalk cw = chunk_walk(B);

    if (warp == NCW) {
        // ------------------------------------------------ producer warp
        // (weights do not depend on the preceding kernel, the expert ids do)
        if (B.sel) grid_dependency_wait();
        const uint64_t pol = policy_evict_first();
        bool ok = true;
        int it = 0;
        // fused allreduce: this call's epoch, read before the first push,
        // once the previous grid on the stream has completed (the weight
        // copies above the wait still start early)
        uint32_t epoch = 0;
        bool have_epoch = false;
        auto reduce = [&](int j) {  // partials of iteration j -> y
            const int s = j % kStages, rd = (j / kStages) & 1;
            const int c = cw.c0 + j * cw.step;
            const int p = chunk_matrix(B, c);
            const int lc = c - B.first_chunk[p];
            const int rows = min(RC, B.N[p] - lc * RC);
            for (int row = lane; row < rows; row += 32) {
                const float* r = red + ((rd * kStages + s) * WK) * RM + row;
                float v = 0.f;
                for (int wk = 0; wk < WK; ++wk) v += r[wk * RM];
                if (B.fused) {  // this rank's partial row, tagged, into every rank's slot
                    const PeerView& P = B.peer;
                    if (!have_epoch) {
                        grid_dependency_wait();
                        epoch = P.ctr[0] + 1u;
                        have_epoch = true;
                    }
                    const int64_t slot = ((int64_t)(epoch & 1u) * (P.world + 1) + P.rank) *
                                             P.max_elems + (int64_t)lc * RC + row;
                    const uint64_t wv = ((uint64_t)epoch << 32) | __float_as_uint(v);
                    for (int q = 0; q < P.world; ++q) st_word(P.data[q] + slot, wv);
                } else {
                    B.y[p][(int64_t)lc * RC + row] = v;
                }
            }
        };
        auto issue = [&](int c, int s) {
            if (lane == 0) {
                const int p = chunk_matrix(B, c);
                const int lc = c - B.first_chunk[p];
                const int rows = min(RC, B.N[p] - lc * RC);
                const uint32_t bytes = (uint32_t)(rows * stride);
                mbar_arrive_expect_tx(&full[s], bytes);
                bulk_g2s(stg + s * stage_bytes, matrix_base(B, p) + (int64_t)lc * RC * stride, bytes,
                         &full[s], pol);
            }
            __syncwarp();
        };
        for (int c = cw.c0; c < cw.cend; c += cw.step, ++it) {
            const int s = it % kStages;
            if (it >= kStages) {
                // consumers are done with iteration it - kStages: refill the
                // stage first, then fold that iteration's partials into y
                ok = mbar_wait_warp(&empty[s], ((it / kStages) - 1) & 1);
                if (!ok) break;
                issue(c, s);
                reduce(it - kStages);
            } else {
                issue(c, s);
            }
        }
        if (B.pf_n > 0 && lane == 0) {
            // this CTA's slice of the next launch's first bytes, into L2
            const int64_t per = ((B.pf_total / gridDim.x) + 15) & ~int64_t(15);
            int64_t lo = (int64_t)blockIdx.x * per;
            const int64_t hi = min(lo + per, B.pf_total);
            int64_t base = 0;
            for (int r = 0; r < B.pf_n && lo < hi; ++r) {
                const int64_t end = base + B.pf_len[r];
                while (lo < hi && lo < end) {
                    const int64_t n = min(min(hi, end) - lo, (int64_t)1 << 20);
                    bulk_prefetch_l2(B.pf_ptr[r] + (lo - base), (uint32_t)n);
                    lo += n;
                }
                base = end;
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
        if (B.fused) fused_allreduce_tail(B, cw, RC);
        return;
    }

    // ---------------------------------------------------- consumer warps
    grid_dependency_wait();  // x may be the preceding kernel's output
    build_planes<kSilu>(cw.x, B.x_up, nsb, warp, NCW, lane, planes, sums, scales);
    named_barrier(1, NCW * 32);

    const int wr = warp / WK, wk = warp % WK;
    const int qd = lane >> 2, t = lane & 3;
    const int sb = wk * 8 + qd;
    const bool valid = sb < nsb;
    const uint32_t use_s2 = t >= 2;          // sub-blocks 4..7 use the split encoding
    const int sh0 = 8 * ((2 * t) & 3);       // byte of sub-block 2t within its word
    const uint32_t mask_a = use_s2 ? 0x0F0Fu : 0x3F3Fu;
    const uint32_t mask_b = use_s2 ? 0x3030u : 0u;
    LaneX X;
    if (valid) {
        const uint4* src = reinterpret_cast<const uint4*>(planes + (sb * 4 + t) * kPlaneWords);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint4 a = src[i], b = src[4 + i], c = src[8 + i];
            X.h[4 * i] = a.x; X.h[4 * i + 1] = a.y; X.h[4 * i + 2] = a.z; X.h[4 * i + 3] = a.w;
            X.m[4 * i] = b.x; X.m[4 * i + 1] = b.y; X.m[4 * i + 2] = b.z; X.m[4 * i + 3] = b.w;
            X.l[4 * i] = c.x; X.l[4 * i + 1] = c.y; X.l[4 * i + 2] = c.z; X.l[4 * i + 3] = c.w;
        }
        X.sum_lo = sums[(sb * 4 + t) * 2];
        X.sum_hi = sums[(sb * 4 + t) * 2 + 1];
        X.scale = scales[sb];
    }

    // Super-blocks past K are computed on in-bounds bytes (clamped) and
    // discarded by a select; rows past the chunk's end are skipped with a
    // branch that is uniform across the warp (the row index depends on the
    // warp only), so the row loop never diverges.
    const int sb_ld = valid ? sb : nsb - 1;
    int it = 0;
    for (int c = cw.c0; c < cw.cend; c += cw.step, ++it) {
        const int s = it % kStages, rd = (it / kStages) & 1;
        if (!mbar_wait_warp(&full[s], (it / kStages) & 1)) break;
        const int p = chunk_matrix(B, c);
        const int rows = min(RC, B.N[p] - (c - B.first_chunk[p]) * RC);
        // bytes per 256 weights: Q4_K 144, Q6_K 210, Q8_0 8 x 34
        constexpr int kUnit = kFmt == kGemvQ6K ? 210 : kFmt == kGemvQ80 ? 272 : 144;
        const uint8_t* base = stg + s * stage_bytes + sb_ld * kUnit + wr * stride;
        float acc[RPW];
#pragma unroll
        for (int i = 0; i < RPW; ++i) {
            acc[i] = 0.f;
            if (wr + WR * i < rows) {
                const uint8_t* rb = base + (WR * i) * stride;
                const float v = kFmt == kGemvQ6K ? q6k_row_partial(rb, t, X)
                              : kFmt == kGemvQ80 ? q80_row_partial(rb, t, X)
                                                 : q4k_row_partial(rb, t, use_s2, sh0, mask_a,
                                                                   mask_b, X);
                acc[i] = valid ? v : 0.f;
            }
        }
        // transposed butterfly: after log2(RPW) halving steps lane l holds one
        // row's partial (row index from its low bits), then a plain reduction
        float v = warp_rows_sum<RPW>(acc, lane);
        const int row = lane_row<RPW>(lane);
        if (lane < RPW) red[((rd * kStages + s) * WK + wk) * RM + wr + WR * row] = v;
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
    }
    if (B.fused) fused_allreduce_tail(B, cw, RC);
}

struct Q4kPlan {
    int WK, WR, RPW, RC, grid, threads;
    size_t smem;
};

bool plan_q4k(int64_t Ntot, int64_t K, int64_t stride, Q4kPlan& p) {
    const int nsb = (int)(K / 256);
    p.WK = (nsb + 7) / 8;
    if (p.WK > 15) return false;
    p.WR = std::max(1, (kMaxThreads / 32 - 1) / p.WK);  // consumer warps + 1 producer
    const int sms = device_sms();
    // rows per chunk: ~48 KB chunks, but small enough that every SM gets two
    int64_t rc = std::max<int64_t>(1, 49152 / stride + p.WR / 2);
    rc = std::min<int64_t>(rc, std::max<int64_t>(p.WR, Ntot / (2 * (int64_t)sms)));
    const int64_t rpw = std::max<int64_t>(1, rc / p.WR);
    p.RPW = rpw >= 4 ? 4 : (rpw >= 2 ? 2 : 1);
    while (p.RPW > 1 && p.RPW * p.WR > 64) p.RPW /= 2;  // the producer reduces <= 2 rows per lane
    if (p.RPW * p.WR > 64) return false;
    const int RC = p.RPW * p.WR;
    p.threads = (p.WK * p.WR + 1) * 32;
    p.smem = (size_t)kStages * RC * stride                 // weight stages
             + (size_t)nsb * 4 * kPlaneWords * 4          // activation planes
             + (size_t)nsb * 9 * 4                         // sums + scales
             + (size_t)2 * kStages * p.WK * RC * 4         // partials, two rounds
             + 16 + 2 * kStages * 8;                        // barriers
    while (p.smem > kMaxSmem && p.RPW > 1) {               // shrink chunks to fit
        p.smem -= (size_t)kStages * (p.RPW / 2) * p.WR * stride;
        p.smem -= (size_t)2 * kStages * p.WK * (p.RPW / 2) * p.WR * 4;
        p.RPW /= 2;
    }
    if (p.smem > kMaxSmem || p.threads > kMaxThreads) return false;
    p.RC = p.RPW * p.WR;
    return true;
}

// Rows per chunk for a batch: the largest RC <= rc_max whose chunk count
// fills the last round of CTAs best (a small launch otherwise ends with one
// mostly idle round).
int balance_rc(int P, const int64_t* N, int rc_max, int sms) {
    int best = rc_max;
    double best_eff = 0.0;
    for (int rc = rc_max; rc >= std::max(1, rc_max / 2); --rc) {
        int64_t ch = 0;
        for (int i = 0; i < P; ++i) ch += (N[i] + rc - 1) / rc;
        const int64_t rounds = (ch + sms - 1) / sms;
        // useful work / (rounds * rc): rewards full rounds and big chunks
        int64_t rows = 0;
        for (int i = 0; i < P; ++i) rows += N[i];
        const double eff = (double)rows / ((double)rounds * sms * rc);
        if (eff > best_eff + 1e-9) {
            best_eff = eff;
            best = rc;
        }
    }
    return best;
}

}  // namespace

// Fast path for Q4_K, M == 1.  Returns FTC_E_UNSUPPORTED when the shape or
// alignment does not fit (the caller then uses the general kernels).
int gemv_q4k_batch(const GemvSpec& g, cudaStream_t st) {
    const int P = g.P;
    if (P < 1 || P > kGemvMaxMats) return FTC_E_UNSUPPORTED;
    if (g.stride % 16 || g.K % 256) return FTC_E_UNSUPPORTED;
    int64_t ntot = 0;
    for (int i = 0; i < P; ++i) {
        if ((uintptr_t)g.W[i] % 16 || g.N[i] <= 0 || g.N[i] > (1 << 30)) return FTC_E_UNSUPPORTED;
        if ((uintptr_t)g.x[g.per_matrix_x ? i : 0] % 16) return FTC_E_UNSUPPORTED;
        ntot += g.N[i];
    }
    if (g.sel && (g.sel_stride % 16 || g.sel_max < 0)) return FTC_E_UNSUPPORTED;
    if (g.peer && (P != 1 || g.per_matrix_x || g.sel || g.N[0] > g.peer->max_elems))
        return FTC_E_UNSUPPORTED;
    if (g.x_up < 0 || g.x_up % 4) return FTC_E_UNSUPPORTED;  // up half 16-byte aligned
    if (g.wfmt && (g.peer || g.x_up || g.sel || g.per_matrix_x)) return FTC_E_UNSUPPORTED;
    Q4kPlan p;
    if (!plan_q4k(ntot, g.K, g.stride, p)) return FTC_E_UNSUPPORTED;
    const int sms = device_sms();
    const int RC = balance_rc(P, g.N, p.RPW * p.WR, sms);
    GemvBatch B = {};
    B.P = P;
    B.per_matrix_x = g.per_matrix_x;
    B.sel = g.sel;
    B.sel_stride = g.sel_stride;
    B.sel_max = g.sel_max;
    B.first_chunk[0] = 0;
    for (int i = 0; i < P; ++i) {
        B.W[i] = g.W[i];
        B.y[i] = g.y[i];
        B.x[i] = g.x[g.per_matrix_x ? i : 0];
        B.N[i] = (int)g.N[i];
        B.sel_slot[i] = g.sel ? g.sel_slot[i] : -1;
        B.first_chunk[i + 1] = B.first_chunk[i] + (int)((g.N[i] + RC - 1) / RC);
    }
    // prefetch hint: the first kGemvPrefetchWindow bytes of the next launch,
    // in 16-byte multiples (a region's tail below 16 bytes is left out)
    B.pf_n = 0;
    B.pf_total = 0;
    for (int r = 0; r < g.pf_n && r < kGemvMaxMats && B.pf_total < kGemvPrefetchWindow; ++r) {
        if (!g.pf_ptr[r] || (uintptr_t)g.pf_ptr[r] % 16 || g.pf_len[r] < 16) continue;
        const int64_t n = std::min(g.pf_len[r] & ~int64_t(15), kGemvPrefetchWindow - B.pf_total);
        B.pf_ptr[B.pf_n] = g.pf_ptr[r];
        B.pf_len[B.pf_n] = n;
        B.pf_total += n;
        ++B.pf_n;
    }
    const int nchunks = B.first_chunk[P];
    p.grid = std::min(nchunks, sms);
    B.fused = g.peer ? 1 : 0;
    B.x_up = g.x_up;
    if (g.peer) {
        B.peer = *g.peer;
    }
    if (g.per_matrix_x) {
        // one CTA per matrix, then each further CTA to the matrix with the
        // most chunks per CTA (no CTA without a chunk)
        int cnt[kGemvMaxMats], used = P;
        for (int i = 0; i < P; ++i) cnt[i] = 1;
        for (const int grid = std::max(p.grid, P); used < grid; ++used) {
            int best = -1;
            double load = 0.0;
            for (int i = 0; i < P; ++i) {
                const int ch = B.first_chunk[i + 1] - B.first_chunk[i];
                if (cnt[i] < ch && (double)ch / cnt[i] > load) {
                    load = (double)ch / cnt[i];
                    best = i;
                }
            }
            if (best < 0) break;
            ++cnt[best];
        }
        B.cta_first[0] = 0;
        for (int i = 0; i < P; ++i) B.cta_first[i + 1] = B.cta_first[i] + cnt[i];
        p.grid = B.cta_first[P];
    }
    const int nsb = (int)(g.K / 256);
    // opt in to large dynamic shared memory once per instantiation and device
    auto launch = [&](auto kern, int) -> int {
        const int orc = opt_in_smem(reinterpret_cast<const void*>(kern), (int)kMaxSmem,
                                    "cudaFuncSetAttribute(gemv_q4k_dp4a)");
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
        const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, B, g.stride, nsb, p.WK, p.WR, RC);
        if (e != cudaSuccess) return cuda_error(e, "launch gemv_q4k_dp4a");
        return FTC_OK;
    };
    int rc;
    if (g.wfmt == kGemvQ6K)
        rc = p.RPW == 4 ? launch(gemv_q4k_dp4a<4, false, kGemvQ6K>, 8)
           : p.RPW == 2 ? launch(gemv_q4k_dp4a<2, false, kGemvQ6K>, 7)
                        : launch(gemv_q4k_dp4a<1, false, kGemvQ6K>, 6);
    else if (g.wfmt == kGemvQ80)
        rc = p.RPW == 4 ? launch(gemv_q4k_dp4a<4, false, kGemvQ80>, 11)
           : p.RPW == 2 ? launch(gemv_q4k_dp4a<2, false, kGemvQ80>, 10)
                        : launch(gemv_q4k_dp4a<1, false, kGemvQ80>, 9);
    else if (g.x_up == 0)
        rc = p.RPW == 4 ? launch(gemv_q4k_dp4a<4, false>, 2)
           : p.RPW == 2 ? launch(gemv_q4k_dp4a<2, false>, 1)
                        : launch(gemv_q4k_dp4a<1, false>, 0);
    else
        rc = p.RPW == 4 ? launch(gemv_q4k_dp4a<4, true>, 5)
           : p.RPW == 2 ? launch(gemv_q4k_dp4a<2, true>, 4)
                        : launch(gemv_q4k_dp4a<1, true>, 3);
    if (rc != FTC_OK) return rc;
    FTC_CUDA(cudaGetLastError());
    return FTC_OK;
}

// Several matrices sharing x (q/k/v, gate/up); optional prefetch hint for
// the next launch (n_next regions, see GemvSpec).
int gemv_q4k_fast_multi(int P, const uint8_t* const* W, const int64_t* N, float* const* y,
                        int64_t stride, int64_t K, const float* x, cudaStream_t st,
                        int n_next = 0, const uint8_t* const* next_w = nullptr,
                        const int64_t* next_bytes = nullptr) {
    if (P < 1 || P > kGemvMaxMats) return FTC_E_UNSUPPORTED;
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
    g.pf_n = std::min(n_next, kGemvMaxMats);
    for (int i = 0; i < g.pf_n; ++i) {
        g.pf_ptr[i] = next_w[i];
        g.pf_len[i] = next_bytes[i];
    }
    return gemv_q4k_batch(g, st);
}

int gemv_q4k_fast(const uint8_t* W, int64_t stride, int64_t N, int64_t K, const float* x,
                  float* y, cudaStream_t st) {
    return gemv_q4k_fast_multi(1, &W, &N, &y, stride, K, x, st);
}

// The same persistent kernel on Q6_K rows (the config-2 output head) or
// Q8_0 rows (config 1), batch 1.  FTC_E_UNSUPPORTED when the shape or
// alignment does not fit.
int gemv_kq_fast(int wfmt, const uint8_t* W, int64_t stride, int64_t N, int64_t K, const float* x,
                 float* y, cudaStream_t st) {
    GemvSpec g = {};
    g.P = 1;
    g.K = K;
    g.stride = stride;
    g.x[0] = x;
    g.W[0] = W;
    g.N[0] = N;
    g.y[0] = y;
    g.wfmt = wfmt;
    return gemv_q4k_batch(g, st);
}

}  // namespace ftc
