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
// One persistent CTA per SM, warp-specialized (15 warps):
//   warp 0      TMA: activation tiles (BN tokens x 64 k, 128-byte swizzle)
//               into the NB-slot B ring.  Also owns TMEM.
//   warp 14     TMA: raw Q4_K tiles (128 rows x one 144-byte super-block)
//               into a 2-6 slot ring, independently of the B ring.
//   warp 1      one thread issues tcgen05.mma 128 x BN x 16 (A = weights,
//               B = tokens, both K-major from shared memory) into a TMEM
//               accumulator (two of them, so the epilogue of tile i overlaps
//               the MMAs of tile i+1).
//   warps 2-5   epilogue: tcgen05.ld 32 lanes x 32 columns, convert, store
//               Y[token][row] (a warp writes 32 consecutive n per token).
//   warps 6-13  dequant: thread (row r, half h) decodes 32 weights of one
//               64-wide k-step (codes of group g, both nibbles) -- packed fp16
//               arithmetic for fp16 operands, fp32 with one rounding for bf16
//               (see dequant_pairs) -- and writes them either in the
//               128-byte-swizzled K-major shared-memory layout the MMA reads
//               (256-token tiles), or with tcgen05.st into tensor memory after
//               the accumulators, where the MMA reads its A operand (128-token
//               tiles: row r in TMEM lane r, two k per 32-bit column).
// Every pipeline wait is bounded in time (sm100.cuh); a kernel that gives up
// records a status and returns.
//
// Grouped mode (MoE experts).  Rows [offsets[g], offsets[g] + counts[g]) of X
// and Y belong to group g and multiply weight plane g (expert g); counts and
// offsets are read on the device, so a router kernel can produce them in the
// same stream with no host round trip.  One or two weight sets (gate and up)
// share the tokens; set s writes columns [s*N, (s+1)*N) of Y.  A tile with
// fewer tokens than BN issues a narrower MMA (N rounded up to 16) and loads a
// shorter activation box (32, 64, ... rows).
//
// Schedule.  Full waves of whole tiles (CTA b: tiles b, b + G, ...), then
// the tiles of the last, partial wave stream-K: their tiles x K/256
// super-block steps cut into one equal contiguous range per CTA, so every SM
// gets the same work (224 tiles on 148 SMs would otherwise be 1.5 waves); a
// tile cut by a range boundary gets fp32 partials from each piece, summed in
// range order by the piece that arrives last.
//
// Row scales.  With row_exp set, output row m is multiplied by 2^row_exp[m]
// in the epilogue (exact): callers feed fp16 rows scaled by 2^-row_exp into
// fp16's range (ftc_rows_to_f16) and get unscaled results.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <cstring>
#include <mutex>
#include <type_traits>

#include "common.cuh"
#include "sm100.cuh"

namespace ftc {

constexpr int kGemmMaxGroups = 256;

// Token groups of one launch (see the grouped mode above).
struct GemmGroups {
    const int32_t* counts;   // device [G] rows per group; nullptr: one group of all M rows
    const int32_t* offsets;  // device [G] first row of each group
    int G;                   // groups = weight planes
    int n_sets;              // weight tensors sharing the tokens (1, or 2 for gate + up)
    int64_t ldy;             // Y row pitch in elements
    const int32_t* row_exp;  // optional: Y row m is multiplied by 2^row_exp[m] (exact)
    // stream-K scratch (set by the launcher; nullptr: whole tiles only)
    uint32_t* counters;  // [CTAs][kEpiWarps] arrivals of cut tiles (zero between launches)
    float* part;         // [2 * CTAs][BN][BM] fp32 partials of cut tiles
};

namespace {

constexpr int kXMaps = 4;  // activation boxes of 32, 64, 128 and BN rows

struct XMaps {
    CUtensorMap m[kXMaps];
};

constexpr int BM = 128;       // weight rows per tile (MMA M)
constexpr int BK = 64;        // k per stage: one 128-byte swizzle row of 16-bit values
constexpr int kRawBytes = BM * 144;
constexpr int kEpiWarps = 4;
constexpr int kTeamWarps = 8;  // dequant warps per team

// Kernel shape.  DT dequant teams of 8 warps take alternate super-blocks;
// each team has its own NAT-stage slice of the dequantized weight ring and
// its own RAWT-slot slice of the raw ring, so every ring has one producer and
// one consumer and an mbarrier is never waited on more than one phase ahead.
// MI MMA-issuing threads (1 or 2, in separate warps) take alternate k-steps
// of every tile, each into its own accumulator; the epilogue adds them in
// issuer order.  One issuing thread spends ~640 cycles of its own per 64-wide
// k-step (waits, fence, descriptors, four MMAs, two commits), which bounds
// small token counts, where the MMAs themselves are short.
template <int BN_, int DT_, int NAT_, int NB_, int RAWT_, bool ATM_ = false, int MI_ = 1>
struct Cfg {
    static constexpr int BN = BN_, DT = DT_, NAT = NAT_, NB = NB_, RAWT = RAWT_, MI = MI_;
    static_assert(MI == 1 || MI == 2, "one or two MMA issuers");
    // ATM: dequantized weight stages live in tensor memory (tcgen05.st by the
    // dequant warps, read by the MMA as its A operand), after the
    // accumulators; otherwise in shared memory (128-byte swizzle).
    static constexpr bool ATM = ATM_;
    // On the 256-token tile every pipeline wait sleeps between tests (the
    // thread wakes when the phase completes), so waiting warps leave their
    // issue slots to the dequant and MMA warps (measured: M = 2048 and 8192
    // 2.7-3.7 % faster).  The smaller tiles, bound by the dequant warps'
    // latency, lose to the wake-up delay (2-4 % at 16-64 tokens) and poll.
    static constexpr uint32_t SLEEP_NS = BN_ >= 256 ? 20000u : 0u;
    static constexpr int NA = DT * NAT;           // dequantized weight stages
    static constexpr int RAW = DT * RAWT;         // raw super-block slots
    static constexpr int WARPS = 2 + kEpiWarps + DT * kTeamWarps + 1 + (MI - 1);
    static constexpr int THREADS = 32 * WARPS;
    static constexpr int RAW_WARP = 2 + kEpiWarps + DT * kTeamWarps;  // issues the raw weight tiles
    static constexpr int MMA2_WARP = RAW_WARP + 1;                     // second issuer (MI == 2)
    static constexpr int A_BYTES = BM * BK * 2;   // 16 KB
    static constexpr int B_BYTES = BN * BK * 2;
    static constexpr int ACC_COLS = 2 * MI * BN;  // [2 tiles in flight][MI issuers] accumulators
    static constexpr int A_COL0 = ACC_COLS;       // first TMEM column of the A stages (ATM)
    static constexpr int A_COLS = BK / 2;         // 32 columns: 64 16-bit k per lane
    static constexpr int TMEM_COLS = ATM ? 512 : (ACC_COLS <= 256 ? 256 : 512);
    static_assert(!ATM || A_COL0 + NA * A_COLS <= 512, "tensor memory");
    // shared layout (all tiles 1024-byte aligned)
    static constexpr int OFF_A = 0;
    static constexpr int OFF_B = OFF_A + (ATM ? 0 : NA * A_BYTES);
    static constexpr int OFF_RAW = OFF_B + NB * B_BYTES;
    static constexpr int OFF_BAR = OFF_RAW + RAW * kRawBytes;
    // barriers: a_full[NA] a_empty[NA] b_full[NB] b_empty[NB] raw_full[RAW]
    // raw_empty[RAW] acc_full[2] acc_empty[2]
    static constexpr int N_BARS = 2 * NA + 2 * NB + 2 * RAW + 4;
    // tile schedule: first tile, first row and row count of each group, then
    // the CTA's work ranges (8 ints)
    static constexpr int OFF_SCHED = OFF_BAR + N_BARS * 8 + 16;
    static constexpr int SMEM = OFF_SCHED + (3 * kGemmMaxGroups + 1 + 8) * 4 + 1024;  // +1024: alignment slack
    static_assert(SMEM <= 227 * 1024, "shared memory");
};

// Ring positions of super-block rc (in kernel order) and its k-step g: the
// owning team, its raw slot and that slot's phase, and the A stage / phase.
template <class C>
struct RingPos {
    int team, raw_slot, a_stage;
    uint32_t raw_phase, a_phase;
    __device__ __forceinline__ RingPos(uint32_t rc, int g) {
        team = (int)(rc % C::DT);
        const uint32_t lr = rc / C::DT;            // team-local super-block
        raw_slot = team * C::RAWT + (int)(lr % C::RAWT);
        raw_phase = (lr / C::RAWT) & 1;
        const uint32_t la = lr * 4 + (uint32_t)g;  // team-local k-step
        a_stage = team * C::NAT + (int)(la % C::NAT);
        a_phase = (la / C::NAT) & 1;
    }
};

// Tile t of the schedule: group, weight set, 128-row block of W, and the
// group's token rows it covers.  Tiles of a group run token tile by token
// tile, weight blocks fastest, so concurrent CTAs share the activation tile.
struct TileRef {
    int g, set, nt, row0, rows;
};

// Cut of the last, partial wave of whole tiles, computed alike by the
// kernel and by the launcher (which sizes a launch with fewer tiles than SMs
// to the CTAs that get work).  Given the scratch, the tail's W = rem x nsb
// super-block steps are cut one of two ways.  Aligned: S CTAs per tail
// tile, each on nsb/S of its steps, so no range crosses a tile boundary (the
// fewest S with the shortest range that fits the grid).  Stream-K: one CTA
// per kMinPiece steps or more, up to the grid, ranges crossing tile
// boundaries (such a CTA drains its pipeline and runs an epilogue twice).
// With W >= Gc every range is non-empty, which the piece bookkeeping relies
// on.  Each is charged its longest range plus an estimate, in super-block
// steps, of its fix-up (128 KB of fp32 partial per piece on the 256-token
// tile) and, for stream-K, the second epilogue; the cheaper runs when it
// shortens the schedule by 5 % or more, else every tile runs whole (a last
// wave that is nearly full, or one of many waves, gains less than the cut
// tiles cost).  Any grid size gives a valid plan.
struct TailPlan {
    int t_full;  // tiles run whole, round robin over the grid
    int W;       // steps of the cut tail (0: none)
    int Gc;      // CTAs sharing them, ranges [b*W/Gc, (b+1)*W/Gc)
};

template <int BN>
__host__ __device__ inline TailPlan plan_tail(int tiles, int nsb, int Gl, bool scratch) {
    constexpr int kMinPiece = BN >= 256 ? 4 : 2;
    constexpr int kCostAligned = BN >= 256 ? 4 : 2;
    constexpr int kCostStreamK = BN >= 256 ? 8 : 3;
    const int waves = tiles / Gl, rem = tiles - waves * Gl;
    const int w_rem = rem * nsb;
    const int span_whole = (waves + (rem ? 1 : 0)) * nsb;
    int s_al = 0;
    if (rem) {
        s_al = Gl / rem < nsb / kMinPiece ? Gl / rem : nsb / kMinPiece;
        if (s_al >= 2) {
            const int len = (nsb + s_al - 1) / s_al;
            s_al = (nsb + len - 1) / len;
        }
    }
    const int span_al = s_al >= 2 ? waves * nsb + (nsb + s_al - 1) / s_al + kCostAligned : (1 << 30);
    const int per = w_rem / kMinPiece > 1 ? w_rem / kMinPiece : 1;
    const int g_sk = Gl < per ? Gl : per;
    const int span_sk = waves * nsb + (w_rem + g_sk - 1) / g_sk + kCostStreamK;
    const bool aligned = span_al <= span_sk;
    const int span_cut = aligned ? span_al : span_sk;
    // (W x (Gl + 1) below 2^31: the range and owner arithmetic is 32-bit)
    const bool cut = scratch && rem > 0 && 20 * span_cut < 19 * span_whole &&
                     (long long)w_rem * (Gl + 1) < 0x7fffffffLL;
    TailPlan p;
    p.t_full = cut ? waves * Gl : tiles;
    p.W = cut ? w_rem : 0;
    p.Gc = cut ? (aligned ? rem * s_al : g_sk) : 0;
    return p;
}

template <int BN>
__device__ __forceinline__ TileRef tile_ref(int tile, const int* s_start, const int* s_base,
                                            const int* s_cnt, int G, int n_tiles, int n_all) {
    int lo = 0, hi = G - 1;  // last group whose first tile is <= tile
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (s_start[mid] <= tile) lo = mid;
        else hi = mid - 1;
    }
    const int local = tile - s_start[lo];
    const int tt = local / n_all, na = local - tt * n_all;
    TileRef r;
    r.g = lo;
    r.set = na / n_tiles;
    r.nt = na - r.set * n_tiles;
    r.row0 = s_base[lo] + tt * BN;
    r.rows = min(BN, s_cnt[lo] - tt * BN);
    return r;
}

// rows of activation box i: 32, 64, 128, then BN (every box at most BN)
__host__ __device__ constexpr int xbox_rows(int i, int BN) {
    return (32 << i) < BN && i < kXMaps - 1 ? (32 << i) : BN;
}



// Scale and min of all 8 sub-blocks of a Q4_K super-block header (d, dmin,
// 12 packed bytes): fdl[j] = d*sc_j and fnml[j] = -dmin*m_j in fp32 (exact),
// and for fp16 operands also as fp16 pairs dl2[j] / nml2[j] (one rounding).
template <typename OP>
__device__ __forceinline__ void decode_scales(const uint4 hd, float (&fdl)[8], float (&fnml)[8],
                                              uint32_t (&dl2)[8], uint32_t (&nml2)[8]) {
    const float d = h2f(hd.x), dmin = h2f(hd.x >> 16);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        int sc, mn;
        q4k_scale_min(hd.y, hd.z, hd.w, j, sc, mn);
        fdl[j] = d * (float)sc;
        fnml[j] = -(dmin * (float)mn);
        if constexpr (std::is_same<OP, __half>::value) {
            const __half2 a = __float2half2_rn(fdl[j]);
            const __half2 b = __float2half2_rn(fnml[j]);
            dl2[j] = *reinterpret_cast<const uint32_t*>(&a);
            nml2[j] = *reinterpret_cast<const uint32_t*>(&b);
        } else {
            dl2[j] = nml2[j] = 0;
        }
    }
}

// packed fp32x2 arithmetic (two floats in one 64-bit register, low = first)
__device__ __forceinline__ uint64_t pack_f2(float a, float b) {
    return (uint64_t)__float_as_uint(a) | ((uint64_t)__float_as_uint(b) << 32);
}

__device__ __forceinline__ uint64_t add_f2(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}

__device__ __forceinline__ uint64_t fma_f2(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}

// (lo, hi) floats -> bf16x2 (round to nearest even), lo in the low half
__device__ __forceinline__ uint32_t bf2_of(uint64_t v) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(__uint_as_float((uint32_t)v),
                                                   __uint_as_float((uint32_t)(v >> 32)));
    return *reinterpret_cast<const uint32_t*>(&h);
}

__device__ __forceinline__ uint32_t hfma2_u(uint32_t a, uint32_t b, uint32_t c) {
    const __half2 r = __hfma2(*reinterpret_cast<const __half2*>(&a),
                              *reinterpret_cast<const __half2*>(&b),
                              *reinterpret_cast<const __half2*>(&c));
    return *reinterpret_cast<const uint32_t*>(&r);
}

__device__ __forceinline__ uint32_t hsub2_u(uint32_t a, uint32_t b) {
    const __half2 r = __hsub2(*reinterpret_cast<const __half2*>(&a),
                              *reinterpret_cast<const __half2*>(&b));
    return *reinterpret_cast<const uint32_t*>(&r);
}


// Eight weights of one code word: byte i holds q_lo (k = 4u + i of the low
// sub-block) and q_hi (same k of the high sub-block).
//  fp16 operands: each pair of neighbouring bytes becomes half2(1024 + q0,
//    1024 + q1) by placing the nibbles in the mantissa of 0x6400 (1024.0);
//    subtracting 1024 is exact, and one fused multiply-add gives
//    fp16(q * fp16(d*sc) - fp16(dmin*m)) with a single rounding.
//  bf16 operands: w = (d*sc)*q - dmin*m in fp32 (the product is exact, the
//    subtraction rounds once, as the reference's dequant_row) and one
//    rounding to bf16 -- bf16's coarser grid leaves no room for the fp16
//    rounding of the scales.
template <typename OP>
__device__ __forceinline__ void dequant_pairs(uint32_t w, uint32_t dl_lo, uint32_t nml_lo,
                                              uint32_t dl_hi, uint32_t nml_hi, float fdl_lo,
                                              float fml_lo, float fdl_hi, float fml_hi,
                                              uint32_t& lo01, uint32_t& lo23, uint32_t& hi01,
                                              uint32_t& hi23) {
    if constexpr (std::is_same<OP, __half>::value) {
        constexpr uint32_t kMagic = 0x64006400u;
        const uint32_t p01 = __byte_perm(w, 0, 0x4140);  // byte1 << 16 | byte0
        const uint32_t p23 = __byte_perm(w, 0, 0x4342);  // byte3 << 16 | byte2
        const uint32_t q_lo01 = hsub2_u((p01 & 0x000F000Fu) | kMagic, kMagic);
        const uint32_t q_lo23 = hsub2_u((p23 & 0x000F000Fu) | kMagic, kMagic);
        const uint32_t q_hi01 = hsub2_u(((p01 >> 4) & 0x000F000Fu) | kMagic, kMagic);
        const uint32_t q_hi23 = hsub2_u(((p23 >> 4) & 0x000F000Fu) | kMagic, kMagic);
        lo01 = hfma2_u(q_lo01, dl_lo, nml_lo);
        lo23 = hfma2_u(q_lo23, dl_lo, nml_lo);
        hi01 = hfma2_u(q_hi01, dl_hi, nml_hi);
        hi23 = hfma2_u(q_hi23, dl_hi, nml_hi);
    } else {
        // q -> float via the 2^23 magic (exact), then packed fp32x2 FMAs:
        // fp32(q*dl - ml) with the product exact, one rounding, then bf16.
        const uint32_t lo4 = w & 0x0F0F0F0Fu, hi4 = (w >> 4) & 0x0F0F0F0Fu;
        auto fpair = [](uint32_t nib4, uint32_t sel_lo, uint32_t sel_hi) {
            // 0x4B0000qq = 2^23 + q for the selected bytes
            return (uint64_t)__byte_perm(nib4, 0x4B000000u, sel_lo) |
                   ((uint64_t)__byte_perm(nib4, 0x4B000000u, sel_hi) << 32);
        };
        const uint64_t m23 = 0xCB000000CB000000ull;  // (-2^23, -2^23)
        const uint64_t dll = pack_f2(fdl_lo, fdl_lo), mll = pack_f2(fml_lo, fml_lo);
        const uint64_t dlh = pack_f2(fdl_hi, fdl_hi), mlh = pack_f2(fml_hi, fml_hi);
        lo01 = bf2_of(fma_f2(add_f2(fpair(lo4, 0x7440, 0x7441), m23), dll, mll));
        lo23 = bf2_of(fma_f2(add_f2(fpair(lo4, 0x7442, 0x7443), m23), dll, mll));
        hi01 = bf2_of(fma_f2(add_f2(fpair(hi4, 0x7440, 0x7441), m23), dlh, mlh));
        hi23 = bf2_of(fma_f2(add_f2(fpair(hi4, 0x7442, 0x7443), m23), dlh, mlh));
    }
}

// y element store in the requested output type
__device__ __forceinline__ void store_out(void* y, int ytype, int64_t idx, float v) {
    if (ytype == FTC_F32) reinterpret_cast<float*>(y)[idx] = v;
    else if (ytype == FTC_BF16) reinterpret_cast<__nv_bfloat16*>(y)[idx] = __float2bfloat16_rn(v);
    else reinterpret_cast<__half*>(y)[idx] = __float2half_rn(v);
}

template <class C, typename OP>
__global__ void __launch_bounds__(C::THREADS, 1)
gemm_q4k_tc(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_w2,
            const __grid_constant__ XMaps tm_x, int M, int N, int K, void* __restrict__ y,
            int ytype, const GemmGroups grp) {
    constexpr int BN = C::BN;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sA = smem + C::OFF_A;
    uint8_t* sB = smem + C::OFF_B;
    uint8_t* sRaw = smem + C::OFF_RAW;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
    uint64_t* a_full = bars;
    uint64_t* a_empty = a_full + C::NA;
    uint64_t* b_full = a_empty + C::NA;
    uint64_t* b_empty = b_full + C::NB;
    uint64_t* raw_full = b_empty + C::NB;
    uint64_t* raw_empty = raw_full + C::RAW;
    uint64_t* acc_full = raw_empty + C::RAW;
    uint64_t* acc_empty = acc_full + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + C::N_BARS);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    int* s_start = reinterpret_cast<int*>(smem + C::OFF_SCHED);  // [G + 1]
    int* s_base = s_start + kGemmMaxGroups + 1;                  // [G]
    int* s_cnt = s_base + kGemmMaxGroups;                        // [G]
    int* s_plan = s_cnt + kGemmMaxGroups;                        // [8] this CTA's schedule
    const int G = grp.G;
    const int n_tiles = (N + BM - 1) / BM;
    const int n_all = n_tiles * grp.n_sets;
    // Programmatic dependent launch: this grid may start while the preceding
    // kernel on the stream still runs.  Grouped launches read device counts
    // for their tile schedule, so every thread waits here; dense launches let
    // the raw-weight producer, the dequant and the MMA warps start at once and
    // wait only where the preceding kernel's outputs are read (activations)
    // or its inputs may still be read (Y, row scales, stream-K scratch).
    if (grp.counts) grid_dependency_wait();
    for (int g = threadIdx.x; g < G; g += blockDim.x) {
        const int base = grp.counts ? min(max(grp.offsets[g], 0), M) : 0;
        s_base[g] = base;
        s_cnt[g] = grp.counts ? min(max(grp.counts[g], 0), M - base) : M;
    }

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < C::NA; ++s) {
            mbar_init(&a_full[s], kTeamWarps);
            mbar_init(&a_empty[s], 1);
        }
        for (int s = 0; s < C::NB; ++s) {
            mbar_init(&b_full[s], 1);
            mbar_init(&b_empty[s], 1);
        }
        for (int s = 0; s < C::RAW; ++s) {
            mbar_init(&raw_full[s], 1);
            mbar_init(&raw_empty[s], kTeamWarps);
        }
        for (int s = 0; s < 2; ++s) {
            mbar_init(&acc_full[s], C::MI);
            mbar_init(&acc_empty[s], kEpiWarps);
        }
        *abort_flag = 0;
        mbar_fence_init();
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        int acc = 0;
        for (int g = 0; g < G; ++g) {
            s_start[g] = acc;
            acc += (s_cnt[g] + BN - 1) / BN * n_all;
        }
        s_start[G] = acc;
        // this CTA's share (one thread: the divisions, issued by every warp,
        // cost ~0.4 us of issue slots per launch)
        const int Gl = (int)gridDim.x, b = (int)blockIdx.x, nsb = K / 256;
        const TailPlan pl = plan_tail<BN>(acc, nsb, Gl, grp.part != nullptr);
        const int it0 = b < pl.Gc ? b * pl.W / pl.Gc : 0;
        const int it1 = b < pl.Gc ? (b + 1) * pl.W / pl.Gc : 0;
        const int n_whole = b < pl.t_full ? (pl.t_full - 1 - b) / Gl + 1 : 0;
        s_plan[0] = pl.t_full;
        s_plan[1] = pl.W;
        s_plan[2] = pl.Gc;
        s_plan[3] = n_whole;
        s_plan[4] = it0;
        s_plan[5] = it1;
        s_plan[6] = n_whole + (it1 > it0 ? (it1 - 1) / nsb - it0 / nsb + 1 : 0);
    }
    if (warp == 0) {
        tmem_alloc(tmem_slot, C::TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    grid_launch_dependents();  // the next kernel's prologue may overlap this grid

    const int nsb = K / 256;
    auto tile_at = [&](int tile) {
        return tile_ref<BN>(tile, s_start, s_base, s_cnt, G, n_tiles, n_all);
    };
    // Work schedule.  Whole tiles b, b + G, ... for every full wave of G
    // CTAs (consecutive CTAs on consecutive tiles, so a wave shares its
    // activation and weight tiles in L2); the tiles of the last, partial
    // wave (all of them when there are fewer tiles than CTAs) may be cut
    // (plan_tail): their W = tiles x nsb super-block steps split into one
    // equal contiguous range per CTA, [b*W/Gc, (b+1)*W/Gc) for the first Gc
    // CTAs, which meets tiles in segments (a tile and a super-block range).
    // A tile cut by range boundaries is finished by the last of its pieces
    // to arrive, adding the pieces' fp32 partials in range order.
    const int Gl = (int)gridDim.x;
    const int b_cta = (int)blockIdx.x;
    const int t_full = s_plan[0];   // tiles run whole, round robin
    const int W = s_plan[1];        // steps of the cut tail
    const int Gc = s_plan[2];       // CTAs sharing them
    const int n_whole = s_plan[3];  // this CTA's whole tiles
    const int it0 = s_plan[4], it1 = s_plan[5];  // its range of the tail (empty unless W)
    const int nseg = s_plan[6];
    // segment k of this CTA: its tile and super-block range [sb0, sb1)
    auto seg_at = [&](int k, int& sb0, int& sb1) -> int {
        if (k < n_whole) {
            sb0 = 0;
            sb1 = nsb;
            return b_cta + k * Gl;
        }
        const int t = it0 / nsb + (k - n_whole);
        const int t0 = t * nsb;
        sb0 = max(it0, t0) - t0;
        sb1 = min(it1, t0 + nsb) - t0;
        return t_full + t;
    };
    // the CTA whose stream-K range holds step q (W > 0)
    auto owner = [&](int q) { return ((q + 1) * Gc + W - 1) / W - 1; };

    if (warp == 0) {
        // ---------------------------------------------------------- TMA
        if (lane == 0) {
            for (int i = 0; i < kXMaps; ++i) prefetch_tensormap(&tm_x.m[i]);
            grid_dependency_wait();  // X may be the preceding kernel's output
            const uint64_t pol_x = policy_evict_last();
            uint32_t kc = 0;
            for (int k = 0; k < nseg && !*abort_flag; ++k) {
                int sb0, sb1;
                const TileRef t = tile_at(seg_at(k, sb0, sb1));
                int xb = 0;  // smallest box covering the tile's rows
                while (xb < kXMaps - 1 && xbox_rows(xb, BN) < t.rows) ++xb;
                const CUtensorMap* xm = &tm_x.m[xb];
                const uint32_t bytes = (uint32_t)xbox_rows(xb, BN) * BK * 2;
                for (int ks = sb0 * 4; ks < sb1 * 4; ++ks) {
                    const int s = kc % C::NB;
                    if (!mbar_wait(&b_empty[s], ((kc / C::NB) & 1) ^ 1, C::SLEEP_NS)) {
                        *abort_flag = 1;
                        break;
                    }
                    mbar_arrive_expect_tx(&b_full[s], bytes);
                    tma_load_2d(sB + s * C::B_BYTES, xm, ks * BK, t.row0, &b_full[s], pol_x);
                    ++kc;
                }
            }
            if (*abort_flag) {  // let issued copies land before the CTA leaves
                for (uint32_t j = kc > (uint32_t)C::NB ? kc - C::NB : 0; j < kc; ++j)
                    mbar_wait(&b_full[j % C::NB], (j / C::NB) & 1, C::SLEEP_NS);
            }
        }
    } else if (warp == C::RAW_WARP) {
        // ------------------------------------------------------ raw TMA
        // Raw weight tiles run up to kRawSlots super-blocks ahead of the
        // dequant warps, independent of the activation ring.
        if (lane == 0) {
            prefetch_tensormap(&tm_w);
            prefetch_tensormap(&tm_w2);
            const uint64_t pol_w = policy_evict_last();  // weights are re-read per token tile
            uint32_t rc = 0;
            for (int k = 0; k < nseg && !*abort_flag; ++k) {
                int sb0, sb1;
                const TileRef t = tile_at(seg_at(k, sb0, sb1));
                const CUtensorMap* wm = t.set ? &tm_w2 : &tm_w;
                for (int sb = sb0; sb < sb1; ++sb) {
                    const RingPos<C> rp(rc, 0);
                    if (!mbar_wait(&raw_empty[rp.raw_slot], rp.raw_phase ^ 1, C::SLEEP_NS)) {
                        *abort_flag = 1;
                        break;
                    }
                    mbar_arrive_expect_tx(&raw_full[rp.raw_slot], kRawBytes);
                    tma_load_3d(sRaw + rp.raw_slot * kRawBytes, wm, sb * 144, t.nt * BM, t.g,
                                &raw_full[rp.raw_slot], pol_w);
                    ++rc;
                }
            }
            if (*abort_flag) {  // let issued copies land before the CTA leaves
                for (uint32_t j = rc > (uint32_t)C::RAW ? rc - C::RAW : 0; j < rc; ++j) {
                    const RingPos<C> rp(j, 0);
                    mbar_wait(&raw_full[rp.raw_slot], rp.raw_phase, C::SLEEP_NS);
                }
            }
        }
    } else if (warp == 1 || (C::MI == 2 && warp == C::MMA2_WARP)) {
        // ---------------------------------------------------------- MMA
        // issuer j takes the k-steps ks of a unit with (ks - first) % MI == j
        const int j = warp == 1 ? 0 : 1;
        if (lane == 0) {
            constexpr uint32_t fmt = std::is_same<OP, __half>::value ? 0u : 1u;
            uint32_t kc = 0, last_kc = 0;
            bool any = false;
            int i = 0;
            for (int k = 0; k < nseg && !*abort_flag; ++k, ++i) {
                const int b = i & 1;
                int sb0, sb1;
                const int tile = seg_at(k, sb0, sb1);
                // MMA N = the tile's tokens rounded up to 16
                const uint32_t idesc = idesc_f16(fmt, BM, (uint32_t)min(BN, (tile_at(tile).rows + 15) & ~15));
                if (!mbar_wait(&acc_empty[b], ((i >> 1) & 1) ^ 1, C::SLEEP_NS)) {
                    *abort_flag = 1;
                    break;
                }
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + (uint32_t)((b * C::MI + j) * BN);
                bool acc = false;  // the issuer's first k-step of the unit overwrites
                for (int ks = sb0 * 4; ks < sb1 * 4; ++ks, ++kc) {
                    if (C::MI == 2 && ((ks - sb0 * 4) & 1) != j) continue;
                    const RingPos<C> rp(kc >> 2, (int)(kc & 3));
                    const int sa = rp.a_stage, s = kc % C::NB;
                    if (!mbar_wait(&a_full[sa], rp.a_phase, C::SLEEP_NS) ||
                        !mbar_wait(&b_full[s], (kc / C::NB) & 1, C::SLEEP_NS)) {
                        *abort_flag = 1;
                        break;
                    }
                    tc_fence_after();
                    const uint64_t db = smem_desc_k_sw128(sB + s * C::B_BYTES);
                    if constexpr (C::ATM) {
                        const uint32_t a_tmem = tmem_base + (uint32_t)(C::A_COL0 + sa * C::A_COLS);
#pragma unroll
                        for (int kk = 0; kk < BK / 16; ++kk)  // 8 columns (16 k) per MMA
                            umma_f16_ts(d_tmem, a_tmem + 8 * kk, db + 2 * kk, idesc, acc || kk != 0);
                    } else {
                        const uint64_t da = smem_desc_k_sw128(sA + sa * C::A_BYTES);
#pragma unroll
                        for (int kk = 0; kk < BK / 16; ++kk)  // +32 bytes along k per MMA
                            umma_f16_ss(d_tmem, da + 2 * kk, db + 2 * kk, idesc, acc || kk != 0);
                    }
                    umma_commit(&a_empty[sa]);
                    umma_commit(&b_empty[s]);
                    acc = true;
                    any = true;
                    last_kc = kc;
                }
                if (*abort_flag) break;
                umma_commit(&acc_full[b]);
            }
            // wait for this issuer's last MMAs to retire before TMEM can be released
            if (any) mbar_wait(&b_empty[last_kc % C::NB], (last_kc / C::NB) & 1, C::SLEEP_NS);
        }
    } else if (warp < 2 + kEpiWarps) {
        // ---------------------------------------------------------- epilogue
        // A cut tile (stream-K): every piece stores its fp32 partial (this
        // warp's 32 columns of the tile); the warp whose arrival completes the
        // tile's count sums all partials in range order, so the result does
        // not depend on which piece finished last.  Each warp counts on its
        // own (no barrier between the epilogue warps).
        const int q = warp & 3;  // TMEM lane quadrant this warp may access
        const int nl = 32 * q + lane;  // column of the tile this lane holds
        grid_dependency_wait();  // Y, row scales and stream-K scratch of earlier kernels
        int i = 0;
        for (int k = 0; k < nseg; ++k, ++i) {
            const int b = i & 1;
            int sb0, sb1;
            const int tile = seg_at(k, sb0, sb1);
            const TileRef t = tile_at(tile);
            if (!mbar_wait_warp(&acc_full[b], (i >> 1) & 1, C::SLEEP_NS)) {
                *abort_flag = 1;
                break;
            }
            tc_fence_after();
            const int n = t.nt * BM + nl;
            const int64_t col = (int64_t)t.set * N + n;
            const uint32_t taddr = tmem_base + ((uint32_t)(32 * q) << 16) + (uint32_t)(b * C::MI * BN);
            // the tile's accumulator: issuer 0's plus (MI == 2) issuer 1's, in that order
            auto load_acc = [&](int c0, uint32_t (&r)[32]) {
                tmem_ld_32x32b_x32(taddr + c0, r);
                if constexpr (C::MI == 2) {
                    uint32_t r2[32];
                    tmem_ld_32x32b_x32(taddr + BN + c0, r2);
                    tmem_ld_wait();
#pragma unroll
                    for (int jj = 0; jj < 32; ++jj)
                        r[jj] = __float_as_uint(__uint_as_float(r[jj]) + __uint_as_float(r2[jj]));
                } else {
                    tmem_ld_wait();
                }
            };
            bool last = true;
            if (sb0 != 0 || sb1 != nsb) {
                // a piece of a tile cut by range boundaries: pieces come from
                // CTAs first .. last_cta in range order; CTA c keeps the piece of
                // its first tile in partial slot 2c and of its last tile in
                // 2c + 1 ([quadrant][row][32 columns] fp32 each); the tile's
                // arrival count sits in row `first` of the counters (no other
                // cut tile has its first piece in CTA `first`)
                const int ts = tile - t_full;  // the tile in the stream-K range
                const int first = owner(ts * nsb);
                const int npieces = owner(ts * nsb + nsb - 1) - first + 1;
                float* mine = grp.part + (size_t)(2 * b_cta + (k == n_whole ? 0 : 1)) * (BM * BN) +
                              q * (BN * 32) + lane;
#pragma unroll 1
                for (int c0 = 0; c0 < t.rows; c0 += 32) {
                    uint32_t r[32];
                    load_acc(c0, r);
                    const int jn = min(32, t.rows - c0);
#pragma unroll
                    for (int j = 0; j < 32; ++j)
                        if (j < jn) __stcg(mine + (c0 + j) * 32, __uint_as_float(r[j]));
                }
                __threadfence();
                __syncwarp();
                uint32_t old = 0;
                uint32_t* cnt = grp.counters + first * kEpiWarps + q;
                if (lane == 0) old = atomicAdd(cnt, 1u);
                old = __shfl_sync(0xffffffffu, old, 0);
                last = old == (uint32_t)(npieces - 1);
                if (last) {
                    if (lane == 0) atomicExch(cnt, 0u);  // ready for the next launch
                    __threadfence();
                    // Sum the pieces' partials of this quadrant in range
                    // order.  A lane takes 4 columns (c4..c4+3) of rows
                    // 4g + rr; loads go out 16 at a time (4 pieces x 4 row
                    // groups) so the fix-up costs one L2 round trip per 16
                    // rows and 4 pieces.
                    const int rr = lane >> 3, c4 = 4 * (lane & 7);
                    // partial slot of piece p (CTA first + p): the tile is the
                    // first tile of every later piece's CTA (slot 2c) and the
                    // last tile of CTA `first` unless its range starts here
                    const int e0 = first * W / Gc != ts * nsb ? 1 : 0;
                    auto piece_slot = [&](int p) {
                        return (size_t)(2 * (first + p) + (p == 0 ? e0 : 0));
                    };
                    const float* qb = grp.part + q * (BN * 32) + c4;
                    const int nq = t.nt * BM + 32 * q + c4;  // first of the lane's 4 columns
                    const int64_t cq = (int64_t)t.set * N + nq;
#pragma unroll 1
                    for (int rb = 0; rb < t.rows; rb += 16) {
                        float4 acc[4];
#pragma unroll 1
                        for (int s0 = 0; s0 < npieces; s0 += 4) {
                            float4 v[4][4];
#pragma unroll
                            for (int u2 = 0; u2 < 4; ++u2)
#pragma unroll
                                for (int g = 0; g < 4; ++g) {
                                    const int row = rb + 4 * g + rr;
                                    v[u2][g] = (s0 + u2 < npieces && row < t.rows)
                                                   ? __ldcg(reinterpret_cast<const float4*>(
                                                         qb + piece_slot(s0 + u2) * (BM * BN) +
                                                         row * 32))
                                                   : make_float4(0.f, 0.f, 0.f, 0.f);
                                }
#pragma unroll
                            for (int u2 = 0; u2 < 4; ++u2) {
                                if (s0 + u2 >= npieces) break;
#pragma unroll
                                for (int g = 0; g < 4; ++g) {
                                    if (s0 + u2 == 0) {
                                        acc[g] = v[u2][g];
                                    } else {
                                        acc[g].x += v[u2][g].x;
                                        acc[g].y += v[u2][g].y;
                                        acc[g].z += v[u2][g].z;
                                        acc[g].w += v[u2][g].w;
                                    }
                                }
                            }
                        }
#pragma unroll
                        for (int g = 0; g < 4; ++g) {
                            const int row = rb + 4 * g + rr;
                            if (row >= t.rows) continue;
                            float f = 1.f;
                            if (grp.row_exp)
                                f = __uint_as_float((uint32_t)(grp.row_exp[t.row0 + row] + 127) << 23);
                            const int64_t yi = (int64_t)(t.row0 + row) * grp.ldy + cq;
                            const float o[4] = {acc[g].x * f, acc[g].y * f, acc[g].z * f, acc[g].w * f};
#pragma unroll
                            for (int e = 0; e < 4; ++e)
                                if (nq + e < N) store_out(y, ytype, yi + e, o[e]);
                        }
                    }
                }
            } else {
#pragma unroll 1
                for (int c0 = 0; c0 < t.rows; c0 += 32) {
                    uint32_t r[32];
                    load_acc(c0, r);
                    const int64_t y0 = (int64_t)(t.row0 + c0) * grp.ldy + col;
                    const int jn = min(32, t.rows - c0);
                    if (grp.row_exp) {  // exact power-of-two row scales (warp-uniform branch)
                        float f = 0.f;
                        if (lane < jn) f = __uint_as_float((uint32_t)(grp.row_exp[t.row0 + c0 + lane] + 127) << 23);
#pragma unroll
                        for (int j = 0; j < 32; ++j)
                            r[j] = __float_as_uint(__uint_as_float(r[j]) * __shfl_sync(0xffffffffu, f, j));
                    }
                    if (n < N) {
#pragma unroll
                        for (int j = 0; j < 32; ++j)
                            if (j < jn) store_out(y, ytype, y0 + (int64_t)j * grp.ldy, __uint_as_float(r[j]));
                    }
                }
            }
            (void)last;
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acc_empty[b]);
            if (*abort_flag) break;
        }
    } else {
        // ---------------------------------------------------------- dequant
        const int dw = warp - (2 + kEpiWarps);
        const int team = dw / kTeamWarps;
        // shared-memory stages: a warp covers rows 16*wi .. 16*wi + 15, both
        // halves of the group; a quarter-warp takes 8 consecutive rows of one
        // half, so its 16-byte stores hit 8 different swizzled chunks (all 32
        // banks) and its raw loads (rows 144 bytes apart) 8 different bank
        // quads.  Tensor-memory stages: a warp may only write the 32 TMEM
        // lanes of its quadrant (warp % 4), so it takes those 32 rows (lane =
        // row) and one half of the group (the other warp of the quadrant the
        // other half).
        const int wi = dw % kTeamWarps;
        const int h = C::ATM ? wi / 4 : (lane >> 3) & 1;           // half of the group
        const int r = C::ATM ? 32 * (warp & 3) + lane
                             : 16 * wi + 8 * (lane >> 4) + (lane & 7);  // weight row in tile
        const int swz = r & 7;
        uint32_t rc = 0;  // super-blocks in kernel order; this team takes rc % DT == team
        for (int k = 0; k < nseg; ++k) {
            int sb0, sb1;
            seg_at(k, sb0, sb1);
            for (int sb = sb0; sb < sb1; ++sb, ++rc) {
                if ((int)(rc % C::DT) != team) continue;
                const RingPos<C> rp0(rc, 0);
                const int rs = rp0.raw_slot;
                if (!mbar_wait_warp(&raw_full[rs], rp0.raw_phase, C::SLEEP_NS)) {
                    *abort_flag = 1;
                    break;
                }
                const uint8_t* blk = sRaw + rs * kRawBytes + r * 144;
                float fdl[8], fnml[8];      // per sub-block: d*sc, -dmin*m
                uint32_t dl2[8], nml2[8];   // the same as fp16 pairs (fp16 operands)
                decode_scales<OP>(*reinterpret_cast<const uint4*>(blk), fdl, fnml, dl2, nml2);
#pragma unroll
                for (int g = 0; g < 4; ++g) {
                    const RingPos<C> rp(rc, g);
                    const int s = rp.a_stage;
                    if (!mbar_wait_warp(&a_empty[s], rp.a_phase ^ 1, C::SLEEP_NS)) {
                        *abort_flag = 1;
                        break;
                    }
                    if constexpr (C::ATM) tc_fence_after();  // the MMA that read the stage is done
                    const uint4 qv = *reinterpret_cast<const uint4*>(blk + 16 + 32 * g + 16 * h);
                    const uint32_t w[4] = {qv.x, qv.y, qv.z, qv.w};
                    uint32_t lo[8], hi[8];  // packed pairs, k = 16h + 2i (+32 for hi)
#pragma unroll
                    for (int u = 0; u < 4; ++u) {
                        dequant_pairs<OP>(w[u], dl2[2 * g], nml2[2 * g], dl2[2 * g + 1],
                                          nml2[2 * g + 1], fdl[2 * g], fnml[2 * g],
                                          fdl[2 * g + 1], fnml[2 * g + 1], lo[2 * u],
                                          lo[2 * u + 1], hi[2 * u], hi[2 * u + 1]);
                    }
                    if constexpr (C::ATM) {
                        // columns (two k each): low nibbles k = 16h + 2i -> 8h + i,
                        // high nibbles k = 32 + 16h + 2i -> 16 + 8h + i
                        const uint32_t tcol = tmem_base + ((uint32_t)(32 * (warp & 3)) << 16) +
                                              (uint32_t)(C::A_COL0 + s * C::A_COLS);
                        tmem_st_32x32b_x8(tcol + 8 * h, lo);
                        tmem_st_32x32b_x8(tcol + 16 + 8 * h, hi);
                        tmem_st_wait();
                        tc_fence_before();
                        __syncwarp();
                        if (lane == 0) mbar_arrive(&a_full[s]);
                        continue;
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
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&raw_empty[rs]);
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

template <class C, typename OP>
int launch(const CUtensorMap& tw, const CUtensorMap& tw2, const XMaps& tx, int M, int N, int K,
           void* y, int ytype, const GemmGroups& grp, int64_t max_units, int sms,
           cudaStream_t st) {
    const int rc = opt_in_smem(reinterpret_cast<const void*>(gemm_q4k_tc<C, OP>), C::SMEM,
                               "cudaFuncSetAttribute(gemm_q4k_tc)");
    if (rc) return rc;
    const int grid = (int)std::max<int64_t>(1, std::min<int64_t>(max_units, sms));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(C::THREADS);
    cfg.dynamicSmemBytes = C::SMEM;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t e =
        cudaLaunchKernelEx(&cfg, gemm_q4k_tc<C, OP>, tw, tw2, tx, M, N, K, y, ytype, grp);
    if (e != cudaSuccess) return cuda_error(e, "launch gemm_q4k_tc");
    return FTC_OK;
}

// W: G planes of N rows of Q4_K blocks, plane g at w + g * plane_stride.
int weight_map(CUtensorMap* m, const void* w, int64_t N, int64_t K, int64_t row_stride, int64_t G,
               int64_t plane_stride, const char* who) {
    auto enc = encode_fn();
    FTC_REQUIRE(enc, FTC_E_CUDA, std::string(who) + ": cuTensorMapEncodeTiled unavailable");
    const cuuint64_t dims[3] = {(cuuint64_t)((K / 256) * 144), (cuuint64_t)N, (cuuint64_t)G};
    const cuuint64_t strides[2] = {(cuuint64_t)row_stride, (cuuint64_t)plane_stride};
    const cuuint32_t box[3] = {144, BM, 1};
    const cuuint32_t es[3] = {1, 1, 1};
    CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(w), dims, strides, box,
                     es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    FTC_REQUIRE(r == CUDA_SUCCESS, FTC_E_CUDA, std::string(who) + ": weight tensor map rejected");
    return FTC_OK;
}

// X: rows x K 16-bit activations; one map per box height 32, 64, ... BN.
int act_maps(XMaps* mx, const void* x, int x_dtype, int64_t rows, int64_t K, int BN,
             const char* who) {
    auto enc = encode_fn();
    FTC_REQUIRE(enc, FTC_E_CUDA, std::string(who) + ": cuTensorMapEncodeTiled unavailable");
    std::memset(mx, 0, sizeof(*mx));
    for (int i = 0; i < kXMaps; ++i) {
        const cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
        const cuuint64_t strides[1] = {(cuuint64_t)(K * 2)};
        const cuuint32_t box[2] = {BK, (cuuint32_t)xbox_rows(i, BN)};
        const cuuint32_t es[2] = {1, 1};
        CUresult r = enc(&mx->m[i],
                         x_dtype == FTC_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                             : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                         2, const_cast<void*>(x), dims, strides, box, es,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        FTC_REQUIRE(r == CUDA_SUCCESS, FTC_E_CUDA,
                    std::string(who) + ": activation tensor map rejected");
    }
    return FTC_OK;
}

// ------------------------------------------------------------- stream-K

// Scratch of the stream-K schedule: two partial slots (a CTA's first and
// last tile) and one row of arrival counters per CTA, one CTA per SM.
constexpr int kSlotsPerSm = 2;

struct SplitScratch {
    int units = 0;  // capacity in partial slots (0: none)
    uint32_t* counters = nullptr;
    float* part = nullptr;
};

std::mutex g_split_mu;
SplitScratch g_split[64];  // per device

// The device's stream-K scratch, allocated on first use (never freed, never
// moved: graphs that captured its address stay valid).  Inside a stream
// capture nothing can be allocated; *out stays empty and the caller runs
// whole tiles.
int split_scratch(cudaStream_t st, int sms, SplitScratch* out) {
    int dev = 0;
    FTC_CUDA(cudaGetDevice(&dev));
    FTC_REQUIRE(dev >= 0 && dev < 64, FTC_E_CUDA, "gemm stream-K: device index out of range");
    std::lock_guard<std::mutex> lk(g_split_mu);
    SplitScratch& sc = g_split[dev];
    if (!sc.units) {
        cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
        FTC_CUDA(cudaStreamIsCapturing(st, &cs));
        if (cs != cudaStreamCaptureStatusNone) {
            *out = SplitScratch{};
            return FTC_OK;
        }
        const int units = kSlotsPerSm * sms;
        const size_t cnt_bytes = ((size_t)units * kEpiWarps * 4 + 255) & ~size_t(255);
        const size_t part_bytes = (size_t)units * BM * 256 * 4;
        void* p = nullptr;
        FTC_CUDA(cudaMalloc(&p, cnt_bytes + part_bytes));
        const cudaError_t e = cudaMemset(p, 0, cnt_bytes);
        if (e != cudaSuccess) {
            cudaFree(p);
            return cuda_error(e, "cudaMemset(gemm stream-K counters)");
        }
        sc.counters = static_cast<uint32_t*>(p);
        sc.part = reinterpret_cast<float*>(static_cast<uint8_t*>(p) + cnt_bytes);
        sc.units = units;
    }
    *out = sc;
    return FTC_OK;
}

int dispatch(int BN, int x_dtype, const CUtensorMap& tw, const CUtensorMap& tw2, const XMaps& tx,
             int M, int N, int K, void* y, int y_dtype, GemmGroups grp, int64_t max_tiles,
             int tile_rows, cudaStream_t st) {
    const bool bf = x_dtype == FTC_BF16;
    const int sms = device_sms();
    (void)tile_rows;
    // stream-K over all SMs when the scratch exists (two partial slots and
    // one counter row per CTA); otherwise whole tiles, one CTA per tile
    grp.counters = nullptr;
    grp.part = nullptr;
    SplitScratch sc;
    const int src = split_scratch(st, sms, &sc);
    if (src != FTC_OK) return src;
    if (sc.units >= 2 * sms) {
        grp.counters = sc.counters;
        grp.part = sc.part;
    }
    if (max_tiles * (K / 256) > INT32_MAX) grp.counters = nullptr, grp.part = nullptr;
    // launch size: with the tile count known on the host (no device-side
    // groups) and under one wave, the CTAs the kernel's plan gives work to
    // (the kernel recomputes it for that grid); otherwise every SM (grouped
    // counts are only known on the device)
    int64_t units = grp.part ? max_tiles * (K / 256) : max_tiles;
    if (!grp.counts && max_tiles < sms) {
        const int t = (int)max_tiles, nsb = K / 256;
        const bool scr = grp.part != nullptr;
        const TailPlan pl = BN == 64    ? plan_tail<64>(t, nsb, sms, scr)
                            : BN == 128 ? plan_tail<128>(t, nsb, sms, scr)
                                        : plan_tail<256>(t, nsb, sms, scr);
        units = std::max(pl.t_full, pl.Gc);
    }
    // up to 64 tokens: two MMA issuers (their accumulators and the A stages
    // all in tensor memory); up to 128: A stages in tensor memory (no
    // shared-memory A stores or A reads by the MMA); larger: the 256-token
    // tile, which halves the weight traffic per FLOP and needs all 512 TMEM
    // columns for its two accumulators.  On that tile a fourth dequantized
    // stage in place of a third raw slot (two raw slots still hold 8 k-steps
    // of lookahead) was 1.5-2 % faster at M = 2048 and 8192.
    using C64 = Cfg<64, 1, 8, 6, 6, true, 2>;
    using C128 = Cfg<128, 1, 4, 5, 3, true>;
    using C256 = Cfg<256, 1, 4, 3, 2>;
    int rc;
    if (BN == 64)
        rc = bf ? launch<C64, __nv_bfloat16>(tw, tw2, tx, M, N, K, y, y_dtype, grp, units, sms, st)
                : launch<C64, __half>(tw, tw2, tx, M, N, K, y, y_dtype, grp, units, sms, st);
    else if (BN == 128)
        rc = bf ? launch<C128, __nv_bfloat16>(tw, tw2, tx, M, N, K, y, y_dtype, grp, units, sms, st)
                : launch<C128, __half>(tw, tw2, tx, M, N, K, y, y_dtype, grp, units, sms, st);
    else
        rc = bf ? launch<C256, __nv_bfloat16>(tw, tw2, tx, M, N, K, y, y_dtype, grp, units, sms, st)
                : launch<C256, __half>(tw, tw2, tx, M, N, K, y, y_dtype, grp, units, sms, st);
    if (rc != FTC_OK) return rc;
    FTC_CUDA(cudaGetLastError());
    return FTC_OK;
}

}  // namespace

// Status reader of this file's kernels.  Clearing a recorded timeout also
// zeroes the stream-K arrival counters, which a launch that gave up part way
// may have left uneven.
int devstat_gemm_q4k(int clear) {
    int v = 0;
    if (cudaMemcpyFromSymbol(&v, g_dev_status, sizeof(int)) != cudaSuccess) return -1;
    if (clear && v) {
        const int z = 0;
        if (cudaMemcpyToSymbol(g_dev_status, &z, sizeof(int)) != cudaSuccess) return -1;
        int dev = 0;
        if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return -1;
        std::lock_guard<std::mutex> lk(g_split_mu);
        const SplitScratch& sc = g_split[dev];
        if (sc.units && cudaMemset(sc.counters, 0, (size_t)sc.units * kEpiWarps * 4) != cudaSuccess)
            return -1;
    }
    return v;
}

namespace {

int check_types(int x_dtype, int y_dtype, const char* who) {
    FTC_REQUIRE(x_dtype == FTC_BF16 || x_dtype == FTC_F16, FTC_E_UNSUPPORTED,
                std::string(who) + ": activations must be bf16 or fp16");
    FTC_REQUIRE(y_dtype == FTC_BF16 || y_dtype == FTC_F16 || y_dtype == FTC_F32, FTC_E_UNSUPPORTED,
                std::string(who) + ": output must be bf16, fp16 or fp32");
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
    int rc = check_types(x_dtype, y_dtype, "ftc_gemm");
    if (rc) return rc;
    FTC_REQUIRE(row_stride >= (K / 256) * 144 && row_stride % 16 == 0 && (uintptr_t)w % 16 == 0,
                FTC_E_INVALID, "ftc_gemm: weight rows must be 16-byte aligned");
    FTC_REQUIRE((uintptr_t)x % 16 == 0, FTC_E_INVALID, "ftc_gemm: activations must be 16-byte aligned");
    const int BN = M <= 64 ? 64 : M <= 128 ? 128 : 256;
    CUtensorMap tw;
    XMaps tx;
    if ((rc = weight_map(&tw, w, N, K, row_stride, 1, N * row_stride, "ftc_gemm"))) return rc;
    if ((rc = act_maps(&tx, x, x_dtype, M, K, BN, "ftc_gemm"))) return rc;
    if (inject_fail("ftc_gemm")) return set_error(FTC_E_INJECTED, "ftc_gemm: injected failure");
    const GemmGroups grp = {nullptr, nullptr, 1, 1, N, nullptr, nullptr, nullptr};
    const int64_t tiles = ((N + BM - 1) / BM) * ((M + BN - 1) / BN);
    return dispatch(BN, x_dtype, tw, tw, tx, (int)M, (int)N, (int)K, y, y_dtype, grp, tiles,
                    (int)std::min<int64_t>(M, BN), st);
}

// Dense GEMM on fp16 rows scaled by 2^-row_exp (ftc_rows_to_f16), output
// rows scaled back by 2^row_exp.
int gemm_q4k_rowscaled(const void* w, int64_t N, int64_t K, int64_t row_stride, const void* x16,
                       int64_t M, void* y, int y_dtype, const int32_t* row_exp, cudaStream_t st) {
    FTC_REQUIRE(w && x16 && y && row_exp, FTC_E_INVALID, "ftc_gemm_rowscaled: null pointer");
    FTC_REQUIRE(M > 0 && N > 0 && K > 0 && K % 256 == 0, FTC_E_INVALID,
                "ftc_gemm_rowscaled: bad shape (K must be a multiple of 256)");
    FTC_REQUIRE(M <= INT32_MAX && N <= INT32_MAX && K <= INT32_MAX, FTC_E_INVALID,
                "ftc_gemm_rowscaled: shape too large");
    int rc = check_types(FTC_F16, y_dtype, "ftc_gemm_rowscaled");
    if (rc) return rc;
    FTC_REQUIRE(row_stride >= (K / 256) * 144 && row_stride % 16 == 0 && (uintptr_t)w % 16 == 0 &&
                    (uintptr_t)x16 % 16 == 0,
                FTC_E_INVALID, "ftc_gemm_rowscaled: operands must be 16-byte aligned");
    const int BN = M <= 64 ? 64 : M <= 128 ? 128 : 256;
    CUtensorMap tw;
    XMaps tx;
    if ((rc = weight_map(&tw, w, N, K, row_stride, 1, N * row_stride, "ftc_gemm_rowscaled")))
        return rc;
    if ((rc = act_maps(&tx, x16, FTC_F16, M, K, BN, "ftc_gemm_rowscaled"))) return rc;
    const GemmGroups grp = {nullptr, nullptr, 1, 1, N, row_exp, nullptr, nullptr};
    const int64_t tiles = ((N + BM - 1) / BM) * ((M + BN - 1) / BN);
    return dispatch(BN, FTC_F16, tw, tw, tx, (int)M, (int)N, (int)K, y, y_dtype, grp, tiles,
                    (int)std::min<int64_t>(M, BN), st);
}

// Grouped form: rows of x are grouped by expert (device counts / offsets);
// w (and w2 when n_sets == 2) hold G planes of N rows.  max_rows_per_group
// bounds every count (it picks the token tile).
int gemm_q4k_grouped(const void* w, const void* w2, int n_sets, int64_t G, int64_t plane_stride,
                     int64_t N, int64_t K, int64_t row_stride, const void* x, int x_dtype,
                     int64_t rows, const int32_t* counts, const int32_t* offsets,
                     int64_t max_rows_per_group, void* y, int y_dtype, int64_t ldy,
                     cudaStream_t st, const int32_t* row_exp) {
    FTC_REQUIRE(w && x && y && counts && offsets && (n_sets == 1 || w2), FTC_E_INVALID,
                "gemm_q4k_grouped: null pointer");
    FTC_REQUIRE(n_sets == 1 || n_sets == 2, FTC_E_INVALID, "gemm_q4k_grouped: 1 or 2 weight sets");
    FTC_REQUIRE(G >= 1 && G <= kGemmMaxGroups, FTC_E_INVALID, "gemm_q4k_grouped: 1..256 groups");
    FTC_REQUIRE(rows > 0 && N > 0 && K > 0 && K % 256 == 0, FTC_E_INVALID,
                "gemm_q4k_grouped: bad shape");
    FTC_REQUIRE(rows <= INT32_MAX && N <= INT32_MAX && K <= INT32_MAX, FTC_E_INVALID,
                "gemm_q4k_grouped: shape too large");
    int rc = check_types(x_dtype, y_dtype, "gemm_q4k_grouped");
    if (rc) return rc;
    FTC_REQUIRE(row_stride >= (K / 256) * 144 && row_stride % 16 == 0 && plane_stride % 16 == 0 &&
                    plane_stride >= N * row_stride && (uintptr_t)w % 16 == 0 &&
                    (uintptr_t)w2 % 16 == 0,
                FTC_E_INVALID, "gemm_q4k_grouped: weight rows and planes must be 16-byte aligned");
    FTC_REQUIRE((uintptr_t)x % 16 == 0, FTC_E_INVALID,
                "gemm_q4k_grouped: activations must be 16-byte aligned");
    FTC_REQUIRE(ldy >= n_sets * N, FTC_E_INVALID, "gemm_q4k_grouped: output pitch too small");
    const int BN = max_rows_per_group <= 64 ? 64 : max_rows_per_group <= 128 ? 128 : 256;
    CUtensorMap tw, tw2;
    XMaps tx;
    if ((rc = weight_map(&tw, w, N, K, row_stride, G, plane_stride, "gemm_q4k_grouped"))) return rc;
    if (n_sets == 2 &&
        (rc = weight_map(&tw2, w2, N, K, row_stride, G, plane_stride, "gemm_q4k_grouped")))
        return rc;
    if ((rc = act_maps(&tx, x, x_dtype, rows, K, BN, "gemm_q4k_grouped"))) return rc;
    const GemmGroups grp = {counts, offsets, (int)G, n_sets, ldy, row_exp, nullptr, nullptr};
    // upper bound on tiles: every non-empty group adds at most one partial token tile
    const int64_t tok_tiles = (rows + BN - 1) / BN + std::min<int64_t>(G, rows);
    const int64_t tiles = tok_tiles * ((N + BM - 1) / BM) * n_sets;
    return dispatch(BN, x_dtype, tw, n_sets == 2 ? tw2 : tw, tx, (int)rows, (int)N, (int)K, y,
                    y_dtype, grp, tiles, (int)std::min<int64_t>(max_rows_per_group, BN), st);
}

}  // namespace ftc
