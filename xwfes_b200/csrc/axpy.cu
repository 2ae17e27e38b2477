// axpy.cu -- the engine's down projection in the reference's transposed
// layout, ft::matmul_down_axpy (ft/src/cpu_backend.cpp:60-75, called for the
// dense FFN and the shared expert at ft/src/engine.cpp:256, 275):
//
//   y[m][j] += sum_i x[m][i] * W_i[j]      i < n_in, j < N
//
// W_i is row i of the weight: N weights in GGUF blocks along j, rows
// row_stride bytes apart (the neuron-major "down" the reference's files
// carry; standard GGUF down projections go through the GEMV/GEMM instead).
// A row with x[m][i] == 0 adds nothing, as in the reference.
//
// Work split: a CTA owns a column tile (8 consecutive weights per thread, so
// a warp covers 256 columns = one K-quant super-block of every row it
// reads) and a slab of consecutive rows, and walks the slab's rows in order
// with its tokens' activations in shared memory; every weight byte is read
// once per 8 tokens.  Each slab's fp32 sums go to a scratch plane and a
// second kernel adds the planes into y in slab order, so the result does not
// depend on scheduling.  With one slab the first kernel adds into y itself.
#include <algorithm>

#include "common.cuh"

namespace ftc {
namespace {

constexpr int kAxpyThreads = 256;  // threads per CTA at most (8 columns each)
constexpr int kAxpyMT = 8;         // tokens per CTA at most (1, 2, 4 or 8)
constexpr int kAxpyMaxRows = 512;  // rows per slab (activations staged in shared memory)
// rows whose bytes are in flight per thread: 8 for 1-2 tokens (a warp then
// has 8 x 144 B of one Q4_K column of blocks outstanding, ~28 KB per SM at 3
// CTAs per SM), 4 when 4-8 tokens per byte make the kernel less
// latency-bound and the sums need the registers
template <int MT>
__host__ __device__ constexpr int axpy_unroll() { return MT <= 2 ? 8 : 4; }
// 3 CTAs per SM: what the one-token Q4_K kernel (79 registers x 256 threads)
// keeps resident, so its grid is a single wave
constexpr int kAxpyTargetCtas = 3 * 148;

enum { kGeneric = -1 };  // element-by-element decoder (any format, any alignment)

struct AxpyArgs {
    const uint8_t* w;
    int64_t stride;
    int64_t n_in;
    int64_t N;
    int dtype;
    const float* x;
    int64_t M;
    int rows;     // rows per slab
    float* part;  // [slabs][M][N] slab sums, or null: add into y directly
    float* y;
};

__device__ __forceinline__ uint32_t ld16(const uint8_t* p) {
    return __ldg(reinterpret_cast<const unsigned short*>(p));
}

// ---------------------------------------------------------------- raw bytes
// Weights j0 .. j0+7 of one row (j0 a multiple of 8, inside the row): the
// bytes each format needs, loaded before any of them is decoded so that
// several rows' loads are in flight together.

struct RawQ4K {
    uint32_t hd, s0, s1, s2;  // d | dmin << 16, the 12 scale bytes
    uint2 q;                  // 8 code bytes (low or high nibbles)
};

// Block start 16-byte aligned (checked on the host).
__device__ __forceinline__ RawQ4K load_q4k(const uint8_t* row, int64_t j0) {
    const uint8_t* b = row + (j0 >> 8) * 144;
    const int i = (int)(j0 & 255);
    const uint4 h = __ldg(reinterpret_cast<const uint4*>(b));
    RawQ4K r;
    r.hd = h.x;
    r.s0 = h.y;
    r.s1 = h.z;
    r.s2 = h.w;
    r.q = __ldg(reinterpret_cast<const uint2*>(b + 16 + 32 * (i >> 6) + (i & 31)));
    return r;
}

// Same arithmetic as decode_elem's Q4_K case: (d*sc)*q - dmin*mn.
__device__ __forceinline__ void dec_q4k(const RawQ4K& r, int64_t j0, float w[8]) {
    const int i = (int)(j0 & 255);
    const int g = i >> 6, hi = (i >> 5) & 1;
    int sc, mn;
    q4k_scale_min(r.s0, r.s1, r.s2, 2 * g + hi, sc, mn);
    const float dl = h2f(r.hd) * (float)sc;
    const float ml = h2f(r.hd >> 16) * (float)mn;
    const int sh = 4 * hi;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
        w[c] = __fsub_rn(__fmul_rn(dl, (float)((r.q.x >> (8 * c + sh)) & 0xF)), ml);
        w[4 + c] = __fsub_rn(__fmul_rn(dl, (float)((r.q.y >> (8 * c + sh)) & 0xF)), ml);
    }
}

struct RawQ6K {
    uint32_t ql0, ql1, qh0, qh1;  // 8 low-bit bytes, 8 high-bit bytes
    uint32_t d;                   // fp16 bits
    int sc;
};

// 210-byte blocks: only 2-byte alignment (checked on the host).
__device__ __forceinline__ RawQ6K load_q6k(const uint8_t* row, int64_t j0) {
    const uint8_t* b = row + (j0 >> 8) * 210;
    const int i = (int)(j0 & 255);
    const int half = i >> 7, r = i & 127, quad = r >> 5, l0 = r & 31;
    const uint8_t* ql = b + 64 * half + l0 + ((quad & 1) ? 32 : 0);
    const uint8_t* qh = b + 128 + 32 * half + l0;
    RawQ6K o;
    o.ql0 = ld16(ql) | (ld16(ql + 2) << 16);
    o.ql1 = ld16(ql + 4) | (ld16(ql + 6) << 16);
    o.qh0 = ld16(qh) | (ld16(qh + 2) << 16);
    o.qh1 = ld16(qh + 4) | (ld16(qh + 6) << 16);
    o.d = ld16(b + 208);
    o.sc = (int)(int8_t)__ldg(b + 192 + 8 * half + (l0 >> 4) + 2 * quad);
    return o;
}

// Same arithmetic as decode_elem's Q6_K case: (d*sc) * (q - 32).
__device__ __forceinline__ void dec_q6k(const RawQ6K& o, int64_t j0, float w[8]) {
    const int quad = (int)((j0 & 127) >> 5);
    const int lsh = (quad & 2) ? 4 : 0, hsh = 2 * quad;
    const float ds = h2f(o.d) * (float)o.sc;
#pragma unroll
    for (int c = 0; c < 8; ++c) {
        const uint32_t ql = c < 4 ? o.ql0 : o.ql1, qh = c < 4 ? o.qh0 : o.qh1;
        const int s = 8 * (c & 3);
        const int low = (int)((ql >> (s + lsh)) & 0xF);
        const int high = (int)((qh >> (s + hsh)) & 3);
        w[c] = __fmul_rn(ds, (float)((low | (high << 4)) - 32));
    }
}

struct RawQ80 {
    uint32_t q0, q1;  // 8 int8 codes
    uint32_t d;       // fp16 bits
};

__device__ __forceinline__ RawQ80 load_q80(const uint8_t* row, int64_t j0) {
    const uint8_t* b = row + (j0 >> 5) * 34;
    const uint8_t* q = b + 2 + (j0 & 31);
    RawQ80 o;
    o.d = ld16(b);
    o.q0 = ld16(q) | (ld16(q + 2) << 16);
    o.q1 = ld16(q + 4) | (ld16(q + 6) << 16);
    return o;
}

__device__ __forceinline__ void dec_q80(const RawQ80& o, int64_t, float w[8]) {
    const float d = h2f(o.d);
#pragma unroll
    for (int c = 0; c < 4; ++c) {
        w[c] = d * (float)(int8_t)(o.q0 >> (8 * c));
        w[4 + c] = d * (float)(int8_t)(o.q1 >> (8 * c));
    }
}

// Any format, any alignment: element by element (columns past N read as 0).
struct RawAny {
    const uint8_t* row;
};

__device__ __forceinline__ RawAny load_any(const uint8_t* row, int64_t) { return RawAny{row}; }

__device__ __forceinline__ void dec_any(const RawAny& r, int dtype, int64_t j0, int64_t N,
                                        float w[8]) {
#pragma unroll
    for (int c = 0; c < 8; ++c) w[c] = j0 + c < N ? decode_elem(dtype, r.row, j0 + c) : 0.f;
}

template <int DT>
struct Fmt8;

template <>
struct Fmt8<FTC_Q4_K> {
    using Raw = RawQ4K;
    static __device__ __forceinline__ Raw load(const uint8_t* row, int64_t j0) { return load_q4k(row, j0); }
    static __device__ __forceinline__ void dec(const Raw& r, int, int64_t j0, int64_t, float w[8]) {
        dec_q4k(r, j0, w);
    }
};

template <>
struct Fmt8<FTC_Q6_K> {
    using Raw = RawQ6K;
    static __device__ __forceinline__ Raw load(const uint8_t* row, int64_t j0) { return load_q6k(row, j0); }
    static __device__ __forceinline__ void dec(const Raw& r, int, int64_t j0, int64_t, float w[8]) {
        dec_q6k(r, j0, w);
    }
};

template <>
struct Fmt8<FTC_Q8_0> {
    using Raw = RawQ80;
    static __device__ __forceinline__ Raw load(const uint8_t* row, int64_t j0) { return load_q80(row, j0); }
    static __device__ __forceinline__ void dec(const Raw& r, int, int64_t j0, int64_t, float w[8]) {
        dec_q80(r, j0, w);
    }
};

template <>
struct Fmt8<kGeneric> {
    using Raw = RawAny;
    static __device__ __forceinline__ Raw load(const uint8_t* row, int64_t j0) { return load_any(row, j0); }
    static __device__ __forceinline__ void dec(const Raw& r, int dtype, int64_t j0, int64_t N,
                                               float w[8]) {
        dec_any(r, dtype, j0, N, w);
    }
};

template <int MT>
__device__ __forceinline__ void axpy8(float (&acc)[MT][8], const float (*xs)[kAxpyMaxRows],
                                      int r, int mc, const float w[8]) {
#pragma unroll
    for (int t = 0; t < MT; ++t) {
        if (t < mc) {  // uniform over the CTA
            const float v = xs[t][r];
            if (v != 0.f) {  // uniform: the reference skips these rows
#pragma unroll
                for (int c = 0; c < 8; ++c) acc[t][c] = fmaf(v, w[c], acc[t][c]);
            }
        }
    }
}

// grid (column tiles, slabs, token groups of MT)
template <int DT, int MT>
__global__ void __launch_bounds__(kAxpyThreads) rows_axpy(AxpyArgs a) {
    using F8 = Fmt8<DT>;
    __shared__ float xs[MT][kAxpyMaxRows];
    const int64_t i0 = (int64_t)blockIdx.y * a.rows;
    const int nr = (int)min((int64_t)a.rows, a.n_in - i0);
    const int64_t m0 = (int64_t)blockIdx.z * MT;
    const int mc = (int)min((int64_t)MT, a.M - m0);
    for (int e = threadIdx.x; e < MT * nr; e += blockDim.x) {
        const int t = e / nr, r = e - t * nr;
        xs[t][r] = t < mc ? a.x[(m0 + t) * a.n_in + i0 + r] : 0.f;
    }
    __syncthreads();
    const int64_t j0 = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) * 8;
    if (j0 >= a.N) return;
    float acc[MT][8];
#pragma unroll
    for (int t = 0; t < MT; ++t)
#pragma unroll
        for (int c = 0; c < 8; ++c) acc[t][c] = 0.f;
    const uint8_t* base = a.w + i0 * a.stride;
    constexpr int UR = axpy_unroll<MT>();
    int r = 0;
    for (; r + UR <= nr; r += UR) {
        typename F8::Raw raw[UR];
#pragma unroll
        for (int u = 0; u < UR; ++u) raw[u] = F8::load(base + (int64_t)(r + u) * a.stride, j0);
#pragma unroll
        for (int u = 0; u < UR; ++u) {
            float w[8];
            F8::dec(raw[u], a.dtype, j0, a.N, w);
            axpy8(acc, xs, r + u, mc, w);
        }
    }
    for (; r < nr; ++r) {
        float w[8];
        F8::dec(F8::load(base + (int64_t)r * a.stride, j0), a.dtype, j0, a.N, w);
        axpy8(acc, xs, r, mc, w);
    }
    const int nc = (int)min((int64_t)8, a.N - j0);
    if (a.part) {
        float* p = a.part + ((int64_t)blockIdx.y * a.M + m0) * a.N + j0;
#pragma unroll
        for (int t = 0; t < MT; ++t)
            if (t < mc)
#pragma unroll
                for (int c = 0; c < 8; ++c)
                    if (c < nc) __stcg(p + (int64_t)t * a.N + c, acc[t][c]);
    } else {
        float* p = a.y + m0 * a.N + j0;
#pragma unroll
        for (int t = 0; t < MT; ++t)
            if (t < mc)
#pragma unroll
                for (int c = 0; c < 8; ++c)
                    if (c < nc) p[(int64_t)t * a.N + c] += acc[t][c];
    }
}

// y[e] += sum over slabs s (ascending) of part[s][e], e < MN.  Block (32, 8):
// lane = element, threadIdx.y = every 8th slab; the 8 sums are combined in
// threadIdx.y order.
__global__ void __launch_bounds__(256)
axpy_reduce(const float* __restrict__ part, int S, int64_t MN, float* __restrict__ y) {
    __shared__ float s[8][33];
    const int64_t e = (int64_t)blockIdx.x * 32 + threadIdx.x;
    float v = 0.f;
    if (e < MN)
        for (int k = threadIdx.y; k < S; k += 8) v += __ldcg(part + (int64_t)k * MN + e);
    s[threadIdx.y][threadIdx.x] = v;
    __syncthreads();
    if (threadIdx.y == 0 && e < MN) {
        float t = s[0][threadIdx.x];
#pragma unroll
        for (int k = 1; k < 8; ++k) t += s[k][threadIdx.x];
        y[e] += t;
    }
}

struct AxpyPlan {
    int mt, threads, col_tiles, slabs, rows, m_groups;
    size_t ws_bytes;
};

// Rows per slab: enough that a slab's partial sums (up to 8 tokens x N
// floats) stay small next to the slab's weight bytes, few enough that the
// grid fills the GPU a few times over; at most kAxpyMaxRows.
AxpyPlan plan(int dtype, int64_t n_in, int64_t N, int64_t M) {
    AxpyPlan p;
    const int64_t lanes = (N + 7) / 8;
    p.threads = (int)std::min<int64_t>(kAxpyThreads, (lanes + 31) / 32 * 32);
    p.col_tiles = (int)((lanes + p.threads - 1) / p.threads);
    p.mt = M <= 1 ? 1 : M <= 2 ? 2 : M <= 4 ? 4 : kAxpyMT;
    p.m_groups = (int)((M + p.mt - 1) / p.mt);
    const int64_t rb = row_bytes(dtype, N);
    const int64_t mt = p.mt;
    const int64_t min_rows = std::max<int64_t>(8, (2 * mt * N * 4 + rb - 1) / rb);
    int64_t slabs = std::max<int64_t>(1, kAxpyTargetCtas / ((int64_t)p.col_tiles * p.m_groups));
    slabs = std::min<int64_t>(slabs, (n_in + min_rows - 1) / min_rows);
    int64_t rows = (n_in + slabs - 1) / slabs;
    rows = std::min<int64_t>(rows, kAxpyMaxRows);
    p.rows = (int)rows;
    p.slabs = (int)((n_in + rows - 1) / rows);
    p.ws_bytes = p.slabs > 1 ? (size_t)p.slabs * (size_t)M * (size_t)N * sizeof(float) : 0;
    return p;
}

constexpr int64_t kMaxSlabs = 65535, kMaxGroups = 65535;

int validate(int dtype, const void* w, int64_t n_in, int64_t N, int64_t row_stride, const float* x,
             int64_t M, const float* y) {
    const Fmt f = fmt_of(dtype);
    FTC_REQUIRE(f.block_elems > 0, FTC_E_UNSUPPORTED, "ftc_matmul_down_axpy: unknown dtype");
    FTC_REQUIRE(M >= 0 && n_in >= 0 && N > 0, FTC_E_INVALID, "ftc_matmul_down_axpy: bad shape");
    FTC_REQUIRE(N % f.block_elems == 0, FTC_E_INVALID,
                "ftc_matmul_down_axpy: a row must be a whole number of blocks");
    FTC_REQUIRE(row_stride >= row_bytes(dtype, N), FTC_E_INVALID,
                "ftc_matmul_down_axpy: row_stride smaller than a row");
    FTC_REQUIRE(n_in <= kMaxSlabs * kAxpyMaxRows && M <= kMaxGroups * kAxpyMT, FTC_E_INVALID,
                "ftc_matmul_down_axpy: n_in or M too large for one launch");
    FTC_REQUIRE(M == 0 || n_in == 0 || (w && x && y), FTC_E_INVALID,
                "ftc_matmul_down_axpy: null pointer");
    return FTC_OK;
}

template <int DT>
void launch(const AxpyPlan& p, const AxpyArgs& a, cudaStream_t st) {
    dim3 grid((unsigned)p.col_tiles, (unsigned)p.slabs, (unsigned)p.m_groups);
    switch (p.mt) {
        case 1: rows_axpy<DT, 1><<<grid, p.threads, 0, st>>>(a); break;
        case 2: rows_axpy<DT, 2><<<grid, p.threads, 0, st>>>(a); break;
        case 4: rows_axpy<DT, 4><<<grid, p.threads, 0, st>>>(a); break;
        default: rows_axpy<DT, kAxpyMT><<<grid, p.threads, 0, st>>>(a); break;
    }
}

}  // namespace

size_t down_axpy_workspace_bytes(int dtype, int64_t n_in, int64_t N, int64_t M) {
    if (fmt_of(dtype).block_elems == 0 || n_in <= 0 || N <= 0 || M <= 0) return 0;
    return plan(dtype, n_in, N, M).ws_bytes;
}

// The vector decoders need Q4_K rows on 16-byte boundaries and Q6_K / Q8_0
// rows on 2-byte boundaries; other weights take the element-by-element
// decoder, which gives the same bits (same plan, same order of sums).
int down_axpy(int dtype, const void* w, int64_t n_in, int64_t N, int64_t row_stride,
              const float* x, int64_t M, float* y, void* ws, size_t ws_bytes, cudaStream_t st) {
    int rc = validate(dtype, w, n_in, N, row_stride, x, M, y);
    if (rc) return rc;
    if (inject_fail("ftc_matmul_down_axpy"))
        return set_error(FTC_E_INJECTED, "ftc_matmul_down_axpy: injected failure");
    if (M == 0 || n_in == 0) return ok();
    const AxpyPlan p = plan(dtype, n_in, N, M);
    FTC_REQUIRE(p.ws_bytes == 0 || (ws && ws_bytes >= p.ws_bytes), FTC_E_INVALID,
                "ftc_matmul_down_axpy: workspace smaller than ftc_matmul_down_axpy_workspace_bytes");
    AxpyArgs a{static_cast<const uint8_t*>(w), row_stride, n_in, N, dtype, x, M, p.rows,
               p.slabs > 1 ? static_cast<float*>(ws) : nullptr, y};
    const uintptr_t wa = (uintptr_t)w;
    if (dtype == FTC_Q4_K && wa % 16 == 0 && row_stride % 16 == 0)
        launch<FTC_Q4_K>(p, a, st);
    else if (dtype == FTC_Q6_K && wa % 2 == 0 && row_stride % 2 == 0)
        launch<FTC_Q6_K>(p, a, st);
    else if (dtype == FTC_Q8_0 && wa % 2 == 0 && row_stride % 2 == 0)
        launch<FTC_Q8_0>(p, a, st);
    else
        launch<kGeneric>(p, a, st);
    FTC_CUDA(cudaGetLastError());
    if (p.slabs > 1) {
        const int64_t MN = M * N;
        axpy_reduce<<<(unsigned)((MN + 31) / 32), dim3(32, 8), 0, st>>>(
            static_cast<const float*>(ws), p.slabs, MN, y);
        FTC_CUDA(cudaGetLastError());
    }
    return ok();
}

}  // namespace ftc
