// attention.cu -- the engine's attention on the device: causal grouped-query
// attention over an fp32 KV cache in HBM, and RoPE.
//
// The B200 form of Engine::Impl::attn (ft/src/engine.cpp:137-177): query row
// m (position base + m) of head h attends positions 0 .. base + m of KV head
// h / (n_head / n_head_kv); positions below `base` come from the cache rows,
// the rest from the current block's rows (the same memory when the caller
// wrote the block into the cache first, as the engine does with write_kv,
// ft/src/engine.cpp:553-565).  Rows are [position][n_head_kv * head_dim]
// fp32, as ft::KvCache keeps them (ft/include/ft/kv_cache.h:12-20).
//
// Decode reads every cached K and V row once per KV head, so the kernel is
// HBM-bound: the positions of a row are cut into splits of L positions (a
// multiple of 32), one CTA per (KV head, group of G query heads, row,
// split), with as many splits as fill one wave of resident CTAs.  A CTA
// walks its split in chunks of 32 positions whose K and V rows it brings
// into shared memory with 16-byte cp.async copies, one chunk ahead of the
// one it computes on:
// G x 32 scores from shared memory, an online softmax (running maximum and
// sum, the accumulator rescaled when the maximum grows) and the weighted V
// sum.  A row with one split is finished in place; else a second kernel
// combines the splits in split order (deterministic):
//   out = sum_s acc_s * exp(max_s - max) / sum_s sum_s * exp(max_s - max).
// The reference normalises before the V sum (w = e / sum) and sums in
// position order; the results agree to fp32 rounding.
//
// RoPE (ft/src/engine.cpp:43-60, applied at 545-551): frequencies, angles,
// cos and sin in double as the reference computes them, rounded to float,
// the rotation in float with every product and sum rounded separately (no
// fused multiply-add), so it matches the reference's float arithmetic.
#include <algorithm>
#include <mutex>

#include "common.cuh"

namespace ftc {
namespace {

constexpr int kAttnThreads = 128;  // 4 warps per CTA

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
    const uint32_t s = (uint32_t)__cvta_generic_to_shared(smem);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(s), "l"(gmem) : "memory");
}

__device__ __forceinline__ void cp_async_wait_all() {
    asm volatile("cp.async.commit_group;\ncp.async.wait_group 0;" ::: "memory");
}

struct AttnArgs {
    const float* q;        // [M][n_head][HD]
    const float* kc;       // cache rows (position < base)
    const float* vc;
    const float* kb;       // block rows (position >= base), row p at (p - base)
    const float* vb;
    float* out;            // [M][n_head][HD]
    float* part;           // [M][n_head][S][HD] split sums (S > 1)
    float2* stat;          // [M][n_head][S] (split maximum, sum of exponentials)
    int64_t kv_stride;     // floats per position row
    int64_t base;
    int n_head, gqa, L, S;
    float scale;
};

// A CTA walks its split in chunks of 32 positions, two chunk buffers in
// shared memory: while chunk c is scored and summed, chunk c + 1 is in
// flight.  Buffer layout: K [32][HD + 4] (padded: the 16-byte loads of 8
// lanes reading 8 consecutive positions at the same k hit 8 different bank
// quads), V [32][HD].  Then q [G][HD], the chunk's exponentials [G][32] and
// per head the running maximum, running sum and this chunk's rescale factor
// (online softmax: the accumulator is multiplied by exp(old max - new max)
// whenever the maximum grows).  The final cross-group V-sum reduction reuses
// buffer 0 (512 G floats, within 32 (2 HD + 4) for every HD and G <= 8).
constexpr int kChunk = 32;
static_assert(512 * 8 <= kChunk * (2 * 64 + 4), "V-sum reduction fits a chunk buffer");

__device__ __forceinline__ void cp_async_commit() {
    asm volatile("cp.async.commit_group;" ::: "memory");
}

template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

template <int HD, int G>
__global__ void __launch_bounds__(kAttnThreads)
attn_split(const AttnArgs a) {
    extern __shared__ __align__(16) float sm[];
    constexpr int KP = HD + 4, C4 = HD / 4, BUF = kChunk * (KP + HD);
    constexpr int NGRP = kAttnThreads / C4;  // position groups of the V sum
    float* qs = sm + 2 * BUF;
    float* es = qs + G * HD;
    float* mrun = es + G * kChunk;
    float* lrun = mrun + G;
    float* alpha = lrun + G;

    const int ngrp = a.gqa / G;
    const int kvh = blockIdx.x / ngrp;
    const int h0 = kvh * a.gqa + (blockIdx.x % ngrp) * G;  // first query head of this CTA
    const int m = blockIdx.y;
    const int s = blockIdx.z;
    const int64_t len = a.base + m + 1;
    const int64_t p0 = (int64_t)s * a.L;
    if (p0 >= len) return;  // this row has fewer splits
    const int n = (int)(len - p0 < a.L ? len - p0 : a.L);
    const int nch = (n + kChunk - 1) / kChunk;
    const int S_m = (int)((len + a.L - 1) / a.L);
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5;

    // chunk c (rows [32c, 32c + rows) of the split) -> buffer c & 1
    auto issue = [&](int c) {
        float* ks = sm + (c & 1) * BUF;
        float* vs = ks + kChunk * KP;
        const int rows = min(kChunk, n - kChunk * c);
        for (int i = t; i < rows * C4; i += kAttnThreads) {
            const int r = i / C4, cc = i - r * C4;
            const int64_t p = p0 + kChunk * c + r;
            const int64_t off =
                (p < a.base ? p : p - a.base) * a.kv_stride + (int64_t)kvh * HD + 4 * cc;
            cp_async16(ks + r * KP + 4 * cc, (p < a.base ? a.kc : a.kb) + off);
            cp_async16(vs + r * HD + 4 * cc, (p < a.base ? a.vc : a.vb) + off);
        }
        cp_async_commit();
    };
    issue(0);
    for (int i = t; i < G * HD; i += kAttnThreads)
        qs[i] = a.q[((int64_t)m * a.n_head + h0) * HD + i];
    if (t < G) {
        mrun[t] = -INFINITY;
        lrun[t] = 0.f;
    }
    const int d4 = t % C4, grp = t / C4;
    float4 acc[G];
#pragma unroll
    for (int g = 0; g < G; ++g) acc[g] = make_float4(0.f, 0.f, 0.f, 0.f);

    for (int c = 0; c < nch; ++c) {
        if (c + 1 < nch) {
            issue(c + 1);
            cp_async_wait<1>();  // chunk c has landed (c + 1 may still fly)
        } else {
            cp_async_wait<0>();
        }
        __syncthreads();
        const float* ks = sm + (c & 1) * BUF;
        const float* vs = ks + kChunk * KP;
        const int rows = min(kChunk, n - kChunk * c);

        // scores: lane j takes position j, warp w heads w, w + 4, ...
        if (lane < rows) {
            const float4* kr = reinterpret_cast<const float4*>(ks + lane * KP);
            for (int g = warp; g < G; g += 4) {
                const float4* qg = reinterpret_cast<const float4*>(qs + g * HD);
                float d0 = 0.f, d1 = 0.f;
#pragma unroll 8
                for (int cc = 0; cc < C4; ++cc) {
                    const float4 k4 = kr[cc], q4 = qg[cc];
                    d0 = fmaf(q4.x, k4.x, d0);
                    d1 = fmaf(q4.y, k4.y, d1);
                    d0 = fmaf(q4.z, k4.z, d0);
                    d1 = fmaf(q4.w, k4.w, d1);
                }
                es[g * kChunk + lane] = (d0 + d1) * a.scale;
            }
        }
        __syncthreads();

        // online softmax: new maximum, this chunk's exponentials, rescale
        for (int g = warp; g < G; g += 4) {
            const float sv = lane < rows ? es[g * kChunk + lane] : -INFINITY;
            float cm = sv;
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) cm = fmaxf(cm, __shfl_xor_sync(0xffffffffu, cm, o));
            const float mo = mrun[g], mn = fmaxf(mo, cm);
            const float e = lane < rows ? expf(sv - mn) : 0.f;
            es[g * kChunk + lane] = e;
            float se = e;
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) se += __shfl_xor_sync(0xffffffffu, se, o);
            if (lane == 0) {
                const float al = expf(mo - mn);  // 0 on the first chunk (mo = -inf)
                alpha[g] = al;
                lrun[g] = lrun[g] * al + se;
                mrun[g] = mn;
            }
        }
        __syncthreads();

        // weighted V sum: thread t takes 4 dimensions (d4) of every NGRP-th row
#pragma unroll
        for (int g = 0; g < G; ++g) {
            const float al = alpha[g];
            acc[g].x *= al;
            acc[g].y *= al;
            acc[g].z *= al;
            acc[g].w *= al;
        }
        for (int r = grp; r < rows; r += NGRP) {
            const float4 v4 = reinterpret_cast<const float4*>(vs + r * HD)[d4];
#pragma unroll
            for (int g = 0; g < G; ++g) {
                const float e = es[g * kChunk + r];
                acc[g].x = fmaf(e, v4.x, acc[g].x);
                acc[g].y = fmaf(e, v4.y, acc[g].y);
                acc[g].z = fmaf(e, v4.z, acc[g].z);
                acc[g].w = fmaf(e, v4.w, acc[g].w);
            }
        }
        __syncthreads();  // buffer c & 1 is refilled by the next iteration's copies
    }

    // add the NGRP group sums in group order
    float4* red = reinterpret_cast<float4*>(sm);  // [NGRP][G][C4] over buffer 0
#pragma unroll
    for (int g = 0; g < G; ++g) red[(grp * G + g) * C4 + d4] = acc[g];
    __syncthreads();
    for (int i = t; i < G * C4; i += kAttnThreads) {
        const int g = i / C4, c = i - g * C4;
        float4 v = red[g * C4 + c];
        for (int k = 1; k < NGRP; ++k) {
            const float4 w = red[(k * G + g) * C4 + c];
            v.x += w.x;
            v.y += w.y;
            v.z += w.z;
            v.w += w.w;
        }
        const int64_t row = (int64_t)m * a.n_head + h0 + g;
        if (S_m == 1) {
            const float inv = 1.f / lrun[g];
            reinterpret_cast<float4*>(a.out + row * HD)[c] =
                make_float4(v.x * inv, v.y * inv, v.z * inv, v.w * inv);
        } else {
            reinterpret_cast<float4*>(a.part + (row * a.S + s) * HD)[c] = v;
            if (c == 0) a.stat[row * a.S + s] = make_float2(mrun[g], lrun[g]);
        }
    }
}

// Rows with more than one split: combine the splits in split order.  The
// split weights exp(max_s - max) go to shared memory once; thread (d, sg)
// sums the splits s = sg, sg + SG, ... of dimension d, and the SG partial
// sums are added in sg order (deterministic).
__global__ void __launch_bounds__(256)
attn_combine(const AttnArgs a, int HD) {
    extern __shared__ float wsm[];  // [S] split weights, then [SG][HD] partial sums
    __shared__ float red[32];
    const int h = blockIdx.x, m = blockIdx.y;
    const int64_t len = a.base + m + 1;
    const int S_m = (int)((len + a.L - 1) / a.L);
    if (S_m == 1) return;  // finished by the split kernel
    const int64_t row = (int64_t)m * a.n_head + h;
    const float2* st = a.stat + row * a.S;
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5, nw = blockDim.x >> 5;
    float mx = -INFINITY;
    for (int s = t; s < S_m; s += blockDim.x) mx = fmaxf(mx, st[s].x);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if (lane == 0) red[warp] = mx;
    __syncthreads();
    mx = red[0];
    for (int w = 1; w < nw; ++w) mx = fmaxf(mx, red[w]);
    for (int s = t; s < S_m; s += blockDim.x) wsm[s] = expf(st[s].x - mx);
    __syncthreads();
    if (t == 0) {
        float tot = 0.f;
        for (int s = 0; s < S_m; ++s) tot += st[s].y * wsm[s];
        red[0] = tot;  // every thread has read red[] above
    }
    const int SG = (int)blockDim.x / HD;
    const int d = t % HD, sg = t / HD;
    float v = 0.f;
    if (sg < SG) {
#pragma unroll 8
        for (int s = sg; s < S_m; s += SG) v = fmaf(a.part[(row * a.S + s) * HD + d], wsm[s], v);
    }
    float* psum = wsm + a.S;
    if (sg < SG) psum[sg * HD + d] = v;
    __syncthreads();
    if (sg == 0) {
        float o = psum[d];
        for (int k = 1; k < SG; ++k) o += psum[k * HD + d];
        a.out[row * HD + d] = o / red[0];
    }
}

// RoPE of rows m at position base + m: block m, thread i takes the pair i of
// every head.
__global__ void rope_kernel(float* x, int heads, int hd, int64_t base, double theta, int neox) {
    const int m = blockIdx.x;
    const int half = hd / 2;
    for (int i = threadIdx.x; i < half; i += blockDim.x) {
        const double f = pow(theta, -2.0 * (double)i / (double)hd);
        const double ang = (double)(base + m) * f;
        double sd, cd;
        sincos(ang, &sd, &cd);
        const float c = (float)cd, s = (float)sd;
        const int i0 = neox ? i : 2 * i, i1 = neox ? i + half : 2 * i + 1;
        for (int h = 0; h < heads; ++h) {
            float* v = x + ((int64_t)m * heads + h) * hd;
            const float av = v[i0], bv = v[i1];
            v[i0] = __fsub_rn(__fmul_rn(av, c), __fmul_rn(bv, s));
            v[i1] = __fadd_rn(__fmul_rn(av, s), __fmul_rn(bv, c));
        }
    }
}

struct AttnPlan {
    int G, L, S;
};

// two chunk buffers, q, the chunk's exponentials, three floats per head
size_t attn_smem(int HD, int G) {
    return (size_t)(2 * kChunk * (2 * HD + 4) + G * HD + G * kChunk + 3 * G) * sizeof(float);
}

// CTAs of attn_split<HD, G> one SM holds at once, queried once per device
// (the attribute and the occupancy belong to the device's context).
template <int HD, int G>
int resident_ctas() {
    static std::mutex mu;
    static int cached[64] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) dev = -1;
    if (dev >= 0) {
        std::lock_guard<std::mutex> lk(mu);
        if (cached[dev]) return cached[dev];
    }
    int n = 0;
    const size_t smem = attn_smem(HD, G);
    const int rc = opt_in_smem(reinterpret_cast<const void*>(attn_split<HD, G>), (int)smem,
                               "cudaFuncSetAttribute(attn_split)");
    if (rc) return 1;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, attn_split<HD, G>, kAttnThreads, smem) !=
            cudaSuccess ||
        n < 1)
        return 1;
    if (dev >= 0) {
        std::lock_guard<std::mutex> lk(mu);
        cached[dev] = n;
    }
    return n;
}

template <int HD>
int resident_ctas_g(int G) {
    return G == 8 ? resident_ctas<HD, 8>() : G == 4 ? resident_ctas<HD, 4>()
         : G == 2 ? resident_ctas<HD, 2>() : resident_ctas<HD, 1>();
}

// Query heads per CTA (a power of two dividing gqa, at most 8) and the
// split length L, a whole number of 32-position chunks: the longest row's
// chunks shared out over as many splits as fit one wave of resident CTAs
// (a CTA per SM slot), so every CTA of a decode launch runs at once.
AttnPlan attn_plan(int64_t M, int64_t n_head_kv, int64_t gqa, int64_t base, int64_t head_dim) {
    AttnPlan p;
    p.G = gqa % 8 == 0 ? 8 : gqa % 4 == 0 ? 4 : gqa % 2 == 0 ? 2 : 1;
    const int res = head_dim == 64 ? resident_ctas_g<64>(p.G)
                  : head_dim == 128 ? resident_ctas_g<128>(p.G) : resident_ctas_g<256>(p.G);
    const int64_t ctas_per_split = n_head_kv * (gqa / p.G) * M;
    const int64_t len_max = base + M;
    const int64_t chunks = (len_max + kChunk - 1) / kChunk;
    const int64_t slots = (int64_t)res * device_sms();
    const int64_t splits = std::max<int64_t>(1, std::min<int64_t>(chunks, slots / ctas_per_split));
    const int64_t per = (chunks + splits - 1) / splits;  // chunks per split
    p.L = (int)(per * kChunk);
    p.S = (int)((len_max + p.L - 1) / p.L);
    return p;
}

template <int HD, int G>
int launch_split(const AttnArgs& a, int64_t M, int64_t n_head_kv, cudaStream_t st) {
    const size_t smem = attn_smem(HD, G);
    const int rc = opt_in_smem(reinterpret_cast<const void*>(attn_split<HD, G>), (int)smem,
                               "cudaFuncSetAttribute(attn_split)");
    if (rc) return rc;
    const dim3 grid((unsigned)(n_head_kv * (a.gqa / G)), (unsigned)M, (unsigned)a.S);
    attn_split<HD, G><<<grid, kAttnThreads, smem, st>>>(a);
    FTC_CUDA(cudaGetLastError());
    return FTC_OK;
}

template <int HD>
int launch_split_g(int G, const AttnArgs& a, int64_t M, int64_t n_head_kv, cudaStream_t st) {
    switch (G) {
        case 8: return launch_split<HD, 8>(a, M, n_head_kv, st);
        case 4: return launch_split<HD, 4>(a, M, n_head_kv, st);
        case 2: return launch_split<HD, 2>(a, M, n_head_kv, st);
        default: return launch_split<HD, 1>(a, M, n_head_kv, st);
    }
}

}  // namespace

int attention_check(int64_t M, int64_t n_head, int64_t n_head_kv, int64_t head_dim, int64_t base,
                    const char* who) {
    FTC_REQUIRE(M > 0 && n_head > 0 && n_head_kv > 0 && base >= 0, FTC_E_INVALID,
                std::string(who) + ": empty shape or negative base");
    FTC_REQUIRE(n_head % n_head_kv == 0, FTC_E_INVALID,
                std::string(who) + ": n_head must be a multiple of n_head_kv");
    FTC_REQUIRE(head_dim == 64 || head_dim == 128 || head_dim == 256, FTC_E_UNSUPPORTED,
                std::string(who) + ": head_dim must be 64, 128 or 256");
    FTC_REQUIRE(M <= 65535 && (base + M + 31) / 32 <= 65535 && n_head <= (1 << 20),
                FTC_E_UNSUPPORTED, std::string(who) + ": too many rows or positions for one launch");
    return FTC_OK;
}

size_t attention_workspace_bytes(int64_t M, int64_t n_head, int64_t n_head_kv, int64_t head_dim,
                                 int64_t base) {
    if (attention_check(M, n_head, n_head_kv, head_dim, base, "ftc_attention_workspace_bytes"))
        return 0;
    const AttnPlan p = attn_plan(M, n_head_kv, n_head / n_head_kv, base, head_dim);
    if (p.S == 1) return 0;
    // split statistics (float2 each), padded to 16 bytes, then the split sums
    const size_t stats = ((size_t)(M * n_head) * (size_t)p.S * sizeof(float2) + 15) & ~size_t(15);
    return stats + (size_t)(M * n_head) * (size_t)p.S * (size_t)head_dim * sizeof(float);
}

int attention(const float* q, int64_t M, int64_t n_head, int64_t n_head_kv, int64_t head_dim,
              const float* k_cache, const float* v_cache, int64_t kv_stride, int64_t base,
              const float* k_blk, const float* v_blk, float* out, void* ws, size_t ws_bytes,
              cudaStream_t st) {
    int rc = attention_check(M, n_head, n_head_kv, head_dim, base, "ftc_attention");
    if (rc) return rc;
    FTC_REQUIRE(q && out && k_blk && v_blk && (base == 0 || (k_cache && v_cache)), FTC_E_INVALID,
                "ftc_attention: null pointer");
    FTC_REQUIRE(kv_stride >= n_head_kv * head_dim && kv_stride % 4 == 0, FTC_E_INVALID,
                "ftc_attention: kv_stride must cover n_head_kv * head_dim and be a multiple of 4");
    auto a16 = [](const void* p) { return p == nullptr || (uintptr_t)p % 16 == 0; };
    FTC_REQUIRE(a16(q) && a16(out) && a16(k_cache) && a16(v_cache) && a16(k_blk) && a16(v_blk),
                FTC_E_INVALID, "ftc_attention: buffers must be 16-byte aligned");
    const int64_t gqa = n_head / n_head_kv;
    const AttnPlan p = attn_plan(M, n_head_kv, gqa, base, head_dim);
    const size_t need = attention_workspace_bytes(M, n_head, n_head_kv, head_dim, base);
    FTC_REQUIRE(ws_bytes >= need && (need == 0 || (ws && a16(ws))), FTC_E_INVALID,
                "ftc_attention: workspace smaller than ftc_attention_workspace_bytes");
    AttnArgs a;
    a.q = q;
    a.kc = k_cache;
    a.vc = v_cache;
    a.kb = k_blk;
    a.vb = v_blk;
    a.out = out;
    const size_t stats = ((size_t)(M * n_head) * (size_t)p.S * sizeof(float2) + 15) & ~size_t(15);
    a.stat = need ? static_cast<float2*>(ws) : nullptr;
    a.part = need ? reinterpret_cast<float*>(static_cast<uint8_t*>(ws) + stats) : nullptr;
    a.kv_stride = kv_stride;
    a.base = base;
    a.n_head = (int)n_head;
    a.gqa = (int)gqa;
    a.L = p.L;
    a.S = p.S;
    a.scale = 1.f / sqrtf((float)head_dim);
    if (head_dim == 64) rc = launch_split_g<64>(p.G, a, M, n_head_kv, st);
    else if (head_dim == 128) rc = launch_split_g<128>(p.G, a, M, n_head_kv, st);
    else rc = launch_split_g<256>(p.G, a, M, n_head_kv, st);
    if (rc) return rc;
    if (p.S > 1) {
        const size_t csm = (size_t)(p.S + 256) * sizeof(float);  // split weights + partial sums
        attn_combine<<<dim3((unsigned)n_head, (unsigned)M), 256, csm, st>>>(a, (int)head_dim);
        FTC_CUDA(cudaGetLastError());
    }
    return FTC_OK;
}

int rope(float* x, int64_t M, int64_t heads, int64_t head_dim, int64_t base, double theta,
         int neox, cudaStream_t st) {
    FTC_REQUIRE(x && M >= 0 && heads > 0 && head_dim > 0 && head_dim % 2 == 0 && base >= 0,
                FTC_E_INVALID, "ftc_rope: bad argument");
    FTC_REQUIRE(M <= 0x7fffffff && heads <= (1 << 20) && head_dim <= 65536, FTC_E_UNSUPPORTED,
                "ftc_rope: shape too large");
    if (M == 0) return FTC_OK;
    const int threads = (int)std::min<int64_t>(256, std::max<int64_t>(32, head_dim / 2));
    rope_kernel<<<(unsigned)M, threads, 0, st>>>(x, (int)heads, (int)head_dim, base, theta,
                                                 neox ? 1 : 0);
    FTC_CUDA(cudaGetLastError());
    return FTC_OK;
}

}  // namespace ftc
