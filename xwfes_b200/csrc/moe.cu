// moe.cu -- routed-expert MoE FFN on the device: the reference's
// Engine::Impl::moe_ffn (ft/src/engine.cpp:179-241) with its expert FFN
// (ft/src/cpu_backend.cpp:106-149) in the standard GGUF down layout.
//
//   route    p = softmax(logits[t]) over E experts (fp32 exps, double sum,
//            ft/src/engine.cpp:62-72); the U most probable experts (ties to
//            the lower index); w[t][u] = p / sum of the U chosen
//            (ft/src/engine.cpp:198-215).
//   group    the T*U (token, slot) pairs sorted by expert, tokens ascending
//            within an expert (the reference's per-expert token lists,
//            ft/src/engine.cpp:212-213); experts ranked by first use.
//   gather   x rows into expert order as fp16, each row scaled by a power of
//            two 2^-xs into [2^14, 2^15) (exact; fp16 keeps 11 bits for any
//            input range).
//   gate/up  one grouped dequant-GEMM launch over both weight sets
//            (gemm_q4k_sm100.cu): gu[row] = [x.gate_e | x.up_e] in fp32.
//   silu     h = silu(g) * u in fp32 (g / (1 + exp(-g)),
//            ft/src/cpu_backend.cpp:127) after undoing 2^-xs, stored as fp16
//            with its own row scale 2^-hs.
//   down     grouped dequant-GEMM: yd[row] = h . down_e  (fp32).
//   combine  out[t] = sum over t's slots of w * (yd * 2^hs), added in the
//            experts' first-use order with separately rounded products and
//            sums, as the reference's tmpo[m] += w * acb
//            (ft/src/engine.cpp:229-236).
//
// Every step reads device-side counts: there is no host round trip, so the
// whole layer can be captured in a CUDA graph.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>

#include "common.cuh"
#include "gemv_batch.cuh"
#include "sm100.cuh"

namespace ftc {

int gemm_q4k_grouped(const void* w, const void* w2, int n_sets, int64_t G, int64_t plane_stride,
                     int64_t N, int64_t K, int64_t row_stride, const void* x, int x_dtype,
                     int64_t rows, const int32_t* counts, const int32_t* offsets,
                     int64_t max_rows_per_group, void* y, int y_dtype, int64_t ldy,
                     cudaStream_t st, const int32_t* row_exp = nullptr);

namespace {

constexpr int kRouteThreads = 1024;
constexpr int kMaxExperts = 256;
constexpr int kMaxTopK = 8;

__device__ __forceinline__ float to_f(float v) { return v; }
__device__ __forceinline__ float to_f(__half v) { return __half2float(v); }
__device__ __forceinline__ float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }

// Power-of-two row scale for fp16 operands: s with amax * 2^-s in
// [2^14, 2^15) (below fp16's 65504), clamped so 2^s and 2^-s are normal
// floats.  Scaling by 2^-s and back by 2^s is exact.
__device__ __forceinline__ int row_scale_exp(float amax) {
    if (!(amax > 0.f) || !isfinite(amax)) return 0;
    const int e = (int)((__float_as_uint(amax) >> 23) & 0xFF) - 127;  // floor(log2) for normals
    return max(-126, min(126, e - 14));
}

__device__ __forceinline__ float exp2i(int s) { return __uint_as_float((uint32_t)(s + 127) << 23); }

__device__ __forceinline__ float block_max(float v, float* red) {
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    const int w = threadIdx.x >> 5, nw = blockDim.x >> 5;
    __syncthreads();  // red may still be read by a previous call
    if ((threadIdx.x & 31) == 0) red[w] = v;
    __syncthreads();
    float m = 0.f;
    for (int i = 0; i < nw; ++i) m = fmaxf(m, red[i]);
    return m;
}

// Inclusive prefix sum of v over the CTA (blockDim a multiple of 32): warp
// scans by shuffles, then one scan of the warp totals -- two barriers
// instead of one per doubling step.  *total gets the CTA's sum; warp_tot
// (32 ints of shared memory) may be reused after the caller's next barrier.
__device__ __forceinline__ int block_incl_scan(int v, int* warp_tot, int* total) {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = blockDim.x >> 5;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int n = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += n;
    }
    if (lane == 31) warp_tot[w] = v;
    __syncthreads();
    if (w == 0) {
        int t = lane < nw ? warp_tot[lane] : 0;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int n = __shfl_up_sync(0xffffffffu, t, o);
            if (lane >= o) t += n;
        }
        if (lane < nw) warp_tot[lane] = t;
    }
    __syncthreads();
    *total = warp_tot[nw - 1];
    return v + (w > 0 ? warp_tot[w - 1] : 0);
}

// Threads of the routing CTA: the tokens rounded up to whole warps (the
// kernel's barriers cost in proportion to the CTA's size, and decode routes
// one token).
int route_threads(int64_t T) {
    const int64_t t = std::max<int64_t>(32, (T + 31) / 32 * 32);
    return (int)std::min<int64_t>(t, kRouteThreads);
}

// One CTA routes all T tokens and builds the expert grouping:
//   idx[t*U+u], w[t*U+u]  chosen experts and renormalised weights
//   counts[e], offsets[e] rows of expert e in expert order (offsets[E] = T*U)
//   rank[e]               order of first use (ft/src/engine.cpp:213-217)
//   pos[t*U+u]            row of pair (t, u) in expert order
//   row_token[row]        token of each row
__global__ void __launch_bounds__(kRouteThreads)
moe_route(const float* __restrict__ logits, int T, int E, int U, int32_t* __restrict__ idx,
          float* __restrict__ wts, int32_t* __restrict__ counts, int32_t* __restrict__ offsets,
          int32_t* __restrict__ rank, int32_t* __restrict__ pos, int32_t* __restrict__ row_token) {
    grid_launch_dependents();  // the next launch may start its prologue
    __shared__ int s_count[kMaxExperts];
    __shared__ int s_first[kMaxExperts];
    __shared__ int s_off[kMaxExperts];
    __shared__ int s_wtot[32];
    for (int e = threadIdx.x; e < E; e += blockDim.x) {
        s_count[e] = 0;
        s_first[e] = INT32_MAX;
    }
    __syncthreads();
    for (int t = threadIdx.x; t < T; t += blockDim.x) {
        const float* r = logits + (int64_t)t * E;
        float mx = r[0];
        for (int j = 1; j < E; ++j) mx = fmaxf(mx, r[j]);
        double sum = 0.0;
        for (int j = 0; j < E; ++j) sum += (double)expf(r[j] - mx);
        const float inv = (float)(1.0 / sum);
        int chosen[kMaxTopK];
        float pr[kMaxTopK];
        for (int u = 0; u < U; ++u) {
            int best = -1;
            float bp = 0.f;
            for (int j = 0; j < E; ++j) {
                bool taken = false;
                for (int v = 0; v < u; ++v) taken |= (chosen[v] == j);
                if (taken) continue;
                const float pj = expf(r[j] - mx) * inv;
                if (best < 0 || pj > bp) {
                    best = j;
                    bp = pj;
                }
            }
            chosen[u] = best;
            pr[u] = bp;
        }
        float wsum = 0.f;
        for (int u = 0; u < U; ++u) wsum += pr[u];
        const float winv = wsum > 0.f ? 1.f / wsum : 0.f;
        for (int u = 0; u < U; ++u) {
            idx[t * U + u] = chosen[u];
            wts[t * U + u] = pr[u] * winv;
            atomicAdd(&s_count[chosen[u]], 1);
            atomicMin(&s_first[chosen[u]], t * U + u);
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        int acc = 0;
        for (int e = 0; e < E; ++e) {
            s_off[e] = acc;
            offsets[e] = acc;
            counts[e] = s_count[e];
            acc += s_count[e];
        }
        offsets[E] = acc;
    }
    for (int e = threadIdx.x; e < E; e += blockDim.x) {
        int rk = 0;
        if (s_first[e] != INT32_MAX)
            for (int f = 0; f < E; ++f) rk += s_first[f] < s_first[e];
        rank[e] = s_first[e] == INT32_MAX ? -1 : rk;
    }
    __syncthreads();
    // rows in expert order, tokens ascending within an expert: the row of
    // (t, e) is offsets[e] + #{t' < t routed to e}, one block scan per expert
    for (int e = 0; e < E; ++e) {
        if (s_count[e] == 0) continue;  // uniform: shared value
        int carry = 0;
        for (int t0 = 0; t0 < T; t0 += blockDim.x) {
            const int t = t0 + threadIdx.x;
            int slot = -1;
            if (t < T)
                for (int u = 0; u < U; ++u)
                    if (idx[t * U + u] == e) slot = u;
            int chunk_total = 0;
            const int incl = block_incl_scan(slot >= 0 ? 1 : 0, s_wtot, &chunk_total);
            if (slot >= 0) {
                const int row = s_off[e] + carry + incl - 1;
                pos[t * U + slot] = row;
                row_token[row] = t;
            }
            carry += chunk_total;
            __syncthreads();  // s_wtot is rewritten by the next chunk's scan
        }
    }
}

// xg[row] = fp16(x[row_token[row]] * 2^-xs[row]), one CTA per row
// (row_token nullptr: x is already in row order)
template <typename TI>
__global__ void moe_gather_scale(const TI* __restrict__ x, const int32_t* __restrict__ row_token,
                                 int K, __half* __restrict__ xg, int32_t* __restrict__ xs) {
    grid_launch_dependents();  // the next launch may start its prologue
    __shared__ float red[32];
    const int row = blockIdx.x;
    const TI* src = x + (int64_t)(row_token ? row_token[row] : row) * K;
    float amax = 0.f;
    for (int k = threadIdx.x; k < K; k += blockDim.x) amax = fmaxf(amax, fabsf(to_f(src[k])));
    const int s = row_scale_exp(block_max(amax, red));
    const float sc = exp2i(-s);
    __half2* dst = reinterpret_cast<__half2*>(xg + (int64_t)row * K);
    for (int k = 2 * threadIdx.x; k < K; k += 2 * blockDim.x)
        dst[k >> 1] = __floats2half2_rn(to_f(src[k]) * sc, to_f(src[k + 1]) * sc);
    if (threadIdx.x == 0) xs[row] = s;
}

// h = silu(g) * u with g, u = gu[row] * 2^xs[row] (fp32, exact rescale);
// h[row] = fp16(h * 2^-hs[row]).  h is kept in shared memory between the
// max pass and the store pass.
__global__ void moe_silu_scale(const float* __restrict__ gu, const int32_t* __restrict__ xs,
                               int n_ff, __half* __restrict__ h, int32_t* __restrict__ hs) {
    grid_launch_dependents();  // the next launch may start its prologue
    extern __shared__ float sh[];
    __shared__ float red[32];
    const int row = blockIdx.x;
    const float* g = gu + (int64_t)row * 2 * n_ff;
    const float* u = g + n_ff;
    const float up = exp2i(xs[row]);
    float amax = 0.f;
    for (int i = threadIdx.x; i < n_ff; i += blockDim.x) {
        const float gv = g[i] * up;
        const float v = gv / (1.f + expf(-gv)) * (u[i] * up);
        sh[i] = v;
        amax = fmaxf(amax, fabsf(v));
    }
    const int s = row_scale_exp(block_max(amax, red));
    const float sc = exp2i(-s);
    __half2* dst = reinterpret_cast<__half2*>(h + (int64_t)row * n_ff);
    for (int i = 2 * threadIdx.x; i < n_ff; i += 2 * blockDim.x)
        dst[i >> 1] = __floats2half2_rn(sh[i] * sc, sh[i + 1] * sc);
    if (threadIdx.x == 0) hs[row] = s;
}

// out[t][k] = sum over slots (in expert first-use order) of w * yd[pos][k]
__global__ void moe_combine(const float* __restrict__ yd, const int32_t* __restrict__ hs,
                            const int32_t* __restrict__ pos, const int32_t* __restrict__ idx,
                            const float* __restrict__ wts, const int32_t* __restrict__ rank, int T,
                            int U, int K, float* __restrict__ out) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < (int64_t)T * (K / 4);
         i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t t = i / (K / 4), k4 = i - t * (K / 4);
        int order[kMaxTopK];
        for (int u = 0; u < U; ++u) {  // insertion sort of the slots by expert rank
            int v = u;
            const int ru = rank[idx[t * U + u]];
            while (v > 0 && rank[idx[t * U + order[v - 1]]] > ru) {
                order[v] = order[v - 1];
                --v;
            }
            order[v] = u;
        }
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int j = 0; j < U; ++j) {
            const int u = order[j];
            const float w = wts[t * U + u];
            const int row = pos ? pos[t * U + u] : (int)(t * U + u);
            float4 y = reinterpret_cast<const float4*>(yd + (int64_t)row * K)[k4];
            const float up = hs ? exp2i(hs[row]) : 1.f;  // undo the row scale of h (exact)
            y.x *= up;
            y.y *= up;
            y.z *= up;
            y.w *= up;
            acc.x = __fadd_rn(acc.x, __fmul_rn(w, y.x));
            acc.y = __fadd_rn(acc.y, __fmul_rn(w, y.y));
            acc.z = __fadd_rn(acc.z, __fmul_rn(w, y.z));
            acc.w = __fadd_rn(acc.w, __fmul_rn(w, y.w));
        }
        reinterpret_cast<float4*>(out + t * K)[k4] = acc;
    }
}

// xf = fp32 copy of x (exact for bf16 / fp16)
template <typename TI>
__global__ void moe_to_f32(const TI* __restrict__ x, int64_t n, float* __restrict__ xf) {
    grid_launch_dependents();  // the next launch may start its prologue
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x)
        xf[i] = to_f(x[i]);
}

// h[r][i] = silu(gu[r][i]) * gu[r][n_ff + i], all fp32
__global__ void moe_silu_f32(const float* __restrict__ gu, int rows, int n_ff,
                             float* __restrict__ h) {
    grid_launch_dependents();  // the next launch may start its prologue
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < (int64_t)rows * n_ff;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = i / n_ff, c = i - r * n_ff;
        const float g = gu[r * 2 * n_ff + c];
        h[i] = g / (1.f + expf(-g)) * gu[r * 2 * n_ff + n_ff + c];
    }
}

int grid_for(int64_t n) {
    const int sms = device_sms();
    return (int)std::max<int64_t>(1, std::min<int64_t>((n + 255) / 256, (int64_t)sms * 8));
}

size_t align256(size_t n) { return (n + 255) & ~(size_t)255; }

constexpr int64_t kMaxFf = 49152;  // h row kept in shared memory by moe_silu_scale
constexpr int64_t kFusedSiluMaxFf = 8192;  // decode down GEMV takes silu(gate) * up itself

// Decode (few tokens): every (token, slot) pair is a GEMV over its expert's
// weights, which streams each chosen expert once at HBM speed; the
// tensor-core GEMM pays a fixed cost per 128-row MMA that dominates there.
// (The GEMV covers K up to 15 * 2048.)
bool decode_path(const ftc_moe_desc& d, int64_t T) {
    return T * d.top_k * 2 <= kGemvMaxMats && d.n_embd <= 30720 && d.n_ff <= 30720 &&
           d.gu_row_stride % 16 == 0 &&
           d.dn_row_stride % 16 == 0 && d.gu_plane_stride % 16 == 0 &&
           d.dn_plane_stride % 16 == 0;
}

// Workspace regions, in order (each 256-byte aligned).
struct MoeLayout {
    size_t idx, wts, counts, offsets, rank, pos, row_token, xs, hs, xg, gu, h, yd, total;
};

MoeLayout moe_layout(const ftc_moe_desc& d, int64_t T) {
    const int64_t R = T * d.top_k, E = d.n_experts;
    MoeLayout L;
    size_t o = 0;
    L.idx = o;       o += align256((size_t)R * 4);
    L.wts = o;       o += align256((size_t)R * 4);
    L.counts = o;    o += align256((size_t)E * 4);
    L.offsets = o;   o += align256((size_t)(E + 1) * 4);
    L.rank = o;      o += align256((size_t)E * 4);
    L.pos = o;       o += align256((size_t)R * 4);
    L.row_token = o; o += align256((size_t)R * 4);
    L.xs = o;        o += align256((size_t)R * 4);
    L.hs = o;        o += align256((size_t)R * 4);
    // xg: fp16 rows (GEMM path) or the fp32 tokens (decode path)
    L.xg = o;        o += align256(std::max((size_t)R * 2, (size_t)T * 4) * d.n_embd);
    L.gu = o;        o += align256((size_t)R * 2 * d.n_ff * 4);
    // h: fp16 rows (GEMM path) or fp32 rows (decode path)
    L.h = o;         o += align256((size_t)R * d.n_ff * (decode_path(d, T) ? 4 : 2));
    L.yd = o;        o += align256((size_t)R * d.n_embd * 4);
    L.total = o;
    return L;
}

// routing: the entry routes tokens (top_k must fit n_experts); the expert
// FFN entries on pre-grouped rows ignore top_k (an expert-parallel rank may
// hold fewer experts than the layer's top_k)
int check_desc(const ftc_moe_desc* d, const char* who, bool routing = true) {
    FTC_REQUIRE(d, FTC_E_INVALID, std::string(who) + ": null descriptor");
    FTC_REQUIRE(d->dtype == FTC_Q4_K, FTC_E_UNSUPPORTED,
                std::string(who) + ": expert weights must be Q4_K");
    FTC_REQUIRE(d->n_experts >= 1 && d->n_experts <= kMaxExperts, FTC_E_INVALID,
                std::string(who) + ": need 1 <= n_experts <= 256");
    FTC_REQUIRE(!routing || (d->top_k >= 1 && d->top_k <= kMaxTopK && d->top_k <= d->n_experts),
                FTC_E_INVALID, std::string(who) + ": need 1 <= top_k <= min(8, n_experts) <= 256");
    FTC_REQUIRE(d->n_embd > 0 && d->n_ff > 0 && d->n_embd % 256 == 0 && d->n_ff % 256 == 0 &&
                    d->n_embd <= INT32_MAX && d->n_ff <= kMaxFf,
                FTC_E_INVALID,
                std::string(who) + ": n_embd and n_ff must be multiples of 256, n_ff <= 49152");
    return FTC_OK;
}

}  // namespace

size_t moe_workspace_bytes(const ftc_moe_desc* d, int64_t T) {
    if (check_desc(d, "ftc_moe_workspace_bytes") != FTC_OK || T < 0) return 0;
    return moe_layout(*d, T).total;
}

int moe_ffn(const ftc_moe_desc* d, const float* logits, const void* x, int x_dtype, int64_t T,
            float* out, void* ws, size_t ws_bytes, cudaStream_t st) {
    int rc = check_desc(d, "ftc_moe_ffn");
    if (rc) return rc;
    FTC_REQUIRE(T >= 0 && T * d->top_k <= INT32_MAX / 2, FTC_E_INVALID, "ftc_moe_ffn: bad T");
    if (T == 0) return FTC_OK;
    FTC_REQUIRE(logits && x && out && ws && d->gate_exps && d->up_exps && d->down_exps,
                FTC_E_INVALID, "ftc_moe_ffn: null pointer");
    FTC_REQUIRE(x_dtype == FTC_F32 || x_dtype == FTC_BF16 || x_dtype == FTC_F16,
                FTC_E_UNSUPPORTED, "ftc_moe_ffn: x must be fp32, bf16 or fp16");
    FTC_REQUIRE((uintptr_t)ws % 256 == 0 && (uintptr_t)out % 16 == 0 && (uintptr_t)x % 16 == 0,
                FTC_E_INVALID, "ftc_moe_ffn: x and out need 16-byte, workspace 256-byte alignment");
    const MoeLayout L = moe_layout(*d, T);
    FTC_REQUIRE(ws_bytes >= L.total, FTC_E_INVALID, "ftc_moe_ffn: workspace too small");
    if (inject_fail("ftc_moe_ffn")) return set_error(FTC_E_INJECTED, "ftc_moe_ffn: injected failure");

    uint8_t* w = static_cast<uint8_t*>(ws);
    auto i32 = [&](size_t off) { return reinterpret_cast<int32_t*>(w + off); };
    int32_t *idx = i32(L.idx), *counts = i32(L.counts), *offsets = i32(L.offsets);
    int32_t *rank = i32(L.rank), *pos = i32(L.pos), *row_token = i32(L.row_token);
    int32_t *xs = i32(L.xs), *hs = i32(L.hs);
    float* wts = reinterpret_cast<float*>(w + L.wts);
    __half* xg = reinterpret_cast<__half*>(w + L.xg);
    float* gu = reinterpret_cast<float*>(w + L.gu);
    __half* h = reinterpret_cast<__half*>(w + L.h);
    float* yd = reinterpret_cast<float*>(w + L.yd);
    const int E = (int)d->n_experts, U = (int)d->top_k, K = (int)d->n_embd, F = (int)d->n_ff;
    const int R = (int)(T * U);

    moe_route<<<1, route_threads(T), 0, st>>>(logits, (int)T, E, U, idx, wts, counts, offsets,
                                              rank, pos, row_token);
    FTC_CUDA(cudaGetLastError());
    if (decode_path(*d, T)) {
        // fp32 tokens, then one GEMV launch for gate and up of every (token,
        // slot) pair, SiLU, one GEMV launch for the pairs' down projections
        const float* xf = static_cast<const float*>(x);
        if (x_dtype != FTC_F32) {
            float* dst = reinterpret_cast<float*>(w + L.xg);
            const int64_t n = T * (int64_t)K;
            if (x_dtype == FTC_BF16)
                moe_to_f32<<<grid_for(n), 256, 0, st>>>(static_cast<const __nv_bfloat16*>(x), n, dst);
            else
                moe_to_f32<<<grid_for(n), 256, 0, st>>>(static_cast<const __half*>(x), n, dst);
            FTC_CUDA(cudaGetLastError());
            xf = dst;
        }
        float* h32 = reinterpret_cast<float*>(w + L.h);
        GemvSpec g = {};
        g.P = 2 * R;
        g.K = K;
        g.stride = d->gu_row_stride;
        g.per_matrix_x = T > 1;
        g.sel = idx;
        g.sel_stride = d->gu_plane_stride;
        g.sel_max = E - 1;
        for (int r = 0; r < R; ++r)
            for (int j = 0; j < 2; ++j) {
                const int i = 2 * r + j;
                g.W[i] = static_cast<const uint8_t*>(j ? d->up_exps : d->gate_exps);
                g.N[i] = F;
                g.y[i] = gu + (int64_t)r * 2 * F + (int64_t)j * F;
                g.x[i] = xf + (int64_t)(r / U) * K;
                g.sel_slot[i] = r;
            }
        if ((rc = gemv_q4k_batch(g, st))) return rc;
        // down: for short n_ff the GEMV takes silu(gate) * up from the pair's
        // [gate | up] row as it loads its activation (the same fp32
        // expression as moe_silu_f32), one launch less; for long rows every
        // CTA reading the whole [gate | up] row costs more than the launch
        // (n_ff = 14336: 72 -> 78 us per layer), so moe_silu_f32 runs first
        GemvSpec dn = {};
        dn.P = R;
        dn.K = F;
        dn.stride = d->dn_row_stride;
        dn.per_matrix_x = R > 1;
        dn.sel = idx;
        dn.sel_stride = d->dn_plane_stride;
        dn.sel_max = E - 1;
        dn.x_up = F <= kFusedSiluMaxFf ? F : 0;
        for (int r = 0; r < R; ++r) {
            dn.W[r] = static_cast<const uint8_t*>(d->down_exps);
            dn.N[r] = K;
            dn.y[r] = yd + (int64_t)r * K;
            dn.x[r] = gu + (int64_t)r * 2 * F;
            dn.sel_slot[r] = r;
        }
        rc = dn.x_up ? gemv_q4k_batch(dn, st) : FTC_E_UNSUPPORTED;
        if (rc == FTC_E_UNSUPPORTED) {
            moe_silu_f32<<<grid_for((int64_t)R * F), 256, 0, st>>>(gu, R, F, h32);
            FTC_CUDA(cudaGetLastError());
            dn.x_up = 0;
            for (int r = 0; r < R; ++r) dn.x[r] = h32 + (int64_t)r * F;
            rc = gemv_q4k_batch(dn, st);
        }
        if (rc) return rc;
        moe_combine<<<grid_for((int64_t)T * K / 4), 256, 0, st>>>(yd, nullptr, nullptr, idx, wts,
                                                                  rank, (int)T, U, K, out);
        FTC_CUDA(cudaGetLastError());
        return FTC_OK;
    }
    if (x_dtype == FTC_F32)
        moe_gather_scale<float><<<R, 256, 0, st>>>(static_cast<const float*>(x), row_token, K, xg, xs);
    else if (x_dtype == FTC_BF16)
        moe_gather_scale<__nv_bfloat16><<<R, 256, 0, st>>>(
            static_cast<const __nv_bfloat16*>(x), row_token, K, xg, xs);
    else
        moe_gather_scale<__half><<<R, 256, 0, st>>>(static_cast<const __half*>(x), row_token, K,
                                                    xg, xs);
    FTC_CUDA(cudaGetLastError());
    rc = gemm_q4k_grouped(d->gate_exps, d->up_exps, 2, E, d->gu_plane_stride, F, K,
                          d->gu_row_stride, xg, FTC_F16, R, counts, offsets, T, gu, FTC_F32,
                          2 * (int64_t)F, st);
    if (rc) return rc;
    {
        const size_t smem = (size_t)F * 4;
        if ((rc = opt_in_smem(reinterpret_cast<const void*>(moe_silu_scale), (int)(kMaxFf * 4),
                              "cudaFuncSetAttribute(moe_silu_scale)")))
            return rc;
        moe_silu_scale<<<R, 512, smem, st>>>(gu, xs, F, h, hs);
        FTC_CUDA(cudaGetLastError());
    }
    rc = gemm_q4k_grouped(d->down_exps, nullptr, 1, E, d->dn_plane_stride, K, F, d->dn_row_stride,
                          h, FTC_F16, R, counts, offsets, T, yd, FTC_F32, K, st);
    if (rc) return rc;
    moe_combine<<<grid_for((int64_t)T * K / 4), 256, 0, st>>>(yd, hs, pos, idx, wts, rank, (int)T,
                                                              U, K, out);
    FTC_CUDA(cudaGetLastError());
    return FTC_OK;
}


// Routing and grouping alone (moe_route): outputs as in the kernel's header.
int moe_route_only(const float* logits, int64_t T, int64_t E, int64_t U, int32_t* idx, float* w,
                   int32_t* counts, int32_t* offsets, int32_t* rank, int32_t* pos,
                   int32_t* row_token, cudaStream_t st) {
    FTC_REQUIRE(E >= 1 && E <= kMaxExperts && U >= 1 && U <= kMaxTopK && U <= E, FTC_E_INVALID,
                "ftc_moe_route: need 1 <= top_k <= min(8, n_experts) <= 256");
    FTC_REQUIRE(T >= 0 && T * U <= INT32_MAX / 2, FTC_E_INVALID, "ftc_moe_route: bad T");
    // T == 0 (e.g. an expert-parallel rank without tokens): only the per-expert
    // arrays are written, the per-token ones may be empty (null)
    FTC_REQUIRE(counts && offsets && rank && (T == 0 || (logits && idx && w && pos && row_token)),
                FTC_E_INVALID, "ftc_moe_route: null pointer");
    moe_route<<<1, route_threads(T), 0, st>>>(logits, (int)T, (int)E, (int)U, idx, w, counts,
                                              offsets, rank, pos, row_token);
    FTC_CUDA(cudaGetLastError());
    return FTC_OK;
}

// out[t] = sum over t's slots (in expert first-use order) of w * y[pos]
int moe_combine_only(const float* y, const int32_t* pos, const int32_t* idx, const float* w,
                     const int32_t* rank, int64_t T, int64_t U, int64_t K, float* out,
                     cudaStream_t st) {
    FTC_REQUIRE(T >= 0 && U >= 1 && U <= kMaxTopK && K > 0 && K % 4 == 0 && (uintptr_t)y % 16 == 0 &&
                    (uintptr_t)out % 16 == 0,
                FTC_E_INVALID, "ftc_moe_combine: bad shape or alignment");
    if (T == 0) return FTC_OK;  // nothing to combine (empty arrays may be null)
    FTC_REQUIRE(y && pos && idx && w && rank && out, FTC_E_INVALID, "ftc_moe_combine: null pointer");
    moe_combine<<<grid_for(T * K / 4), 256, 0, st>>>(y, nullptr, pos, idx, w, rank, (int)T, (int)U,
                                                   (int)K, out);
    FTC_CUDA(cudaGetLastError());
    return FTC_OK;
}

// Expert FFNs on rows already grouped by expert (the local half of an
// expert-parallel MoE layer): rows [offsets[e], offsets[e] + counts[e]) of x
// go through expert e of d (gate/up, silu, down) into y (fp32, unscaled).
// counts / offsets: device int32 [E]; rows: total rows; max_rows: bound on
// any count.  Workspace: moe_experts_workspace_bytes.
size_t moe_experts_workspace_bytes(const ftc_moe_desc* d, int64_t rows) {
    if (check_desc(d, "ftc_moe_experts_workspace_bytes", false) != FTC_OK || rows < 0) return 0;
    size_t o = 0;
    o += align256((size_t)rows * 4);                    // xs
    o += align256((size_t)rows * 4);                    // hs
    o += align256((size_t)rows * d->n_embd * 2);        // xg
    o += align256((size_t)rows * 2 * d->n_ff * 4);      // gu
    o += align256((size_t)rows * d->n_ff * 2);          // h
    return o;
}

int moe_experts(const ftc_moe_desc* d, const void* x, int x_dtype, int64_t rows,
                const int32_t* counts, const int32_t* offsets, int64_t max_rows, float* y,
                void* ws, size_t ws_bytes, cudaStream_t st) {
    int rc = check_desc(d, "ftc_moe_experts", false);
    if (rc) return rc;
    FTC_REQUIRE(rows >= 0 && rows <= INT32_MAX / 2 && max_rows >= 0, FTC_E_INVALID,
                "ftc_moe_experts: bad row count");
    if (rows == 0) return FTC_OK;
    FTC_REQUIRE(x && y && ws && counts && offsets && d->gate_exps && d->up_exps && d->down_exps,
                FTC_E_INVALID, "ftc_moe_experts: null pointer");
    FTC_REQUIRE(x_dtype == FTC_F32 || x_dtype == FTC_BF16 || x_dtype == FTC_F16,
                FTC_E_UNSUPPORTED, "ftc_moe_experts: x must be fp32, bf16 or fp16");
    FTC_REQUIRE((uintptr_t)ws % 256 == 0 && (uintptr_t)y % 16 == 0 && (uintptr_t)x % 16 == 0,
                FTC_E_INVALID, "ftc_moe_experts: x and y need 16-byte, workspace 256-byte alignment");
    FTC_REQUIRE(ws_bytes >= moe_experts_workspace_bytes(d, rows), FTC_E_INVALID,
                "ftc_moe_experts: workspace too small");
    const int E = (int)d->n_experts, K = (int)d->n_embd, F = (int)d->n_ff, R = (int)rows;
    uint8_t* w = static_cast<uint8_t*>(ws);
    int32_t* xs = reinterpret_cast<int32_t*>(w);
    w += align256((size_t)R * 4);
    int32_t* hs = reinterpret_cast<int32_t*>(w);
    w += align256((size_t)R * 4);
    __half* xg = reinterpret_cast<__half*>(w);
    w += align256((size_t)R * K * 2);
    float* gu = reinterpret_cast<float*>(w);
    w += align256((size_t)R * 2 * F * 4);
    __half* h = reinterpret_cast<__half*>(w);
    if (x_dtype == FTC_F32)
        moe_gather_scale<float><<<R, 256, 0, st>>>(static_cast<const float*>(x), nullptr, K, xg, xs);
    else if (x_dtype == FTC_BF16)
        moe_gather_scale<__nv_bfloat16><<<R, 256, 0, st>>>(
            static_cast<const __nv_bfloat16*>(x), nullptr, K, xg, xs);
    else
        moe_gather_scale<__half><<<R, 256, 0, st>>>(static_cast<const __half*>(x), nullptr, K, xg, xs);
    FTC_CUDA(cudaGetLastError());
    const int64_t mr = std::max<int64_t>(1, std::min<int64_t>(max_rows, rows));
    rc = gemm_q4k_grouped(d->gate_exps, d->up_exps, 2, E, d->gu_plane_stride, F, K,
                          d->gu_row_stride, xg, FTC_F16, R, counts, offsets, mr, gu, FTC_F32,
                          2 * (int64_t)F, st);
    if (rc) return rc;
    if ((rc = opt_in_smem(reinterpret_cast<const void*>(moe_silu_scale), (int)(kMaxFf * 4),
                          "cudaFuncSetAttribute(moe_silu_scale)")))
        return rc;
    moe_silu_scale<<<R, 512, (size_t)F * 4, st>>>(gu, xs, F, h, hs);
    FTC_CUDA(cudaGetLastError());
    // down projection; the epilogue undoes h's row scales (exact)
    return gemm_q4k_grouped(d->down_exps, nullptr, 1, E, d->dn_plane_stride, K, F,
                            d->dn_row_stride, h, FTC_F16, R, counts, offsets, mr, y, FTC_F32, K,
                            st, hs);
}

}  // namespace ftc
