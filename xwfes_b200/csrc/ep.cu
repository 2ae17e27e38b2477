// ep.cu -- device-side bookkeeping of the expert-parallel MoE layer (config
// 5, experts split over G GPUs) for an exchange with fixed capacity:
//
// Every rank sends every other rank the same number of rows (cap = this
// rank's maximum token count x top_k), so the all-to-alls use equal splits,
// no split size ever goes to the host and the whole layer can be captured
// in a CUDA graph.  The row order is the reference's grouping of rows by
// expert (Engine::Impl::moe_ffn, ft/src/engine.cpp:179-241, as ftc_moe_route
// produces it); these kernels only move rows between that order and the
// padded exchange layout.
//
//   ep_pack     send[d][i] = x[row_token[off_d + i]] for the i < cnt_d rows
//               routed to rank d (its experts are contiguous in the expert
//               order: off_d / cnt_d are prefix sums of the expert counts);
//               pos_padded[t][u] = the slot d * cap + i that carries token
//               t's u-th row, i.e. where its expert output comes back.
//   ep_regroup  from the received per-(source, local expert) counts: the
//               local experts' row counts and offsets and a permutation of
//               the world * cap received slots that puts the valid rows in
//               expert-major order (source-major within an expert, the
//               order a single GPU would see them) and the padding after
//               them; and its inverse, to send outputs back.
#include "common.cuh"

namespace ftc {
namespace {

constexpr int kEpMaxExperts = 256;

// first row and row count of rank d's experts in the expert-sorted order
__device__ __forceinline__ void rank_span(const int32_t* counts, int El, int d, int& off, int& cnt) {
    off = 0;
    for (int e = 0; e < d * El; ++e) off += counts[e];
    cnt = 0;
    for (int e = d * El; e < (d + 1) * El; ++e) cnt += counts[e];
}

// One CTA per send slot (d, i); 16-byte copies of the row.
__global__ void ep_pack_rows(const uint4* __restrict__ x, int64_t row_vecs,
                             const int32_t* __restrict__ counts, const int32_t* __restrict__ row_token,
                             int El, int cap, uint4* __restrict__ send) {
    const int d = blockIdx.x / cap, i = blockIdx.x - d * cap;
    __shared__ int s_src;
    if (threadIdx.x == 0) {
        int off, cnt;
        rank_span(counts, El, d, off, cnt);
        s_src = i < cnt ? row_token[off + i] : -1;
    }
    __syncthreads();
    const int src = s_src;
    if (src < 0) return;  // padding: never read by the receiver
    const uint4* a = x + (int64_t)src * row_vecs;
    uint4* b = send + (int64_t)blockIdx.x * row_vecs;
    for (int64_t v = threadIdx.x; v < row_vecs; v += blockDim.x) b[v] = a[v];
}

__global__ void ep_pos_padded(const int32_t* __restrict__ idx, const int32_t* __restrict__ pos,
                              const int32_t* __restrict__ counts, int R, int El, int cap,
                              int32_t* __restrict__ out) {
    const int r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= R) return;
    const int d = idx[r] / El;
    int off, cnt;
    rank_span(counts, El, d, off, cnt);
    out[r] = d * cap + (pos[r] - off);
}

// One CTA.  rc[src][e]: rows of local expert e received from rank src, stored
// at slots src * cap + (rows of src's earlier local experts) + i.
__global__ void ep_regroup_kernel(const int32_t* __restrict__ rc, int world, int El, int cap,
                                  int32_t* __restrict__ perm, int32_t* __restrict__ inv,
                                  int32_t* __restrict__ counts, int32_t* __restrict__ offsets) {
    __shared__ int s_rc[kEpMaxExperts];      // [src][e]
    __shared__ int s_base[kEpMaxExperts];    // start of (src, e) within src's slots
    __shared__ int s_dst[kEpMaxExperts];     // first destination of (src, e)
    __shared__ int s_cnt_src[kEpMaxExperts]; // valid rows from src
    __shared__ int s_pad0[kEpMaxExperts];    // first destination of src's padding
    const int n = world * El;
    for (int j = threadIdx.x; j < n; j += blockDim.x) s_rc[j] = max(0, min(rc[j], cap));
    __syncthreads();
    if (threadIdx.x == 0) {
        int total = 0;
        for (int e = 0; e < El; ++e) {
            int c = 0;
            for (int s = 0; s < world; ++s) {
                s_dst[s * El + e] = total + c;
                c += s_rc[s * El + e];
            }
            counts[e] = c;
            offsets[e] = total;
            total += c;
        }
        int pad = total;
        for (int s = 0; s < world; ++s) {
            int b = 0;
            for (int e = 0; e < El; ++e) {
                s_base[s * El + e] = b;
                b += s_rc[s * El + e];
            }
            b = min(b, cap);
            s_cnt_src[s] = b;
            s_pad0[s] = pad;
            pad += cap - b;
        }
    }
    __syncthreads();
    for (int slot = threadIdx.x; slot < world * cap; slot += blockDim.x) {
        const int s = slot / cap, i = slot - s * cap;
        int dst;
        if (i < s_cnt_src[s]) {
            int e = 0;
            while (e + 1 < El && i >= s_base[s * El + e + 1]) ++e;
            dst = s_dst[s * El + e] + (i - s_base[s * El + e]);
        } else {
            dst = s_pad0[s] + (i - s_cnt_src[s]);
        }
        perm[dst] = slot;
        inv[slot] = dst;
    }
}

}  // namespace

int ep_pack(const void* x, int x_dtype, int64_t T, int64_t n_embd, const int32_t* idx,
            const int32_t* counts, const int32_t* pos, const int32_t* row_token, int64_t n_experts,
            int64_t top_k, int64_t world, int64_t cap, void* send, int32_t* pos_padded,
            cudaStream_t st) {
    FTC_REQUIRE(counts && send && (T == 0 || (x && idx && pos && row_token && pos_padded)),
                FTC_E_INVALID, "ftc_ep_pack: null pointer");
    FTC_REQUIRE(x_dtype == FTC_F32 || x_dtype == FTC_BF16 || x_dtype == FTC_F16,
                FTC_E_UNSUPPORTED, "ftc_ep_pack: x must be fp32, bf16 or fp16");
    FTC_REQUIRE(world >= 1 && n_experts >= 1 && n_experts <= kEpMaxExperts && n_experts % world == 0,
                FTC_E_INVALID, "ftc_ep_pack: experts must split evenly over 1..256 ranks");
    FTC_REQUIRE(T >= 0 && top_k >= 1 && cap >= T * top_k && world * cap <= INT32_MAX,
                FTC_E_INVALID, "ftc_ep_pack: capacity below T * top_k");
    const int64_t es = x_dtype == FTC_F32 ? 4 : 2;
    FTC_REQUIRE(n_embd > 0 && (n_embd * es) % 16 == 0 && (uintptr_t)x % 16 == 0 &&
                    (uintptr_t)send % 16 == 0,
                FTC_E_INVALID, "ftc_ep_pack: rows must be 16-byte multiples, 16-byte aligned");
    const int El = (int)(n_experts / world);
    if (world * cap > 0)
        ep_pack_rows<<<(int)(world * cap), 128, 0, st>>>(
            static_cast<const uint4*>(x), n_embd * es / 16, counts, row_token, El, (int)cap,
            static_cast<uint4*>(send));
    const int R = (int)(T * top_k);
    if (R > 0) ep_pos_padded<<<(R + 255) / 256, 256, 0, st>>>(idx, pos, counts, R, El, (int)cap, pos_padded);
    FTC_CUDA(cudaGetLastError());
    return FTC_OK;
}

int ep_regroup(const int32_t* recv_counts, int64_t world, int64_t n_local, int64_t cap,
               int32_t* perm, int32_t* inv, int32_t* counts, int32_t* offsets, cudaStream_t st) {
    FTC_REQUIRE(recv_counts && perm && inv && counts && offsets, FTC_E_INVALID,
                "ftc_ep_regroup: null pointer");
    FTC_REQUIRE(world >= 1 && n_local >= 1 && world * n_local <= kEpMaxExperts && cap >= 0 &&
                    world * cap <= INT32_MAX,
                FTC_E_INVALID, "ftc_ep_regroup: world * n_local must be in 1..256");
    ep_regroup_kernel<<<1, 1024, 0, st>>>(recv_counts, (int)world, (int)n_local, (int)cap, perm, inv,
                                         counts, offsets);
    FTC_CUDA(cudaGetLastError());
    return FTC_OK;
}

}  // namespace ftc
