// peer_ar.cu -- one-shot allreduce of fp32 partials over NVLink peer memory,
// for the small row-parallel outputs of the tensor-parallel block (config 4:
// the [M, n_embd] partials of o and down, 32 KB per rank at M = 1).
//
// The reference has no tensor parallelism (one process runs every matmul of
// ft/src/engine.cpp:485-600); the allreduce is the exchange step the
// row-parallel split adds.  At these sizes an allreduce is all latency, so
// the exchange carries its own completion flags: every fp32 value travels
// with the call's epoch in the same 8-byte word (value bits low, epoch
// high), written with one store, so a reader that sees the epoch also sees
// the value -- no memory fence and no separate flag round trip.
//
// Layout.  Every rank owns one device region, mapped by every other rank
// through a CUDA IPC handle:
//   data  [2 parities][world source ranks + 1][max_elems] u64 (value | epoch << 32);
//         the extra slot holds the owners' sums of a two-shot call
//   ctr   [2] uint32: this rank's call epoch, and the CTAs of the current
//         call that have finished (the last one advances the epoch)
// A call runs kArBlocks CTAs; CTA b owns slice b of the vector.  It
//   1. stores its slice of `in` into slot [parity][rank] of every rank's data
//      (its own included) -- 8-byte stores to peer addresses over NVLink;
//   2. reads its slice of every source slot of its own region, waiting per
//      word until the word carries this call's epoch (bounded in time);
//   3. sums the sources in rank order 0, 1, ... world-1 into `out`.
// Every rank adds the same values in the same order, so all ranks hold the
// same bits.  The epoch counts this rank's calls in device memory (graph
// replays advance it): every CTA of a call reads it once the previous call
// on the stream has completed, and the CTA that finishes last advances it.
// One epoch per call, not per CTA, because a given element is written by
// different CTAs in different kinds of calls (slices here, row chunks in the
// fused GEMV).  The two parities keep a rank that has moved on to the next
// call from overwriting a slot a slower peer is still reading: a rank can
// only be one call ahead, because finishing a call needs every peer's words
// of that call.
//
// A peer that never arrives makes the wait give up after the same bound as
// every other wait of this library (FTC_DEVSTAT_WAIT_TIMEOUT) and the CTA
// returns without writing its slice.
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "common.cuh"
#include "gemv_batch.cuh"
#include "sm100.cuh"

namespace ftc {

FTC_DEVSTAT_READER(devstat_peer_ar)

namespace {

constexpr int kArBlocks = kPeerBlocks;  // one CTA per SM, every call (the call counters are per CTA)
constexpr int kArThreads = 256;
constexpr int kArBatch = 4;     // elements a thread gathers at once
constexpr int kArMaxRanks = kPeerMaxRanks;

struct ArPeers {
    uint64_t* data[kArMaxRanks];  // each rank's data region (this rank's own included)
};

__device__ __forceinline__ void st_word(uint64_t* p, uint64_t v) {
    asm volatile("st.volatile.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ uint64_t ld_word(const uint64_t* p) {
    uint64_t v;
    asm volatile("ld.volatile.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

// Waits (bounded) until the words of elements [lo, hi) from `nsrc` sources
// (source s at d + s * stride) carry `epoch`, then calls emit(i, sum) with the
// sources summed in order.  A thread keeps the loads of kArBatch elements x
// all sources in flight together.  Returns false when the wait gave up.
template <class Emit>
__device__ __forceinline__ bool gather_sum(const uint64_t* d, int nsrc, int64_t stride, int64_t lo,
                                           int64_t hi, uint32_t epoch, volatile int* ok,
                                           Emit emit) {
    uint64_t t0 = 0;
    for (int64_t base = lo + threadIdx.x; base < hi && *ok; base += kArThreads * kArBatch) {
        uint64_t w[kArBatch][kArMaxRanks];
        uint32_t pending = 0;  // bit e * kArMaxRanks + s: word (element e, source s) not seen yet
#pragma unroll
        for (int e = 0; e < kArBatch; ++e)
            if (base + e * kArThreads < hi) pending |= ((1u << nsrc) - 1u) << (e * kArMaxRanks);
        while (pending) {
#pragma unroll
            for (int e = 0; e < kArBatch; ++e)
#pragma unroll
                for (int s = 0; s < kArMaxRanks; ++s)
                    if ((pending >> (e * kArMaxRanks + s)) & 1u)
                        w[e][s] = ld_word(d + s * stride + base + e * kArThreads);
#pragma unroll
            for (int e = 0; e < kArBatch; ++e)
#pragma unroll
                for (int s = 0; s < kArMaxRanks; ++s)
                    if (((pending >> (e * kArMaxRanks + s)) & 1u) && (w[e][s] >> 32) == epoch)
                        pending &= ~(1u << (e * kArMaxRanks + s));
            if (pending) {
                const uint64_t now = global_ns();
                if (t0 == 0) {
                    t0 = now;
                } else if (now - t0 > kWaitLimitNs) {
                    record_timeout();
                    *ok = 0;
                }
                if (!*ok) return false;
            }
        }
#pragma unroll
        for (int e = 0; e < kArBatch; ++e) {
            const int64_t i = base + e * kArThreads;
            if (i >= hi) break;
            float a = __uint_as_float((uint32_t)w[e][0]);
#pragma unroll
            for (int s = 1; s < kArMaxRanks; ++s)
                if (s < nsrc) a += __uint_as_float((uint32_t)w[e][s]);
            emit(i, a);
        }
    }
    return *ok != 0;
}

// One-shot (two_shot == 0): every rank pushes its slice of every element to
// every rank and sums all sources itself.  Two-shot: within each CTA's slice
// [i0, i1), rank o owns the o-th of `world` sub-slices; every rank pushes
// each element only to its owner (slot [par][rank]), the owner sums the
// sources in rank order and pushes the sum to every rank (slot [par][world]),
// and every rank waits for those -- 2 words per element leave a rank instead
// of `world`, for one more NVLink hop.
__global__ void __launch_bounds__(kArThreads)
peer_ar_f32(const __grid_constant__ ArPeers P, int rank, int world, int64_t max_elems,
            const float* __restrict__ in, float* __restrict__ out, int64_t n, int two_shot,
            uint32_t* __restrict__ ctr) {
    const int b = blockIdx.x;
    __shared__ uint32_t s_epoch;
    __shared__ int s_ok;
    if (threadIdx.x == 0) {
        s_epoch = ctr[0] + 1u;  // the previous call on the stream has completed
        s_ok = 1;
    }
    __syncthreads();
    const uint32_t epoch = s_epoch;
    const int par = (int)(epoch & 1u);
    const int64_t i0 = n * b / kArBlocks, i1 = n * (b + 1) / kArBlocks;
    const int64_t pstride = (int64_t)(world + 1) * max_elems;  // slots of one parity
    const int64_t slot = par * pstride + (int64_t)rank * max_elems;
    const uint64_t tag = (uint64_t)epoch << 32;
    const uint64_t* mine = P.data[rank] + par * pstride;
    volatile int* ok = &s_ok;

    if (!two_shot) {
        for (int64_t i = i0 + threadIdx.x; i < i1; i += kArThreads) {
            const uint64_t w = tag | __float_as_uint(in[i]);
            for (int q = 0; q < world; ++q) st_word(P.data[q] + slot + i, w);
        }
        gather_sum(mine, world, max_elems, i0, i1, epoch, ok,
                   [&](int64_t i, float a) { out[i] = a; });
    } else {
        const int64_t len = i1 - i0;
        auto owner_lo = [&](int o) { return i0 + len * o / world; };
        for (int64_t i = i0 + threadIdx.x; i < i1; i += kArThreads) {
            int o = 0;  // owner: the sub-slice holding i
            while (o + 1 < world && owner_lo(o + 1) <= i) ++o;
            st_word(P.data[o] + slot + i, tag | __float_as_uint(in[i]));
        }
        // the owner's sub-slice: sum the sources, push the sum to every rank
        const uint64_t* sumslot = mine + (int64_t)world * max_elems;
        if (gather_sum(mine, world, max_elems, owner_lo(rank), owner_lo(rank + 1), epoch, ok,
                       [&](int64_t i, float a) {
                           const uint64_t w = tag | __float_as_uint(a);
                           for (int q = 0; q < world; ++q)
                               st_word(P.data[q] + par * pstride + (int64_t)world * max_elems + i, w);
                       }))
            gather_sum(sumslot, 1, 0, i0, i1, epoch, ok, [&](int64_t i, float a) { out[i] = a; });
    }
    __syncthreads();
    if (threadIdx.x == 0) peer_call_done(ctr, epoch);
}

}  // namespace

}  // namespace ftc

struct ftc_peer_ar {
    int rank = 0, world = 0, device = 0;
    int64_t max_elems = 0;
    void* base = nullptr;  // this rank's region
    uint32_t* ctr = nullptr;
    void* peer_base[ftc::kArMaxRanks] = {};  // opened IPC mappings (nullptr for self)
    ftc::ArPeers peers = {};
    bool open = false;
};

namespace ftc {

// The buffer of an opened ftc_peer_ar, for kernels that push their partial
// results into it themselves (the fused GEMV + allreduce).
int peer_ar_view(const ftc_peer_ar* ar, PeerView* v) {
    FTC_REQUIRE(ar && ar->open, FTC_E_INVALID, "peer allreduce: ftc_peer_ar_open not called");
    for (int q = 0; q < kPeerMaxRanks; ++q) v->data[q] = q < ar->world ? ar->peers.data[q] : nullptr;
    v->world = ar->world;
    v->rank = ar->rank;
    v->max_elems = ar->max_elems;
    v->ctr = ar->ctr;
    return FTC_OK;
}

}  // namespace ftc

namespace {

size_t region_bytes(int world, int64_t max_elems) {
    // per parity: one slot per source rank + one for the owners' sums (two-shot)
    const size_t data = (size_t)2 * (world + 1) * max_elems * sizeof(uint64_t);
    return ((data + 255) & ~size_t(255)) + ftc::kArBlocks * sizeof(uint32_t);
}

}  // namespace

extern "C" {

int ftc_peer_ar_create(int rank, int world, int64_t max_elems, ftc_peer_ar** out, void* handle) {
    using namespace ftc;
    FTC_REQUIRE(out && handle, FTC_E_INVALID, "ftc_peer_ar_create: null pointer");
    FTC_REQUIRE(world >= 1 && world <= kArMaxRanks && rank >= 0 && rank < world, FTC_E_INVALID,
                "ftc_peer_ar_create: 1..8 ranks, 0 <= rank < world");
    FTC_REQUIRE(max_elems > 0 && max_elems <= ((int64_t)1 << 28), FTC_E_INVALID,
                "ftc_peer_ar_create: max_elems must be in 1..2^28");
    if (inject_fail("ftc_peer_ar_create"))
        return set_error(FTC_E_INJECTED, "ftc_peer_ar_create: injected failure");
    auto* ar = new ftc_peer_ar();
    ar->rank = rank;
    ar->world = world;
    ar->max_elems = max_elems;
    cudaError_t e = cudaGetDevice(&ar->device);
    const size_t bytes = region_bytes(world, max_elems);
    if (e == cudaSuccess) e = cudaMalloc(&ar->base, bytes);
    if (e == cudaSuccess) e = cudaMemset(ar->base, 0, bytes);
    cudaIpcMemHandle_t h;
    if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, ar->base);
    if (e != cudaSuccess) {
        if (ar->base) cudaFree(ar->base);
        delete ar;
        return cuda_error(e, "ftc_peer_ar_create");
    }
    std::memcpy(handle, &h, sizeof(h));
    ar->ctr = reinterpret_cast<uint32_t*>(static_cast<uint8_t*>(ar->base) + bytes -
                                          kArBlocks * sizeof(uint32_t));
    *out = ar;
    return ok();
}

int ftc_peer_ar_open(ftc_peer_ar* ar, const void* handles) {
    using namespace ftc;
    FTC_REQUIRE(ar && handles, FTC_E_INVALID, "ftc_peer_ar_open: null pointer");
    FTC_REQUIRE(!ar->open, FTC_E_INVALID, "ftc_peer_ar_open: already open");
    for (int q = 0; q < ar->world; ++q) {
        void* p = ar->base;
        if (q != ar->rank) {
            cudaIpcMemHandle_t h;
            std::memcpy(&h, static_cast<const uint8_t*>(handles) + q * FTC_IPC_HANDLE_BYTES,
                        sizeof(h));
            const cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
            if (e != cudaSuccess) {
                for (int j = 0; j < q; ++j)
                    if (ar->peer_base[j]) {
                        cudaIpcCloseMemHandle(ar->peer_base[j]);
                        ar->peer_base[j] = nullptr;  // destroy must not close it again
                    }
                return cuda_error(e, "ftc_peer_ar_open: cudaIpcOpenMemHandle");
            }
            ar->peer_base[q] = p;
        }
        ar->peers.data[q] = static_cast<uint64_t*>(p);
    }
    ar->open = true;
    return ok();
}

int64_t ftc_peer_ar_max_elems(const ftc_peer_ar* ar) { return ar ? ar->max_elems : 0; }

int ftc_peer_ar_sum_f32(ftc_peer_ar* ar, const float* in, float* out, int64_t n, void* stream) {
    using namespace ftc;
    FTC_REQUIRE(ar && in && out, FTC_E_INVALID, "ftc_peer_ar_sum_f32: null pointer");
    FTC_REQUIRE(ar->open, FTC_E_INVALID, "ftc_peer_ar_sum_f32: ftc_peer_ar_open not called");
    FTC_REQUIRE(n >= 0 && n <= ar->max_elems, FTC_E_INVALID,
                "ftc_peer_ar_sum_f32: n exceeds the buffer's max_elems");
    if (n == 0) return ok();
    if (inject_fail("ftc_peer_ar_sum_f32"))
        return set_error(FTC_E_INJECTED, "ftc_peer_ar_sum_f32: injected failure");
    // Two-shot once the one-shot's world-fold traffic outweighs the extra hop:
    // from 16384 elements on 4 or more ranks (with 2 ranks both move the same
    // bytes).  FTC_PEER_AR_TWO_SHOT=<elements> overrides the threshold.
    static const int64_t env_min = [] {
        const char* e = std::getenv("FTC_PEER_AR_TWO_SHOT");
        return e ? std::atoll(e) : (int64_t)-1;
    }();
    const int64_t two_min = env_min >= 0 ? env_min : (ar->world > 2 ? 16384 : INT64_MAX);
    const int two_shot = ar->world > 1 && n >= two_min;
    peer_ar_f32<<<kArBlocks, kArThreads, 0, (cudaStream_t)stream>>>(
        ar->peers, ar->rank, ar->world, ar->max_elems, in, out, n, two_shot, ar->ctr);
    FTC_CUDA(cudaGetLastError());
    return ok();
}

int ftc_mul_mat_vec_allreduce(ftc_peer_ar* ar, int dtype, const void* w, int64_t N, int64_t K,
                               int64_t row_stride, const float* x, float* y, void* stream) {
    using namespace ftc;
    FTC_REQUIRE(ar && w && x && y, FTC_E_INVALID, "ftc_mul_mat_vec_allreduce: null pointer");
    FTC_REQUIRE(dtype == FTC_Q4_K, FTC_E_UNSUPPORTED,
                "ftc_mul_mat_vec_allreduce: Q4_K weights only");
    FTC_REQUIRE(N > 0 && K > 0 && K % 256 == 0 && row_stride >= (K / 256) * 144, FTC_E_INVALID,
                "ftc_mul_mat_vec_allreduce: bad shape");
    FTC_REQUIRE(N <= ar->max_elems, FTC_E_INVALID,
                "ftc_mul_mat_vec_allreduce: N exceeds the buffer's max_elems");
    if (inject_fail("ftc_mul_mat_vec_allreduce"))
        return set_error(FTC_E_INJECTED, "ftc_mul_mat_vec_allreduce: injected failure");
    PeerView v;
    int rc = peer_ar_view(ar, &v);
    if (rc) return rc;
    GemvSpec g = {};
    g.P = 1;
    g.K = K;
    g.stride = row_stride;
    g.W[0] = static_cast<const uint8_t*>(w);
    g.N[0] = N;
    g.y[0] = y;
    g.x[0] = x;
    g.peer = &v;
    rc = gemv_q4k_batch(g, (cudaStream_t)stream);
    if (rc == FTC_E_UNSUPPORTED)
        return set_error(rc, "ftc_mul_mat_vec_allreduce: shape or alignment not supported by the "
                             "fused kernel (16-byte aligned rows and x; use ftc_mul_mat_vec + "
                             "ftc_peer_ar_sum_f32)");
    return rc ? rc : ok();
}

int ftc_mul_mat_vec_silu(ftc_peer_ar* ar, int dtype, const void* w, int64_t N, int64_t K,
                         int64_t row_stride, const float* gu, int64_t up_offset, float* y,
                         void* stream) {
    using namespace ftc;
    FTC_REQUIRE(w && gu && y, FTC_E_INVALID, "ftc_mul_mat_vec_silu: null pointer");
    FTC_REQUIRE(dtype == FTC_Q4_K, FTC_E_UNSUPPORTED, "ftc_mul_mat_vec_silu: Q4_K weights only");
    FTC_REQUIRE(N > 0 && K > 0 && K % 256 == 0 && row_stride >= (K / 256) * 144, FTC_E_INVALID,
                "ftc_mul_mat_vec_silu: bad shape");
    FTC_REQUIRE(up_offset >= K && up_offset % 4 == 0, FTC_E_INVALID,
                "ftc_mul_mat_vec_silu: up_offset must be >= K and a multiple of 4");
    FTC_REQUIRE(!ar || N <= ar->max_elems, FTC_E_INVALID,
                "ftc_mul_mat_vec_silu: N exceeds the buffer's max_elems");
    if (inject_fail("ftc_mul_mat_vec_silu"))
        return set_error(FTC_E_INJECTED, "ftc_mul_mat_vec_silu: injected failure");
    PeerView v;
    if (ar) {
        int rc = peer_ar_view(ar, &v);
        if (rc) return rc;
    }
    GemvSpec g = {};
    g.P = 1;
    g.K = K;
    g.stride = row_stride;
    g.W[0] = static_cast<const uint8_t*>(w);
    g.N[0] = N;
    g.y[0] = y;
    g.x[0] = gu;
    g.x_up = up_offset;
    g.peer = ar ? &v : nullptr;
    const int rc = gemv_q4k_batch(g, (cudaStream_t)stream);
    if (rc == FTC_E_UNSUPPORTED)
        return set_error(rc, "ftc_mul_mat_vec_silu: shape or alignment not supported by the "
                             "fused kernel (16-byte aligned rows and gu; use ftc_silu_mul_rows + "
                             "ftc_mul_mat_vec)");
    return rc ? rc : ok();
}

int ftc_peer_ar_destroy(ftc_peer_ar* ar) {
    using namespace ftc;
    if (!ar) return ok();
    cudaError_t first = cudaSuccess;
    for (int q = 0; q < ar->world; ++q)
        if (ar->peer_base[q]) {
            const cudaError_t e = cudaIpcCloseMemHandle(ar->peer_base[q]);
            if (first == cudaSuccess) first = e;
        }
    if (ar->base) {
        const cudaError_t e = cudaFree(ar->base);
        if (first == cudaSuccess) first = e;
    }
    delete ar;
    if (first != cudaSuccess) return cuda_error(first, "ftc_peer_ar_destroy");
    return ok();
}

}  // extern "C"
