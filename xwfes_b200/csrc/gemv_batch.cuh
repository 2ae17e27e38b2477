// gemv_batch.cuh -- host description of a batched Q4_K decode GEMV launch
// (gemv_q4k.cu), shared with the MoE decode path (moe.cu).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace ftc {

constexpr int kGemvMaxMats = 8;

// P matrices with the same K and row pitch in one launch:
//   y_p[n] = sum_k x_p[k] * W_p[n][k]
// x_p = x[0] for every p unless per_matrix_x.  With sel set, matrix p with
// sel_slot[p] >= 0 starts at W[p] + sel[sel_slot[p]] * sel_stride (expert
// ids read on the device after the preceding kernel, clamped to [0, sel_max]).
// A peer allreduce buffer as the kernels see it (see peer_ar.cu): every
// rank's data region ([2 parities][world + 1][max_elems] words of fp32 value
// | epoch << 32), this rank's call epoch and finished-CTA count.
constexpr int kPeerMaxRanks = 8;
constexpr int kPeerBlocks = 148;
struct PeerView {
    uint64_t* data[kPeerMaxRanks];
    int world, rank;
    int64_t max_elems;
    uint32_t* ctr;  // [0] epoch of the last completed call, [1] CTAs done in this call
};

// Called once per CTA at the end of a call: the last CTA to finish makes
// `epoch` the last completed call and resets the count for the next call.
__device__ __forceinline__ void peer_call_done(uint32_t* ctr, uint32_t epoch) {
    if (atomicAdd(&ctr[1], 1u) == gridDim.x - 1) {
        ctr[1] = 0;
        ctr[0] = epoch;
    }
}

struct GemvSpec {
    int P;
    int64_t K, stride;
    const uint8_t* W[kGemvMaxMats];
    int64_t N[kGemvMaxMats];
    float* y[kGemvMaxMats];
    const float* x[kGemvMaxMats];
    int per_matrix_x;
    const int32_t* sel;
    int64_t sel_stride;
    int sel_max;
    int sel_slot[kGemvMaxMats];
    // Prefetch hint: the weight regions the NEXT launch on the stream reads,
    // in the order it reads them (its first chunks first).  After issuing its
    // own last copy, every CTA prefetches its share of their first
    // kGemvPrefetchWindow bytes into L2, so the next launch starts on L2 hits
    // while this one drains.
    int pf_n;
    const uint8_t* pf_ptr[kGemvMaxMats];
    int64_t pf_len[kGemvMaxMats];
    // Allreduce over a tensor-parallel group (one matrix, y the sum over the
    // ranks of their partial products): nullptr for a plain GEMV.
    const PeerView* peer;
    // 0: x is the activation.  > 0: x holds a [gate | up] row, up at
    // x + x_up floats (a multiple of 4), and the activation is
    // silu_gate(gate[k], up[k]) -- the SiLU product folded into the
    // activation load, bit for bit what a separate silu kernel would give.
    int64_t x_up;
    // Weight format: 0 Q4_K; kGemvQ6K / kGemvQ80: Q6_K super-blocks (210
    // bytes) / Q8_0 blocks (34 bytes), one matrix per x, no allreduce, no
    // SiLU activation, no expert selection.
    int wfmt;
};

constexpr int kGemvQ6K = 1;
constexpr int kGemvQ80 = 2;

constexpr int64_t kGemvPrefetchWindow = 24ll << 20;

// FTC_E_UNSUPPORTED when the shape or alignment does not fit the kernel.
int gemv_q4k_batch(const GemvSpec& g, cudaStream_t st);

}  // namespace ftc
