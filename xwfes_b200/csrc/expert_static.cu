// expert_static.cu -- the expert chunk with library-owned scratch, for
// callers that cannot allocate device memory.
//
// ftc_backend_run_expert_chunk allocates (and grows) staging and scratch
// buffers on first use.  Some callers cannot allow that: an engine that has
// handed a fixed slice of HBM to its own allocator, code running between the
// begin and end of someone else's stream capture, or a host runtime that
// forbids cudaMalloc on its serving thread.  ftc_expert_chunk_static runs
// the same kernels on device buffers the caller owns and keeps its
// intermediate activations (gate, up and silu(gate)*up: 3 x M x IC floats)
// in one file-scope __device__ array of fixed size, so it never allocates.
//
// Limits and sharing:
//   * M * IC must not exceed FTC_EXPERT_STATIC_MAX_HC (65536); larger calls
//     are rejected with FTC_E_INVALID before anything is launched.
//   * Every GPU that loads the library holds the 768 KB array until the
//     process exits.
//   * All calls on a device share the array and it keeps the previous call's
//     contents.  Every element a call reads is written by that call first
//     (the GEMVs fill gate/up, silu_mul fills h), so nothing is cleared; calls
//     that overlap on the GPU (different streams, no ordering) race on it.
//   * The first call on each device looks up the array's device address with
//     cudaGetSymbolAddress (with that device current) and caches it; make
//     that first call before any stream capture.  The cached address belongs
//     to the device's primary context: after cudaDeviceReset (which destroys
//     that context and the array with it) do not call this entry again in
//     the same process.
#include <mutex>

#include "common.cuh"

namespace ftc {

int expert_chunk_dev(int dtype, const float* x, float* out, const void* gate, const void* up,
                     const void* down, int64_t M, int64_t K, int64_t IC, int64_t gu_stride,
                     int64_t dn_stride, float* gbuf, float* ubuf, float* hbuf, cudaStream_t st);

namespace {

constexpr int64_t kMaxHC = FTC_EXPERT_STATIC_MAX_HC;

// gate | up | h, kMaxHC floats each.  In host code this name is only a
// handle for cudaGetSymbolAddress, never a device address.
static __device__ __align__(256) float g_expert_scratch[3 * kMaxHC];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
float* g_addr[kMaxDevices] = {};

// Device address of g_expert_scratch on the current device (looked up once).
int scratch_on_current_device(float** out) {
    int dev = 0;
    FTC_CUDA(cudaGetDevice(&dev));
    FTC_REQUIRE(dev >= 0 && dev < kMaxDevices, FTC_E_UNSUPPORTED,
                "ftc_expert_chunk_static: device ordinal out of range");
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g_addr[dev]) {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_expert_scratch);
        if (e != cudaSuccess) return cuda_error(e, "cudaGetSymbolAddress(g_expert_scratch)");
        g_addr[dev] = static_cast<float*>(p);
    }
    *out = g_addr[dev];
    return FTC_OK;
}

}  // namespace
}  // namespace ftc

using namespace ftc;

extern "C" int ftc_expert_chunk_static(int dtype, const float* x, float* out, const void* gate,
                                       const void* up, const void* down, int64_t M, int64_t K,
                                       int64_t IC, int64_t gate_up_row_stride,
                                       int64_t down_row_stride, void* stream) {
    if (IC <= 0 || M <= 0 || K <= 0) return ok();  // nothing to add, as the reference
    const Fmt f = fmt_of(dtype);
    FTC_REQUIRE(f.block_elems > 0, FTC_E_UNSUPPORTED, "ftc_expert_chunk_static: unknown dtype");
    FTC_REQUIRE(x && out && gate && up && down, FTC_E_INVALID,
                "ftc_expert_chunk_static: null pointer");
    FTC_REQUIRE(K % f.block_elems == 0, FTC_E_INVALID,
                "ftc_expert_chunk_static: K must be a whole number of blocks");
    const int64_t rb = row_bytes(dtype, K);
    FTC_REQUIRE(gate_up_row_stride >= rb && down_row_stride >= rb, FTC_E_INVALID,
                "ftc_expert_chunk_static: stride smaller than a row");
    FTC_REQUIRE(M <= kMaxHC && IC <= kMaxHC && M * IC <= kMaxHC, FTC_E_INVALID,
                "ftc_expert_chunk_static: M * IC exceeds FTC_EXPERT_STATIC_MAX_HC (65536); "
                "split the window or use ftc_backend_run_expert_chunk");
    if (inject_fail("ftc_expert_chunk_static"))
        return set_error(FTC_E_INJECTED, "ftc_expert_chunk_static: injected failure");
    float* s = nullptr;
    int rc = scratch_on_current_device(&s);
    if (rc) return rc;
    rc = expert_chunk_dev(dtype, x, out, gate, up, down, M, K, IC, gate_up_row_stride,
                          down_row_stride, s, s + kMaxHC, s + 2 * kMaxHC, (cudaStream_t)stream);
    return rc ? rc : ok();
}
