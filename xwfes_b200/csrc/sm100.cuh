// sm100.cuh -- thin inline-PTX wrappers for the sm_100a features the kernels
// use: mbarriers with bounded waits, bulk (TMA) copies, tensor-map loads,
// and the tcgen05 tensor-memory / MMA instructions.  Every copy is issued
// for the calling CTA alone.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace ftc {

// Device-side status word, one per translation unit (no relocatable device
// code): kernels that give up on a bounded wait record FTC_DEVSTAT_* here
// (first writer wins) and return.  Each unit defines a host reader with
// FTC_DEVSTAT_READER; ftc_device_status() polls them all.
enum : int { FTC_DEVSTAT_OK = 0, FTC_DEVSTAT_WAIT_TIMEOUT = 1 };
static __device__ int g_dev_status = 0;

#define FTC_DEVSTAT_READER(fn)                                                   \
    int fn(int clear) {                                                          \
        int v = 0;                                                               \
        if (cudaMemcpyFromSymbol(&v, g_dev_status, sizeof(int)) != cudaSuccess)  \
            return -1;                                                           \
        if (clear && v) {                                                        \
            const int z = 0;                                                     \
            if (cudaMemcpyToSymbol(g_dev_status, &z, sizeof(int)) != cudaSuccess) \
                return -1;                                                       \
        }                                                                        \
        return v;                                                                \
    }

// A wait that has not completed after this many nanoseconds of wall time is
// declared stuck (a legitimate wait in these kernels lasts microseconds).
constexpr uint64_t kWaitLimitNs = 2000000000ull;

__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void mbar_fence_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// The same test, but a thread whose phase is not complete yet may sleep for
// up to `suspend_ns` (it wakes when the phase completes): for warps that wait
// long (a whole tile) and would otherwise take issue slots from the warps
// doing the work.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t* bar, uint32_t parity,
                                                    uint32_t suspend_ns) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "r"(suspend_ns)
        : "memory");
    return ok != 0;
}

__device__ __forceinline__ void record_timeout() {
    atomicCAS(&g_dev_status, FTC_DEVSTAT_OK, FTC_DEVSTAT_WAIT_TIMEOUT);
}

// Single-thread wait for the phase with the given parity.  Returns false
// (and records FTC_DEVSTAT_WAIT_TIMEOUT) after kWaitLimitNs.
// suspend_ns > 0: sleep between tests (see mbar_try_wait_sleep).
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity,
                                          uint32_t suspend_ns = 0) {
    uint64_t t0 = 0;
    for (uint32_t i = 0;; ++i) {
        if (suspend_ns ? mbar_try_wait_sleep(bar, parity, suspend_ns) : mbar_try_wait(bar, parity))
            return true;
        if ((i & 255u) == 255u) {
            const uint64_t now = global_ns();
            if (t0 == 0) {
                t0 = now;
            } else if (now - t0 > kWaitLimitNs) {
                record_timeout();
                return false;
            }
        }
    }
}

// Whole-warp wait: every lane polls (so every lane acquires the phase), the
// decision to stop is warp-uniform, and lane 0 owns the time limit.
__device__ __forceinline__ bool mbar_wait_warp(uint64_t* bar, uint32_t parity,
                                               uint32_t suspend_ns = 0) {
    const int lane = threadIdx.x & 31;
    uint64_t t0 = 0;
    for (uint32_t i = 0;; ++i) {
        const bool done = suspend_ns ? mbar_try_wait_sleep(bar, parity, suspend_ns)
                                     : mbar_try_wait(bar, parity);
        if (__all_sync(0xffffffffu, done)) return true;
        if ((i & 255u) == 255u) {
            int late = 0;
            if (lane == 0) {
                const uint64_t now = global_ns();
                if (t0 == 0) t0 = now;
                else late = (now - t0 > kWaitLimitNs);
            }
            if (__shfl_sync(0xffffffffu, late, 0)) {
                if (lane == 0) record_timeout();
                return false;
            }
        }
    }
}

// ------------------------------------------------------------ bulk copies

// Global -> shared bulk copy of `bytes` (multiple of 16; both addresses
// 16-byte aligned), completing on `bar` by transaction count.
__device__ __forceinline__ void bulk_g2s(void* dst_smem, const void* src, uint32_t bytes,
                                         uint64_t* bar, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1], %2, [%3], %4;" ::"r"(smem_u32(dst_smem)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}

// Pull [src, src + bytes) into L2 without a destination (16-byte aligned,
// bytes a multiple of 16).
__device__ __forceinline__ void bulk_prefetch_l2(const void* src, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

// L2 policy for data read exactly once (streamed weights).
__device__ __forceinline__ uint64_t policy_evict_first() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}

__device__ __forceinline__ uint64_t policy_evict_last() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
    return p;
}

// 2-D tiled tensor-map load for this CTA: box at (x, y) -> dst_smem.
__device__ __forceinline__ void tma_load_2d(void* dst_smem, const CUtensorMap* map, int x, int y,
                                            uint64_t* bar, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        ".L2::cache_hint [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(smem_u32(dst_smem)),
        "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}

__device__ __forceinline__ void tma_load_3d(void* dst_smem, const CUtensorMap* map, int x, int y,
                                            int z, uint64_t* bar, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        ".L2::cache_hint [%0], [%1, {%2, %3, %4}], [%5], %6;" ::"r"(smem_u32(dst_smem)),
        "l"(map), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}

__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(map) : "memory");
}

// Make generic-proxy shared-memory writes visible to the async proxy
// (tensor cores / TMA) before signalling them.
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void named_barrier(int id, int threads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// ------------------------------------------------------------ PDL

// Programmatic dependent launch: wait for the preceding grid's memory to be
// visible (no-op without a programmatic dependency) ...
__device__ __forceinline__ void grid_dependency_wait() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
}
// ... and let the next grid start its prologue.
__device__ __forceinline__ void grid_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ------------------------------------------------------------ tcgen05

__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(dst_smem)),
                 "r"(ncols)
                 : "memory");
}

__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
                 : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem desc] * B[smem desc]^T, kind::f16 (fp16/bf16 in, fp32
// accumulate), issued by one thread.
__device__ __forceinline__ void umma_f16_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                            uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// The same with A read from tensor memory: a_tmem addresses lane 0 of the
// M x 16 operand (row m in lane m, two consecutive k per 32-bit column).
__device__ __forceinline__ void umma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                            uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// 32 lanes x 8 consecutive 32-bit columns of TMEM <- 8 registers per thread
// (the warp's lane quadrant); completes at tmem_st_wait.
__device__ __forceinline__ void tmem_st_32x32b_x8(uint32_t taddr, const uint32_t (&r)[8]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
        : "memory");
}

__device__ __forceinline__ void tmem_st_wait() {
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// Arrive on `bar` once every tcgen05.mma issued so far by this thread is done.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     smem_u32(bar))
                 : "memory");
}

// 32 lanes x 32 consecutive 32-bit columns of TMEM -> 32 registers per thread.
__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
        "%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
          "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
          "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
          "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld_wait() {
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Shared-memory matrix descriptor for a K-major tile in the 128-byte swizzle
// layout (rows of 128 B, 8-row groups 1024 B apart), tcgen05 format:
// start address >> 4 in bits 0-13, leading byte offset (unused for this
// layout, 1) in 16-29, stride byte offset 1024 >> 4 in 32-45, version 1 in
// 46-47, layout SWIZZLE_128B (2) in 61-63.
__device__ __forceinline__ uint64_t smem_desc_k_sw128(const void* tile) {
    const uint64_t addr = smem_u32(tile);
    uint64_t d = 0;
    d |= (addr >> 4) & 0x3FFFull;
    d |= 1ull << 16;
    d |= (uint64_t)(1024 >> 4) << 32;
    d |= 1ull << 46;
    d |= 2ull << 61;
    return d;
}

// Instruction descriptor, kind::f16: fp32 accumulate, A and B of the same
// 16-bit type (0 = f16, 1 = bf16), both K-major, M x N tile.
__host__ __device__ constexpr uint32_t idesc_f16(uint32_t ab_format, uint32_t M, uint32_t N) {
    return (1u << 4)                 // D format: f32
           | (ab_format << 7)        // A format
           | (ab_format << 10)       // B format
           | ((N >> 3) << 17)        // N / 8
           | ((M >> 4) << 24);       // M / 16
}

}  // namespace ftc
