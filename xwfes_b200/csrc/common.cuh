// common.cuh -- shared helpers of libftcuda.so: status plumbing, load
// intrinsics and the per-format block decoders used by every kernel.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "../../include/ftc.h"

namespace ftc {

// ------------------------------------------------------------ status

// Records `msg` as this thread's last error and returns `code`.
int set_error(int code, const std::string& msg);
int cuda_error(cudaError_t e, const char* what);
int ok();

#define FTC_CUDA(call)                                            \
    do {                                                          \
        cudaError_t e_ = (call);                                  \
        if (e_ != cudaSuccess) return ::ftc::cuda_error(e_, #call); \
    } while (0)

#define FTC_REQUIRE(cond, code, msg)                              \
    do {                                                          \
        if (!(cond)) return ::ftc::set_error((code), (msg));      \
    } while (0)

// Multiprocessor count of the current device (cached per device).
int device_sms();

// Lets kernel `fn` use `bytes` of dynamic shared memory on the current
// device.  The attribute belongs to the device's context, so it is set once
// per (kernel, device, size), not once per process.
int opt_in_smem(const void* fn, int bytes, const char* what);

// Host-side fault injection: when the environment variable FTC_INJECT_FAIL
// names an entry point (or "all"), that entry point returns FTC_E_INJECTED
// before launching anything.  Used by the failure-path tests; no GPU fault.
bool inject_fail(const char* entry);

// ------------------------------------------------------------ formats

struct Fmt {
    int block_elems;
    int block_bytes;
};

inline Fmt fmt_of(int dtype) {
    switch (dtype) {
        case FTC_F32: return {1, 4};
        case FTC_F16: case FTC_BF16: return {1, 2};
        case FTC_Q4_0: return {32, 18};
        case FTC_Q4_1: return {32, 20};
        case FTC_Q8_0: return {32, 34};
        case FTC_Q4_K: return {256, 144};
        case FTC_Q6_K: return {256, 210};
        default: return {0, 0};
    }
}

inline int64_t row_bytes(int dtype, int64_t k) {
    Fmt f = fmt_of(dtype);
    if (f.block_elems == 0) return -1;
    return (k + f.block_elems - 1) / f.block_elems * f.block_bytes;
}

// ------------------------------------------------------------ loads

// 16-byte streaming load of weight bytes: read-only path, not kept in L1
// (L1 holds the activations every warp re-reads).
__device__ __forceinline__ uint4 ld_stream16(const void* p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

__device__ __forceinline__ float h2f(uint32_t bits16) {
    return __half2float(__ushort_as_half((unsigned short)(bits16 & 0xFFFFu)));
}

__device__ __forceinline__ float bf2f(uint32_t bits16) {
    return __uint_as_float((bits16 & 0xFFFFu) << 16);
}

__device__ __forceinline__ uint32_t ld_u16(const uint8_t* p) {
    return (uint32_t)p[0] | ((uint32_t)p[1] << 8);
}

// ------------------------------------------------------------ Q4_K scales

// Scale and min of sub-block j (0..7) from the 12 packed bytes, held as
// three little-endian words s0 = bytes 0-3, s1 = bytes 4-7, s2 = bytes 8-11.
// Sub-blocks 0..3: low 6 bits of byte j (scale) and byte j+4 (min).
// Sub-blocks 4..7: nibbles of byte j+4 (scale low, min high) plus the top
// two bits of bytes j-4 (scale) and j (min).
__device__ __forceinline__ void q4k_scale_min(uint32_t s0, uint32_t s1, uint32_t s2, int j,
                                              int& sc, int& mn) {
    if (j < 4) {
        sc = (s0 >> (8 * j)) & 63;
        mn = (s1 >> (8 * j)) & 63;
    } else {
        const int i = j - 4;
        const uint32_t b = (s2 >> (8 * i)) & 0xFF;
        sc = (int)((b & 0x0F) | (((s0 >> (8 * i + 6)) & 3) << 4));
        mn = (int)((b >> 4) | (((s1 >> (8 * i + 6)) & 3) << 4));
    }
}

// ------------------------------------------------------------ element decode

// Weight j of a row (generic, one element at a time).  Used by the generic
// kernels that cover every format and any alignment; the fast kernels decode
// whole vectors instead.  Bit-exact with ft::dequant_row
// (ft/include/ft/quant.h:10-84) and with the GGUF K-quant formulas: every
// product is exact in fp32, so fused or unfused evaluation agree.
__device__ __forceinline__ float decode_elem(int dtype, const uint8_t* row, int64_t j) {
    switch (dtype) {
        case FTC_F32: {
            const uint8_t* p = row + 4 * j;
            uint32_t u = (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) |
                         ((uint32_t)p[3] << 24);
            return __uint_as_float(u);
        }
        case FTC_F16: return h2f(ld_u16(row + 2 * j));
        case FTC_BF16: return bf2f(ld_u16(row + 2 * j));
        case FTC_Q8_0: {
            const uint8_t* b = row + (j >> 5) * 34;
            return h2f(ld_u16(b)) * (float)(int8_t)b[2 + (j & 31)];
        }
        case FTC_Q4_0: {  // reference layout: weight i in byte i>>1, odd i high nibble
            const uint8_t* b = row + (j >> 5) * 18;
            const int i = (int)(j & 31);
            const uint8_t byte = b[2 + (i >> 1)];
            const int nib = (i & 1) ? (byte >> 4) : (byte & 0xF);
            return h2f(ld_u16(b)) * (float)(nib - 8);
        }
        case FTC_Q4_1: {  // reference layout: w = h0 + h1 * nib
            const uint8_t* b = row + (j >> 5) * 20;
            const int i = (int)(j & 31);
            const uint8_t byte = b[4 + (i >> 1)];
            const int nib = (i & 1) ? (byte >> 4) : (byte & 0xF);
            return h2f(ld_u16(b)) + h2f(ld_u16(b + 2)) * (float)nib;
        }
        case FTC_Q4_K: {
            const uint8_t* b = row + (j >> 8) * 144;
            const int i = (int)(j & 255);
            const int g = i >> 6, hi = (i >> 5) & 1, l = i & 31;
            const uint8_t* s = b + 4;
            uint32_t s0 = s[0] | (s[1] << 8) | (s[2] << 16) | ((uint32_t)s[3] << 24);
            uint32_t s1 = s[4] | (s[5] << 8) | (s[6] << 16) | ((uint32_t)s[7] << 24);
            uint32_t s2 = s[8] | (s[9] << 8) | (s[10] << 16) | ((uint32_t)s[11] << 24);
            int sc, mn;
            q4k_scale_min(s0, s1, s2, 2 * g + hi, sc, mn);
            const uint8_t byte = b[16 + 32 * g + l];
            const int q = hi ? (byte >> 4) : (byte & 0xF);
            const float dl = h2f(ld_u16(b)) * (float)sc;
            const float ml = h2f(ld_u16(b + 2)) * (float)mn;
            return __fsub_rn(__fmul_rn(dl, (float)q), ml);
        }
        case FTC_Q6_K: {
            const uint8_t* b = row + (j >> 8) * 210;
            const int i = (int)(j & 255);
            const int half = i >> 7, r = i & 127;
            const int quad = r >> 5, l = r & 31;  // quad: 0..3 -> weights l, l+32, l+64, l+96
            const uint8_t* ql = b + 64 * half;
            const uint8_t* qh = b + 128 + 32 * half;
            const int8_t* sc = (const int8_t*)(b + 192 + 8 * half);
            const uint8_t lb = ql[l + ((quad & 1) ? 32 : 0)];
            const int low = (quad & 2) ? (lb >> 4) : (lb & 0xF);
            const int high = (qh[l] >> (2 * quad)) & 3;
            const int q = (low | (high << 4)) - 32;
            const float d = h2f(ld_u16(b + 208));
            return __fmul_rn(d * (float)sc[(l >> 4) + 2 * quad], (float)q);
        }
        default: return 0.f;
    }
}

// ------------------------------------------------------------ activation

// silu(g) * u = g / (1 + exp(-g)) * u in fp32, the reference's expert FFN
// activation (ft/src/cpu_backend.cpp:127); every kernel that applies it uses
// this one expression, so fused and separate evaluations give the same bits.
__device__ __forceinline__ float silu_gate(float g, float u) { return g / (1.f + expf(-g)) * u; }

}  // namespace ftc
