/*
 * ftoracle.c -- CPU restatement of the reference's GGUF dequant-matmul path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker for the CUDA path and
 * the "port" CPU baseline; nothing in the product library links or calls it.
 * Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg may
 * load it.
 *
 * Reference: Dark-hub-cat/xwfes, project ft-igpu-src (cited as ft/...).
 *   - block decoders:  ft/include/ft/quant.h:10-84 (F32/F16/BF16/Q8_0/Q4_0/Q4_1)
 *   - dot product:     ft/include/ft/quant.h:86-103 (dot_row_f32)
 *   - fp16 helpers:    ft/include/ft/types.h:60-117
 *   - row-parallel matmul: ft/src/cpu_backend.cpp:39-58, 90-104
 *   - expert chunk:    ft/src/cpu_backend.cpp:106-149
 *   - MoE routing:     ft/src/engine.cpp:62-72 (softmax), 179-241 (moe_ffn)
 *   - attention:       ft/src/engine.cpp:137-177 (Engine::Impl::attn), 43-60 and
 *                      545-551 (RoPE)
 *
 * Q4_K and Q6_K do not exist in the reference (ft/include/ft/types.h:20-27,
 * ft/src/gguf.cpp:129-137).  Their decoders below are written from the
 * published GGUF block-format description (super-blocks of 256 weights) and
 * are pinned against golden vectors produced by the GGUF format's own Python
 * package (gguf-py 0.19.0), see tests/golden/gen_golden.py.
 *
 * Compile with -ffp-contract=off: the reference is built for generic x86-64
 * (no FMA), so every product and sum below is rounded separately, in the
 * order written, exactly as the reference's loops round them.
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include "ftoracle.h"

/* ---------------------------------------------------------------- fp16 */

/* ft/include/ft/types.h:60-82: bit-exact fp16 -> fp32 incl. subnormals. */
float ftor_half_to_float(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t ex = (h >> 10) & 0x1Fu;
    uint32_t man = h & 0x3FFu;
    uint32_t bits;
    if (ex == 0) {
        if (man == 0) {
            bits = sign;
        } else {
            /* normalise the subnormal: shift until the implicit bit appears */
            /* value = man * 2^-24; after `shifts` left shifts the leading one
             * sits at bit 10, so the value is 1.frac * 2^(-14 - shifts). */
            int shifts = 0;
            while (!(man & 0x400u)) { man <<= 1; ++shifts; }
            man &= 0x3FFu;
            bits = sign | ((uint32_t)(127 - 14 - shifts) << 23) | (man << 13);
        }
    } else if (ex == 31) {
        bits = sign | 0x7F800000u | (man << 13);
    } else {
        bits = sign | ((ex - 15 + 127) << 23) | (man << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

/* ft/include/ft/types.h:84-111: fp32 -> fp16, round to nearest even.  Used
 * only by generators that build quant blocks, as the reference tests do
 * (ft/src/tests/test_core.cpp:250,262,279). */
uint16_t ftor_float_to_half(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    uint32_t sign = (x >> 16) & 0x8000u;
    int32_t ex = (int32_t)((x >> 23) & 0xFFu) - 127 + 15;
    uint32_t man = x & 0x007FFFFFu;
    if (((x >> 23) & 0xFFu) == 0xFF) return (uint16_t)(sign | 0x7C00u | (man ? 0x200u : 0));
    if (ex >= 31) return (uint16_t)(sign | 0x7C00u);
    if (ex <= 0) {
        if (ex < -10) return (uint16_t)sign;
        man |= 0x00800000u;
        int shift = 14 - ex;
        uint32_t hm = man >> shift;
        uint32_t rem = man & ((1u << shift) - 1u);
        uint32_t halfway = 1u << (shift - 1);
        if (rem > halfway || (rem == halfway && (hm & 1u))) hm++;
        return (uint16_t)(sign | hm);
    }
    uint32_t hr = man >> 13;
    uint32_t rem = man & 0x1FFFu;
    if (rem > 0x1000u || (rem == 0x1000u && (hr & 1u))) hr++;
    /* As in the reference, the rounded mantissa is OR-ed (not added) into
     * the exponent field, so a rounding carry is lost when ex is odd. */
    return (uint16_t)(sign | ((uint32_t)ex << 10) | hr);
}

static float bf16_to_float(uint16_t b) {
    uint32_t bits = (uint32_t)b << 16;
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

static uint16_t rd16(const uint8_t* p) { return (uint16_t)(p[0] | (p[1] << 8)); }

/* ------------------------------------------------------- block geometry */

int64_t ftor_block_elems(int dtype) {
    switch (dtype) {
        case FTOR_Q4_0: case FTOR_Q4_1: case FTOR_Q8_0: return 32;
        case FTOR_Q4_K: case FTOR_Q6_K: return 256;
        case FTOR_F32: case FTOR_F16: case FTOR_BF16: return 1;
        default: return -1;
    }
}

int64_t ftor_block_bytes(int dtype) {
    switch (dtype) {
        case FTOR_F32: return 4;
        case FTOR_F16: case FTOR_BF16: return 2;
        case FTOR_Q4_0: return 18;
        case FTOR_Q4_1: return 20;
        case FTOR_Q8_0: return 34;
        case FTOR_Q4_K: return 144;
        case FTOR_Q6_K: return 210;
        default: return -1;
    }
}

/* ft/include/ft/types.h:51-55 (dtype_row_bytes): whole blocks per row. */
int64_t ftor_row_bytes(int dtype, int64_t n_cols) {
    int64_t eb = ftor_block_elems(dtype), bb = ftor_block_bytes(dtype);
    if (eb <= 0) return -1;
    return ((n_cols + eb - 1) / eb) * bb;
}

/* --------------------------------------------------------- K-quant scales */

/* Q4_K: 12 packed bytes hold eight 6-bit scales and eight 6-bit mins.
 * Sub-blocks 0..3 keep their values in the low 6 bits of bytes j (scale) and
 * j+4 (min); sub-blocks 4..7 keep their low 4 bits in the nibbles of byte j+4
 * (scale low, min high) and their top 2 bits in the top 2 bits of bytes j-4
 * (scale) and j (min). */
static void q4k_scale_min(const uint8_t* sc12, int j, int* sc, int* mn) {
    if (j < 4) {
        *sc = sc12[j] & 63;
        *mn = sc12[j + 4] & 63;
    } else {
        *sc = (sc12[j + 4] & 0x0F) | ((sc12[j - 4] >> 6) << 4);
        *mn = (sc12[j + 4] >> 4) | ((sc12[j] >> 6) << 4);
    }
}

/* Q4_K super-block (144 B): fp16 d, fp16 dmin, 12 B scales, 128 B codes.
 * Codes: 4 groups of 32 bytes; group g holds sub-block 2g in the low nibbles
 * and sub-block 2g+1 in the high nibbles, byte l giving weight l of each.
 * w = (d*sc)*q - (dmin*m).  d*sc, dmin*m and (d*sc)*q are exact in fp32
 * (11+6+4 significant bits), so only the final subtraction rounds. */
static void dequant_q4k_block(float* y, const uint8_t* b) {
    const float d = ftor_half_to_float(rd16(b));
    const float dmin = ftor_half_to_float(rd16(b + 2));
    const uint8_t* sc12 = b + 4;
    const uint8_t* qs = b + 16;
    for (int g = 0; g < 4; ++g) {
        int s0, m0, s1, m1;
        q4k_scale_min(sc12, 2 * g, &s0, &m0);
        q4k_scale_min(sc12, 2 * g + 1, &s1, &m1);
        const float d0 = d * (float)s0, n0 = dmin * (float)m0;
        const float d1 = d * (float)s1, n1 = dmin * (float)m1;
        for (int l = 0; l < 32; ++l) {
            y[64 * g + l] = d0 * (float)(qs[32 * g + l] & 0x0F) - n0;
            y[64 * g + 32 + l] = d1 * (float)(qs[32 * g + l] >> 4) - n1;
        }
    }
}

/* Q6_K super-block (210 B): 128 B low nibbles (ql), 64 B high 2-bit pairs
 * (qh), 16 int8 sub-block scales (one per 16 weights), fp16 d.
 * Each half of 128 weights uses 64 B of ql and 32 B of qh; within a half,
 * byte l (<32) of qh carries the top 2 bits of weights l, l+32, l+64, l+96
 * (bits 0-1, 2-3, 4-5, 6-7); ql byte l gives the low nibbles of weights l
 * (low nibble) and l+64 (high nibble), ql byte l+32 those of l+32 and l+96.
 * w = (d*sc)*(q-32), exact in fp32 (11+7+5 significant bits). */
static void dequant_q6k_block(float* y, const uint8_t* b) {
    const uint8_t* ql = b;
    const uint8_t* qh = b + 128;
    const int8_t* sc = (const int8_t*)(b + 192);
    const float d = ftor_half_to_float(rd16(b + 208));
    for (int half = 0; half < 2; ++half) {
        const uint8_t* l4 = ql + 64 * half;
        const uint8_t* h2 = qh + 32 * half;
        const int8_t* s = sc + 8 * half;
        float* o = y + 128 * half;
        for (int l = 0; l < 32; ++l) {
            const int q0 = (int)((l4[l] & 0x0F) | (((h2[l] >> 0) & 3) << 4)) - 32;
            const int q1 = (int)((l4[l + 32] & 0x0F) | (((h2[l] >> 2) & 3) << 4)) - 32;
            const int q2 = (int)((l4[l] >> 4) | (((h2[l] >> 4) & 3) << 4)) - 32;
            const int q3 = (int)((l4[l + 32] >> 4) | (((h2[l] >> 6) & 3) << 4)) - 32;
            const int is = l / 16;
            o[l] = (d * (float)s[is + 0]) * (float)q0;
            o[l + 32] = (d * (float)s[is + 2]) * (float)q1;
            o[l + 64] = (d * (float)s[is + 4]) * (float)q2;
            o[l + 96] = (d * (float)s[is + 6]) * (float)q3;
        }
    }
}

/* ------------------------------------------------------------- dequant */

/* ft/include/ft/quant.h:10-84 (dequant_row) for the reference's own formats,
 * extended with Q4_K / Q6_K.  Note the reference's Q4_0/Q4_1 layouts: weight
 * j of a block sits in byte j>>1, odd j in the high nibble (quant.h:52-54),
 * and Q4_1 stores (base, step) as w = h0 + h1*nib (quant.h:64-75). */
int ftor_dequant_row(float* dst, const uint8_t* src, int dtype, int64_t n) {
    switch (dtype) {
        case FTOR_F32:
            memcpy(dst, src, (size_t)n * 4);
            return 0;
        case FTOR_F16:
            for (int64_t i = 0; i < n; ++i) dst[i] = ftor_half_to_float(rd16(src + 2 * i));
            return 0;
        case FTOR_BF16:
            for (int64_t i = 0; i < n; ++i) dst[i] = bf16_to_float(rd16(src + 2 * i));
            return 0;
        case FTOR_Q8_0: { /* quant.h:31-44 */
            const int64_t nb = (n + 31) / 32;
            for (int64_t b = 0; b < nb; ++b) {
                const uint8_t* p = src + b * 34;
                const float d = ftor_half_to_float(rd16(p));
                const int64_t base = b * 32;
                const int64_t cnt = (n - base) < 32 ? (n - base) : 32;
                for (int64_t j = 0; j < cnt; ++j) dst[base + j] = d * (float)(int8_t)p[2 + j];
            }
            return 0;
        }
        case FTOR_Q4_0: { /* quant.h:45-61 */
            const int64_t nb = (n + 31) / 32;
            for (int64_t b = 0; b < nb; ++b) {
                const uint8_t* p = src + b * 18;
                const float d = ftor_half_to_float(rd16(p));
                const int64_t base = b * 32;
                const int64_t cnt = (n - base) < 32 ? (n - base) : 32;
                for (int64_t j = 0; j < cnt; ++j) {
                    const uint8_t byte = p[2 + (j >> 1)];
                    const int nib = (j & 1) ? ((byte >> 4) & 0xF) : (byte & 0xF);
                    dst[base + j] = d * (float)(nib - 8);
                }
            }
            return 0;
        }
        case FTOR_Q4_1: { /* quant.h:62-79 */
            const int64_t nb = (n + 31) / 32;
            for (int64_t b = 0; b < nb; ++b) {
                const uint8_t* p = src + b * 20;
                const float h0 = ftor_half_to_float(rd16(p));
                const float h1 = ftor_half_to_float(rd16(p + 2));
                const int64_t base = b * 32;
                const int64_t cnt = (n - base) < 32 ? (n - base) : 32;
                for (int64_t j = 0; j < cnt; ++j) {
                    const uint8_t byte = p[4 + (j >> 1)];
                    const int nib = (j & 1) ? ((byte >> 4) & 0xF) : (byte & 0xF);
                    dst[base + j] = h0 + h1 * (float)nib;
                }
            }
            return 0;
        }
        case FTOR_Q4_K:
        case FTOR_Q6_K: {
            if (n % 256) return -2; /* K-quant rows are whole super-blocks */
            const int64_t bb = ftor_block_bytes(dtype);
            for (int64_t b = 0; b < n / 256; ++b) {
                if (dtype == FTOR_Q4_K) dequant_q4k_block(dst + 256 * b, src + bb * b);
                else dequant_q6k_block(dst + 256 * b, src + bb * b);
            }
            return 0;
        }
        default:
            return -1;
    }
}

/* ft/include/ft/quant.h:86-103 (dot_row_f32): dequantize 2048-element chunks
 * and accumulate x[i]*w[i] sequentially into one fp32 running sum. */
float ftor_dot_row_f32(const float* x, const uint8_t* w, int dtype, int64_t n) {
    if (dtype == FTOR_F32) {
        const float* wf = (const float*)w;
        float acc = 0.f;
        for (int64_t i = 0; i < n; ++i) acc += x[i] * wf[i];
        return acc;
    }
    float buf[2048];
    float acc = 0.f;
    for (int64_t i = 0; i < n;) {
        const int64_t chunk = (n - i) < 2048 ? (n - i) : 2048;
        if (ftor_dequant_row(buf, w + ftor_row_bytes(dtype, i), dtype, chunk) != 0) return NAN;
        for (int64_t j = 0; j < chunk; ++j) acc += x[i + j] * buf[j];
        i += chunk;
    }
    return acc;
}

/* ---------------------------------------------------------- threading */

/* ft/src/cpu_backend.cpp:39-58 (parallel_for): static contiguous split of n
 * items over at most min(threads, n, 256) threads, created per call. */
typedef void (*range_fn)(void* ctx, int64_t b, int64_t e);
struct range_job { range_fn fn; void* ctx; int64_t b, e; };

static void* range_thread(void* p) {
    struct range_job* j = (struct range_job*)p;
    j->fn(j->ctx, j->b, j->e);
    return NULL;
}

static void parallel_for(int64_t n, int threads, range_fn fn, void* ctx) {
    if (n <= 0) return;
    int nt = threads > 0 ? threads : 1;
    if (nt > 256) nt = 256;
    if (nt > n) nt = (int)n;
    if (nt == 1) { fn(ctx, 0, n); return; }
    const int64_t chunk = (n + nt - 1) / nt;
    pthread_t tid[256];
    struct range_job jobs[256];
    int started = 0;
    for (int t = 1; t < nt; ++t) {
        const int64_t b = t * chunk;
        if (b >= n) break;
        jobs[t].fn = fn; jobs[t].ctx = ctx; jobs[t].b = b;
        jobs[t].e = (b + chunk < n) ? b + chunk : n;
        if (pthread_create(&tid[t], NULL, range_thread, &jobs[t]) != 0) {
            fn(ctx, jobs[t].b, jobs[t].e); /* run inline if no thread */
            tid[t] = 0;
        }
        started = t;
    }
    fn(ctx, 0, chunk < n ? chunk : n);
    for (int t = 1; t <= started; ++t)
        if (tid[t]) pthread_join(tid[t], NULL);
}

/* ------------------------------------------------------------- matmul */

struct mm_ctx {
    const float* x; int64_t M, K, N; const uint8_t* W; int64_t stride; int dtype; float* y;
};

static void mm_rows(void* p, int64_t b, int64_t e) {
    struct mm_ctx* c = (struct mm_ctx*)p;
    for (int64_t r = b; r < e; ++r) {
        const uint8_t* wrow = c->W + c->stride * r;
        for (int64_t m = 0; m < c->M; ++m)
            c->y[m * c->N + r] = ftor_dot_row_f32(c->x + m * c->K, wrow, c->dtype, c->K);
    }
}

/* ft/src/cpu_backend.cpp:90-104 (CpuBackend::matmul) with the intended
 * per-row semantics y[m][n] = dot(x_m, W_n).  The reference folds all M rows
 * into y[n] (a bug for M>1); at M=1 both agree bit for bit. */
int ftor_matmul(const float* x, int64_t M, int64_t K, const uint8_t* W, int dtype,
                int64_t N, int64_t row_stride, float* y, int threads) {
    if (ftor_block_elems(dtype) <= 0) return -1;
    if (row_stride <= 0) row_stride = ftor_row_bytes(dtype, K);
    struct mm_ctx c = {x, M, K, N, W, row_stride, dtype, y};
    parallel_for(N, threads, mm_rows, &c);
    return 0;
}

/* --------------------------------------------------------- expert chunk */

static float silu_ref(float g) { return g / (1.f + expf(-g)); }

struct ph_a_ctx {
    const float* x; int64_t K, IC; const uint8_t* gate; const uint8_t* up;
    int64_t gu_stride; int dtype; float* h;
};

static void phase_a(void* p, int64_t b, int64_t e) {
    struct ph_a_ctx* c = (struct ph_a_ctx*)p;
    for (int64_t idx = b; idx < e; ++idx) {
        const int64_t m = idx / c->IC, i = idx % c->IC;
        float g = ftor_dot_row_f32(c->x + m * c->K, c->gate + c->gu_stride * i, c->dtype, c->K);
        const float u = ftor_dot_row_f32(c->x + m * c->K, c->up + c->gu_stride * i, c->dtype, c->K);
        g = silu_ref(g);
        c->h[idx] = g * u;
    }
}

struct ph_b_ctx {
    const float* h; int64_t M, K, IC; const uint8_t* down; int64_t dn_stride; int dtype;
    float* out; int err;
};

static void phase_b(void* p, int64_t kb, int64_t ke) {
    struct ph_b_ctx* c = (struct ph_b_ctx*)p;
    float* row = (float*)malloc((size_t)c->K * sizeof(float));
    if (!row) { c->err = 1; return; }
    for (int64_t m = 0; m < c->M; ++m) {
        const float* hm = c->h + m * c->IC;
        float* om = c->out + m * c->K;
        for (int64_t i = 0; i < c->IC; ++i) {
            ftor_dequant_row(row, c->down + c->dn_stride * i, c->dtype, c->K);
            const float v = hm[i];
            if (v == 0.f) continue;
            for (int64_t k = kb; k < ke; ++k) om[k] += v * row[k];
        }
    }
    free(row);
}

/* ft/src/cpu_backend.cpp:106-149 (CpuBackend::run_expert_chunk).
 * Phase A: h[m,i] = silu(x_m . gate_i) * (x_m . up_i).
 * Phase B: out[m,k] += sum_i h[m,i] * down[i][k]  (the reference's
 * neuron-major down layout: IC rows of K weights).  `out` accumulates. */
int ftor_expert_chunk(const float* x, float* out, const uint8_t* gate, const uint8_t* up,
                      const uint8_t* down, int dtype, int64_t M, int64_t K, int64_t IC,
                      int64_t gu_stride, int64_t dn_stride, int threads) {
    if (IC <= 0 || M <= 0 || K <= 0) return 0;
    if (ftor_block_elems(dtype) <= 0) return -1;
    float* h = (float*)malloc((size_t)(M * IC) * sizeof(float));
    if (!h) return -3;
    struct ph_a_ctx a = {x, K, IC, gate, up, gu_stride, dtype, h};
    parallel_for(M * IC, threads, phase_a, &a);
    struct ph_b_ctx bctx = {h, M, K, IC, down, dn_stride, dtype, out, 0};
    parallel_for(K, threads, phase_b, &bctx);
    free(h);
    return bctx.err ? -3 : 0;
}

/* ft/src/cpu_backend.cpp:60-75 (ft::matmul_down_axpy, the engine's dense
 * and shared-expert down projection, ft/src/engine.cpp:256, 275):
 * y[m][j] += x[m][i] * W_i[j] for i < n_in in ascending order, rows with
 * x[m][i] == 0 skipped; W_i = row i of N weights.  Every y[m][j] sees the
 * same sequence of separately rounded products and sums as the reference's
 * single-threaded loop, so the column split over threads changes no bit. */
int ftor_matmul_down_axpy(const float* x, int64_t M, int64_t n_in, const uint8_t* W, int dtype,
                          int64_t N, int64_t row_stride, float* y, int threads) {
    if (ftor_block_elems(dtype) <= 0) return -1;
    if (M <= 0 || n_in <= 0 || N <= 0) return 0;
    if (row_stride <= 0) row_stride = ftor_row_bytes(dtype, N);
    struct ph_b_ctx c = {x, M, N, n_in, W, row_stride, dtype, y, 0};
    parallel_for(N, threads, phase_b, &c);
    return c.err ? -3 : 0;
}

/* Standard GGUF layout for the down projection (ffn_down rows = outputs):
 * out[m][o] += dot(h_m, down_o) over n_ff.  Phase A is the reference's
 * (cpu_backend.cpp:115-130); phase B is its matmul (cpu_backend.cpp:90-104)
 * applied to h with per-row semantics. */
int ftor_expert_ffn(const float* x, float* out, const uint8_t* gate, const uint8_t* up,
                    const uint8_t* down, int dtype, int64_t M, int64_t K, int64_t n_ff,
                    int64_t gu_stride, int64_t dn_stride, int threads) {
    if (n_ff <= 0 || M <= 0 || K <= 0) return 0;
    if (ftor_block_elems(dtype) <= 0) return -1;
    float* h = (float*)malloc((size_t)(M * n_ff) * sizeof(float));
    float* y = (float*)malloc((size_t)(M * K) * sizeof(float));
    if (!h || !y) { free(h); free(y); return -3; }
    struct ph_a_ctx a = {x, K, n_ff, gate, up, gu_stride, dtype, h};
    parallel_for(M * n_ff, threads, phase_a, &a);
    ftor_matmul(h, M, n_ff, down, dtype, K, dn_stride, y, threads);
    for (int64_t i = 0; i < M * K; ++i) out[i] += y[i];
    free(h);
    free(y);
    return 0;
}

/* ------------------------------------------------------------ routing */

/* ft/src/engine.cpp:62-72 (softmax_inplace): float exps, double sum. */
static void softmax_inplace(float* p, int64_t n) {
    float mx = p[0];
    for (int64_t i = 1; i < n; ++i) mx = p[i] > mx ? p[i] : mx;
    double sum = 0;
    for (int64_t i = 0; i < n; ++i) {
        p[i] = expf(p[i] - mx);
        sum += p[i];
    }
    const float inv = (float)(1.0 / sum);
    for (int64_t i = 0; i < n; ++i) p[i] *= inv;
}

/* ft/src/engine.cpp:198-215: optional bias, softmax over all E, top-U by
 * probability, renormalise the U chosen weights by their float sum.
 * std::partial_sort leaves ties in unspecified order; here ties go to the
 * lower expert index.  Writes idx[T][U] and w[T][U]. */
int ftor_route_topk(const float* logits, const float* bias, int64_t T, int64_t E, int64_t U,
                    int32_t* idx, float* w) {
    if (E <= 0 || U <= 0 || U > E || E > 1024) return -1;
    float r[1024];
    for (int64_t m = 0; m < T; ++m) {
        for (int64_t j = 0; j < E; ++j) r[j] = logits[m * E + j] + (bias ? bias[j] : 0.f);
        softmax_inplace(r, E);
        int32_t* id = idx + m * U;
        for (int64_t u = 0; u < U; ++u) {
            int64_t best = -1;
            for (int64_t j = 0; j < E; ++j) {
                int taken = 0;
                for (int64_t v = 0; v < u; ++v) taken |= (id[v] == j);
                if (taken) continue;
                if (best < 0 || r[j] > r[best]) best = j;
            }
            id[u] = (int32_t)best;
        }
        float wsum = 0.f;
        for (int64_t u = 0; u < U; ++u) wsum += r[id[u]];
        const float inv = wsum > 0 ? 1.f / wsum : 0.f;
        for (int64_t u = 0; u < U; ++u) w[m * U + u] = r[id[u]] * inv;
    }
    return 0;
}

/* ft/src/engine.cpp:179-241 (moe_ffn) for the routed experts: route, gather
 * each used expert's tokens in first-use order, run the expert FFN on them
 * (standard down layout), and add w * expert_out into out[m] in the same
 * expert order.  Expert e's tensors start at base + e * plane_bytes. */
int ftor_moe_ffn(const float* x, const float* logits, int64_t T, int64_t K, int64_t n_ff,
                 int64_t E, int64_t U, const uint8_t* gate_exps, const uint8_t* up_exps,
                 const uint8_t* down_exps, int dtype, float* out, int threads) {
    if (T <= 0) return 0;
    const int64_t gu_stride = ftor_row_bytes(dtype, K);
    const int64_t dn_stride = ftor_row_bytes(dtype, n_ff);
    const int64_t gu_plane = gu_stride * n_ff, dn_plane = dn_stride * K;
    int32_t* idx = (int32_t*)malloc((size_t)(T * U) * sizeof(int32_t));
    float* w = (float*)malloc((size_t)(T * U) * sizeof(float));
    int64_t* order = (int64_t*)malloc((size_t)E * sizeof(int64_t));
    int64_t* list = (int64_t*)malloc((size_t)(T * U) * sizeof(int64_t));
    float* xe = (float*)malloc((size_t)(T * K) * sizeof(float));
    float* acb = (float*)malloc((size_t)(T * K) * sizeof(float));
    int rc = (idx && w && order && list && xe && acb) ? 0 : -3;
    if (!rc) rc = ftor_route_topk(logits, NULL, T, E, U, idx, w);
    int64_t n_used = 0;
    if (!rc) {
        for (int64_t m = 0; m < T; ++m)
            for (int64_t u = 0; u < U; ++u) {
                int64_t e = idx[m * U + u], seen = 0;
                for (int64_t k = 0; k < n_used; ++k) seen |= (order[k] == e);
                if (!seen) order[n_used++] = e;
            }
    }
    for (int64_t oi = 0; !rc && oi < n_used; ++oi) {
        const int64_t e = order[oi];
        int64_t S = 0;
        for (int64_t m = 0; m < T; ++m)
            for (int64_t u = 0; u < U; ++u)
                if (idx[m * U + u] == e) list[S++] = m * U + u;
        for (int64_t s = 0; s < S; ++s) memcpy(xe + s * K, x + (list[s] / U) * K, (size_t)K * 4);
        memset(acb, 0, (size_t)(S * K) * 4);
        rc = ftor_expert_ffn(xe, acb, gate_exps + gu_plane * e, up_exps + gu_plane * e,
                             down_exps + dn_plane * e, dtype, S, K, n_ff, gu_stride, dn_stride,
                             threads);
        for (int64_t s = 0; !rc && s < S; ++s) {
            const float wgt = w[list[s]];
            float* trow = out + (list[s] / U) * K;
            const float* arow = acb + s * K;
            for (int64_t j = 0; j < K; ++j) trow[j] += wgt * arow[j];
        }
    }
    free(idx); free(w); free(order); free(list); free(xe); free(acb);
    return rc;
}

/* ---------------------------------------------------------- attention */

/* ft/src/engine.cpp:62-72 (softmax_inplace): max, exp of the shifted
 * scores in float, their sum in double, one float reciprocal applied. */
static void softmax_ref(float* p, int64_t n) {
    float mx = p[0];
    for (int64_t i = 1; i < n; ++i) mx = p[i] > mx ? p[i] : mx;
    double sum = 0;
    for (int64_t i = 0; i < n; ++i) {
        p[i] = expf(p[i] - mx);
        sum += p[i];
    }
    const float inv = (float)(1.0 / sum);
    for (int64_t i = 0; i < n; ++i) p[i] *= inv;
}

struct attn_ctx {
    const float *q, *kc, *vc, *kb, *vb;
    float* out;
    int64_t nh, gqa, hd, dk, base;
    float scale;
};

/* ft/src/engine.cpp:137-177 (Engine::Impl::attn), one (row, head) item:
 * causal length base + m + 1; positions below base from the cache, the rest
 * from the current block; scores d * scale with d summed in k order;
 * output summed in position order, positions of weight zero skipped. */
static void attn_items(void* vctx, int64_t b, int64_t e) {
    const struct attn_ctx* c = (const struct attn_ctx*)vctx;
    float* sc = NULL;
    int64_t cap = 0;
    for (int64_t idx = b; idx < e; ++idx) {
        const int64_t m = idx / c->nh, h = idx % c->nh, kvh = h / c->gqa;
        const float* qs = c->q + (m * c->nh + h) * c->hd;
        const int64_t len = c->base + m + 1;
        if (len > cap) {
            free(sc);
            sc = (float*)malloc((size_t)len * sizeof(float));
            cap = len;
            if (!sc) return;
        }
        for (int64_t p = 0; p < len; ++p) {
            const float* kp = (p < c->base ? c->kc + p * c->dk : c->kb + (p - c->base) * c->dk) +
                              kvh * c->hd;
            float d = 0.f;
            for (int64_t t = 0; t < c->hd; ++t) d += qs[t] * kp[t];
            sc[p] = d * c->scale;
        }
        softmax_ref(sc, len);
        float* o = c->out + (m * c->nh + h) * c->hd;
        for (int64_t t = 0; t < c->hd; ++t) o[t] = 0.f;
        for (int64_t p = 0; p < len; ++p) {
            const float w = sc[p];
            if (w == 0.f) continue;
            const float* vp = (p < c->base ? c->vc + p * c->dk : c->vb + (p - c->base) * c->dk) +
                              kvh * c->hd;
            for (int64_t t = 0; t < c->hd; ++t) o[t] += w * vp[t];
        }
    }
    free(sc);
}

int ftor_attention(const float* q, int64_t M, int64_t n_head, int64_t n_head_kv,
                   int64_t head_dim, const float* k_cache, const float* v_cache, int64_t base,
                   const float* k_blk, const float* v_blk, float* out, int threads) {
    if (M <= 0 || n_head <= 0 || n_head_kv <= 0 || head_dim <= 0 || n_head % n_head_kv || base < 0)
        return -1;
    struct attn_ctx c = {q, k_cache, v_cache, k_blk, v_blk, out, n_head, n_head / n_head_kv,
                         head_dim, n_head_kv * head_dim, base,
                         1.f / sqrtf((float)head_dim)};
    parallel_for(M * n_head, threads, attn_items, &c);
    return 0;
}

/* ft/src/engine.cpp:43-60 (rope_vec): frequency and angle in double, cos and
 * sin rounded to float, the rotation in float (pairs (i, i + hd/2) for NeoX,
 * (2i, 2i + 1) otherwise). */
void ftor_rope_vec(float* v, int64_t hd, int64_t pos, double theta, int neox) {
    for (int64_t i = 0; i < hd / 2; ++i) {
        const double f = pow(theta, -2.0 * (double)i / (double)hd);
        const double ang = (double)pos * f;
        const float c = (float)cos(ang);
        const float s = (float)sin(ang);
        const int64_t i0 = neox ? i : 2 * i, i1 = neox ? i + hd / 2 : 2 * i + 1;
        const float a = v[i0], b = v[i1];
        v[i0] = a * c - b * s;
        v[i1] = a * s + b * c;
    }
}

/* ft/src/engine.cpp:545-551: every head of rows m = 0..M-1 at position
 * base + m; x is [M][heads][hd]. */
int ftor_rope(float* x, int64_t M, int64_t heads, int64_t hd, int64_t base, double theta,
              int neox) {
    if (M < 0 || heads <= 0 || hd <= 0 || hd % 2) return -1;
    for (int64_t m = 0; m < M; ++m)
        for (int64_t h = 0; h < heads; ++h)
            ftor_rope_vec(x + (m * heads + h) * hd, hd, base + m, theta, neox);
    return 0;
}
