/*
 * ftc.h -- C ABI of libftcuda.so, the B200 (sm_100a) GGUF dequant-matmul
 * backend.  Plain pointers and sizes only; every function returns an int
 * status (FTC_OK = 0) and ftc_last_error() describes the last failure on the
 * calling thread.
 *
 * Two layers:
 *   1. ftc_backend_*  -- one backend instance = one device + one stream +
 *      a weight cache.  These take HOST buffers, copy inputs in and results
 *      out, and return with the results complete on the host: the contract
 *      of the reference's operator interface ft::IBackend
 *      (ft/include/ft/backend.h:21-40).  A C++ ft::IBackend adapter over
 *      these lives in xwfes_b200/host/cuda_backend.{h,cpp}.
 *   2. ftc_* kernel entry points -- DEVICE pointers, launched on the given
 *      cudaStream_t (passed as void*), asynchronous, no allocation.
 *
 * Weight layout everywhere: GGUF blocks exactly as the loader produces them
 * (ft::HostTensor, ft/include/ft/types.h:119-140): W[n][k] is n rows of
 * row_stride bytes, each row ceil(k / block) whole blocks along k.
 */
#ifndef FTC_H
#define FTC_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------ status */
#define FTC_OK 0
#define FTC_E_INVALID (-1)     /* bad argument: null pointer, shape, stride, alignment */
#define FTC_E_UNSUPPORTED (-2) /* dtype / shape combination not implemented */
#define FTC_E_CUDA (-3)        /* CUDA runtime error (message has the CUDA text) */
#define FTC_E_NOMEM (-4)       /* device or pinned host allocation failed */
#define FTC_E_INJECTED (-5)    /* host-side fault injection (FTC_INJECT_FAIL) fired */
#define FTC_E_DEVICE (-6)      /* a kernel reported a bounded wait that ran out */

/* ------------------------------------------------------------ dtypes */
/* The reference's ft::DType values (ft/include/ft/types.h:20-27) plus the
 * GGUF type ids of Q4_K and Q6_K, which its loader rejects
 * (ft/src/gguf.cpp:129-137). */
enum ftc_dtype {
    FTC_F32 = 0,
    FTC_F16 = 1,
    FTC_Q4_0 = 2,
    FTC_Q4_1 = 3,
    FTC_Q8_0 = 8,
    FTC_Q4_K = 12,
    FTC_Q6_K = 14,
    FTC_BF16 = 30
};

/* Message of the last failing call on this thread ("" if none). */
const char* ftc_last_error(void);
/* ABI version, bumped on incompatible changes. */
int ftc_abi_version(void);
/* Bytes of one row of k weights of `dtype` (whole blocks), or -1. */
int64_t ftc_row_bytes(int dtype, int64_t k);

/* ============================================================ backend */

typedef struct ftc_backend ftc_backend;

/* Replaces constructing a backend (ft::CpuBackend / ft::VulkanBackend,
 * ft/src/cpu_backend.cpp:77-86, ft/src/vulkan_backend.cpp:128-277): binds
 * `device`, creates its stream and pinned staging.  On failure *out is NULL
 * and the engine keeps its CPU backend (ft/src/engine.cpp:291-300). */
int ftc_backend_create(int device, ftc_backend** out);
void ftc_backend_destroy(ftc_backend* be);

/* ft::IBackend::name() / info() (ft/include/ft/types.h:142-147 DeviceInfo):
 * device name into `name` (NUL-terminated, truncated to cap) and its total
 * memory.  integrated/uma are always false for a B200. */
int ftc_backend_info(ftc_backend* be, char* name, size_t cap, uint64_t* mem_bytes);

/* Upload a GGUF tensor's raw blocks to HBM once (Engine::load time,
 * ft/src/engine.cpp:318-382).  The cache is keyed by the host address range
 * [host, host + nbytes); later calls whose weight pointer falls inside that
 * range use the device copy.  Re-uploading the same range is a no-op.
 * Lifetime rule: the caller keeps [host, host + nbytes) mapped and unchanged
 * until ftc_backend_evict or ftc_backend_destroy (the engine's GGUF mapping
 * outlives its backend).  Only ranges passed here are ever cached: weights
 * the entry points below meet outside every uploaded range are copied to
 * the device for that call alone, so freeing or rewriting such a buffer
 * after the call is always safe. */
int ftc_backend_upload(ftc_backend* be, const void* host, size_t nbytes);
/* Drop the cached copy of the range that starts at `host`. */
int ftc_backend_evict(ftc_backend* be, const void* host);
/* Bytes currently cached on the device. */
int ftc_backend_cached_bytes(ftc_backend* be, uint64_t* bytes);

/* ft::IBackend::matmul (ft/include/ft/backend.h:28-29):
 *   y[m][n] = sum_k x[m][k] * W[n][k]   for m < M, n < N
 * x: host fp32 [M][K]; w_host: the tensor's host data pointer (HostTensor::
 * data), dtype and N rows of ceil(K/block) blocks; y: host fp32 [M][N].
 * A W inside an uploaded range is read from HBM; any other W is copied to
 * the device for this call only (nothing is cached implicitly).  Returns
 * with y written.  Unlike the reference's CpuBackend::matmul
 * (ft/src/cpu_backend.cpp:90-104), which folds all M rows into y[n], every
 * row m gets its own output row.  Q4_K with M > 8 runs on the tensor cores
 * (ftc_rows_to_f16 + ftc_gemm_rowscaled: fp16 operands, fp32 accumulation);
 * everything else on the fp32 GEMV, 8 rows per pass over the weight.
 * Per-call latency: x and y of up to 1 MiB move through the backend's pinned
 * buffers by a copy kernel and direct stores instead of the copy engines,
 * and a call on an uploaded weight replays a CUDA graph of its copy-in,
 * matmul and copy-out, captured on the first call with that (weight, M, K,
 * N, dtype) and kept until the staging buffers move or the backend is
 * destroyed.  FTC_BACKEND_GRAPHS=0 in the environment at ftc_backend_create
 * turns the graphs off. */
int ftc_backend_matmul(ftc_backend* be, const float* x, int64_t M, int64_t K,
                       const void* w_host, int dtype, int64_t N, float* y);

/* ft::ExpertChunkJob (ft/include/ft/backend.h:7-19), same fields. */
typedef struct ftc_expert_chunk_job {
    const float* x;      /* host fp32 [M][K] */
    float* out;          /* host fp32 [M][K], accumulated into (+=) */
    const void* gate;    /* host block pointers (inside a cached range or not) */
    const void* up;
    const void* down;
    int dtype;
    int64_t M;
    int64_t K;
    int64_t IC;          /* neurons in this window */
    size_t gate_up_row_stride;
    size_t down_row_stride;
} ftc_expert_chunk_job;

/* ft::IBackend::run_expert_chunk (ft/include/ft/backend.h:31), the maths of
 * ft/src/cpu_backend.cpp:106-149:
 *   h[m][i]   = silu(x_m . gate_i) * (x_m . up_i)          i < IC
 *   out[m][k] += sum_i h[m][i] * down_i[k]                  (down_i = row i)
 * Windows not inside a cached range are copied to the device per call. */
int ftc_backend_run_expert_chunk(ftc_backend* be, const ftc_expert_chunk_job* job);

/* The engine's down projection, ft::matmul_down_axpy (ft/src/cpu_backend.cpp:
 * 60-75; a free function the engine calls beside the interface, at
 * ft/src/engine.cpp:256, 275), with host buffers:
 *   y[m][j] += sum_i x[m][i] * W_i[j]      i < n_in, j < N
 * W_i = row i of w_host (N weights, row_bytes(dtype, N) bytes per row; the
 * reference's transposed "down" layout, n_in rows = neurons); rows with
 * x[m][i] == 0 add nothing.  x: host fp32 [M][n_in]; y: host fp32 [M][N],
 * accumulated.  The weight resolves like ftc_backend_matmul's: the HBM
 * copy of an uploaded range, else a copy for this call only.  M == 0 or
 * n_in == 0 changes nothing. */
int ftc_backend_matmul_down_axpy(ftc_backend* be, const float* x, int64_t M, int64_t n_in,
                                 const void* w_host, int dtype, int64_t N, float* y);

/* The routed experts of the engine's moe_ffn (ft/src/engine.cpp:179-241)
 * after its router matmul, with host buffers: the reference's router bias
 * (bias[E], may be NULL) is added to the logits, then ftc_moe_ffn runs on
 * the device and its result is added into out:
 *   out[t] += sum over t's top_k experts e of w_e * down_e . (silu(gate_e . x_t) * (up_e . x_t))
 * desc: as for ftc_moe_ffn but gate_exps / up_exps / down_exps are the
 * tensors' HOST data pointers (the GGUF mapping), resolved like
 * ftc_backend_matmul's weights (uploaded: HBM copy; else copied for this
 * call); down planes in the standard layout
 * (n_embd rows of n_ff).  logits: host fp32 [T][E]; x: host fp32 [T][n_embd];
 * out: host fp32 [T][n_embd] (the engine's tmpo).  T == 0 changes nothing. */
struct ftc_moe_desc; /* defined with the device MoE entry points below */
int ftc_backend_moe_ffn(ftc_backend* be, const struct ftc_moe_desc* desc, const float* logits,
                        const float* bias, const float* x, int64_t T, float* out);

/* ft::IBackend::sync (ft/include/ft/backend.h:39). */
int ftc_backend_sync(ftc_backend* be);

/* The backend's cudaStream_t (as void*), for callers mixing in kernel calls. */
void* ftc_backend_stream(ftc_backend* be);
/* Device pointer of the cached copy of `host` (NULL if not cached). */
const void* ftc_backend_device_ptr(ftc_backend* be, const void* host);

/* Kernels never trap or spin forever: a pipeline wait that exceeds its
 * bound (far above any legitimate wait) makes the kernel record a status and
 * return.  This synchronizes `stream`, returns the OR of the recorded
 * statuses in *status (0 = none; 1 = a bounded wait ran out) and clears
 * them. */
int ftc_device_status(void* stream, int* status);

/* ====================================================== kernel entry points
 * Device pointers; asynchronous on `stream` (a cudaStream_t; NULL = legacy
 * default stream).  They allocate nothing. */

/* Dequantize n_rows rows of k weights to fp32: out[r][j] (row pitch k).
 * Bit-exact with the reference's ft::dequant_row (ft/include/ft/quant.h:10-84)
 * for F32/F16/BF16/Q8_0/Q4_0/Q4_1, and with the GGUF K-quant formulas for
 * Q4_K/Q6_K.  k must be a whole number of blocks. */
int ftc_dequant(int dtype, const void* w, int64_t n_rows, int64_t k, int64_t row_stride,
                float* out, void* stream);

/* Decode GEMV/GEMM on CUDA cores, fp32 activations and accumulation:
 *   y[m][n] = sum_k x[m][k] * W[n][k]     m < M (1..8), n < N
 * x fp32 with row pitch k, y fp32 with row pitch N.  The per-row arithmetic
 * of ft::dot_row_f32 (ft/include/ft/quant.h:86-103) in a different
 * summation order. */
int ftc_mul_mat_vec(int dtype, const void* w, int64_t N, int64_t K, int64_t row_stride,
                    const float* x, int64_t M, float* y, void* stream);

/* Several decode GEMVs that read the same activations (q/k/v, gate/up) in
 * one launch: for i < n_mats, y_i[m][n] = sum_k x[m][k] * W_i[n][k], n < N[i].
 * w, N, y: host arrays of n_mats (<= 8) device pointers / row counts; all
 * matrices share dtype, K and row_stride.  Each y_i equals what
 * ftc_mul_mat_vec gives for that matrix alone, bit for bit. */
int ftc_mul_mat_vec_multi(int dtype, int n_mats, const void* const* w, const int64_t* N,
                          int64_t K, int64_t row_stride, const float* x, int64_t M,
                          float* const* y, void* stream);

/* ftc_mul_mat_vec_multi plus a prefetch hint for the launch that follows on
 * the same stream: next_w[i] / next_bytes[i] (i < n_next <= 8) are the
 * weight regions that launch reads, in the order it reads them.  Once this
 * launch has issued its last weight copy, its CTAs pull the first 24 MB of
 * those regions into L2, so the next launch's first copies hit L2 instead of
 * waiting on HBM while this one drains (batch 1, Q4_K; otherwise the hint is
 * ignored).  Regions must stay valid until the next launch has run.  No
 * counterpart in the reference (it has no device-side pipeline). */
int ftc_mul_mat_vec_multi_hint(int dtype, int n_mats, const void* const* w, const int64_t* N,
                               int64_t K, int64_t row_stride, const float* x, int64_t M,
                               float* const* y, int n_next, const void* const* next_w,
                               const int64_t* next_bytes, void* stream);

/* Prefill dequant-GEMM on the tcgen05 tensor cores:
 *   y[m][n] = sum_k x[m][k] * W[n][k]      m < M, n < N
 * W: Q4_K rows (16-byte aligned, row_stride % 16 == 0, K % 256 == 0).
 * x: [M][K] bf16 or fp16 (x_dtype), 16-byte aligned.  Each weight tile is
 * dequantized on chip to x's 16-bit type (fp32 arithmetic, one rounding to
 * 16 bits) and multiplied with fp32 accumulation.  y: [M][N] in y_dtype
 * (FTC_F32, FTC_BF16 or FTC_F16).  The per-row semantics of
 * ft::CpuBackend::matmul (ft/src/cpu_backend.cpp:90-104) for M > 1. */
int ftc_gemm(int dtype, const void* w, int64_t N, int64_t K, int64_t row_stride, const void* x,
             int x_dtype, int64_t M, void* y, int y_dtype, void* stream);

/* The prefill GEMM on fp16 rows produced by ftc_rows_to_f16: output row m is
 * multiplied by 2^row_exp[m] (exact), undoing the input row's scale.  Same
 * weight and output rules as ftc_gemm; x16: [M][K] fp16, 16-byte aligned. */
int ftc_gemm_rowscaled(int dtype, const void* w, int64_t N, int64_t K, int64_t row_stride,
                       const void* x16, int64_t M, void* y, int y_dtype, const int32_t* row_exp,
                       void* stream);

/* Activation rows to fp16 tensor-core operands without overflow or loss of
 * precision: out[m][k] = fp16(x[m][k] * 2^-row_exp[m]), row_exp[m] chosen so
 * the row's largest magnitude lands in [2^14, 2^15).  x: [rows][ld] in
 * x_dtype (FTC_F32, FTC_BF16, FTC_F16); out: [rows][K] fp16; K even. */
int ftc_rows_to_f16(const void* x, int x_dtype, int64_t rows, int64_t K, int64_t ld, void* out,
                    int32_t* row_exp, void* stream);

/* ftc_backend_matmul_down_axpy on DEVICE buffers: y[m][j] += sum_i x[m][i] *
 * W_i[j] (W: n_in rows of N weights, row_stride bytes apart; x fp32
 * [M][n_in]; y fp32 [M][N], accumulated; zero activations skipped).  N must
 * be a whole number of blocks.  ws: device scratch of at least
 * ftc_matmul_down_axpy_workspace_bytes(dtype, n_in, N, M) bytes (NULL when
 * that is 0); the partial sums of row slabs are added in a fixed order, so
 * the result is the same on every run. */
size_t ftc_matmul_down_axpy_workspace_bytes(int dtype, int64_t n_in, int64_t N, int64_t M);
int ftc_matmul_down_axpy(int dtype, const void* w, int64_t n_in, int64_t N, int64_t row_stride,
                         const float* x, int64_t M, float* y, void* ws, size_t ws_bytes,
                         void* stream);

/* h[i] = silu(g[i]) * u[i] = g / (1 + exp(-g)) * u in fp32, the expert FFN's
 * activation (ft/src/cpu_backend.cpp:127). */
int ftc_silu_mul(const float* g, const float* u, int64_t n, float* h, void* stream);

/* The same on rows that hold [gate (n values) | up (n values)] side by side
 * (pitch ld >= 2n: the output of one matmul over stacked gate and up
 * weights): row m of the result is silu(gate) * up, written either to h
 * (fp32 rows, pitch n) or, when h is NULL, to out16 as fp16 rows with
 * power-of-two scales exactly as ftc_rows_to_f16 would give for that fp32
 * row (out16 pitch n, n even, row_exp[rows]). */
int ftc_silu_mul_rows(const float* gu, int64_t rows, int64_t n, int64_t ld, float* h, void* out16,
                      int32_t* row_exp, void* stream);

/* Routed-expert MoE FFN layer on the device: the reference's
 * Engine::Impl::moe_ffn (ft/src/engine.cpp:179-241) after the router matmul,
 * with each expert's FFN (ft/src/cpu_backend.cpp:106-149) in the standard
 * GGUF layout (down_exps planes are [n_embd rows][n_ff cols]).
 *   p = softmax(logits[t]); the top_k experts by p (ties: lower index);
 *   w = p / sum of the chosen p;
 *   out[t] = sum over chosen e of w_e * down_e . (silu(gate_e . x_t) * (up_e . x_t))
 * Expert e's weights start at base + e * plane_stride.  Tokens are grouped by
 * expert on the device and every expert matmul is a tcgen05 dequant-GEMM
 * over all of its tokens with fp16 operands and fp32 accumulation: each row of
 * x and of h is scaled by a power of two into fp16's range first (undone
 * exactly afterwards), so no input range overflows.  Nothing returns to the
 * host, so a call can be captured in a CUDA graph.  n_ff <= 49152. */
typedef struct ftc_moe_desc {
    int dtype;                 /* expert weight format: FTC_Q4_K */
    int64_t n_experts;         /* E, 1..256 */
    int64_t top_k;             /* experts per token, 1..min(8, E) */
    int64_t n_embd;            /* model width K (multiple of 256) */
    int64_t n_ff;              /* expert hidden width (multiple of 256) */
    const void* gate_exps;     /* device: E planes of n_ff rows x n_embd */
    const void* up_exps;       /* device: E planes of n_ff rows x n_embd */
    const void* down_exps;     /* device: E planes of n_embd rows x n_ff */
    int64_t gu_row_stride;     /* bytes per gate/up row (16-byte multiple) */
    int64_t gu_plane_stride;   /* bytes per gate/up expert plane */
    int64_t dn_row_stride;     /* bytes per down row */
    int64_t dn_plane_stride;   /* bytes per down expert plane */
} ftc_moe_desc;

/* Device workspace bytes ftc_moe_ffn needs for T tokens (0 for a bad desc). */
size_t ftc_moe_workspace_bytes(const ftc_moe_desc* desc, int64_t T);

/* logits: device fp32 [T][E]; x: device [T][n_embd] in x_dtype (FTC_F32,
 * FTC_BF16 or FTC_F16; 16-byte aligned); out: device fp32 [T][n_embd],
 * overwritten.  workspace: 256-byte aligned device memory of at least
 * ftc_moe_workspace_bytes.  After the call the workspace starts with the
 * routing: int32 idx[T*top_k], then at the next 256-byte boundary fp32
 * weights[T*top_k], then int32 counts[E] (tokens per expert), each region
 * 256-byte aligned. */
int ftc_moe_ffn(const ftc_moe_desc* desc, const float* logits, const void* x, int x_dtype,
                int64_t T, float* out, void* workspace, size_t workspace_bytes, void* stream);

/* The routing half of ftc_moe_ffn (ft/src/engine.cpp:198-217): per token the
 * top_k experts (idx[T][top_k]) and renormalised weights (w[T][top_k]), the
 * rows of each expert in expert order (counts[E], offsets[E + 1]), each
 * expert's rank by first use (first_use_rank[E], -1 when unused), the row of
 * every (token, slot) pair (pos[T][top_k]) and the token of every row
 * (row_token[T * top_k]).  All device int32 / fp32 arrays. */
int ftc_moe_route(const float* logits, int64_t T, int64_t n_experts, int64_t top_k, int32_t* idx,
                  float* w, int32_t* counts, int32_t* offsets, int32_t* first_use_rank,
                  int32_t* pos, int32_t* row_token, void* stream);

/* The combine of ftc_moe_ffn: out[t] = sum over t's slots, in the experts'
 * first-use order, of w[t][u] * y[pos[t][u]] (separately rounded products
 * and sums, as ft/src/engine.cpp:229-236); y, out: device fp32, row pitch
 * n_embd (a multiple of 4). */
int ftc_moe_combine(const float* y, const int32_t* pos, const int32_t* idx, const float* w,
                    const int32_t* first_use_rank, int64_t T, int64_t top_k, int64_t n_embd,
                    float* out, void* stream);

/* The expert half of ftc_moe_ffn on rows already grouped by expert (the
 * local step of an expert-parallel layer, after the token exchange): rows
 * [offsets[e], offsets[e] + counts[e]) of x (device [rows][n_embd], x_dtype
 * FTC_F32 / FTC_BF16 / FTC_F16) go through expert e of desc (gate/up, silu,
 * down; same operand rules as ftc_moe_ffn) into y (device fp32
 * [rows][n_embd]).  counts / offsets: device int32 [n_experts]; max_rows:
 * an upper bound on every count.  workspace: 256-byte aligned device memory
 * of at least ftc_moe_experts_workspace_bytes(desc, rows).  desc->top_k is
 * not used here (a rank may hold fewer experts than the layer's top_k). */
size_t ftc_moe_experts_workspace_bytes(const ftc_moe_desc* desc, int64_t rows);
int ftc_moe_experts(const ftc_moe_desc* desc, const void* x, int x_dtype, int64_t rows,
                    const int32_t* counts, const int32_t* offsets, int64_t max_rows, float* y,
                    void* workspace, size_t workspace_bytes, void* stream);

/* The expert chunk of ftc_backend_run_expert_chunk on DEVICE buffers,
 * without allocating anything: for callers that cannot call cudaMalloc (an
 * engine whose HBM is owned by its own allocator, code inside someone
 * else's stream capture, a serving thread where allocation is forbidden).
 * No counterpart in the reference: its backends always own their buffers.
 *   h[m][i]   = silu(x_m . gate_i) * (x_m . up_i)      i < IC
 *   out[m][k] += sum_i h[m][i] * down_i[k]
 * x, out: device fp32 [M][K]; gate/up/down: device block pointers.  The
 * intermediate gate, up and h live in one library-owned __device__ array
 * (768 KB on every GPU that loads the library): M * IC must be at most
 * FTC_EXPERT_STATIC_MAX_HC, else FTC_E_INVALID.  All calls on a device share
 * that array, so calls that overlap on the GPU race; the first call on a
 * device looks up the array's address (make it before any stream capture). */
#define FTC_EXPERT_STATIC_MAX_HC 65536
int ftc_expert_chunk_static(int dtype, const float* x, float* out, const void* gate,
                            const void* up, const void* down, int64_t M, int64_t K, int64_t IC,
                            int64_t gate_up_row_stride, int64_t down_row_stride, void* stream);

/* ---- expert-parallel exchange with fixed capacity ----
 *
 * The expert-parallel MoE layer (experts split evenly over `world` GPUs,
 * rank d holding experts [d*E/world, (d+1)*E/world)) exchanges rows with
 * all-to-alls of equal splits: every rank sends every rank `cap` rows
 * (cap >= this rank's T * top_k, the same on all ranks), so no split size
 * goes to the host and the layer can be captured in a CUDA graph.
 *
 * ftc_ep_pack, after ftc_moe_route on this rank's T tokens: send[d][i] (rows
 * of n_embd x_dtype values) = x[row_token[off_d + i]] for the cnt_d rows
 * routed to rank d (off_d, cnt_d: prefix sums of counts over rank d's
 * experts; slots past cnt_d are left as they are); pos_padded[t][u] =
 * d * cap + i, the slot of token t's u-th row, i.e. where its expert output
 * comes back in the reverse exchange (pass it to ftc_moe_combine as pos).
 * With T == 0 (a rank without tokens) only counts and send are read.
 * The per-expert counts themselves are the [world][E/world] counts to send.
 *
 * ftc_ep_regroup, on the receiving rank with recv_counts[src][e] (rows of
 * local expert e from rank src): counts[e] / offsets[e] of the local
 * experts and a permutation of the world * cap received slots: perm[j] is
 * the slot that goes to position j (valid rows in expert-major,
 * source-major order first, then the padding), inv its inverse. */
int ftc_ep_pack(const void* x, int x_dtype, int64_t T, int64_t n_embd, const int32_t* idx,
                const int32_t* counts, const int32_t* pos, const int32_t* row_token,
                int64_t n_experts, int64_t top_k, int64_t world, int64_t cap, void* send,
                int32_t* pos_padded, void* stream);
int ftc_ep_regroup(const int32_t* recv_counts, int64_t world, int64_t n_local, int64_t cap,
                   int32_t* perm, int32_t* inv, int32_t* counts, int32_t* offsets, void* stream);

/* ---- tensor-parallel exchange: allreduce over NVLink peer memory ----
 *
 * One-shot allreduce (sum) of fp32 vectors between the ranks of a
 * tensor-parallel group, one process per GPU.  The row-parallel matmuls of
 * the tensor-parallel block (config 4) produce [M, n_embd] fp32 partials
 * that every rank needs summed; the reference has no such step (one process
 * runs every matmul, ft/src/engine.cpp:485-600).  Each rank's CTAs store
 * their slice into every rank's buffer, raise per-block flags and sum the
 * slots in rank order, so every rank gets the same bits.  Meant for small
 * vectors (up to a few MB); use NCCL for large ones.
 *
 * Setup: every rank calls ftc_peer_ar_create (same world and max_elems),
 * the FTC_IPC_HANDLE_BYTES handles are exchanged out of band (e.g. an
 * all-gather over the process group) and every rank calls ftc_peer_ar_open
 * with all handles in rank order.  Calls must then be made by every rank in
 * the same order (stream-ordered on each rank; CUDA-graph capture is fine).
 * A rank that does not join a call makes the others' kernels give up after
 * the library's wait bound and record status 1 (ftc_device_status).
 * Vectors of 16384+ elements on 4+ ranks use a two-shot exchange (each
 * element to an owner rank, the owner's rank-ordered sum to every rank);
 * the environment variable FTC_PEER_AR_TWO_SHOT=<elements> sets that
 * threshold for any group size. */
#define FTC_IPC_HANDLE_BYTES 64
typedef struct ftc_peer_ar ftc_peer_ar;
int ftc_peer_ar_create(int rank, int world, int64_t max_elems, ftc_peer_ar** out, void* handle);
int ftc_peer_ar_open(ftc_peer_ar* ar, const void* handles);
int64_t ftc_peer_ar_max_elems(const ftc_peer_ar* ar);
/* out[i] = sum over ranks of in[i], i < n <= max_elems; out may equal in. */
int ftc_peer_ar_sum_f32(ftc_peer_ar* ar, const float* in, float* out, int64_t n, void* stream);
int ftc_peer_ar_destroy(ftc_peer_ar* ar);

/* A row-parallel decode GEMV and its allreduce in one kernel: every rank
 * passes its shard w (N rows of Q4_K, its K columns) and its x (fp32, K);
 * y = sum over the ranks of x . w^T (fp32, N <= max_elems), the same bits on
 * every rank.  The kernel's producer pushes each finished row of the rank's
 * partial into every rank's buffer and each CTA then sums its own rows over
 * the ranks in rank order (bounded waits, as ftc_peer_ar_sum_f32).  Shares
 * ar's call counters with ftc_peer_ar_sum_f32; every rank makes the same
 * calls in the same order.  FTC_E_UNSUPPORTED if the shape or alignment does
 * not fit the fused kernel. */
int ftc_mul_mat_vec_allreduce(ftc_peer_ar* ar, int dtype, const void* w, int64_t N, int64_t K,
                               int64_t row_stride, const float* x, float* y, void* stream);

/* The row-parallel down projection of a SiLU FFN at one token, with the
 * activation computed as it is loaded:
 *   y[n] = sum_k silu(gu[k]) * gu[up_offset + k] * W[n][k]
 * silu(g) * u = g / (1 + exp(-g)) * u in fp32 (ft/src/cpu_backend.cpp:127),
 * bit for bit what ftc_silu_mul_rows + ftc_mul_mat_vec give.  gu: DEVICE
 * fp32 [gate (K) | ... | up (K)] (the output row of a stacked gate/up
 * matmul), 16-byte aligned, up_offset >= K and a multiple of 4.  With ar
 * (may be NULL) the product is also summed over the ranks in the kernel, as
 * ftc_mul_mat_vec_allreduce.  Q4_K, 16-byte aligned rows. */
int ftc_mul_mat_vec_silu(ftc_peer_ar* ar, int dtype, const void* w, int64_t N, int64_t K,
                         int64_t row_stride, const float* gu, int64_t up_offset, float* y,
                         void* stream);

/* ------------------------------------------------------------ attention */

/* Bytes of workspace ftc_attention needs for this shape (0: none). */
size_t ftc_attention_workspace_bytes(int64_t M, int64_t n_head, int64_t n_head_kv,
                                     int64_t head_dim, int64_t base);

/* Causal grouped-query attention on DEVICE buffers, Engine::Impl::attn
 * (ft/src/engine.cpp:137-177): query row m (position base + m) of head h
 * attends positions 0 .. base + m of KV head h / (n_head / n_head_kv), with
 * scores q . k / sqrt(head_dim) and a softmax over them.  q and out are fp32
 * [M][n_head][head_dim]; K and V rows are fp32 [position][kv_stride] with the
 * head's head_dim values at kv_head * head_dim.  Positions below base are
 * read from k_cache / v_cache (row p at p * kv_stride; may be NULL when base
 * is 0), the rest from k_blk / v_blk (position p at (p - base) * kv_stride),
 * which is the cache itself at row base when the caller stored the block
 * there first (the engine's write_kv path, ft/src/engine.cpp:553-565).
 * head_dim 64, 128 or 256; kv_stride >= n_head_kv * head_dim, a multiple of
 * 4; every buffer 16-byte aligned; ws at least
 * ftc_attention_workspace_bytes (may be NULL when that is 0). */
int ftc_attention(const float* q, int64_t M, int64_t n_head, int64_t n_head_kv, int64_t head_dim,
                  const float* k_cache, const float* v_cache, int64_t kv_stride, int64_t base,
                  const float* k_blk, const float* v_blk, float* out, void* ws, size_t ws_bytes,
                  void* stream);

/* Rotary position embedding in place on DEVICE fp32 x [M][heads][head_dim],
 * row m at position base + m: rope_vec (ft/src/engine.cpp:43-60) as the
 * engine applies it to q and k (ft/src/engine.cpp:545-551); neox != 0 rotates
 * the pairs (i, i + head_dim/2), else (2i, 2i + 1).  Angles in double, the
 * rotation in float with separately rounded products, as the reference. */
int ftc_rope(float* x, int64_t M, int64_t heads, int64_t head_dim, int64_t base, double theta,
             int neox, void* stream);

/* The engine's KV cache in this backend's HBM: ft::KvCache::alloc
 * (ft/include/ft/kv_cache.h:12-20), n_layers x capacity rows of dim fp32 for
 * K and for V, zero-filled; replaces any cache the backend held. */
int ftc_backend_kv_alloc(ftc_backend* be, int64_t n_layers, int64_t capacity, int64_t dim);

/* The engine's per-layer attention step with HOST buffers: q [M][n_head *
 * head_dim] and the block's k_new / v_new [M][n_head_kv * head_dim] (all fp32,
 * after RoPE), out [M][n_head * head_dim].  With write_kv the block's rows
 * are stored into the device cache at rows [base, base + M) of `layer` first
 * (ft/src/engine.cpp:553-559), else they are used for this call only.  Then
 * ftc_attention over the cache's rows [0, base) and the block.  Synchronous,
 * like the engine's CPU attention.  Requires ftc_backend_kv_alloc with dim =
 * n_head_kv * head_dim and base + M <= capacity. */
int ftc_backend_attention(ftc_backend* be, int64_t layer, int64_t base, int64_t M, int64_t n_head,
                          int64_t n_head_kv, int64_t head_dim, const float* q,
                          const float* k_new, const float* v_new, int write_kv, float* out);

/* Rows [pos0, pos0 + n) of `layer` of the device KV cache to HOST k / v
 * ([n][dim] fp32 each): the copies the engine's prefix cache makes when it
 * stores a snapshot (ft/src/engine.cpp:630-645).  Synchronous. */
int ftc_backend_kv_read(ftc_backend* be, int64_t layer, int64_t pos0, int64_t n, float* k,
                        float* v);

/* HOST k / v ([n][dim] fp32 each) into rows [pos0, pos0 + n) of `layer` of
 * the device KV cache: the copies the engine makes when it restores a
 * prefix-cache snapshot (ft/src/engine.cpp:608-616).  Synchronous. */
int ftc_backend_kv_write(ftc_backend* be, int64_t layer, int64_t pos0, int64_t n, const float* k,
                         const float* v);

#ifdef __cplusplus
}
#endif
#endif /* FTC_H */
