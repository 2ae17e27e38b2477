// api.cu -- the C ABI of libftcuda.so (include/ftc.h): status plumbing, the
// backend instance (device, stream, HBM weight cache, pinned staging) and
// the extern "C" entry points.
#include <cstdlib>
#include <cstring>
#include <atomic>
#include <map>
#include <mutex>
#include <set>
#include <string>
#include <tuple>

#include "common.cuh"

namespace ftc {

// ------------------------------------------------------------ status

namespace {
thread_local std::string g_last_error;
}

int set_error(int code, const std::string& msg) {
    g_last_error = msg;
    return code;
}

int cuda_error(cudaError_t e, const char* what) {
    return set_error(FTC_E_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

int ok() {
    g_last_error.clear();
    return FTC_OK;
}

int device_sms() {
    constexpr int kMaxDevices = 64;
    static std::atomic<int> sms[kMaxDevices] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return 148;
    int v = sms[dev].load(std::memory_order_relaxed);
    if (!v) {
        if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || v <= 0)
            return 148;
        sms[dev].store(v, std::memory_order_relaxed);
    }
    return v;
}

int opt_in_smem(const void* fn, int bytes, const char* what) {
    int dev = 0;
    FTC_CUDA(cudaGetDevice(&dev));
    static std::mutex mu;
    static std::set<std::tuple<const void*, int, int>> done;
    std::lock_guard<std::mutex> lk(mu);
    if (done.count(std::make_tuple(fn, dev, bytes))) return FTC_OK;
    const cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e != cudaSuccess) return cuda_error(e, what);
    done.insert(std::make_tuple(fn, dev, bytes));
    return FTC_OK;
}

bool inject_fail(const char* entry) {
    const char* v = std::getenv("FTC_INJECT_FAIL");
    if (!v || !*v) return false;
    if (std::strcmp(v, "all") == 0) return true;
    // comma-separated list of entry-point names
    const size_t n = std::strlen(entry);
    for (const char* p = v; *p;) {
        const char* e = std::strchr(p, ',');
        const size_t len = e ? (size_t)(e - p) : std::strlen(p);
        if (len == n && std::strncmp(p, entry, n) == 0) return true;
        if (!e) break;
        p = e + 1;
    }
    return false;
}

// kernels (gemv.cu, dequant.cu, expert.cu)
int mul_mat_vec(int dtype, const void* w, int64_t N, int64_t K, int64_t row_stride,
                const float* x, int64_t M, float* y, cudaStream_t st);
int dequant(int dtype, const void* w, int64_t n_rows, int64_t k, int64_t row_stride, float* out,
            cudaStream_t st);
int mul_mat_vec_multi(int dtype, int P, const void* const* w, const int64_t* N, int64_t K,
                      int64_t row_stride, const float* x, int64_t M, float* const* y,
                      cudaStream_t st, int n_next, const void* const* next_w,
                      const int64_t* next_bytes);
int expert_chunk_dev(int dtype, const float* x, float* out, const void* gate, const void* up,
                     const void* down, int64_t M, int64_t K, int64_t IC, int64_t gu_stride,
                     int64_t dn_stride, float* gbuf, float* ubuf, float* hbuf, cudaStream_t st);

int gemm_q4k(const void* w, int64_t N, int64_t K, int64_t row_stride, const void* x, int x_dtype,
             int64_t M, void* y, int y_dtype, cudaStream_t st);
int gemm_q4k_rowscaled(const void* w, int64_t N, int64_t K, int64_t row_stride, const void* x16,
                       int64_t M, void* y, int y_dtype, const int32_t* row_exp, cudaStream_t st);
int copy_f32(float* dst, const float* src, int64_t n, cudaStream_t st);
int rows_to_f16(const void* x, int x_dtype, int64_t rows, int64_t K, int64_t ld, void* out,
                int32_t* row_exp, cudaStream_t st);
int silu_mul_rows(const float* gu, int64_t rows, int64_t n, int64_t ld, float* h, void* out16,
                  int32_t* row_exp, cudaStream_t st);
int ep_pack(const void* x, int x_dtype, int64_t T, int64_t n_embd, const int32_t* idx,
            const int32_t* counts, const int32_t* pos, const int32_t* row_token, int64_t n_experts,
            int64_t top_k, int64_t world, int64_t cap, void* send, int32_t* pos_padded,
            cudaStream_t st);
int ep_regroup(const int32_t* recv_counts, int64_t world, int64_t n_local, int64_t cap,
               int32_t* perm, int32_t* inv, int32_t* counts, int32_t* offsets, cudaStream_t st);
int silu_mul(const float* g, const float* u, int64_t n, float* h, cudaStream_t st);
size_t down_axpy_workspace_bytes(int dtype, int64_t n_in, int64_t N, int64_t M);
int down_axpy(int dtype, const void* w, int64_t n_in, int64_t N, int64_t row_stride,
              const float* x, int64_t M, float* y, void* ws, size_t ws_bytes, cudaStream_t st);
size_t moe_workspace_bytes(const ftc_moe_desc* d, int64_t T);
size_t moe_experts_workspace_bytes(const ftc_moe_desc* d, int64_t rows);
int moe_route_only(const float* logits, int64_t T, int64_t E, int64_t U, int32_t* idx, float* w,
                   int32_t* counts, int32_t* offsets, int32_t* rank, int32_t* pos,
                   int32_t* row_token, cudaStream_t st);
int moe_combine_only(const float* y, const int32_t* pos, const int32_t* idx, const float* w,
                     const int32_t* rank, int64_t T, int64_t U, int64_t K, float* out,
                     cudaStream_t st);
int moe_experts(const ftc_moe_desc* d, const void* x, int x_dtype, int64_t rows,
                const int32_t* counts, const int32_t* offsets, int64_t max_rows, float* y,
                void* ws, size_t ws_bytes, cudaStream_t st);
int moe_ffn(const ftc_moe_desc* d, const float* logits, const void* x, int x_dtype, int64_t T,
            float* out, void* ws, size_t ws_bytes, cudaStream_t st);
size_t attention_workspace_bytes(int64_t M, int64_t n_head, int64_t n_head_kv, int64_t head_dim,
                                 int64_t base);
int attention(const float* q, int64_t M, int64_t n_head, int64_t n_head_kv, int64_t head_dim,
              const float* k_cache, const float* v_cache, int64_t kv_stride, int64_t base,
              const float* k_blk, const float* v_blk, float* out, void* ws, size_t ws_bytes,
              cudaStream_t st);
int attention_check(int64_t M, int64_t n_head, int64_t n_head_kv, int64_t head_dim, int64_t base,
                    const char* who);
int rope(float* x, int64_t M, int64_t heads, int64_t head_dim, int64_t base, double theta,
         int neox, cudaStream_t st);

// status readers of the translation units whose kernels use bounded waits
int devstat_gemv_q4k(int clear);
int devstat_gemv_imma(int clear);
int devstat_gemm_q4k(int clear);
int devstat_peer_ar(int clear);

}  // namespace ftc

using namespace ftc;

// ------------------------------------------------------------ backend

namespace {

// Growable device / pinned-host buffer owned by a backend.
// ftc_backend_matmul moves x and y of at most this many bytes with a copy
// kernel and direct stores into pinned memory instead of the copy engines.
constexpr size_t kKernelCopyMax = 1 << 20;

struct DevBuf {
    void* p = nullptr;
    size_t cap = 0;
    bool pinned = false;
    int ensure(size_t bytes) {
        if (bytes <= cap) return FTC_OK;
        release();
        size_t want = bytes < 4096 ? 4096 : bytes;
        cudaError_t e = pinned ? cudaMallocHost(&p, want) : cudaMalloc(&p, want);
        if (e != cudaSuccess) {
            p = nullptr;
            cap = 0;
            return set_error(FTC_E_NOMEM, std::string("staging allocation: ") + cudaGetErrorString(e));
        }
        cap = want;
        return FTC_OK;
    }
    void release() {
        if (p) pinned ? cudaFreeHost(p) : cudaFree(p);
        p = nullptr;
        cap = 0;
    }
};

struct CacheEntry {
    const uint8_t* host;
    size_t nbytes;
    void* dev;
};

}  // namespace

struct ftc_backend {
    int device = 0;
    cudaStream_t stream = nullptr;
    std::string name;
    uint64_t mem = 0;
    std::map<uintptr_t, CacheEntry> cache;  // keyed by host start address
    uint64_t cached = 0;
    DevBuf pin_in{nullptr, 0, true}, pin_out{nullptr, 0, true};
    DevBuf dx, dy, dwin, dtmp;
    std::mutex mu;

    // the engine's KV cache in HBM (ftc_backend_kv_alloc): K of all layers,
    // then V, each [layer][capacity][dim] fp32; dattn stages one attention
    // call's q, block rows, workspace and output
    float* kv = nullptr;
    int64_t kv_layers = 0, kv_cap = 0, kv_dim = 0;
    DevBuf dattn;

    // ftc_backend_matmul's per-call work (copy in, GEMV or GEMM, copy out)
    // captured once per (weight, shape) and replayed as a CUDA graph: one
    // launch instead of three to six API calls.  On unless
    // FTC_BACKEND_GRAPHS=0 at creation.  The graphs hold the staging
    // buffers' addresses, so all of them are dropped when a buffer moves.
    bool use_graphs = false;
    bool uva = false;  // pinned host buffers are addressable from kernels
    std::map<std::tuple<const void*, int64_t, int64_t, int64_t, int>, cudaGraphExec_t> graphs;
    void* graph_bufs[5] = {nullptr, nullptr, nullptr, nullptr, nullptr};
    void drop_graphs() {
        for (auto& kv : graphs) cudaGraphExecDestroy(kv.second);
        graphs.clear();
    }

    // Cached entry that fully covers [p, p + n), or nullptr.
    const CacheEntry* find(const void* p, size_t n) const {
        const uintptr_t a = (uintptr_t)p;
        auto it = cache.upper_bound(a);
        if (it == cache.begin()) return nullptr;
        --it;
        const CacheEntry& e = it->second;
        if (a >= (uintptr_t)e.host && a + n <= (uintptr_t)e.host + e.nbytes) return &e;
        return nullptr;
    }

    int upload(const void* host, size_t nbytes) {
        if (find(host, nbytes)) return FTC_OK;
        void* d = nullptr;
        cudaError_t e = cudaMalloc(&d, nbytes);
        if (e != cudaSuccess)
            return set_error(FTC_E_NOMEM, std::string("weight upload: ") + cudaGetErrorString(e));
        e = cudaMemcpyAsync(d, host, nbytes, cudaMemcpyHostToDevice, stream);
        if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
        if (e != cudaSuccess) {
            cudaFree(d);
            return cuda_error(e, "weight upload copy");
        }
        cache[(uintptr_t)host] = CacheEntry{static_cast<const uint8_t*>(host), nbytes, d};
        cached += nbytes;
        return FTC_OK;
    }

    // Device addresses of n host ranges.  A range inside a tensor passed to
    // upload() uses that HBM copy; any other range is copied, on the
    // backend's stream, into the per-call window buffer `dwin` and used from
    // there for this call only.  Nothing is cached implicitly, so a host
    // buffer that the caller frees or rewrites after the call can never be
    // served later from a stale device copy.  *streamed tells whether any
    // range went through the window buffer.
    int resolve(int n, const void* const* host, const size_t* bytes, const void** dev,
                bool* streamed) {
        size_t off[4] = {0, 0, 0, 0}, total = 0;
        for (int i = 0; i < n; ++i) {
            const CacheEntry* e = find(host[i], bytes[i]);
            if (e) {
                dev[i] = static_cast<const uint8_t*>(e->dev) + ((const uint8_t*)host[i] - e->host);
            } else {
                dev[i] = nullptr;
                off[i] = total;
                total += (bytes[i] + 255) & ~(size_t)255;
            }
        }
        *streamed = total > 0;
        if (!total) return FTC_OK;
        int rc = dwin.ensure(total);
        if (rc) return rc;
        for (int i = 0; i < n; ++i)
            if (!dev[i]) {
                void* d = static_cast<uint8_t*>(dwin.p) + off[i];
                FTC_CUDA(cudaMemcpyAsync(d, host[i], bytes[i], cudaMemcpyHostToDevice, stream));
                dev[i] = d;
            }
        return FTC_OK;
    }
};

namespace {

int bind(ftc_backend* be) {
    FTC_REQUIRE(be, FTC_E_INVALID, "null backend");
    FTC_CUDA(cudaSetDevice(be->device));
    return FTC_OK;
}

}  // namespace

extern "C" {

const char* ftc_last_error(void) { return g_last_error.c_str(); }

int ftc_abi_version(void) { return 1; }

int64_t ftc_row_bytes(int dtype, int64_t k) { return row_bytes(dtype, k); }

int ftc_backend_create(int device, ftc_backend** out) {
    FTC_REQUIRE(out, FTC_E_INVALID, "ftc_backend_create: null out");
    *out = nullptr;
    if (inject_fail("ftc_backend_create"))
        return set_error(FTC_E_INJECTED, "ftc_backend_create: injected failure");
    int n = 0;
    FTC_CUDA(cudaGetDeviceCount(&n));
    FTC_REQUIRE(device >= 0 && device < n, FTC_E_INVALID, "ftc_backend_create: no such device");
    FTC_CUDA(cudaSetDevice(device));
    cudaDeviceProp prop;
    FTC_CUDA(cudaGetDeviceProperties(&prop, device));
    FTC_REQUIRE(prop.major == 10, FTC_E_UNSUPPORTED,
                "ftc_backend_create: libftcuda is built for sm_100a (B200) only");
    ftc_backend* be = new ftc_backend();
    be->device = device;
    const char* g = std::getenv("FTC_BACKEND_GRAPHS");
    be->use_graphs = !(g && std::strcmp(g, "0") == 0);
    be->uva = prop.unifiedAddressing != 0;
    be->name = std::string("CUDA:") + prop.name;
    be->mem = prop.totalGlobalMem;
    cudaError_t e = cudaStreamCreateWithFlags(&be->stream, cudaStreamNonBlocking);
    if (e != cudaSuccess) {
        delete be;
        return cuda_error(e, "cudaStreamCreate");
    }
    *out = be;
    return ok();
}

void ftc_backend_destroy(ftc_backend* be) {
    if (!be) return;
    cudaSetDevice(be->device);
    if (be->stream) cudaStreamSynchronize(be->stream);
    be->drop_graphs();
    for (auto& kv : be->cache) cudaFree(kv.second.dev);
    be->pin_in.release();
    be->pin_out.release();
    be->dx.release();
    be->dy.release();
    be->dwin.release();
    be->dtmp.release();
    be->dattn.release();
    if (be->kv) cudaFree(be->kv);
    if (be->stream) cudaStreamDestroy(be->stream);
    delete be;
}

int ftc_backend_info(ftc_backend* be, char* name, size_t cap, uint64_t* mem_bytes) {
    FTC_REQUIRE(be, FTC_E_INVALID, "ftc_backend_info: null backend");
    if (name && cap) {
        std::strncpy(name, be->name.c_str(), cap - 1);
        name[cap - 1] = 0;
    }
    if (mem_bytes) *mem_bytes = be->mem;
    return ok();
}

int ftc_backend_upload(ftc_backend* be, const void* host, size_t nbytes) {
    int rc = bind(be);
    if (rc) return rc;
    FTC_REQUIRE(host && nbytes, FTC_E_INVALID, "ftc_backend_upload: empty range");
    if (inject_fail("ftc_backend_upload"))
        return set_error(FTC_E_INJECTED, "ftc_backend_upload: injected failure");
    std::lock_guard<std::mutex> lk(be->mu);
    rc = be->upload(host, nbytes);
    return rc ? rc : ok();
}

int ftc_backend_evict(ftc_backend* be, const void* host) {
    int rc = bind(be);
    if (rc) return rc;
    std::lock_guard<std::mutex> lk(be->mu);
    auto it = be->cache.find((uintptr_t)host);
    FTC_REQUIRE(it != be->cache.end(), FTC_E_INVALID, "ftc_backend_evict: range not cached");
    FTC_CUDA(cudaStreamSynchronize(be->stream));
    be->drop_graphs();  // they may read the evicted copy
    cudaFree(it->second.dev);
    be->cached -= it->second.nbytes;
    be->cache.erase(it);
    return ok();
}

int ftc_backend_cached_bytes(ftc_backend* be, uint64_t* bytes) {
    FTC_REQUIRE(be && bytes, FTC_E_INVALID, "ftc_backend_cached_bytes: null argument");
    *bytes = be->cached;
    return ok();
}

void* ftc_backend_stream(ftc_backend* be) { return be ? (void*)be->stream : nullptr; }

const void* ftc_backend_device_ptr(ftc_backend* be, const void* host) {
    if (!be) return nullptr;
    std::lock_guard<std::mutex> lk(be->mu);
    const CacheEntry* e = be->find(host, 1);
    return e ? static_cast<const uint8_t*>(e->dev) + ((const uint8_t*)host - e->host) : nullptr;
}

int ftc_backend_matmul(ftc_backend* be, const float* x, int64_t M, int64_t K, const void* w_host,
                       int dtype, int64_t N, float* y) {
    int rc = bind(be);
    if (rc) return rc;
    const Fmt f = fmt_of(dtype);
    FTC_REQUIRE(f.block_elems > 0, FTC_E_UNSUPPORTED, "ftc_backend_matmul: unknown dtype");
    FTC_REQUIRE(x && w_host && y, FTC_E_INVALID, "ftc_backend_matmul: null pointer");
    FTC_REQUIRE(M > 0 && K > 0 && N > 0, FTC_E_INVALID, "ftc_backend_matmul: empty shape");
    FTC_REQUIRE(K % f.block_elems == 0, FTC_E_INVALID,
                "ftc_backend_matmul: K must be a whole number of blocks");
    if (inject_fail("ftc_backend_matmul"))
        return set_error(FTC_E_INJECTED, "ftc_backend_matmul: injected failure");
    std::lock_guard<std::mutex> lk(be->mu);
    const int64_t stride = row_bytes(dtype, K);
    const void* dW = nullptr;
    const size_t wb = (size_t)(stride * N);
    bool streamed = false;
    if ((rc = be->resolve(1, &w_host, &wb, &dW, &streamed))) return rc;
    const size_t xb = (size_t)(M * K) * 4, yb = (size_t)(M * N) * 4;
    if ((rc = be->pin_in.ensure(xb)) || (rc = be->pin_out.ensure(yb)) || (rc = be->dx.ensure(xb)) ||
        (rc = be->dy.ensure(yb)))
        return rc;
    // Q4_K beyond 8 rows (prefill, speculative verify): the tensor-core GEMM
    // on fp16 rows with power-of-two row scales, one pass over the weight;
    // otherwise the fp32 GEMV, 8 rows per pass.
    const bool tc = dtype == FTC_Q4_K && M > 8 && M <= INT32_MAX && N <= INT32_MAX &&
                    (uintptr_t)dW % 16 == 0 && stride % 16 == 0;
    const size_t x16b = tc ? ((size_t)(M * K) * 2 + 255) & ~(size_t)255 : 0;
    if (tc && (rc = be->dtmp.ensure(x16b + (size_t)M * 4))) return rc;
    std::memcpy(be->pin_in.p, x, xb);
    const float* dx = static_cast<const float*>(be->dx.p);
    // Small calls (decode): a copy engine transfer on each side of the GEMV
    // costs more than the GEMV (~7 us each on B200).  Instead a copy kernel
    // reads x from the pinned buffer (the GEMV behind it starts early and
    // prefetches its weights meanwhile), and the GEMV stores y straight into
    // the pinned output buffer; both reached through unified addressing.
    const bool small = be->uva && !tc && xb <= kKernelCopyMax && yb <= kKernelCopyMax;
    float* dy = small ? static_cast<float*>(be->pin_out.p) : static_cast<float*>(be->dy.p);
    cudaStream_t st = be->stream;
    auto enqueue = [&]() -> int {
        if (small) {
            const int crc = copy_f32(static_cast<float*>(be->dx.p),
                                     static_cast<const float*>(be->pin_in.p), M * K, st);
            if (crc) return crc;
        } else {
            FTC_CUDA(cudaMemcpyAsync(be->dx.p, be->pin_in.p, xb, cudaMemcpyHostToDevice, st));
        }
        int erc;
        if (tc) {
            void* x16 = be->dtmp.p;
            int32_t* row_exp = reinterpret_cast<int32_t*>(static_cast<uint8_t*>(be->dtmp.p) + x16b);
            if ((erc = rows_to_f16(dx, FTC_F32, M, K, K, x16, row_exp, st)) ||
                (erc = gemm_q4k_rowscaled(dW, N, K, stride, x16, M, dy, FTC_F32, row_exp, st)))
                return erc;
        } else {
            for (int64_t m0 = 0; m0 < M; m0 += 8) {
                const int64_t mc = M - m0 < 8 ? M - m0 : 8;
                if ((erc = mul_mat_vec(dtype, dW, N, K, stride, dx + m0 * K, mc, dy + m0 * N, st)))
                    return erc;
            }
        }
        if (!small) FTC_CUDA(cudaMemcpyAsync(be->pin_out.p, dy, yb, cudaMemcpyDeviceToHost, st));
        return FTC_OK;
    };
    // Graphs only for resident weights: a streamed weight's copy is per call.
    if (be->use_graphs && !streamed) {
        void* bufs[5] = {be->pin_in.p, be->pin_out.p, be->dx.p, be->dy.p, be->dtmp.p};
        if (std::memcmp(bufs, be->graph_bufs, sizeof(bufs)) != 0) {
            be->drop_graphs();
            std::memcpy(be->graph_bufs, bufs, sizeof(bufs));
        }
        const auto key = std::make_tuple(dW, M, K, N, dtype);
        auto it = be->graphs.find(key);
        if (it == be->graphs.end()) {
            // relaxed: a kernel's first launch may set its shared-memory attribute
            FTC_CUDA(cudaStreamBeginCapture(st, cudaStreamCaptureModeRelaxed));
            const int erc = enqueue();
            cudaGraph_t g = nullptr;
            const cudaError_t ce = cudaStreamEndCapture(st, &g);
            if (erc || ce != cudaSuccess) {
                if (g) cudaGraphDestroy(g);
                return erc ? erc : cuda_error(ce, "ftc_backend_matmul: graph capture");
            }
            cudaGraphExec_t ex = nullptr;
            const cudaError_t ie = cudaGraphInstantiate(&ex, g, 0);
            cudaGraphDestroy(g);
            if (ie != cudaSuccess) return cuda_error(ie, "ftc_backend_matmul: graph instantiate");
            it = be->graphs.emplace(key, ex).first;
        }
        FTC_CUDA(cudaGraphLaunch(it->second, st));
    } else if ((rc = enqueue())) {
        return rc;
    }
    FTC_CUDA(cudaStreamSynchronize(st));
    std::memcpy(y, be->pin_out.p, yb);
    return ok();
}

int ftc_backend_run_expert_chunk(ftc_backend* be, const ftc_expert_chunk_job* job) {
    int rc = bind(be);
    if (rc) return rc;
    FTC_REQUIRE(job, FTC_E_INVALID, "ftc_backend_run_expert_chunk: null job");
    const int64_t M = job->M, K = job->K, IC = job->IC;
    if (IC <= 0 || M <= 0 || K <= 0) return ok();  // as ft/src/cpu_backend.cpp:110
    const Fmt f = fmt_of(job->dtype);
    FTC_REQUIRE(f.block_elems > 0, FTC_E_UNSUPPORTED, "ftc_backend_run_expert_chunk: unknown dtype");
    FTC_REQUIRE(job->x && job->out && job->gate && job->up && job->down, FTC_E_INVALID,
                "ftc_backend_run_expert_chunk: null pointer");
    FTC_REQUIRE(K % f.block_elems == 0, FTC_E_INVALID,
                "ftc_backend_run_expert_chunk: K must be a whole number of blocks");
    const int64_t rb = row_bytes(job->dtype, K);
    FTC_REQUIRE((int64_t)job->gate_up_row_stride >= rb && (int64_t)job->down_row_stride >= rb,
                FTC_E_INVALID, "ftc_backend_run_expert_chunk: stride smaller than a row");
    if (inject_fail("ftc_backend_run_expert_chunk"))
        return set_error(FTC_E_INJECTED, "ftc_backend_run_expert_chunk: injected failure");
    std::lock_guard<std::mutex> lk(be->mu);
    // Windows: cached ranges are used in place; anything else is streamed in
    // (the reference's staging upload, ft/include/ft/chunker.h:126-147).
    const size_t gu_bytes = (size_t)((IC - 1) * (int64_t)job->gate_up_row_stride + rb);
    const size_t dn_bytes = (size_t)((IC - 1) * (int64_t)job->down_row_stride + rb);
    const void* win[3] = {job->gate, job->up, job->down};
    const size_t wbytes[3] = {gu_bytes, gu_bytes, dn_bytes};
    const void* dev[3] = {nullptr, nullptr, nullptr};
    bool streamed = false;
    if ((rc = be->resolve(3, win, wbytes, dev, &streamed))) return rc;
    const size_t xb = (size_t)(M * K) * 4, hb = (size_t)(M * IC) * 4;
    if ((rc = be->pin_in.ensure(2 * xb)) || (rc = be->pin_out.ensure(xb)) ||
        (rc = be->dx.ensure(2 * xb)) || (rc = be->dtmp.ensure(3 * hb + 768)))
        return rc;
    std::memcpy(be->pin_in.p, job->x, xb);
    std::memcpy(static_cast<uint8_t*>(be->pin_in.p) + xb, job->out, xb);
    FTC_CUDA(cudaMemcpyAsync(be->dx.p, be->pin_in.p, 2 * xb, cudaMemcpyHostToDevice, be->stream));
    float* dxp = static_cast<float*>(be->dx.p);
    float* dout = reinterpret_cast<float*>(static_cast<uint8_t*>(be->dx.p) + xb);
    uint8_t* t = static_cast<uint8_t*>(be->dtmp.p);
    float* g = reinterpret_cast<float*>(t);
    float* u = reinterpret_cast<float*>(t + ((hb + 255) & ~(size_t)255));
    float* h = reinterpret_cast<float*>(t + 2 * ((hb + 255) & ~(size_t)255));
    if ((rc = expert_chunk_dev(job->dtype, dxp, dout, dev[0], dev[1], dev[2], M, K, IC,
                               (int64_t)job->gate_up_row_stride, (int64_t)job->down_row_stride, g,
                               u, h, be->stream)))
        return rc;
    FTC_CUDA(cudaMemcpyAsync(be->pin_out.p, dout, xb, cudaMemcpyDeviceToHost, be->stream));
    FTC_CUDA(cudaStreamSynchronize(be->stream));
    std::memcpy(job->out, be->pin_out.p, xb);
    return ok();
}

int ftc_backend_kv_alloc(ftc_backend* be, int64_t n_layers, int64_t capacity, int64_t dim) {
    int rc = bind(be);
    if (rc) return rc;
    FTC_REQUIRE(n_layers > 0 && capacity > 0 && dim > 0 && dim % 4 == 0, FTC_E_INVALID,
                "ftc_backend_kv_alloc: empty shape or dim not a multiple of 4");
    FTC_REQUIRE(n_layers <= (1 << 20) && capacity <= (1 << 28) && dim <= (1 << 20) &&
                    n_layers * capacity <= ((int64_t)1 << 40) / dim,
                FTC_E_INVALID, "ftc_backend_kv_alloc: cache too large");
    std::lock_guard<std::mutex> lk(be->mu);
    FTC_CUDA(cudaStreamSynchronize(be->stream));  // no call may still read the old cache
    if (be->kv) cudaFree(be->kv);
    be->kv = nullptr;
    be->kv_layers = be->kv_cap = be->kv_dim = 0;
    const size_t bytes = (size_t)(2 * n_layers * capacity * dim) * sizeof(float);
    void* p = nullptr;
    const cudaError_t e = cudaMalloc(&p, bytes);
    if (e != cudaSuccess)
        return set_error(FTC_E_NOMEM, std::string("ftc_backend_kv_alloc: ") + cudaGetErrorString(e));
    const cudaError_t z = cudaMemsetAsync(p, 0, bytes, be->stream);  // KvCache::alloc zero-fills
    if (z != cudaSuccess) {
        cudaFree(p);
        return cuda_error(z, "ftc_backend_kv_alloc: cudaMemsetAsync");
    }
    be->kv = static_cast<float*>(p);
    be->kv_layers = n_layers;
    be->kv_cap = capacity;
    be->kv_dim = dim;
    return ok();
}

int ftc_backend_attention(ftc_backend* be, int64_t layer, int64_t base, int64_t M, int64_t n_head,
                          int64_t n_head_kv, int64_t head_dim, const float* q,
                          const float* k_new, const float* v_new, int write_kv, float* out) {
    int rc = bind(be);
    if (rc) return rc;
    if ((rc = attention_check(M, n_head, n_head_kv, head_dim, base, "ftc_backend_attention")))
        return rc;
    FTC_REQUIRE(q && k_new && v_new && out, FTC_E_INVALID, "ftc_backend_attention: null pointer");
    if (inject_fail("ftc_backend_attention"))
        return set_error(FTC_E_INJECTED, "ftc_backend_attention: injected failure");
    std::lock_guard<std::mutex> lk(be->mu);
    FTC_REQUIRE(be->kv, FTC_E_INVALID, "ftc_backend_attention: no KV cache (ftc_backend_kv_alloc)");
    const int64_t dk = n_head_kv * head_dim;
    FTC_REQUIRE(dk == be->kv_dim, FTC_E_INVALID,
                "ftc_backend_attention: n_head_kv * head_dim differs from the cache's dim");
    FTC_REQUIRE(layer >= 0 && layer < be->kv_layers, FTC_E_INVALID,
                "ftc_backend_attention: layer out of range");
    FTC_REQUIRE(base + M <= be->kv_cap, FTC_E_INVALID,
                "ftc_backend_attention: base + M exceeds the cache capacity");
    // staging: [q | k_new | v_new | out | workspace], each 256-byte aligned
    auto up = [](size_t b) { return (b + 255) & ~size_t(255); };
    const size_t qb = (size_t)(M * n_head * head_dim) * 4, rb = (size_t)(M * dk) * 4;
    const size_t wsb = attention_workspace_bytes(M, n_head, n_head_kv, head_dim, base);
    const size_t in_b = up(qb) + 2 * up(rb);
    if ((rc = be->pin_in.ensure(in_b)) || (rc = be->pin_out.ensure(qb)) ||
        (rc = be->dattn.ensure(in_b + up(qb) + up(wsb))))
        return rc;
    uint8_t* hp = static_cast<uint8_t*>(be->pin_in.p);
    std::memcpy(hp, q, qb);
    std::memcpy(hp + up(qb), k_new, rb);
    std::memcpy(hp + up(qb) + up(rb), v_new, rb);
    uint8_t* dp = static_cast<uint8_t*>(be->dattn.p);
    cudaStream_t st = be->stream;
    FTC_CUDA(cudaMemcpyAsync(dp, hp, in_b, cudaMemcpyHostToDevice, st));
    const float* dq = reinterpret_cast<const float*>(dp);
    const float* dkn = reinterpret_cast<const float*>(dp + up(qb));
    const float* dvn = reinterpret_cast<const float*>(dp + up(qb) + up(rb));
    float* dout = reinterpret_cast<float*>(dp + in_b);
    void* dws = wsb ? dp + in_b + up(qb) : nullptr;
    float* kc = be->kv + layer * be->kv_cap * dk;
    float* vc = be->kv + (be->kv_layers + layer) * be->kv_cap * dk;
    const float* kb = dkn;
    const float* vb = dvn;
    if (write_kv) {  // the block joins the cache (ft/src/engine.cpp:553-559)
        FTC_CUDA(cudaMemcpyAsync(kc + base * dk, dkn, rb, cudaMemcpyDeviceToDevice, st));
        FTC_CUDA(cudaMemcpyAsync(vc + base * dk, dvn, rb, cudaMemcpyDeviceToDevice, st));
        kb = kc + base * dk;
        vb = vc + base * dk;
    }
    if ((rc = attention(dq, M, n_head, n_head_kv, head_dim, kc, vc, dk, base, kb, vb, dout, dws,
                        wsb, st)))
        return rc;
    FTC_CUDA(cudaMemcpyAsync(be->pin_out.p, dout, qb, cudaMemcpyDeviceToHost, st));
    FTC_CUDA(cudaStreamSynchronize(st));
    std::memcpy(out, be->pin_out.p, qb);
    return ok();
}

namespace {

// rows [pos0, pos0 + n) of `layer`: K and V device pointers, or an error
int kv_rows(ftc_backend* be, int64_t layer, int64_t pos0, int64_t n, float** k, float** v,
            const char* who) {
    FTC_REQUIRE(be->kv, FTC_E_INVALID, std::string(who) + ": no KV cache (ftc_backend_kv_alloc)");
    FTC_REQUIRE(layer >= 0 && layer < be->kv_layers, FTC_E_INVALID,
                std::string(who) + ": layer out of range");
    FTC_REQUIRE(pos0 >= 0 && n >= 0 && pos0 + n <= be->kv_cap, FTC_E_INVALID,
                std::string(who) + ": rows outside the cache");
    *k = be->kv + (layer * be->kv_cap + pos0) * be->kv_dim;
    *v = be->kv + ((be->kv_layers + layer) * be->kv_cap + pos0) * be->kv_dim;
    return FTC_OK;
}

}  // namespace

int ftc_backend_kv_read(ftc_backend* be, int64_t layer, int64_t pos0, int64_t n, float* k,
                        float* v) {
    int rc = bind(be);
    if (rc) return rc;
    FTC_REQUIRE(k && v, FTC_E_INVALID, "ftc_backend_kv_read: null pointer");
    std::lock_guard<std::mutex> lk(be->mu);
    float *dk, *dv;
    if ((rc = kv_rows(be, layer, pos0, n, &dk, &dv, "ftc_backend_kv_read"))) return rc;
    const size_t bytes = (size_t)(n * be->kv_dim) * sizeof(float);
    FTC_CUDA(cudaMemcpyAsync(k, dk, bytes, cudaMemcpyDeviceToHost, be->stream));
    FTC_CUDA(cudaMemcpyAsync(v, dv, bytes, cudaMemcpyDeviceToHost, be->stream));
    FTC_CUDA(cudaStreamSynchronize(be->stream));
    return ok();
}

int ftc_backend_kv_write(ftc_backend* be, int64_t layer, int64_t pos0, int64_t n, const float* k,
                         const float* v) {
    int rc = bind(be);
    if (rc) return rc;
    FTC_REQUIRE(k && v, FTC_E_INVALID, "ftc_backend_kv_write: null pointer");
    std::lock_guard<std::mutex> lk(be->mu);
    float *dk, *dv;
    if ((rc = kv_rows(be, layer, pos0, n, &dk, &dv, "ftc_backend_kv_write"))) return rc;
    const size_t bytes = (size_t)(n * be->kv_dim) * sizeof(float);
    FTC_CUDA(cudaMemcpyAsync(dk, k, bytes, cudaMemcpyHostToDevice, be->stream));
    FTC_CUDA(cudaMemcpyAsync(dv, v, bytes, cudaMemcpyHostToDevice, be->stream));
    FTC_CUDA(cudaStreamSynchronize(be->stream));  // the host buffers may go after the call
    return ok();
}

int ftc_backend_matmul_down_axpy(ftc_backend* be, const float* x, int64_t M, int64_t n_in,
                                 const void* w_host, int dtype, int64_t N, float* y) {
    int rc = bind(be);
    if (rc) return rc;
    const Fmt f = fmt_of(dtype);
    FTC_REQUIRE(f.block_elems > 0, FTC_E_UNSUPPORTED, "ftc_backend_matmul_down_axpy: unknown dtype");
    FTC_REQUIRE(M >= 0 && n_in >= 0 && N > 0 && N % f.block_elems == 0, FTC_E_INVALID,
                "ftc_backend_matmul_down_axpy: bad shape (N must be whole blocks)");
    if (M == 0 || n_in == 0) return ok();  // the reference's loops do nothing
    FTC_REQUIRE(x && w_host && y, FTC_E_INVALID, "ftc_backend_matmul_down_axpy: null pointer");
    if (inject_fail("ftc_backend_matmul_down_axpy"))
        return set_error(FTC_E_INJECTED, "ftc_backend_matmul_down_axpy: injected failure");
    std::lock_guard<std::mutex> lk(be->mu);
    const int64_t stride = row_bytes(dtype, N);
    const void* dW = nullptr;
    const size_t wb = (size_t)(stride * n_in);
    bool streamed = false;
    if ((rc = be->resolve(1, &w_host, &wb, &dW, &streamed))) return rc;
    const size_t xb = (size_t)(M * n_in) * 4, yb = (size_t)(M * N) * 4;
    const size_t xo = (xb + 255) & ~(size_t)255;
    const size_t wsb = down_axpy_workspace_bytes(dtype, n_in, N, M);
    if ((rc = be->pin_in.ensure(xo + yb)) || (rc = be->pin_out.ensure(yb)) ||
        (rc = be->dx.ensure(xo + yb)) || (rc = be->dtmp.ensure(wsb ? wsb : 1)))
        return rc;
    std::memcpy(be->pin_in.p, x, xb);
    std::memcpy(static_cast<uint8_t*>(be->pin_in.p) + xo, y, yb);
    FTC_CUDA(cudaMemcpyAsync(be->dx.p, be->pin_in.p, xo + yb, cudaMemcpyHostToDevice, be->stream));
    const float* dx = static_cast<const float*>(be->dx.p);
    float* dy = reinterpret_cast<float*>(static_cast<uint8_t*>(be->dx.p) + xo);
    if ((rc = down_axpy(dtype, dW, n_in, N, stride, dx, M, dy, be->dtmp.p, be->dtmp.cap,
                        be->stream)))
        return rc;
    FTC_CUDA(cudaMemcpyAsync(be->pin_out.p, dy, yb, cudaMemcpyDeviceToHost, be->stream));
    FTC_CUDA(cudaStreamSynchronize(be->stream));
    std::memcpy(y, be->pin_out.p, yb);
    return ok();
}

int ftc_backend_moe_ffn(ftc_backend* be, const ftc_moe_desc* desc, const float* logits,
                        const float* bias, const float* x, int64_t T, float* out) {
    int rc = bind(be);
    if (rc) return rc;
    FTC_REQUIRE(desc && T >= 0, FTC_E_INVALID, "ftc_backend_moe_ffn: null desc or T < 0");
    if (T == 0) return ok();
    FTC_REQUIRE(logits && x && out, FTC_E_INVALID, "ftc_backend_moe_ffn: null pointer");
    // the desc is checked before any of its host ranges is touched
    if (moe_workspace_bytes(desc, T) == 0) return FTC_E_INVALID;  // message set by the check
    FTC_REQUIRE(desc->gate_exps && desc->up_exps && desc->down_exps, FTC_E_INVALID,
                "ftc_backend_moe_ffn: null expert tensor");
    FTC_REQUIRE(desc->gu_row_stride >= row_bytes(FTC_Q4_K, desc->n_embd) &&
                    desc->gu_plane_stride >= desc->n_ff * desc->gu_row_stride &&
                    desc->dn_row_stride >= row_bytes(FTC_Q4_K, desc->n_ff) &&
                    desc->dn_plane_stride >= desc->n_embd * desc->dn_row_stride,
                FTC_E_INVALID, "ftc_backend_moe_ffn: row or plane stride smaller than its rows");
    if (inject_fail("ftc_backend_moe_ffn"))
        return set_error(FTC_E_INJECTED, "ftc_backend_moe_ffn: injected failure");
    std::lock_guard<std::mutex> lk(be->mu);
    ftc_moe_desc d = *desc;
    const int64_t E = d.n_experts, K = d.n_embd;
    const void* dev[3] = {nullptr, nullptr, nullptr};
    const void* host[3] = {d.gate_exps, d.up_exps, d.down_exps};
    // each tensor's extent: E - 1 whole planes and the last plane's rows
    const size_t gu_ext = (size_t)((E - 1) * d.gu_plane_stride + d.n_ff * d.gu_row_stride);
    const size_t dn_ext = (size_t)((E - 1) * d.dn_plane_stride + K * d.dn_row_stride);
    const size_t bytes[3] = {gu_ext, gu_ext, dn_ext};
    bool streamed = false;
    if ((rc = be->resolve(3, host, bytes, dev, &streamed))) return rc;
    d.gate_exps = dev[0];
    d.up_exps = dev[1];
    d.down_exps = dev[2];
    const size_t wsb = moe_workspace_bytes(&d, T);
    FTC_REQUIRE(wsb > 0, FTC_E_INVALID, "ftc_backend_moe_ffn: bad desc");
    const size_t lb = (size_t)(T * E) * 4, lo = (lb + 255) & ~(size_t)255;
    const size_t xb = (size_t)(T * K) * 4;
    if ((rc = be->pin_in.ensure(lo + xb)) || (rc = be->pin_out.ensure(xb)) ||
        (rc = be->dx.ensure(lo + xb)) || (rc = be->dy.ensure(xb)) || (rc = be->dtmp.ensure(wsb)))
        return rc;
    float* pl = static_cast<float*>(be->pin_in.p);
    std::memcpy(pl, logits, lb);
    if (bias)  // r[j] += rbias[j] before the softmax (ft/src/engine.cpp:200-201)
        for (int64_t t = 0; t < T; ++t)
            for (int64_t e = 0; e < E; ++e) pl[t * E + e] += bias[e];
    std::memcpy(static_cast<uint8_t*>(be->pin_in.p) + lo, x, xb);
    FTC_CUDA(cudaMemcpyAsync(be->dx.p, be->pin_in.p, lo + xb, cudaMemcpyHostToDevice, be->stream));
    const float* dl = static_cast<const float*>(be->dx.p);
    const void* dxp = static_cast<const uint8_t*>(be->dx.p) + lo;
    float* dy = static_cast<float*>(be->dy.p);
    if ((rc = moe_ffn(&d, dl, dxp, FTC_F32, T, dy, be->dtmp.p, be->dtmp.cap, be->stream))) return rc;
    FTC_CUDA(cudaMemcpyAsync(be->pin_out.p, dy, xb, cudaMemcpyDeviceToHost, be->stream));
    FTC_CUDA(cudaStreamSynchronize(be->stream));
    const float* po = static_cast<const float*>(be->pin_out.p);
    for (int64_t i = 0; i < T * K; ++i) out[i] += po[i];
    return ok();
}

int ftc_backend_sync(ftc_backend* be) {
    int rc = bind(be);
    if (rc) return rc;
    FTC_CUDA(cudaStreamSynchronize(be->stream));
    return ok();
}

int ftc_device_status(void* stream, int* status) {
    FTC_REQUIRE(status, FTC_E_INVALID, "ftc_device_status: null status");
    FTC_CUDA(cudaStreamSynchronize((cudaStream_t)stream));
    int v = 0;
    for (int (*rd)(int) : {devstat_gemv_q4k, devstat_gemv_imma, devstat_gemm_q4k, devstat_peer_ar}) {
        const int s = rd(1);
        FTC_REQUIRE(s >= 0, FTC_E_CUDA, "ftc_device_status: cannot read the status word");
        v |= s;
    }
    *status = v;
    return ok();
}

int ftc_dequant(int dtype, const void* w, int64_t n_rows, int64_t k, int64_t row_stride,
                float* out, void* stream) {
    int rc = dequant(dtype, w, n_rows, k, row_stride, out, (cudaStream_t)stream);
    return rc ? rc : ok();
}

int ftc_mul_mat_vec(int dtype, const void* w, int64_t N, int64_t K, int64_t row_stride,
                    const float* x, int64_t M, float* y, void* stream) {
    int rc = mul_mat_vec(dtype, w, N, K, row_stride, x, M, y, (cudaStream_t)stream);
    return rc ? rc : ok();
}

int ftc_mul_mat_vec_multi(int dtype, int n_mats, const void* const* w, const int64_t* N,
                          int64_t K, int64_t row_stride, const float* x, int64_t M,
                          float* const* y, void* stream) {
    int rc = mul_mat_vec_multi(dtype, n_mats, w, N, K, row_stride, x, M, y, (cudaStream_t)stream,
                               0, nullptr, nullptr);
    return rc ? rc : ok();
}

int ftc_mul_mat_vec_multi_hint(int dtype, int n_mats, const void* const* w, const int64_t* N,
                               int64_t K, int64_t row_stride, const float* x, int64_t M,
                               float* const* y, int n_next, const void* const* next_w,
                               const int64_t* next_bytes, void* stream) {
    int rc = mul_mat_vec_multi(dtype, n_mats, w, N, K, row_stride, x, M, y, (cudaStream_t)stream,
                               n_next, next_w, next_bytes);
    return rc ? rc : ok();
}

int ftc_gemm(int dtype, const void* w, int64_t N, int64_t K, int64_t row_stride, const void* x,
             int x_dtype, int64_t M, void* y, int y_dtype, void* stream) {
    FTC_REQUIRE(dtype == FTC_Q4_K, FTC_E_UNSUPPORTED, "ftc_gemm: only Q4_K weights");
    int rc = gemm_q4k(w, N, K, row_stride, x, x_dtype, M, y, y_dtype, (cudaStream_t)stream);
    return rc ? rc : ok();
}

int ftc_gemm_rowscaled(int dtype, const void* w, int64_t N, int64_t K, int64_t row_stride,
                       const void* x16, int64_t M, void* y, int y_dtype, const int32_t* row_exp,
                       void* stream) {
    FTC_REQUIRE(dtype == FTC_Q4_K, FTC_E_UNSUPPORTED, "ftc_gemm_rowscaled: only Q4_K weights");
    int rc = gemm_q4k_rowscaled(w, N, K, row_stride, x16, M, y, y_dtype, row_exp,
                                (cudaStream_t)stream);
    return rc ? rc : ok();
}

int ftc_rows_to_f16(const void* x, int x_dtype, int64_t rows, int64_t K, int64_t ld, void* out,
                    int32_t* row_exp, void* stream) {
    int rc = rows_to_f16(x, x_dtype, rows, K, ld, out, row_exp, (cudaStream_t)stream);
    return rc ? rc : ok();
}

size_t ftc_matmul_down_axpy_workspace_bytes(int dtype, int64_t n_in, int64_t N, int64_t M) {
    return down_axpy_workspace_bytes(dtype, n_in, N, M);
}

int ftc_matmul_down_axpy(int dtype, const void* w, int64_t n_in, int64_t N, int64_t row_stride,
                         const float* x, int64_t M, float* y, void* ws, size_t ws_bytes,
                         void* stream) {
    int rc = down_axpy(dtype, w, n_in, N, row_stride, x, M, y, ws, ws_bytes, (cudaStream_t)stream);
    return rc ? rc : ok();
}

size_t ftc_attention_workspace_bytes(int64_t M, int64_t n_head, int64_t n_head_kv,
                                     int64_t head_dim, int64_t base) {
    return attention_workspace_bytes(M, n_head, n_head_kv, head_dim, base);
}

int ftc_attention(const float* q, int64_t M, int64_t n_head, int64_t n_head_kv, int64_t head_dim,
                  const float* k_cache, const float* v_cache, int64_t kv_stride, int64_t base,
                  const float* k_blk, const float* v_blk, float* out, void* ws, size_t ws_bytes,
                  void* stream) {
    if (inject_fail("ftc_attention"))
        return set_error(FTC_E_INJECTED, "ftc_attention: injected failure");
    int rc = attention(q, M, n_head, n_head_kv, head_dim, k_cache, v_cache, kv_stride, base, k_blk,
                       v_blk, out, ws, ws_bytes, (cudaStream_t)stream);
    return rc ? rc : ok();
}

int ftc_rope(float* x, int64_t M, int64_t heads, int64_t head_dim, int64_t base, double theta,
             int neox, void* stream) {
    int rc = rope(x, M, heads, head_dim, base, theta, neox, (cudaStream_t)stream);
    return rc ? rc : ok();
}

int ftc_silu_mul(const float* g, const float* u, int64_t n, float* h, void* stream) {
    int rc = silu_mul(g, u, n, h, (cudaStream_t)stream);
    return rc ? rc : ok();
}

int ftc_silu_mul_rows(const float* gu, int64_t rows, int64_t n, int64_t ld, float* h, void* out16,
                      int32_t* row_exp, void* stream) {
    int rc = silu_mul_rows(gu, rows, n, ld, h, out16, row_exp, (cudaStream_t)stream);
    return rc ? rc : ok();
}

int ftc_ep_pack(const void* x, int x_dtype, int64_t T, int64_t n_embd, const int32_t* idx,
                const int32_t* counts, const int32_t* pos, const int32_t* row_token,
                int64_t n_experts, int64_t top_k, int64_t world, int64_t cap, void* send,
                int32_t* pos_padded, void* stream) {
    int rc = ep_pack(x, x_dtype, T, n_embd, idx, counts, pos, row_token, n_experts, top_k, world,
                     cap, send, pos_padded, (cudaStream_t)stream);
    return rc ? rc : ok();
}

int ftc_ep_regroup(const int32_t* recv_counts, int64_t world, int64_t n_local, int64_t cap,
                   int32_t* perm, int32_t* inv, int32_t* counts, int32_t* offsets, void* stream) {
    int rc = ep_regroup(recv_counts, world, n_local, cap, perm, inv, counts, offsets,
                        (cudaStream_t)stream);
    return rc ? rc : ok();
}

int ftc_moe_route(const float* logits, int64_t T, int64_t n_experts, int64_t top_k, int32_t* idx,
                  float* w, int32_t* counts, int32_t* offsets, int32_t* first_use_rank,
                  int32_t* pos, int32_t* row_token, void* stream) {
    int rc = moe_route_only(logits, T, n_experts, top_k, idx, w, counts, offsets, first_use_rank,
                            pos, row_token, (cudaStream_t)stream);
    return rc ? rc : ok();
}

int ftc_moe_combine(const float* y, const int32_t* pos, const int32_t* idx, const float* w,
                    const int32_t* first_use_rank, int64_t T, int64_t top_k, int64_t n_embd,
                    float* out, void* stream) {
    int rc = moe_combine_only(y, pos, idx, w, first_use_rank, T, top_k, n_embd, out,
                              (cudaStream_t)stream);
    return rc ? rc : ok();
}

size_t ftc_moe_experts_workspace_bytes(const ftc_moe_desc* desc, int64_t rows) {
    return moe_experts_workspace_bytes(desc, rows);
}

int ftc_moe_experts(const ftc_moe_desc* desc, const void* x, int x_dtype, int64_t rows,
                    const int32_t* counts, const int32_t* offsets, int64_t max_rows, float* y,
                    void* workspace, size_t workspace_bytes, void* stream) {
    int rc = moe_experts(desc, x, x_dtype, rows, counts, offsets, max_rows, y, workspace,
                         workspace_bytes, (cudaStream_t)stream);
    return rc ? rc : ok();
}

size_t ftc_moe_workspace_bytes(const ftc_moe_desc* desc, int64_t T) {
    return moe_workspace_bytes(desc, T);
}

int ftc_moe_ffn(const ftc_moe_desc* desc, const float* logits, const void* x, int x_dtype,
                int64_t T, float* out, void* workspace, size_t workspace_bytes, void* stream) {
    int rc = moe_ffn(desc, logits, x, x_dtype, T, out, workspace, workspace_bytes,
                     (cudaStream_t)stream);
    return rc ? rc : ok();
}

}  // extern "C"
