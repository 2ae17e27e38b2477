// test_cuda_backend.cpp -- ft::CudaBackend (the C++ IBackend drop-in) on a
// B200, in the style of the reference's own test binary
// (ft/src/tests/test_core.cpp: CHECK macro, failure count, exit status).
// Checked against the CPU oracle (oracle/ftoracle.c, linked as a checker).
#include <cmath>
#include <cstdio>
#include <cstring>
#include <stdexcept>
#include <vector>

#include "cuda_backend.h"
#include "ft/gguf.h"
#include "ftoracle.h"

using namespace ft;

static int g_fails = 0;

#define CHECK(cond, msg)                                     \
    do {                                                     \
        if (!(cond)) {                                       \
            std::printf("FAIL %d: %s\n", __LINE__, msg);     \
            ++g_fails;                                       \
        }                                                    \
    } while (0)

static uint32_t g_lcg = 123456789u;
static uint32_t next_u32() {
    g_lcg = g_lcg * 1664525u + 1013904223u;
    return g_lcg;
}
static float rnd() { return ((float)((next_u32() >> 9) & 0x7FFF) / 32768.f) * 2.f - 1.f; }

// Random blocks with sane fp16 scales for the formats under test.
static std::vector<uint8_t> random_blocks(DType t, int64_t rows, int64_t cols) {
    const size_t rb = dtype_row_bytes(t, cols);
    std::vector<uint8_t> b(rb * (size_t)rows);
    for (auto& v : b) v = (uint8_t)(next_u32() >> 24);
    const size_t bb = dtype_bytes_per_block(t);
    const size_t nblk = b.size() / bb;
    for (size_t i = 0; i < nblk; ++i) {
        uint8_t* p = b.data() + i * bb;
        const uint16_t d = ftor_float_to_half(0.01f + 0.01f * std::fabs(rnd()));
        if (t == DType::Q8_0) std::memcpy(p, &d, 2);
        if (t == DType::Q4_K) { std::memcpy(p, &d, 2); std::memcpy(p + 2, &d, 2); }
        if (t == DType::Q6_K) std::memcpy(p + 208, &d, 2);
    }
    return b;
}

static HostTensor view(const std::vector<uint8_t>& b, DType t, int64_t cols, int64_t rows) {
    HostTensor h;
    h.name = "w";
    h.ne[0] = cols;
    h.ne[1] = rows;
    h.n_dims = 2;
    h.dtype = t;
    h.data = b.data();
    h.nbytes = b.size();
    return h;
}

// max |a-b| / max |b|: the tensor-core path's bound (fp16 operands)
static double norm_err(const std::vector<float>& a, const std::vector<float>& b) {
    double d = 0, r = 0;
    for (size_t i = 0; i < b.size(); ++i) {
        d = std::fmax(d, std::fabs((double)a[i] - b[i]));
        r = std::fmax(r, std::fabs((double)b[i]));
    }
    return d / r;
}

// max |a-b| / (|b| + 1e-2 * rms(b))
static double rel_err(const std::vector<float>& a, const std::vector<float>& b) {
    double ss = 0;
    for (float v : b) ss += (double)v * v;
    const double rms = std::sqrt(ss / (double)b.size());
    double m = 0;
    for (size_t i = 0; i < b.size(); ++i)
        m = std::fmax(m, std::fabs((double)a[i] - b[i]) / (std::fabs((double)b[i]) + 1e-2 * rms));
    return m;
}

static void test_matmul(CudaBackend& be, DType t, int64_t N, int64_t K, int64_t M) {
    auto w = random_blocks(t, N, K);
    HostTensor W = view(w, t, K, N);
    std::vector<float> x((size_t)(M * K));
    for (auto& v : x) v = rnd();
    std::vector<float> y((size_t)(M * N), NAN), ref((size_t)(M * N));
    be.matmul(x.data(), M, K, W, y.data());
    ftor_matmul(x.data(), M, K, w.data(), (int)t, N, (int64_t)W.row_stride_bytes(), ref.data(), 8);
    char msg[96];
    std::snprintf(msg, sizeof msg, "matmul dtype %u N %lld K %lld M %lld", (unsigned)t,
                  (long long)N, (long long)K, (long long)M);
    // Q4_K beyond 8 rows runs on the tensor cores (fp16 operands)
    const bool tc = t == DType::Q4_K && M > 8;
    CHECK((tc ? norm_err(y, ref) : rel_err(y, ref)) <= 2e-3, msg);
}

// The reference chunker test's shapes (ft/src/tests/test_core.cpp:307-346):
// F32 K=16, FF=48, M=3 in windows of 8, accumulated window by window.
static void test_expert_chunk_windows(CudaBackend& be) {
    const int64_t K = 16, FF = 48, M = 3, C = 8;
    std::vector<float> gate((size_t)(K * FF)), up((size_t)(K * FF)), down((size_t)(K * FF));
    for (auto& v : gate) v = rnd() * 0.5f;
    for (auto& v : up) v = rnd() * 0.5f;
    for (auto& v : down) v = rnd() * 0.5f;
    std::vector<float> x((size_t)(M * K));
    for (auto& v : x) v = rnd();
    std::vector<float> out((size_t)(M * K), 0.f), ref((size_t)(M * K), 0.f);
    const size_t stride = (size_t)K * 4;
    for (int64_t i0 = 0; i0 < FF; i0 += C) {
        ExpertChunkJob job;
        job.x = x.data();
        job.out = out.data();
        job.gate = gate.data() + i0 * K;
        job.up = up.data() + i0 * K;
        job.down = down.data() + i0 * K;
        job.dt = DType::F32;
        job.M = M;
        job.K = K;
        job.IC = C;
        job.gate_up_row_stride = stride;
        job.down_row_stride = stride;
        be.run_expert_chunk(job);
        ftor_expert_chunk(x.data(), ref.data(), (const uint8_t*)(gate.data() + i0 * K),
                          (const uint8_t*)(up.data() + i0 * K), (const uint8_t*)(down.data() + i0 * K),
                          FTOR_F32, M, K, C, (int64_t)stride, (int64_t)stride, 1);
    }
    double maxerr = 0;
    for (size_t j = 0; j < ref.size(); ++j)
        maxerr = std::fmax(maxerr, std::fabs(ref[j] - out[j]) / (std::fabs(ref[j]) + 1e-3));
    CHECK(maxerr < 1e-4, "chunked expert equivalence (reference test bound)");
}

// The engine's FFN down projection (ft/src/engine.cpp:256, 275) in both
// layouts: neuron-major through matmul_down_axpy (checked against the
// reference's loop, ftor_matmul_down_axpy), output-major through matmul.
static void test_down_project(CudaBackend& be, DType t, int64_t n_ff, int64_t n_embd, int64_t M) {
    std::vector<float> h((size_t)(M * n_ff));
    for (size_t i = 0; i < h.size(); ++i) h[i] = (i % 5 == 0) ? 0.f : rnd();
    std::vector<float> y0((size_t)(M * n_embd));
    for (auto& v : y0) v = rnd();
    char msg[128];
    {  // neuron-major: n_ff rows of n_embd weights
        auto w = random_blocks(t, n_ff, n_embd);
        HostTensor W = view(w, t, n_embd, n_ff);
        std::vector<float> y = y0, ref = y0;
        be.down_project(h.data(), M, n_ff, W, y.data());
        ftor_matmul_down_axpy(h.data(), M, n_ff, w.data(), (int)t, n_embd,
                              (int64_t)W.row_stride_bytes(), ref.data(), 8);
        std::snprintf(msg, sizeof msg, "down_project neuron rows dtype %u n_ff %lld M %lld",
                      (unsigned)t, (long long)n_ff, (long long)M);
        CHECK(rel_err(y, ref) <= 2e-3, msg);
    }
    if (n_ff != n_embd) {  // output-major: n_embd rows of n_ff weights
        auto w = random_blocks(t, n_embd, n_ff);
        HostTensor W = view(w, t, n_ff, n_embd);
        std::vector<float> y = y0, ref((size_t)(M * n_embd));
        be.down_project(h.data(), M, n_ff, W, y.data());
        ftor_matmul(h.data(), M, n_ff, w.data(), (int)t, n_embd, (int64_t)W.row_stride_bytes(),
                    ref.data(), 8);
        for (size_t i = 0; i < ref.size(); ++i) ref[i] += y0[i];
        std::snprintf(msg, sizeof msg, "down_project output rows dtype %u n_ff %lld M %lld",
                      (unsigned)t, (long long)n_ff, (long long)M);
        CHECK(rel_err(y, ref) <= 2e-3, msg);
    }
}

// The engine's routed experts through moe_ffn against the oracle's MoE
// (the reference's routing and expert arithmetic, standard down layout).
static void test_moe_ffn(CudaBackend& be, int64_t T, bool with_bias) {
    const int64_t E = 8, U = 2, K = 1024, FF = 2048;
    auto g = random_blocks(DType::Q4_K, E * FF, K), u = random_blocks(DType::Q4_K, E * FF, K);
    auto dn = random_blocks(DType::Q4_K, E * K, FF);
    HostTensor G = view(g, DType::Q4_K, K, FF), Uu = view(u, DType::Q4_K, K, FF);
    HostTensor D = view(dn, DType::Q4_K, FF, K);
    G.ne[2] = Uu.ne[2] = D.ne[2] = E;
    std::vector<float> x((size_t)(T * K)), logits((size_t)(T * E)), bias;
    for (auto& v : x) v = rnd();
    for (auto& v : logits) v = rnd() * 2.f;
    if (with_bias) {
        bias.resize((size_t)E);
        for (auto& v : bias) v = rnd();
    }
    std::vector<float> out((size_t)(T * K)), ref((size_t)(T * K), 0.f), biased = logits;
    for (auto& v : out) v = rnd();
    const std::vector<float> out0 = out;
    CHECK(be.moe_ffn(x.data(), logits.data(), bias, T, U, G, Uu, D, out.data()), "moe_ffn handled");
    if (with_bias)
        for (int64_t t = 0; t < T; ++t)
            for (int64_t e = 0; e < E; ++e) biased[(size_t)(t * E + e)] += bias[(size_t)e];
    ftor_moe_ffn(x.data(), biased.data(), T, K, FF, E, U, g.data(), u.data(), dn.data(), FTOR_Q4_K,
                 ref.data(), 8);
    for (size_t i = 0; i < ref.size(); ++i) ref[i] += out0[i];
    char msg[96];
    std::snprintf(msg, sizeof msg, "moe_ffn T %lld bias %d", (long long)T, (int)with_bias);
    CHECK(norm_err(out, ref) <= 2e-3, msg);
    HostTensor Dn = view(dn, DType::Q4_K, K, FF);  // neuron-major down: not handled
    Dn.ne[2] = E;
    CHECK(!be.moe_ffn(x.data(), logits.data(), bias, T, U, G, Uu, Dn, out.data()),
          "neuron-major down left to the streamer");
}

// Host-only checks (no device): the down-weight layout by shape.
static void test_down_layout() {
    std::vector<uint8_t> b(16);
    HostTensor a = view(b, DType::Q4_K, 4096, 14336);   // n_ff rows
    HostTensor o = view(b, DType::Q4_K, 14336, 4096);   // n_ff columns
    HostTensor sq = view(b, DType::Q4_K, 4096, 4096);
    CHECK(down_layout(a, 14336) == DownLayout::NeuronRows, "n_ff rows -> neuron rows");
    CHECK(down_layout(o, 14336) == DownLayout::OutputRows, "n_ff columns -> output rows");
    CHECK(down_layout(sq, 4096) == DownLayout::NeuronRows, "square -> the reference's layout");
    bool threw = false;
    try {
        down_layout(a, 1000);
    } catch (const std::runtime_error&) {
        threw = true;
    }
    CHECK(threw, "no n_ff dimension throws");
    // MoE expert planes: standard down handled on the device, others not
    HostTensor g = view(b, DType::Q4_K, 4096, 14336), d = view(b, DType::Q4_K, 14336, 4096);
    HostTensor dn = view(b, DType::Q4_K, 4096, 14336), g8 = view(b, DType::Q8_0, 4096, 14336);
    g.ne[2] = d.ne[2] = dn.ne[2] = g8.ne[2] = 8;
    CHECK(CudaBackend::moe_supported(g, g, d), "Q4_K standard down: device MoE");
    CHECK(!CudaBackend::moe_supported(g, g, dn), "neuron-major down: streamer");
    CHECK(!CudaBackend::moe_supported(g8, g8, d), "Q8_0 experts: streamer");
}

static void test_upload_and_errors(CudaBackend& be) {
    auto w = random_blocks(DType::Q4_K, 256, 4096);
    HostTensor W = view(w, DType::Q4_K, 4096, 256);
    be.upload(W);
    std::vector<float> x(4096, 0.25f), y(256);
    be.matmul(x.data(), 1, 4096, W, y.data());
    bool threw = false;
    try {
        be.matmul(x.data(), 1, 2048, W, y.data());  // K does not match W
    } catch (const std::runtime_error&) {
        threw = true;
    }
    CHECK(threw, "mismatched K throws std::runtime_error");
    be.evict(W);  // before w's memory is freed
    be.sync();
}

// One host buffer rewritten with other weights between calls (same address,
// other blocks and formats): a weight that was never uploaded is copied per
// call, so every call must see the current bytes.
static void test_reused_host_buffer(CudaBackend& be) {
    const int64_t K = 4096, M = 3;
    std::vector<uint8_t> buf(dtype_row_bytes(DType::Q4_K, K) * 1024);
    std::vector<float> x((size_t)(M * K));
    for (auto& v : x) v = rnd();
    const DType types[4] = {DType::Q4_K, DType::Q4_K, DType::Q8_0, DType::Q6_K};
    const int64_t rows[4] = {1024, 1024, 512, 512};
    for (int c = 0; c < 4; ++c) {
        auto w = random_blocks(types[c], rows[c], K);
        std::memcpy(buf.data(), w.data(), w.size());
        HostTensor W = view(buf, types[c], K, rows[c]);
        std::vector<float> y((size_t)(M * rows[c]), NAN), ref((size_t)(M * rows[c]));
        be.matmul(x.data(), M, K, W, y.data());
        ftor_matmul(x.data(), M, K, w.data(), (int)types[c], rows[c],
                    (int64_t)W.row_stride_bytes(), ref.data(), 8);
        char msg[96];
        std::snprintf(msg, sizeof msg, "reused host buffer, case %d", c);
        CHECK(rel_err(y, ref) <= 2e-3, msg);
    }
}

// A model file through the engine's load path: ft::Gguf maps it, upload_all
// puts every tensor's blocks into HBM unchanged (ft/src/gguf.cpp:129-137 plus
// the K-quants), then matmuls on the 2-D weights and expert-chunk windows
// inside the 3-D expert tensor run from the device copies, against the
// oracle on the mapped bytes.
static void test_gguf_model(CudaBackend& be, const char* path) {
    Gguf model(path);
    size_t total = 0;
    for (const auto& kv : model.tensors()) total += kv.second.nbytes;
    const size_t up = be.upload_all(model);
    CHECK(up == total, "upload_all uploads every tensor");
    int matmuls = 0, chunks = 0;
    for (const auto& kv : model.tensors()) {
        const HostTensor& W = kv.second;
        const int t = (int)W.dtype;
        if (W.dim2() == 1 && (t == FTOR_Q4_K || t == FTOR_Q6_K || t == FTOR_Q8_0)) {
            for (int64_t M : {1, 3, 16}) {
                const int64_t K = W.cols(), N = W.rows();
                std::vector<float> x((size_t)(M * K));
                for (auto& v : x) v = rnd();
                std::vector<float> y((size_t)(M * N), NAN), ref((size_t)(M * N));
                be.matmul(x.data(), M, K, W, y.data());
                ftor_matmul(x.data(), M, K, W.data, t, N, (int64_t)W.row_stride_bytes(),
                            ref.data(), 8);
                const bool tc = t == FTOR_Q4_K && M > 8;
                char msg[160];
                std::snprintf(msg, sizeof msg, "gguf matmul %s M %lld", W.name.c_str(),
                              (long long)M);
                CHECK((tc ? norm_err(y, ref) : rel_err(y, ref)) <= 2e-3, msg);
                ++matmuls;
            }
        }
        if (W.dim2() > 1 && t == FTOR_Q4_K) {  // expert planes: windows of plane 1 in place
            const int64_t K = W.cols(), FF = W.rows(), M = 4, C = 128;
            const size_t rs = W.row_stride_bytes();
            const uint8_t* plane = W.slice(1);
            std::vector<float> x((size_t)(M * K)), out((size_t)(M * K), 0.f),
                ref((size_t)(M * K), 0.f);
            for (auto& v : x) v = rnd();
            for (int64_t i0 = 0; i0 + C <= FF; i0 += C) {
                ExpertChunkJob job;
                job.x = x.data();
                job.out = out.data();
                job.gate = plane + i0 * rs;
                job.up = plane + i0 * rs;
                job.down = plane + i0 * rs;
                job.dt = W.dtype;
                job.M = M;
                job.K = K;
                job.IC = C;
                job.gate_up_row_stride = rs;
                job.down_row_stride = rs;
                be.run_expert_chunk(job);
                ftor_expert_chunk(x.data(), ref.data(), plane + i0 * rs, plane + i0 * rs,
                                  plane + i0 * rs, t, M, K, C, (int64_t)rs, (int64_t)rs, 8);
                ++chunks;
            }
            CHECK(rel_err(out, ref) <= 2e-3, "gguf expert chunks from the uploaded planes");
        }
    }
    CHECK(matmuls >= 3 && chunks >= 1, "the model has 2-D weights and an expert tensor");
    for (const auto& kv : model.tensors()) be.evict(kv.second);
}

// ft::CudaBackend::kv_alloc + attention as the engine's layer loop uses them
// (ft/src/engine.cpp:553-566): a prefill block written into the device cache,
// decode steps after it, and a look-ahead call without write_kv; each output
// against the oracle's restatement of Engine::Impl::attn over the same rows.
static void test_attention(CudaBackend& be) {
    const int64_t nh = 16, nkv = 4, hd = 64, dk = nkv * hd, layers = 2, cap = 96;
    be.kv_alloc(layers, cap, dk);
    std::vector<std::vector<float>> kc(layers), vc(layers);
    int64_t base = 0;
    for (int64_t M : {9, 1, 1, 4}) {
        for (int64_t l = 0; l < layers; ++l) {
            for (int pass = 0; pass < 2; ++pass) {  // pass 0: look-ahead, not written
                const bool write = pass == 1;
                const int64_t rows = write ? M : 1;
                std::vector<float> q((size_t)(rows * nh * hd)), k((size_t)(rows * dk)),
                    v((size_t)(rows * dk)), out(q.size()), ref(q.size());
                for (auto& x : q) x = rnd();
                for (auto& x : k) x = rnd();
                for (auto& x : v) x = rnd();
                be.attention(l, base, rows, nh, nkv, hd, q.data(), k.data(), v.data(), write,
                             out.data());
                const float* kp = kc[l].empty() ? k.data() : kc[l].data();
                const float* vp = vc[l].empty() ? v.data() : vc[l].data();
                CHECK(ftor_attention(q.data(), rows, nh, nkv, hd, kp, vp, base, k.data(),
                                     v.data(), ref.data(), 4) == 0,
                      "oracle attention");
                double num = 0, den = 0;
                for (size_t i = 0; i < out.size(); ++i) {
                    num += (double)(out[i] - ref[i]) * (out[i] - ref[i]);
                    den += (double)ref[i] * ref[i];
                }
                CHECK(std::sqrt(num / den) < 5e-5, "attention vs oracle (normwise)");
                if (write) {
                    kc[l].insert(kc[l].end(), k.begin(), k.end());
                    vc[l].insert(vc[l].end(), v.begin(), v.end());
                }
            }
        }
        base += M;
    }
    // snapshot of layer 1 read back bit for bit, then written over and read again
    std::vector<float> sk((size_t)(base * dk)), sv(sk.size());
    be.kv_read(1, 0, base, sk.data(), sv.data());
    CHECK(std::memcmp(sk.data(), kc[1].data(), sk.size() * sizeof(float)) == 0 &&
              std::memcmp(sv.data(), vc[1].data(), sv.size() * sizeof(float)) == 0,
          "kv_read returns the rows attention wrote");
    be.kv_write(0, 0, base, sk.data(), sv.data());
    std::vector<float> rk(sk.size()), rv(sk.size());
    be.kv_read(0, 0, base, rk.data(), rv.data());
    CHECK(rk == sk && rv == sv, "kv_write then kv_read");
    bool threw = false;
    try {  // beyond the cache's capacity
        std::vector<float> q((size_t)(nh * hd)), k((size_t)dk), v((size_t)dk), o(q.size());
        be.attention(0, cap, 1, nh, nkv, hd, q.data(), k.data(), v.data(), true, o.data());
    } catch (const std::runtime_error&) {
        threw = true;
    }
    CHECK(threw, "attention past the capacity throws");
}

int main(int argc, char** argv) {
    test_down_layout();
    const char* mode = argc > 1 ? argv[1] : "";
    if (std::strcmp(mode, "--gguf") == 0 && argc > 2) {
        try {
            CudaBackend be(0);
            test_gguf_model(be, argv[2]);
            be.sync();
        } catch (const std::exception& e) {
            std::printf("FAIL exception: %s\n", e.what());
            ++g_fails;
        }
        if (g_fails) {
            std::printf("%d checks FAILED\n", g_fails);
            return 1;
        }
        std::printf("all tests passed\n");
        return 0;
    }
    if (std::strcmp(mode, "--attention") == 0) {
        try {
            CudaBackend be(0);
            test_attention(be);
            be.sync();
        } catch (const std::exception& e) {
            std::printf("FAIL exception: %s\n", e.what());
            ++g_fails;
        }
        if (g_fails) {
            std::printf("%d checks FAILED\n", g_fails);
            return 1;
        }
        std::printf("all tests passed\n");
        return 0;
    }
    if (std::strcmp(mode, "--host-only") == 0) {
        if (g_fails) return 1;
        std::printf("all tests passed\n");
        return 0;
    }
    // --down-project: only the down projection (run late in the suite)
    const bool down_only = std::strcmp(mode, "--down-project") == 0;
    try {
        CudaBackend be(0);
        if (down_only) {
            test_down_project(be, DType::Q4_K, 14336, 4096, 1);
            test_down_project(be, DType::Q4_K, 1024, 512, 3);
            test_down_project(be, DType::Q8_0, 96, 4096, 9);
            test_down_project(be, DType::Q6_K, 512, 512, 2);
            test_moe_ffn(be, 1, false);
            test_moe_ffn(be, 37, true);
            be.sync();
            if (g_fails) {
                std::printf("%d checks FAILED\n", g_fails);
                return 1;
            }
            std::printf("all tests passed\n");
            return 0;
        }
        CHECK(be.ready(), "backend ready");
        CHECK(be.info().mem_bytes > (100ull << 30), "device memory reported");
        CHECK(be.alloc_staging(1 << 20) == nullptr, "no staging buffers");
        test_matmul(be, DType::Q4_K, 512, 4096, 1);
        test_matmul(be, DType::Q4_K, 1024, 14336, 3);
        test_matmul(be, DType::Q8_0, 256, 4096, 1);
        test_matmul(be, DType::Q6_K, 300, 4096, 2);
        test_matmul(be, DType::Q4_K, 1024, 4096, 9);     // tensor-core path from 9 rows
        test_matmul(be, DType::Q4_K, 4096, 14336, 128);  // a prefill chunk
        test_matmul(be, DType::Q8_0, 512, 4096, 20);     // GEMV, 8 rows per pass
        test_expert_chunk_windows(be);
        test_upload_and_errors(be);
        test_reused_host_buffer(be);
    } catch (const std::exception& e) {
        std::printf("FAIL exception: %s\n", e.what());
        ++g_fails;
    }
    if (g_fails) {
        std::printf("%d checks FAILED\n", g_fails);
        return 1;
    }
    std::printf("all tests passed\n");
    return 0;
}
