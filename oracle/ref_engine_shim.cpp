// ref_engine_shim.cpp -- C entry points onto the reference engine's OWN
// attention code: Engine::Impl::attn (ft/src/engine.cpp:137-177), rope_vec
// (ft/src/engine.cpp:43-60) and softmax_inplace (ft/src/engine.cpp:62-72).
// oracle/Makefile compiles it with the reference's engine.cpp included into
// this translation unit (so its file-local helpers and the engine's private
// Impl are reachable) and links the reference's other sources that
// engine.cpp needs (gguf, graph, tokenizer, spec, cpu_backend; no Vulkan),
// into oracle/_ref/libftref_engine.so.
//
// TEST INFRASTRUCTURE ONLY: used to pin the oracle's restatement of the
// attention path in tests/.  Nothing here is reference source; it only
// calls it.
//
// The standard headers come first: the access override below must only
// reach the reference's own classes.
#include <algorithm>
#include <array>
#include <atomic>
#include <chrono>
#include <cmath>
#include <condition_variable>
#include <cstring>
#include <deque>
#include <exception>
#include <fstream>
#include <functional>
#include <iostream>
#include <map>
#include <memory>
#include <mutex>
#include <optional>
#include <random>
#include <set>
#include <sstream>
#include <string>
#include <thread>
#include <unordered_map>
#include <unordered_set>
#include <vector>

#define private public
#include "engine.cpp"
#undef private

extern "C" {

// One call of Engine::Impl::attn for one layer: q [M][n_head][hd] (after
// RoPE), the layer's cache rows [0, base) of k_cache / v_cache ([pos][dk],
// dk = n_head_kv * hd), the current block's rows k_blk / v_blk ([M][dk]);
// out [M][n_head][hd].  Returns -1 if the reference throws.
int ftref_attn(const float* q, int64_t M, int64_t n_head, int64_t n_head_kv, int64_t hd,
               const float* k_cache, const float* v_cache, int64_t base, const float* k_blk,
               const float* v_blk, float* out, int threads) {
    try {
        ft::Engine::Impl I;
        I.cfg.head_dim = hd;
        I.cfg.n_head = n_head;
        I.cfg.n_head_kv = n_head_kv;
        I.opt.threads = threads;
        const int64_t dk = n_head_kv * hd;
        I.kv.alloc(1, base + M, dk, dk);
        if (base > 0) {
            std::memcpy(I.kv.k(0), k_cache, (size_t)(base * dk) * sizeof(float));
            std::memcpy(I.kv.v(0), v_cache, (size_t)(base * dk) * sizeof(float));
        }
        I.q.assign(q, q + M * n_head * hd);
        I.attout.assign((size_t)(M * n_head * hd), 0.f);
        I.attn(0, base, M, k_blk, v_blk);
        std::memcpy(out, I.attout.data(), I.attout.size() * sizeof(float));
        return 0;
    } catch (const std::exception&) {
        return -1;
    }
}

void ftref_rope_vec(float* v, int64_t hd, int64_t pos, double theta, int neox) {
    ft::rope_vec(v, hd, pos, theta, neox != 0);
}

void ftref_softmax(float* p, int64_t n) { ft::softmax_inplace(p, n); }

}  // extern "C"
