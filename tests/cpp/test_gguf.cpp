// Probe of the GGUF reader (xwfes_b200/host/gguf.cpp) for tests/test_gguf_loader.py:
//   test_gguf <file> tensors          one line per tensor (sorted by name):
//                                     name n_dims ne0 ne1 ne2 ne3 dtype nbytes offset fnv1a64
//   test_gguf <file> <getter> <key>   str | i64 | f64 | bool | str_arr | f32_arr | i32_arr | has
//   test_gguf <file> dequant <tensor> <plane> <row>
//                                     fnv1a64 of the row's fp32 values, dequantized by
//                                     the oracle (oracle/ftoracle.c) through the
//                                     reader's view (slice + row stride)
// A load or lookup error prints "error: <message>" and exits with status 2.
#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <stdexcept>
#include <string>
#include <vector>

#include "ft/gguf.h"
#include "ftoracle.h"

static unsigned long long fnv1a(const uint8_t* p, size_t n) {
    unsigned long long h = 1469598103934665603ull;
    for (size_t i = 0; i < n; ++i) h = (h ^ p[i]) * 1099511628211ull;
    return h;
}

int main(int argc, char** argv) {
    if (argc < 3) return 1;
    try {
        ft::Gguf g(argv[1]);
        const std::string what = argv[2];
        if (what == "tensors") {
            std::vector<std::string> names;
            for (const auto& kv : g.tensors()) names.push_back(kv.first);
            std::sort(names.begin(), names.end());
            const uint8_t* first = nullptr;
            for (const auto& n : names) {
                const ft::HostTensor* t = g.tensor(n);
                if (!first || t->data < first) first = t->data;
            }
            for (const auto& n : names) {
                const ft::HostTensor* t = g.tensor(n);
                std::printf("%s %d %lld %lld %lld %lld %u %zu %lld %llu\n", n.c_str(), t->n_dims,
                            (long long)t->ne[0], (long long)t->ne[1], (long long)t->ne[2],
                            (long long)t->ne[3], (unsigned)t->dtype, t->nbytes,
                            (long long)(t->data - first), fnv1a(t->data, t->nbytes));
            }
            return 0;
        }
        if (argc < 4) return 1;
        const std::string key = argv[3];
        if (what == "dequant" && argc >= 6) {
            const ft::HostTensor* t = g.tensor(key);
            if (!t) throw std::runtime_error("no tensor " + key);
            const long plane = std::atol(argv[4]), row = std::atol(argv[5]);
            std::vector<float> v((size_t)t->ne[0]);
            const uint8_t* src = t->slice(plane) + (size_t)row * t->row_stride_bytes();
            if (ftor_dequant_row(v.data(), src, (int)t->dtype, t->ne[0]) != 0)
                throw std::runtime_error("oracle dequant failed");
            std::printf("%llu\n", fnv1a(reinterpret_cast<const uint8_t*>(v.data()), v.size() * 4));
            return 0;
        }
        if (what == "has") std::printf("%d\n", g.has(key) ? 1 : 0);
        else if (what == "str") std::printf("%s\n", g.get_str(key, "<default>").c_str());
        else if (what == "i64") std::printf("%lld\n", (long long)g.get_i64(key, -12345));
        else if (what == "f64") std::printf("%.17g\n", g.get_f64(key, -1.5));
        else if (what == "bool") std::printf("%d\n", g.get_bool(key, false) ? 1 : 0);
        else if (what == "str_arr") {
            for (const auto& s : g.get_str_arr(key)) std::printf("%s\n", s.c_str());
        } else if (what == "f32_arr") {
            for (float v : g.get_f32_arr(key)) std::printf("%.9g\n", (double)v);
        } else if (what == "i32_arr") {
            for (int32_t v : g.get_i32_arr(key)) std::printf("%d\n", v);
        } else {
            return 1;
        }
        return 0;
    } catch (const std::exception& e) {
        std::printf("error: %s\n", e.what());
        return 2;
    }
}
