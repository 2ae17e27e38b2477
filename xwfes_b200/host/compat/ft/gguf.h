// ft/gguf.h -- the GGUF model-file reader interface of the reference engine
// (ft/include/ft/gguf.h), restated so that the adapter builds without the
// reference tree.  The class name, methods and their meaning are the
// reference's, so the engine's loader code (Engine::load,
// ft/src/engine.cpp:282-396) compiles unchanged against this header; the
// implementation (xwfes_b200/host/gguf.cpp) is this repository's own and
// accepts the GGUF K-quant tensor types Q4_K (12) and Q6_K (14) besides the
// reference's F32, F16, BF16, Q4_0, Q4_1 and Q8_0.
#pragma once

#include <cstdint>
#include <memory>
#include <string>
#include <unordered_map>
#include <vector>

#include "ft/types.h"

namespace ft {

class Gguf {
public:
    // Maps the file read-only; throws std::runtime_error when it is not a
    // version 2 or 3 GGUF file, is truncated, holds an unsupported tensor
    // type or a tensor whose blocks lie outside the file.
    explicit Gguf(const std::string& path);
    ~Gguf();

    Gguf(const Gguf&) = delete;
    Gguf& operator=(const Gguf&) = delete;

    bool has(const std::string& key) const;

    // Scalar metadata; `def` when the key is absent (a key of another type
    // throws).
    std::string get_str(const std::string& key, const std::string& def = "") const;
    int64_t get_i64(const std::string& key, int64_t def = 0) const;
    double get_f64(const std::string& key, double def = 0) const;
    bool get_bool(const std::string& key, bool def = false) const;

    // Array metadata; empty when the key is absent.
    std::vector<std::string> get_str_arr(const std::string& key) const;
    std::vector<float> get_f32_arr(const std::string& key) const;
    std::vector<int32_t> get_i32_arr(const std::string& key) const;

    // Views into the mapping (valid while this object lives); nullptr when
    // the name is absent.
    const HostTensor* tensor(const std::string& name) const;
    const std::unordered_map<std::string, HostTensor>& tensors() const { return tensors_; }

private:
    struct Impl;
    std::unique_ptr<Impl> impl_;
    std::unordered_map<std::string, HostTensor> tensors_;
};

}  // namespace ft
