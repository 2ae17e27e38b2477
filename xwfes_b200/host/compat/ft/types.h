// ft/types.h -- the subset of the reference engine's interface types that a
// backend implementation needs (reference: ft/include/ft/types.h:16-147),
// restated so this repository's C++ adapter and its tests compile without
// the reference tree.  Names, enumerator values and field layout match the
// reference's, so cuda_backend.cpp compiles unchanged against either header.
// The two K-quant enumerators (GGUF type ids 12 and 14) are the ones a
// maintainer adds to the reference's DType to load Q4_K / Q6_K tensors.
#pragma once

#include <cstddef>
#include <cstdint>
#include <stdexcept>
#include <string>

namespace ft {

enum class DType : uint32_t {
    F32 = 0,
    F16 = 1,
    Q4_0 = 2,
    Q4_1 = 3,
    Q8_0 = 8,
    Q4_K = 12,
    Q6_K = 14,
    BF16 = 30,
};

constexpr size_t QK = 32;
constexpr size_t QK_K = 256;

inline size_t dtype_elems_per_block(DType t) {
    switch (t) {
        case DType::Q4_0: case DType::Q4_1: case DType::Q8_0: return QK;
        case DType::Q4_K: case DType::Q6_K: return QK_K;
        default: return 1;
    }
}

inline size_t dtype_bytes_per_block(DType t) {
    switch (t) {
        case DType::F32: return 4;
        case DType::F16: case DType::BF16: return 2;
        case DType::Q4_0: return 18;
        case DType::Q4_1: return 20;
        case DType::Q8_0: return 34;
        case DType::Q4_K: return 144;
        case DType::Q6_K: return 210;
        default: throw std::runtime_error("unknown dtype");
    }
}

inline size_t dtype_row_bytes(DType t, int64_t n_cols) {
    const size_t eb = dtype_elems_per_block(t), bb = dtype_bytes_per_block(t);
    return (size_t)((n_cols + (int64_t)eb - 1) / (int64_t)eb) * bb;
}

// Non-owning view of a tensor's blocks: ne[0] = columns (K, the block
// axis), ne[1] = rows (N), ne[2] = expert planes.
struct HostTensor {
    std::string name;
    int64_t ne[4] = {1, 1, 1, 1};
    int32_t n_dims = 0;
    DType dtype = DType::F32;
    const uint8_t* data = nullptr;
    size_t nbytes = 0;

    int64_t cols() const { return ne[0]; }
    int64_t rows() const { return ne[1]; }
    int64_t dim2() const { return ne[2]; }
    int64_t dim3() const { return ne[3]; }
    size_t row_stride_bytes() const { return dtype_row_bytes(dtype, ne[0]); }
    size_t slice_bytes() const { return row_stride_bytes() * (size_t)ne[1]; }
    const uint8_t* slice(int64_t i2, int64_t i3 = 0) const {
        return data + slice_bytes() * ((size_t)i3 * (size_t)ne[2] + (size_t)i2);
    }
};

struct DeviceInfo {
    std::string name;
    bool integrated = false;
    bool uma = false;
    uint64_t mem_bytes = 0;
};

}  // namespace ft
