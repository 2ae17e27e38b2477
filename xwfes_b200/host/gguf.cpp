// gguf.cpp -- GGUF model-file reader for the engine's loader (ft::Gguf, the
// interface of ft/include/ft/gguf.h), written from the GGUF file format:
//
//   header   "GGUF" magic (u32 0x46554747), version (2 or 3), tensor count
//            (u64), metadata count (u64)
//   metadata key (u64 length + bytes), value type (u32), value; types 0-12:
//            u8 i8 u16 i16 u32 i32 f32 bool string array u64 i64 f64, an
//            array being element type (u32) + count (u64) + elements
//   tensors  name, dimension count (u32), dims (u64 each, dims[0] the
//            contiguous axis), GGML type (u32), offset (u64) from the start
//            of the data section
//   data     starts at the first multiple of general.alignment (default 32)
//            after the tensor records
//
// Differences from the reference reader (ft/src/gguf.cpp): the GGUF
// K-quant types Q4_K (12) and Q6_K (14) load as ft::DType::Q4_K / Q6_K (the
// reference stops at ft/src/gguf.cpp:129-137), and every tensor is checked
// to lie inside the file and to hold whole blocks per row, so a damaged file
// fails at load instead of at the first matmul.
#include "ft/gguf.h"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstring>
#include <stdexcept>

namespace ft {

namespace {

enum : uint32_t {
    kU8 = 0, kI8, kU16, kI16, kU32, kI32, kF32, kBool, kStr, kArr, kU64, kI64, kF64
};

size_t scalar_size(uint32_t t) {
    switch (t) {
        case kU8: case kI8: case kBool: return 1;
        case kU16: case kI16: return 2;
        case kU32: case kI32: case kF32: return 4;
        case kU64: case kI64: case kF64: return 8;
        default: return 0;
    }
}

// One metadata value: numbers are kept as both int64 and double (the getters
// convert), arrays of numbers element-wise, arrays of strings as strings.
struct Meta {
    uint32_t type = 0;
    int64_t i = 0;
    double f = 0.0;
    std::string s;
    uint32_t elem = 0;
    std::vector<int64_t> ai;
    std::vector<double> af;
    std::vector<std::string> as;
};

// Bounds-checked little-endian cursor over the mapped file.
struct Cursor {
    const uint8_t* base;
    size_t size;
    size_t at = 0;

    const uint8_t* take(size_t n, const char* what) {
        if (n > size || at > size - n)
            throw std::runtime_error(std::string("gguf: truncated file (") + what + ")");
        const uint8_t* p = base + at;
        at += n;
        return p;
    }
    template <typename T>
    T get(const char* what) {
        T v;
        std::memcpy(&v, take(sizeof(T), what), sizeof(T));
        return v;
    }
    std::string str(const char* what) {
        const uint64_t n = get<uint64_t>(what);
        if (n > size) throw std::runtime_error(std::string("gguf: bad string length (") + what + ")");
        const uint8_t* p = take((size_t)n, what);
        return std::string(reinterpret_cast<const char*>(p), (size_t)n);
    }
    // a number of type t as (int, float)
    void number(uint32_t t, int64_t& i, double& f, const char* what) {
        switch (t) {
            case kU8: i = get<uint8_t>(what); f = (double)i; break;
            case kI8: i = get<int8_t>(what); f = (double)i; break;
            case kU16: i = get<uint16_t>(what); f = (double)i; break;
            case kI16: i = get<int16_t>(what); f = (double)i; break;
            case kU32: i = get<uint32_t>(what); f = (double)i; break;
            case kI32: i = get<int32_t>(what); f = (double)i; break;
            case kU64: i = (int64_t)get<uint64_t>(what); f = (double)(uint64_t)i; break;
            case kI64: i = get<int64_t>(what); f = (double)i; break;
            case kBool: i = get<uint8_t>(what) != 0; f = (double)i; break;
            case kF32: f = get<float>(what); i = (int64_t)f; break;
            case kF64: f = get<double>(what); i = (int64_t)f; break;
            default: throw std::runtime_error(std::string("gguf: bad number type (") + what + ")");
        }
    }
    Meta meta(uint32_t t, const char* what) {
        Meta m;
        m.type = t;
        if (t == kStr) {
            m.s = str(what);
        } else if (t == kArr) {
            m.elem = get<uint32_t>(what);
            const uint64_t n = get<uint64_t>(what);
            if (m.elem == kStr) {
                if (n > size) throw std::runtime_error(std::string("gguf: bad array length (") + what + ")");
                m.as.reserve((size_t)n);
                for (uint64_t k = 0; k < n; ++k) m.as.push_back(str(what));
            } else if (scalar_size(m.elem)) {
                if (n > size / scalar_size(m.elem))
                    throw std::runtime_error(std::string("gguf: bad array length (") + what + ")");
                m.ai.resize((size_t)n);
                m.af.resize((size_t)n);
                for (uint64_t k = 0; k < n; ++k) number(m.elem, m.ai[(size_t)k], m.af[(size_t)k], what);
            } else {
                throw std::runtime_error(std::string("gguf: unsupported array element type (") + what + ")");
            }
        } else if (scalar_size(t)) {
            number(t, m.i, m.f, what);
        } else {
            throw std::runtime_error(std::string("gguf: unsupported metadata type (") + what + ")");
        }
        return m;
    }
};

bool to_dtype(uint32_t ggml, DType& out) {
    switch (ggml) {
        case 0: out = DType::F32; return true;
        case 1: out = DType::F16; return true;
        case 2: out = DType::Q4_0; return true;
        case 3: out = DType::Q4_1; return true;
        case 8: out = DType::Q8_0; return true;
        case 12: out = DType::Q4_K; return true;
        case 14: out = DType::Q6_K; return true;
        case 30: out = DType::BF16; return true;
        default: return false;
    }
}

}  // namespace

struct Gguf::Impl {
    int fd = -1;
    const uint8_t* map = nullptr;
    size_t size = 0;
    std::unordered_map<std::string, Meta> kv;

    ~Impl() {
        if (map) munmap(const_cast<uint8_t*>(map), size);
        if (fd >= 0) ::close(fd);
    }
    const Meta* find(const std::string& key) const {
        auto it = kv.find(key);
        return it == kv.end() ? nullptr : &it->second;
    }
};

Gguf::Gguf(const std::string& path) : impl_(new Impl) {
    Impl& I = *impl_;
    I.fd = ::open(path.c_str(), O_RDONLY);
    if (I.fd < 0) throw std::runtime_error("gguf: cannot open " + path);
    struct stat st {};
    if (fstat(I.fd, &st) != 0) throw std::runtime_error("gguf: cannot stat " + path);
    I.size = (size_t)st.st_size;
    if (I.size < 24) throw std::runtime_error("gguf: file too small: " + path);
    void* p = mmap(nullptr, I.size, PROT_READ, MAP_PRIVATE, I.fd, 0);
    if (p == MAP_FAILED) throw std::runtime_error("gguf: cannot map " + path);
    I.map = static_cast<const uint8_t*>(p);

    Cursor c{I.map, I.size};
    if (c.get<uint32_t>("magic") != 0x46554747u) throw std::runtime_error("gguf: not a GGUF file: " + path);
    const uint32_t version = c.get<uint32_t>("version");
    if (version != 2 && version != 3)
        throw std::runtime_error("gguf: unsupported version " + std::to_string(version));
    const uint64_t n_tensors = c.get<uint64_t>("tensor count");
    const uint64_t n_kv = c.get<uint64_t>("metadata count");
    if (n_tensors > I.size || n_kv > I.size) throw std::runtime_error("gguf: bad counts");

    for (uint64_t k = 0; k < n_kv; ++k) {
        std::string key = c.str("metadata key");
        const uint32_t t = c.get<uint32_t>("metadata type");
        Meta m = c.meta(t, key.c_str());
        I.kv[std::move(key)] = std::move(m);
    }
    uint64_t align = 32;
    if (const Meta* a = I.find("general.alignment")) {
        if (a->type == kStr || a->type == kArr || a->i <= 0 || (a->i & (a->i - 1)) != 0)
            throw std::runtime_error("gguf: general.alignment must be a power of two");
        align = (uint64_t)a->i;
    }

    struct Rec {
        std::string name;
        HostTensor t;
        uint64_t offset;
    };
    std::vector<Rec> recs;
    recs.reserve((size_t)n_tensors);
    for (uint64_t k = 0; k < n_tensors; ++k) {
        Rec r;
        r.name = c.str("tensor name");
        const uint32_t nd = c.get<uint32_t>(r.name.c_str());
        if (nd < 1 || nd > 4) throw std::runtime_error("gguf: " + r.name + " has " + std::to_string(nd) + " dims");
        for (uint32_t d = 0; d < nd; ++d) {
            const uint64_t v = c.get<uint64_t>(r.name.c_str());
            if (v == 0 || v > ((uint64_t)1 << 40))
                throw std::runtime_error("gguf: " + r.name + " has a bad dimension");
            r.t.ne[d] = (int64_t)v;
        }
        r.t.n_dims = (int32_t)nd;
        const uint32_t ggml = c.get<uint32_t>(r.name.c_str());
        if (!to_dtype(ggml, r.t.dtype))
            throw std::runtime_error("gguf: " + r.name + " has unsupported tensor type " + std::to_string(ggml));
        r.offset = c.get<uint64_t>(r.name.c_str());
        r.t.name = r.name;
        recs.push_back(std::move(r));
    }

    const uint64_t data0 = (c.at + align - 1) / align * align;
    for (Rec& r : recs) {
        HostTensor& t = r.t;
        if ((uint64_t)t.ne[0] % dtype_elems_per_block(t.dtype) != 0)
            throw std::runtime_error("gguf: " + r.name + ": rows are not whole blocks");
        const uint64_t nbytes = (uint64_t)t.slice_bytes() * (uint64_t)t.ne[2] * (uint64_t)t.ne[3];
        if (r.offset % align != 0 || data0 + r.offset > I.size || nbytes > I.size - (data0 + r.offset))
            throw std::runtime_error("gguf: " + r.name + " lies outside the file");
        t.data = I.map + data0 + r.offset;
        t.nbytes = (size_t)nbytes;
        if (!tensors_.emplace(r.name, t).second)
            throw std::runtime_error("gguf: duplicate tensor " + r.name);
    }
}

Gguf::~Gguf() = default;

bool Gguf::has(const std::string& key) const { return impl_->find(key) != nullptr; }

namespace {

[[noreturn]] void wrong_type(const std::string& key, const char* want) {
    throw std::runtime_error("gguf: metadata " + key + " is not " + want);
}

}  // namespace

std::string Gguf::get_str(const std::string& key, const std::string& def) const {
    const Meta* m = impl_->find(key);
    if (!m) return def;
    if (m->type != kStr) wrong_type(key, "a string");
    return m->s;
}

int64_t Gguf::get_i64(const std::string& key, int64_t def) const {
    const Meta* m = impl_->find(key);
    if (!m) return def;
    if (m->type == kStr || m->type == kArr) wrong_type(key, "a number");
    return m->i;
}

double Gguf::get_f64(const std::string& key, double def) const {
    const Meta* m = impl_->find(key);
    if (!m) return def;
    if (m->type == kStr || m->type == kArr) wrong_type(key, "a number");
    return m->f;
}

bool Gguf::get_bool(const std::string& key, bool def) const {
    const Meta* m = impl_->find(key);
    if (!m) return def;
    if (m->type == kStr || m->type == kArr) wrong_type(key, "a bool");
    return m->i != 0;
}

std::vector<std::string> Gguf::get_str_arr(const std::string& key) const {
    const Meta* m = impl_->find(key);
    if (!m) return {};
    if (m->type != kArr || m->elem != kStr) wrong_type(key, "an array of strings");
    return m->as;
}

std::vector<float> Gguf::get_f32_arr(const std::string& key) const {
    const Meta* m = impl_->find(key);
    if (!m) return {};
    if (m->type != kArr || m->elem == kStr) wrong_type(key, "an array of numbers");
    return std::vector<float>(m->af.begin(), m->af.end());
}

std::vector<int32_t> Gguf::get_i32_arr(const std::string& key) const {
    const Meta* m = impl_->find(key);
    if (!m) return {};
    if (m->type != kArr || m->elem == kStr) wrong_type(key, "an array of numbers");
    std::vector<int32_t> out;
    out.reserve(m->ai.size());
    for (int64_t v : m->ai) out.push_back((int32_t)v);
    return out;
}

const HostTensor* Gguf::tensor(const std::string& name) const {
    auto it = tensors_.find(name);
    return it == tensors_.end() ? nullptr : &it->second;
}

}  // namespace ft
